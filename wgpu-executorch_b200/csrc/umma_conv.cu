// tcgen05 / TMEM implicit-GEMM convolution (fp16 in, fp32 accumulate).
//
// Replaces the register-tiled WGSL implicit-im2col GEMMs of the reference
// (src/shaders/convolution/conv2d-tile64-f16.wgsl.ts:8-181,
// conv2d-tile32-f16.wgsl.ts, conv2d-gemm-f16.wgsl.ts,
// conv2d-1x1-tile64-f16.wgsl.ts, conv2d-1x1-tile32-f16.wgsl.ts and the
// conv-with-clamp twins). Same GEMM: M = OC, N = output positions,
// K = IC*KH*KW, bias (+ clamp / SiLU) epilogue, NCHW store. The reference
// accumulates in f16 (vec4<f16> acc); here products accumulate in fp32 in
// tensor memory and the epilogue rounds once.
//
// Data layout (B200 design, no materialised im2col):
//  * input re-laid by pack_input into a zero-padded, channel-blocked
//    layout xs[b][c/8][Hp][Wp][8] (Hp = IH+2pH, Wp = IW+2pW, for the
//    transposed variant rounded up to a multiple of 8 where that costs at
//    most 5 %; channels padded to a multiple of 32). One "row" = one padded position = 16 bytes.
//    Flattening (hp, wp) to p = hp*Wp + wp turns a stride-1 convolution into
//    out[p] = sum_taps W_tap . xs[p + kh*dH*Wp + kw*dW]: every tap is a pure
//    row shift.
//  * a stride-s convolution (dilation 1) is run as a stride-1 convolution
//    over a space-to-depth view of its input: writing each tap offset
//    kh - pH = s*d + ph (0 <= ph < s), input row s*oh + kh - pH is row
//    oh + d of phase ph. The re-layout stores phase (ph, pw) of input
//    channel c as virtual channel (phase index)*IC + c, the virtual filter
//    spans the d range (3x3 / stride 2 / pad 1 -> 2x2 over 4*IC channels)
//    and the packed weights hold w[oc][c][s*d + ph + pH][...] at virtual
//    tap d, zero where that tap falls outside the real filter.
//  * operands in shared memory use the canonical K-major no-swizzle layout
//    (core matrix = 8 rows x 16 bytes, rows 16 bytes apart, 8-channel chunks
//    one plane apart). A row shift is then just a 16-byte move of the
//    descriptor start address, so one staged activation tile feeds all KW
//    taps of a filter row.
//  * weights packed by pack_weights into [oc_tile][kh][cblk][kw][chunk][128][8]
//    so the A operand of one pipeline stage is one contiguous bulk copy.
//
// Persistent kernel: one CTA per SM loops over tiles of 128 output channels
// x 256 positions. Pipeline stage = (kh, 32-channel block): A = KW x 128 x 32
// weights, B = (256 + (KW-1)*dW) activation rows x 32 channels. When all
// weights of the (single) output-channel tile fit next to the pipeline they
// are loaded once per CTA and stay resident; otherwise each stage streams
// its A block. Two TMEM accumulators of 256 columns ping-pong, so the
// epilogue of tile i overlaps the MMAs of tile i+1.
// Warp roles: warp 0 issues bulk copies, warp 1 owns TMEM and issues
// tcgen05.mma (with positions on M and several M blocks per tile, warp 2
// issues every other M block: two issuers keep the tensor pipe busier on
// short MMAs), warps 4-19 drain TMEM (four warps per TMEM lane quadrant,
// 64 columns each) through bias + activation to NCHW global memory.
//
// Every mbarrier wait is bounded (about 2 s of %globaltimer); on expiry the
// waiting role sets a bit in the device error word and stops, so a broken
// pipeline returns an error instead of hanging the GPU.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>

#include "tcgen05.h"
#include "tma.h"
#include "umma_conv.h"

namespace wgx {

constexpr int UM = 128;          // MMA M: output channels per tile
constexpr int UN = 256;          // MMA N: positions per tile
constexpr int EPI_WARP0 = 4;     // first epilogue warp
constexpr int EPI_WARPS = 16;    // four per TMEM lane quadrant
constexpr int THREADS = 32 * (EPI_WARP0 + EPI_WARPS);
constexpr uint32_t TMEM_COLS = 512;  // two accumulators of UN fp32 columns
constexpr int MAX_KW = 7;
constexpr int EPI_COLS = 16;     // positions per staged epilogue block
constexpr int EPI_ROWB = 48;     // staged channel row: 16 fp16 + 16 B pad
constexpr uint32_t EPI_BYTES = EPI_WARPS * 32 * EPI_ROWB;
// transposed epilogue: bias (<= 64 floats) in the first 1 KB, then 1 KB of
// transpose rows per warp
static_assert(1024 + EPI_WARPS * 1024 <= EPI_BYTES, "epilogue staging");
constexpr uint32_t SMEM_MAX = 227u * 1024u;

constexpr int kMaxSrc = 8;
constexpr int kMaxOut = 4;

// space-to-depth tap masks: filter-row groups x phases
constexpr int kMaxKhg = 4, kMaxPhases = 16;

struct UmmaGeom {
  // IC, KH, KW, dH, dW, pH, pW describe the stride-1 convolution the MMA
  // pipeline runs (for a strided convolution: the space-to-depth view);
  // the x* fields and the phase tables describe the real one.
  int B, IC, IH, IW, OC, OH, OW, KH, KW, dH, dW, pH, pW;
  int sH, sW, xIC, xKH, xKW, xpH, xpW;
  int nphH, nphW, phH[4], phW[4];    // input phases the filter touches
  // trans = 1: positions on the MMA M side (128 per MMA, G M-blocks per
  // tile), output channels on N (NT = OC rounded up to 16/32/64). Used for
  // OC <= 64, where channels on M would leave TMEM lane quadrants idle.
  int trans, NT, G, lgNT;
  int tile_pos;                      // positions of one tile's accumulator (M rows)
  int tile_stride;                   // first positions of consecutive tiles: tile_pos,
                                     // or tile_pos - 8 when hs > 0 (see below)
  // hs > 0 (positions on M, stride 1, filter width hs = 3): the filter
  // columns are folded into N. The MMA pipeline runs the KW = 1 convolution
  // Y[q][kw*ocp + oc] = sum_{kh,c} xs[q + kh*dH*Wp][c] w[oc][c][kh][kw]
  // (N = 3*ocp rounded up to 16, ocp = OC rounded up to 8 / 16 / 32 / 64), one MMA per
  // filter row and 16 channels instead of three, and the epilogue forms
  // out[p][oc] = Y[p][oc] + Y[p+1][ocp+oc] + Y[p+2][2*ocp+oc]. A tile's
  // last 8 positions only feed its own outputs, so tiles advance by
  // tile_pos - 8.
  int hs, ocp;
  // position -> padded row: pos / Wp = __umulhi(pos, wp_magic) with
  // wp_magic = ceil(2^32 / Wp), exact for every position the kernel forms
  // (checked on the host: pos_max * (wp_magic * Wp - 2^32) < 2^32); 0 =
  // plain division
  uint32_t wp_magic;
  int wrows;                         // packed weight rows per oc tile (UM or NT)
  int acc_cols;                      // TMEM columns per accumulator
  int bk, chunks;                    // channels per stage, 16-byte chunks per stage
  int khs, n_khg;                    // filter rows per stage, filter-row groups
  int Hp, Wp, C8, ncb, n_oct, tiles_per_img, total_tiles, R, R_alloc, stages, n_kstages;
  int resident;                      // all weights of the oc tile stay in smem
  long long plane_rows;              // Hp*Wp
  uint32_t a_stage_bytes, b_stage_bytes, w_region_bytes;
  int has_bias, act;
  float lo, hi;
  uint32_t *err;
  // output layout: omode 0 = NCHW `out`; 1 = the re-laid input of a
  // consuming tcgen05 convolution (its xs layout, described below), written
  // 16 bytes (8 channels of one position) at a time
  int omode;
  int oHp, oWp, oplanes, opH, opW, osH, osW, onphW, oxIC;
  int ophase_h[4], ophase_w[4];  // consumer phase index of (row mod osH), -1 when unused
  uint4 *oxs;
  // input: up to kMaxSrc channel ranges (a concatenation along channels),
  // source s holding channels [src_c0[s], src_c0[s+1]) of the input
  int nsrc;
  int src_c0[kMaxSrc + 1];
  const __half *src[kMaxSrc];
  // direct = 1 (1x1, stride 1, no padding): the producer loads activation
  // tiles straight from the NCHW sources with TMA (boxes of 64 positions x
  // dbox channels, 128-byte swizzle, zero fill past the image and past a
  // source's channels) and the MMAs read them MN-major; no re-layout runs
  int direct, dbox;
  // transposed variant, NCHW output (or split pieces) with Wp % 8 == 0,
  // OW % 8 == 0 and 16-byte aligned outputs: 16-byte epilogue stores
  int tvec;
  // channels-on-M space-to-depth stages whose channel block lies within one
  // phase (xIC % bk == 0): taps (bit khl*KW + kw) of filter-row group khg and
  // phase whose packed weights are not all zero. The MMAs of the other taps
  // add zeros and are skipped; a stage with none is neither loaded nor
  // issued (3x3 / stride 2: 9 of the 16 phase x tap pairs, and a quarter of
  // the stages). tapskip = 0: every stage uses every tap. cbpp = channel
  // blocks per phase.
  int tapskip, cbpp;
  uint16_t tapmask[kMaxKhg][kMaxPhases];
  // NCHW output options (omode 0): `resid` (same shape as the output) is
  // added after the activation; nout > 0 splits the output channels into
  // tensors outp[k] holding channels [out_c0[k], out_c0[k+1])
  const __half *resid;
  int nout;
  int out_c0[kMaxOut + 1];
  __half *outp[kMaxOut];
  // failure-detection tests (WGX_INJECT_SKIP_LOADS): the producer issues no
  // copies, so the other roles' bounded waits run out
  int inject_skip;
  // split = 1: each stage's copies are split across several issuing threads
  // (see the producer); 0: one issuer
  int split;
  // per-image weights (a batched GEMM: aten.bmm as a 1x1 convolution whose
  // weights differ per image): packed weight bytes per image, 0 = shared
  uint64_t w_img_bytes;
  // buffer extents in bytes, checked by the bounds-checking build
  // (WGX_BOUNDS): out (and resid), the re-laid input xs, the consumer's xs,
  // the packed weights, the split pieces
  uint64_t out_bytes, xs_bytes, oxs_bytes, wpk_bytes, outp_bytes[kMaxOut];
};

// Bounds checks of the epilogue stores (WGX_BOUNDS build; true otherwise):
// an NCHW store lands in `out` or, with split outputs, in one of the pieces.
__device__ __forceinline__ bool out_ok(const UmmaGeom &g, const __half *out, const void *p,
                                       int n) {
#ifdef WGX_BOUNDS
  if (g.nout == 0) return bounds_ok(p, uint64_t(n), out, g.out_bytes, g.err);
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  for (int k = 0; k < kMaxOut; ++k) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(g.outp[k]);
    if (k < g.nout && a >= b && a + uint64_t(n) <= b + g.outp_bytes[k]) return true;
  }
  atomicOr(g.err, kErrBounds);
  return false;
#else
  return true;
#endif
}
__device__ __forceinline__ bool oxs_ok(const UmmaGeom &g, const void *p) {
  return WGX_IN_BOUNDS(p, 16, g.oxs, g.oxs_bytes, g.err);
}

// MMA groups (filter tap x 16-channel step) of one stage whose descriptor
// offsets the generic staging keeps in shared memory
constexpr int kMaxGroups = 128;
// generic staging: stages of at most this many MMA groups issue as one
// straight-line sequence
constexpr int kSeqGroups = 8;

static uint32_t smem_need(const UmmaGeom &g) {
  return g.w_region_bytes + uint32_t(g.stages) * g.b_stage_bytes + EPI_BYTES +
         (2 * g.stages + 9) * 8 + 16 + kMaxGroups * 8 + kMaxKhg * kMaxPhases * 4 + 1024;
}

// Geometry for one staging choice: each pipeline stage carries `bk` input
// channels and `khs` filter rows (khs = 1: one stage per filter row;
// khs = KH: the whole filter, so one staged activation tile feeds every tap).
static int floor_div(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

// Phases ph in [0, s) with (kh - pad) mod s == ph for some filter tap kh,
// and the range [d0, d1] of (kh - pad - ph) / s.
static void phases(int K, int pad, int s, int &n, int *ph, int &d0, int &d1) {
  bool used[4] = {false, false, false, false};
  for (int k = 0; k < K; ++k) used[(((k - pad) % s) + s) % s] = true;
  n = 0;
  for (int q = 0; q < s; ++q)
    if (used[q]) ph[n++] = q;
  d0 = floor_div(-pad, s);
  d1 = floor_div(K - 1 - pad, s);
}

static UmmaGeom geom_for(const wgx_conv2d_params &p, int khs, int bk, int trans, int hs = 0,
                         bool no_resident = false) {
  UmmaGeom g{};
  g.trans = trans;
  if (trans) {
    // G M blocks per tile, interleaved MMA by MMA: 8 for N = 16 / 32, 4 for
    // N = 64 (a tile's accumulator then spans 128 or 256 TMEM columns)
    g.NT = p.OC <= 16 ? 16 : p.OC <= 32 ? 32 : 64;
    g.lgNT = g.NT == 16 ? 4 : g.NT == 32 ? 5 : 6;
    g.G = g.NT == 64 ? 4 : 8;
    g.tile_pos = 128 * g.G;
    g.wrows = g.NT;
    g.acc_cols = g.G * g.NT;
  } else {
    g.NT = UN;
    g.G = 1;
    g.tile_pos = UN;
    g.wrows = UM;
    g.acc_cols = UN;
  }
  g.B = p.B;
  g.IH = p.IH;
  g.IW = p.IW;
  g.OC = p.OC;
  g.OH = p.OH;
  g.OW = p.OW;
  g.sH = p.sH;
  g.sW = p.sW;
  g.xIC = p.IC;
  g.xKH = p.KH;
  g.xKW = p.KW;
  g.xpH = p.pH;
  g.xpW = p.pW;
  if (p.sH == 1 && p.sW == 1) {
    g.IC = p.IC;
    g.KH = p.KH;
    g.KW = p.KW;
    g.dH = p.dH;
    g.dW = p.dW;
    g.pH = p.pH;
    g.pW = p.pW;
    g.nphH = g.nphW = 1;
    g.Hp = p.IH + 2 * p.pH;
    g.Wp = p.IW + 2 * p.pW;
  } else {
    int d0h, d1h, d0w, d1w;
    phases(p.KH, p.pH, p.sH, g.nphH, g.phH, d0h, d1h);
    phases(p.KW, p.pW, p.sW, g.nphW, g.phW, d0w, d1w);
    g.IC = g.nphH * g.nphW * p.IC;
    g.KH = d1h - d0h + 1;
    g.KW = d1w - d0w + 1;
    g.dH = g.dW = 1;
    g.pH = -d0h;
    g.pW = -d0w;
    g.Hp = p.OH + g.KH - 1;
    g.Wp = p.OW + g.KW - 1;
  }
  // transposed variant: the padded row pitch is rounded up to a multiple of
  // 8 (extra zero columns, whose outputs are discarded), so that 8-position
  // groups never straddle an output row (vector epilogue stores), when that
  // adds at most 1/6 of the positions for unfolded stride-1 filters, whose
  // NCHW and residual stores otherwise take the 2-byte path (YOLO26-N
  // bottlenecks on 80^2 / 40^2 planes: pitch 82 -> 88, 42 -> 48, 30 % faster
  // measured), and at most 5 % for strided and folded ones, whose MMA work
  // grows with the pitch while their stores gain less. 1x1 stride-1
  // unpadded convolutions keep Wp = IW: the direct mode reads NCHW rows as
  // they are.
  const bool plain_1x1 =
      p.KH == 1 && p.KW == 1 && p.sH == 1 && p.sW == 1 && p.pH == 0 && p.pW == 0;
  const int wp8 = (g.Wp + 7) / 8 * 8;
  const int pitch_div = (hs || p.sH != 1 || p.sW != 1) ? 20 : 6;
  if (trans && !plain_1x1 && (wp8 - g.Wp) * pitch_div <= g.Wp) g.Wp = wp8;
  if (hs) {
    // filter columns folded into N (stride 1, dW = 1, KW = hs): the
    // pipeline runs a KW = 1 convolution with N = hs*ocp columns per M block
    g.hs = hs;
    // ocp = 8 / 16 / 32 / 64: N = 32 / 48 / 96 / 192 with 8 / 4 / 2 / 1 M
    // blocks (two accumulators fit TMEM; 8 (M block, 8-channel) epilogue
    // items per tile)
    g.ocp = p.OC <= 8 ? 8 : p.OC <= 16 ? 16 : p.OC <= 32 ? 32 : 64;
    g.NT = (hs * g.ocp + 15) / 16 * 16;
    g.G = g.ocp == 8 ? 8 : g.ocp == 16 ? 4 : g.ocp == 32 ? 2 : 1;
    g.lgNT = 0;
    g.tile_pos = 128 * g.G;
    g.wrows = g.NT;
    g.acc_cols = g.G * g.NT;
    g.KW = 1;
  }
  if (khs <= 0) khs = g.KH;
  g.bk = bk;
  g.chunks = bk / 8;
  g.khs = khs;
  g.n_khg = g.KH / khs;
  g.C8 = (g.IC + bk - 1) / bk * bk;
  g.ncb = g.C8 / bk;
  g.n_oct = (p.OC + g.wrows - 1) / g.wrows;
  g.plane_rows = (long long)g.Hp * g.Wp;
  long long p_out = (long long)(p.OH - 1) * g.Wp + p.OW;
  if (trans && !hs && g.G == 8 && p_out <= 512) {
    // small planes: 4 M blocks (512 positions) instead of 8, most of whose
    // positions would lie past the image
    g.G = 4;
    g.tile_pos = 128 * g.G;
    g.acc_cols = g.G * g.NT;
  }
  g.tile_stride = hs ? g.tile_pos - 8 : g.tile_pos;
  g.tiles_per_img = int((p_out + g.tile_stride - 1) / g.tile_stride);
  g.wp_magic = 0;
  if (g.Wp >= 2) {
    const uint64_t m = ((1ull << 32) + uint64_t(g.Wp) - 1) / uint64_t(g.Wp);
    const uint64_t e = m * uint64_t(g.Wp) - (1ull << 32);
    const uint64_t pos_max = uint64_t(g.tiles_per_img) * g.tile_stride + g.tile_pos;
    if (m < (1ull << 32) && pos_max * e < (1ull << 32)) g.wp_magic = uint32_t(m);
  }
  g.total_tiles = g.tiles_per_img * g.n_oct * g.B;
  long long r = g.tile_pos + (long long)(khs - 1) * g.dH * g.Wp + (long long)(g.KW - 1) * g.dW;
  g.R = r > (1 << 20) ? (1 << 20) : int(r);
  g.R_alloc = (g.R + 7) / 8 * 8;
  g.a_stage_bytes = uint32_t(khs * g.KW) * g.chunks * g.wrows * 16;
  g.b_stage_bytes = uint32_t(g.chunks) * g.R_alloc * 16;
  g.n_kstages = g.n_khg * g.ncb;
  // resident weights: one oc tile, all stages' A blocks plus >= 2 B stages
  uint64_t w_all = uint64_t(g.n_kstages) * g.a_stage_bytes;
  g.resident = 0;
  g.stages = 0;
  if (g.n_oct == 1 && w_all < SMEM_MAX && !no_resident) {
    g.w_region_bytes = uint32_t(w_all);
    g.stages = 2;
    if (smem_need(g) <= SMEM_MAX) {
      g.resident = 1;
      // stages are reused across tiles, so short filters (few stages per
      // tile) still prefetch the next tiles' activations
      while (g.stages < 6) {
        ++g.stages;
        if (smem_need(g) > SMEM_MAX) {
          --g.stages;
          break;
        }
      }
    }
  }
  if (!g.resident) {
    g.stages = 1;
    g.w_region_bytes = g.a_stage_bytes;
    while (g.stages < 6) {
      g.stages += 1;
      g.w_region_bytes = uint32_t(g.stages) * g.a_stage_bytes;
      if (smem_need(g) > SMEM_MAX) {
        g.stages -= 1;
        g.w_region_bytes = uint32_t(g.stages) * g.a_stage_bytes;
        break;
      }
    }
  }
  // tap masks of channels-on-M space-to-depth stages (the rule of the weight
  // packing); the positions-on-M variant issues short MMAs whose rate
  // depends on full stages, so it keeps every tap
  g.tapskip = 0;
  g.cbpp = 1;
  const int nph = g.nphH * g.nphW;
  // (positions-on-M: only with the generic staging, whose per-stage MMA
  // group lists are compacted per filter-row group and phase and must fit
  // the group table after the full list)
  const int ngroups_ = g.khs * g.KW * (g.bk / 16);
  const bool spec_ = g.khs == 1 && g.bk == 32 && g.KW <= 3;
  const bool trans_ok = !spec_ && ngroups_ <= kSeqGroups &&
                        ngroups_ * (1 + g.n_khg * g.nphH * g.nphW) <= kMaxGroups;
  if ((!trans || trans_ok) && nph > 1 && g.xIC % g.bk == 0 && g.n_khg <= kMaxKhg &&
      nph <= kMaxPhases && g.khs * g.KW <= 16) {
    g.cbpp = g.xIC / g.bk;
    for (int khg = 0; khg < g.n_khg; ++khg)
      for (int ph = 0; ph < nph; ++ph) {
        uint16_t m = 0;
        for (int khl = 0; khl < g.khs; ++khl) {
          const int rkh = g.sH * (khg * g.khs + khl - g.pH) + g.phH[ph / g.nphW] + g.xpH;
          if (rkh < 0 || rkh >= g.xKH) continue;
          for (int kw = 0; kw < g.KW; ++kw) {
            const int rkw = g.sW * (kw - g.pW) + g.phW[ph % g.nphW] + g.xpW;
            if (rkw >= 0 && rkw < g.xKW) m |= uint16_t(1u << (khl * g.KW + kw));
          }
        }
        g.tapmask[khg][ph] = m;
        if (m != uint16_t((1u << (g.khs * g.KW)) - 1)) g.tapskip = 1;
      }
  }
  g.has_bias = p.has_bias;
  g.act = p.act;
  g.lo = p.out_min;
  g.hi = p.out_max;
  return g;
}

// Filter columns folded into N (UmmaGeom::hs): stride-1 3-wide filters of
// the positions-on-M variant (OC <= 64) without dilation across, where it
// pays. The fold cuts the MMAs per position threefold (their cost grows
// with the 16-channel input blocks) but its epilogue costs about as much
// per tile and 8 output channels as a 3x3 filter's MMAs per 16 input
// channels cost unfolded at N = 16 (measured per role on B200: ~3 K cycles
// per tile and 8-channel chunk, against ~5.8 K cycles of unfolded MMAs per
// 1024 positions and input block): folded when ocp < 14 * ceil(IC / 16),
// and on small planes up to ocp = 16 * ceil(IC / 16) (below).
// The environment variable WGX_CONV_HSUM=0 turns the fold off, =2 applies
// it wherever it is possible (both forms compute the same convolution).
static bool hsum_eligible(const wgx_conv2d_params &p) {
  static const int mode = [] {
    const char *e = std::getenv("WGX_CONV_HSUM");
    return (e && e[0] == '0') ? 0 : (e && e[0] == '2') ? 2 : 1;
  }();
  if (!mode || p.OC > 64 || p.sH != 1 || p.sW != 1 || p.dW != 1 || p.KW != 3 || p.groups != 1)
    return false;
  const int ocp = p.OC <= 8 ? 8 : p.OC <= 16 ? 16 : p.OC <= 32 ? 32 : 64;
  const int c16 = (p.IC + 15) / 16;
  // planes of at most 512 flattened positions fit inside one unfolded tile
  // of 4 M blocks; the fold's smaller tiles spread them over more SMs
  // (64 -> 64 channels at 20^2: 31 -> 23 us measured), so there it is
  // taken up to ocp = 16 * ceil(IC / 16)
  const long long p_out = (long long)(p.OH - 1) * (p.IW + 2 * p.pW) + p.OW;
  return mode == 2 || ocp < 14 * c16 || (p_out <= 512 && ocp <= 16 * c16);
}

// 64-channel stages for channels-on-M convolutions (input channels a
// multiple of 64): WGX_CONV_BK64=0 never, =1 (default) 1x1 filters with at
// least 256 input channels, =2 1x1 filters with at least 192, =3 1x1
// filters, =4 every filter size (all forms compute the same convolution).
static bool bk64_wanted(const wgx_conv2d_params &p) {
  static const int mode = [] {
    const char *e = std::getenv("WGX_CONV_BK64");
    return (e && e[0] >= '0' && e[0] <= '4') ? e[0] - '0' : 1;
  }();
  const bool one = p.KH == 1 && p.KW == 1;
  switch (mode) {
    case 0: return false;
    case 1: return one && p.IC >= 256;
    case 2: return one && p.IC >= 192;
    case 3: return one;
    default: return true;
  }
}

// Copy issue of the activation stages: WGX_CONV_SPLIT=0 one issuing
// thread, =1 (default) several (the same copies either way).
static int split_mode() {
  static const int mode = [] {
    const char *e = std::getenv("WGX_CONV_SPLIT");
    return (e && e[0] >= '0' && e[0] <= '1') ? e[0] - '0' : 1;
  }();
  return mode;
}

// Pick the staging: per-filter-row stages of 32 channels measured fastest
// on config 2 (41 % tensor-pipe activity against 30 % for whole-filter
// stages of 16 channels); whole-filter and 16-channel stages are the
// fallbacks for shapes where fewer than three 32-channel stages fit.
// per_image_w: the weights differ per image (batched GEMM), so they are
// streamed per stage, never resident.
static UmmaGeom make_geom(const wgx_conv2d_params &p, bool per_image_w = false) {
  // (khs, bk); khs 0 = the whole filter. Below 16 (virtual) channels,
  // 16-channel stages halve the zero padding of the K dimension.
  int cand[4][2] = {{1, 32}, {0, 16}, {1, 16}, {0, 32}};
  const int trans = p.OC <= 64 ? 1 : 0;
  const int hs = hsum_eligible(p) ? p.KW : 0;
  if (hs) {
    // one MMA per filter row: whole-filter stages keep several MMAs per
    // stage (per-stage waits and commits cost several MMA times)
    const int c4[4][2] = {{0, 32}, {0, 16}, {1, 32}, {1, 16}};
    std::memcpy(cand, c4, sizeof cand);
    if (p.IC <= 16) std::swap(cand[0][1], cand[1][1]);
  } else if (geom_for(p, 1, 32, trans).IC <= 16) {
    if (trans) {
      // positions on M with at most 16 (virtual) channels: one stage per
      // filter row carries only KW x G MMAs, and each stage's wait, fence
      // and commit cost several MMA times; whole-filter stages measured
      // faster on every such YOLO26-N layer (stem 235 -> 225 us, 8 -> 16
      // channels at 160^2 74 -> 63 us, 16 -> 16 at 80^2 41 -> 37 us)
      const int c4[4][2] = {{0, 16}, {1, 16}, {1, 32}, {0, 32}};
      std::memcpy(cand, c4, sizeof cand);
    } else {
      cand[0][1] = 16;
      cand[2][1] = 32;
    }
  } else if (!trans && p.IC % 64 == 0 && bk64_wanted(p)) {
    // channels on M, input channels a multiple of 64: 64-channel stages.
    // The per-SM copy engine finishes pipeline stages at a roughly fixed
    // cost per barrier round and per copy (measured on B200: 4 KB copies,
    // four to a stage, feed ~11 B/clk per SM; 8 KB copies ~20 B/clk), so
    // twice the bytes per stage and per copy (8 KB boxes, 8 KB chunk rows)
    // nearly double what the tensor cores are fed (1x1 layers of YOLO26-N
    // at batch 64: 512 -> 256 at 20^2 40.0 -> 29.8 us, 384 -> 128 at 40^2
    // 48.1 -> 40.2 us). With at most two stages per tile (128 input
    // channels) and for 3x3 filters they measured slower, and 128-channel
    // stages for 512 input channels and whole-filter 32-channel stages
    // for 3x3 filters no faster.
    const int c4[4][2] = {{1, 64}, {1, 32}, {0, 16}, {1, 16}};
    std::memcpy(cand, c4, sizeof cand);
  } else if (trans && (p.sH > 1 || p.sW > 1)) {
    // strided, positions on M, more than 16 virtual channels: whole-filter
    // stages of 32 channels first (the 64 -> 64 / stride-2 layer of
    // YOLO26-N at 160^2: 102 -> 85 us against 16-channel stages; stride-1
    // layers measured neutral and keep the per-row order)
    const int c4[4][2] = {{0, 32}, {0, 16}, {1, 32}, {1, 16}};
    std::memcpy(cand, c4, sizeof cand);
  }
  UmmaGeom best{};
  bool have = false;
  for (int min_stages : {3, 2}) {
    for (auto &c : cand) {
      UmmaGeom g = geom_for(p, c[0], c[1], trans, hs, per_image_w);
      if (g.stages >= min_stages && smem_need(g) <= SMEM_MAX && g.R_alloc * 16 < (1 << 18)) {
        return g;
      }
      if (!have) {
        best = g;
        have = true;
      }
    }
  }
  return best;
}

// Dynamic shared memory of one CTA; never below 120 KB so that exactly one
// CTA is resident per SM (the 512-column TMEM allocation never waits).
static uint32_t smem_bytes(const UmmaGeom &g) {
  uint32_t need = smem_need(g);
  return need < 120u * 1024u ? 120u * 1024u : need;
}

bool umma_conv_supported(const wgx_conv2d_params &p, bool per_image_w) {
  if (p.dtype != WGX_FLOAT16 || p.groups != 1) return false;
  if (p.sH < 1 || p.sW < 1 || p.sH > 4 || p.sW > 4) return false;
  if (p.dH < 1 || p.dW < 1 || p.pH < 0 || p.pW < 0) return false;
  if (p.sH == 1 && p.sW == 1) {
    if (p.IC < 8) return false;
    // stride-1 geometry must be consistent with the padded flattening
    if (p.OH != p.IH + 2 * p.pH - p.dH * (p.KH - 1)) return false;
    if (p.OW != p.IW + 2 * p.pW - p.dW * (p.KW - 1)) return false;
  } else {
    // strided: space-to-depth view, dilation 1
    if (p.dH != 1 || p.dW != 1) return false;
    if (p.IH + 2 * p.pH < p.KH || p.IW + 2 * p.pW < p.KW) return false;
    if (p.OH != (p.IH + 2 * p.pH - p.KH) / p.sH + 1) return false;
    if (p.OW != (p.IW + 2 * p.pW - p.KW) / p.sW + 1) return false;
  }
  UmmaGeom g = make_geom(p, per_image_w);
  if (g.KW > MAX_KW || g.IC < 8) return false;
  if (g.khs * g.KW * (g.bk / 16) > kMaxGroups) return false;
  if (g.stages < 2) return false;
  if (smem_need(g) > SMEM_MAX) return false;
  if (g.R_alloc * 16 >= (1 << 18)) return false;  // LBO field range
  if (g.total_tiles < 1) return false;
  // positions and per-image output offsets are handled in 32-bit integers
  if ((long long)g.tiles_per_img * g.tile_pos + g.plane_rows >= (1ll << 31)) return false;
  if ((long long)g.OH * g.OW >= (1ll << 31)) return false;
  return true;
}

static int sm_count() {
  int dev = 0, n = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "SM count");
  return n;
}

std::string umma_conv_describe(const wgx_conv2d_params &p) {
  const UmmaGeom g = make_geom(p);
  char buf[256];
  snprintf(buf, sizeof buf,
           "umma %s N=%d G=%d tile=%d positions bk=%d khs=%d stages=%d/%d kstages=%d%s%s%s "
           "Wp=%d tiles=%d",
           g.trans ? "positions-on-M" : "channels-on-M", g.trans ? g.NT : UN, g.G, g.tile_pos,
           g.bk, g.khs, g.stages, g.n_kstages, g.n_kstages, g.resident ? " resident" : "",
           g.tapskip ? " tapskip" : "", g.hs ? " kw-folded" : "", g.Wp, g.total_tiles);
  return buf;
}

uint64_t umma_conv_grid(const wgx_conv2d_params &p) {
  UmmaGeom g = make_geom(p);
  return uint64_t(g.total_tiles);
}

uint64_t umma_conv_packed_weight_bytes(const wgx_conv2d_params &p, bool per_image_w) {
  UmmaGeom g = make_geom(p, per_image_w);
  return uint64_t(g.n_oct) * g.n_kstages * g.a_stage_bytes;
}

// Rows the main kernel may read: the last tile's B stage of the last filter
// row starts at (tiles-1)*tile_pos + (KH-1)*dH*Wp and spans R rows. Rows past the
// image only feed output positions that are discarded.
static uint64_t input_rows_total(const UmmaGeom &g) {
  uint64_t planes = uint64_t(g.B) * (g.C8 / 8);
  uint64_t last_end = uint64_t(g.tiles_per_img - 1) * g.tile_stride +
                      uint64_t(g.n_khg - 1) * g.khs * g.dH * g.Wp + g.R;
  uint64_t slack = last_end > uint64_t(g.plane_rows) ? last_end - g.plane_rows : 0;
  return planes * g.plane_rows + slack;
}

uint64_t umma_conv_input_bytes(const wgx_conv2d_params &p, bool per_image_w) {
  UmmaGeom g = make_geom(p, per_image_w);
  return (input_rows_total(g) * 16 + 255) / 256 * 256;
}

// --------------------------------------------------------------- re-layout
// Plane (b, c) of the (possibly concatenated) input: the source holding
// channel c and c's channel within it.
__device__ __forceinline__ const __half *src_plane(const UmmaGeom &g, long long b, int c) {
  int s = 0;
#pragma unroll
  for (int k = 1; k < kMaxSrc; ++k)
    if (k < g.nsrc && c >= g.src_c0[k]) s = k;
  const int cs = g.src_c0[s + 1] - g.src_c0[s];
  return g.src[s] + (b * cs + (c - g.src_c0[s])) * (long long)g.IH * g.IW;
}

// xs[b][cb][hp][wp][8] <- x[b][c][hp-pH][wp-pW], zero outside the image and
// for channels >= IC. One thread per 16-byte row slot; consecutive threads
// take consecutive wp, so the 2-byte gathers of one channel are coalesced
// and the 16-byte stores are contiguous.
__global__ void pack_input(UmmaGeom g, const __half *__restrict__ x, uint4 *__restrict__ xs,
                           long long n_slots) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_slots) return;
  int wp = int(i % g.Wp);
  long long t = i / g.Wp;
  int hp = int(t % g.Hp);
  t /= g.Hp;
  int cb = int(t % (g.C8 / 8));
  long long b = t / (g.C8 / 8);
  int ih = hp - g.pH, iw = wp - g.pW;
  __align__(16) __half v[8];
  bool inside = ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    int c = cb * 8 + e;
    v[e] = (inside && c < g.IC) ? src_plane(g, b, c)[(long long)ih * g.IW + iw]
                                : __float2half_rn(0.f);
  }
  if (WGX_IN_BOUNDS(xs + i, 16, xs, g.xs_bytes, g.err)) xs[i] = *reinterpret_cast<const uint4 *>(v);
}

// Warp-cooperative store of 4 consecutive 16-byte slots per lane: lane l's
// slots k (lo_l <= k < hi_l) go to dst_l + k. Written directly, every warp
// store would put 16 bytes into each of 32 lines 64 bytes apart; staged in
// the warp's 2 KB of shared memory (16-byte units XOR-swizzled within each
// 128 bytes: conflict-free both ways), each store instruction writes 32
// consecutive entries (lane l's run continues lane l + 1's when they share a
// row, which is the common case). All 32 lanes must call it.
__device__ __forceinline__ int slot_swz(int j) { return j ^ ((j >> 3) & 7); }
__device__ __forceinline__ void warp_store4(const UmmaGeom &g, const uint4 *xs, uint4 *wbuf,
                                            const uint4 (&v)[4], uint4 *dst, int lo, int hi) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; ++k) wbuf[slot_swz(lane * 4 + k)] = v[k];
  __syncwarp();
  const unsigned long long dptr = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int j = m * 32 + lane, t = j >> 2, k = j & 3;
    const unsigned long long d = __shfl_sync(0xffffffffu, dptr, t);
    const int tlo = __shfl_sync(0xffffffffu, lo, t), thi = __shfl_sync(0xffffffffu, hi, t);
    if (k >= tlo && k < thi &&
        WGX_IN_BOUNDS(reinterpret_cast<uint4 *>(d) + k, 16, xs, g.xs_bytes, g.err))
      reinterpret_cast<uint4 *>(d)[k] = wbuf[slot_swz(j)];
  }
  __syncwarp();
}

// Vector form of pack_input for IW % 4 == 0: one thread re-lays 4
// consecutive padded positions of one 8-channel block. The first position
// wp0 = 4t + (pW % 4) - 4 is chosen so that its input column iw0 = wp0 - pW
// is a multiple of 4: each channel row contributes one aligned 8-byte load,
// the 8x4 block is transposed in registers (prmt) and written as four
// 16-byte slots (64 contiguous bytes). Positions outside [0, Wp) are
// skipped; padding positions and channels >= IC are written as zeros.
__global__ void __launch_bounds__(256)
    pack_input_v4(UmmaGeom g, const __half *__restrict__ x, uint4 *__restrict__ xs,
                  int groups_per_row, long long n_threads) {
  __shared__ uint4 wstage[8][128];
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = i < n_threads;
  if (!active) i = n_threads - 1;  // inactive lanes still join the warp store
  const int t = int(i % groups_per_row);
  long long r = i / groups_per_row;
  const int hp = int(r % g.Hp);
  r /= g.Hp;
  const int cb = int(r % (g.C8 / 8));
  const long long b = r / (g.C8 / 8);
  const int wp0 = 4 * t + (g.pW & 3) - 4;
  const int iw0 = wp0 - g.pW;
  const int ih = hp - g.pH;
  const bool row_in = ih >= 0 && ih < g.IH;
  uint2 ch[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int c = cb * 8 + e;
    ch[e] = make_uint2(0u, 0u);
    if (row_in && c < g.IC) {
      const __half *src = src_plane(g, b, c) + (long long)ih * g.IW;
      if (iw0 >= 0 && iw0 + 3 < g.IW) {
        ch[e] = *reinterpret_cast<const uint2 *>(src + iw0);
      } else {
        __align__(8) __half v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int iw = iw0 + k;
          v[k] = (iw >= 0 && iw < g.IW) ? src[iw] : __float2half_rn(0.f);
        }
        ch[e] = *reinterpret_cast<const uint2 *>(v);
      }
    }
  }
  uint4 *dst = xs + ((b * (g.C8 / 8) + cb) * g.Hp + hp) * (long long)g.Wp + wp0;
  uint4 vv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    // halves of position k: low (k even) or high (k odd) half of word k/2
    const uint32_t sel = (k & 1) ? 0x7632u : 0x5410u;
    const bool lo = k < 2;
    vv[k] = make_uint4(__byte_perm(lo ? ch[0].x : ch[0].y, lo ? ch[1].x : ch[1].y, sel),
                       __byte_perm(lo ? ch[2].x : ch[2].y, lo ? ch[3].x : ch[3].y, sel),
                       __byte_perm(lo ? ch[4].x : ch[4].y, lo ? ch[5].x : ch[5].y, sel),
                       __byte_perm(lo ? ch[6].x : ch[6].y, lo ? ch[7].x : ch[7].y, sel));
  }
  // positions outside [0, Wp) are skipped
  const int klo = active ? max(0, -wp0) : 4, khi = active ? min(4, g.Wp - wp0) : 0;
  warp_store4(g, xs, wstage[threadIdx.x >> 5], vv, dst, klo, khi);
}

// Vector form of pack_input for IW % 8 == 0: one thread re-lays 8
// consecutive padded positions of one 8-channel block. The first position
// wp0 = 8t + (pW % 8) - 8 is chosen so that its input column iw0 = wp0 - pW
// is a multiple of 8: each channel row contributes one aligned 16-byte load,
// the 8x8 block is transposed in registers (prmt) and written as eight
// 16-byte slots (128 contiguous bytes). Positions outside [0, Wp) are
// skipped; padding positions and channels >= IC are written as zeros.
__device__ __forceinline__ void pack_weights_body(const UmmaGeom &g, const __half *__restrict__ w,
                                                  uint4 *__restrict__ packed, int i);

// One launch re-lays the input and, when `w` is not null, packs the weights
// (blocks past n_in_blocks): the small weight packing costs no launch of its
// own on the per-call path. Each input thread handles one 8-position group
// of one padded row (b, 8-channel block, hp); index math is 32-bit (the
// host checks the ranges). The CTA's items are consecutive (row, group)
// pairs, so the slots they write form one contiguous run of xs: the threads
// put their slots in shared memory (16-byte units XOR-swizzled within each
// 128 bytes, so that a thread's 8 consecutive slots and 8 threads' equal
// slots fall in distinct banks) and the CTA then stores the run with
// coalesced 16-byte writes (a thread's own 8 slots, written directly, would
// make every warp store touch 32 different 128-byte lines).
constexpr int PACK_SLOTS = 256 * 8;
__device__ __forceinline__ int pack_swz(int s) { return s ^ ((s >> 3) & 7); }

__global__ void __launch_bounds__(256, 4)
    pack_input_v8(UmmaGeom g, const __half *__restrict__ x, uint4 *__restrict__ xs,
                  int groups_per_row, int n_items, int n_in_blocks,
                  const __half *__restrict__ w, uint4 *__restrict__ packed, int n_w) {
  if (int(blockIdx.x) >= n_in_blocks) {
    const int i = (int(blockIdx.x) - n_in_blocks) * 256 + threadIdx.x;
    if (w && i < n_w) pack_weights_body(g, w, packed, i);
    return;
  }
  __shared__ uint4 stage[PACK_SLOTS];
  const int ipw = g.pW & 7;
  // the CTA's slot run [s0, s1]
  const int item0 = blockIdx.x * 256;
  const int item1 = min(n_items, item0 + 256) - 1;
  const int r0 = item0 / groups_per_row, r1 = item1 / groups_per_row;
  const long long s0 = (long long)r0 * g.Wp + max(0, 8 * (item0 - r0 * groups_per_row) + ipw - 8);
  const long long s1 =
      (long long)r1 * g.Wp + min(g.Wp - 1, 8 * (item1 - r1 * groups_per_row) + ipw - 1);
  const int item = item0 + threadIdx.x;
  if (item < n_items) {
    const int row = item / groups_per_row;
    const int t = item - row * groups_per_row;
    const int ncb = g.C8 / 8;
    const int hp = row % g.Hp;
    const int rest = row / g.Hp;
    const int cb = rest % ncb, b = rest / ncb;
    const int ih = hp - g.pH;
    const bool row_in = ih >= 0 && ih < g.IH;
    const int nch = min(8, g.IC - cb * 8);
    const size_t cstride = size_t(g.IH) * g.IW;
    // every 8-channel block lies in one source (source boundaries are multiples of 8)
    const __half *src0 = (nch > 0 ? src_plane(g, b, cb * 8) : x) + size_t(row_in ? ih : 0) * g.IW;
    const int wp0 = 8 * t + ipw - 8;
    const int iw0 = wp0 - g.pW;  // a multiple of 8
    // IW % 8 == 0 and iw0 % 8 == 0: the 16-byte chunk [iw0, iw0 + 8) lies
    // either entirely inside the input row or entirely in the padding
    const bool inside = row_in && iw0 >= 0 && iw0 < g.IW;
    uint4 ch[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      ch[e] = (inside && e < nch) ? *reinterpret_cast<const uint4 *>(src0 + e * cstride + iw0)
                                  : make_uint4(0u, 0u, 0u, 0u);
    const int srow = int((long long)row * g.Wp - s0);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int wp = wp0 + k;
      if (wp < 0 || wp >= g.Wp) continue;
      // position k sits in word k/2 of every channel vector, low or high half
      const uint32_t sel = (k & 1) ? 0x7632u : 0x5410u;
      uint32_t wd[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint4 &v = ch[e];
        wd[e] = (k >> 1) == 0 ? v.x : (k >> 1) == 1 ? v.y : (k >> 1) == 2 ? v.z : v.w;
      }
      stage[pack_swz(srow + wp)] =
          make_uint4(__byte_perm(wd[0], wd[1], sel), __byte_perm(wd[2], wd[3], sel),
                     __byte_perm(wd[4], wd[5], sel), __byte_perm(wd[6], wd[7], sel));
    }
  }
  __syncthreads();
  const int n = int(s1 - s0 + 1);
  uint4 *dst = xs + s0;
  for (int i = threadIdx.x; i < n; i += 256)
    if (WGX_IN_BOUNDS(dst + i, 16, xs, g.xs_bytes, g.err)) dst[i] = stage[pack_swz(i)];
}

// Space-to-depth re-layout for stride 2 with few input channels (XIC < 8,
// e.g. an RGB stem): one thread takes staged row hp of image b and four
// consecutive positions wp = q0 + pW .. q0 + pW + 3 (input columns 2*q0 ..
// 2*q0 + 7, q0 a multiple of 4): one aligned 16-byte load per input channel
// and row phase, then the C8/8 slots (8 virtual channels each) of the four
// positions. Virtual channel vc = (2*ph + pw)*XIC + c, all index math
// compile-time in XIC.
template <int XIC>
__global__ void __launch_bounds__(256)
    pack_input_s2d_small(UmmaGeom g, uint4 *__restrict__ xs, int groups_per_row, int qbase,
                         int n_items) {
  __shared__ uint4 wstage[8][128];
  int item = blockIdx.x * 256 + threadIdx.x;
  const bool active = item < n_items;
  if (!active) item = n_items - 1;  // inactive lanes still join the warp stores
  const int t = item % groups_per_row;
  const int r = item / groups_per_row;
  const int hp = r % g.Hp, b = r / g.Hp;
  const int q0 = 4 * t + qbase;
  const int iw0 = 2 * q0;  // a multiple of 8: the 8 columns are all in or all out
  const bool col_in = iw0 >= 0 && iw0 < g.IW;
  uint4 v[2][XIC];
#pragma unroll
  for (int ph = 0; ph < 2; ++ph) {
    const int ih = 2 * (hp - g.pH) + ph;
    const bool in = col_in && ih >= 0 && ih < g.IH;
#pragma unroll
    for (int c = 0; c < XIC; ++c)
      v[ph][c] = in ? *reinterpret_cast<const uint4 *>(src_plane(g, b, c) + (long long)ih * g.IW + iw0)
                    : make_uint4(0u, 0u, 0u, 0u);
  }
  const int planes = g.C8 / 8;
  const size_t plane_rows = size_t(g.Hp) * g.Wp;
  const int wp0 = q0 + g.pW;
  // positions outside [0, Wp) are skipped
  const int klo = active ? max(0, -wp0) : 4, khi = active ? min(4, g.Wp - wp0) : 0;
#pragma unroll
  for (int pl = 0; pl < 4; ++pl) {
    if (pl >= planes) break;  // uniform across the CTA
    uint4 vv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t w32[4];
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        uint32_t h2 = 0;
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int vc = pl * 8 + 2 * e2 + hi;
          uint32_t hv = 0;
          if (vc < 4 * XIC) {
            const int phase = vc / XIC, c = vc % XIC;
            const uint4 &src = v[phase >> 1][c];
            // column 2k + pw of the 8 loaded: half pw of word k
            const uint32_t word = k == 0 ? src.x : k == 1 ? src.y : k == 2 ? src.z : src.w;
            hv = (phase & 1) ? (word >> 16) : (word & 0xffffu);
          }
          h2 |= hv << (16 * hi);
        }
        w32[e2] = h2;
      }
      vv[k] = make_uint4(w32[0], w32[1], w32[2], w32[3]);
    }
    warp_store4(g, xs, wstage[threadIdx.x >> 5], vv,
                xs + (size_t(b) * planes + pl) * plane_rows + size_t(hp) * g.Wp + wp0, klo, khi);
  }
}

// packed[oct][khg][cb][kh_local][kw][chunk][row < wrows][8] <- w[oc][c][kh][kw]
// (kh = khg*khs + kh_local): one pipeline stage's A operand is contiguous.
__device__ __forceinline__ void pack_weights_body(const UmmaGeom &g, const __half *__restrict__ w,
                                                  uint4 *__restrict__ packed, int i) {
  const int row = i % g.wrows;
  int t = i / g.wrows;
  const int chunk = t % g.chunks;
  t /= g.chunks;
  const int kw = t % g.KW;
  t /= g.KW;
  const int khl = t % g.khs;
  t /= g.khs;
  const int cb = t % g.ncb;
  t /= g.ncb;
  const int khg = t % g.n_khg;
  const int oct = t / g.n_khg;
  const int kh = khg * g.khs + khl;
  __align__(16) __half v[8];
  if (g.hs) {
    // folded filter columns: row = kw*ocp + oc (stride 1, one output tile)
    const int fkw = row / g.ocp, foc = row - fkw * g.ocp;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = cb * g.bk + chunk * 8 + e;
      v[e] = (fkw < g.hs && foc < g.OC && c < g.IC)
                 ? w[((size_t(foc) * g.IC + c) * g.xKH + kh) * g.xKW + fkw]
                 : __float2half_rn(0.f);
    }
    packed[i] = *reinterpret_cast<const uint4 *>(v);
    return;
  }
  const int oc = oct * g.wrows + row;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int cv = cb * g.bk + chunk * 8 + e;  // virtual channel
    __half val = __float2half_rn(0.f);
    if (oc < g.OC && cv < g.IC) {
      // virtual channel -> (phase, real channel); virtual tap -> real tap
      // (stride 1: one phase, identity)
      const int phase = cv / g.xIC, c = cv - phase * g.xIC;
      const int ph = g.phH[phase / g.nphW], pw = g.phW[phase % g.nphW];
      const int rkh = g.sH * (kh - g.pH) + ph + g.xpH;
      const int rkw = g.sW * (kw - g.pW) + pw + g.xpW;
      if (rkh >= 0 && rkh < g.xKH && rkw >= 0 && rkw < g.xKW)
        val = w[((size_t(oc) * g.xIC + c) * g.xKH + rkh) * g.xKW + rkw];
    }
    v[e] = val;
  }
  packed[i] = *reinterpret_cast<const uint4 *>(v);
}

// ------------------------------------------------- space-to-depth re-layout
// xs[b][cb][hp][wp][8] <- phase (ph, pw) of input channel c at
// x[b][c][sH*(hp-pH)+ph][sW*(wp-pW)+pw] for virtual channel
// cv = (phase index)*IC + c, zero outside the image and for cv >= the
// virtual channel count. One thread per 16-byte slot (any shape).
__global__ void pack_input_s2d(UmmaGeom g, const __half *__restrict__ x, uint4 *__restrict__ xs,
                               long long n_slots) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_slots) return;
  const int wp = int(i % g.Wp);
  long long t = i / g.Wp;
  const int hp = int(t % g.Hp);
  t /= g.Hp;
  const int cb = int(t % (g.C8 / 8));
  const long long b = t / (g.C8 / 8);
  __align__(16) __half v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int cv = cb * 8 + e;
    __half val = __float2half_rn(0.f);
    if (cv < g.IC) {
      const int phase = cv / g.xIC, c = cv - phase * g.xIC;
      const int ih = g.sH * (hp - g.pH) + g.phH[phase / g.nphW];
      const int iw = g.sW * (wp - g.pW) + g.phW[phase % g.nphW];
      if (ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW)
        val = src_plane(g, b, c)[(long long)ih * g.IW + iw];
    }
    v[e] = val;
  }
  if (WGX_IN_BOUNDS(xs + i, 16, xs, g.xs_bytes, g.err)) xs[i] = *reinterpret_cast<const uint4 *>(v);
}

// Vector form for stride 2 across with both column phases used, IC % 8 == 0
// and IW % 8 == 0 (then the virtual channel count is a multiple of 8 and
// every 8-channel block of xs holds one phase). One thread takes one
// 8-channel block of one input row (phase ph of virtual row hp) and 8
// consecutive input columns iw0 = 2*q0 (q0 a multiple of 4): eight aligned
// 16-byte loads, a register transpose, and four 16-byte slots for each of
// the two column phases (64 contiguous bytes each).
__global__ void __launch_bounds__(256)
    pack_input_s2d_v8(UmmaGeom g, const __half *__restrict__ x, uint4 *__restrict__ xs,
                      int groups_per_row, int qbase, int n_items) {
  __shared__ uint4 wstage[8][128];
  int item = blockIdx.x * 256 + threadIdx.x;
  const bool active = item < n_items;
  if (!active) item = n_items - 1;  // inactive lanes still join the warp stores
  const int t = item % groups_per_row;
  int r = item / groups_per_row;
  const int iph = r % g.nphH;
  r /= g.nphH;
  const int hp = r % g.Hp;
  r /= g.Hp;
  const int nb = g.xIC / 8;
  const int cb = r % nb, b = r / nb;
  const int ih = g.sH * (hp - g.pH) + g.phH[iph];
  const int q0 = 4 * t + qbase;
  const int iw0 = 2 * q0;  // a multiple of 8: the 8 columns are all in or all out
  const bool inside = ih >= 0 && ih < g.IH && iw0 >= 0 && iw0 < g.IW;
  uint4 ch[8];
  const size_t cstride = size_t(g.IH) * g.IW;
  const __half *src0 = src_plane(g, b, cb * 8) + size_t(inside ? ih : 0) * g.IW + (inside ? iw0 : 0);
#pragma unroll
  for (int e = 0; e < 8; ++e)
    ch[e] = inside ? *reinterpret_cast<const uint4 *>(src0 + e * cstride)
                   : make_uint4(0u, 0u, 0u, 0u);
  const size_t plane_rows = size_t(g.Hp) * g.Wp;
  const int wp0 = q0 + g.pW;
  // positions outside [0, Wp) are skipped
  const int klo = active ? max(0, -wp0) : 4, khi = active ? min(4, g.Wp - wp0) : 0;
#pragma unroll
  for (int pw = 0; pw < 2; ++pw) {
    // virtual block of phase (iph, pw), real block cb
    const int vb = (iph * 2 + pw) * nb + cb;
    uint4 *dst = xs + (size_t(b) * (g.C8 / 8) + vb) * plane_rows + size_t(hp) * g.Wp + wp0;
    const uint32_t sel = pw ? 0x7632u : 0x5410u;
    uint4 vv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // column 2k+pw of each channel: half pw of word k
      uint32_t wd[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint4 &v = ch[e];
        wd[e] = k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
      }
      vv[k] = make_uint4(__byte_perm(wd[0], wd[1], sel), __byte_perm(wd[2], wd[3], sel),
                         __byte_perm(wd[4], wd[5], sel), __byte_perm(wd[6], wd[7], sel));
    }
    warp_store4(g, xs, wstage[threadIdx.x >> 5], vv, dst, klo, khi);
  }
}

__global__ void pack_weights(UmmaGeom g, const __half *__restrict__ w, uint4 *__restrict__ packed,
                             int n_slots) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_slots) pack_weights_body(g, w, packed, i);
}

// Per-image weights (batched GEMM): image img's OIHW weights at
// w + img * w_img_elems pack into packed + img * n_img_slots.
__global__ void pack_weights_batched(UmmaGeom g, const __half *__restrict__ w,
                                     uint4 *__restrict__ packed, int n_img_slots,
                                     long long w_img_elems, long long n_slots) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_slots) return;
  const long long img = i / n_img_slots;
  pack_weights_body(g, w + img * w_img_elems, packed + img * n_img_slots, int(i - img * n_img_slots));
}

// PTX helpers: tcgen05.h

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// bias + activation of one accumulator value. SiLU(v) = v*sigmoid(v) is
// evaluated as h + h*tanh(h) with h = v/2 (the identity
// sigmoid(v) = (1 + tanh(v/2)) / 2): two FMAs and one MUFU op; the bias is
// folded into the first FMA (hb = bias/2).
template <int ACT>
__device__ __forceinline__ float epi_act(float acc, float bias, float hb, float lo, float hi) {
  if constexpr (ACT == WGX_ACT_SILU) {
    const float h = fmaf(acc, 0.5f, hb);
    return fmaf(h, tanh_approx(h), h);
  } else if constexpr (ACT == WGX_ACT_CLAMP) {
    return fminf(fmaxf(acc + bias, lo), hi);
  } else {
    return acc + bias;
  }
}

// Two epilogue values (with their biases) -> packed fp16x2. SiLU runs in
// half precision after one rounding of h = (acc + bias)/2: one
// tanh.approx.f16x2 for both values and y = h + h*tanh(h) as one HFMA2
// (the output is fp16, so the half-precision tail adds at most about one
// fp16 rounding); the other activations round once from fp32. For SiLU the
// bias arguments are the HALF biases (bias/2, staged that way by the
// epilogues: one FMA per value).
template <int ACT>
__device__ __forceinline__ uint32_t epi_act2(float a0, float a1, float b0, float b1, float lo,
                                             float hi) {
  if constexpr (ACT == WGX_ACT_SILU) {
    const __half2 h = __floats2half2_rn(fmaf(a0, 0.5f, b0), fmaf(a1, 0.5f, b1));
    const uint32_t hu = *reinterpret_cast<const uint32_t *>(&h);
    uint32_t tu;
    asm("tanh.approx.f16x2 %0, %1;" : "=r"(tu) : "r"(hu));
    const __half2 y = __hfma2(h, *reinterpret_cast<const __half2 *>(&tu), h);
    return *reinterpret_cast<const uint32_t *>(&y);
  } else {
    const __half2 y = __floats2half2_rn(epi_act<ACT>(a0, b0, 0.f, lo, hi),
                                        epi_act<ACT>(a1, b1, 0.f, lo, hi));
    return *reinterpret_cast<const uint32_t *>(&y);
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// pos / Wp for a position of the padded plane (see UmmaGeom::wp_magic)
__device__ __forceinline__ int div_wp(const UmmaGeom &g, int pos) {
  return g.wp_magic ? int(__umulhi(uint32_t(pos), g.wp_magic)) : pos / g.Wp;
}

// The consumer's re-layout slot (16 bytes: virtual channels vc..vc+7 of one
// staged position) that holds output channels [c, c+8) of image b at output
// position (oh, ow), or null when the consumer stages no such slot (an input
// phase its filter never touches, or a row or column past its staged plane).
__device__ __forceinline__ uint4 *xs_slot(const UmmaGeom &g, int b, int c, int oh, int ow) {
  int hp, wp, vc;
  if (g.osH == 1 && g.osW == 1) {
    hp = oh + g.opH;
    wp = ow + g.opW;
    vc = c;
  } else if (g.osH == 2 && g.osW == 2) {
    const int iph = g.ophase_h[oh & 1], ipw = g.ophase_w[ow & 1];
    if (iph < 0 || ipw < 0) return nullptr;
    vc = (iph * g.onphW + ipw) * g.oxIC + c;
    hp = (oh >> 1) + g.opH;
    wp = (ow >> 1) + g.opW;
  } else {
    const int iph = g.ophase_h[oh % g.osH], ipw = g.ophase_w[ow % g.osW];
    if (iph < 0 || ipw < 0) return nullptr;
    vc = (iph * g.onphW + ipw) * g.oxIC + c;
    hp = oh / g.osH + g.opH;
    wp = ow / g.osW + g.opW;
  }
  if (hp >= g.oHp || wp >= g.oWp) return nullptr;
  return g.oxs + ((size_t(b) * g.oplanes + (vc >> 3)) * g.oHp + hp) * g.oWp + wp;
}

// v (two fp16 outputs) + the residual pair r, added in fp32 and rounded once
// (what the separate add operator computes on the stored conv output).
__device__ __forceinline__ uint32_t add_resid2(uint32_t v, uint32_t r) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&v));
  const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&r));
  const __half2 y = __floats2half2_rn(a.x + b.x, a.y + b.y);
  return *reinterpret_cast<const uint32_t *>(&y);
}
__device__ __forceinline__ __half add_resid1(__half v, __half r) {
  return __float2half_rn(__half2float(v) + __half2float(r));
}

// Start of output plane (b, c): `out` itself, or the split piece holding
// channel c.
__device__ __forceinline__ __half *out_plane(const UmmaGeom &g, __half *out, int b, int c,
                                             size_t plane) {
  if (g.nout == 0) return out + (size_t(b) * g.OC + c) * plane;
  int k = 0;
#pragma unroll
  for (int j = 1; j < kMaxOut; ++j)
    if (j < g.nout && c >= g.out_c0[j]) k = j;
  const int ck = g.out_c0[k + 1] - g.out_c0[k];
  return g.outp[k] + (size_t(b) * ck + (c - g.out_c0[k])) * plane;
}

// tile index -> (image, first position, output-channel tile); oc tile
// fastest so that CTAs working on the same positions run together.
// Pipeline stage walk: (filter-row group khg, channel block cbk) and the
// space-to-depth phase of cbk, advanced without divisions.
struct StageWalk {
  int khg = 0, cbk = 0, pc = 0, phase = 0;
  __device__ __forceinline__ void next(const UmmaGeom &g) {
    if (++cbk == g.ncb) {
      cbk = pc = phase = 0;
      ++khg;
    } else if (++pc == g.cbpp) {
      pc = 0;
      ++phase;
    }
  }
  __device__ __forceinline__ uint32_t taps(const UmmaGeom &g) const {
    return g.tapskip ? g.tapmask[khg][phase] : 0xFFFFu;
  }
};

// Optional per-role cycle counters (compile with -DWGX_PROF): per CTA,
// [0] producer waiting for free slots, [1] MMA thread waiting for a free
// accumulator, [2] MMA thread waiting for staged data, [3] MMA thread
// issuing, [4] epilogue warp 4 waiting for a full accumulator, [5] epilogue
// warp 4 working, [6] MMA thread total, [7] tiles of the CTA; folded-column
// epilogue (warp 4): [8] TMEM loads, [9] exchange wait, [10] outputs;
// %globaltimer (ns) at [11] kernel entry, [12] end of the set-up, [13] the
// MMA thread's last commit, [14] the end of epilogue warp 4, [15] kernel exit.
#ifdef WGX_PROF
__device__ unsigned long long g_umma_prof[256][20];
#define WGX_PROF_T(v) const long long v = clock64()
#define WGX_PROF_ADD(acc, t0) acc += (unsigned long long)(clock64() - (t0))
#else
#define WGX_PROF_T(v)
#define WGX_PROF_ADD(acc, t0)
#endif

__device__ __forceinline__ void tile_coords(const UmmaGeom &g, int t, int &b, long long &p0,
                                            int &oct) {
  oct = t % g.n_oct;
  const int rest = t / g.n_oct;
  b = rest / g.tiles_per_img;
  p0 = (long long)(rest % g.tiles_per_img) * g.tile_stride;
}

// ---------------------------------------- epilogue of the folded-column form
// tcgen05.ld of 8 columns without waiting (completed by tmem_wait_3x8)
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, float *r) {
  uint32_t *u = reinterpret_cast<uint32_t *>(r);
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]),
                 "=r"(u[6]), "=r"(u[7])
               : "r"(taddr));
}
// Waits for this thread's outstanding tcgen05.ld's. The 24 destination
// registers are operands, so no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait_3x8(float *a, float *b, float *c) {
  uint32_t *x = reinterpret_cast<uint32_t *>(a), *y = reinterpret_cast<uint32_t *>(b),
           *z = reinterpret_cast<uint32_t *>(c);
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(x[0]), "+r"(x[1]), "+r"(x[2]), "+r"(x[3]), "+r"(x[4]), "+r"(x[5]),
                 "+r"(x[6]), "+r"(x[7]), "+r"(y[0]), "+r"(y[1]), "+r"(y[2]), "+r"(y[3]),
                 "+r"(y[4]), "+r"(y[5]), "+r"(y[6]), "+r"(y[7]), "+r"(z[0]), "+r"(z[1]),
                 "+r"(z[2]), "+r"(z[3]), "+r"(z[4]), "+r"(z[5]), "+r"(z[6]), "+r"(z[7])
               :
               : "memory");
}

// Exchange area of the folded-column epilogue inside the epilogue staging
// region (after the bias and the per-warp transpose rows): per tile parity
// 32 entries (group of 32 positions x 8-channel chunk) of 24 floats: Y's
// second column group at the group's lane 0, its third at lanes 0 and 1.
constexpr uint32_t HS_XCH_OFF = 1024 + EPI_WARPS * 1024;
static_assert(HS_XCH_OFF + 2 * 32 * 24 * 4 <= EPI_BYTES, "folded-column exchange");

// Epilogue of the folded-column form (UmmaGeom::hs). Accumulator column
// kw*OCP + oc of M block mb holds Y[p][kw][oc] for position p = tile start +
// mb*128 + TMEM lane; out[p][oc] = Y[p][0][oc] + Y[p+1][1][oc] + Y[p+2][2][oc].
// Warp w reads TMEM lane quadrant q = w % 4 (positions 32q..32q+31 of every
// M block). The tile's 8 items (M block, 8-channel chunk) go two to each of
// the four warps of a quadrant. For an item a lane loads its position's
// three 8-column groups; the next positions' values come by warp shuffles,
// and lanes 30 and 31 take them from the next 32-position group's lanes 0
// and 1, which that group's warp publishes in shared memory (waited for on
// an mbarrier per tile parity, bounded like every wait here). Outputs:
// the consumer's re-laid input (one 16-byte slot per position), NCHW through
// a per-warp transpose (16-byte runs of 8 positions), or 2-byte NCHW stores;
// residual adds and channel splits in the NCHW paths.
template <int ACT_T, int NT_C, int G_C>
__device__ __forceinline__ void hsum_epilogue(const UmmaGeom &g, uint32_t tmem,
                                              const __half *__restrict__ bias,
                                              __half *__restrict__ out, uint8_t *sE,
                                              uint64_t *accf, uint64_t *acce, uint64_t *xbar,
                                              int warp, int lane) {
  constexpr int OCP = NT_C == 32 ? 8 : NT_C / 3;
  constexpr int NCHUNK = OCP / 8;
  constexpr int ACC_COLS = G_C * NT_C;
  static_assert(G_C * NCHUNK == 8, "two items per epilogue warp");
  const int ew = warp - EPI_WARP0;
  const int q = warp & 3, cq = ew / 4;
  const size_t plane = size_t(g.OH) * g.OW;
  float *sbias = reinterpret_cast<float *>(sE);
  for (int i = threadIdx.x - EPI_WARP0 * 32; i < NT_C; i += EPI_WARPS * 32)
    sbias[i] = ((g.has_bias && i < g.OC) ? __half2float(bias[i]) : 0.f) *
                (ACT_T == WGX_ACT_SILU ? 0.5f : 1.f);
  asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32) : "memory");
  uint16_t *tstage = reinterpret_cast<uint16_t *>(sE + 1024 + ew * 1024);
  float *xch = reinterpret_cast<float *>(sE + HS_XCH_OFF);
  const bool tvec = g.tvec != 0;
  int it = 0;
  [[maybe_unused]] unsigned long long ph_wait = 0, ph_ld = 0, ph_x = 0, ph_out = 0;
  for (int t = blockIdx.x; t < g.total_tiles; t += gridDim.x, ++it) {
    const int acc = it & 1, use_acc = it >> 1;
    int b, oct;
    long long p0;
    tile_coords(g, t, b, p0, oct);
    WGX_PROF_T(th0);
    if (!mbar_wait(smem_u32(&accf[acc]), use_acc & 1)) {
      if (lane == 0) atomicOr(g.err, kErrEpilogueTimeout);
      break;
    }
    WGX_PROF_ADD(ph_wait, th0);
    WGX_PROF_T(th1);
    tc_fence_after();
    float y[2][3][8];
    const uint32_t tq = tmem + (uint32_t(q * 32) << 16) + uint32_t(acc * ACC_COLS);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int item = cq + 4 * k, mb = item / NCHUNK, ch = item % NCHUNK;
#pragma unroll
      for (int kw = 0; kw < 3; ++kw)
        tmem_ld8_nowait(tq + uint32_t(mb * NT_C + kw * OCP + ch * 8), y[k][kw]);
    }
    tmem_wait_3x8(y[0][0], y[0][1], y[0][2]);
    tmem_wait_3x8(y[1][0], y[1][1], y[1][2]);
    WGX_PROF_ADD(ph_ld, th1);
    // the accumulator is free again
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&acce[acc]));
    // publish what the previous group's lanes 30 and 31 need
    float *xb = xch + (it & 1) * 32 * 24;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int item = cq + 4 * k, mb = item / NCHUNK, ch = item % NCHUNK;
      float *e = xb + ((mb * 4 + q) * NCHUNK + ch) * 24;
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          e[j] = y[k][1][j];
          e[8 + j] = y[k][2][j];
        }
      } else if (lane == 1) {
#pragma unroll
        for (int j = 0; j < 8; ++j) e[16 + j] = y[k][2][j];
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&xbar[it & 1]));
    WGX_PROF_T(th2);
    if (!mbar_wait(smem_u32(&xbar[it & 1]), (it >> 1) & 1)) {
      if (lane == 0) atomicOr(g.err, kErrEpilogueTimeout);
      break;
    }
    WGX_PROF_ADD(ph_x, th2);
    WGX_PROF_T(th3);
    // sums: own column group 0 + next position's group 1 + the one after's
    // group 2; lanes 30 and 31 patch theirs from the next group's entry
    float v[2][8];
    int mbk[2], chk[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int item = cq + 4 * k;
      mbk[k] = item / NCHUNK;
      chk[k] = item % NCHUNK;
      float a1[8], a2[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a1[j] = __shfl_down_sync(0xffffffffu, y[k][1][j], 1);
        a2[j] = __shfl_down_sync(0xffffffffu, y[k][2][j], 2);
      }
      if (lane >= 30) {
        // the next 32 positions: quadrant q + 1 of this M block, or quadrant
        // 0 of the next (none after the tile's last group, whose lanes 30
        // and 31 lie past the tile's outputs)
        const int mb = mbk[k];
        const int ngrp = q < 3 ? mb * 4 + q + 1 : (mb + 1 < G_C ? (mb + 1) * 4 : -1);
        const float4 *e4 =
            reinterpret_cast<const float4 *>(xb + (ngrp < 0 ? 0 : (ngrp * NCHUNK + chk[k]) * 24));
        if (lane == 31) {
          const float4 p0v = e4[0], p1v = e4[1], p4v = e4[4], p5v = e4[5];
          a1[0] = p0v.x, a1[1] = p0v.y, a1[2] = p0v.z, a1[3] = p0v.w;
          a1[4] = p1v.x, a1[5] = p1v.y, a1[6] = p1v.z, a1[7] = p1v.w;
          a2[0] = p4v.x, a2[1] = p4v.y, a2[2] = p4v.z, a2[3] = p4v.w;
          a2[4] = p5v.x, a2[5] = p5v.y, a2[6] = p5v.z, a2[7] = p5v.w;
        } else {
          const float4 p2v = e4[2], p3v = e4[3];
          a2[0] = p2v.x, a2[1] = p2v.y, a2[2] = p2v.z, a2[3] = p2v.w;
          a2[4] = p3v.x, a2[5] = p3v.y, a2[6] = p3v.z, a2[7] = p3v.w;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[k][j] = y[k][0][j] + a1[j] + a2[j];
    }
    uint32_t pr[2][4];
    int ohk[2], owk[2];
    bool validk[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int oc0 = chk[k] * 8;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        pr[k][j] = epi_act2<ACT_T>(v[k][2 * j], v[k][2 * j + 1], sbias[oc0 + 2 * j],
                                   sbias[oc0 + 2 * j + 1], g.lo, g.hi);
      const int i = mbk[k] * 128 + q * 32 + lane;
      const int pos = int(p0) + i;
      ohk[k] = div_wp(g, pos);
      owk[k] = pos - ohk[k] * g.Wp;
      validk[k] = i < g.tile_stride && ohk[k] < g.OH && owk[k] < g.OW;
    }
    if (g.omode) {
      // 8 channels of one position: one slot of the consumer's input
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int oc0 = chk[k] * 8;
        if (validk[k] && oc0 < g.OC) {
          uint4 *slot = xs_slot(g, b, oc0, ohk[k], owk[k]);
          if (slot && oxs_ok(g, slot)) *slot = make_uint4(pr[k][0], pr[k][1], pr[k][2], pr[k][3]);
        }
      }
    } else if (tvec) {
      // [item][channel][32 positions] through the warp's staging rows; lane
      // -> channel lane / 4 of each item, positions 8 * (lane % 4) .. + 7
      // (Wp % 8 == 0 and OW % 8 == 0: an 8-group is entirely valid or
      // entirely padding; tile_stride % 8 == 0: entirely inside or past the
      // tile's outputs)
#pragma unroll
      for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          tstage[(k * 8 + 2 * j) * 32 + lane] = uint16_t(pr[k][j] & 0xFFFFu);
          tstage[(k * 8 + 2 * j + 1) * 32 + lane] = uint16_t(pr[k][j] >> 16);
        }
      __syncwarp();
      const int row = lane >> 2, part = lane & 3;
      uint4 val[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) val[k] = reinterpret_cast<const uint4 *>(tstage)[(k * 8 + row) * 4 + part];
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        // (oh, ow) of the group's first position, from the lane holding it
        const int oh8 = __shfl_sync(0xffffffffu, ohk[k], part * 8);
        const int ow8 = __shfl_sync(0xffffffffu, owk[k], part * 8);
        const int i8 = mbk[k] * 128 + q * 32 + part * 8;
        const int oc = chk[k] * 8 + row;
        if (i8 < g.tile_stride && oh8 < g.OH && ow8 < g.OW && oc < g.OC) {
          const size_t off = size_t(oh8) * g.OW + ow8;
          uint4 w4 = val[k];
          if (g.resid) {
            const __half *rsrc = g.resid + (size_t(b) * g.OC + oc) * plane + off;
            const uint4 rr = WGX_IN_BOUNDS(rsrc, 16, g.resid, g.out_bytes, g.err)
                                 ? *reinterpret_cast<const uint4 *>(rsrc)
                                 : make_uint4(0u, 0u, 0u, 0u);
            w4 = make_uint4(add_resid2(w4.x, rr.x), add_resid2(w4.y, rr.y),
                            add_resid2(w4.z, rr.z), add_resid2(w4.w, rr.w));
          }
          __half *dst16 = out_plane(g, out, b, oc, plane) + off;
          if (out_ok(g, out, dst16, 16)) *reinterpret_cast<uint4 *>(dst16) = w4;
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (!validk[k]) continue;
        const size_t posoff = size_t(ohk[k]) * g.OW + owk[k];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int oc = chk[k] * 8 + 2 * j;
          uint32_t vv = pr[k][j];
          if (g.resid) {
            const __half *rp = g.resid + size_t(b) * g.OC * plane + posoff;
            const uint32_t lo =
                oc < g.OC ? uint32_t(__half_as_ushort(rp[size_t(oc) * plane])) : 0u;
            const uint32_t hi =
                oc + 1 < g.OC ? uint32_t(__half_as_ushort(rp[size_t(oc + 1) * plane])) : 0u;
            vv = add_resid2(vv, lo | (hi << 16));
          }
          const __half2 h2 = *reinterpret_cast<const __half2 *>(&vv);
          if (oc < g.OC && out_ok(g, out, out_plane(g, out, b, oc, plane) + posoff, 2))
            out_plane(g, out, b, oc, plane)[posoff] = __low2half(h2);
          if (oc + 1 < g.OC && out_ok(g, out, out_plane(g, out, b, oc + 1, plane) + posoff, 2))
            out_plane(g, out, b, oc + 1, plane)[posoff] = __high2half(h2);
        }
      }
    }
    WGX_PROF_ADD(ph_out, th3);
  }
#ifdef WGX_PROF
  if (warp == EPI_WARP0 && lane == 0) {
    g_umma_prof[blockIdx.x][4] = ph_wait;
    g_umma_prof[blockIdx.x][8] = ph_ld;
    g_umma_prof[blockIdx.x][9] = ph_x;
    g_umma_prof[blockIdx.x][10] = ph_out;
  }
#endif
}

// ------------------------------------------------------------ main kernel
// KW_T > 0: compile-time filter width with one filter row and 32 channels
// per stage (the common staging); the MMA issue loop is then fully unrolled
// over precomputed descriptor offsets. KW_T == 0: any staging, runtime loops.
// TRANS > 0 (geometry trans = 1, NT = TRANS): positions are the MMA's M
// rows and output channels its N columns; the staged activation rows become the A operand
// and the packed weights the B operand, with no change to either layout.
// EXT: NCHW output with a residual add and/or a channel split (separate
// instantiations keep the common epilogue free of those branches).
template <int KW_T, int ACT_T, int TRANS, int EXT, int HS = 0>
__global__ void __launch_bounds__(THREADS, 1)
    umma_conv_kernel(const UmmaGeom g, const uint8_t *__restrict__ xs,
                     const uint8_t *__restrict__ wpk, const __half *__restrict__ bias,
                     __half *__restrict__ out, const __grid_constant__ TmapSet tm) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
#ifdef WGX_PROF
  if (threadIdx.x == 0) g_umma_prof[blockIdx.x][11] = global_ns();
#endif
  // transposed variant: output channels per M block (N), M blocks per tile
  // (TRANS = 17 / 33: N = 16 / 32 with 4 M blocks, for planes of at most
  // 512 positions)
  constexpr int NT_C = TRANS > 0 ? (TRANS & ~1) : UN;
  // folded filter columns (HS > 0): N = 32 / 48 / 96 / 192 with 8 / 4 / 2 / 1 M blocks
  constexpr int G_C = HS > 0 ? (NT_C == 32 ? 8 : NT_C == 48 ? 4 : NT_C == 96 ? 2 : 1)
                      : TRANS == 0 ? 1 : (TRANS == 64 || (TRANS & 1)) ? 4 : 8;
  constexpr int LG_NT = NT_C == 16 ? 4 : NT_C == 32 ? 5 : 6;
  // positions on M with several M blocks per tile: two MMA threads (warps 1
  // and 2), each issuing every other M block of every stage; a single
  // thread's back-to-back tcgen05.mma issue (~56 cycles per MMA measured)
  // is slower than the tensor pipe takes short MMAs from two issuers (~40
  // cycles for N <= 32)
  constexpr bool DUAL = TRANS > 0 && G_C >= 2;
  constexpr int NISS = DUAL ? 2 : 1;
  // copy-issuing threads (see the producer)
  constexpr int NPI = DUAL ? 2 : 3;
  const int npi = g.split ? NPI : 1;
  // activation stages first, on a 1024-byte boundary (128-byte swizzle atoms
  // of the direct mode); stage sizes are multiples of 1024 bytes there
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int S = g.stages;
  uint8_t *sB = smem;                                  // activation stages
  uint8_t *sW = sB + size_t(S) * g.b_stage_bytes;      // weights (resident or per stage)
  uint8_t *sE = sW + g.w_region_bytes;                 // epilogue staging
  uint64_t *bars = reinterpret_cast<uint64_t *>(sE + EPI_BYTES);
  uint64_t *full = bars, *empty = bars + S;
  uint64_t *accf = bars + 2 * S, *acce = accf + 2, *wbar = acce + 2;
  uint64_t *xbar = wbar + 1;  // folded-column epilogue exchange, per tile parity
  uint64_t *dbar = xbar + 2;  // each MMA thread's drain of its MMAs after a timeout
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(dbar + 2);
  // generic staging: (activation, weight) descriptor offsets of every MMA
  // group of a stage, in 16-byte units (written and read by the MMA thread)
  uint2 *grp_off = reinterpret_cast<uint2 *>(tmem_slot + 4);
  // positions-on-M with tap masks: (start, count) of the compacted group list
  // of each (filter-row group, phase) inside grp_off
  uint16_t *grp_list = reinterpret_cast<uint16_t *>(grp_off + kMaxGroups);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), npi);
      mbar_init(smem_u32(&empty[s]), NISS);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&accf[a]), NISS);
      mbar_init(smem_u32(&acce[a]), EPI_WARPS);
    }
    mbar_init(smem_u32(wbar), 1);
    for (int j = 0; j < 2; ++j) mbar_init(smem_u32(&xbar[j]), EPI_WARPS);
    mbar_init(smem_u32(&dbar[0]), 1);
    mbar_init(smem_u32(&dbar[1]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if constexpr (KW_T == 0) {
    if (threadIdx.x == 32) {
      // generic staging: the (activation, weight) descriptor offsets of every
      // MMA group of a stage, read by the MMA thread(s) after the barrier
      const uint32_t a_lbo = uint32_t(g.wrows) * 16, b_lbo = uint32_t(g.R_alloc) * 16;
      const int ngroups = g.khs * g.KW * (g.bk / 16);
      int j = 0;
      for (int khl = 0; khl < g.khs; ++khl)
        for (int kw = 0; kw < g.KW; ++kw)
          for (int ks = 0; ks < g.bk / 16; ++ks, ++j) {
            const uint32_t tap = uint32_t(khl * g.KW + kw);
            const uint32_t shift = uint32_t(khl * g.dH * g.Wp + kw * g.dW);
            grp_off[j] = make_uint2((shift * 16 + uint32_t(ks) * 2 * b_lbo) >> 4,
                                    (tap * uint32_t(g.chunks) * a_lbo + uint32_t(ks) * 2 * a_lbo) >> 4);
          }
      if (TRANS && g.tapskip) {
        // compacted lists: the groups whose tap meets real filter taps
        int e = ngroups;
        for (int khg = 0; khg < g.n_khg; ++khg)
          for (int ph = 0; ph < g.nphH * g.nphW; ++ph) {
            const uint32_t m = g.tapmask[khg][ph];
            const int start = e;
            for (int jj = 0; jj < ngroups; ++jj)
              if ((m >> (jj / (g.bk / 16))) & 1) grp_off[e++] = grp_off[jj];
            grp_list[2 * (khg * kMaxPhases + ph)] = uint16_t(start);
            grp_list[2 * (khg * kMaxPhases + ph) + 1] = uint16_t(e - start);
          }
      }
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
#ifdef WGX_PROF
  if (threadIdx.x == 0) g_umma_prof[blockIdx.x][12] = global_ns();
#endif

  if (warp == 0 || warp == 3 || (!DUAL && warp == 2)) {
    const int pi = warp == 0 ? 0 : warp == 3 ? 1 : 2;
    if (lane == 0 && !g.inject_skip && pi < npi) {
      // ---------------- producers: bulk copies of weights + activation rows.
      // NPI threads (lane 0 of warps 0, 3 and, without a second MMA issuer,
      // 2) walk the same stage sequence and split each stage's copies: the
      // per-SM copy engine takes copies from several issuing threads faster
      // than from one (measured on B200: eight 4 KB copies per stage, one
      // issuer ~16 B/clk per SM, four issuers ~22 B/clk). Each issuer
      // arrives on the stage's full barrier once with its own byte count;
      // issuer 0 also copies the weights. In the direct mode the issuers
      // take every npi-th 64-position atom of each channel box (YOLO26-N
      // batch 64, 1x1 layers over concatenations of 16-channel sources:
      // 48 -> 64 at 160^2 105 -> 86 us against one issuer).
      const uint32_t b_copy = uint32_t(g.R) * 16;
      if (g.resident && pi == 0) {
        // (one copy: splitting it into per-stage pieces, each on its own
        // barrier, or into one piece per issuer, measured no faster on B200)
        const uint32_t wb = smem_u32(wbar);
        mbar_expect_tx(wb, g.w_region_bytes);
        if (WGX_IN_BOUNDS(wpk, g.w_region_bytes, wpk, g.wpk_bytes, g.err))
          bulk_g2s(smem_u32(sW), wpk, g.w_region_bytes, wb);
      }
      // this issuer's share of a stage: chunk copies ch = pi, pi + npi, ...;
      // direct-mode atoms j = pi, pi + npi, ... of every channel box
      const int my_chunks = g.chunks > pi ? (g.chunks - pi + npi - 1) / npi : 0;
      const int nj = g.tile_pos / 64;
      const int my_boxes = g.direct && nj > pi ? (g.bk / g.dbox) * ((nj - pi + npi - 1) / npi) : 0;
      const uint32_t my_bytes =
          (g.resident || pi != 0 ? 0u : g.a_stage_bytes) +
          (g.direct ? uint32_t(my_boxes) * uint32_t(g.dbox) * 128u : uint32_t(my_chunks) * b_copy);
      int slot = S - 1, use = -1;  // pipeline slot and its use count, advanced per loaded stage
      bool ok = true;
      [[maybe_unused]] unsigned long long pr_empty = 0;
      for (int t = blockIdx.x; t < g.total_tiles && ok; t += gridDim.x) {
        int b, oct;
        long long p0;
        tile_coords(g, t, b, p0, oct);
        StageWalk sw;
        for (int s = 0; s < g.n_kstages; ++s, sw.next(g)) {
          if (!sw.taps(g)) continue;  // all-zero weights: not loaded
          if (++slot == S) {
            slot = 0;
            ++use;
          }
          WGX_PROF_T(tw0);
          if (use > 0 && !mbar_wait(smem_u32(&empty[slot]), (use - 1) & 1)) {
            atomicOr(g.err, kErrLoadTimeout);
            ok = false;
            // this stage was not issued: step back so the drain below
            // waits only for copies in flight
            if (slot == 0) {
              slot = S - 1;
              --use;
            } else {
              --slot;
            }
            break;
          }
          WGX_PROF_ADD(pr_empty, tw0);
          const int khg = sw.khg, cbk = sw.cbk;
          const uint32_t fb = smem_u32(&full[slot]);
          mbar_expect_tx(fb, my_bytes);
          if (!g.resident && pi == 0) {
            const uint8_t *wsrc = wpk + size_t(b) * g.w_img_bytes +
                                  (size_t(oct) * g.n_kstages + s) * g.a_stage_bytes;
            if (WGX_IN_BOUNDS(wsrc, g.a_stage_bytes, wpk, g.wpk_bytes, g.err))
              bulk_g2s(smem_u32(sW + size_t(slot) * g.a_stage_bytes), wsrc, g.a_stage_bytes, fb);
          }
          if (g.direct) {
            // TMA boxes of 64 positions x dbox channels: atom j (64 positions,
            // bk rows of 128 bytes) at j * bk * 128, channel group rows inside
            // (this issuer: atoms j = pi, pi + npi, ... of every channel box;
            // no per-box division or source search, the issuing thread's
            // own instruction time bounds how fast small boxes go out)
            const uint32_t stage = smem_u32(sB + size_t(slot) * g.b_stage_bytes);
            const uint32_t jstep = uint32_t(npi) * uint32_t(g.bk) * 128u;
            for (int c = cbk * g.bk, row = 0; row < g.bk; c += g.dbox, row += g.dbox) {
              int src = 0;
              for (int k = 1; k < g.nsrc; ++k)
                if (c >= g.src_c0[k]) src = k;
              const int y = c - g.src_c0[src];
              const void *map = &tm.m[src];
              uint32_t dst = stage + uint32_t(pi) * uint32_t(g.bk) * 128u + uint32_t(row) * 128u;
              for (int j = pi; j < nj; j += npi, dst += jstep)
                tma_load_3d(dst, map, int(p0) + 64 * j, y, b, fb);
            }
            continue;
          }
          const long long row0 = p0 + (long long)khg * g.khs * g.dH * g.Wp;
          for (int ch = pi; ch < g.chunks; ch += npi) {
            const long long plane = (long long)b * (g.C8 / 8) + cbk * g.chunks + ch;
            const uint8_t *xsrc = xs + (plane * g.plane_rows + row0) * 16;
            if (WGX_IN_BOUNDS(xsrc, b_copy, xs, g.xs_bytes, g.err))
              bulk_g2s(smem_u32(sB + size_t(slot) * g.b_stage_bytes + size_t(ch) * g.R_alloc * 16),
                       xsrc, b_copy, fb);
          }
        }
      }
      // Before the CTA exits, every copy this thread issued must have landed
      // (bounded waits). Slot j's last fill is use (j <= slot) or use - 1;
      // its barrier completed no later phase, so the parity test is exact.
      // On the normal path every wait succeeds at its first try.
      if (g.resident && pi == 0 && !mbar_wait(smem_u32(wbar), 0))
        atomicOr(g.err, kErrLoadTimeout);
      for (int j = 0; j < S; ++j) {
        const int last = j <= slot ? use : use - 1;
        if (last >= 0 && !mbar_wait(smem_u32(&full[j]), uint32_t(last) & 1)) {
          atomicOr(g.err, kErrLoadTimeout);
          break;
        }
      }
#ifdef WGX_PROF
      if (pi == 0) g_umma_prof[blockIdx.x][0] = pr_empty;
#endif
    }
  } else if (warp == 1 || (DUAL && warp == 2)) {
    if (lane == 0) {
      // ---------------- MMA issuer (iss 0: warp 1; with DUAL, iss 1: warp 2,
      // the odd M blocks)
      const int iss = warp - 1;
      WGX_PROF_T(tm_start);
      [[maybe_unused]] unsigned long long pm_acce = 0, pm_full = 0, pm_issue = 0, pm_tiles = 0;
      // (a = packed weights, b = staged activation rows, whichever MMA
      // operand slot they take)
      const uint32_t idesc = (1u << 4)                                  // D = f32
                             | (uint32_t(NT_C >> 3) << 17)                  // N
                             | (uint32_t(128 >> 4) << 24);              // M; f16 K-major
      const uint32_t a_lbo = uint32_t(g.wrows) * 16;        // chunk plane of the weights
      const uint32_t b_lbo = uint32_t(g.R_alloc) * 16;      // chunk plane of the activations
      bool ok = true;
      WGX_PROF_T(tw_res);
      if (g.resident && !mbar_wait(smem_u32(wbar), 0)) {
        atomicOr(g.err, kErrMmaTimeout);
        ok = false;
      }
#ifdef WGX_PROF
      if (iss == 0) {
        g_umma_prof[blockIdx.x][16] = (unsigned long long)(clock64() - tw_res);
        g_umma_prof[blockIdx.x][17] = global_ns();
      }
#endif
      // per-MMA start-address offsets (16-byte units) of the specialised path:
      // MMA i = (kw, ks) reads A tap kw chunk pair ks, B shifted kw*dW rows
      uint32_t a_off[KW_T > 0 ? 2 * KW_T : 1], b_off[KW_T > 0 ? 2 * KW_T : 1];
      if constexpr (KW_T > 0) {
#pragma unroll
        for (int kw = 0; kw < KW_T; ++kw)
#pragma unroll
          for (int ks = 0; ks < 2; ++ks) {
            a_off[2 * kw + ks] = (uint32_t(kw) * 4 * a_lbo + uint32_t(ks) * 2 * a_lbo) >> 4;
            b_off[2 * kw + ks] = (uint32_t(kw * g.dW) * 16 + uint32_t(ks) * 2 * b_lbo) >> 4;
          }
      }
      const int ngroups = g.khs * g.KW * (g.bk / 16);
      int it = 0, slot = S - 1, use = -1;
      for (int t = blockIdx.x; t < g.total_tiles && ok; t += gridDim.x, ++it) {
        const int acc = it & 1, use_acc = it >> 1;
        WGX_PROF_T(ta0);
        if (use_acc > 0 && !mbar_wait(smem_u32(&acce[acc]), (use_acc - 1) & 1)) {
          atomicOr(g.err, kErrMmaTimeout);
          ok = false;
          break;
        }
        WGX_PROF_ADD(pm_acce, ta0);
#ifdef WGX_PROF
        ++pm_tiles;
#endif
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(acc * g.acc_cols);
        uint32_t acc_on = 0;  // the tile's accumulator already holds a product
        StageWalk sw;
        for (int s = 0; s < g.n_kstages; ++s, sw.next(g)) {
          const uint32_t tmask = sw.taps(g);
          if (!tmask) continue;  // all-zero weights: not loaded, no MMA
          if (++slot == S) {
            slot = 0;
            ++use;
          }
          WGX_PROF_T(tf0);
          if (!mbar_wait(smem_u32(&full[slot]), use & 1)) {
            atomicOr(g.err, kErrMmaTimeout);
            ok = false;
            break;
          }
          WGX_PROF_ADD(pm_full, tf0);
#ifdef WGX_PROF
          if (iss == 0 && it == 0 && g_umma_prof[blockIdx.x][18] == 0)
            g_umma_prof[blockIdx.x][18] = global_ns();  // first stage landed
          // issue time: from the data's arrival to the stage's commit
          // (measured at the next stage's wait start: approximated by the
          // commit below)
          const long long ti0 = clock64();
          struct IssueTimer {
            unsigned long long &acc;
            long long t0;
            __device__ ~IssueTimer() { acc += (unsigned long long)(clock64() - t0); }
          } issue_timer{pm_issue, ti0};
#endif
          tc_fence_after();
          const uint32_t a_base =
              smem_u32(sW + size_t(g.resident ? s : slot) * g.a_stage_bytes);
          const uint32_t b_base = smem_u32(sB + size_t(slot) * g.b_stage_bytes);
          if (g.direct) {
            // activations MN-major (128-byte swizzle): atoms of 64 positions
            // bk*128 bytes apart, 8-channel groups 1024 bytes apart; one MMA
            // takes two groups (K = 16); weights K-major as always
            const uint32_t x_lbo = uint32_t(g.bk) * 128;
            const uint32_t idesc_mn = idesc | (TRANS ? (1u << 15) : (1u << 16));
            for (int ks = 0; ks < g.bk / 16; ++ks) {
              const uint64_t wdesc = kmajor_desc(a_base + uint32_t(ks) * 2 * a_lbo, a_lbo);
              const uint32_t xaddr = b_base + uint32_t(ks) * 2 * 1024;
              if constexpr (TRANS) {
#pragma unroll
                for (int k2 = 0; k2 < G_C / NISS; ++k2) {
                  const int mb = k2 * NISS + iss;
                  mma_f16(d + uint32_t(mb * NT_C),
                          sw128_mn_desc(xaddr + uint32_t(mb) * 2 * x_lbo, x_lbo, 1024), wdesc,
                          idesc_mn, (acc_on | ks) != 0);
                }
              } else {
                mma_f16(d, wdesc, sw128_mn_desc(xaddr, x_lbo, 1024), idesc_mn, (acc_on | ks) != 0);
              }
            }
            acc_on = 1;
            mma_commit(smem_u32(&empty[slot]));
            continue;
          }
          if constexpr (KW_T > 0) {
            // descriptors differ from the stage's base descriptors only in
            // the start-address field: add precomputed (offset >> 4) values
            const uint64_t a0 = kmajor_desc(a_base, a_lbo), b0 = kmajor_desc(b_base, b_lbo);
            if constexpr (TRANS) {
              // M-block mb: activation rows mb*128.., accumulator columns
              // mb*NT..; M blocks innermost so that consecutive MMAs feed
              // different accumulators (a short MMA would otherwise wait on
              // the previous one's accumulation)
#pragma unroll
              for (int i = 0; i < 2 * KW_T; ++i)
#pragma unroll
                for (int k2 = 0; k2 < G_C / NISS; ++k2) {
                  const int mb = k2 * NISS + iss;
                  mma_f16(d + uint32_t(mb * NT_C), b0 + uint64_t(mb * 128) + b_off[i],
                          a0 + a_off[i], idesc, (acc_on | i) != 0);
                }
              acc_on = 1;
            } else {
              // (taps whose weights are all zero are skipped: tapskip)
#pragma unroll
              for (int i = 0; i < 2 * KW_T; ++i) {
                if (!((tmask >> (i >> 1)) & 1)) continue;
                mma_f16(d, a0 + a_off[i], b0 + b_off[i], idesc, acc_on);
                acc_on = 1;
              }
            }
            mma_commit(smem_u32(&empty[slot]));
            continue;
          }
          {
            // generic staging: one MMA group per (filter tap, 16-channel
            // step), offsets from the table. Up to kSeqGroups groups are
            // issued as straight-line code entered once per stage (a branch
            // between MMAs stalls the issuing thread far longer than an MMA
            // takes to issue): the stage's offsets are loaded first, last
            // group in the last slot, and the switch falls through the
            // groups in table order.
            const uint64_t x0 = kmajor_desc(b_base, b_lbo), w0 = kmajor_desc(a_base, a_lbo);
            uint32_t acc_flag = acc_on;
            // the stage's group list: all groups, or the compacted list of
            // its (filter-row group, phase) under tap masks
            int gstart = 0, gcount = ngroups;
            if (TRANS && g.tapskip) {
              gstart = grp_list[2 * (sw.khg * kMaxPhases + sw.phase)];
              gcount = grp_list[2 * (sw.khg * kMaxPhases + sw.phase) + 1];
            }
            // batches of at most kSeqGroups groups (a branch between
            // batches, none inside one)
            for (int base = 0; base < gcount; base += kSeqGroups) {
              const int nb = gcount - base < kSeqGroups ? gcount - base : kSeqGroups;
              uint2 e[kSeqGroups];
#pragma unroll
              for (int k = 0; k < kSeqGroups; ++k) {
                const int j = k - (kSeqGroups - nb);
                e[k] = grp_off[gstart + base + (j < 0 ? 0 : j)];
              }
#define WGX_GROUP(K)                                                                      \
  {                                                                                       \
    const uint64_t xd = x0 + e[K].x, wd = w0 + e[K].y;                                    \
    if constexpr (TRANS) {                                                                \
      _Pragma("unroll") for (int k2 = 0; k2 < G_C / NISS; ++k2)                          \
          mma_f16(d + uint32_t((k2 * NISS + iss) * NT_C), xd + uint64_t((k2 * NISS + iss) * 128), \
                  wd, idesc, acc_flag);                                                   \
    } else {                                                                              \
      mma_f16(d, wd, xd, idesc, acc_flag);                                                \
    }                                                                                     \
    acc_flag = 1;                                                                         \
  }
              switch (nb) {
                case 8: WGX_GROUP(0) [[fallthrough]];
                case 7: WGX_GROUP(1) [[fallthrough]];
                case 6: WGX_GROUP(2) [[fallthrough]];
                case 5: WGX_GROUP(3) [[fallthrough]];
                case 4: WGX_GROUP(4) [[fallthrough]];
                case 3: WGX_GROUP(5) [[fallthrough]];
                case 2: WGX_GROUP(6) [[fallthrough]];
                default: WGX_GROUP(7)
              }
#undef WGX_GROUP
            }
          }
          acc_on = 1;
          mma_commit(smem_u32(&empty[slot]));
        }
        if (ok) mma_commit(smem_u32(&accf[acc]));
      }
      if (!ok) {
        // a wait ran out: let the MMAs already issued finish (bounded)
        // before TMEM is released at the end of the kernel
        mma_commit(smem_u32(&dbar[iss]));
        if (!mbar_wait(smem_u32(&dbar[iss]), 0)) atomicOr(g.err, kErrMmaTimeout);
      }
#ifdef WGX_PROF
      if (iss == 0) {
      g_umma_prof[blockIdx.x][1] = pm_acce;
      g_umma_prof[blockIdx.x][2] = pm_full;
      g_umma_prof[blockIdx.x][3] = pm_issue;
      g_umma_prof[blockIdx.x][6] = (unsigned long long)(clock64() - tm_start);
      g_umma_prof[blockIdx.x][13] = global_ns();
      g_umma_prof[blockIdx.x][7] = pm_tiles;
      }
#endif
    }
  } else if (warp >= EPI_WARP0) {
  if constexpr (HS > 0) {
    hsum_epilogue<ACT_T, NT_C, G_C>(g, tmem, bias, out, sE, accf, acce, xbar, warp, lane);
  } else if constexpr (TRANS > 0) {
    // ---------------- epilogue (positions on TMEM lanes): warp w reads lane
    // quadrant w % 4 (32 positions of every M block) and 32 of the 128
    // accumulator columns; column c is channel c % NT of M block c / NT.
    // For each channel the warp stores 32 consecutive positions (64 bytes
    // of one output row unless the block wraps a row).
    const int ew = warp - EPI_WARP0;
    const int q = warp & 3, cq = ew / 4;
    const size_t plane = size_t(g.OH) * g.OW;
    // bias (and its half, for SiLU) of the NT channels, staged once in the
    // otherwise unused epilogue staging area
    float *sbias = reinterpret_cast<float *>(sE);
    for (int i = threadIdx.x - EPI_WARP0 * 32; i < NT_C; i += EPI_WARPS * 32)
      sbias[i] = ((g.has_bias && i < g.OC) ? __half2float(bias[i]) : 0.f) *
                (ACT_T == WGX_ACT_SILU ? 0.5f : 1.f);
    asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32) : "memory");
    // per-warp transpose rows of the vector-store path: 16 rows x 64 bytes
    // after the bias (1 KB reserved), 16 KB in all
    uint32_t *tstage = reinterpret_cast<uint32_t *>(sE + 1024 + ew * 1024);
    const bool tvec = g.tvec != 0;
    float r[EXT ? 16 : 32];
    int it = 0;
    [[maybe_unused]] unsigned long long pe_wait = 0, pe_work = 0;
    [[maybe_unused]] long long te_mark = 0;
    for (int t = blockIdx.x; t < g.total_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1, use_acc = it >> 1;
      int b, oct;
      long long p0;
      tile_coords(g, t, b, p0, oct);
#ifdef WGX_PROF
      if (warp == EPI_WARP0 && lane == 0 && it > 0) pe_work += (unsigned long long)(clock64() - te_mark);
#endif
      WGX_PROF_T(te0);
      if (!mbar_wait(smem_u32(&accf[acc]), use_acc & 1)) {
        if (lane == 0) atomicOr(g.err, kErrEpilogueTimeout);
        break;
      }
      WGX_PROF_ADD(pe_wait, te0);
#ifdef WGX_PROF
      te_mark = clock64();
#endif
      tc_fence_after();
      if constexpr (EXT) {
      // the warp's acc_cols / 4 columns, 16 at a time (16 columns always lie
      // in one M block, NT >= 16)
      const int n16 = g.acc_cols / 64;
      __half *base = out + size_t(b) * g.OC * plane;
      for (int h = 0; h < n16; ++h) {
        const int c0 = cq * (g.acc_cols / 4) + h * 16;
        tmem_ld16(tmem + (uint32_t(q * 32) << 16) + uint32_t(acc * g.acc_cols + c0), r);
        if (h == n16 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&acce[acc]));
        }
        const int mb = c0 >> LG_NT;
        const int pos = int(p0) + mb * 128 + q * 32 + lane;
        const int oh = div_wp(g, pos), ow = pos - oh * g.Wp;
        const bool okp = oh < g.OH && ow < g.OW;
        const int oc0 = c0 & (NT_C - 1);  // first of this lane's 16 channels
        // columns 2j, 2j+1: channels oc0+2j, oc0+2j+1 of one position
        uint32_t pr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int oc = oc0 + 2 * j;
          pr[j] = epi_act2<ACT_T>(r[2 * j], r[2 * j + 1], sbias[oc], sbias[oc + 1], g.lo, g.hi);
        }
        if (!okp) continue;
        if (g.omode) {
          // 8 consecutive columns = 8 channels of one position: one 16-byte slot
#pragma unroll
          for (int q8 = 0; q8 < 2; ++q8) {
            const int oc = oc0 + 8 * q8;
            if (oc >= g.OC) continue;
            uint4 *slot = xs_slot(g, b, oc, oh, ow);
            if (slot && oxs_ok(g, slot))
              *slot = make_uint4(pr[4 * q8], pr[4 * q8 + 1], pr[4 * q8 + 2], pr[4 * q8 + 3]);
          }
          continue;
        }
        const size_t posoff = size_t(oh) * g.OW + ow;
        if (g.nout == 0 && !g.resid) {
          __half *d = base + posoff;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int oc = oc0 + 2 * j;
            const __half2 h2 = *reinterpret_cast<const __half2 *>(&pr[j]);
            if (oc < g.OC && out_ok(g, out, d + size_t(oc) * plane, 2))
              d[size_t(oc) * plane] = __low2half(h2);
            if (oc + 1 < g.OC && out_ok(g, out, d + size_t(oc + 1) * plane, 2))
              d[size_t(oc + 1) * plane] = __high2half(h2);
          }
          continue;
        }
        // residual pairs of the 16 channels, all loads issued before use
        uint32_t rres[8];
        if (g.resid) {
          const __half *rp = g.resid + size_t(b) * g.OC * plane + posoff;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int oc = oc0 + 2 * j;
            const uint32_t lo = oc < g.OC ? uint32_t(__half_as_ushort(rp[size_t(oc) * plane])) : 0u;
            const uint32_t hi =
                oc + 1 < g.OC ? uint32_t(__half_as_ushort(rp[size_t(oc + 1) * plane])) : 0u;
            rres[j] = lo | (hi << 16);
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int oc = oc0 + 2 * j;
          const uint32_t v = g.resid ? add_resid2(pr[j], rres[j]) : pr[j];
          const __half2 h2 = *reinterpret_cast<const __half2 *>(&v);
          if (oc < g.OC && out_ok(g, out, out_plane(g, out, b, oc, plane) + posoff, 2))
            out_plane(g, out, b, oc, plane)[posoff] = __low2half(h2);
          if (oc + 1 < g.OC && out_ok(g, out, out_plane(g, out, b, oc + 1, plane) + posoff, 2))
            out_plane(g, out, b, oc + 1, plane)[posoff] = __high2half(h2);
        }
      }
      } else {
      // the warp's ACC_COLS / 4 columns in pieces of 16 (each within one M
      // block, NT >= 16). TMEM reads are software-pipelined: piece h + 1 is
      // requested as soon as piece h has arrived, so its latency hides
      // behind piece h's conversion and stores.
      constexpr int ACC_COLS = G_C * NT_C;
      constexpr int WC = ACC_COLS / 4;
      constexpr int NP = WC / 16;
      __half *base = out + size_t(b) * g.OC * plane;
      float rb[2][16];
      const uint32_t tw = tmem + (uint32_t(q * 32) << 16) + uint32_t(acc * ACC_COLS + cq * WC);
      tmem_ld16_async(tw, rb[0]);
#pragma unroll
      for (int h = 0; h < NP; ++h) {
        float *rr = rb[h & 1];
        tmem_wait16(rr);
        if (h + 1 < NP) tmem_ld16_async(tw + uint32_t((h + 1) * 16), rb[(h + 1) & 1]);
        if (h == NP - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&acce[acc]));
        }
        const int c0 = cq * WC + h * 16;
        const int mb = c0 >> LG_NT;
        const int oc0 = c0 & (NT_C - 1);  // first of the piece's 16 channels
        const int pos = int(p0) + mb * 128 + q * 32 + lane;
        const int oh = div_wp(g, pos), ow = pos - oh * g.Wp;
        const bool okp = oh < g.OH && ow < g.OW;
        // columns 2j, 2j+1: channels oc0 + 2j, oc0 + 2j + 1 of this lane's position
        uint32_t pr[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 bb = reinterpret_cast<const float2 *>(sbias)[(oc0 >> 1) + j];
          pr[j] = epi_act2<ACT_T>(rr[2 * j], rr[2 * j + 1], bb.x, bb.y, g.lo, g.hi);
        }
        if (tvec) {
          // transpose through the warp's staging rows: lanes l, l^1 swap
          // halves so that even lanes hold positions (l, l+1) of column 2k
          // and odd lanes positions (l-1, l) of column 2k+1; row = column
          // (64 bytes: 32 positions). Then lane -> row lane/4 (+8), 8
          // positions from (lane%4)*8: one 16-byte store of 8 consecutive
          // outputs (Wp % 8 == 0: an 8-group never leaves its output row;
          // OW % 8 == 0: it is entirely valid or entirely padding)
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const uint32_t v = pr[k];
            const uint32_t o = __shfl_xor_sync(0xffffffffu, v, 1);
            const bool odd = lane & 1;
            tstage[(2 * k + (odd ? 1 : 0)) * 16 + (lane >> 1)] =
                odd ? __byte_perm(o, v, 0x7632) : __byte_perm(v, o, 0x5410);
          }
          __syncwarp();
          const int part = lane & 3;
          // (oh, ow) of the 8-group's first position, from the lane holding it
          const int oh8 = __shfl_sync(0xffffffffu, oh, part * 8);
          const int ow8 = __shfl_sync(0xffffffffu, ow, part * 8);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int row = (lane >> 2) + 8 * k;
            const uint4 val = reinterpret_cast<const uint4 *>(tstage)[row * 4 + part];
            const int oc = oc0 + row;
            if (oc < g.OC && oh8 < g.OH && ow8 < g.OW) {
              const size_t off = size_t(oh8) * g.OW + ow8;
              uint4 v = val;
              if (g.resid) {
                // residual add after the activation, one rounding (as the
                // separate add would compute it)
                const __half *rsrc = g.resid + (size_t(b) * g.OC + oc) * plane + off;
                const uint4 rr4 = WGX_IN_BOUNDS(rsrc, 16, g.resid, g.out_bytes, g.err)
                                      ? *reinterpret_cast<const uint4 *>(rsrc)
                                      : make_uint4(0u, 0u, 0u, 0u);
                v = make_uint4(add_resid2(val.x, rr4.x), add_resid2(val.y, rr4.y),
                               add_resid2(val.z, rr4.z), add_resid2(val.w, rr4.w));
              }
              __half *dst16 = out_plane(g, out, b, oc, plane) + off;
              if (out_ok(g, out, dst16, 16)) *reinterpret_cast<uint4 *>(dst16) = v;
            }
          }
          __syncwarp();
          continue;
        }
        if (!okp) continue;
        if (g.omode) {
          // 8 consecutive columns = 8 channels of one position: one 16-byte
          // slot; the slot of channel c is that of channel 0 plus c / 8
          // planes (the consumer's channel count is a multiple of 8)
          const size_t pstride = size_t(g.oHp) * g.oWp;
          uint4 *slot = xs_slot(g, b, 0, oh, ow);
          if (slot) {
#pragma unroll
            for (int q8 = 0; q8 < 2; ++q8) {
              const int oc = oc0 + 8 * q8;
              if (oc < g.OC)
                if (oxs_ok(g, slot + size_t(oc >> 3) * pstride))
                  slot[size_t(oc >> 3) * pstride] =
                    make_uint4(pr[4 * q8], pr[4 * q8 + 1], pr[4 * q8 + 2], pr[4 * q8 + 3]);
            }
          }
          continue;
        }
        __half *d = base + size_t(oh) * g.OW + ow;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int oc = oc0 + 2 * j;
          const __half2 h2 = *reinterpret_cast<const __half2 *>(&pr[j]);
          if (oc < g.OC && out_ok(g, out, d + size_t(oc) * plane, 2))
            d[size_t(oc) * plane] = __low2half(h2);
          if (oc + 1 < g.OC && out_ok(g, out, d + size_t(oc + 1) * plane, 2))
            d[size_t(oc + 1) * plane] = __high2half(h2);
        }
      }
      }
    }
#ifdef WGX_PROF
    if (warp == EPI_WARP0 && lane == 0) {
      if (it > 0) pe_work += (unsigned long long)(clock64() - te_mark);
      g_umma_prof[blockIdx.x][4] = pe_wait;
      g_umma_prof[blockIdx.x][5] = pe_work;
    }
#endif
  } else {
    // ---------------- epilogue: TMEM -> bias + activation -> NCHW fp16.
    // Warp w reads TMEM lane quadrant w % 4 (32 output channels) and one
    // quarter (64 columns) of the accumulator. Per block of 16 positions it
    // converts its 32x16 tile to fp16 into its private staging rows (48 B,
    // conflict-free row writes), then stores four channel rows per
    // instruction: 8 lanes x 2 positions = one full 32-byte sector per row
    // when OW and Wp are even (pairs never straddle an output row), 2-byte
    // stores otherwise.
    const int ew = warp - EPI_WARP0;
    constexpr int WCOLS = UN / (EPI_WARPS / 4);  // accumulator columns per warp
    const int q = warp & 3, colh = ew / 4;
    uint8_t *stage = sE + size_t(ew) * 32 * EPI_ROWB;
    const bool pairs = ((g.OW | g.Wp) & 1) == 0;
    const size_t plane = size_t(g.OH) * g.OW;
    const int sub = lane & 7, rsel = lane >> 3;  // position pair, row within 4
    float rb[2][EPI_COLS];
    int it = 0;
    for (int t = blockIdx.x; t < g.total_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1, use_acc = it >> 1;
      int b, oct;
      long long p0;
      tile_coords(g, t, b, p0, oct);
      const bool ok = mbar_wait(smem_u32(&accf[acc]), use_acc & 1);
      if (!ok) {
        if (lane == 0) atomicOr(g.err, kErrEpilogueTimeout);
        break;
      }
#ifdef WGX_PROF
      if (it == 0 && ew == 0 && lane == 0) g_umma_prof[blockIdx.x][19] = global_ns();
#endif
      tc_fence_after();
      const int oc0 = oct * UM + q * 32;  // first channel of this quadrant
      const int oc_lane = oc0 + lane;
      // (halved for SiLU: see epi_act2)
      const float bv = ((g.has_bias && oc_lane < g.OC) ? __half2float(bias[oc_lane]) : 0.f) *
                       (ACT_T == WGX_ACT_SILU ? 0.5f : 1.f);
      const int nrows = min(32, g.OC - oc0);  // valid channel rows of the quadrant
      // this lane stores rows rsel, rsel+4, ..., rsel+28 of the quadrant
      __half *rowp = out + (size_t(b) * g.OC + oc0 + rsel) * plane;
      // (oh, ow) of this lane's first position pair; advanced per block
      const int pos0 = int(p0) + colh * WCOLS + 2 * sub;
      int oh = div_wp(g, pos0), ow = pos0 - oh * g.Wp;
      constexpr int NBLK = WCOLS / EPI_COLS;
      // TMEM reads are software-pipelined: block blk + 1 is requested right
      // after block blk has arrived, so its latency hides behind blk's stores
      const uint32_t tq = tmem + (uint32_t(q * 32) << 16) + uint32_t(acc * g.acc_cols + colh * WCOLS);
      tmem_ld16_async(tq, rb[0]);
#pragma unroll
      for (int blk = 0; blk < NBLK; ++blk) {
        const int col0 = colh * WCOLS + blk * EPI_COLS;
        float *r = rb[blk & 1];
        tmem_wait16(r);
        if (blk + 1 < NBLK) tmem_ld16_async(tq + uint32_t((blk + 1) * EPI_COLS), rb[(blk + 1) & 1]);
        if (blk == NBLK - 1) {
          // all TMEM reads of this accumulator are done: hand it back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&acce[acc]));
        }
        uint32_t pw[EPI_COLS / 2];
#pragma unroll
        for (int j = 0; j < EPI_COLS / 2; ++j)
          pw[j] = epi_act2<ACT_T>(r[2 * j], r[2 * j + 1], bv, bv, g.lo, g.hi);
        uint4 *dst = reinterpret_cast<uint4 *>(stage + lane * EPI_ROWB);
        dst[0] = make_uint4(pw[0], pw[1], pw[2], pw[3]);
        dst[1] = make_uint4(pw[4], pw[5], pw[6], pw[7]);
        __syncwarp();
        if (g.omode) {
          // staged [32 channels][16 positions] -> 64 slots of 8 channels x 1
          // position; lane k takes slots k and k + 32
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int id = lane + 32 * k;
            const int pos = id & 15, grp = id >> 4;
            const uint8_t *colp = stage + pos * 2;
            uint32_t wv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t lo = *reinterpret_cast<const uint16_t *>(colp + (grp * 8 + 2 * e) * EPI_ROWB);
              const uint32_t hi =
                  *reinterpret_cast<const uint16_t *>(colp + (grp * 8 + 2 * e + 1) * EPI_ROWB);
              wv[e] = lo | (hi << 16);
            }
            const int P = int(p0) + col0 + pos;
            const int ohh = div_wp(g, P), oww = P - ohh * g.Wp;
            const int c = oc0 + grp * 8;
            if (ohh < g.OH && oww < g.OW && c < g.OC) {
              uint4 *slot = xs_slot(g, b, c, ohh, oww);
              if (slot && oxs_ok(g, slot)) *slot = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
          }
          __syncwarp();
          ow += EPI_COLS;
          while (ow >= g.Wp) {
            ow -= g.Wp;
            ++oh;
          }
          continue;
        }
        const bool v0 = oh < g.OH && ow < g.OW;
        const int off0 = oh * g.OW + ow;
        // second position: next column, or the first column of the next row
        const bool wrap = ow + 1 >= g.Wp;
        const bool v1 = wrap ? (oh + 1 < g.OH) : (oh < g.OH && ow + 1 < g.OW);
        const int off1 = wrap ? (oh + 1) * g.OW : off0 + 1;
        if constexpr (EXT) {
        const uint8_t *src = stage + rsel * EPI_ROWB + 4 * sub;
        // residual pairs of this lane's 8 rows, all loads issued before use
        uint32_t rv[8];
        if (g.resid) {
#pragma unroll
          for (int r4 = 0; r4 < 8; ++r4) {
            rv[r4] = 0;
            if (4 * r4 + rsel < nrows) {
              const __half *rrow = g.resid + (size_t(b) * g.OC + oc0 + rsel + 4 * r4) * plane;
              if (pairs) {
                if (v0) rv[r4] = *reinterpret_cast<const uint32_t *>(rrow + off0);
              } else {
                const uint32_t lo =
                    v0 ? uint32_t(*reinterpret_cast<const uint16_t *>(rrow + off0)) : 0u;
                const uint32_t hi =
                    v1 ? uint32_t(*reinterpret_cast<const uint16_t *>(rrow + off1)) : 0u;
                rv[r4] = lo | (hi << 16);
              }
            }
          }
        }
#pragma unroll
        for (int r4 = 0; r4 < 8; ++r4) {
          uint32_t val = *reinterpret_cast<const uint32_t *>(src + r4 * 4 * EPI_ROWB);
          if (4 * r4 + rsel < nrows) {
            const int c = oc0 + rsel + 4 * r4;
            __half *orow = g.nout ? out_plane(g, out, b, c, plane) : rowp + size_t(r4) * 4 * plane;
            if (g.resid) val = add_resid2(val, rv[r4]);
            if (pairs) {
              if (v0 && out_ok(g, out, orow + off0, 4))
                *reinterpret_cast<uint32_t *>(orow + off0) = val;
            } else {
              const __half2 h2 = *reinterpret_cast<const __half2 *>(&val);
              if (v0 && out_ok(g, out, orow + off0, 2)) orow[off0] = __low2half(h2);
              if (v1 && out_ok(g, out, orow + off1, 2)) orow[off1] = __high2half(h2);
            }
          }
        }
        } else {
        const uint8_t *src = stage + rsel * EPI_ROWB + 4 * sub;
#pragma unroll
        for (int r4 = 0; r4 < 8; ++r4) {
          const uint32_t val = *reinterpret_cast<const uint32_t *>(src + r4 * 4 * EPI_ROWB);
          if (4 * r4 + rsel < nrows) {
            __half *orow = rowp + size_t(r4) * 4 * plane;
            if (pairs) {
              if (v0 && out_ok(g, out, orow + off0, 4))
                *reinterpret_cast<uint32_t *>(orow + off0) = val;
            } else {
              const __half2 h2 = *reinterpret_cast<const __half2 *>(&val);
              if (v0 && out_ok(g, out, orow + off0, 2)) orow[off0] = __low2half(h2);
              if (v1 && out_ok(g, out, orow + off1, 2)) orow[off1] = __high2half(h2);
            }
          }
        }
        }
        __syncwarp();
        ow += EPI_COLS;
        while (ow >= g.Wp) {
          ow -= g.Wp;
          ++oh;
        }
      }
    }
  }
  }
#ifdef WGX_PROF
  if (warp == EPI_WARP0 && lane == 0) g_umma_prof[blockIdx.x][14] = global_ns();
#endif
  tc_fence_before();
  __syncthreads();
#ifdef WGX_PROF
  if (threadIdx.x == 0) g_umma_prof[blockIdx.x][15] = global_ns();
#endif
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

void umma_conv_pack_weights(const wgx_conv2d_params &p, const __half *w, void *packed,
                            cudaStream_t stream) {
  UmmaGeom g = make_geom(p);
  const uint64_t n = umma_conv_packed_weight_bytes(p) / 16;
  if (n >= (1ull << 31)) fail("conv2d: weights too large for the tensor-core path");
  pack_weights<<<unsigned((n + 255) / 256), 256, 0, stream>>>(g, w, static_cast<uint4 *>(packed),
                                                              int(n));
  check_cuda(cudaGetLastError(), "pack_weights launch");
}

bool umma_conv_link_ok(const wgx_conv2d_params &prod, const wgx_conv2d_params &cons) {
  return umma_conv_supported(prod) && umma_conv_supported(cons) && prod.B == cons.B &&
         prod.OC == cons.IC && prod.OH == cons.IH && prod.OW == cons.IW && prod.OC % 8 == 0;
}

void umma_conv_run(const wgx_conv2d_params &p, const __half *in, void *packed,
                   const __half *w_to_pack, const __half *bias, __half *out, void *xs,
                   cudaStream_t stream, const UmmaLink *link) {
  const bool per_image_w = link && link->per_image_weights;
  if (!umma_conv_supported(p, per_image_w))
    fail("conv2d: shape not supported by the tensor-core path");
  UmmaGeom g = make_geom(p, per_image_w);
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  g.err = device_error_word(dev);
  g.inject_skip = inject_skip_loads() ? 1 : 0;
  g.split = split_mode() != 0;
  // extents for the bounds-checking build
  g.out_bytes = uint64_t(p.B) * p.OC * p.OH * p.OW * 2;
  g.xs_bytes = umma_conv_input_bytes(p, per_image_w);
  g.wpk_bytes = uint64_t(per_image_w ? p.B : 1) * umma_conv_packed_weight_bytes(p, per_image_w);
  if ((reinterpret_cast<uintptr_t>(xs) & 15) || (reinterpret_cast<uintptr_t>(packed) & 15))
    fail("conv2d: scratch must be 16-byte aligned");
  // ---- input sources
  bool srcs_aligned = (reinterpret_cast<uintptr_t>(in) & 15) == 0;
  if (link && link->nsrc > 0) {
    if (link->nsrc > kMaxSrc) fail("conv2d: too many concatenated inputs");
    g.nsrc = link->nsrc;
    g.src_c0[0] = 0;
    srcs_aligned = true;
    for (int k = 0; k < link->nsrc; ++k) {
      if (link->src_ch[k] % 8) fail("conv2d: concatenated input channels must be multiples of 8");
      g.src[k] = link->src[k];
      g.src_c0[k + 1] = g.src_c0[k] + link->src_ch[k];
      srcs_aligned = srcs_aligned && (reinterpret_cast<uintptr_t>(link->src[k]) & 15) == 0;
    }
    if (g.src_c0[g.nsrc] != p.IC) fail("conv2d: concatenated inputs do not add up to IC");
  } else {
    g.nsrc = 1;
    g.src[0] = in;
    g.src_c0[0] = 0;
    g.src_c0[1] = p.IC;
  }
  // ---- output into the consumer's re-laid input
  if (link && link->consumer) {
    if (!umma_conv_link_ok(p, *link->consumer)) fail("conv2d: invalid producer/consumer link");
    if (reinterpret_cast<uintptr_t>(link->consumer_xs) & 15)
      fail("conv2d: consumer buffer must be 16-byte aligned");
    const UmmaGeom c = make_geom(*link->consumer);
    g.omode = 1;
    g.oHp = c.Hp;
    g.oWp = c.Wp;
    g.oplanes = c.C8 / 8;
    g.opH = c.pH;
    g.opW = c.pW;
    g.osH = c.sH;
    g.osW = c.sW;
    g.onphW = c.nphW;
    g.oxIC = c.xIC;
    for (int k = 0; k < 4; ++k) g.ophase_h[k] = g.ophase_w[k] = -1;
    if (c.sH == 1 && c.sW == 1) {
      g.ophase_h[0] = g.ophase_w[0] = 0;
    } else {
      for (int k = 0; k < c.nphH; ++k) g.ophase_h[c.phH[k]] = k;
      for (int k = 0; k < c.nphW; ++k) g.ophase_w[c.phW[k]] = k;
    }
    g.oxs = static_cast<uint4 *>(link->consumer_xs);
    g.oxs_bytes = umma_conv_input_bytes(*link->consumer);
  }
  const bool xs_ready = link && link->xs_ready;
  if (xs_ready && w_to_pack) fail("conv2d: weights must be packed before a linked launch");
  // ---- NCHW output options
  if (link && (link->resid || link->nout > 0)) {
    if (g.omode) fail("conv2d: a linked output cannot also be split or take a residual");
    g.resid = link->resid;
    if (link->nout > 0) {
      if (link->nout > kMaxOut) fail("conv2d: too many output pieces");
      g.nout = link->nout;
      g.out_c0[0] = 0;
      for (int k = 0; k < link->nout; ++k) {
        g.outp[k] = link->outp[k];
        g.out_c0[k + 1] = g.out_c0[k] + link->out_ch[k];
        g.outp_bytes[k] = uint64_t(p.B) * link->out_ch[k] * p.OH * p.OW * 2;
      }
      if (g.out_c0[g.nout] != p.OC) fail("conv2d: output pieces do not add up to OC");
    }
  }
  // ---- direct mode: 1x1 / stride 1 / no padding reads NCHW through TMA
  TmapSet tm;
  std::memset(&tm, 0, sizeof tm);
  {
    const int64_t hw = int64_t(p.IH) * p.IW;
    bool direct = !xs_ready && (!link || link->allow_direct) && p.KH == 1 && p.KW == 1 &&
                  p.sH == 1 && p.sW == 1 && p.pH == 0 &&
                  p.pW == 0 && hw % 8 == 0 && srcs_aligned && g.tile_pos % 64 == 0 &&
                  hw < (1ll << 31) && g.b_stage_bytes % 1024 == 0;
    // channel box: a whole stage (bk channels) for one source; for a
    // concatenation the largest of bk, 16, 8 dividing every source's channel
    // count, so that no box straddles two sources
    int dbox = g.bk;
    while (g.nsrc > 1 && dbox > 8) {
      bool fits = true;
      for (int k = 0; k < g.nsrc; ++k) fits = fits && (g.src_c0[k + 1] - g.src_c0[k]) % dbox == 0;
      if (fits) break;
      dbox /= 2;
    }
    for (int k = 0; k < g.nsrc && direct; ++k)
      direct = (g.src_c0[k + 1] - g.src_c0[k]) % dbox == 0 || g.nsrc == 1;
    if (direct) {
      g.direct = 1;
      g.dbox = dbox;
      for (int k = 0; k < g.nsrc; ++k)
        encode_nchw_tmap(&tm.m[k], g.src[k], p.B, g.src_c0[k + 1] - g.src_c0[k], int(hw), dbox);
    }
  }
  // per-image weights: packed image after image (streamed per stage)
  g.w_img_bytes = 0;
  if (per_image_w) {
    g.w_img_bytes = umma_conv_packed_weight_bytes(p, true);
    if (w_to_pack) {
      const long long n_img = (long long)(g.w_img_bytes / 16);
      if (n_img >= (1ll << 31)) fail("conv2d: weights too large for the tensor-core path");
      const long long total = n_img * p.B;
      pack_weights_batched<<<unsigned((total + 255) / 256), 256, 0, stream>>>(
          g, w_to_pack, static_cast<uint4 *>(packed), int(n_img),
          (long long)p.OC * p.IC * p.KH * p.KW, total);
      check_cuda(cudaGetLastError(), "pack_weights launch");
    }
  }
  // shared weights still to pack (fused into the re-layout launch where it can be)
  const __half *wtp = per_image_w ? nullptr : w_to_pack;
  const uint64_t n_w64 = wtp ? umma_conv_packed_weight_bytes(p) / 16 : 0;
  if (n_w64 >= (1ull << 31)) fail("conv2d: weights too large for the tensor-core path");
  const int n_w = int(n_w64);
  const bool strided = g.sH != 1 || g.sW != 1;
  const int th_pack = (xs_ready || g.direct) ? -1 : timer_begin("umma_conv_pack", stream);
  if (xs_ready) {
    // re-laid by the producer
  } else if (g.direct) {
    // read from NCHW by the kernel's TMA loads; only the weights may need packing
    if (wtp)
      pack_weights<<<unsigned((n_w + 255) / 256), 256, 0, stream>>>(
          g, wtp, static_cast<uint4 *>(packed), n_w);
  } else if (strided) {
    if (wtp)
      pack_weights<<<unsigned((n_w + 255) / 256), 256, 0, stream>>>(
          g, wtp, static_cast<uint4 *>(packed), n_w);
    if (g.sW == 2 && g.nphW == 2 && g.phW[0] == 0 && g.phW[1] == 1 && g.xIC % 8 == 0 &&
        g.IW % 8 == 0 && g.C8 == g.IC && srcs_aligned) {
      const int qbase = -4 * ((g.pW + 3) / 4);
      const int groups_per_row = (g.Wp - g.pW - qbase + 3) / 4;
      const long long n_items =
          (long long)g.B * (g.xIC / 8) * g.Hp * g.nphH * groups_per_row;
      if (n_items >= (1ll << 31) - 256) fail("conv2d: input too large for the re-layout kernel");
      pack_input_s2d_v8<<<unsigned((n_items + 255) / 256), 256, 0, stream>>>(
          g, in, static_cast<uint4 *>(xs), groups_per_row, qbase, int(n_items));
    } else if (g.sH == 2 && g.sW == 2 && g.nphH == 2 && g.nphW == 2 && g.xIC < 8 &&
               g.C8 <= 32 && g.IW % 8 == 0 && srcs_aligned) {
      const int qbase = -4 * ((g.pW + 3) / 4);
      const int groups_per_row = (g.Wp - g.pW - qbase + 3) / 4;
      const long long n_items = (long long)g.B * g.Hp * groups_per_row;
      if (n_items >= (1ll << 31) - 256) fail("conv2d: input too large for the re-layout kernel");
      const unsigned blocks = unsigned((n_items + 255) / 256);
      uint4 *o = static_cast<uint4 *>(xs);
      switch (g.xIC) {
        case 1: pack_input_s2d_small<1><<<blocks, 256, 0, stream>>>(g, o, groups_per_row, qbase, int(n_items)); break;
        case 2: pack_input_s2d_small<2><<<blocks, 256, 0, stream>>>(g, o, groups_per_row, qbase, int(n_items)); break;
        case 3: pack_input_s2d_small<3><<<blocks, 256, 0, stream>>>(g, o, groups_per_row, qbase, int(n_items)); break;
        case 4: pack_input_s2d_small<4><<<blocks, 256, 0, stream>>>(g, o, groups_per_row, qbase, int(n_items)); break;
        case 5: pack_input_s2d_small<5><<<blocks, 256, 0, stream>>>(g, o, groups_per_row, qbase, int(n_items)); break;
        case 6: pack_input_s2d_small<6><<<blocks, 256, 0, stream>>>(g, o, groups_per_row, qbase, int(n_items)); break;
        default: pack_input_s2d_small<7><<<blocks, 256, 0, stream>>>(g, o, groups_per_row, qbase, int(n_items)); break;
      }
    } else {
      const long long n_slots = (long long)g.B * (g.C8 / 8) * g.plane_rows;
      pack_input_s2d<<<unsigned((n_slots + 255) / 256), 256, 0, stream>>>(
          g, in, static_cast<uint4 *>(xs), n_slots);
    }
  } else if (g.IW % 8 == 0 && srcs_aligned) {
    // input re-layout and weight packing in one launch
    const int groups_per_row = (g.Wp - (g.pW & 7) + 8 + 7) / 8;
    const long long n_items = (long long)g.B * (g.C8 / 8) * g.Hp * groups_per_row;
    if (n_items >= (1ll << 31) - 256) fail("conv2d: input too large for the re-layout kernel");
    const int n_in_blocks = int((n_items + 255) / 256);
    const int n_wblk = (n_w + 255) / 256;
    pack_input_v8<<<unsigned(n_in_blocks + n_wblk), 256, 0, stream>>>(
        g, in, static_cast<uint4 *>(xs), groups_per_row, int(n_items), n_in_blocks, wtp,
        static_cast<uint4 *>(packed), n_w);
  } else {
    if (wtp)
      pack_weights<<<unsigned((n_w + 255) / 256), 256, 0, stream>>>(
          g, wtp, static_cast<uint4 *>(packed), n_w);
    if (g.IW % 4 == 0 && srcs_aligned) {
      const int groups_per_row = (g.Wp - (g.pW & 3) + 4 + 3) / 4;
      long long n = (long long)g.B * (g.C8 / 8) * g.Hp * groups_per_row;
      pack_input_v4<<<unsigned((n + 255) / 256), 256, 0, stream>>>(
          g, in, static_cast<uint4 *>(xs), groups_per_row, n);
    } else {
      long long n_slots = (long long)g.B * (g.C8 / 8) * g.plane_rows;
      pack_input<<<unsigned((n_slots + 255) / 256), 256, 0, stream>>>(
          g, in, static_cast<uint4 *>(xs), n_slots);
    }
  }
  check_cuda(cudaGetLastError(), "pack_input launch");
  timer_end(th_pack, stream);
  uint32_t smem = smem_bytes(g);
  using KernelFn = void (*)(const UmmaGeom, const uint8_t *, const uint8_t *, const __half *,
                           __half *, const TmapSet);
  // specialisations: filter width (1/3/5/7, per-row 32-channel staging) x
  // epilogue activation
#define WGX_UMMA_ROW(KW, T) \
  { umma_conv_kernel<KW, 0, T, 0>, umma_conv_kernel<KW, 1, T, 0>, umma_conv_kernel<KW, 2, T, 0> }
#define WGX_UMMA_TRANS(T)                                                                  \
  {WGX_UMMA_ROW(0, T), WGX_UMMA_ROW(1, T), WGX_UMMA_ROW(2, T), WGX_UMMA_ROW(3, T),          \
   WGX_UMMA_ROW(0, T), WGX_UMMA_ROW(0, T), WGX_UMMA_ROW(0, T)}
  // [standard, transposed N = 16 / 32 / 64, N = 16 / 32 with 4 M blocks]
  // [filter width][activation]
  static const KernelFn table[6][7][3] = {
      {WGX_UMMA_ROW(0, 0), WGX_UMMA_ROW(1, 0), WGX_UMMA_ROW(2, 0), WGX_UMMA_ROW(3, 0),
       WGX_UMMA_ROW(4, 0), WGX_UMMA_ROW(5, 0), WGX_UMMA_ROW(7, 0)},
      WGX_UMMA_TRANS(16), WGX_UMMA_TRANS(32), WGX_UMMA_TRANS(64), WGX_UMMA_TRANS(17),
      WGX_UMMA_TRANS(33)};
#undef WGX_UMMA_TRANS
#undef WGX_UMMA_ROW
  int kw_idx = 0;
  if (g.khs == 1 && g.bk == 32)
    kw_idx = g.KW == 7 ? 6 : (g.KW >= 1 && g.KW <= 5) ? g.KW : 0;
  if (g.trans && kw_idx > 3) kw_idx = 0;  // transposed: specialised for KW <= 3 only
  const int act_idx = (g.act >= 0 && g.act <= 2) ? g.act : 0;
  // residual / split outputs: generic MMA loop, EXT epilogue
#define WGX_UMMA_EXT(T) \
  { umma_conv_kernel<0, 0, T, 1>, umma_conv_kernel<0, 1, T, 1>, umma_conv_kernel<0, 2, T, 1> }
  static const KernelFn table_ext[6][3] = {WGX_UMMA_EXT(0),  WGX_UMMA_EXT(16), WGX_UMMA_EXT(32),
                                           WGX_UMMA_EXT(64), WGX_UMMA_EXT(17), WGX_UMMA_EXT(33)};
#undef WGX_UMMA_EXT
  const int nt_idx = !g.trans ? 0 : g.NT == 64 ? 3 : (g.NT == 16 ? 1 : 2) + (g.G == 4 ? 3 : 0);
  if (g.trans && !g.hs && g.NT != 16 && g.NT != 32 && g.NT != 64)
    fail("conv2d: bad transposed tile");
  // 16-byte stores of the transposed epilogue (split pieces and residual
  // loads included)
  {
    bool aligned = g.nout > 0 || (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    for (int k = 0; k < g.nout; ++k)
      aligned = aligned && (reinterpret_cast<uintptr_t>(g.outp[k]) & 15) == 0;
    aligned = aligned && (reinterpret_cast<uintptr_t>(g.resid) & 15) == 0;
    g.tvec = g.trans && !g.omode && ((g.Wp | g.OW) & 7) == 0 && aligned;
  }
  // residual adds and split outputs the vector path cannot store: the EXT
  // epilogue
  const bool ext = (g.resid != nullptr || g.nout > 0) && !g.tvec;
  // folded filter columns: N = 32 / 48 / 96 / 192, generic MMA loop, own
  // epilogue (residual adds and splits included)
#define WGX_UMMA_HS(T) \
  { umma_conv_kernel<0, 0, T, 0, 1>, umma_conv_kernel<0, 1, T, 0, 1>, umma_conv_kernel<0, 2, T, 0, 1> }
  static const KernelFn table_hs[4][3] = {WGX_UMMA_HS(32), WGX_UMMA_HS(48), WGX_UMMA_HS(96),
                                          WGX_UMMA_HS(192)};
#undef WGX_UMMA_HS
  const int hs_idx = g.NT == 32 ? 0 : g.NT == 48 ? 1 : g.NT == 96 ? 2 : 3;
  if (g.hs && (g.NT != 32 && g.NT != 48 && g.NT != 96 && g.NT != 192))
    fail("conv2d: bad folded-column tile");
  KernelFn kern = g.hs  ? table_hs[hs_idx][act_idx]
                  : ext ? table_ext[nt_idx][act_idx]
                        : table[nt_idx][kw_idx][act_idx];
  const int kidx = g.hs  ? 144 + hs_idx * 3 + act_idx
                   : ext ? 126 + nt_idx * 3 + act_idx
                         : (nt_idx * 7 + kw_idx) * 3 + act_idx;
  // per (device, kernel) set-up, cached; host threads launching on one
  // device share the tables, so they are read and written under a lock
  static std::mutex setup_mu;
  static bool attr_set[64][160] = {};
  static int sms[64] = {};
  int n_sm = 0;
  {
    std::lock_guard<std::mutex> lock(setup_mu);
    if (dev >= 64 || !attr_set[dev][kidx]) {
      check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(SMEM_MAX)),
                 "umma_conv smem attr");
      if (dev < 64) attr_set[dev][kidx] = true;
    }
    if (dev < 64 && !sms[dev]) sms[dev] = sm_count();
    n_sm = dev < 64 ? sms[dev] : sm_count();
  }
  const int grid = g.total_tiles < n_sm ? g.total_tiles : n_sm;
  int th = timer_begin("umma_conv_kernel", stream);
  kern<<<grid, THREADS, smem, stream>>>(g, static_cast<const uint8_t *>(xs),
                                        static_cast<const uint8_t *>(packed), bias, out, tm);
  check_cuda(cudaGetLastError(), "umma_conv launch");
  timer_end(th, stream);
}

// ------------------------------------------------------- batched GEMM
// aten.bmm in fp16 on the tensor cores (src/shaders/bmm/index.ts:33-55:
// C[b] = A[b] B[b], A [batch, M, K], B [batch, K, N], row-major): the 1x1
// convolution of image b = B[b] (K channels of N positions, 1 x N) with
// the per-image weights A[b] (M output channels x K input channels), so the
// same tcgen05 pipeline, TMA reads of the [K][N] image (N % 8 == 0) and
// epilogue serve it; each image's packed weights stream per stage.
static wgx_conv2d_params bmm_params(int64_t batch, int64_t M, int64_t K, int64_t N) {
  wgx_conv2d_params p{};
  p.B = int(batch);
  p.IC = int(K);
  p.IH = 1;
  p.IW = int(N);
  p.OC = int(M);
  p.OH = 1;
  p.OW = int(N);
  p.KH = p.KW = 1;
  p.sH = p.sW = 1;
  p.dH = p.dW = 1;
  p.groups = 1;
  p.has_bias = 0;
  p.dtype = WGX_FLOAT16;
  p.act = WGX_ACT_NONE;
  p.out_min = -INFINITY;
  p.out_max = INFINITY;
  return p;
}

bool umma_bmm_supported(int64_t batch, int64_t M, int64_t K, int64_t N) {
  if (batch < 1 || M < 1 || K < 1 || N < 1 || batch > INT32_MAX || M > INT32_MAX ||
      K > INT32_MAX || N > INT32_MAX)
    return false;
  return umma_conv_supported(bmm_params(batch, M, K, N), true);
}

static uint64_t align256(uint64_t v) { return (v + 255) / 256 * 256; }

uint64_t umma_bmm_scratch_bytes(int64_t batch, int64_t M, int64_t K, int64_t N) {
  const wgx_conv2d_params p = bmm_params(batch, M, K, N);
  return align256(uint64_t(batch) * umma_conv_packed_weight_bytes(p, true)) +
         umma_conv_input_bytes(p, true);
}

void umma_bmm_run(const __half *A, const __half *B, __half *C, int64_t batch, int64_t M, int64_t K,
                  int64_t N, void *scratch, uint64_t scratch_bytes, cudaStream_t stream) {
  const wgx_conv2d_params p = bmm_params(batch, M, K, N);
  if (scratch_bytes < umma_bmm_scratch_bytes(batch, M, K, N))
    fail("aten.bmm.default: scratch too small");
  UmmaLink link;
  link.per_image_weights = true;
  char *base = static_cast<char *>(scratch);
  void *xs = base + align256(uint64_t(batch) * umma_conv_packed_weight_bytes(p, true));
  umma_conv_run(p, B, base, A, nullptr, C, xs, stream, &link);
}

}  // namespace wgx

#ifdef WGX_PROF
// Reads (and clears) the per-CTA role counters of the last launches.
extern "C" __attribute__((visibility("default"))) int wgx_umma_prof_read(unsigned long long *out) {
  if (cudaDeviceSynchronize() != cudaSuccess) return 1;
  if (cudaMemcpyFromSymbol(out, wgx::g_umma_prof, sizeof(wgx::g_umma_prof)) != cudaSuccess) return 1;
  static unsigned long long zero[256][20] = {};
  return cudaMemcpyToSymbol(wgx::g_umma_prof, zero, sizeof(zero)) != cudaSuccess;
}
#endif
