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
//    layout xs[b][c/8][Hp][Wp][8] (Hp = IH+2pH, Wp = IW+2pW, channels padded
//    to a multiple of 32). One "row" = one padded position = 16 bytes.
//    Flattening (hp, wp) to p = hp*Wp + wp turns a stride-1 convolution into
//    out[p] = sum_taps W_tap . xs[p + kh*dH*Wp + kw*dW]: every tap is a pure
//    row shift.
//  * operands in shared memory use the canonical K-major no-swizzle layout
//    (core matrix = 8 rows x 16 bytes, rows 16 bytes apart, 8-channel chunks
//    one plane apart). A row shift is then just a 16-byte move of the
//    descriptor start address, so one staged activation tile feeds all KW
//    taps of a filter row.
//  * weights packed by pack_weights into [oc_tile][kh][cblk][kw][chunk][128][8]
//    so the A operand of one pipeline stage is one contiguous bulk copy.
//
// CTA = 128 output channels x 512 positions (two N=256 accumulators, 512
// TMEM columns). Pipeline stage = (kh, 32-channel block): A = KW x 128 x 32,
// B = (512 + (KW-1)*dW) rows x 32 channels. Warp roles: warp 0 issues the
// bulk copies, warp 1 owns TMEM and issues tcgen05.mma, warps 4-7 drain TMEM
// (tcgen05.ld) through bias + activation to global memory.
//
// Every mbarrier wait is bounded (about 2 s of %globaltimer); on expiry the
// waiting role sets a bit in the device error word and stops, so a broken
// pipeline returns an error instead of hanging the GPU.
#include "umma_conv.h"

namespace wgx {

constexpr int UM = 128;        // MMA M (output channels per CTA)
constexpr int UN = 256;        // MMA N per instruction
constexpr int NACC = 2;        // accumulators per CTA
constexpr int NT = UN * NACC;  // positions per CTA
constexpr int BK = 32;         // channels per pipeline stage
constexpr int CHUNKS = BK / 8;
constexpr int THREADS = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr int MAX_KW = 7;
constexpr uint64_t WAIT_NS = 2000000000ull;

struct UmmaGeom {
  int B, IC, IH, IW, OC, OH, OW, KH, KW, dH, dW, pH, pW;
  int Hp, Wp, C8, ncb, n_oct, tiles_per_img, R, R_alloc, stages, n_kstages;
  long long plane_rows;  // Hp*Wp
  uint32_t a_stage_bytes, b_stage_bytes;
  int has_bias, act;
  float lo, hi;
  uint32_t *err;
};

static UmmaGeom make_geom(const wgx_conv2d_params &p) {
  UmmaGeom g{};
  g.B = p.B;
  g.IC = p.IC;
  g.IH = p.IH;
  g.IW = p.IW;
  g.OC = p.OC;
  g.OH = p.OH;
  g.OW = p.OW;
  g.KH = p.KH;
  g.KW = p.KW;
  g.dH = p.dH;
  g.dW = p.dW;
  g.pH = p.pH;
  g.pW = p.pW;
  g.Hp = p.IH + 2 * p.pH;
  g.Wp = p.IW + 2 * p.pW;
  g.C8 = (p.IC + BK - 1) / BK * BK;
  g.ncb = g.C8 / BK;
  g.n_oct = (p.OC + UM - 1) / UM;
  g.plane_rows = (long long)g.Hp * g.Wp;
  long long p_out = (long long)(p.OH - 1) * g.Wp + p.OW;
  g.tiles_per_img = int((p_out + NT - 1) / NT);
  g.R = NT + (p.KW - 1) * p.dW;
  g.R_alloc = (g.R + 7) / 8 * 8;
  g.a_stage_bytes = uint32_t(p.KW) * CHUNKS * UM * 16;
  g.b_stage_bytes = uint32_t(CHUNKS) * g.R_alloc * 16;
  g.n_kstages = p.KH * g.ncb;
  uint32_t stage = g.a_stage_bytes + g.b_stage_bytes;
  int st = int((220u * 1024u) / stage);
  if (st > 6) st = 6;
  if (st > g.n_kstages) st = g.n_kstages;
  if (st < 1) st = 1;
  g.stages = st;
  g.has_bias = p.has_bias;
  g.act = p.act;
  g.lo = p.out_min;
  g.hi = p.out_max;
  return g;
}

// Dynamic shared memory of one CTA. Never below 120 KB, so that at most
// one CTA is resident per SM and the 512-column TMEM allocation of a CTA
// never waits on another CTA of the same kernel.
static uint32_t smem_bytes(const UmmaGeom &g) {
  uint32_t need = uint32_t(g.stages) * (g.a_stage_bytes + g.b_stage_bytes) +
                  (2 * g.stages + 1) * 8 + 16 + 128;
  return need < 120u * 1024u ? 120u * 1024u : need;
}

bool umma_conv_supported(const wgx_conv2d_params &p) {
  if (p.dtype != WGX_FLOAT16 || p.groups != 1) return false;
  if (p.sH != 1 || p.sW != 1) return false;
  if (p.KW > MAX_KW || p.IC < 8) return false;
  if (p.dH < 1 || p.dW < 1) return false;
  // stride-1 geometry must be consistent with the padded flattening
  if (p.OH != p.IH + 2 * p.pH - p.dH * (p.KH - 1)) return false;
  if (p.OW != p.IW + 2 * p.pW - p.dW * (p.KW - 1)) return false;
  UmmaGeom g = make_geom(p);
  if (g.stages < 2 && g.n_kstages > 1) return false;
  if (smem_bytes(g) > 227u * 1024u) return false;
  if (g.R_alloc * 16 >= (1 << 18)) return false;  // LBO field range
  if (g.B > 65535 || g.n_oct > 65535) return false;
  return true;
}

uint64_t umma_conv_grid(const wgx_conv2d_params &p) {
  UmmaGeom g = make_geom(p);
  return uint64_t(g.tiles_per_img) * g.n_oct * g.B;
}

uint64_t umma_conv_packed_weight_bytes(const wgx_conv2d_params &p) {
  UmmaGeom g = make_geom(p);
  return uint64_t(g.n_oct) * g.KH * g.ncb * g.a_stage_bytes;
}

// Rows the main kernel may read: the last tile's B stage of the last filter
// row starts at (tiles*NT - NT) + (KH-1)*dH*Wp and spans R rows. Rows past
// the image only feed output positions that are discarded.
static uint64_t input_rows_total(const UmmaGeom &g) {
  uint64_t planes = uint64_t(g.B) * (g.C8 / 8);
  uint64_t last_end = uint64_t(g.tiles_per_img - 1) * NT + uint64_t(g.KH - 1) * g.dH * g.Wp + g.R;
  uint64_t slack = last_end > uint64_t(g.plane_rows) ? last_end - g.plane_rows : 0;
  return planes * g.plane_rows + slack;
}

uint64_t umma_conv_input_bytes(const wgx_conv2d_params &p) {
  UmmaGeom g = make_geom(p);
  return (input_rows_total(g) * 16 + 255) / 256 * 256;
}

// --------------------------------------------------------------- re-layout
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
  const __half *src = x + ((b * g.IC + cb * 8) * g.IH + ih) * (long long)g.IW + iw;
  long long cstride = (long long)g.IH * g.IW;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    int c = cb * 8 + e;
    v[e] = (inside && c < g.IC) ? src[e * cstride] : __float2half_rn(0.f);
  }
  xs[i] = *reinterpret_cast<const uint4 *>(v);
}

// packed[oct][kh][cbk][kw][chunk][row 0..127][8] <- w[oc][c][kh][kw]
__global__ void pack_weights(UmmaGeom g, const __half *__restrict__ w, uint4 *__restrict__ packed,
                             long long n_slots) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_slots) return;
  int row = int(i % UM);
  long long t = i / UM;
  int chunk = int(t % CHUNKS);
  t /= CHUNKS;
  int kw = int(t % g.KW);
  t /= g.KW;
  int cbk = int(t % g.ncb);
  t /= g.ncb;
  int kh = int(t % g.KH);
  int oct = int(t / g.KH);
  int oc = oct * UM + row;
  __align__(16) __half v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    int c = cbk * BK + chunk * 8 + e;
    v[e] = (oc < g.OC && c < g.IC) ? w[(((long long)oc * g.IC + c) * g.KH + kh) * g.KW + kw]
                                   : __float2half_rn(0.f);
  }
  packed[i] = *reinterpret_cast<const uint4 *>(v);
}

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Bounded wait: true when the phase with `parity` completed, false after
// WAIT_NS (the caller then records the error and stops its role).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  uint64_t t0 = global_ns();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (global_ns() - t0 > WAIT_NS) return false;
  }
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// K-major, no swizzle: rows 16 B apart (SBO = 128 B between 8-row core
// matrices), the two 8-element K chunks of one MMA `lbo` bytes apart.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= uint64_t((addr & 0x3FFFF) >> 4);
  d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
  d |= uint64_t((128u >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;  // descriptor version for sm_100
  return d;                // base offset 0, layout SWIZZLE_NONE (0)
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *r) {
  uint32_t *u = reinterpret_cast<uint32_t *>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
        "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]),
        "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]), "=r"(u[25]),
        "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float epi_act(float v, int act, float lo, float hi) {
  if (act == WGX_ACT_CLAMP) return fminf(fmaxf(v, lo), hi);
  if (act == WGX_ACT_SILU) return v / (1.0f + __expf(-v));
  return v;
}

// ------------------------------------------------------------ main kernel
__global__ void __launch_bounds__(THREADS, 1)
    umma_conv_kernel(const UmmaGeom g, const uint8_t *__restrict__ xs,
                     const uint8_t *__restrict__ wpk, const __half *__restrict__ bias,
                     __half *__restrict__ out) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                              ~uintptr_t(127));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tile = blockIdx.x, oct = blockIdx.y, b = blockIdx.z;
  const int S = g.stages;
  uint8_t *sA = smem;
  uint8_t *sB = smem + size_t(S) * g.a_stage_bytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sB + size_t(S) * g.b_stage_bytes);
  uint64_t *full = bars, *empty = bars + S, *accf = bars + 2 * S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accf + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(accf), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
  const long long p0 = (long long)tile * NT;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: bulk copies of weights + activation rows
      const uint32_t b_bytes_copied = uint32_t(g.R) * 16;
      for (int s = 0; s < g.n_kstages; ++s) {
        const int slot = s % S, use = s / S;
        if (use > 0 && !mbar_wait(smem_u32(&empty[slot]), (use - 1) & 1)) {
          atomicOr(g.err, kErrLoadTimeout);
          break;
        }
        const int kh = s / g.ncb, cbk = s % g.ncb;
        const uint32_t fb = smem_u32(&full[slot]);
        mbar_expect_tx(fb, g.a_stage_bytes + CHUNKS * b_bytes_copied);
        const uint8_t *asrc = wpk + ((size_t(oct) * g.KH + kh) * g.ncb + cbk) * g.a_stage_bytes;
        bulk_g2s(smem_u32(sA + size_t(slot) * g.a_stage_bytes), asrc, g.a_stage_bytes, fb);
        const long long row0 = p0 + (long long)kh * g.dH * g.Wp;
        for (int ch = 0; ch < CHUNKS; ++ch) {
          const long long plane = (long long)b * (g.C8 / 8) + cbk * CHUNKS + ch;
          const uint8_t *bsrc = xs + (plane * g.plane_rows + row0) * 16;
          bulk_g2s(smem_u32(sB + size_t(slot) * g.b_stage_bytes + size_t(ch) * g.R_alloc * 16),
                   bsrc, b_bytes_copied, fb);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc = (1u << 4)                      // D = f32
                             | (uint32_t(UN >> 3) << 17)    // N
                             | (uint32_t(UM >> 4) << 24);   // M; A,B f16 K-major
      const uint32_t a_lbo = UM * 16;                       // chunk plane of A
      const uint32_t b_lbo = uint32_t(g.R_alloc) * 16;      // chunk plane of B
      bool ok = true;
      for (int s = 0; s < g.n_kstages && ok; ++s) {
        const int slot = s % S, use = s / S;
        if (!mbar_wait(smem_u32(&full[slot]), use & 1)) {
          atomicOr(g.err, kErrMmaTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + size_t(slot) * g.a_stage_bytes);
        const uint32_t b_base = smem_u32(sB + size_t(slot) * g.b_stage_bytes);
        for (int kw = 0; kw < g.KW; ++kw) {
#pragma unroll
          for (int ks = 0; ks < BK / 16; ++ks) {
            const uint64_t adesc =
                kmajor_desc(a_base + uint32_t(kw) * CHUNKS * UM * 16 + ks * 2 * a_lbo, a_lbo);
#pragma unroll
            for (int h = 0; h < NACC; ++h) {
              const uint64_t bdesc = kmajor_desc(
                  b_base + uint32_t(h * UN + kw * g.dW) * 16 + ks * 2 * b_lbo, b_lbo);
              mma_f16(tmem + h * UN, adesc, bdesc, idesc, (s | kw | ks) != 0);
            }
          }
        }
        mma_commit(smem_u32(&empty[slot]));
      }
      mma_commit(smem_u32(accf));
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: TMEM -> bias + activation -> NCHW fp16
    const int q = warp & 3;
    const int oc = oct * UM + q * 32 + lane;
    const bool ok = mbar_wait(smem_u32(accf), 0);
    if (!ok && lane == 0) atomicOr(g.err, kErrEpilogueTimeout);
    tc_fence_after();
    const float bv = (g.has_bias && oc < g.OC) ? __half2float(bias[oc]) : 0.f;
    __half *obase = out + ((long long)b * g.OC + (oc < g.OC ? oc : 0)) * g.OH * (long long)g.OW;
    float r[32];
    for (int h = 0; h < NACC; ++h) {
      for (int c = 0; c < UN / 32; ++c) {
        tmem_ld32(tmem + (uint32_t(q * 32) << 16) + h * UN + c * 32, r);
        long long pb = p0 + h * UN + c * 32;
        int oh = int(pb / g.Wp), ow = int(pb % g.Wp);
        if (ok && oc < g.OC) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (oh < g.OH && ow < g.OW)
              obase[(long long)oh * g.OW + ow] =
                  __float2half_rn(epi_act(r[j] + bv, g.act, g.lo, g.hi));
            if (++ow == g.Wp) {
              ow = 0;
              ++oh;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
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
  long long n = (long long)(umma_conv_packed_weight_bytes(p) / 16);
  pack_weights<<<unsigned((n + 255) / 256), 256, 0, stream>>>(g, w, static_cast<uint4 *>(packed),
                                                              n);
  check_cuda(cudaGetLastError(), "pack_weights launch");
}

void umma_conv_run(const wgx_conv2d_params &p, const __half *in, const void *packed,
                   const __half *bias, __half *out, void *xs, cudaStream_t stream) {
  if (!umma_conv_supported(p)) fail("conv2d: shape not supported by the tensor-core path");
  UmmaGeom g = make_geom(p);
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  g.err = device_error_word(dev);
  if ((reinterpret_cast<uintptr_t>(xs) & 15) || (reinterpret_cast<uintptr_t>(packed) & 15))
    fail("conv2d: scratch must be 16-byte aligned");
  long long n_slots = (long long)g.B * (g.C8 / 8) * g.plane_rows;
  pack_input<<<unsigned((n_slots + 255) / 256), 256, 0, stream>>>(g, in, static_cast<uint4 *>(xs),
                                                                 n_slots);
  check_cuda(cudaGetLastError(), "pack_input launch");
  uint32_t smem = smem_bytes(g);
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    check_cuda(cudaFuncSetAttribute(umma_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    227 * 1024),
               "umma_conv smem attr");
    attr_set[dev] = true;
  }
  dim3 grid(unsigned(g.tiles_per_img), unsigned(g.n_oct), unsigned(g.B));
  umma_conv_kernel<<<grid, THREADS, smem, stream>>>(g, static_cast<const uint8_t *>(xs),
                                                    static_cast<const uint8_t *>(packed), bias,
                                                    out);
  check_cuda(cudaGetLastError(), "umma_conv launch");
}

}  // namespace wgx
