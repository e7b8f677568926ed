// CUDA-core convolution kernels and the convolution dispatcher.
//
// The reference computes every aten.convolution / et_vk.conv_with_clamp
// variant with WGSL kernels (src/shaders/convolution/*.wgsl.ts,
// src/shaders/conv-with-clamp/*.wgsl.ts) selected in
// src/shaders/convolution/index.ts:171-238 and
// src/shaders/conv-with-clamp/index.ts:173-243. Here the dense fp16 case
// runs on tcgen05 tensor cores (umma_conv.cu); this file holds the
// remaining variants:
//   * simt_gemm_conv: fp32 (and odd-shaped fp16) implicit-im2col GEMM,
//     the FFMA path for fp32 models (fp32 accumulation);
//   * depthwise: groups == IC == OC, memory bound, smem row tile, f32 acc;
//   * direct: any other grouping (grouped direct conv of conv2d.wgsl.ts);
//   * conv_transpose: transposed conv gather (conv-transpose2d.wgsl.ts);
//   * pointwise_single: 1x1 conv with one output channel, f32 accumulation
//     (conv-with-clamp-1x1-single-channel*.wgsl.ts).
// All of them apply bias, then the activation (clamp or SiLU) in fp32 and
// round once to the storage type.
#include <algorithm>
#include <mutex>

#include "internal.h"
#include "umma_conv.h"

namespace wgx {

template <class T>
__device__ __forceinline__ float ld_f(const T *p) {
  return float(*p);
}
template <>
__device__ __forceinline__ float ld_f<__half>(const __half *p) {
  return __half2float(*p);
}
template <class T>
__device__ __forceinline__ T to_t(float v);
template <>
__device__ __forceinline__ float to_t<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half to_t<__half>(float v) {
  return __float2half_rn(v);
}

__device__ __forceinline__ float apply_act(float v, int act, float lo, float hi) {
  if (act == WGX_ACT_CLAMP) return fminf(fmaxf(v, lo), hi);
  if (act == WGX_ACT_SILU) return v / (1.0f + __expf(-v));
  return v;
}

struct ConvGeom {
  int B, IC, IH, IW, OC, OH, OW, KH, KW, sH, sW, pH, pW, dH, dW, groups, has_bias, act;
  float lo, hi;
};

static ConvGeom geom_of(const wgx_conv2d_params &p) {
  return ConvGeom{p.B,  p.IC, p.IH, p.IW, p.OC, p.OH, p.OW,     p.KH,       p.KW,  p.sH, p.sW,
                  p.pH, p.pW, p.dH, p.dW, p.groups, p.has_bias, p.act, p.out_min, p.out_max};
}

// ---------------------------------------------------------------------------
// simt_gemm_conv: implicit-im2col GEMM on CUDA cores, groups == 1.
// GEMM view (as in conv2d-tile64.wgsl.ts:35-41): M = OC, N = B*OH*OW,
// K = IC*KH*KW, weights OIHW = [M, K] row-major, input gathered per
// element with zero fill outside the image. 64x64 tile, 256 threads, 4x4
// outputs per thread, K step 16, fp32 accumulation.
// ---------------------------------------------------------------------------
template <class T>
__global__ void __launch_bounds__(256) simt_gemm_conv(ConvGeom g, const T *__restrict__ x,
                                                      const T *__restrict__ w,
                                                      const T *__restrict__ bias,
                                                      T *__restrict__ out) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const long long M = g.OC;
  const long long ohw = (long long)g.OH * g.OW;
  const long long N = (long long)g.B * ohw;
  const long long K = (long long)g.IC * g.KH * g.KW;
  const int khw = g.KH * g.KW;
  const long long m0 = (long long)blockIdx.y * BM;
  const long long n0 = (long long)blockIdx.x * BN;

  // Each thread loads 4 weights (row a_r, k cols a_c..) and 4 inputs.
  const int a_r = tid / 4, a_c = (tid % 4) * 4;  // 64 rows x 16 k
  const int b_k = tid / 16, b_n = (tid % 16) * 4;  // 16 k x 64 n
  long long nb[4];
  int ihb[4], iwb[4];
  bool nv[4];
  for (int j = 0; j < 4; ++j) {
    long long n = n0 + b_n + j;
    nv[j] = n < N;
    long long nn = nv[j] ? n : 0;
    long long b = nn / ohw, sp = nn % ohw;
    int oh = int(sp / g.OW), ow = int(sp % g.OW);
    nb[j] = b;
    ihb[j] = oh * g.sH - g.pH;
    iwb[j] = ow * g.sW - g.pW;
  }
  float acc[4][4] = {};
  for (long long k0 = 0; k0 < K; k0 += BK) {
    for (int j = 0; j < 4; ++j) {
      long long m = m0 + a_r, k = k0 + a_c + j;
      As[a_c + j][a_r] = (m < M && k < K) ? ld_f(&w[m * K + k]) : 0.f;
    }
    {
      long long k = k0 + b_k;
      int ic = 0, kh = 0, kw = 0;
      bool kv = k < K;
      if (kv) {
        ic = int(k / khw);
        int r = int(k % khw);
        kh = r / g.KW;
        kw = r % g.KW;
      }
      for (int j = 0; j < 4; ++j) {
        float v = 0.f;
        if (kv && nv[j]) {
          int ih = ihb[j] + kh * g.dH, iw = iwb[j] + kw * g.dW;
          if (ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW)
            v = ld_f(&x[((nb[j] * g.IC + ic) * g.IH + ih) * (long long)g.IW + iw]);
        }
        Bs[b_k][b_n + j] = v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
      for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i) {
    long long m = m0 + ty * 4 + i;
    if (m >= M) continue;
    float bv = g.has_bias ? ld_f(&bias[m]) : 0.f;
    for (int j = 0; j < 4; ++j) {
      long long n = n0 + tx * 4 + j;
      if (n >= N) continue;
      long long b = n / ohw, sp = n % ohw;
      float v = apply_act(acc[i][j] + bv, g.act, g.lo, g.hi);
      out[(b * g.OC + m) * ohw + sp] = to_t<T>(v);
    }
  }
}

// ---------------------------------------------------------------------------
// direct grouped conv: one thread per output element (conv2d.wgsl.ts).
// ---------------------------------------------------------------------------
template <class T>
__global__ void direct_conv(ConvGeom g, const T *__restrict__ x, const T *__restrict__ w,
                            const T *__restrict__ bias, T *__restrict__ out, long long total) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int ow = int(i % g.OW);
  long long t = i / g.OW;
  int oh = int(t % g.OH);
  t /= g.OH;
  int oc = int(t % g.OC);
  long long b = t / g.OC;
  int icpg = g.IC / g.groups, ocpg = g.OC / g.groups;
  int grp = oc / ocpg;
  float acc = g.has_bias ? ld_f(&bias[oc]) : 0.f;
  for (int c = 0; c < icpg; ++c) {
    int ic = grp * icpg + c;
    for (int kh = 0; kh < g.KH; ++kh) {
      int ih = oh * g.sH - g.pH + kh * g.dH;
      if (ih < 0 || ih >= g.IH) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        int iw = ow * g.sW - g.pW + kw * g.dW;
        if (iw < 0 || iw >= g.IW) continue;
        acc = fmaf(ld_f(&x[((b * g.IC + ic) * g.IH + ih) * (long long)g.IW + iw]),
                   ld_f(&w[((long long)(oc * icpg + c) * g.KH + kh) * g.KW + kw]), acc);
      }
    }
  }
  out[i] = to_t<T>(apply_act(acc, g.act, g.lo, g.hi));
}

// ---------------------------------------------------------------------------
// transposed conv gather (conv-transpose2d.wgsl.ts): weight [IC, OC/g, KH, KW]
// ---------------------------------------------------------------------------
template <class T>
__global__ void conv_transpose_gather(ConvGeom g, const T *__restrict__ x, const T *__restrict__ w,
                                      const T *__restrict__ bias, T *__restrict__ out,
                                      long long total) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  int ow = int(i % g.OW);
  long long t = i / g.OW;
  int oh = int(t % g.OH);
  t /= g.OH;
  int oc = int(t % g.OC);
  long long b = t / g.OC;
  int icpg = g.IC / g.groups, ocpg = g.OC / g.groups;
  int grp = oc / ocpg, ocl = oc % ocpg;
  float acc = g.has_bias ? ld_f(&bias[oc]) : 0.f;
  for (int c = 0; c < icpg; ++c) {
    int ic = grp * icpg + c;
    for (int kh = 0; kh < g.KH; ++kh) {
      int th = oh + g.pH - kh * g.dH;
      if (th < 0 || th % g.sH) continue;
      int ih = th / g.sH;
      if (ih >= g.IH) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        int tw = ow + g.pW - kw * g.dW;
        if (tw < 0 || tw % g.sW) continue;
        int iw = tw / g.sW;
        if (iw >= g.IW) continue;
        acc = fmaf(ld_f(&x[((b * g.IC + ic) * g.IH + ih) * (long long)g.IW + iw]),
                   ld_f(&w[((long long)(ic * ocpg + ocl) * g.KH + kh) * g.KW + kw]), acc);
      }
    }
  }
  out[i] = to_t<T>(apply_act(acc, g.act, g.lo, g.hi));
}

// ---------------------------------------------------------------------------
// depthwise: groups == IC == OC, one input channel per output channel.
// The reference's conv2d-depthwise-f16.wgsl.ts reads every tap straight
// from global memory with 2-element strides; here one CTA owns a band of
// TH output rows of one (b, c) plane, stages the input rows it needs (with
// zero padding) in shared memory using 16-byte loads when the rows are
// 16-byte aligned, and each thread produces 8 consecutive outputs of a row
// so the stores are 16-byte vectors. Accumulation is fp32 starting from
// the bias like the reference (acc = bias; acc += x*w), the activation is
// applied in fp32, one rounding at the store.
// Shared tile: (TH*sH + (KH-1)*dH) rows x TWs columns (input width + pads).
// ---------------------------------------------------------------------------
constexpr int DW_THREADS = 256;
constexpr int DW_MAX_TAPS = 64;

template <class T>
__global__ void __launch_bounds__(DW_THREADS)
    depthwise_conv(ConvGeom g, int TH, int TWs, int P, long long planes, const T *__restrict__ x,
                   const T *__restrict__ w, const T *__restrict__ bias, T *__restrict__ out,
                   int vec_in, int vec_out) {
  // P planes per CTA (small planes: one band each), or one plane's band of
  // TH output rows (P = 1)
  extern __shared__ __align__(16) unsigned char dw_smem[];
  float *wsm = reinterpret_cast<float *>(dw_smem);  // [P][DW_MAX_TAPS] weights
  T *tile = reinterpret_cast<T *>(dw_smem + size_t(P) * DW_MAX_TAPS * sizeof(float));
  const long long plane0 = (long long)blockIdx.x * P;
  const int np = int(min((long long)P, planes - plane0));
  const int oh0 = blockIdx.y * TH;
  const int taps = g.KH * g.KW;
  for (int i = threadIdx.x; i < np * taps; i += blockDim.x) {
    const int pp = i / taps, t = i - pp * taps;
    const int c = int((plane0 + pp) % g.OC);
    wsm[pp * DW_MAX_TAPS + t] = ld_f(&w[(long long)c * taps + t]);
  }
  const int rows = (TH - 1) * g.sH + (g.KH - 1) * g.dH + 1;
  const int ih0 = oh0 * g.sH - g.pH;
  const size_t ptile = size_t(rows) * TWs;
  // stage rows [ih0, ih0+rows) x cols [-pW, -pW+TWs) of each plane; column
  // j of a tile is input column j - pW.
  for (int pp = 0; pp < np; ++pp) {
    const T *xp = x + (plane0 + pp) * (long long)g.IH * g.IW;
    T *tl = tile + pp * ptile;
    if (vec_in) {
      // interior: 16-byte vectors of 8 (f16) / 4 (f32) elements
      constexpr int V = 16 / sizeof(T);
      const int nvec = g.IW / V;
      for (int idx = threadIdx.x; idx < rows * nvec; idx += blockDim.x) {
        int r = idx / nvec, v = idx % nvec;
        int ih = ih0 + r;
        T *dst = tl + (long long)r * TWs + g.pW + v * V;
        if (ih >= 0 && ih < g.IH) {
          uint4 val = *reinterpret_cast<const uint4 *>(xp + (long long)ih * g.IW + v * V);
          const T *vv = reinterpret_cast<const T *>(&val);
#pragma unroll
          for (int e = 0; e < V; ++e) dst[e] = vv[e];
        } else {
#pragma unroll
          for (int e = 0; e < V; ++e) dst[e] = to_t<T>(0.f);
        }
      }
      // left/right padding columns
      const int padc = TWs - g.IW;
      for (int idx = threadIdx.x; idx < rows * padc; idx += blockDim.x) {
        int r = idx / padc, j = idx % padc;
        int col = j < g.pW ? j : g.IW + j;
        tl[(long long)r * TWs + col] = to_t<T>(0.f);
      }
    } else {
      for (int idx = threadIdx.x; idx < rows * TWs; idx += blockDim.x) {
        int r = idx / TWs, j = idx % TWs;
        int ih = ih0 + r, iw = j - g.pW;
        T v = to_t<T>(0.f);
        if (ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW) v = xp[(long long)ih * g.IW + iw];
        tl[(long long)r * TWs + j] = v;
      }
    }
  }
  __syncthreads();
  const int ohn = min(TH, g.OH - oh0);
  const int ngrp = (g.OW + 7) / 8;
  const int per_plane = ohn * ngrp;
  for (int idx = threadIdx.x; idx < np * per_plane; idx += blockDim.x) {
    const int pp = idx / per_plane, rq = idx - pp * per_plane;
    const int r = rq / ngrp, q = rq - r * ngrp;
    const int c = int((plane0 + pp) % g.OC);
    const float bv = g.has_bias ? ld_f(&bias[c]) : 0.f;
    const float *wp = wsm + pp * DW_MAX_TAPS;
    const T *tl = tile + pp * ptile;
    T *op = out + (plane0 + pp) * (long long)g.OH * g.OW;
    int ow0 = q * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = bv;
    for (int kh = 0; kh < g.KH; ++kh) {
      const T *trow = tl + (long long)(r * g.sH + kh * g.dH) * TWs;
      for (int kw = 0; kw < g.KW; ++kw) {
        float wv = wp[kh * g.KW + kw];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          int col = (ow0 + e) * g.sW + kw * g.dW;  // tile column (input col + pW)
          if (col < TWs) acc[e] = fmaf(ld_f(&trow[col]), wv, acc[e]);
        }
      }
    }
    T *orow = op + (long long)(oh0 + r) * g.OW;
    if (vec_out && ow0 + 8 <= g.OW) {
      alignas(16) T res[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) res[e] = to_t<T>(apply_act(acc[e], g.act, g.lo, g.hi));
      if (sizeof(T) == 2) {
        *reinterpret_cast<uint4 *>(orow + ow0) = *reinterpret_cast<const uint4 *>(res);
      } else {
        reinterpret_cast<uint4 *>(orow + ow0)[0] = reinterpret_cast<const uint4 *>(res)[0];
        reinterpret_cast<uint4 *>(orow + ow0)[1] = reinterpret_cast<const uint4 *>(res)[1];
      }
    } else {
      for (int e = 0; e < 8 && ow0 + e < g.OW; ++e)
        orow[ow0 + e] = to_t<T>(apply_act(acc[e], g.act, g.lo, g.hi));
    }
  }
}

// ---------------------------------------------------------------------------
// 1x1 conv with a single output channel: out[b,0,p] = sum_c x[b,c,p]*w[c]
// with fp32 accumulation (conv-with-clamp-1x1-single-channel-f16.wgsl.ts:44-58).
// ---------------------------------------------------------------------------
template <class T>
__global__ void pointwise_single(ConvGeom g, const T *__restrict__ x, const T *__restrict__ w,
                                 const T *__restrict__ bias, T *__restrict__ out) {
  long long hw = (long long)g.OH * g.OW;
  long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  int b = blockIdx.y;
  if (p >= hw) return;
  const T *xb = x + (long long)b * g.IC * hw + p;
  float acc = 0.f;
  for (int c = 0; c < g.IC; ++c) acc = fmaf(ld_f(&xb[c * hw]), ld_f(&w[c]), acc);
  if (g.has_bias) acc += ld_f(&bias[0]);
  out[(long long)b * hw + p] = to_t<T>(apply_act(acc, g.act, g.lo, g.hi));
}

// ------------------------------------------- stride-1 depthwise, K x K
// One CTA stages P whole planes, or a band of TH output rows of one plane,
// in shared memory: staged row r of a plane is input row oh0 - pH + r and
// staged column DW_PADL + iw holds input column iw (the interior starts on
// a 16-byte boundary, the zero halo sits on both sides). Each thread owns
// DW_R output rows x 8 output columns: it walks the DW_R + K - 1 input rows
// once, holding the 8 + K - 1 values of the current row in registers and
// adding them into every output row whose filter touches that row, then
// writes each output row's 8 values with one 16-byte store.
constexpr int DW_PADL = 8;  // staged columns left of the interior (>= pW)
constexpr int DW_R = 4;     // output rows per thread
constexpr int DW_SMEM = 46 * 1024;

struct DwTile {
  int P, TH, bands, rows, TWs, n_cg, n_rg;
  long long planes;
};

// Stages np planes' rows [ih0, ih0 + rows) into the tiles with 16-byte
// vectors: per staged row one zero vector left of the interior, IW / V
// interior vectors, one zero vector right of it (rows outside the image are
// zero). Each thread issues DW_STAGE_U loads before storing any of them, so
// several loads are in flight per thread.
constexpr int DW_STAGE_U = 4;
template <class T>
__device__ __forceinline__ void dw_stage_vec(const ConvGeom &g, const DwTile &d,
                                             const T *__restrict__ x, T *tile, long long plane0,
                                             int np, int ih0, size_t plane_tile) {
  constexpr int V = 16 / sizeof(T);
  const int vrow = g.IW / V + 2;
  const int total = np * d.rows * vrow;
  for (int base = threadIdx.x; base < total; base += blockDim.x * DW_STAGE_U) {
    uint4 val[DW_STAGE_U];
    T *dst[DW_STAGE_U];
#pragma unroll
    for (int u = 0; u < DW_STAGE_U; ++u) {
      const int i = base + u * blockDim.x;
      val[u] = make_uint4(0u, 0u, 0u, 0u);
      dst[u] = nullptr;
      if (i < total) {
        const int v = i % vrow;
        const int rr = i / vrow;
        const int r = rr % d.rows, p = rr / d.rows;
        const int ih = ih0 + r;
        const int col = v == 0 ? DW_PADL - V : DW_PADL + (v - 1) * V;
        dst[u] = tile + p * plane_tile + size_t(r) * d.TWs + col;
        if (v > 0 && v < vrow - 1 && ih >= 0 && ih < g.IH)
          val[u] = *reinterpret_cast<const uint4 *>(
              x + ((plane0 + p) * g.IH + ih) * (long long)g.IW + (v - 1) * V);
      }
    }
#pragma unroll
    for (int u = 0; u < DW_STAGE_U; ++u)
      if (dst[u]) *reinterpret_cast<uint4 *>(dst[u]) = val[u];
  }
}

// Rows whose width is a whole number of 8-byte units (IW * sizeof(T) % 8 ==
// 0, e.g. 20-wide fp16 planes): every 8-byte unit of every staged row is
// written once, the interior from global memory (8-byte aligned loads),
// the halo columns and the rows outside the image as zeros (DW_PADL is a
// whole number of units, so a unit is entirely inside or outside).
template <class T>
__device__ __forceinline__ void dw_stage_vec8b(const ConvGeom &g, const DwTile &d,
                                               const T *__restrict__ x, T *tile, long long plane0,
                                               int np, int ih0, size_t plane_tile) {
  constexpr int U = 8 / sizeof(T);  // elements per unit
  const int urow = d.TWs / U;
  const int total = np * d.rows * urow;
  for (int base = threadIdx.x; base < total; base += blockDim.x * DW_STAGE_U) {
    uint2 val[DW_STAGE_U];
    int dst[DW_STAGE_U];
#pragma unroll
    for (int u = 0; u < DW_STAGE_U; ++u) {
      const int i = base + u * blockDim.x;
      val[u] = make_uint2(0u, 0u);
      dst[u] = -1;
      if (i < total) {
        const int v = i % urow;
        const int rr = i / urow;
        const int r = rr % d.rows, p = rr / d.rows;
        const int ih = ih0 + r, iw = v * U - DW_PADL;
        dst[u] = int(p * plane_tile + size_t(r) * d.TWs + v * U);
        if (ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW)
          val[u] = *reinterpret_cast<const uint2 *>(x + ((plane0 + p) * g.IH + ih) * (long long)g.IW + iw);
      }
    }
#pragma unroll
    for (int u = 0; u < DW_STAGE_U; ++u)
      if (dst[u] >= 0) *reinterpret_cast<uint2 *>(tile + dst[u]) = val[u];
  }
}

// Staging for rows that are not whole 16-byte vectors: a plane's row band
// is one contiguous run of memory, so it is read as aligned 16-byte vectors
// (the plane size is a multiple of the vector width) and each element is
// scattered to its staged row and column; the tiles are zeroed first.
template <class T>
__device__ __forceinline__ void dw_stage_flat(const ConvGeom &g, const DwTile &d,
                                              const T *__restrict__ x, T *tile, long long plane0,
                                              int np, int ih0, size_t plane_tile) {
  constexpr int V = 16 / sizeof(T);
  const int zero_vecs = int(size_t(np) * plane_tile / V);
  for (int i = threadIdx.x; i < zero_vecs; i += blockDim.x)
    reinterpret_cast<uint4 *>(tile)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  const int r_lo = max(ih0, 0), r_hi = min(ih0 + d.rows, g.IH);
  if (r_hi <= r_lo) return;
  const int s = r_lo * g.IW, e = r_hi * g.IW;  // plane-local element range
  const int v0 = s / V, nvec = (e + V - 1) / V - v0;
  const int total = np * nvec;
  for (int base = threadIdx.x; base < total; base += blockDim.x * DW_STAGE_U) {
    uint4 val[DW_STAGE_U];
#pragma unroll
    for (int u = 0; u < DW_STAGE_U; ++u) {
      const int i = base + u * blockDim.x;
      if (i < total) {
        const int p = i / nvec, v = v0 + i % nvec;
        val[u] = *reinterpret_cast<const uint4 *>(x + (plane0 + p) * g.IH * (long long)g.IW +
                                                  (long long)v * V);
      }
    }
#pragma unroll
    for (int u = 0; u < DW_STAGE_U; ++u) {
      const int i = base + u * blockDim.x;
      if (i >= total) continue;
      const int p = i / nvec, v = v0 + i % nvec;
      const T *vals = reinterpret_cast<const T *>(&val[u]);
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const int idx = v * V + k;
        if (idx < s || idx >= e) continue;
        const int row = idx / g.IW, col = idx - row * g.IW;
        tile[p * plane_tile + size_t(row - ih0) * d.TWs + DW_PADL + col] = vals[k];
      }
    }
  }
}

template <class T, int K>
__global__ void __launch_bounds__(256)
    depthwise_tiled(ConvGeom g, DwTile d, const T *__restrict__ x, const T *__restrict__ w,
                    const T *__restrict__ bias, T *__restrict__ out, int vec_in, int vec_out) {
  extern __shared__ __align__(16) unsigned char dw_smem[];
  T *tile = reinterpret_cast<T *>(dw_smem);
  const long long cta = blockIdx.x;
  const long long plane0 = (cta / d.bands) * d.P;
  const int oh0 = int(cta % d.bands) * d.TH;
  const int np = int(min((long long)d.P, d.planes - plane0));
  const int ih0 = oh0 - g.pH;
  const size_t plane_tile = size_t(d.rows) * d.TWs;
  // ---- stage: interior (vectorised when rows are whole 16-byte vectors),
  // zero halo columns on both sides, zero rows outside the image
  constexpr int V = 16 / sizeof(T);
  if (vec_in == 1) {
    dw_stage_vec<T>(g, d, x, tile, plane0, np, ih0, plane_tile);
  } else if (vec_in == 3) {
    dw_stage_vec8b<T>(g, d, x, tile, plane0, np, ih0, plane_tile);
  } else if (vec_in == 2) {
    dw_stage_flat<T>(g, d, x, tile, plane0, np, ih0, plane_tile);
  } else {
    const int total = np * d.rows * d.TWs;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int col = i % d.TWs;
      const int rr = i / d.TWs;
      const int r = rr % d.rows, p = rr / d.rows;
      const int ih = ih0 + r, iw = col - DW_PADL;
      T v = to_t<T>(0.f);
      if (ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW)
        v = x[((plane0 + p) * g.IH + ih) * (long long)g.IW + iw];
      tile[p * plane_tile + size_t(r) * d.TWs + col] = v;
    }
  }
  __syncthreads();
  // ---- compute
  const int oh_end = min(oh0 + d.TH, g.OH);
  const int items = np * d.n_rg * d.n_cg;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int cg = it % d.n_cg;
    const int t = it / d.n_cg;
    const int rg = t % d.n_rg, p = t / d.n_rg;
    const long long plane = plane0 + p;
    const int c = int(plane % g.OC);
    float wr[K * K];
#pragma unroll
    for (int i = 0; i < K * K; ++i) wr[i] = ld_f(&w[size_t(c) * K * K + i]);
    const float bv = g.has_bias ? ld_f(&bias[c]) : 0.f;
    const int r0 = rg * DW_R, ow0 = cg * 8;
    float acc[DW_R][8];
#pragma unroll
    for (int r = 0; r < DW_R; ++r)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[r][e] = bv;
    const T *tb = tile + p * plane_tile + (DW_PADL - g.pW + ow0);
#pragma unroll
    for (int ir = 0; ir < DW_R + K - 1; ++ir) {
      float v[8 + K - 1];
      const T *src = tb + size_t(r0 + ir) * d.TWs;
#pragma unroll
      for (int j = 0; j < 8 + K - 1; ++j) v[j] = ld_f(&src[j]);
#pragma unroll
      for (int r = 0; r < DW_R; ++r) {
        const int kh = ir - r;
        if (kh < 0 || kh >= K) continue;
#pragma unroll
        for (int kw = 0; kw < K; ++kw)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[r][e] = fmaf(v[e + kw], wr[kh * K + kw], acc[r][e]);
      }
    }
    T *op = out + plane * g.OH * (long long)g.OW;
#pragma unroll
    for (int r = 0; r < DW_R; ++r) {
      const int oh = oh0 + r0 + r;
      if (oh >= oh_end) break;
      T *orow = op + (long long)oh * g.OW;
      if (vec_out && ow0 + 8 <= g.OW) {
        alignas(16) T res[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) res[e] = to_t<T>(apply_act(acc[r][e], g.act, g.lo, g.hi));
#pragma unroll
        for (int q = 0; q < 8 / V; ++q)
          reinterpret_cast<uint4 *>(orow + ow0)[q] = reinterpret_cast<const uint4 *>(res)[q];
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (ow0 + e < g.OW) orow[ow0 + e] = to_t<T>(apply_act(acc[r][e], g.act, g.lo, g.hi));
      }
    }
  }
}

// fp16 form of depthwise_tiled for "same" padding (pW = (K-1)/2): packed
// half2 arithmetic, accumulating in f16 from the bias like the reference's
// f16 depthwise kernel (src/shaders/convolution/conv2d-depthwise-f16.wgsl.ts:
// f16 accumulator initialised with the bias). Each staged input row is read
// as three aligned 16-byte vectors (staged columns ow0-8 .. ow0+15 around
// the thread's 8 outputs); the half2 pairs a filter tap needs are taken
// from those words directly (even offset) or with one byte permute (odd).
// The CTA's weights sit in shared memory behind the tiles as (w, w) pairs.
template <int K>
__global__ void __launch_bounds__(256)
    depthwise_tiled_h2(ConvGeom g, DwTile d, const __half *__restrict__ x,
                       const __half *__restrict__ w, const __half *__restrict__ bias,
                       __half *__restrict__ out, int vec_in, int vec_out) {
  constexpr int PW = (K - 1) / 2;
  extern __shared__ __align__(16) unsigned char dw_smem[];
  __half *tile = reinterpret_cast<__half *>(dw_smem);
  const long long cta = blockIdx.x;
  const long long plane0 = (cta / d.bands) * d.P;
  const int oh0 = int(cta % d.bands) * d.TH;
  const int np = int(min((long long)d.P, d.planes - plane0));
  const int ih0 = oh0 - g.pH;
  const size_t plane_tile = size_t(d.rows) * d.TWs;
  __half2 *wsm = reinterpret_cast<__half2 *>(tile + size_t(d.P) * plane_tile);
  // vec_out == 2: the CTA's outputs are staged after the weights (16-byte
  // aligned) and stored contiguously at the end
  __half *ostg = reinterpret_cast<__half *>(
      (reinterpret_cast<uintptr_t>(wsm + size_t(d.P) * (K * K + 1)) + 15) & ~uintptr_t(15));
  for (int i = threadIdx.x; i < np * (K * K + 1); i += blockDim.x) {
    const int p = i / (K * K + 1), t = i % (K * K + 1);
    const int c = int((plane0 + p) % g.OC);
    const __half v = t < K * K ? w[size_t(c) * K * K + t]
                               : (g.has_bias ? bias[c] : __float2half_rn(0.f));
    wsm[i] = __halves2half2(v, v);
  }
  if (vec_in == 1) {
    dw_stage_vec<__half>(g, d, x, tile, plane0, np, ih0, plane_tile);
  } else if (vec_in == 3) {
    dw_stage_vec8b<__half>(g, d, x, tile, plane0, np, ih0, plane_tile);
  } else if (vec_in == 2) {
    dw_stage_flat<__half>(g, d, x, tile, plane0, np, ih0, plane_tile);
  } else {
    const int total = np * d.rows * d.TWs;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
      const int col = i % d.TWs;
      const int rr = i / d.TWs;
      const int r = rr % d.rows, p = rr / d.rows;
      const int ih = ih0 + r, iw = col - DW_PADL;
      __half v = __float2half_rn(0.f);
      if (ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW)
        v = x[((plane0 + p) * g.IH + ih) * (long long)g.IW + iw];
      tile[p * plane_tile + size_t(r) * d.TWs + col] = v;
    }
  }
  __syncthreads();
  const int oh_end = min(oh0 + d.TH, g.OH);
  const int items = np * d.n_rg * d.n_cg;
  for (int it = threadIdx.x; it < items; it += blockDim.x) {
    const int cg = it % d.n_cg;
    const int t = it / d.n_cg;
    const int rg = t % d.n_rg, p = t / d.n_rg;
    const long long plane = plane0 + p;
    const __half2 *wp = wsm + p * (K * K + 1);
    const int r0 = rg * DW_R, ow0 = cg * 8;
    __half2 acc[DW_R][4];
#pragma unroll
    for (int r = 0; r < DW_R; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[r][j] = wp[K * K];
    // staged columns ow0 - 8 + 8 .. : window start (16-byte aligned)
    const __half *wbase = tile + p * plane_tile + (DW_PADL - 8 + ow0);
#pragma unroll
    for (int ir = 0; ir < DW_R + K - 1; ++ir) {
      const uint4 *src = reinterpret_cast<const uint4 *>(wbase + size_t(r0 + ir) * d.TWs);
      const uint4 a = src[0], b = src[1], c = src[2];
      const uint32_t wd[12] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w};
#pragma unroll
      for (int r = 0; r < DW_R; ++r) {
        const int kh = ir - r;
        if (kh < 0 || kh >= K) continue;
#pragma unroll
        for (int kw = 0; kw < K; ++kw) {
          const __half2 wv = wp[kh * K + kw];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // outputs 2j, 2j+1 read window halves h, h+1 with h = 8 - PW + kw + 2j
            const int h = 8 - PW + kw + 2 * j;
            const uint32_t pr = (h & 1) ? __byte_perm(wd[h >> 1], wd[(h >> 1) + 1], 0x5432)
                                        : wd[h >> 1];
            acc[r][j] = __hfma2(*reinterpret_cast<const __half2 *>(&pr), wv, acc[r][j]);
          }
        }
      }
    }
    __half *op = out + plane * g.OH * (long long)g.OW;
#pragma unroll
    for (int r = 0; r < DW_R; ++r) {
      const int oh = oh0 + r0 + r;
      if (oh >= oh_end) break;
      __half *orow = op + (long long)oh * g.OW;
      uint32_t res[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __half2 v = acc[r][j];
        if (g.act == WGX_ACT_SILU) {
          // v * sigmoid(v) = h + h * tanh(h), h = v / 2
          const __half2 h = __hmul2(v, __float2half2_rn(0.5f));
          const uint32_t hu = *reinterpret_cast<const uint32_t *>(&h);
          uint32_t tu;
          asm("tanh.approx.f16x2 %0, %1;" : "=r"(tu) : "r"(hu));
          v = __hfma2(h, *reinterpret_cast<const __half2 *>(&tu), h);
        } else if (g.act == WGX_ACT_CLAMP) {
          const float2 f = __half22float2(v);
          v = __floats2half2_rn(fminf(fmaxf(f.x, g.lo), g.hi), fminf(fmaxf(f.y, g.lo), g.hi));
        }
        res[j] = *reinterpret_cast<const uint32_t *>(&v);
      }
      if (vec_out == 1 && ow0 + 8 <= g.OW) {
        *reinterpret_cast<uint4 *>(orow + ow0) = make_uint4(res[0], res[1], res[2], res[3]);
      } else if (vec_out == 2) {
        // into the CTA's output image (stored below, coalesced)
        __half *srow = ostg + (size_t(p) * g.OH + oh) * g.OW;
        const __half *hv = reinterpret_cast<const __half *>(res);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (ow0 + e < g.OW) srow[ow0 + e] = hv[e];
      } else {
        const __half *hv = reinterpret_cast<const __half *>(res);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (ow0 + e < g.OW) orow[ow0 + e] = hv[e];
      }
    }
  }
  if (vec_out == 2) {
    // whole planes (one band): the CTA's np planes are one contiguous run of
    // the output; copy the staged image with 16-byte stores
    __syncthreads();
    const int n16 = int(size_t(np) * g.OH * g.OW / 8);
    uint4 *dst = reinterpret_cast<uint4 *>(out + plane0 * g.OH * (long long)g.OW);
    const uint4 *src = reinterpret_cast<const uint4 *>(ostg);
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
  }
}

// ------------------------------- fp16 depthwise, sliding window per thread
// Stride 1, dilation 1, square K in {3, 5, 7} with "same" padding
// (pH = pW = (K-1)/2), rows of whole 16-byte vectors (IW % 8 == 0), 16-byte
// aligned tensors. Same arithmetic as depthwise_tiled_h2 (and the
// reference's conv2d-depthwise-f16.wgsl.ts: f16 accumulator started at the
// bias, taps added in (kh, kw) order), so the results are identical; what
// changes is the work per instruction, which the half2 FMA pipe bounds:
//  * one CTA stages P whole planes (or a band of TH output rows of one
//    plane) with cp.async 16-byte copies, zero-filled outside the image
//    (no per-element index arithmetic; the loop steps are precomputed);
//  * each thread owns 8 output columns x RB output rows and slides down
//    RB + K - 1 staged input rows: per input row three shared loads (the 8
//    + K - 1 columns it needs), the odd-offset column pairs by one byte
//    permute each, and K*K*4 HFMA2 into the (at most K) output rows the
//    row feeds, with the K*K weight pairs in registers; an output row is
//    stored (16 bytes) as soon as its last input row is added.
// Staged column 8 + iw holds input column iw; columns 0-7 and those past
// the image are zero (the halo).
struct DwSlide {
  int P, TH, bands, rows, TWs, n_cg, n_rb, threads;
  long long planes;
  // extents of x and out in bytes and the device error word (bounds-checking
  // build)
  uint64_t in_bytes, out_bytes;
  uint32_t *err;
};
constexpr int DWS_RB = 8;  // output rows per thread

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = valid ? 16 : 0;  // 0: no bytes read, 16 zero bytes written
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}

template <int K>
__global__ void __launch_bounds__(256, 2)
    depthwise_slide_h2(ConvGeom g, DwSlide d, const __half *__restrict__ x,
                       const __half *__restrict__ w, const __half *__restrict__ bias,
                       __half *__restrict__ out) {
  constexpr int PW = (K - 1) / 2;
  constexpr int RB = DWS_RB;
  constexpr int KK1 = K * K + 1;  // weights + bias of one plane
  extern __shared__ __align__(16) unsigned char dw_smem[];
  __half *tile = reinterpret_cast<__half *>(dw_smem);
  const int tid = threadIdx.x;
  const long long plane0 = (long long)(blockIdx.x / d.bands) * d.P;
  const int oh0 = int(blockIdx.x % d.bands) * d.TH;
  const int np = int(min((long long)d.P, d.planes - plane0));
  const int plane_tile = d.rows * d.TWs;
  __half2 *wsm = reinterpret_cast<__half2 *>(tile + size_t(d.P) * plane_tile);
  {
    // staging: thread -> (vector column v, first row r0), rows step rstep
    const int vrow = d.TWs / 8;
    const int v = tid % vrow, r0 = tid / vrow, rstep = blockDim.x / vrow;
    const int iw0 = v * 8 - 8;
    const bool col_in = iw0 >= 0 && iw0 < g.IW;
    const size_t hw = size_t(g.IH) * g.IW;
    if (r0 < rstep) {
      for (int p = 0; p < np; ++p) {
        const __half *src = x + size_t(plane0 + p) * hw;
        __half *dst = tile + p * plane_tile + v * 8;
        for (int r = r0; r < d.rows; r += rstep) {
          const int ih = oh0 - PW + r;
          const bool ok = col_in && ih >= 0 && ih < g.IH;
          const __half *gsrc = ok ? src + size_t(ih) * g.IW + iw0 : src;
          cp_async16(dst + r * d.TWs, gsrc,
                     ok && WGX_IN_BOUNDS(gsrc, 16, x, d.in_bytes, d.err));
        }
      }
    }
  }
  for (int i = tid; i < np * KK1; i += blockDim.x) {
    const int p = i / KK1, t = i - p * KK1;
    const int c = int((plane0 + p) % g.OC);
    const __half v = t < K * K ? w[size_t(c) * K * K + t]
                               : (g.has_bias ? bias[c] : __float2half_rn(0.f));
    wsm[i] = __halves2half2(v, v);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  // compute: thread -> (plane p, row block rb, column group cg)
  const int cg = tid % d.n_cg;
  const int rest = tid / d.n_cg;
  const int rb = rest % d.n_rb, p = rest / d.n_rb;
  if (p >= np) return;
  const int ow0 = cg * 8, r0 = rb * RB;  // r0: first output row of the block in the band
  const int oh_end = min(oh0 + d.TH, g.OH);
  __half2 wv[K * K];
  const __half2 *wp = wsm + p * KK1;
#pragma unroll
  for (int t = 0; t < K * K; ++t) wv[t] = wp[t];
  const __half2 b2 = wp[K * K];
  // staged columns ow0 .. ow0 + 23 (input columns ow0 - 8 .. ow0 + 15)
  const __half *rowp = tile + p * plane_tile + r0 * d.TWs + ow0;
  __half *op = out + size_t(plane0 + p) * g.OH * g.OW + ow0;
  __half2 acc[RB][4];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[r][j] = b2;
#pragma unroll
  for (int ir = 0; ir < RB + K - 1; ++ir) {
    // window words wd[k] = staged halves 2k, 2k + 1 of the row from column
    // ow0; only those the filter reaches are loaded
    const __half *src = rowp + ir * d.TWs;
    uint32_t wd[12];
    {
      const uint4 bq = *reinterpret_cast<const uint4 *>(src + 8);
      wd[4] = bq.x, wd[5] = bq.y, wd[6] = bq.z, wd[7] = bq.w;
      if constexpr (PW <= 2) {
        wd[3] = *reinterpret_cast<const uint32_t *>(src + 6);
        wd[8] = *reinterpret_cast<const uint32_t *>(src + 16);
      } else {
        const uint2 a = *reinterpret_cast<const uint2 *>(src + 4);
        const uint2 c = *reinterpret_cast<const uint2 *>(src + 16);
        wd[2] = a.x, wd[3] = a.y, wd[8] = c.x, wd[9] = c.y;
      }
    }
    // pair i = input columns ow0 - PW + i, +1 (odd offsets: one permute);
    // (output pair j, tap kw) reads pair 2j + kw <= K + 5
    uint32_t pr[K + 6];
#pragma unroll
    for (int i = 0; i < K + 6; ++i) {
      const int h = 8 - PW + i;
      pr[i] = (h & 1) ? __byte_perm(wd[h >> 1], wd[(h >> 1) + 1], 0x5432) : wd[h >> 1];
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const int kh = ir - r;
      if (kh < 0 || kh >= K) continue;
#pragma unroll
      for (int kw = 0; kw < K; ++kw)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[r][j] = __hfma2(*reinterpret_cast<const __half2 *>(&pr[2 * j + kw]),
                              wv[kh * K + kw], acc[r][j]);
    }
    // output row ir - (K - 1) is complete
    if (ir >= K - 1) {
      const int r = ir - (K - 1);
      const int oh = oh0 + r0 + r;
      if (oh < oh_end) {
        uint32_t res[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __half2 v = acc[r][j];
          if (g.act == WGX_ACT_SILU) {
            // v * sigmoid(v) = h + h * tanh(h), h = v / 2
            const __half2 h = __hmul2(v, __float2half2_rn(0.5f));
            const uint32_t hu = *reinterpret_cast<const uint32_t *>(&h);
            uint32_t tu;
            asm("tanh.approx.f16x2 %0, %1;" : "=r"(tu) : "r"(hu));
            v = __hfma2(h, *reinterpret_cast<const __half2 *>(&tu), h);
          } else if (g.act == WGX_ACT_CLAMP) {
            const float2 f = __half22float2(v);
            v = __floats2half2_rn(fminf(fmaxf(f.x, g.lo), g.hi), fminf(fmaxf(f.y, g.lo), g.hi));
          }
          res[j] = *reinterpret_cast<const uint32_t *>(&v);
        }
        if (WGX_IN_BOUNDS(op + size_t(oh) * g.OW, 16, out, d.out_bytes, d.err))
          *reinterpret_cast<uint4 *>(op + size_t(oh) * g.OW) =
              make_uint4(res[0], res[1], res[2], res[3]);
      }
    }
  }
}

// Tiling of depthwise_slide_h2 (see there), or false when it does not apply.
static int dw_sm_count() {
  int dev = 0, n = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "SM count");
  return n > 0 ? n : 1;
}

static bool dw_slide_tiling(const wgx_conv2d_params &p, DwSlide &d, size_t &smem, int n_sm) {
  const int K = p.KH;
  if (p.dtype != WGX_FLOAT16 || p.KW != K || (K != 3 && K != 5 && K != 7)) return false;
  if (p.sH != 1 || p.sW != 1 || p.dH != 1 || p.dW != 1) return false;
  if (p.pH != (K - 1) / 2 || p.pW != (K - 1) / 2 || p.IW % 8 != 0) return false;
  if (p.OH != p.IH || p.OW != p.IW) return false;
  d.n_cg = p.OW / 8;
  // staged row: 8 zero columns, the interior, then zeros up to the last
  // column group's window end (ow0 + 24)
  d.TWs = 8 * d.n_cg + 16;
  d.planes = (long long)p.B * p.OC;
  const size_t wbytes = size_t(K * K + 1) * 4;
  // whole planes when one plane's items fit 256 threads and its tile fits
  // the shared-memory budget, else bands of TH output rows
  const int budget = 96 * 1024;
  int TH = p.OH;
  auto items = [&](int th) { return d.n_cg * ((th + DWS_RB - 1) / DWS_RB); };
  auto tbytes = [&](int th) {
    return size_t((th + DWS_RB - 1) / DWS_RB * DWS_RB + K - 1) * d.TWs * 2 + wbytes;
  };
  while (TH > DWS_RB && (items(TH) > 256 || tbytes(TH) > size_t(budget)))
    TH = (TH / 2 + DWS_RB - 1) / DWS_RB * DWS_RB;
  if (items(TH) > 256 || tbytes(TH) > size_t(budget)) return false;
  d.TH = TH;
  d.bands = (p.OH + TH - 1) / TH;
  d.n_rb = (TH + DWS_RB - 1) / DWS_RB;
  d.rows = d.n_rb * DWS_RB + K - 1;
  d.P = 1;
  if (d.bands == 1) {
    // as many planes as fill 256 threads and the budget, but no fewer than
    // two CTAs per SM when there are planes enough (small planes: 16^2 has
    // 4 items per plane)
    const long long per_sm2 = (d.planes + 2ll * n_sm - 1) / (2ll * n_sm);
    d.P = int(std::max(1ll, std::min<long long>({(long long)(256 / items(TH)),
                                                  (long long)(budget / tbytes(TH)), d.planes,
                                                  per_sm2})));
  }
  const int vrow = d.TWs / 8;
  auto threads_for = [&](int P) {
    return std::min(256, std::max((P * items(TH) + 31) / 32 * 32, (vrow + 31) / 32 * 32));
  };
  d.threads = threads_for(d.P);
  smem = size_t(d.P) * (size_t(d.rows) * d.TWs * 2 + wbytes);
  const long long ctas = (d.planes + d.P - 1) / d.P * d.bands;
  return ctas < (1ll << 31) && vrow <= d.threads && d.P * items(TH) <= d.threads;
}

// Tiling of depthwise_tiled for p (stride 1, dilation 1, square K in
// {3,5,7}, pW <= DW_PADL), or false when it does not apply.
static bool dw_tiling(const wgx_conv2d_params &p, int esize, DwTile &d) {
  const int K = p.KH;
  if (p.KW != K || (K != 3 && K != 5 && K != 7)) return false;
  if (p.sH != 1 || p.sW != 1 || p.dH != 1 || p.dW != 1) return false;
  // the zero halo on each side of a staged row is one 16-byte vector wide
  if (p.pW > 16 / esize || p.pH < 0 || p.pW < 0) return false;
  if (p.OH != p.IH + 2 * p.pH - K + 1 || p.OW != p.IW + 2 * p.pW - K + 1) return false;
  const int V = 16 / esize;
  d.n_cg = (p.OW + 7) / 8;
  // staged row: zero halo vector + interior + zero halo vector, wide enough
  // for every tap of the last column group and for the fp16 kernel's
  // 24-column read window starting at staged column 8 * cg
  const int right = std::max({p.IW + V, 8 * d.n_cg - p.pW + K - 1, 8 * d.n_cg + 8});
  d.TWs = (DW_PADL + right + 7) / 8 * 8;
  d.planes = (long long)p.B * p.OC;
  // shared memory of one plane: its tile plus (fp16 kernel) K*K + 1 weight pairs
  const size_t wbytes = esize == 2 ? size_t(K * K + 1) * 4 : 0;
  auto tile_bytes = [&](int th) {
    return size_t((th + DW_R - 1) / DW_R * DW_R + K - 1) * d.TWs * esize + wbytes;
  };
  int TH = p.OH;
  while (TH > DW_R && tile_bytes(TH) > size_t(DW_SMEM)) TH = (TH / 2 + DW_R - 1) / DW_R * DW_R;
  if (tile_bytes(TH) > size_t(DW_SMEM)) return false;
  d.TH = TH;
  d.bands = (p.OH + TH - 1) / TH;
  d.n_rg = (TH + DW_R - 1) / DW_R;
  d.rows = d.n_rg * DW_R + K - 1;
  d.P = 1;
  if (d.bands == 1) {
    // planes per CTA: of floor and ceil of 256 / (items per plane), the one
    // whose items (4 x 8 outputs each) fill the rounds of the CTA's 256
    // threads best, the larger on a tie (20 x 20 planes: 17 planes = 255
    // items in one round rather than 18 = 270 in two; 80 x 80: 2 planes =
    // 400 items in two rounds, as full as 1 plane's one)
    const int per_plane = d.n_rg * d.n_cg;
    auto fill = [&](int np) {
      const int items = np * per_plane;
      return double(items) / (double((items + 255) / 256) * 256.0);
    };
    const int lo = std::max(1, 256 / per_plane), hi = std::max(1, (256 + per_plane - 1) / per_plane);
    const int want = fill(lo) > fill(hi) + 1e-9 ? lo : hi;
    const int fit = int(size_t(DW_SMEM) / tile_bytes(TH));
    d.P = std::max(1, std::min(want, fit));
  }
  const long long ctas = (d.planes + d.P - 1) / d.P * d.bands;
  return ctas < (1ll << 31);
}

// ---------------------------------------------------------------- dispatch
static bool is_depthwise(const wgx_conv2d_params &p) {
  return p.groups == p.OC && p.IC == p.OC && p.groups > 1;
}

wgx_conv2d_plan plan_conv2d(const wgx_conv2d_params &p) {
  wgx_conv2d_plan plan{};
  if (p.dtype != WGX_FLOAT32 && p.dtype != WGX_FLOAT16) fail("conv2d: dtype must be fp32 or fp16");
  if (p.groups < 1 || p.IC % p.groups || p.OC % p.groups) fail("conv2d: bad groups");
  if (p.B <= 0 || p.IC <= 0 || p.OC <= 0 || p.OH <= 0 || p.OW <= 0 || p.KH <= 0 || p.KW <= 0)
    fail("conv2d: non-positive dimension");
  bool unit1x1 = p.KH == 1 && p.KW == 1 && p.sH == 1 && p.sW == 1 && p.pH == 0 && p.pW == 0;
  if (p.groups == 1 && p.dtype == WGX_FLOAT16 && umma_conv_supported(p)) {
    plan.variant = WGX_CONV_UMMA;
    plan.scratch_bytes = conv2d_scratch_bytes(p, true);
    plan.grid_ctas = umma_conv_grid(p);
    plan.n_launches = 2;
  } else if (p.groups == 1 && p.OC == 1 && unit1x1) {
    plan.variant = WGX_CONV_POINTWISE1;
    plan.n_launches = 1;
    plan.grid_ctas = uint64_t((int64_t(p.OH) * p.OW + 255) / 256) * p.B;
  } else if (p.groups == 1) {
    plan.variant = WGX_CONV_SIMT_GEMM;
    plan.n_launches = 1;
    plan.grid_ctas = uint64_t((int64_t(p.B) * p.OH * p.OW + 63) / 64) * ((p.OC + 63) / 64);
  } else if (is_depthwise(p) && p.KH * p.KW <= DW_MAX_TAPS) {
    plan.variant = WGX_CONV_DEPTHWISE;
    plan.n_launches = 1;
  } else {
    plan.variant = WGX_CONV_DIRECT;
    plan.n_launches = 1;
  }
  return plan;
}

bool conv2d_in_place_safe(const wgx_conv2d_params &p) {
  wgx_conv2d_plan plan;
  try {
    plan = plan_conv2d(p);
  } catch (const Error &) {
    return false;
  }
  // tensor cores: the first kernel stages the whole input before the second writes
  if (plan.variant == WGX_CONV_UMMA) return true;
  // tiled depthwise with whole planes per CTA: each CTA stages its planes in
  // shared memory before writing them, and no other CTA reads those planes
  // (either depthwise kernel may run: the sliding-window one when the
  // pointers are 16-byte aligned; both must stage whole planes)
  DwTile d{};
  DwSlide ds{};
  size_t ds_smem = 0;
  const int esize = p.dtype == WGX_FLOAT16 ? 2 : 4;
  // (the band split does not depend on the SM count)
  const bool slide_whole = !dw_slide_tiling(p, ds, ds_smem, 1) || ds.bands == 1;
  return plan.variant == WGX_CONV_DEPTHWISE && dw_tiling(p, esize, d) && d.bands == 1 &&
         slide_whole && p.OH == p.IH && p.OW == p.IW;
}

uint64_t conv2d_packed_weight_bytes(const wgx_conv2d_params &p) {
  if (plan_conv2d(p).variant != WGX_CONV_UMMA) return 0;
  return umma_conv_packed_weight_bytes(p);
}
uint64_t conv2d_input_scratch_bytes(const wgx_conv2d_params &p) {
  if (p.groups != 1 || p.dtype != WGX_FLOAT16 || !umma_conv_supported(p)) return 0;
  return umma_conv_input_bytes(p);
}
uint64_t conv2d_scratch_bytes(const wgx_conv2d_params &p, bool include_packed) {
  if (p.groups != 1 || p.dtype != WGX_FLOAT16 || !umma_conv_supported(p)) return 0;
  uint64_t b = umma_conv_input_bytes(p);
  if (include_packed) b += umma_conv_packed_weight_bytes(p);
  return b;
}
int conv2d_kernel_launches(const wgx_conv2d_params &p, bool packed_ready) {
  wgx_conv2d_plan plan = plan_conv2d(p);
  if (plan.variant == WGX_CONV_UMMA) return 2;
  return plan.n_launches;
}

void conv2d_pack_weights(const wgx_conv2d_params &p, const void *w, void *packed,
                         cudaStream_t stream) {
  umma_conv_pack_weights(p, static_cast<const __half *>(w), packed, stream);
}

template <class T>
static void launch_simt(const wgx_conv2d_params &p, int variant, const T *in, const T *w,
                        const T *bias, T *out, cudaStream_t s) {
  ConvGeom g = geom_of(p);
  DwTile dt{};
  DwSlide ds{};
  size_t ds_smem = 0;
  if (variant == WGX_CONV_SIMT_GEMM) {
    long long N = (long long)p.B * p.OH * p.OW;
    dim3 grid(unsigned((N + 63) / 64), unsigned((p.OC + 63) / 64));
    if (grid.y > 65535) fail("conv2d: too many output channels for the FFMA path");
    simt_gemm_conv<T><<<grid, 256, 0, s>>>(g, in, w, bias, out);
  } else if (variant == WGX_CONV_POINTWISE1) {
    long long hw = (long long)p.OH * p.OW;
    if (p.B > 65535) fail("conv2d: batch too large for the single-channel kernel");
    dim3 grid(unsigned((hw + 255) / 256), unsigned(p.B));
    pointwise_single<T><<<grid, 256, 0, s>>>(g, in, w, bias, out);
  } else if (variant == WGX_CONV_DEPTHWISE && sizeof(T) == 2 &&
             ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0 &&
             dw_slide_tiling(p, ds, ds_smem, dw_sm_count())) {
    const __half *hin = reinterpret_cast<const __half *>(in);
    const __half *hw = reinterpret_cast<const __half *>(w);
    const __half *hb = reinterpret_cast<const __half *>(bias);
    __half *hout = reinterpret_cast<__half *>(out);
    {
      int dev = 0;
      check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
      ds.err = device_error_word(dev);
      ds.in_bytes = uint64_t(p.B) * p.IC * p.IH * p.IW * 2;
      ds.out_bytes = uint64_t(p.B) * p.OC * p.OH * p.OW * 2;
    }
    auto fn = p.KH == 3 ? depthwise_slide_h2<3> : p.KH == 5 ? depthwise_slide_h2<5> : depthwise_slide_h2<7>;
    static std::mutex mu;
    static bool attr[3] = {};
    {
      std::lock_guard<std::mutex> lock(mu);
      if (!attr[p.KH / 2 - 1]) {
        check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024),
                   "depthwise smem attr");
        attr[p.KH / 2 - 1] = true;
      }
    }
    if (ds_smem > 100 * 1024) fail("conv2d: depthwise tile exceeds 100 KB");
    const unsigned grid = unsigned((ds.planes + ds.P - 1) / ds.P * ds.bands);
    if (p.KH == 3)
      depthwise_slide_h2<3><<<grid, ds.threads, ds_smem, s>>>(g, ds, hin, hw, hb, hout);
    else if (p.KH == 5)
      depthwise_slide_h2<5><<<grid, ds.threads, ds_smem, s>>>(g, ds, hin, hw, hb, hout);
    else
      depthwise_slide_h2<7><<<grid, ds.threads, ds_smem, s>>>(g, ds, hin, hw, hb, hout);
  } else if (variant == WGX_CONV_DEPTHWISE && dw_tiling(p, int(sizeof(T)), dt)) {
    constexpr int V = 16 / sizeof(T);
    // staging: 1 = whole-vector rows, 3 = whole 8-byte-unit rows, 2 = vector
    // reads of contiguous row bands scattered into the tile, 0 = per element
    const bool aligned = (reinterpret_cast<uintptr_t>(in) & 15) == 0;
    const int vec_in = !aligned ? 0
                       : p.IW % V == 0 ? 1
                       : (p.IW * int(sizeof(T))) % 8 == 0 && dt.TWs % (8 / int(sizeof(T))) == 0 ? 3
                       : (int64_t(p.IH) * p.IW) % V == 0 ? 2 : 0;
    const int vec_out = (p.OW % 8 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    const size_t smem = size_t(dt.P) * dt.rows * dt.TWs * sizeof(T);
    const unsigned grid = unsigned((dt.planes + dt.P - 1) / dt.P * dt.bands);
    if constexpr (sizeof(T) == 2) {
      if (p.pW == (p.KW - 1) / 2) {
        // rows that are not whole 16-byte vectors: whole planes are staged in
        // shared memory and stored contiguously (a thread's 8 outputs of one
        // row would otherwise be 2-byte stores to addresses far from its
        // neighbours'), with fewer planes per CTA if needed
        int vo = vec_out;
        DwTile dh = dt;
        const bool out16 = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
        if (!vo && dh.bands == 1 && (int64_t(p.OH) * p.OW) % 8 == 0 && out16) {
          const size_t per_plane = size_t(dh.rows) * dh.TWs * 2 + size_t(p.KH * p.KW + 1) * 4 +
                                   size_t(p.OH) * p.OW * 2;
          dh.P = std::max(1, std::min(dh.P, int(size_t(DW_SMEM) / per_plane)));
          vo = 2;
        }
        const size_t smem_h2 = size_t(dh.P) * dh.rows * dh.TWs * 2 +
                               size_t(dh.P) * (p.KH * p.KW + 1) * 4 +
                               (vo == 2 ? size_t(dh.P) * p.OH * p.OW * 2 + 16 : 0);
        const unsigned grid_h2 = unsigned((dh.planes + dh.P - 1) / dh.P * dh.bands);
        const __half *hin = reinterpret_cast<const __half *>(in);
        const __half *hw = reinterpret_cast<const __half *>(w);
        const __half *hb = reinterpret_cast<const __half *>(bias);
        __half *hout = reinterpret_cast<__half *>(out);
        if (smem_h2 > 48 * 1024) fail("conv2d: depthwise tile exceeds 48 KB");
        if (p.KH == 3)
          depthwise_tiled_h2<3><<<grid_h2, 256, smem_h2, s>>>(g, dh, hin, hw, hb, hout, vec_in, vo);
        else if (p.KH == 5)
          depthwise_tiled_h2<5><<<grid_h2, 256, smem_h2, s>>>(g, dh, hin, hw, hb, hout, vec_in, vo);
        else
          depthwise_tiled_h2<7><<<grid_h2, 256, smem_h2, s>>>(g, dh, hin, hw, hb, hout, vec_in, vo);
        check_cuda(cudaGetLastError(), "conv2d launch");
        return;
      }
    }
    if (p.KH == 3)
      depthwise_tiled<T, 3><<<grid, 256, smem, s>>>(g, dt, in, w, bias, out, vec_in, vec_out);
    else if (p.KH == 5)
      depthwise_tiled<T, 5><<<grid, 256, smem, s>>>(g, dt, in, w, bias, out, vec_in, vec_out);
    else
      depthwise_tiled<T, 7><<<grid, 256, smem, s>>>(g, dt, in, w, bias, out, vec_in, vec_out);
  } else if (variant == WGX_CONV_DEPTHWISE) {
    // rows per CTA: keep the staged tile under ~40 KB
    int TWs = p.IW + 2 * p.pW;
    int TH = 32;
    auto tile_bytes = [&](int th) {
      return (uint64_t)((th - 1) * p.sH + (p.KH - 1) * p.dH + 1) * TWs * sizeof(T);
    };
    while (TH > 1 && tile_bytes(TH) > 40 * 1024) TH /= 2;
    if (TH > p.OH) TH = p.OH;
    long long planes = (long long)p.B * p.OC;
    // small planes (one band): several per CTA, so that the CTA's 256
    // threads have work (a 16x16 -> 8x8 plane has 8 items of 8 outputs)
    int P = 1;
    if (TH >= p.OH) {
      const long long items = (long long)p.OH * ((p.OW + 7) / 8);
      const uint64_t per_plane = DW_MAX_TAPS * sizeof(float) + tile_bytes(TH);
      P = int(std::max<long long>(1, std::min<long long>({(long long)(DW_THREADS / items),
                                                          (long long)(40 * 1024 / per_plane),
                                                          planes})));
    }
    uint64_t smem = uint64_t(P) * (DW_MAX_TAPS * sizeof(float) + tile_bytes(TH)) + 16;
    if (smem > 200 * 1024) fail("conv2d: depthwise plane too wide");
    if (smem > 48 * 1024)
      check_cuda(cudaFuncSetAttribute(depthwise_conv<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(smem)),
                 "depthwise smem attr");
    constexpr int V = 16 / sizeof(T);
    int vec_in = (p.IW % V == 0) && ((reinterpret_cast<uintptr_t>(in) & 15) == 0) &&
                 (((long long)p.IH * p.IW) % V == 0) && ((p.pW * sizeof(T)) % 1 == 0);
    // the interior copy writes tile columns [pW, pW+IW): vector stores into
    // smem need no alignment (element stores are used), so only global
    // alignment matters.
    int vec_out = (p.OW % 8 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0) &&
                  (((long long)p.OH * p.OW) % 8 == 0);
    if (planes > 0x7fffffffLL) fail("conv2d: too many depthwise planes");
    if ((p.OH + TH - 1) / TH > 65535) fail("conv2d: depthwise plane too tall");
    // plane groups on x (up to 2^31-1 blocks), row bands on y
    dim3 grid(unsigned((planes + P - 1) / P), unsigned((p.OH + TH - 1) / TH));
    depthwise_conv<T><<<grid, DW_THREADS, smem, s>>>(g, TH, TWs, P, planes, in, w, bias, out,
                                                      vec_in, vec_out);
  } else {
    long long total = (long long)p.B * p.OC * p.OH * p.OW;
    direct_conv<T><<<unsigned((total + 255) / 256), 256, 0, s>>>(g, in, w, bias, out, total);
  }
  check_cuda(cudaGetLastError(), "conv2d launch");
}

void launch_conv2d(const wgx_conv2d_params &p, const void *in, const void *w, const void *packed,
                   const void *bias, void *out, void *scratch, uint64_t scratch_bytes,
                   cudaStream_t stream) {
  wgx_conv2d_plan plan = plan_conv2d(p);
  if (!p.has_bias) bias = nullptr;
  if (plan.variant == WGX_CONV_UMMA) {
    uint64_t need = conv2d_scratch_bytes(p, packed == nullptr);
    if (!scratch || scratch_bytes < need)
      fail("conv2d: scratch too small (" + std::to_string(scratch_bytes) + " < " +
           std::to_string(need) + " bytes)");
    char *sp = static_cast<char *>(scratch);
    void *xs = sp;
    if (!packed) {
      // pack the weights into the scratch behind the input re-layout
      umma_conv_run(p, static_cast<const __half *>(in), sp + umma_conv_input_bytes(p),
                    static_cast<const __half *>(w), static_cast<const __half *>(bias),
                    static_cast<__half *>(out), xs, stream);
    } else {
      umma_conv_run(p, static_cast<const __half *>(in), const_cast<void *>(packed), nullptr,
                    static_cast<const __half *>(bias), static_cast<__half *>(out), xs, stream);
    }
    return;
  }
  if (p.dtype == WGX_FLOAT16)
    launch_simt<__half>(p, plan.variant, static_cast<const __half *>(in),
                        static_cast<const __half *>(w), static_cast<const __half *>(bias),
                        static_cast<__half *>(out), stream);
  else
    launch_simt<float>(p, plan.variant, static_cast<const float *>(in),
                       static_cast<const float *>(w), static_cast<const float *>(bias),
                       static_cast<float *>(out), stream);
}

void launch_conv_transpose2d(const wgx_conv2d_params &p, int, int, const void *in, const void *w,
                             const void *bias, void *out, cudaStream_t s) {
  ConvGeom g = geom_of(p);
  if (!p.has_bias) bias = nullptr;
  long long total = (long long)p.B * p.OC * p.OH * p.OW;
  unsigned blocks = unsigned((total + 255) / 256);
  if (p.dtype == WGX_FLOAT16)
    conv_transpose_gather<__half><<<blocks, 256, 0, s>>>(
        g, static_cast<const __half *>(in), static_cast<const __half *>(w),
        static_cast<const __half *>(bias), static_cast<__half *>(out), total);
  else
    conv_transpose_gather<float><<<blocks, 256, 0, s>>>(
        g, static_cast<const float *>(in), static_cast<const float *>(w),
        static_cast<const float *>(bias), static_cast<float *>(out), total);
  check_cuda(cudaGetLastError(), "conv_transpose2d launch");
}

// ------------------------------------------------------------------- mm
// aten.mm is the 1x1 convolution W[OC=M, IC=K] x X[1, K, 1, N]: the same
// kernels serve both (mm-64x64.wgsl.ts computes the identical GEMM).
static wgx_conv2d_params mm_params(int64_t M, int64_t N, int64_t K, int dtype) {
  if (M <= 0 || N <= 0 || K <= 0) fail("aten.mm.default: non-positive dimension");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) fail("aten.mm.default: dimension too large");
  wgx_conv2d_params p{};
  p.B = 1;
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
  p.dtype = dtype;
  p.act = WGX_ACT_NONE;
  p.out_min = -INFINITY;
  p.out_max = INFINITY;
  return p;
}

uint64_t mm_scratch_bytes(int64_t M, int64_t N, int64_t K, int dtype) {
  return conv2d_scratch_bytes(mm_params(M, N, K, dtype), true);
}

// fp32 aten.mm, C[M,N] = A[M,K] B[K,N] row-major (mm-64x64.wgsl.ts's GEMM:
// fp32 FMAs, K ascending within each part). A 64x64 output tile per CTA of
// 256 threads, 4x4 outputs per thread. K advances in 32-deep steps through a
// 4-stage cp.async pipeline (A rows [64][32 + 4 pad], B rows [32][64], zero
// fill past the matrix), so three steps' loads are in flight while one
// step's FMAs run; per 4 k a thread reads its 4 A rows and 4 B rows as
// 16-byte words (8 shared loads for 64 FMAs). The K range is split over the
// S CTAs of a thread-block cluster (S = 1, 2, 4 or 8, chosen so that the grid
// covers the SMs: a 512 x 512 product has 64 tiles, S = 4 gives 256 CTAs);
// each CTA leaves its partial tile in shared memory and, after a cluster
// barrier, CTA r sums rows [r*64/S, (r+1)*64/S) of the S partials in rank
// order through distributed shared memory (deterministic) and stores them.
namespace {
constexpr int MM_T = 64, MM_BK = 32, MM_AS = MM_BK + 4, MM_NS = 4;
constexpr int MM_STAGE_FLOATS = MM_T * MM_AS + MM_BK * MM_T;
constexpr uint32_t MM_SMEM = MM_NS * MM_STAGE_FLOATS * 4;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// the shared-memory address `p` of this CTA, seen in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t dsmem_addr(const void *p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(out)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
  return out;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}
// 4 consecutive floats src[0..3] into shared memory: one 16-byte copy when
// `vec`, else four 4-byte copies. Elements i >= valid (past the matrix) are
// zero-filled and read nothing; their copies take the (aligned) matrix base
// `base` as their source address.
__device__ __forceinline__ void cp_async_f4(float *dst, const float *src, const float *base,
                                            bool vec, int valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  if (vec) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d),
                 "l"(valid >= 4 ? src : base), "r"(valid >= 4 ? 16 : 0)
                 : "memory");
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d + 4 * i),
                   "l"(i < valid ? src + i : base), "r"(i < valid ? 4 : 0)
                   : "memory");
  }
}

__global__ void __launch_bounds__(256) mm_f32_kernel(const float *__restrict__ A,
                                                     const float *__restrict__ B,
                                                     float *__restrict__ C, int M, int N, int K,
                                                     int kchunk, int avec, int bvec) {
  extern __shared__ __align__(16) float mm_smem[];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * MM_T, n0 = blockIdx.x * MM_T;
  const int S = gridDim.z;
  const int kb = blockIdx.z * kchunk, ke = min(K, kb + kchunk);
  const int nsteps = ke > kb ? (ke - kb + MM_BK - 1) / MM_BK : 0;
  // copies per stage: A rows m = tid/8 and tid/8 + 32, k quad tid%8; B rows
  // k = tid/16 and tid/16 + 16, column quad tid%16
  // (avec / bvec: 16-byte copies; K % 4 == 0 / N % 4 == 0 and 16-byte
  // aligned bases, checked on the host)
  auto issue = [&](int step) {
    float *As = mm_smem + (step % MM_NS) * MM_STAGE_FLOATS;
    float *Bs = As + MM_T * MM_AS;
    const int k0 = kb + step * MM_BK;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = (tid >> 3) + 32 * h, kq = (tid & 7) * 4;
      const int k = k0 + kq;
      const int valid = (m0 + m < M) ? max(0, min(4, ke - k)) : 0;
      cp_async_f4(As + m * MM_AS + kq, valid > 0 ? A + size_t(m0 + m) * K + k : A, A, avec != 0,
                  valid);
      const int kr = (tid >> 4) + 16 * h, nq = (tid & 15) * 4;
      const int kk = k0 + kr;
      const int bvalid = (kk < ke) ? max(0, min(4, N - (n0 + nq))) : 0;
      cp_async_f4(Bs + kr * MM_T + nq, bvalid > 0 ? B + size_t(kk) * N + n0 + nq : B, B,
                  bvec != 0, bvalid);
    }
  };
  float acc[4][4] = {};
#pragma unroll
  for (int st = 0; st < MM_NS - 1; ++st) {
    if (st < nsteps) issue(st);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int step = 0; step < nsteps; ++step) {
    // step's copies are complete once at most MM_NS - 2 newer groups remain
    asm volatile("cp.async.wait_group %0;" ::"n"(MM_NS - 2) : "memory");
    __syncthreads();
    // refill the stage consumed one step ago (every thread is past it)
    if (step + MM_NS - 1 < nsteps) issue(step + MM_NS - 1);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const float *As = mm_smem + (step % MM_NS) * MM_STAGE_FLOATS;
    const float *Bs = As + MM_T * MM_AS;
#pragma unroll
    for (int k4 = 0; k4 < MM_BK; k4 += 4) {
      float4 a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4 *>(As + (ty * 4 + i) * MM_AS + k4);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) b[kk] = *reinterpret_cast<const float4 *>(Bs + (k4 + kk) * MM_T + tx * 4);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float bv[4] = {b[kk].x, b[kk].y, b[kk].z, b[kk].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float av = kk == 0 ? a[i].x : kk == 1 ? a[i].y : kk == 2 ? a[i].z : a[i].w;
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av, bv[j], acc[i][j]);
        }
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (S == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
        if (m < M && n < N) C[size_t(m) * N + n] = acc[i][j];
      }
    return;
  }
  // the partial tile [64][64] over the (now idle) pipeline stages
  __syncthreads();
  float *Ps = mm_smem;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4 *>(Ps + (ty * 4 + i) * MM_T + tx * 4) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  cluster_sync_all();
  // rows [r*64/S, (r+1)*64/S) of the tile: sum of the S partials, rank order
  const uint32_t r = cluster_rank();
  const int rows = MM_T / S, row0 = int(r) * rows;
  for (int e = tid; e < rows * (MM_T / 4); e += blockDim.x) {
    const int row = row0 + e / (MM_T / 4), c4 = (e % (MM_T / 4)) * 4;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < S; ++q) {
      const float4 v = ld_dsmem_f4(dsmem_addr(Ps + row * MM_T + c4, uint32_t(q)));
      sum.x += v.x, sum.y += v.y, sum.z += v.z, sum.w += v.w;
    }
    const int m = m0 + row;
    if (m < M) {
      const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n0 + c4 + j < N) C[size_t(m) * N + n0 + c4 + j] = sv[j];
    }
  }
  // no CTA leaves while another may still read its partial
  cluster_sync_all();
}
}  // namespace

void launch_mm(const void *a, const void *b, void *out, int64_t M, int64_t N, int64_t K,
               int dtype, void *scratch, uint64_t scratch_bytes, cudaStream_t stream) {
  wgx_conv2d_params p = mm_params(M, N, K, dtype);
  if (dtype == WGX_FLOAT32 && mm_tf32_supported(a, b, out, M, N, K)) {
    mm_tf32_run(static_cast<const float *>(a), static_cast<const float *>(b),
                static_cast<float *>(out), M, N, K, dw_sm_count(), stream);
    return;
  }
  if (dtype == WGX_FLOAT32) {
    const int64_t gy = (M + MM_T - 1) / MM_T, gx = (N + MM_T - 1) / MM_T;
    if (gy > 65535 || gx > INT32_MAX) fail("aten.mm.default: matrix too large");
    // split K over a cluster of S CTAs until the grid covers the SMs
    // (S divides the tile's 64 rows; each part keeps at least 64 of K)
    const int64_t tiles = gx * gy;
    int S = 1;
    while (S < 8 && tiles * S < dw_sm_count() && K / (2 * S) >= 64) S *= 2;
    const int kchunk = int(((K + S - 1) / S + MM_BK - 1) / MM_BK * MM_BK);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(gx), unsigned(gy), unsigned(S));
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = MM_SMEM;
    cfg.stream = stream;
    {
      static std::mutex mu;
      static bool attr_set[64] = {};
      int dev = 0;
      check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
      std::lock_guard<std::mutex> lock(mu);
      if (dev >= 64 || !attr_set[dev]) {
        check_cuda(cudaFuncSetAttribute(mm_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(MM_SMEM)),
                   "mm smem attr");
        if (dev < 64) attr_set[dev] = true;
      }
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = unsigned(S);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_cuda(cudaLaunchKernelEx(&cfg, mm_f32_kernel, static_cast<const float *>(a),
                                  static_cast<const float *>(b), static_cast<float *>(out), int(M),
                                  int(N), int(K), kchunk,
                                  int(K % 4 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0),
                                  int(N % 4 == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0)),
               "mm launch");
    return;
  }
  launch_conv2d(p, b, a, nullptr, nullptr, out, scratch, scratch_bytes, stream);
}

}  // namespace wgx
