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
    depthwise_conv(ConvGeom g, int TH, int TWs, const T *__restrict__ x, const T *__restrict__ w,
                   const T *__restrict__ bias, T *__restrict__ out, int vec_in, int vec_out) {
  extern __shared__ __align__(16) unsigned char dw_smem[];
  float *wsm = reinterpret_cast<float *>(dw_smem);  // KH*KW weights
  T *tile = reinterpret_cast<T *>(dw_smem + DW_MAX_TAPS * sizeof(float));
  const int plane = blockIdx.x;  // b*C + c
  const int c = plane % g.OC;
  const int oh0 = blockIdx.y * TH;
  const int taps = g.KH * g.KW;
  for (int i = threadIdx.x; i < taps; i += blockDim.x) wsm[i] = ld_f(&w[(long long)c * taps + i]);
  const int rows = (TH - 1) * g.sH + (g.KH - 1) * g.dH + 1;
  const int ih0 = oh0 * g.sH - g.pH;
  const T *xp = x + (long long)plane * g.IH * g.IW;
  // stage rows [ih0, ih0+rows) x cols [-pW, -pW+TWs) into the tile; column j
  // of the tile is input column j - pW.
  if (vec_in) {
    // interior: 16-byte vectors of 8 (f16) / 4 (f32) elements
    constexpr int V = 16 / sizeof(T);
    const int nvec = g.IW / V;
    for (int idx = threadIdx.x; idx < rows * nvec; idx += blockDim.x) {
      int r = idx / nvec, v = idx % nvec;
      int ih = ih0 + r;
      T *dst = tile + (long long)r * TWs + g.pW + v * V;
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
      tile[(long long)r * TWs + col] = to_t<T>(0.f);
    }
  } else {
    for (int idx = threadIdx.x; idx < rows * TWs; idx += blockDim.x) {
      int r = idx / TWs, j = idx % TWs;
      int ih = ih0 + r, iw = j - g.pW;
      T v = to_t<T>(0.f);
      if (ih >= 0 && ih < g.IH && iw >= 0 && iw < g.IW) v = xp[(long long)ih * g.IW + iw];
      tile[(long long)r * TWs + j] = v;
    }
  }
  __syncthreads();
  const float bv = g.has_bias ? ld_f(&bias[c]) : 0.f;
  const int ohn = min(TH, g.OH - oh0);
  const int ngrp = (g.OW + 7) / 8;
  T *op = out + (long long)plane * g.OH * g.OW;
  for (int idx = threadIdx.x; idx < ohn * ngrp; idx += blockDim.x) {
    int r = idx / ngrp, q = idx % ngrp;
    int ow0 = q * 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = bv;
    for (int kh = 0; kh < g.KH; ++kh) {
      const T *trow = tile + (long long)(r * g.sH + kh * g.dH) * TWs;
      for (int kw = 0; kw < g.KW; ++kw) {
        float wv = wsm[kh * g.KW + kw];
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
  DwTile d{};
  const int esize = p.dtype == WGX_FLOAT16 ? 2 : 4;
  return plan.variant == WGX_CONV_DEPTHWISE && dw_tiling(p, esize, d) && d.bands == 1 &&
         p.OH == p.IH && p.OW == p.IW;
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
    uint64_t smem = DW_MAX_TAPS * sizeof(float) + tile_bytes(TH) + 16;
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
    long long planes = (long long)p.B * p.OC;
    if (planes > 0x7fffffffLL) fail("conv2d: too many depthwise planes");
    if ((p.OH + TH - 1) / TH > 65535) fail("conv2d: depthwise plane too tall");
    // planes on x (up to 2^31-1 blocks), row bands on y
    dim3 grid(unsigned(planes), unsigned((p.OH + TH - 1) / TH));
    depthwise_conv<T><<<grid, DW_THREADS, smem, s>>>(g, TH, TWs, in, w, bias, out, vec_in,
                                                      vec_out);
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

// fp32 aten.mm, C[M,N] = A[M,K] B[K,N] row-major (mm-64x64.wgsl.ts's GEMM,
// fp32 FMAs in K order as there): a 32x32 output tile per CTA of 256
// threads, 2x2 outputs per thread, 64-deep K steps through shared memory,
// the next step's global loads held in registers while this step's FMAs
// run. 32x32 tiles give a 512 x 512 product 256 CTAs (64x64 tiles: 64 CTAs
// for 148 SMs, each with a long serial K loop). A is stored k-major
// (As[k][m], one pad column: conflict-free transposing stores), B as is.
namespace {
constexpr int MM_T = 32, MM_BK = 64, MM_LD = MM_T * MM_BK / 256;  // loads per thread and operand

__global__ void __launch_bounds__(256) mm_f32_kernel(const float *__restrict__ A,
                                                     const float *__restrict__ B,
                                                     float *__restrict__ C, int M, int N, int K) {
  __shared__ float As[MM_BK][MM_T + 1];
  __shared__ __align__(16) float Bs[MM_BK][MM_T];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * MM_T, n0 = blockIdx.x * MM_T;
  float ra[MM_LD], rb[MM_LD];
  auto load = [&](int k0) {
#pragma unroll
    for (int u = 0; u < MM_LD; ++u) {
      const int e = tid + 256 * u;
      const int ar = e / MM_BK, ac = e % MM_BK;  // A: row m, column k
      const int br = e / MM_T, bc = e % MM_T;    // B: row k, column n
      ra[u] = (m0 + ar < M && k0 + ac < K) ? A[size_t(m0 + ar) * K + k0 + ac] : 0.f;
      rb[u] = (k0 + br < K && n0 + bc < N) ? B[size_t(k0 + br) * N + n0 + bc] : 0.f;
    }
  };
  float acc[2][2] = {};
  load(0);
  for (int k0 = 0; k0 < K; k0 += MM_BK) {
#pragma unroll
    for (int u = 0; u < MM_LD; ++u) {
      const int e = tid + 256 * u;
      As[e % MM_BK][e / MM_BK] = ra[u];
      Bs[e / MM_T][e % MM_T] = rb[u];
    }
    __syncthreads();
    if (k0 + MM_BK < K) load(k0 + MM_BK);
#pragma unroll
    for (int kk = 0; kk < MM_BK; ++kk) {
      const float a0 = As[kk][2 * ty], a1 = As[kk][2 * ty + 1];
      const float2 b = *reinterpret_cast<const float2 *>(&Bs[kk][2 * tx]);
      acc[0][0] = fmaf(a0, b.x, acc[0][0]);
      acc[0][1] = fmaf(a0, b.y, acc[0][1]);
      acc[1][0] = fmaf(a1, b.x, acc[1][0]);
      acc[1][1] = fmaf(a1, b.y, acc[1][1]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int m = m0 + 2 * ty + i, n = n0 + 2 * tx + j;
      if (m < M && n < N) C[size_t(m) * N + n] = acc[i][j];
    }
}
}  // namespace

void launch_mm(const void *a, const void *b, void *out, int64_t M, int64_t N, int64_t K,
               int dtype, void *scratch, uint64_t scratch_bytes, cudaStream_t stream) {
  wgx_conv2d_params p = mm_params(M, N, K, dtype);
  if (dtype == WGX_FLOAT32) {
    const int64_t gy = (M + MM_T - 1) / MM_T, gx = (N + MM_T - 1) / MM_T;
    if (gy > 65535 || gx > INT32_MAX) fail("aten.mm.default: matrix too large");
    mm_f32_kernel<<<dim3(unsigned(gx), unsigned(gy)), 256, 0, stream>>>(
        static_cast<const float *>(a), static_cast<const float *>(b), static_cast<float *>(out),
        int(M), int(N), int(K));
    check_cuda(cudaGetLastError(), "mm launch");
    return;
  }
  launch_conv2d(p, b, a, nullptr, nullptr, out, scratch, scratch_bytes, stream);
}

}  // namespace wgx
