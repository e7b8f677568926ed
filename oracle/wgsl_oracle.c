/*
 * wgsl_oracle.c - TEST INFRASTRUCTURE ONLY. CPU restatement of the
 * reference's WGSL arithmetic for the hot path (aten.mm, aten.convolution,
 * et_vk.conv_with_clamp). Used by tests/ as the parity checker and by
 * bench.py's cpu_baseline / --impl reference leg as the timed CPU
 * baseline. The product never links or calls it.
 *
 * Reference: barhanc/wgpu-executorch (TypeScript + WGSL; the WGSL runs under
 * WebGPU, which has no CPU path on these machines, so this restatement is
 * the oracle). Pinned against the reference's own known-answer tests
 * (tests/shaders/mm.test.ts, convolution.test.ts, conv-with-clamp.test.ts),
 * see tests/test_oracle.py.
 *
 * Two modes:
 *   ORACLE_EXACT (0): products of the stored (fp32 / fp16) inputs summed in
 *       double, bias added, activation in double, one rounding to the
 *       storage type. The mathematical result the tensor-core path targets.
 *   ORACLE_WGSL  (1): the reference kernel's own arithmetic: the variant the
 *       reference's selection picks (src/shaders/convolution/index.ts:171-238,
 *       src/shaders/conv-with-clamp/index.ts:173-243, src/shaders/mm/index.ts:
 *       65-78), its accumulation type (f16 for the f16 kernels, f32 for the
 *       single-channel and transposed f16 kernels), its summation order and
 *       where the bias enters. f16 arithmetic uses _Float16 with
 *       -fexcess-precision=standard so every operation rounds to f16 like
 *       shader f16 math (mul and add rounded separately: no FMA contraction).
 *
 * Accumulation orders restated (all sequential):
 *   GEMM family (conv2d-tile64/-tile32/-gemm/-1x1-*, mm-*): acc = 0; for k in
 *       0..K-1 (k = ic*KH*KW + kh*KW + kw): acc = acc + x*w; then acc + bias
 *       (conv2d-tile64-f16.wgsl.ts:128-160, conv2d-gemm-f16.wgsl.ts:147-160,
 *       mm-64x64.wgsl.ts:74-92).
 *   depthwise (conv2d-depthwise-f16.wgsl.ts:61-119, -3x3 :81-127): acc = bias;
 *       for kh, kw (in-bounds taps): acc = acc + x*w.
 *   direct grouped (conv2d-f16.wgsl.ts:57-86): acc = bias; for icg, kh, kw.
 *   transposed (conv-transpose2d-f16.wgsl.ts:58-95): f32 acc = bias; kh, kw, icg.
 *   single output channel 1x1 (conv-with-clamp-1x1-single-channel-f16.wgsl.ts:
 *       44-58): f32 acc over ic, + bias, clamp, one rounding.
 *   clamp (conv-with-clamp-*): clamp(acc + bias, f16(min), f16(max)) last.
 *
 * The conv2d-tile32 kernels of aten.convolution store out[m*N + n] with
 * N = B*OH*OW (conv2d-tile32-f16.wgsl.ts:193-196), i.e. [OC, B, OH, OW]; that
 * is NCHW only for B == 1. `bug_tile32` reproduces that layout; it is off in
 * every parity test (the engine computes the mathematically correct NCHW).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef _Float16 f16;

#define ORACLE_EXACT 0
#define ORACLE_WGSL 1
#define DT_F32 0
#define DT_F16 1
#define ACT_NONE 0
#define ACT_CLAMP 1
#define ACT_SILU 2

typedef struct {
  int32_t B, IC, IH, IW, OC, OH, OW, KH, KW, sH, sW, pH, pW, dH, dW, groups, has_bias, dtype, act;
  float out_min, out_max;
} conv_params;

/* ------------------------------------------------------------ threads */
/* Dynamic parallel-for over [0, n) on ORACLE_THREADS (default: all online
 * cores) pthreads; chunks of one index are claimed from an atomic counter. */
typedef void (*range_fn)(void *ctx, long i);
typedef struct {
  range_fn fn;
  void *ctx;
  long n;
  long next;
} pf_job;

static void *pf_worker(void *arg) {
  pf_job *j = arg;
  for (;;) {
    long i = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
    if (i >= j->n) break;
    j->fn(j->ctx, i);
  }
  return NULL;
}

int oracle_num_threads(void) {
  const char *e = getenv("ORACLE_THREADS");
  if (e && atoi(e) > 0) return atoi(e);
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static void parallel_for(long n, range_fn fn, void *ctx) {
  int nt = oracle_num_threads();
  if (nt > n) nt = (int)n;
  pf_job job = {fn, ctx, n, 0};
  if (nt <= 1) {
    pf_worker(&job);
    return;
  }
  pthread_t th[256];
  if (nt > 256) nt = 256;
  for (int t = 1; t < nt; ++t) pthread_create(&th[t], NULL, pf_worker, &job);
  pf_worker(&job);
  for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
}

static inline double ld(int dt, const void *p, long i) {
  return dt == DT_F16 ? (double)((const f16 *)p)[i] : (double)((const float *)p)[i];
}
static inline void st(int dt, void *p, long i, double v) {
  if (dt == DT_F16)
    ((f16 *)p)[i] = (f16)v; /* double -> f16: one RNE rounding */
  else
    ((float *)p)[i] = (float)v;
}
static inline double act_d(int act, double v, double lo, double hi) {
  if (act == ACT_CLAMP) return v < lo ? lo : (v > hi ? hi : v);
  if (act == ACT_SILU) return v / (1.0 + exp(-v));
  return v;
}

/* ------------------------------------------------------------------ mm */
typedef struct {
  int dt, mode;
  const void *a, *b;
  void *out;
  long M, N, K;
} mm_job;

static void mm_row(void *vctx, long m) {
  const mm_job *j = vctx;
  const int dt = j->dt, mode = j->mode;
  const void *a = j->a, *b = j->b;
  void *out = j->out;
  const long N = j->N, K = j->K;
  {
    for (long n = 0; n < N; ++n) {
      if (mode == ORACLE_EXACT) {
        double acc = 0;
        for (long k = 0; k < K; ++k) acc += ld(dt, a, m * K + k) * ld(dt, b, k * N + n);
        st(dt, out, m * N + n, acc);
      } else if (dt == DT_F16) {
        const f16 *A = a, *Bm = b;
        f16 acc = 0;
        for (long k = 0; k < K; ++k) {
          f16 prod = A[m * K + k] * Bm[k * N + n];
          acc = acc + prod;
        }
        ((f16 *)out)[m * N + n] = acc;
      } else {
        const float *A = a, *Bm = b;
        float acc = 0;
        for (long k = 0; k < K; ++k) {
          volatile float prod = A[m * K + k] * Bm[k * N + n];
          acc = acc + prod;
        }
        ((float *)out)[m * N + n] = acc;
      }
    }
  }
}

void oracle_mm(int dt, int mode, const void *a, const void *b, void *out, long M, long N, long K) {
  mm_job j = {dt, mode, a, b, out, M, N, K};
  parallel_for(M, mm_row, &j);
}

/* which reference kernel family handles this forward convolution */
enum { FAM_GEMM = 0, FAM_DEPTHWISE = 1, FAM_DIRECT = 2, FAM_SINGLE = 3 };

static int conv_family(const conv_params *p, int is_clamp_op) {
  int is1x1 = p->KH == 1 && p->KW == 1 && p->sH == 1 && p->sW == 1 && p->pH == 0 && p->pW == 0 &&
              p->dH == 1 && p->dW == 1;
  long ohw = (long)p->OH * p->OW;
  if (is_clamp_op && is1x1 && p->groups == 1 && p->OC == 1 && p->IC <= 32 && ohw % 4 == 0 &&
      (ohw + 255) / 256 <= 65535 && p->B <= 65535)
    return FAM_SINGLE;
  int icpg = p->IC / p->groups;
  if (p->groups == p->OC && p->IC == p->OC && icpg == 1 && p->KH * p->KW <= 49 &&
      (long)p->B * p->OC <= 65535)
    return FAM_DEPTHWISE;
  if (p->groups == 1) return FAM_GEMM;
  return FAM_DIRECT;
}

/* tile32 selection of aten.convolution (convolution/index.ts:184-190, with
 * the 1x1-tile32/64 kernels taking precedence when B == 1) */
static int uses_tile32_layout(const conv_params *p) {
  int is1x1 = p->KH == 1 && p->KW == 1 && p->sH == 1 && p->sW == 1 && p->pH == 0 && p->pW == 0 &&
              p->dH == 1 && p->dW == 1;
  long ohw = (long)p->OH * p->OW;
  int is1x1Vec4 = is1x1 && p->IC % 4 == 0 && ohw % 4 == 0 && p->OC % 4 == 0;
  int is1x1Tile = is1x1Vec4 && p->B == 1 && ohw >= 64 && p->IC >= 16;
  long K = (long)p->IC * p->KH * p->KW;
  return p->groups == 1 && !is1x1Tile && p->OC <= 32 && p->OC >= 8 &&
         (long)p->B * ohw >= 64 && K % 4 == 0;
}

/* is_clamp_op: 1 for et_vk.conv_with_clamp (selects the single-channel
 * kernel and the clamp epilogue), 0 for aten.convolution. */
typedef struct {
  int mode, is_clamp_op, bug_tile32;
  const conv_params *p;
  const void *x, *w, *bias;
  void *out;
} conv_job;

static void conv_plane(void *vctx, long idx) {
  const conv_job *j = vctx;
  const conv_params *p = j->p;
  const int mode = j->mode, is_clamp_op = j->is_clamp_op;
  const void *x = j->x, *w = j->w, *bias = j->bias;
  void *out = j->out;
  const int dt = p->dtype;
  const int fam = conv_family(p, is_clamp_op);
  const int icpg = p->IC / p->groups, ocpg = p->OC / p->groups;
  const long ohw = (long)p->OH * p->OW;
  const int tile32_bug = j->bug_tile32 && !is_clamp_op && uses_tile32_layout(p);
  const double lo = p->out_min, hi = p->out_max;
  const int b = (int)(idx / p->OC), oc = (int)(idx % p->OC);
  {
    {
      const int g = oc / ocpg;
      const double bv = p->has_bias ? ld(dt, bias, oc) : 0.0;
      for (int oh = 0; oh < p->OH; ++oh) {
        for (int ow = 0; ow < p->OW; ++ow) {
          long oidx = ((long)b * p->OC + oc) * ohw + (long)oh * p->OW + ow;
          if (tile32_bug) oidx = (long)oc * ((long)p->B * ohw) + (long)b * ohw + (long)oh * p->OW + ow;
          if (mode == ORACLE_EXACT) {
            double acc = 0;
            for (int c = 0; c < icpg; ++c) {
              int ic = g * icpg + c;
              for (int kh = 0; kh < p->KH; ++kh) {
                int ih = oh * p->sH - p->pH + kh * p->dH;
                if (ih < 0 || ih >= p->IH) continue;
                for (int kw = 0; kw < p->KW; ++kw) {
                  int iw = ow * p->sW - p->pW + kw * p->dW;
                  if (iw < 0 || iw >= p->IW) continue;
                  acc += ld(dt, x, (((long)b * p->IC + ic) * p->IH + ih) * p->IW + iw) *
                         ld(dt, w, (((long)oc * icpg + c) * p->KH + kh) * p->KW + kw);
                }
              }
            }
            st(dt, out, oidx, act_d(p->act, acc + bv, lo, hi));
            continue;
          }
          /* ---- wgsl-faithful */
          if (fam == FAM_SINGLE) {
            float acc = 0.f; /* f32 accumulation of widened f16 operands */
            for (int ic = 0; ic < p->IC; ++ic) {
              float xv = (float)ld(dt, x, ((long)b * p->IC + ic) * ohw + (long)oh * p->OW + ow);
              float wv = (float)ld(dt, w, ic);
              volatile float prod = xv * wv;
              acc = acc + prod;
            }
            if (p->has_bias) acc = acc + (float)bv;
            float lof = p->out_min, hif = p->out_max;
            acc = acc < lof ? lof : (acc > hif ? hif : acc);
            st(dt, out, oidx, acc);
            continue;
          }
          if (dt == DT_F16) {
            const f16 *X = x, *W = w;
            f16 acc = (fam == FAM_GEMM) ? (f16)0 : (f16)bv;
            for (int c = 0; c < icpg; ++c) {
              int ic = g * icpg + c;
              for (int kh = 0; kh < p->KH; ++kh) {
                int ih = oh * p->sH - p->pH + kh * p->dH;
                if (ih < 0 || ih >= p->IH) continue;
                for (int kw = 0; kw < p->KW; ++kw) {
                  int iw = ow * p->sW - p->pW + kw * p->dW;
                  if (iw < 0 || iw >= p->IW) continue;
                  f16 prod = X[(((long)b * p->IC + ic) * p->IH + ih) * p->IW + iw] *
                             W[(((long)oc * icpg + c) * p->KH + kh) * p->KW + kw];
                  acc = acc + prod;
                }
              }
            }
            if (fam == FAM_GEMM) acc = acc + (f16)bv;
            if (p->act == ACT_CLAMP) {
              f16 l = (f16)p->out_min, h = (f16)p->out_max;
              acc = acc < l ? l : (acc > h ? h : acc);
            } else if (p->act == ACT_SILU) {
              /* reference: sigmoid then mul, each in f16 (sigmoid-f16 / mul-elementwise-f16) */
              f16 e = (f16)expf(-(float)acc);
              f16 sg = (f16)1.0f / ((f16)1.0f + e);
              acc = acc * sg;
            }
            ((f16 *)out)[oidx] = acc;
          } else {
            const float *X = x, *W = w;
            float acc = (fam == FAM_GEMM) ? 0.f : (float)bv;
            for (int c = 0; c < icpg; ++c) {
              int ic = g * icpg + c;
              for (int kh = 0; kh < p->KH; ++kh) {
                int ih = oh * p->sH - p->pH + kh * p->dH;
                if (ih < 0 || ih >= p->IH) continue;
                for (int kw = 0; kw < p->KW; ++kw) {
                  int iw = ow * p->sW - p->pW + kw * p->dW;
                  if (iw < 0 || iw >= p->IW) continue;
                  volatile float prod = X[(((long)b * p->IC + ic) * p->IH + ih) * p->IW + iw] *
                                        W[(((long)oc * icpg + c) * p->KH + kh) * p->KW + kw];
                  acc = acc + prod;
                }
              }
            }
            if (fam == FAM_GEMM) acc = acc + (float)bv;
            if (p->act == ACT_CLAMP) {
              acc = acc < p->out_min ? p->out_min : (acc > p->out_max ? p->out_max : acc);
            } else if (p->act == ACT_SILU) {
              float sg = 1.0f / (1.0f + expf(-acc));
              acc = acc * sg;
            }
            ((float *)out)[oidx] = acc;
          }
        }
      }
    }
  }
}

/* Exact mode, plane-wise: for output plane (b, oc) the products of the
 * stored inputs (pre-widened to double once, `xd`) are accumulated in a
 * double plane, input channel and filter tap outermost, so the inner loop
 * runs over contiguous output columns of one row with the in-bounds column
 * range computed up front. Same value as the per-output loop of conv_plane
 * (double sums of the same products; only the order of the additions
 * differs, far below one rounding of the storage type). */
typedef struct {
  const conv_job *j;
  const double *xd;
} exact_job;

static void conv_plane_exact(void *vctx, long idx) {
  const exact_job *e = vctx;
  const conv_job *j = e->j;
  const conv_params *p = j->p;
  const int dt = p->dtype;
  const int icpg = p->IC / p->groups, ocpg = p->OC / p->groups;
  const long ohw = (long)p->OH * p->OW, ihw = (long)p->IH * p->IW;
  const int tile32_bug = j->bug_tile32 && !j->is_clamp_op && uses_tile32_layout(p);
  const int b = (int)(idx / p->OC), oc = (int)(idx % p->OC);
  const int g = oc / ocpg;
  double *acc = calloc((size_t)ohw, sizeof(double));
  if (!acc) abort();
  for (int c = 0; c < icpg; ++c) {
    const double *xp = e->xd + ((long)b * p->IC + g * icpg + c) * ihw;
    for (int kh = 0; kh < p->KH; ++kh)
      for (int kw = 0; kw < p->KW; ++kw) {
        const double wv = ld(dt, j->w, (((long)oc * icpg + c) * p->KH + kh) * p->KW + kw);
        /* in-bounds output columns: 0 <= ow*sW + off < IW */
        const int off = kw * p->dW - p->pW;
        int ow0 = off >= 0 ? 0 : (-off + p->sW - 1) / p->sW;
        int ow1 = (p->IW - 1 - off) >= 0 ? (p->IW - 1 - off) / p->sW + 1 : 0;
        if (ow1 > p->OW) ow1 = p->OW;
        for (int oh = 0; oh < p->OH; ++oh) {
          const int ih = oh * p->sH - p->pH + kh * p->dH;
          if (ih < 0 || ih >= p->IH) continue;
          const double *row = xp + (long)ih * p->IW + off;
          double *a = acc + (long)oh * p->OW;
          for (int ow = ow0; ow < ow1; ++ow) a[ow] += row[(long)ow * p->sW] * wv;
        }
      }
  }
  const double bv = p->has_bias ? ld(dt, j->bias, oc) : 0.0;
  for (long i = 0; i < ohw; ++i) {
    long oidx = ((long)b * p->OC + oc) * ohw + i;
    if (tile32_bug) oidx = (long)oc * ((long)p->B * ohw) + (long)b * ohw + i;
    st(dt, j->out, oidx, act_d(p->act, acc[i] + bv, p->out_min, p->out_max));
  }
  free(acc);
}

typedef struct {
  int dt;
  const void *src;
  double *dst;
  long n, chunk;
} widen_job;

static void widen_chunk(void *vctx, long c) {
  const widen_job *w = vctx;
  const long i0 = c * w->chunk, i1 = i0 + w->chunk < w->n ? i0 + w->chunk : w->n;
  for (long i = i0; i < i1; ++i) w->dst[i] = ld(w->dt, w->src, i);
}

void oracle_conv2d(int mode, int is_clamp_op, const conv_params *p, const void *x, const void *w,
                   const void *bias, void *out, int bug_tile32) {
  conv_job j = {mode, is_clamp_op, bug_tile32, p, x, w, bias, out};
  if (mode == ORACLE_EXACT) {
    const long n = (long)p->B * p->IC * p->IH * p->IW;
    double *xd = malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
    if (!xd) abort();
    widen_job wj = {p->dtype, x, xd, n, 1 << 16};
    parallel_for((n + wj.chunk - 1) / wj.chunk, widen_chunk, &wj);
    exact_job e = {&j, xd};
    parallel_for((long)p->B * p->OC, conv_plane_exact, &e);
    free(xd);
    return;
  }
  parallel_for((long)p->B * p->OC, conv_plane, &j);
}

/* transposed conv (conv-transpose2d{,-f16}.wgsl.ts); weight [IC, OC/g, KH, KW] */
static void convt_plane(void *vctx, long idx) {
  const conv_job *j = vctx;
  const conv_params *p = j->p;
  const int mode = j->mode;
  const void *x = j->x, *w = j->w, *bias = j->bias;
  void *out = j->out;
  const int dt = p->dtype;
  const int icpg = p->IC / p->groups, ocpg = p->OC / p->groups;
  const int b = (int)(idx / p->OC), oc = (int)(idx % p->OC);
  {
      int g = oc / ocpg, ocl = oc % ocpg;
      for (int oh = 0; oh < p->OH; ++oh)
        for (int ow = 0; ow < p->OW; ++ow) {
          double accd = p->has_bias ? ld(dt, bias, oc) : 0.0;
          float accf = (float)accd;
          for (int kh = 0; kh < p->KH; ++kh) {
            int nh = oh + p->pH - kh * p->dH;
            if (nh % p->sH != 0) continue;
            int ih = nh / p->sH;
            if (ih < 0 || ih >= p->IH) continue;
            for (int kw = 0; kw < p->KW; ++kw) {
              int nw = ow + p->pW - kw * p->dW;
              if (nw % p->sW != 0) continue;
              int iw = nw / p->sW;
              if (iw < 0 || iw >= p->IW) continue;
              for (int c = 0; c < icpg; ++c) {
                int ic = g * icpg + c;
                double xv = ld(dt, x, (((long)b * p->IC + ic) * p->IH + ih) * p->IW + iw);
                double wv = ld(dt, w, (((long)ic * ocpg + ocl) * p->KH + kh) * p->KW + kw);
                accd += xv * wv;
                volatile float prod = (float)xv * (float)wv;
                accf = accf + prod;
              }
            }
          }
          long oidx = (((long)b * p->OC + oc) * p->OH + oh) * p->OW + ow;
          st(dt, out, oidx, mode == ORACLE_EXACT ? accd : (double)accf);
        }
    }
}

void oracle_conv_transpose2d(int mode, const conv_params *p, const void *x, const void *w,
                             const void *bias, void *out) {
  conv_job j = {mode, 0, 0, p, x, w, bias, out};
  parallel_for((long)p->B * p->OC, convt_plane, &j);
}

/* f16 <-> f32 helpers (RNE), so Python can round without numpy quirks */
void oracle_f32_to_f16(const float *src, uint16_t *dst, long n) {
  for (long i = 0; i < n; ++i) {
    f16 h = (f16)src[i];
    memcpy(&dst[i], &h, 2);
  }
}
void oracle_f16_to_f32(const uint16_t *src, float *dst, long n) {
  for (long i = 0; i < n; ++i) {
    f16 h;
    memcpy(&h, &src[i], 2);
    dst[i] = (float)h;
  }
}
