// Elementwise operators needed to run whole programs around the
// convolutions: aten.add.Tensor / aten.sub.Tensor (in1 +/- alpha*in2),
// aten.mul.Tensor (in1*in2) with trailing-dimension broadcasting
// (src/shaders/add/index.ts:33-120, src/shaders/utils/broadcasting.ts),
// aten.sigmoid / aten.relu / aten.hardswish (src/shaders/sigmoid,
// relu, hardswish). Arithmetic is done in fp32 and rounded once to the
// storage type.
#include "internal.h"

namespace wgx {

constexpr int EW_MAX_DIM = 8;
struct BcastIdx {
  int ndim;
  int64_t out_shape[EW_MAX_DIM];
  int64_t sa[EW_MAX_DIM];  // element strides of in1 per out dim (0 = broadcast)
  int64_t sb[EW_MAX_DIM];
};

enum BinOp { kAdd = 0, kSub = 1, kMul = 2 };
enum UnOp { kSigmoid = 0, kRelu = 1, kHardswish = 2 };

template <class T>
__device__ __forceinline__ float lf(T v) {
  return float(v);
}
template <>
__device__ __forceinline__ float lf<__half>(__half v) {
  return __half2float(v);
}
template <class T>
__device__ __forceinline__ T st(float v) {
  return T(v);
}
template <>
__device__ __forceinline__ __half st<__half>(float v) {
  return __float2half_rn(v);
}

__device__ __forceinline__ float binop(int op, float a, float b, float alpha) {
  return op == kAdd ? a + alpha * b : op == kSub ? a - alpha * b : a * b;
}
__device__ __forceinline__ float unop(int op, float v) {
  if (op == kSigmoid) return 1.0f / (1.0f + __expf(-v));
  if (op == kRelu) return fmaxf(v, 0.0f);
  return fminf(fmaxf(v + 3.0f, 0.0f), 6.0f) * v / 6.0f;
}

template <class T>
__global__ void ew_binary_same(int op, float alpha, const T *__restrict__ a,
                               const T *__restrict__ b, T *__restrict__ out, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) out[i] = st<T>(binop(op, lf(a[i]), lf(b[i]), alpha));
}

// fp16, n % 8 == 0, 16-byte aligned operands: eight elements per 16-byte
// access (the same per-element fp32 arithmetic and single rounding)
__device__ __forceinline__ uint4 map8(uint4 v, uint4 w, int op, float alpha) {
  const __half2 *a = reinterpret_cast<const __half2 *>(&v), *b = reinterpret_cast<const __half2 *>(&w);
  uint4 r;
  __half2 *o = reinterpret_cast<__half2 *>(&r);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 fa = __half22float2(a[k]), fb = __half22float2(b[k]);
    o[k] = __floats2half2_rn(binop(op, fa.x, fb.x, alpha), binop(op, fa.y, fb.y, alpha));
  }
  return r;
}
__global__ void ew_binary_same_h8(int op, float alpha, const uint4 *__restrict__ a,
                                  const uint4 *__restrict__ b, uint4 *__restrict__ out,
                                  long long n8) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < n8; i += stride) out[i] = map8(a[i], b[i], op, alpha);
}

// fp16 operands that are contiguous over the output's trailing dimensions
// and repeated over its leading ones (index = i mod period, the period a
// multiple of 8): eight elements per 16-byte access.
__global__ void ew_binary_period_h8(int op, float alpha, const uint4 *__restrict__ a,
                                    const uint4 *__restrict__ b, uint4 *__restrict__ out,
                                    long long n8, long long pa8, long long pb8) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < n8; i += stride) out[i] = map8(a[i % pa8], b[i % pb8], op, alpha);
}

template <class T>
__global__ void ew_binary_bcast(int op, float alpha, BcastIdx ix, const T *__restrict__ a,
                                const T *__restrict__ b, T *__restrict__ out, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    long long r = i, ia = 0, ib = 0;
    for (int d = ix.ndim - 1; d >= 0; --d) {
      long long c = r % ix.out_shape[d];
      r /= ix.out_shape[d];
      ia += c * ix.sa[d];
      ib += c * ix.sb[d];
    }
    out[i] = st<T>(binop(op, lf(a[ia]), lf(b[ib]), alpha));
  }
}

template <class T>
__global__ void ew_unary(int op, const T *__restrict__ x, T *__restrict__ out, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long stride = (long long)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    out[i] = st<T>(unop(op, lf(x[i])));
  }
}

// sigmoid for fp16 outputs: 0.5 * tanh(v / 2) + 0.5 with tanh.approx.f32
// (one multi-function-unit op and two FMAs; tanh.approx's relative error is
// at most 2^-11, i.e. 2.4e-4 on the sigmoid, the size of the fp16 rounding
// that follows) instead of 1 / (1 + exp(-v)), whose IEEE division made the
// kernel instruction bound
__device__ __forceinline__ float sigmoid_h(float v) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * v));
  return fmaf(0.5f, t, 0.5f);
}

__global__ void ew_unary_h8(int op, const uint4 *__restrict__ x, uint4 *__restrict__ out,
                            long long n8) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  if (op == kSigmoid) {
    for (; i < n8; i += stride) {
      const uint4 v = x[i];
      const __half2 *a = reinterpret_cast<const __half2 *>(&v);
      uint4 r;
      __half2 *o = reinterpret_cast<__half2 *>(&r);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(a[k]);
        o[k] = __floats2half2_rn(sigmoid_h(f.x), sigmoid_h(f.y));
      }
      out[i] = r;
    }
    return;
  }
  for (; i < n8; i += stride) {
    const uint4 v = x[i];
    const __half2 *a = reinterpret_cast<const __half2 *>(&v);
    uint4 r;
    __half2 *o = reinterpret_cast<__half2 *>(&r);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(a[k]);
      o[k] = __floats2half2_rn(unop(op, f.x), unop(op, f.y));
    }
    out[i] = r;
  }
}

static bool vec8(long long n, const void *p0, const void *p1, const void *p2 = nullptr) {
  return n % 8 == 0 && ((reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1) |
                         reinterpret_cast<uintptr_t>(p2)) & 15) == 0;
}

static unsigned ew_blocks(long long n) {
  long long b = (n + 255) / 256;
  return unsigned(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}

static bool broadcastable(const wgx_tensor *t, const wgx_tensor *out) {
  if (t->ndim > out->ndim) return false;
  for (int i = 0; i < t->ndim; ++i) {
    int64_t d = t->shape[t->ndim - 1 - i], td = out->shape[out->ndim - 1 - i];
    if (d != 1 && d != td) return false;
  }
  return true;
}

static void bcast_strides(const wgx_tensor *t, const wgx_tensor *out, int64_t *s) {
  int64_t stride = 1;
  for (int d = out->ndim - 1; d >= 0; --d) {
    int td = d - (out->ndim - t->ndim);
    if (td < 0) {
      s[d] = 0;
      continue;
    }
    s[d] = t->shape[td] == 1 ? 0 : stride;
    stride *= t->shape[td];
  }
}

// Number of output elements after which operand t repeats when t equals the
// output's trailing dimensions from some dimension on and is 1 (or absent)
// before it; 0 when t broadcasts in another pattern.
static int64_t repeat_period(const wgx_tensor *t, const wgx_tensor *out) {
  const int off = out->ndim - t->ndim;
  int k = out->ndim;  // first dimension of the contiguous trailing block
  for (int d = out->ndim - 1; d >= 0; --d) {
    const int td = d - off;
    const int64_t ts = td >= 0 ? t->shape[td] : 1;
    if (ts == out->shape[d]) {
      k = d;
      continue;
    }
    break;
  }
  for (int d = 0; d < k; ++d) {
    const int td = d - off;
    if (td >= 0 && t->shape[td] != 1) return 0;
  }
  int64_t period = 1;
  for (int d = k; d < out->ndim; ++d) period *= out->shape[d];
  return period;
}

static bool same_shape(const wgx_tensor *a, const wgx_tensor *b) {
  if (a->ndim != b->ndim) return false;
  for (int i = 0; i < a->ndim; ++i)
    if (a->shape[i] != b->shape[i]) return false;
  return true;
}

static void record_binary(wgx_context *ctx, const std::vector<wgx_arg> &args, const char *name,
                          int op, bool has_alpha) {
  if (args.size() < 3) fail(std::string(name) + ": expected at least 3 args");
  wgx_tensor *a = args[0].kind == WGX_ARG_TENSOR ? args[0].v.tensor : nullptr;
  wgx_tensor *b = args[1].kind == WGX_ARG_TENSOR ? args[1].v.tensor : nullptr;
  float alpha = 1.0f;
  wgx_tensor *out;
  if (has_alpha && args.size() == 4) {
    if (args[2].kind == WGX_ARG_NUMBER) alpha = float(args[2].v.number);
    out = args[3].kind == WGX_ARG_TENSOR ? args[3].v.tensor : nullptr;
  } else {
    out = args[2].kind == WGX_ARG_TENSOR ? args[2].v.tensor : nullptr;
  }
  if (!a || !b || !out) fail(std::string(name) + ": expected Tensor arguments");
  if ((a->dtype != WGX_FLOAT32 && a->dtype != WGX_FLOAT16) || b->dtype != a->dtype ||
      out->dtype != a->dtype)
    fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
  if (!broadcastable(a, out) || !broadcastable(b, out))
    fail(std::string(name) + ": Input shapes are not broadcastable to output shape");
  const void *pa = a->data(), *pb = b->data();
  void *po = out->data();
  long long n = out->numel;
  int dtype = a->dtype;
  Command c;
  c.name = name;
  c.kernel_launches = 1;
  if (same_shape(a, out) && same_shape(b, out)) {
    const bool v8 = dtype == WGX_FLOAT16 && vec8(n, pa, pb, po);
    c.run = [=](const ExecEnv &env) {
      if (v8)
        ew_binary_same_h8<<<ew_blocks(n / 8), 256, 0, env.stream>>>(
            op, alpha, (const uint4 *)pa, (const uint4 *)pb, (uint4 *)po, n / 8);
      else if (dtype == WGX_FLOAT16)
        ew_binary_same<__half><<<ew_blocks(n), 256, 0, env.stream>>>(
            op, alpha, (const __half *)pa, (const __half *)pb, (__half *)po, n);
      else
        ew_binary_same<float><<<ew_blocks(n), 256, 0, env.stream>>>(
            op, alpha, (const float *)pa, (const float *)pb, (float *)po, n);
      check_cuda(cudaGetLastError(), "elementwise launch");
    };
  } else if (dtype == WGX_FLOAT16 && vec8(n, pa, pb, po) && repeat_period(a, out) % 8 == 0 &&
             repeat_period(b, out) % 8 == 0 && repeat_period(a, out) > 0 &&
             repeat_period(b, out) > 0) {
    const long long pa8 = repeat_period(a, out) / 8, pb8 = repeat_period(b, out) / 8;
    c.run = [=](const ExecEnv &env) {
      ew_binary_period_h8<<<ew_blocks(n / 8), 256, 0, env.stream>>>(
          op, alpha, (const uint4 *)pa, (const uint4 *)pb, (uint4 *)po, n / 8, pa8, pb8);
      check_cuda(cudaGetLastError(), "elementwise launch");
    };
  } else {
    BcastIdx ix{};
    ix.ndim = out->ndim;
    for (int d = 0; d < out->ndim; ++d) ix.out_shape[d] = out->shape[d];
    bcast_strides(a, out, ix.sa);
    bcast_strides(b, out, ix.sb);
    c.run = [=](const ExecEnv &env) {
      if (dtype == WGX_FLOAT16)
        ew_binary_bcast<__half><<<ew_blocks(n), 256, 0, env.stream>>>(
            op, alpha, ix, (const __half *)pa, (const __half *)pb, (__half *)po, n);
      else
        ew_binary_bcast<float><<<ew_blocks(n), 256, 0, env.stream>>>(
            op, alpha, ix, (const float *)pa, (const float *)pb, (float *)po, n);
      check_cuda(cudaGetLastError(), "elementwise launch");
    };
  }
  ctx->commands.push_back(std::move(c));
}

static void record_unary(wgx_context *ctx, const std::vector<wgx_arg> &args, const char *name,
                         int op) {
  if (args.size() < 2 || args[0].kind != WGX_ARG_TENSOR || args[1].kind != WGX_ARG_TENSOR)
    fail(std::string(name) + ": expected [input, output] tensors");
  wgx_tensor *x = args[0].v.tensor, *out = args[1].v.tensor;
  if ((x->dtype != WGX_FLOAT32 && x->dtype != WGX_FLOAT16) || out->dtype != x->dtype)
    fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
  if (x->numel != out->numel) fail(std::string(name) + ": input numel != output numel");
  const void *px = x->data();
  void *po = out->data();
  long long n = out->numel;
  int dtype = x->dtype;
  Command c;
  c.name = name;
  c.kernel_launches = 1;
  const bool v8 = dtype == WGX_FLOAT16 && vec8(n, px, po);
  c.run = [=](const ExecEnv &env) {
    if (v8)
      ew_unary_h8<<<ew_blocks(n / 8), 256, 0, env.stream>>>(op, (const uint4 *)px, (uint4 *)po,
                                                             n / 8);
    else if (dtype == WGX_FLOAT16)
      ew_unary<__half><<<ew_blocks(n), 256, 0, env.stream>>>(op, (const __half *)px,
                                                              (__half *)po, n);
    else
      ew_unary<float><<<ew_blocks(n), 256, 0, env.stream>>>(op, (const float *)px, (float *)po,
                                                             n);
    check_cuda(cudaGetLastError(), "elementwise launch");
  };
  ctx->commands.push_back(std::move(c));
}

void register_elementwise_ops(std::unordered_map<std::string, OpRecorder> &r) {
  r["aten.add.Tensor"] = [](wgx_context *c, const std::vector<wgx_arg> &a) {
    record_binary(c, a, "aten.add.Tensor", kAdd, true);
  };
  r["aten.sub.Tensor"] = [](wgx_context *c, const std::vector<wgx_arg> &a) {
    record_binary(c, a, "aten.sub.Tensor", kSub, true);
  };
  r["aten.mul.Tensor"] = [](wgx_context *c, const std::vector<wgx_arg> &a) {
    record_binary(c, a, "aten.mul.Tensor", kMul, false);
  };
  r["aten.sigmoid.default"] = [](wgx_context *c, const std::vector<wgx_arg> &a) {
    record_unary(c, a, "aten.sigmoid.default", kSigmoid);
  };
  r["aten.relu.default"] = [](wgx_context *c, const std::vector<wgx_arg> &a) {
    record_unary(c, a, "aten.relu.default", kRelu);
  };
  r["aten.hardswish.default"] = [](wgx_context *c, const std::vector<wgx_arg> &a) {
    record_unary(c, a, "aten.hardswish.default", kHardswish);
  };
}


}  // namespace wgx
