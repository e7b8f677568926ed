// Data-movement, pooling, reduction and resampling operators that the
// shipped YOLO26-N / DepthART / selfie-segmentation programs chain around
// their convolutions. Each recorder follows the reference operator's
// argument layout and validation (file:line per op); arithmetic is fp32 with
// one rounding to the storage type.
//
//   aten.view_copy / clone / squeeze_copy.dims / unsqueeze_copy,
//   et_vk.prepack       flat byte copies   (src/shaders/utils/flat-copy.ts:31-60)
//   aten.cat            pitched copies     (src/shaders/cat/index.ts:27-113)
//   aten.split_with_sizes_copy  pitched    (src/shaders/split-with-sizes/index.ts:30-82)
//   aten.permute_copy   index remap        (src/shaders/permute/index.ts:34-73)
//   aten.bmm            batched GEMM       (src/shaders/bmm/index.ts:33-55)
//   aten.max_pool2d_with_indices           (src/shaders/max-pool-2d/index.ts:36-94)
//   aten._softmax                          (src/shaders/softmax/index.ts:60-90)
//   aten.upsample_nearest2d.vec            (src/shaders/upsample-nearest-2d/index.ts:30-54)
//   aten.upsample_bilinear2d.vec           (src/shaders/upsample-bilinear2d/index.ts:28-60)
//   aten.mean.dim                          (src/shaders/mean-dim/index.ts:26-112)
//   aten.constant_pad_nd                   (src/shaders/constant-pad-nd/index.ts:20-76)
#include <algorithm>
#include <cmath>

#include "internal.h"
#include "umma_conv.h"

namespace wgx {

namespace {

const wgx_arg &at(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  if (i >= a.size()) fail(std::string(op) + ": missing argument " + std::to_string(i));
  return a[i];
}
wgx_tensor *tensor_at(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = at(a, i, op);
  if (x.kind != WGX_ARG_TENSOR || !x.v.tensor)
    fail(std::string(op) + ": argument " + std::to_string(i) + " must be a Tensor");
  return x.v.tensor;
}
std::vector<wgx_tensor *> tensors_at(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = at(a, i, op);
  if (x.kind == WGX_ARG_TENSOR) return {x.v.tensor};
  if (x.kind != WGX_ARG_TENSOR_LIST)
    fail(std::string(op) + ": argument " + std::to_string(i) + " must be a Tensor list");
  return std::vector<wgx_tensor *>(x.v.tensors, x.v.tensors + x.count);
}
double num_at(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = at(a, i, op);
  if (x.kind == WGX_ARG_NUMBER) return x.v.number;
  if (x.kind == WGX_ARG_BOOL) return x.v.boolean;
  fail(std::string(op) + ": argument " + std::to_string(i) + " must be a number");
}
std::vector<int64_t> list_at(const std::vector<wgx_arg> &a, size_t i, const char *op) {
  const wgx_arg &x = at(a, i, op);
  if (x.kind == WGX_ARG_NULL) return {};
  if (x.kind == WGX_ARG_NUMBER) return {int64_t(x.v.number)};
  if (x.kind != WGX_ARG_INT_LIST)
    fail(std::string(op) + ": argument " + std::to_string(i) + " must be an int list");
  return std::vector<int64_t>(x.v.ints, x.v.ints + x.count);
}
bool is_float(int dt) { return dt == WGX_FLOAT32 || dt == WGX_FLOAT16; }
void require_float_pair(const wgx_tensor *a, const wgx_tensor *b, const char *op) {
  if (!is_float(a->dtype) || b->dtype != a->dtype)
    fail(std::string(op) + ": Tensors must have matching float32 or float16 dtype");
}

template <class T>
__device__ __forceinline__ float lf(T v) {
  return float(v);
}
template <>
__device__ __forceinline__ float lf<__half>(__half v) {
  return __half2float(v);
}
template <class T>
__device__ __forceinline__ T sf(float v) {
  return T(v);
}
template <>
__device__ __forceinline__ __half sf<__half>(float v) {
  return __float2half_rn(v);
}

unsigned blocks_for(long long n, int threads = 256) {
  long long b = (n + threads - 1) / threads;
  return unsigned(std::min<long long>(std::max<long long>(b, 1), 148LL * 64));
}

void push(wgx_context *ctx, const char *name, int launches, std::function<void(const ExecEnv &)> f) {
  Command c;
  c.name = name;
  c.kernel_launches = launches;
  c.run = std::move(f);
  ctx->commands.push_back(std::move(c));
}

// ------------------------------------------------------------ flat copies
void record_flat_copy(wgx_context *ctx, const std::vector<wgx_arg> &a, const char *name,
                      size_t in_idx, size_t out_idx) {
  wgx_tensor *in = tensor_at(a, in_idx, name), *out = tensor_at(a, out_idx, name);
  if (in->dtype != out->dtype)
    fail(std::string(name) + ": dtype mismatch (" + dtype_name(in->dtype) + " != " +
         dtype_name(out->dtype) + ")");
  if (in->numel != out->numel)
    fail(std::string(name) + ": numel mismatch (" + std::to_string(in->numel) + " != " +
         std::to_string(out->numel) + ")");
  if (in->buffer == out->buffer) return;  // aliased: already in place (flat-copy.ts:46-48)
  const void *s = in->data();
  void *d = out->data();
  const uint64_t bytes = in->byte_length();
  push(ctx, name, 0, [=](const ExecEnv &env) {
    check_cuda(cudaMemcpyAsync(d, s, bytes, cudaMemcpyDeviceToDevice, env.stream), name);
  });
}

// --------------------------------------------------------- cat / split
// Up to kMaxPieces pitched 2-D copies in one launch: piece p copies `rows`
// rows of width[p] bytes from src[p] (row pitch spitch[p]) to dst[p] (row
// pitch dpitch[p]). The pieces tile one virtual row of `row16` 16-byte
// vectors (col0 = first vector of each piece); every pointer, pitch and
// width is a multiple of 16 bytes (the host falls back to pitched memcpy
// otherwise), so each thread moves whole 16-byte vectors.
constexpr int kMaxPieces = 8;
struct MultiCopy {
  int n;
  long long rows, row16;
  const char *src[kMaxPieces];
  char *dst[kMaxPieces];
  long long spitch[kMaxPieces], dpitch[kMaxPieces], col0[kMaxPieces + 1];
};

__global__ void __launch_bounds__(256) multi_copy_kernel(MultiCopy m) {
  const long long total = m.rows * m.row16;
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    const long long row = i / m.row16, c = i - row * m.row16;
    int p = 0;
#pragma unroll
    for (int q = 1; q < kMaxPieces; ++q)
      if (q < m.n && c >= m.col0[q]) p = q;
    const long long off = (c - m.col0[p]) * 16;
    const uint4 v = *reinterpret_cast<const uint4 *>(m.src[p] + row * m.spitch[p] + off);
    *reinterpret_cast<uint4 *>(m.dst[p] + row * m.dpitch[p] + off) = v;
  }
}

struct CopyPiece {
  const char *src;
  char *dst;
  size_t spitch, dpitch, width;
};

// Launch pitched copies: whole-vector pieces through multi_copy_kernel (in
// groups of kMaxPieces), anything unaligned through cudaMemcpy2DAsync.
void run_pieces(const std::vector<CopyPiece> &pieces, size_t rows, cudaStream_t stream,
                const char *what) {
  auto aligned = [](const CopyPiece &p) {
    return ((reinterpret_cast<uintptr_t>(p.src) | reinterpret_cast<uintptr_t>(p.dst) | p.spitch |
             p.dpitch | p.width) &
            15) == 0;
  };
  MultiCopy m{};
  auto flush = [&] {
    if (m.n == 0) return;
    m.rows = (long long)rows;
    m.row16 = m.col0[m.n];
    const long long total = m.rows * m.row16;
    multi_copy_kernel<<<blocks_for(total), 256, 0, stream>>>(m);
    check_cuda(cudaGetLastError(), what);
    m = MultiCopy{};
  };
  for (const CopyPiece &p : pieces) {
    if (!p.width || !rows) continue;
    if (!aligned(p)) {
      check_cuda(cudaMemcpy2DAsync(p.dst, p.dpitch, p.src, p.spitch, p.width, rows,
                                   cudaMemcpyDeviceToDevice, stream),
                 what);
      continue;
    }
    m.src[m.n] = p.src;
    m.dst[m.n] = p.dst;
    m.spitch[m.n] = (long long)p.spitch;
    m.dpitch[m.n] = (long long)p.dpitch;
    m.col0[m.n + 1] = m.col0[m.n] + (long long)(p.width / 16);
    if (++m.n == kMaxPieces) flush();
  }
  flush();
}

// outer x (extent along dim x inner) blocks: one pitched 2-D copy per input
struct Blocks {
  int64_t outer = 1, inner = 1;
};
Blocks blocks_of(const wgx_tensor *t, int dim) {
  Blocks b;
  for (int i = 0; i < dim; ++i) b.outer *= t->shape[i];
  for (int i = dim + 1; i < t->ndim; ++i) b.inner *= t->shape[i];
  return b;
}

void record_cat(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.cat.default";
  std::vector<wgx_tensor *> ins = tensors_at(a, 0, name);
  int dim = int(num_at(a, 1, name));
  wgx_tensor *out = tensor_at(a, 2, name);
  if (ins.empty()) fail(std::string(name) + ": empty input list");
  const int ndim = out->ndim;
  if (dim < 0) dim += ndim;
  if (dim < 0 || dim >= ndim) fail(std::string(name) + ": dim out of range");
  int64_t total = 0;
  for (auto *t : ins) {
    if (!is_float(t->dtype) || t->dtype != out->dtype)
      fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
    if (t->ndim != ndim) fail(std::string(name) + ": input rank != output rank");
    for (int d = 0; d < ndim; ++d)
      if (d != dim && t->shape[d] != out->shape[d])
        fail(std::string(name) + ": non-concat dim " + std::to_string(d) + " size mismatch");
    total += t->shape[dim];
  }
  if (total != out->shape[dim]) fail(std::string(name) + ": concat dim sizes do not sum to output");
  const int es = dtype_size(out->dtype);
  const Blocks ob = blocks_of(out, dim);
  const size_t dpitch = size_t(out->shape[dim] * ob.inner) * es;
  std::vector<CopyPiece> pieces;
  int64_t off = 0;
  for (auto *t : ins) {
    const size_t width = size_t(t->shape[dim] * ob.inner) * es;
    pieces.push_back({static_cast<const char *>(t->data()),
                      static_cast<char *>(out->data()) + size_t(off * ob.inner) * es, width,
                      dpitch, width});
    off += t->shape[dim];
  }
  const size_t rows = size_t(ob.outer);
  push(ctx, name, 1, [=](const ExecEnv &env) { run_pieces(pieces, rows, env.stream, "cat copy"); });
}

void record_split(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.split_with_sizes_copy.default";
  wgx_tensor *in = tensor_at(a, 0, name);
  std::vector<int64_t> sizes = list_at(a, 1, name);
  int dim = int(num_at(a, 2, name));
  std::vector<wgx_tensor *> outs = tensors_at(a, 3, name);
  const int ndim = in->ndim;
  if (dim < 0) dim += ndim;
  if (dim < 0 || dim >= ndim) fail(std::string(name) + ": dim out of range");
  if (outs.size() != sizes.size())
    fail(std::string(name) + ": outputs (" + std::to_string(outs.size()) + ") != sizes (" +
         std::to_string(sizes.size()) + ")");
  int64_t sum = 0;
  for (auto s : sizes) {
    if (s < 0) fail(std::string(name) + ": negative split size");
    sum += s;
  }
  if (sum != in->shape[dim]) fail(std::string(name) + ": sizes must sum to the split dim extent");
  for (size_t i = 0; i < outs.size(); ++i) {
    if (!is_float(in->dtype) || outs[i]->dtype != in->dtype)
      fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
    if (outs[i]->ndim != ndim || outs[i]->shape[dim] != sizes[i])
      fail(std::string(name) + ": output " + std::to_string(i) + " dim " + std::to_string(dim) +
           " != split size");
  }
  const int es = dtype_size(in->dtype);
  const Blocks ib = blocks_of(in, dim);
  const size_t spitch = size_t(in->shape[dim] * ib.inner) * es;
  std::vector<CopyPiece> pieces;
  int64_t off = 0;
  for (size_t i = 0; i < outs.size(); ++i) {
    const size_t width = size_t(sizes[i] * ib.inner) * es;
    pieces.push_back({static_cast<const char *>(in->data()) + size_t(off * ib.inner) * es,
                      static_cast<char *>(outs[i]->data()), spitch, width, width});
    off += sizes[i];
  }
  const size_t rows = size_t(ib.outer);
  push(ctx, name, 1,
       [=](const ExecEnv &env) { run_pieces(pieces, rows, env.stream, "split copy"); });
}

// -------------------------------------------------------------- permute
struct PermIdx {
  int rank;
  int64_t out_shape[8];
  int64_t in_stride_of_out_dim[8];  // input element stride of output dim d
};

template <class T>
__global__ void permute_kernel(PermIdx p, const T *__restrict__ x, T *__restrict__ y,
                               long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i, src = 0;
    for (int d = p.rank - 1; d >= 0; --d) {
      const long long c = r % p.out_shape[d];
      r /= p.out_shape[d];
      src += c * p.in_stride_of_out_dim[d];
    }
    y[i] = x[src];
  }
}

// y[b][c][r] = x[b][r][c] for an R x C matrix per batch: 32x32 tiles staged
// in shared memory (one padding column against bank conflicts).
template <class T>
__global__ void transpose_kernel(const T *__restrict__ x, T *__restrict__ y, int R, int C) {
  __shared__ T tile[32][33];
  const size_t base = size_t(blockIdx.z) * R * C;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = x[base + size_t(r) * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) y[base + size_t(c) * R + r] = tile[threadIdx.x][i];
  }
}

void record_permute(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.permute_copy.default";
  wgx_tensor *in = tensor_at(a, 0, name);
  std::vector<int64_t> dims = list_at(a, 1, name);
  wgx_tensor *out = tensor_at(a, 2, name);
  require_float_pair(in, out, name);
  const int rank = in->ndim;
  if (out->ndim != rank) fail(std::string(name) + ": output rank != input rank");
  if (int(dims.size()) != rank)
    fail(std::string(name) + ": dims count (" + std::to_string(dims.size()) + ") != input rank (" +
         std::to_string(rank) + ")");
  int perm[8];
  bool seen[8] = {};
  for (int d = 0; d < rank; ++d) {
    int64_t q = dims[d] < 0 ? dims[d] + rank : dims[d];
    if (q < 0 || q >= rank || seen[q]) fail(std::string(name) + ": invalid permute dims");
    seen[q] = true;
    perm[d] = int(q);
  }
  for (int d = 0; d < rank; ++d)
    if (out->shape[d] != in->shape[perm[d]])
      fail(std::string(name) + ": output shape does not match permuted input shape");
  PermIdx p{};
  p.rank = rank;
  int64_t in_stride[8];
  int64_t s = 1;
  for (int d = rank - 1; d >= 0; --d) {
    in_stride[d] = s;
    s *= in->shape[d];
  }
  for (int d = 0; d < rank; ++d) {
    p.out_shape[d] = out->shape[d];
    p.in_stride_of_out_dim[d] = in_stride[perm[d]];
  }
  const void *px = in->data();
  void *py = out->data();
  const long long n = out->numel;
  const int dt = in->dtype;
  // swap of the last two dims with the leading dims in place: a batched
  // transpose through shared-memory tiles (coalesced on both sides)
  bool last_two = rank >= 2 && perm[rank - 1] == rank - 2 && perm[rank - 2] == rank - 1;
  for (int d = 0; d < rank - 2; ++d) last_two = last_two && perm[d] == d;
  if (last_two && n > 0) {
    const long long R = in->shape[rank - 2], C = in->shape[rank - 1];
    const long long batch = n / (R * C);
    if (batch <= 65535 && (R + 31) / 32 <= 65535) {
      const dim3 grid(unsigned((C + 31) / 32), unsigned((R + 31) / 32), unsigned(batch));
      push(ctx, name, 1, [=](const ExecEnv &env) {
        if (dt == WGX_FLOAT16)
          transpose_kernel<__half><<<grid, dim3(32, 8), 0, env.stream>>>(
              (const __half *)px, (__half *)py, int(R), int(C));
        else
          transpose_kernel<float><<<grid, dim3(32, 8), 0, env.stream>>>(
              (const float *)px, (float *)py, int(R), int(C));
        check_cuda(cudaGetLastError(), "permute launch");
      });
      return;
    }
  }
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (dt == WGX_FLOAT16)
      permute_kernel<__half><<<blocks_for(n), 256, 0, env.stream>>>(p, (const __half *)px,
                                                                    (__half *)py, n);
    else
      permute_kernel<float><<<blocks_for(n), 256, 0, env.stream>>>(p, (const float *)px,
                                                                   (float *)py, n);
    check_cuda(cudaGetLastError(), "permute launch");
  });
}

// ------------------------------------------------------------------ bmm
// out[b] = a[b] @ b[b]: 64x64 output tile per CTA, each of the 256 threads
// accumulates a 4x4 block in fp32 over K steps of 16 staged in shared
// memory (A stored k-major so both operands are read as float4).
template <class T>
__global__ void __launch_bounds__(256) bmm_kernel(const T *__restrict__ A, const T *__restrict__ Bm,
                                                  T *__restrict__ C, int M, int N, int K) {
  __shared__ __align__(16) float As[16][64 + 4];  // As[k][m]
  __shared__ __align__(16) float Bs[16][64 + 4];  // Bs[k][n]
  const int bz = blockIdx.z;
  const T *a = A + size_t(bz) * M * K;
  const T *b = Bm + size_t(bz) * K * N;
  T *c = C + size_t(bz) * M * N;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = threadIdx.x + 256 * r;
      const int am = i / 16, ak = i % 16;
      As[ak][am] = (m0 + am < M && k0 + ak < K) ? lf(a[size_t(m0 + am) * K + k0 + ak]) : 0.f;
      const int bk = i / 64, bn = i % 64;
      Bs[bk][bn] = (k0 + bk < K && n0 + bn < N) ? lf(b[size_t(k0 + bk) * N + n0 + bn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float4 av = *reinterpret_cast<const float4 *>(&As[k][ty * 4]);
      const float4 bv = *reinterpret_cast<const float4 *>(&Bs[k][tx * 4]);
      const float ar[4] = {av.x, av.y, av.z, av.w}, br[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) c[size_t(m) * N + n] = sf<T>(acc[i][j]);
    }
  }
}

void record_bmm(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.bmm.default";
  wgx_tensor *A = tensor_at(a, 0, name), *B = tensor_at(a, 1, name), *out = tensor_at(a, 2, name);
  if (!is_float(A->dtype) || B->dtype != A->dtype || out->dtype != A->dtype)
    fail(std::string(name) + ": Tensors must have matching float32 or float16 dtype");
  if (A->ndim != 3 || B->ndim != 3 || out->ndim != 3)
    fail(std::string(name) + ": inputs and output must be 3D");
  const int64_t batch = A->shape[0], m = A->shape[1], k = A->shape[2], n = B->shape[2];
  if (B->shape[0] != batch || B->shape[1] != k)
    fail(std::string(name) + ": batch/K mismatch between a and b");
  if (out->shape[0] != batch || out->shape[1] != m || out->shape[2] != n)
    fail(std::string(name) + ": output shape != [" + std::to_string(batch) + ", " +
         std::to_string(m) + ", " + std::to_string(n) + "]");
  if (batch > 65535 || (m + 63) / 64 > 65535) fail(std::string(name) + ": shape too large");
  const void *pa = A->data(), *pb = B->data();
  void *pc = out->data();
  const int dt = A->dtype;
  if (dt == WGX_FLOAT16 && umma_bmm_supported(batch, m, k, n)) {
    // tcgen05 path: one weight-pack launch and the tensor-core kernel (plus
    // the input re-layout when N % 8 != 0)
    Command c;
    c.name = name;
    c.workspace_bytes = umma_bmm_scratch_bytes(batch, m, k, n);
    c.kernel_launches = n % 8 == 0 ? 2 : 3;
    c.run = [=](const ExecEnv &env) {
      umma_bmm_run(static_cast<const __half *>(pa), static_cast<const __half *>(pb),
                   static_cast<__half *>(pc), batch, m, k, n, env.workspace, env.workspace_bytes,
                   env.stream);
    };
    ctx->commands.push_back(std::move(c));
    return;
  }
  const dim3 grid(unsigned((n + 63) / 64), unsigned((m + 63) / 64), unsigned(batch));
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (dt == WGX_FLOAT16)
      bmm_kernel<__half><<<grid, 256, 0, env.stream>>>((const __half *)pa, (const __half *)pb,
                                                       (__half *)pc, int(m), int(n), int(k));
    else
      bmm_kernel<float><<<grid, 256, 0, env.stream>>>((const float *)pa, (const float *)pb,
                                                      (float *)pc, int(m), int(n), int(k));
    check_cuda(cudaGetLastError(), "bmm launch");
  });
}

// ------------------------------------------------------------- max pool
struct PoolGeom {
  int N, C, IH, IW, OH, OW, kH, kW, sH, sW, pH, pW, dH, dW;
};

template <class T>
__global__ void maxpool_kernel(PoolGeom g, const T *__restrict__ x, T *__restrict__ y,
                               int32_t *__restrict__ idx, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int ow = int(i % g.OW);
    long long t = i / g.OW;
    const int oh = int(t % g.OH);
    const long long plane = t / g.OH;
    const T *xp = x + plane * g.IH * (long long)g.IW;
    // -65504 / -FLT_MAX start and strict '>' like max-pool-2d-f16.wgsl.ts:52-72
    float best = sizeof(T) == 2 ? -65504.0f : -3.402823466e38f;
    int best_idx = 0;
    for (int kh = 0; kh < g.kH; ++kh) {
      const int ih = oh * g.sH - g.pH + kh * g.dH;
      if (ih < 0 || ih >= g.IH) continue;
      for (int kw = 0; kw < g.kW; ++kw) {
        const int iw = ow * g.sW - g.pW + kw * g.dW;
        if (iw < 0 || iw >= g.IW) continue;
        const float v = lf(xp[(long long)ih * g.IW + iw]);
        if (v > best) {
          best = v;
          best_idx = ih * g.IW + iw;
        }
      }
    }
    y[i] = sf<T>(best);
    if (idx) idx[i] = best_idx;
  }
}

// Small planes (IH*IW <= 4096, IH*OW <= 4096): one CTA per plane, separable
// in shared memory. Pass 1 takes, for every input row and output column,
// the maximum over the window's columns and the first column reaching it
// (strict '>', left to right); pass 2 scans the window's rows top to bottom
// over those row maxima with strict '>', so the winner is the first
// maximum in the reference's row-major window order, with the same start
// value and flat index ih*IW + iw as maxpool_kernel.
// Small planes: each block takes `ppb` consecutive planes (ppb * (hw + rw)
// floats + ppb * rw indices of shared memory), so that a block has work for
// all of its threads; the planes are independent.
template <class T>
__global__ void __launch_bounds__(256) maxpool_plane_kernel(PoolGeom g, const T *__restrict__ x,
                                                            T *__restrict__ y,
                                                            int32_t *__restrict__ idx, int ppb,
                                                            long long planes) {
  extern __shared__ __align__(16) unsigned char mp_smem[];
  const int hw = g.IH * g.IW;
  const int rw = g.IH * g.OW;
  const long long plane0 = (long long)blockIdx.x * ppb;
  const int np = int(min((long long)ppb, planes - plane0));
  float *tile = reinterpret_cast<float *>(mp_smem);
  float *rmax = tile + size_t(ppb) * hw;
  int16_t *rarg = reinterpret_cast<int16_t *>(rmax + size_t(ppb) * rw);
  const T *xp = x + plane0 * hw;
  for (int i = threadIdx.x; i < np * hw; i += 256) tile[i] = lf(xp[i]);
  __syncthreads();
  const float start = sizeof(T) == 2 ? -65504.0f : -3.402823466e38f;
  for (int pi = threadIdx.x; pi < np * rw; pi += 256) {
    const int pl = pi / rw, i = pi - pl * rw;
    const int ih = i / g.OW, ow = i - ih * g.OW;
    float best = start;
    int arg = -1;
    for (int kw = 0; kw < g.kW; ++kw) {
      const int iw = ow * g.sW - g.pW + kw * g.dW;
      if (iw < 0 || iw >= g.IW) continue;
      const float v = tile[pl * hw + ih * g.IW + iw];
      if (v > best) {
        best = v;
        arg = iw;
      }
    }
    rmax[pi] = best;
    rarg[pi] = int16_t(arg);
  }
  __syncthreads();
  const int ohw = g.OH * g.OW;
  for (int po = threadIdx.x; po < np * ohw; po += 256) {
    const int pl = po / ohw, o = po - pl * ohw;
    const int oh = o / g.OW, ow = o - oh * g.OW;
    float best = start;
    int best_idx = 0;
    for (int kh = 0; kh < g.kH; ++kh) {
      const int ih = oh * g.sH - g.pH + kh * g.dH;
      if (ih < 0 || ih >= g.IH) continue;
      const float v = rmax[pl * rw + ih * g.OW + ow];
      if (v > best) {
        best = v;
        best_idx = ih * g.IW + rarg[pl * rw + ih * g.OW + ow];
      }
    }
    y[plane0 * ohw + po] = sf<T>(best);
    if (idx) idx[plane0 * ohw + po] = best_idx;
  }
}

// Stride-1, dilation-1, K x K pooling of small planes (compile-time K), in
// the same two passes as maxpool_plane_kernel: row maxima with the first
// maximising column, then a top-to-bottom scan of those with strict '>'
// (the first maximum in (kh, kw) order, as max-pool-2d's shader scans).
// The CTA's `ppb` consecutive planes are staged in shared memory padded by
// (pH, pW) with the start value, which never wins a strict '>', so no tap
// needs a bounds check; threads map to (row, column) pairs of a plane
// (consecutive threads take consecutive columns: coalesced global stores)
// and every output is independent work. Values are compared in fp32 (the
// order of fp16 values is that of their fp32 images). A cascade of o.n
// same-size poolings (the SPPF block: pool(x), pool(pool(x)), ...) runs in
// one launch: each stage's output also replaces the staged tile's interior
// as the next stage's input. IDX = false: no stage writes indices (the
// caller found them unread), so no maximising position is tracked.
template <class T>
struct MpOut {
  T *y[3];
  int32_t *idx[3];
  int n;
};

template <class T, int K, bool IDX>
__global__ void __launch_bounds__(256) maxpool_rows_kernel(PoolGeom g, const T *__restrict__ x,
                                                           MpOut<T> o, int ppb, long long planes) {
  extern __shared__ __align__(16) unsigned char mp_smem[];
  const int IH = g.IH, IW = g.IW, OH = g.OH, OW = g.OW, pH = g.pH, pW = g.pW;
  const int Hp = IH + 2 * pH, Wp = IW + 2 * pW;  // OH = Hp - K + 1, OW = Wp - K + 1
  const long long plane0 = (long long)blockIdx.x * ppb;
  const int np = int(min((long long)ppb, planes - plane0));
  T *tile = reinterpret_cast<T *>(mp_smem);              // [ppb][Hp][Wp]
  T *rmax = tile + size_t(ppb) * Hp * Wp;                 // [ppb][Hp][OW]
  int8_t *rarg = reinterpret_cast<int8_t *>(rmax + size_t(ppb) * Hp * OW);  // [ppb][Hp][OW]
  const float start = sizeof(T) == 2 ? -65504.0f : -3.402823466e38f;
  const T startv = sf<T>(start);
  // padding (and the row-maxima of the pad rows, which never change)
  for (int i = threadIdx.x; i < np * Hp * Wp; i += 256) tile[i] = startv;
  for (int i = threadIdx.x; i < np * Hp * OW; i += 256) rmax[i] = startv;
  __syncthreads();
  // (row, column) mappings of the 256 threads for rows of IW and of OW
  // columns (the host keeps IW, OW <= 256)
  const int ic = threadIdx.x % IW, ir0 = threadIdx.x / IW, irs = 256 / IW;
  const int oc = threadIdx.x % OW, or0 = threadIdx.x / OW, ors = 256 / OW;
  for (int pl = 0; pl < np; ++pl) {
    const T *xp = x + (plane0 + pl) * IH * IW;
    T *tp = tile + (size_t(pl) * Hp + pH) * Wp + pW;
    for (int r = ir0; r < IH && ir0 < irs; r += irs) tp[r * Wp + ic] = xp[r * IW + ic];
  }
  __syncthreads();
  for (int st = 0; st < o.n; ++st) {
    // pass 1: row maxima of the real rows
    if (or0 < ors) {
      for (int pl = 0; pl < np; ++pl) {
#pragma unroll 2
        for (int r = pH + or0; r < pH + IH; r += ors) {
          const T *src = tile + (size_t(pl) * Hp + r) * Wp + oc;
          float best = start;
          int arg = -1;
#pragma unroll
          for (int kw = 0; kw < K; ++kw) {
            const float v = lf(src[kw]);
            if (v > best) {
              best = v;
              if (IDX) arg = kw;
            }
          }
          const size_t ri = (size_t(pl) * Hp + r) * OW + oc;
          rmax[ri] = sf<T>(best);
          if (IDX) rarg[ri] = int8_t(arg);
        }
      }
    }
    __syncthreads();
    // pass 2: column scans of the row maxima
    T *y = o.y[st];
    int32_t *idx = IDX ? o.idx[st] : nullptr;
    const bool next = st + 1 < o.n;  // (same-size poolings: OH = IH, OW = IW)
    if (or0 < ors) {
      for (int pl = 0; pl < np; ++pl) {
        T *yp = y + (plane0 + pl) * OH * OW;
        int32_t *ip = idx ? idx + (plane0 + pl) * OH * OW : nullptr;
#pragma unroll 2
        for (int oh = or0; oh < OH; oh += ors) {
          const T *col = rmax + (size_t(pl) * Hp + oh) * OW + oc;
          float best = start;
          int bk = -1;
#pragma unroll
          for (int kh = 0; kh < K; ++kh) {
            const float v = lf(col[kh * OW]);
            if (v > best) {
              best = v;
              if (IDX) bk = kh;
            }
          }
          const T bv = sf<T>(best);
          yp[oh * OW + oc] = bv;
          if (next) tile[(size_t(pl) * Hp + oh + pH) * Wp + oc + pW] = bv;
          if (IDX && ip) {
            int bi = 0;
            if (bk >= 0) {
              const int ih = oh + bk - pH;
              const int iw = oc + rarg[(size_t(pl) * Hp + oh + bk) * OW + oc] - pW;
              bi = ih * IW + iw;
            }
            ip[oh * OW + oc] = bi;
          }
        }
      }
    }
    __syncthreads();
  }
}

// fp16 form of maxpool_rows_kernel without indices (IW, OW and pW even):
// a thread takes two adjacent output columns as one half2 word. The window
// of output columns 2c, 2c+1 and tap kw is the word at half 2c + kw (even
// kw) or the two halves straddling two words (odd kw, one byte permute);
// each tap is one packed compare (__hgt2_mask, strict '>', false for NaN)
// and a bitwise select, so values and ties resolve exactly as the scalar
// kernel's fp32 compares do. Same shared-memory layout (the index plane is
// left unused).
template <int K>
__global__ void __launch_bounds__(256) maxpool_rows_h2_kernel(PoolGeom g,
                                                              const __half *__restrict__ x,
                                                              MpOut<__half> o, int ppb,
                                                              long long planes) {
  extern __shared__ __align__(16) unsigned char mp_smem[];
  const int IH = g.IH, IW = g.IW, OH = g.OH, OW = g.OW, pH = g.pH;
  const int Hp = IH + 2 * pH, Wp2 = (IW + 2 * g.pW) / 2, OW2 = OW / 2, IW2 = IW / 2;
  const int pW2 = g.pW / 2;
  const long long plane0 = (long long)blockIdx.x * ppb;
  const int np = int(min((long long)ppb, planes - plane0));
  uint32_t *tile = reinterpret_cast<uint32_t *>(mp_smem);  // [ppb][Hp][Wp/2] half pairs
  uint32_t *rmax = tile + size_t(ppb) * Hp * Wp2;          // [ppb][Hp][OW/2]
  constexpr uint32_t kStart = 0xFBFFFBFFu;                 // (-65504, -65504)
  for (int i = threadIdx.x; i < np * Hp * Wp2; i += 256) tile[i] = kStart;
  for (int i = threadIdx.x; i < np * Hp * OW2; i += 256) rmax[i] = kStart;
  __syncthreads();
  const int ic = threadIdx.x % IW2, ir0 = threadIdx.x / IW2, irs = 256 / IW2;
  const int oc = threadIdx.x % OW2, or0 = threadIdx.x / OW2, ors = 256 / OW2;
  for (int pl = 0; pl < np; ++pl) {
    const uint32_t *xp = reinterpret_cast<const uint32_t *>(x + (plane0 + pl) * IH * IW);
    uint32_t *tp = tile + (size_t(pl) * Hp + pH) * Wp2 + pW2;
    for (int r = ir0; r < IH && ir0 < irs; r += irs) tp[r * Wp2 + ic] = xp[r * IW2 + ic];
  }
  __syncthreads();
  auto take = [](uint32_t v, uint32_t best) {
    const uint32_t m = __hgt2_mask(*reinterpret_cast<const __half2 *>(&v),
                                   *reinterpret_cast<const __half2 *>(&best));
    return (v & m) | (best & ~m);
  };
  for (int st = 0; st < o.n; ++st) {
    if (or0 < ors) {
      for (int pl = 0; pl < np; ++pl) {
#pragma unroll 2
        for (int r = pH + or0; r < pH + IH; r += ors) {
          const uint32_t *src = tile + (size_t(pl) * Hp + r) * Wp2 + oc;
          uint32_t w[(K + 1) / 2];
#pragma unroll
          for (int j = 0; j < (K + 1) / 2; ++j) w[j] = src[j];
          uint32_t best = kStart;
#pragma unroll
          for (int kw = 0; kw < K; ++kw)
            best = take((kw & 1) ? __byte_perm(w[kw >> 1], w[(kw >> 1) + 1], 0x5432) : w[kw >> 1],
                        best);
          rmax[(size_t(pl) * Hp + r) * OW2 + oc] = best;
        }
      }
    }
    __syncthreads();
    uint32_t *y = reinterpret_cast<uint32_t *>(o.y[st]);
    const bool next = st + 1 < o.n;  // (same-size poolings: OH = IH, OW = IW)
    if (or0 < ors) {
      for (int pl = 0; pl < np; ++pl) {
        uint32_t *yp = y + (plane0 + pl) * OH * OW2;
#pragma unroll 2
        for (int oh = or0; oh < OH; oh += ors) {
          const uint32_t *col = rmax + (size_t(pl) * Hp + oh) * OW2 + oc;
          uint32_t best = kStart;
#pragma unroll
          for (int kh = 0; kh < K; ++kh) best = take(col[kh * OW2], best);
          yp[oh * OW2 + oc] = best;
          if (next) tile[(size_t(pl) * Hp + oh + pH) * Wp2 + oc + pW2] = best;
        }
      }
    }
    __syncthreads();
  }
}

// Shared memory of one plane for maxpool_rows_kernel.
static size_t mp_rows_plane_bytes(const PoolGeom &g, size_t esz) {
  const size_t Hp = size_t(g.IH) + 2 * g.pH, Wp = size_t(g.IW) + 2 * g.pW;
  return Hp * Wp * esz + Hp * g.OW * esz + Hp * g.OW;
}

void parse_hw(const std::vector<int64_t> &v, const char *name, const char *what, int *h, int *w) {
  if (v.size() == 1) {
    *h = *w = int(v[0]);
  } else if (v.size() == 2) {
    *h = int(v[0]);
    *w = int(v[1]);
  } else {
    fail(std::string(name) + ": " + what + " must be 1 or 2 elements");
  }
}

void record_maxpool(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.max_pool2d_with_indices.default";
  wgx_tensor *in = tensor_at(a, 0, name);
  PoolGeom g{};
  parse_hw(list_at(a, 1, name), name, "kernel_size", &g.kH, &g.kW);
  std::vector<int64_t> st = list_at(a, 2, name);
  if (st.empty()) st = {g.kH, g.kW};  // stride defaults to the kernel size
  parse_hw(st, name, "stride", &g.sH, &g.sW);
  parse_hw(list_at(a, 3, name), name, "padding", &g.pH, &g.pW);
  parse_hw(list_at(a, 4, name), name, "dilation", &g.dH, &g.dW);
  const bool ceil_mode = num_at(a, 5, name) != 0;
  std::vector<wgx_tensor *> outs = tensors_at(a, 6, name);
  if (outs.size() != 2)
    fail(std::string(name) + ": expected 2 outputs [values, indices], got " +
         std::to_string(outs.size()));
  wgx_tensor *vals = outs[0], *idx = outs[1];
  if (!is_float(in->dtype) || vals->dtype != in->dtype)
    fail(std::string(name) + ": values tensors must have matching float32 or float16 dtype");
  if (idx->dtype != WGX_INT32) fail(std::string(name) + ": indices output must be int32");
  if (in->ndim != 4) fail(std::string(name) + ": input must be 4D NCHW");
  g.N = int(in->shape[0]);
  g.C = int(in->shape[1]);
  g.IH = int(in->shape[2]);
  g.IW = int(in->shape[3]);
  const int ohn = g.IH + 2 * g.pH - (g.dH * (g.kH - 1) + 1);
  const int own = g.IW + 2 * g.pW - (g.dW * (g.kW - 1) + 1);
  // max-pool-2d/index.ts:72-75: floor or ceil of the real quotient
  auto div = [&](int num, int s) {
    const double q = double(num) / double(s);
    return int(ceil_mode ? std::ceil(q) : std::floor(q));
  };
  g.OH = std::max(0, div(ohn, g.sH) + 1);
  g.OW = std::max(0, div(own, g.sW) + 1);
  for (auto *t : {vals, idx})
    if (t->ndim != 4 || t->shape[0] != g.N || t->shape[1] != g.C || t->shape[2] != g.OH ||
        t->shape[3] != g.OW)
      fail(std::string(name) + (t == vals ? ": values" : ": indices") + " output shape != [" +
           std::to_string(g.N) + ", " + std::to_string(g.C) + ", " + std::to_string(g.OH) +
           ", " + std::to_string(g.OW) + "]");
  const void *px = in->data();
  void *py = vals->data();
  int32_t *pi = static_cast<int32_t *>(idx->data());
  const long long n = vals->numel;
  const int dt = in->dtype;
  const long long planes = (long long)g.N * g.C;
  const int Kp = g.kH;
  if (g.sH == 1 && g.sW == 1 && g.dH == 1 && g.dW == 1 && g.kW == Kp &&
      (Kp == 3 || Kp == 5 || Kp == 7) && (long long)g.IH * g.IW <= 4096 &&
      (long long)g.IH * g.OW <= 4096 && g.IW <= 256 && g.OW <= 256 && g.OW >= 1 &&
      g.OH >= 1 && planes > 0 && planes < (1ll << 31)) {
    // about 40 KB of planes per block
    const size_t esz = dt == WGX_FLOAT16 ? 2 : 4;
    const size_t per_plane = mp_rows_plane_bytes(g, esz);
    const int ppb = int(std::max<size_t>(1, std::min<size_t>(64, 40 * 1024 / per_plane)));
    const size_t smem = per_plane * ppb + 16;
    if (smem > 48 * 1024) fail(std::string(name) + ": plane too large for the tiled kernel");
    const long long blocks = (planes + ppb - 1) / ppb;
    push(ctx, name, 1, [=](const ExecEnv &env) {
#define WGX_MP_ROWS(TT, KK)                                                             \
  maxpool_rows_kernel<TT, KK, true><<<unsigned(blocks), 256, smem, env.stream>>>(        \
      g, (const TT *)px, MpOut<TT>{{(TT *)py, nullptr, nullptr}, {pi, nullptr, nullptr}, 1}, \
      ppb, planes)
      if (dt == WGX_FLOAT16) {
        if (Kp == 3) WGX_MP_ROWS(__half, 3);
        else if (Kp == 5) WGX_MP_ROWS(__half, 5);
        else WGX_MP_ROWS(__half, 7);
      } else {
        if (Kp == 3) WGX_MP_ROWS(float, 3);
        else if (Kp == 5) WGX_MP_ROWS(float, 5);
        else WGX_MP_ROWS(float, 7);
      }
#undef WGX_MP_ROWS
      check_cuda(cudaGetLastError(), "maxpool launch");
    });
    return;
  }
  if ((long long)g.IH * g.IW <= 4096 && (long long)g.IH * g.OW <= 4096 && g.IW <= 32767 &&
      planes > 0 && planes < (1ll << 31)) {
    // planes per block: about 1024 input elements per block, within 40 KB
    const size_t per_plane = (size_t(g.IH) * g.IW + size_t(g.IH) * g.OW) * 4 +
                             size_t(g.IH) * g.OW * 2;
    int ppb = int(std::max<long long>(1, 1024 / ((long long)g.IH * g.IW)));
    ppb = int(std::min<size_t>(size_t(ppb), std::max<size_t>(1, 40 * 1024 / per_plane)));
    const size_t smem = per_plane * ppb + 16;
    const long long blocks = (planes + ppb - 1) / ppb;
    push(ctx, name, 1, [=](const ExecEnv &env) {
      if (dt == WGX_FLOAT16)
        maxpool_plane_kernel<__half><<<unsigned(blocks), 256, smem, env.stream>>>(
            g, (const __half *)px, (__half *)py, pi, ppb, planes);
      else
        maxpool_plane_kernel<float><<<unsigned(blocks), 256, smem, env.stream>>>(
            g, (const float *)px, (float *)py, pi, ppb, planes);
      check_cuda(cudaGetLastError(), "maxpool launch");
    });
    return;
  }
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (dt == WGX_FLOAT16)
      maxpool_kernel<__half><<<blocks_for(n), 256, 0, env.stream>>>(g, (const __half *)px,
                                                                    (__half *)py, pi, n);
    else
      maxpool_kernel<float><<<blocks_for(n), 256, 0, env.stream>>>(g, (const float *)px,
                                                                   (float *)py, pi, n);
    check_cuda(cudaGetLastError(), "maxpool launch");
  });
}

// -------------------------------------------------------------- softmax
// One warp per (outer, inner) line of length R: max, sum of exp, normalise.
template <class T>
__global__ void softmax_kernel(const T *__restrict__ x, T *__restrict__ y, long long lines, int R,
                               long long inner) {
  const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= lines) return;
  const long long o = warp / inner, in = warp % inner;
  const T *xp = x + o * R * inner + in;
  T *yp = y + o * R * inner + in;
  float mx = -INFINITY;
  for (int r = lane; r < R; r += 32) mx = fmaxf(mx, lf(xp[r * inner]));
  for (int s = 16; s > 0; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
  float sum = 0.f;
  for (int r = lane; r < R; r += 32) sum += __expf(lf(xp[r * inner]) - mx);
  for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
  const float inv = 1.0f / sum;
  for (int r = lane; r < R; r += 32) yp[r * inner] = sf<T>(__expf(lf(xp[r * inner]) - mx) * inv);
}

void record_softmax(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten._softmax.default";
  wgx_tensor *in = tensor_at(a, 0, name);
  int dim = int(num_at(a, 1, name));
  wgx_tensor *out = tensor_at(a, 3, name);
  require_float_pair(in, out, name);
  if (in->ndim == 0) fail(std::string(name) + ": scalar input unsupported");
  if (in->numel != out->numel) fail(std::string(name) + ": input/output numel mismatch");
  if (dim < 0) dim += in->ndim;
  if (dim < 0 || dim >= in->ndim) fail(std::string(name) + ": dim out of range");
  int64_t outer = 1, inner = 1;
  for (int i = 0; i < dim; ++i) outer *= in->shape[i];
  for (int i = dim + 1; i < in->ndim; ++i) inner *= in->shape[i];
  const int R = int(in->shape[dim]);
  if (outer == 0 || R == 0 || inner == 0) fail(std::string(name) + ": zero-sized reduction");
  const void *px = in->data();
  void *py = out->data();
  const long long lines = outer * inner;
  const int dt = in->dtype;
  const unsigned blocks = unsigned((lines * 32 + 255) / 256);
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (dt == WGX_FLOAT16)
      softmax_kernel<__half><<<blocks, 256, 0, env.stream>>>((const __half *)px, (__half *)py,
                                                             lines, R, inner);
    else
      softmax_kernel<float><<<blocks, 256, 0, env.stream>>>((const float *)px, (float *)py, lines,
                                                            R, inner);
    check_cuda(cudaGetLastError(), "softmax launch");
  });
}

// ------------------------------------------------------------ resampling
struct Resample {
  int N, C, IH, IW, OH, OW, align;
};

template <class T>
__global__ void nearest_kernel(Resample r, const T *__restrict__ x, T *__restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int ow = int(i % r.OW);
    long long t = i / r.OW;
    const int oh = int(t % r.OH);
    const long long plane = t / r.OH;
    // source index (dst * in) / out, upsample-nearest-2d-f16.wgsl.ts:40-42
    const int ih = int((long long)oh * r.IH / r.OH), iw = int((long long)ow * r.IW / r.OW);
    y[i] = x[(plane * r.IH + ih) * r.IW + iw];
  }
}

__device__ __forceinline__ float src_index(int dst, int insz, int outsz, int align) {
  if (align) return outsz <= 1 ? 0.f : float(dst) * float(insz - 1) / float(outsz - 1);
  return (float(dst) + 0.5f) * float(insz) / float(outsz) - 0.5f;
}

template <class T>
__global__ void bilinear_kernel(Resample r, const T *__restrict__ x, T *__restrict__ y,
                                long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int ow = int(i % r.OW);
    long long t = i / r.OW;
    const int oh = int(t % r.OH);
    const long long plane = t / r.OH;
    // upsample-bilinear2d-f16.wgsl.ts:28-77 (interpolation here in fp32)
    const float sh = src_index(oh, r.IH, r.OH, r.align), sw = src_index(ow, r.IW, r.OW, r.align);
    const int h0 = int(floorf(sh)), w0 = int(floorf(sw));
    const float lh = sh - float(h0), lw = sw - float(w0);
    const int h0c = min(max(h0, 0), r.IH - 1), h1c = min(max(h0 + 1, 0), r.IH - 1);
    const int w0c = min(max(w0, 0), r.IW - 1), w1c = min(max(w0 + 1, 0), r.IW - 1);
    const T *p = x + plane * r.IH * (long long)r.IW;
    const float v00 = lf(p[h0c * (long long)r.IW + w0c]), v01 = lf(p[h0c * (long long)r.IW + w1c]);
    const float v10 = lf(p[h1c * (long long)r.IW + w0c]), v11 = lf(p[h1c * (long long)r.IW + w1c]);
    const float top = v00 + (v01 - v00) * lw, bot = v10 + (v11 - v10) * lw;
    y[i] = sf<T>(top + (bot - top) * lh);
  }
}

// Bilinear, fp16, OW % 8 == 0, 32-bit index range: each thread writes 8
// consecutive outputs of one output row with one 16-byte store. The CTA
// first tabulates every output column's source columns and weight in shared
// memory (one fp32 division per column instead of per output); the row's
// source rows and weight (h0, h1, lh) are computed once per thread. Same
// fp32 arithmetic as bilinear_kernel (identical results); thread -> (row,
// group) by one 32-bit division.
struct BilinCol {
  int16_t w0, w1;
  float lw;
};
__global__ void __launch_bounds__(256) bilinear_v8_kernel(Resample r, const __half *__restrict__ x,
                                                          uint4 *__restrict__ y, int n8) {
  extern __shared__ BilinCol bcol[];
  for (int ow = threadIdx.x; ow < r.OW; ow += 256) {
    const float sw = src_index(ow, r.IW, r.OW, r.align);
    const int w0 = int(floorf(sw));
    bcol[ow] = BilinCol{int16_t(min(max(w0, 0), r.IW - 1)), int16_t(min(max(w0 + 1, 0), r.IW - 1)),
                        sw - float(w0)};
  }
  __syncthreads();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= n8) return;
  const int ow8 = r.OW / 8;
  const int row = i / ow8, g = i - row * ow8;
  const int plane = row / r.OH, oh = row - plane * r.OH;
  const float sh = src_index(oh, r.IH, r.OH, r.align);
  const int h0 = int(floorf(sh));
  const float lh = sh - float(h0);
  const int h0c = min(max(h0, 0), r.IH - 1), h1c = min(max(h0 + 1, 0), r.IH - 1);
  const __half *p0 = x + (size_t(plane) * r.IH + h0c) * r.IW;
  const __half *p1 = x + (size_t(plane) * r.IH + h1c) * r.IW;
  __align__(16) __half v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const BilinCol cc = bcol[8 * g + k];
    const float lw = cc.lw;
    const float v00 = __half2float(__ldg(p0 + cc.w0)), v01 = __half2float(__ldg(p0 + cc.w1));
    const float v10 = __half2float(__ldg(p1 + cc.w0)), v11 = __half2float(__ldg(p1 + cc.w1));
    const float top = v00 + (v01 - v00) * lw, bot = v10 + (v11 - v10) * lw;
    v[k] = __float2half_rn(top + (bot - top) * lh);
  }
  y[i] = *reinterpret_cast<const uint4 *>(v);
}

// fp16, OW % 8 == 0: each thread writes 8 consecutive outputs of one row
// with one 16-byte store (the 8 source reads hit the same cache lines).
__global__ void nearest_v8_kernel(Resample r, const __half *__restrict__ x, uint4 *__restrict__ y,
                                  long long n8) {
  const int ow8 = r.OW / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const int g = int(i % ow8);
    const long long t = i / ow8;
    const int oh = int(t % r.OH);
    const long long plane = t / r.OH;
    const int ih = int((long long)oh * r.IH / r.OH);
    const __half *row = x + (plane * r.IH + ih) * r.IW;
    __align__(16) __half v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = row[int((long long)(8 * g + k) * r.IW / r.OW)];
    y[i] = *reinterpret_cast<const uint4 *>(v);
  }
}

// Integer scale: OW = 2*IW, OH = sH*IH (the 2x upsample of detection necks).
// One thread reads 4 input values (8 bytes) of input row `row` and writes
// the 8 duplicated values (16 bytes) into each of the sH output rows
// row*sH .. row*sH + sH - 1 (output row of (plane, ih*sH + k) =
// (plane*IH + ih)*sH + k); 32-bit indices (checked by the host).
__global__ void nearest_x2_kernel(const uint2 *__restrict__ x, uint4 *__restrict__ y, int ow8,
                                  int sH, int n_items) {
  const int item = blockIdx.x * blockDim.x + threadIdx.x;
  if (item >= n_items) return;
  const int row = item / ow8, g = item - row * ow8;
  const uint2 v = x[item];  // input row `row`, columns 4g .. 4g + 3
  const uint4 o = make_uint4(__byte_perm(v.x, 0, 0x1010), __byte_perm(v.x, 0, 0x3232),
                             __byte_perm(v.y, 0, 0x1010), __byte_perm(v.y, 0, 0x3232));
  for (int k = 0; k < sH; ++k) y[(size_t(row) * sH + k) * ow8 + g] = o;
}

void record_nearest(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.upsample_nearest2d.vec";
  wgx_tensor *in = tensor_at(a, 0, name), *out = tensor_at(a, 3, name);
  require_float_pair(in, out, name);
  if (in->ndim != 4 || out->ndim != 4) fail(std::string(name) + ": input and output must be 4D NCHW");
  if (out->shape[0] != in->shape[0] || out->shape[1] != in->shape[1])
    fail(std::string(name) + ": output batch/channels must match input");
  if (out->shape[2] < in->shape[2] || out->shape[3] < in->shape[3])
    fail(std::string(name) + ": output spatial dims must be >= input spatial dims");
  Resample r{int(in->shape[0]), int(in->shape[1]), int(in->shape[2]), int(in->shape[3]),
             int(out->shape[2]), int(out->shape[3]), 0};
  const void *px = in->data();
  void *py = out->data();
  const long long n = out->numel;
  const int dt = in->dtype;
  const long long in_rows = (long long)r.N * r.C * r.IH;
  if (dt == WGX_FLOAT16 && r.OW == 2 * r.IW && r.OH % r.IH == 0 && r.IW % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(py) & 15) == 0 && (reinterpret_cast<uintptr_t>(px) & 7) == 0 &&
      in_rows * (r.OW / 8) < (1ll << 31)) {
    const int ow8 = r.OW / 8, sH = r.OH / r.IH;
    const int n_items = int(in_rows * ow8);
    push(ctx, name, 1, [=](const ExecEnv &env) {
      nearest_x2_kernel<<<unsigned((n_items + 255) / 256), 256, 0, env.stream>>>(
          (const uint2 *)px, (uint4 *)py, ow8, sH, n_items);
      check_cuda(cudaGetLastError(), "upsample launch");
    });
    return;
  }
  if (dt == WGX_FLOAT16 && r.OW % 8 == 0 && (reinterpret_cast<uintptr_t>(py) & 15) == 0) {
    const long long n8 = n / 8;
    push(ctx, name, 1, [=](const ExecEnv &env) {
      nearest_v8_kernel<<<blocks_for(n8), 256, 0, env.stream>>>(r, (const __half *)px,
                                                                (uint4 *)py, n8);
      check_cuda(cudaGetLastError(), "upsample launch");
    });
    return;
  }
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (dt == WGX_FLOAT16)
      nearest_kernel<__half><<<blocks_for(n), 256, 0, env.stream>>>(r, (const __half *)px,
                                                                    (__half *)py, n);
    else
      nearest_kernel<float><<<blocks_for(n), 256, 0, env.stream>>>(r, (const float *)px,
                                                                   (float *)py, n);
    check_cuda(cudaGetLastError(), "upsample launch");
  });
}

void record_bilinear(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.upsample_bilinear2d.vec";
  wgx_tensor *in = tensor_at(a, 0, name), *out = tensor_at(a, 4, name);
  const bool align = num_at(a, 2, name) != 0;
  require_float_pair(in, out, name);
  if (in->ndim != 4 || out->ndim != 4) fail(std::string(name) + ": expected 4D in/out tensors");
  if (out->shape[0] != in->shape[0] || out->shape[1] != in->shape[1])
    fail(std::string(name) + ": N/C mismatch");
  Resample r{int(in->shape[0]), int(in->shape[1]), int(in->shape[2]), int(in->shape[3]),
             int(out->shape[2]), int(out->shape[3]), align ? 1 : 0};
  const void *px = in->data();
  void *py = out->data();
  const long long n = out->numel;
  const int dt = in->dtype;
  // (the column table: 8 bytes per output column in shared memory; int16
  // source columns)
  const bool v8 = dt == WGX_FLOAT16 && r.OW % 8 == 0 && n / 8 < (1ll << 31) - 256 &&
                  (reinterpret_cast<uintptr_t>(py) & 15) == 0 &&
                  (long long)r.N * r.C * r.OH < (1ll << 31) && r.OW <= 6144 && r.IW <= 32767;
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (v8) {
      const int n8 = int(n / 8);
      bilinear_v8_kernel<<<unsigned((n8 + 255) / 256), 256, size_t(r.OW) * sizeof(BilinCol),
                           env.stream>>>(r, (const __half *)px, (uint4 *)py, n8);
    } else if (dt == WGX_FLOAT16)
      bilinear_kernel<__half><<<blocks_for(n), 256, 0, env.stream>>>(r, (const __half *)px,
                                                                     (__half *)py, n);
    else
      bilinear_kernel<float><<<blocks_for(n), 256, 0, env.stream>>>(r, (const float *)px,
                                                                    (float *)py, n);
    check_cuda(cudaGetLastError(), "upsample launch");
  });
}

// ---------------------------------------------------------- mean.dim
template <class T>
__global__ void mean_kernel(const T *__restrict__ x, T *__restrict__ y, long long lines, long long R,
                            long long inner) {
  const long long warp = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= lines) return;
  const long long o = warp / inner, in = warp % inner;
  const T *xp = x + o * R * inner + in;
  float sum = 0.f;
  for (long long r = lane; r < R; r += 32) sum += lf(xp[r * inner]);
  for (int s = 16; s > 0; s >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, s);
  if (lane == 0) y[warp] = sf<T>(sum / float(R));
}

void record_mean(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.mean.dim";
  wgx_tensor *in = tensor_at(a, 0, name), *out = tensor_at(a, 4, name);
  std::vector<int64_t> dims = list_at(a, 1, name);
  const int nd = in->ndim;
  if (nd == 0 || dims.empty()) fail(std::string(name) + ": dim out of range");
  for (auto &d : dims) {
    if (d < 0) d += nd;
    if (d < 0 || d >= nd) fail(std::string(name) + ": dim out of range");
  }
  std::sort(dims.begin(), dims.end());
  for (size_t i = 1; i < dims.size(); ++i) {
    if (dims[i] == dims[i - 1]) fail(std::string(name) + ": duplicate reduced dim");
    if (dims[i] != dims[i - 1] + 1) fail(std::string(name) + ": only contiguous reduced dims supported");
  }
  require_float_pair(in, out, name);
  int64_t outer = 1, R = 1, inner = 1;
  for (int i = 0; i < dims.front(); ++i) outer *= in->shape[i];
  for (int64_t i = dims.front(); i <= dims.back(); ++i) R *= in->shape[i];
  for (int i = int(dims.back()) + 1; i < nd; ++i) inner *= in->shape[i];
  if (R == 0) fail(std::string(name) + ": zero-sized reduction");
  if (outer * inner != out->numel) fail(std::string(name) + ": output numel mismatch");
  const void *px = in->data();
  void *py = out->data();
  const long long lines = outer * inner;
  const int dt = in->dtype;
  const unsigned blocks = unsigned((lines * 32 + 255) / 256);
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (dt == WGX_FLOAT16)
      mean_kernel<__half><<<blocks, 256, 0, env.stream>>>((const __half *)px, (__half *)py, lines,
                                                          R, inner);
    else
      mean_kernel<float><<<blocks, 256, 0, env.stream>>>((const float *)px, (float *)py, lines, R,
                                                         inner);
    check_cuda(cudaGetLastError(), "mean launch");
  });
}

// ------------------------------------------------------ constant_pad_nd
struct Pad4 {
  int64_t in[4], out[4], left[4];
  float value;
};

template <class T>
__global__ void pad_kernel(Pad4 p, const T *__restrict__ x, T *__restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    long long r = i, src = 0, stride = 1;
    bool inside = true;
    for (int d = 3; d >= 0; --d) {
      const long long c = r % p.out[d] - p.left[d];
      r /= p.out[d];
      if (c < 0 || c >= p.in[d]) inside = false;
      src += c * stride;
      stride *= p.in[d];
    }
    y[i] = inside ? x[src] : sf<T>(p.value);
  }
}

void record_pad(wgx_context *ctx, const std::vector<wgx_arg> &a) {
  const char *name = "aten.constant_pad_nd.default";
  wgx_tensor *in = tensor_at(a, 0, name);
  std::vector<int64_t> pad = list_at(a, 1, name);
  double value = 0.0;
  wgx_tensor *out;
  if (a.size() == 4) {
    value = num_at(a, 2, name);
    out = tensor_at(a, 3, name);
  } else {
    out = tensor_at(a, 2, name);
  }
  require_float_pair(in, out, name);
  const int nd = in->ndim;
  if (nd == 0 || nd > 4) fail(std::string(name) + ": rank must be 1..4 (got " + std::to_string(nd) + ")");
  if (out->ndim != nd)
    fail(std::string(name) + ": in/out rank mismatch (" + std::to_string(nd) + " !== " +
         std::to_string(out->ndim) + ")");
  if (pad.size() % 2) fail(std::string(name) + ": pad must be even-length");
  const int npad = int(pad.size() / 2);
  if (npad > nd) fail(std::string(name) + ": pad longer than rank");
  Pad4 p{};
  int64_t left[4] = {0, 0, 0, 0}, right[4] = {0, 0, 0, 0};
  for (int k = 0; k < npad; ++k) {
    left[nd - 1 - k] = pad[2 * k];
    right[nd - 1 - k] = pad[2 * k + 1];
  }
  for (int d = 0; d < nd; ++d) {
    if (left[d] < 0 || right[d] < 0) fail(std::string(name) + ": negative pad (cropping) not supported");
    const int64_t e = in->shape[d] + left[d] + right[d];
    if (out->shape[d] != e)
      fail(std::string(name) + ": output dim " + std::to_string(d) + " mismatch (" +
           std::to_string(e) + " != " + std::to_string(out->shape[d]) + ")");
  }
  for (int d = 0; d < 4; ++d) {  // right-align into 4-D
    const int sd = d - (4 - nd);
    p.in[d] = sd >= 0 ? in->shape[sd] : 1;
    p.out[d] = sd >= 0 ? out->shape[sd] : 1;
    p.left[d] = sd >= 0 ? left[sd] : 0;
  }
  p.value = float(value);
  const void *px = in->data();
  void *py = out->data();
  const long long n = out->numel;
  const int dt = in->dtype;
  push(ctx, name, 1, [=](const ExecEnv &env) {
    if (dt == WGX_FLOAT16)
      pad_kernel<__half><<<blocks_for(n), 256, 0, env.stream>>>(p, (const __half *)px,
                                                                (__half *)py, n);
    else
      pad_kernel<float><<<blocks_for(n), 256, 0, env.stream>>>(p, (const float *)px, (float *)py,
                                                               n);
    check_cuda(cudaGetLastError(), "pad launch");
  });
}

}  // namespace

// A cascade of 2 or 3 same-size max-pools (stride 1, dilation 1, K x K with
// K in {3, 5, 7}, padding (K-1)/2), each reading the previous one's values
// (the SPPF block): one launch of maxpool_rows_kernel that writes every
// stage's values and indices. An index tensor given as null is one that no
// later operator reads and that is no program output: it is not written
// (with all of them null, no maximising position is tracked). False
// (nothing recorded) when the shapes do not qualify; the caller then
// records the operators one by one.
bool record_maxpool_cascade(wgx_context *ctx, wgx_tensor *in,
                            const std::vector<std::pair<wgx_tensor *, wgx_tensor *>> &outs, int K) {
  const int n = int(outs.size());
  if (n < 2 || n > 3 || (K != 3 && K != 5 && K != 7)) return false;
  if (in->ndim != 4 || (in->dtype != WGX_FLOAT16 && in->dtype != WGX_FLOAT32)) return false;
  bool any_idx = false;
  for (auto &o : outs) {
    const wgx_tensor *v = o.first, *ix = o.second;
    if (v->dtype != in->dtype || v->ndim != 4) return false;
    if (ix && (ix->dtype != WGX_INT32 || ix->ndim != 4)) return false;
    for (int d = 0; d < 4; ++d)
      if (v->shape[d] != in->shape[d] || (ix && ix->shape[d] != in->shape[d])) return false;
    any_idx = any_idx || ix != nullptr;
  }
  PoolGeom g{};
  g.N = int(in->shape[0]);
  g.C = int(in->shape[1]);
  g.IH = g.OH = int(in->shape[2]);
  g.IW = g.OW = int(in->shape[3]);
  g.kH = g.kW = K;
  g.sH = g.sW = g.dH = g.dW = 1;
  g.pH = g.pW = (K - 1) / 2;
  const long long planes = (long long)g.N * g.C;
  if ((long long)g.IH * g.IW > 4096 || g.IW > 256 || planes <= 0 || planes >= (1ll << 31))
    return false;
  const size_t esz = in->dtype == WGX_FLOAT16 ? 2 : 4;
  const size_t per_plane = mp_rows_plane_bytes(g, esz);
  const int ppb = int(std::max<size_t>(1, std::min<size_t>(64, 40 * 1024 / per_plane)));
  const size_t smem = per_plane * ppb + 16;
  if (smem > 48 * 1024) return false;
  const long long blocks = (planes + ppb - 1) / ppb;
  const void *px = in->data();
  void *py[3] = {}, *pi[3] = {};
  for (int k = 0; k < n; ++k) {
    py[k] = outs[k].first->data();
    pi[k] = outs[k].second ? outs[k].second->data() : nullptr;
  }
  const int dt = in->dtype;
  // packed fp16 form: no indices, even widths and padding, 4-byte aligned planes
  bool h2 = dt == WGX_FLOAT16 && !any_idx && g.IW % 2 == 0 && g.pW % 2 == 0 &&
            g.IW / 2 <= 256 && (reinterpret_cast<uintptr_t>(px) & 3) == 0;
  for (int k = 0; k < n; ++k) h2 = h2 && (reinterpret_cast<uintptr_t>(py[k]) & 3) == 0;
  std::string name = "aten.max_pool2d_with_indices.default x" + std::to_string(n) + " (cascade)";
  Command c;
  c.name = name;
  c.kernel_launches = 1;
  c.run = [=](const ExecEnv &env) {
#define WGX_MP_CASCADE(TT, KK, ID)                                                          \
  maxpool_rows_kernel<TT, KK, ID><<<unsigned(blocks), 256, smem, env.stream>>>(             \
      g, (const TT *)px,                                                                    \
      MpOut<TT>{{(TT *)py[0], (TT *)py[1], (TT *)py[2]},                                   \
                {(int32_t *)pi[0], (int32_t *)pi[1], (int32_t *)pi[2]}, n},                 \
      ppb, planes)
    if (h2) {
      const MpOut<__half> mo{{(__half *)py[0], (__half *)py[1], (__half *)py[2]},
                             {nullptr, nullptr, nullptr}, n};
      if (K == 3)
        maxpool_rows_h2_kernel<3><<<unsigned(blocks), 256, smem, env.stream>>>(
            g, (const __half *)px, mo, ppb, planes);
      else if (K == 5)
        maxpool_rows_h2_kernel<5><<<unsigned(blocks), 256, smem, env.stream>>>(
            g, (const __half *)px, mo, ppb, planes);
      else
        maxpool_rows_h2_kernel<7><<<unsigned(blocks), 256, smem, env.stream>>>(
            g, (const __half *)px, mo, ppb, planes);
    } else if (dt == WGX_FLOAT16) {
      if (any_idx) {
        if (K == 3) WGX_MP_CASCADE(__half, 3, true);
        else if (K == 5) WGX_MP_CASCADE(__half, 5, true);
        else WGX_MP_CASCADE(__half, 7, true);
      } else {
        if (K == 3) WGX_MP_CASCADE(__half, 3, false);
        else if (K == 5) WGX_MP_CASCADE(__half, 5, false);
        else WGX_MP_CASCADE(__half, 7, false);
      }
    } else {
      if (K == 3) WGX_MP_CASCADE(float, 3, true);
      else if (K == 5) WGX_MP_CASCADE(float, 5, true);
      else WGX_MP_CASCADE(float, 7, true);
    }
#undef WGX_MP_CASCADE
    check_cuda(cudaGetLastError(), "maxpool launch");
  };
  ctx->commands.push_back(std::move(c));
  return true;
}

void register_data_ops(std::unordered_map<std::string, OpRecorder> &r) {
  auto flat = [](const char *name) {
    return [name](wgx_context *c, const std::vector<wgx_arg> &a) {
      record_flat_copy(c, a, name, 0, a.size() - 1);
    };
  };
  r["aten.view_copy.default"] = flat("aten.view_copy.default");
  r["aten.clone.default"] = flat("aten.clone.default");
  r["aten.squeeze_copy.dims"] = flat("aten.squeeze_copy.dims");
  r["aten.unsqueeze_copy.default"] = flat("aten.unsqueeze_copy.default");
  r["et_vk.prepack.default"] = flat("et_vk.prepack.default");
  r["aten.cat.default"] = record_cat;
  r["aten.split_with_sizes_copy.default"] = record_split;
  r["aten.permute_copy.default"] = record_permute;
  r["aten.bmm.default"] = record_bmm;
  r["aten.max_pool2d_with_indices.default"] = record_maxpool;
  r["aten._softmax.default"] = record_softmax;
  r["aten.upsample_nearest2d.vec"] = record_nearest;
  r["aten.upsample_bilinear2d.vec"] = record_bilinear;
  r["aten.mean.dim"] = record_mean;
  r["aten.constant_pad_nd.default"] = record_pad;
}

}  // namespace wgx
