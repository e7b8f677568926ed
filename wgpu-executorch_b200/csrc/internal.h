// Internal declarations shared by the runtime, the operator registry and the
// kernels. Nothing here is part of the C ABI (that is include/wgx.h).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "wgx.h"

namespace wgx {

// ---------------------------------------------------------------- errors
// Thread-local last-error text (wgx_last_error). set_error returns its code
// so call sites can write `return set_error(...)`.
int set_error(int code, const std::string &msg);
void clear_error();

struct Error {
  int code;
  std::string msg;
};
// Validation helper used by the op recorders: throws Error, which the C ABI
// entry points catch and turn into a status code + message.
[[noreturn]] void fail(const std::string &msg, int code = WGX_ERR_INVALID);
void check_cuda(cudaError_t e, const char *what);

int dtype_size(int dtype);
const char *dtype_name(int dtype);

// Device-side error word. Kernels that wait on a barrier give up after a
// bounded number of polls and OR a code in here instead of hanging.
enum DeviceErrorBits : uint32_t {
  kErrMmaTimeout = 1u << 0,
  kErrLoadTimeout = 1u << 1,
  kErrEpilogueTimeout = 1u << 2,
  kErrTmemAlloc = 1u << 3,
  kErrBounds = 1u << 4,  // bounds-checking build: an access outside its buffer was skipped
};

// Bounds-checking debug build (-DWGX_BOUNDS; `make bounds` builds
// lib/libwgx_bounds.so). The hot-path kernels check their global accesses
// against the extent of the buffer they belong to; an access outside it is
// skipped and kErrBounds is set in the device error word, so the next sync()
// fails with WGX_ERR_DEVICE instead of the kernel writing (or reading) out of
// bounds. compute-sanitizer is closed on this pool; this build and the
// odd-shape parity tests stand in for it. In the normal build the checks
// compile to nothing.
#ifdef WGX_BOUNDS
__device__ __forceinline__ bool bounds_ok(const void *p, uint64_t n, const void *base,
                                          uint64_t extent, uint32_t *err) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p), b = reinterpret_cast<uintptr_t>(base);
  if (base != nullptr && a >= b && a + n <= b + extent) return true;
  if (err) atomicOr(err, kErrBounds);
  return false;
}
#define WGX_IN_BOUNDS(p, n, base, extent, err) ::wgx::bounds_ok((p), (n), (base), (extent), (err))
#else
#define WGX_IN_BOUNDS(p, n, base, extent, err) true
#endif
uint32_t *device_error_word(int device);

// Device allocations of the library go through device_malloc, which
// honours the test-only fault injection of wgx_debug_inject
// (WGX_INJECT_ALLOC_FAIL fails the next one with cudaErrorMemoryAllocation).
cudaError_t device_malloc(void **p, uint64_t bytes);
// WGX_INJECT_SKIP_LOADS is set: tensor-core kernels launched now issue no
// copies, so their bounded waits run out (failure-detection tests).
bool inject_skip_loads();

// Opt-in CUDA-event timing of individual kernels (wgx_kernel_timing). Both
// are no-ops unless timing is enabled and the stream is not capturing.
int timer_begin(const char *kernel, cudaStream_t stream);
void timer_end(int handle, cudaStream_t stream);

// ------------------------------------------------------------- objects
struct Arena;

}  // namespace wgx

struct wgx_buffer {
  wgx_context *ctx = nullptr;  // owner (null: external buffer)
  void *dptr = nullptr;
  uint64_t size = 0;
  uint32_t usage = 0;
  int device = 0;
  bool owns_alloc = false;  // cudaFree(dptr) on destroy
  bool destroyed = false;
  bool constant = false;    // holds program weights (immutable after upload)
};

struct wgx_tensor {
  wgx_buffer *buffer = nullptr;
  int dtype = 0;
  int ndim = 0;
  int64_t shape[WGX_MAX_NDIM] = {0};
  int64_t numel = 1;
  uint64_t byte_length() const { return uint64_t(numel) * wgx::dtype_size(dtype); }
  void *data() const { return buffer->dptr; }
};

namespace wgx {

// Execution environment handed to every recorded command when it is
// replayed (inside stream capture on the first submit).
struct ExecEnv {
  cudaStream_t stream;
  void *workspace;        // shared scratch, sized to the max any command asked for
  uint64_t workspace_bytes;
};

struct Command {
  std::string name;
  int kernel_launches = 0;
  uint64_t workspace_bytes = 0;  // shared scratch this command needs
  std::function<void(const ExecEnv &)> run;  // throws Error on failure
};

// Program-level connections of the convolution being recorded, set by the
// program recorder around that one recording call (null otherwise).
struct ConvRecordLink {
  // write the output into this buffer: the re-laid input of `consumer`
  void *out_xs = nullptr;
  wgx_conv2d_params consumer{};
  // the input has already been re-laid into this buffer by its producer
  void *in_xs = nullptr;
  // the input is the channel concatenation of these tensors
  std::vector<wgx_tensor *> cat;
  // NCHW output: add this tensor (same shape) after the activation
  const wgx_tensor *resid = nullptr;
  // NCHW output split along channels into these tensors (replaces `out`)
  std::vector<wgx_tensor *> split;
  // write the output into this tensor instead of the op's own output (the
  // result of a residual add folded into the convolution)
  wgx_tensor *out_override = nullptr;
};

}  // namespace wgx

struct wgx_context {
  int device = 0;
  bool destroyed = false;
  cudaStream_t stream = nullptr;
  std::vector<wgx_buffer *> owned;          // buffers freed on destroy
  std::vector<void *> allocations;          // raw device allocations (arenas, caches)
  std::vector<wgx::Command> commands;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  bool graph_valid = false;
  void *workspace = nullptr;
  uint64_t workspace_bytes = 0;
  int64_t launches_per_submit = 0;
  std::vector<std::unique_ptr<wgx_tensor>> program_tensors;  // views made by record_program
  const wgx::ConvRecordLink *conv_link = nullptr;  // see ConvRecordLink

  void *alloc_device(uint64_t bytes);  // tracked device allocation (freed on destroy)
  void invalidate_graph();
};

namespace wgx {

// ------------------------------------------------------ op registry
// A recorder validates the resolved positional args exactly like the
// reference operator's recordIn and appends one or more Commands.
using OpRecorder = std::function<void(wgx_context *, const std::vector<wgx_arg> &)>;
const std::unordered_map<std::string, OpRecorder> &op_registry();

// ------------------------------------------------------ kernel front-ends
// All of these enqueue work on `stream` and throw Error on bad input.
struct ConvLaunch;  // defined in conv.cu

void launch_mm(const void *a, const void *b, void *out, int64_t M, int64_t N, int64_t K,
               int dtype, void *scratch, uint64_t scratch_bytes, cudaStream_t stream);
// fp32 mm on the tensor cores (3xTF32, mm_tf32.cu) for the sizes it tiles
// (M, N multiples of 128, K of 32, 16-byte aligned, at least 2^29
// multiply-adds); launch_mm uses it when mm_tf32_supported. WGX_MM_TF32=0
// keeps every fp32 mm on the FFMA kernel, =2 takes every size it tiles.
bool mm_tf32_supported(const void *a, const void *b, const void *c, int64_t M, int64_t N,
                       int64_t K);
void mm_tf32_run(const float *a, const float *b, float *c, int64_t M, int64_t N, int64_t K,
                 int n_sm, cudaStream_t stream);
uint64_t mm_scratch_bytes(int64_t M, int64_t N, int64_t K, int dtype);

// Fused attention O^T[c][i] = sum_j V^T[c][j] softmax_j(sum_d Q[i][d] K^T[d][j])
// per head (csrc/attention.cu): Q [n, L, dq], K^T [n, dq, L], V^T [n, dv, L],
// O^T [n, dv, L], all fp16.
bool attention_supported(int64_t n, int64_t L, int64_t dq, int64_t dv);
void launch_attention(const __half *Q, const __half *KT, const __half *VT, __half *OT, int64_t n,
                      int64_t L, int64_t dq, int64_t dv, cudaStream_t stream);

wgx_conv2d_plan plan_conv2d(const wgx_conv2d_params &p);
// true when the convolution may write its output over its own input
bool conv2d_in_place_safe(const wgx_conv2d_params &p);
// packed-weight layout size for the tcgen05 path (0 when the plan is not UMMA)
uint64_t conv2d_packed_weight_bytes(const wgx_conv2d_params &p);
uint64_t conv2d_input_scratch_bytes(const wgx_conv2d_params &p);
// pack OIHW weights into the tcgen05 operand layout (one small kernel)
void conv2d_pack_weights(const wgx_conv2d_params &p, const void *w, void *packed,
                         cudaStream_t stream);
// full convolution; `packed` may be null (then weights are packed into the
// front of scratch first). scratch must hold conv2d_scratch_bytes(p, packed==null).
uint64_t conv2d_scratch_bytes(const wgx_conv2d_params &p, bool include_packed_weights);
void launch_conv2d(const wgx_conv2d_params &p, const void *in, const void *w, const void *packed,
                   const void *bias, void *out, void *scratch, uint64_t scratch_bytes,
                   cudaStream_t stream);
int conv2d_kernel_launches(const wgx_conv2d_params &p, bool packed_ready);

// transposed / grouped direct conv used by aten.convolution for shapes
// outside the hot path
void launch_conv_transpose2d(const wgx_conv2d_params &p, int opH, int opW, const void *in,
                             const void *w, const void *bias, void *out, cudaStream_t stream);

// conv recorder with a fused epilogue activation (program fusion pass):
// args are aten.convolution's positional args.
void record_convolution_act(wgx_context *ctx, const std::vector<wgx_arg> &args, int act);

// SPPF-style cascade of 2-3 same-size max-pools in one launch (program
// pass); false when the shapes do not qualify (nothing recorded).
bool record_maxpool_cascade(wgx_context *ctx, wgx_tensor *in,
                            const std::vector<std::pair<wgx_tensor *, wgx_tensor *>> &outs, int K);

}  // namespace wgx
