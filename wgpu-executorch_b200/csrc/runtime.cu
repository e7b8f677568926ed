// Runtime: the C-ABI context / buffer / tensor objects and the command list
// that replaces WebGPU command encoding.
//
// Reference behaviour followed (src/context.ts, src/tensor.ts):
//  * storageBuffer rounds the size up to 4 bytes, minimum 4 (context.ts:86-92)
//  * tensor() with no buffer allocates an owned buffer, with a buffer wraps
//    it without taking ownership (context.ts:135-147)
//  * Tensor validation: rank <= 8, positive integer dims, buffer large
//    enough, STORAGE usage (tensor.ts:50-71)
//  * setData: prefix write padded with zeros to 4 bytes, error when larger
//    than the tensor (tensor.ts:115-135); getData returns byteLength bytes
//    after all submitted work (tensor.ts:142-158)
//  * copy(): COPY_SRC / COPY_DST / size checks, size rounded up to 4
//    (context.ts:172-192)
//  * submit(): no-op when nothing is recorded; replays every command
//    recorded since the last reset (context.ts:323-370)
//  * destroy(): idempotent, afterwards every call throws /destroyed/
//    (context.ts:52-72)
//
// B200 design: submit() captures the command list once into a CUDA graph
// and relaunches the instantiated graph on later submits, so the per-submit
// host cost is one cudaGraphLaunch instead of re-encoding every dispatch.
#include <cstdio>

#include "umma_conv.h"
#include <cstring>
#include <atomic>
#include <mutex>

#include "internal.h"

namespace wgx {

static thread_local std::string g_last_error;

int set_error(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}
void clear_error() { g_last_error.clear(); }

[[noreturn]] void fail(const std::string &msg, int code) { throw Error{code, msg}; }

void check_cuda(cudaError_t e, const char *what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(std::string(what) + ": " + cudaGetErrorString(e),
         e == cudaErrorMemoryAllocation ? WGX_ERR_NOMEM : WGX_ERR_CUDA);
  }
}

int dtype_size(int dtype) {
  switch (dtype) {
    case WGX_FLOAT32: return 4;
    case WGX_FLOAT16: return 2;
    case WGX_INT32: return 4;
    case WGX_INT8: return 1;
    case WGX_UINT8: return 1;
    case WGX_BOOL: return 1;
    case WGX_FLOAT64: return 8;
    case WGX_INT64: return 8;
  }
  fail("unknown dtype " + std::to_string(dtype));
}

const char *dtype_name(int dtype) {
  static const char *names[] = {"float32", "float16", "int32", "int8",
                                "uint8",   "bool",    "float64", "int64"};
  if (dtype < 0 || dtype > 7) return "unknown";
  return names[dtype];
}

__device__ uint32_t g_device_error;

uint32_t *device_error_word(int device) {
  // One word per device; the symbol address is resolved with the device
  // current (cudaGetSymbolAddress is per device).
  static std::mutex mu;
  static std::unordered_map<int, uint32_t *> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  void *p = nullptr;
  check_cuda(cudaGetSymbolAddress(&p, g_device_error), "cudaGetSymbolAddress(error word)");
  cache[device] = static_cast<uint32_t *>(p);
  return static_cast<uint32_t *>(p);
}

// ------------------------------------------------------- kernel timing
struct TimedLaunch {
  std::string kernel;
  cudaEvent_t start, stop;
  bool closed;
};
struct TimingState {
  std::mutex mu;
  bool enabled = false;
  std::vector<TimedLaunch> pending;
  std::unordered_map<std::string, std::pair<double, int64_t>> totals;
};
static TimingState &timing() {
  static TimingState t;
  return t;
}

int timer_begin(const char *kernel, cudaStream_t stream) {
  TimingState &t = timing();
  std::lock_guard<std::mutex> lock(t.mu);
  if (!t.enabled) return -1;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return -1;
  }
  TimedLaunch l{kernel, nullptr, nullptr, false};
  check_cuda(cudaEventCreate(&l.start), "timer event");
  check_cuda(cudaEventCreate(&l.stop), "timer event");
  check_cuda(cudaEventRecord(l.start, stream), "timer record");
  t.pending.push_back(l);
  return int(t.pending.size()) - 1;
}

void timer_end(int handle, cudaStream_t stream) {
  if (handle < 0) return;
  TimingState &t = timing();
  std::lock_guard<std::mutex> lock(t.mu);
  if (handle >= int(t.pending.size())) return;
  check_cuda(cudaEventRecord(t.pending[handle].stop, stream), "timer record");
  t.pending[handle].closed = true;
}

// ------------------------------------------------ fault injection (tests)
static std::atomic<uint32_t> g_inject{0};

cudaError_t device_malloc(void **p, uint64_t bytes) {
  uint32_t f = g_inject.load();
  while (f & WGX_INJECT_ALLOC_FAIL) {
    // one-shot: the flag is consumed by the allocation it fails
    if (g_inject.compare_exchange_weak(f, f & ~uint32_t(WGX_INJECT_ALLOC_FAIL))) {
      *p = nullptr;
      return cudaErrorMemoryAllocation;
    }
  }
  return cudaMalloc(p, bytes);
}

bool inject_skip_loads() { return (g_inject.load() & WGX_INJECT_SKIP_LOADS) != 0; }

}  // namespace wgx

using namespace wgx;

void *wgx_context::alloc_device(uint64_t bytes) {
  void *p = nullptr;
  if (bytes == 0) bytes = 16;
  check_cuda(device_malloc(&p, bytes), "cudaMalloc");
  allocations.push_back(p);
  return p;
}

void wgx_context::invalidate_graph() {
  if (graph_exec) cudaGraphExecDestroy(graph_exec);
  if (graph) cudaGraphDestroy(graph);
  graph_exec = nullptr;
  graph = nullptr;
  graph_valid = false;
}

// Wrap a C-ABI body: Error -> status code + message.
template <class F>
static int guarded(F &&f) {
  try {
    clear_error();
    f();
    return WGX_OK;
  } catch (const Error &e) {
    return set_error(e.code, e.msg);
  } catch (const std::bad_alloc &) {
    return set_error(WGX_ERR_NOMEM, "host allocation failed");
  } catch (const std::exception &e) {
    return set_error(WGX_ERR_INVALID, e.what());
  }
}

static void assert_alive(const wgx_context *ctx) {
  if (!ctx) fail("null context");
  if (ctx->destroyed) fail("WgpuExecutionContext is destroyed", WGX_ERR_DESTROYED);
}

static void set_device(int device) { check_cuda(cudaSetDevice(device), "cudaSetDevice"); }

static wgx_buffer *make_buffer(wgx_context *ctx, int device, uint64_t size, uint32_t usage,
                               bool owned) {
  auto *b = new wgx_buffer();
  b->ctx = owned ? ctx : nullptr;
  b->size = size;
  b->usage = usage;
  b->device = device;
  set_device(device);
  cudaError_t e = device_malloc(&b->dptr, size);
  if (e != cudaSuccess) {
    delete b;
    cudaGetLastError();
    fail(std::string("cudaMalloc(") + std::to_string(size) + "): " + cudaGetErrorString(e),
         WGX_ERR_NOMEM);
  }
  b->owns_alloc = true;
  if (owned) ctx->owned.push_back(b);
  return b;
}

extern "C" {

const char *wgx_last_error(void) { return g_last_error.c_str(); }

int wgx_version(void) { return 1; }

int wgx_build_flags(uint32_t *flags) {
  return guarded([&] {
    if (!flags) fail("wgx_build_flags: null pointer");
#ifdef WGX_BOUNDS
    *flags = WGX_BUILD_BOUNDS;
#else
    *flags = 0;
#endif
  });
}

int wgx_debug_inject(uint32_t flags) {
  return guarded([&] {
    if (flags & ~uint32_t(WGX_INJECT_ALLOC_FAIL | WGX_INJECT_SKIP_LOADS))
      fail("wgx_debug_inject: unknown flags");
    g_inject.store(flags);
  });
}

int wgx_device_count(int *count) {
  return guarded([&] {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    *count = n;
  });
}

int wgx_context_create(int device, wgx_context **out) {
  return guarded([&] {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
      cudaGetLastError();
      fail("no CUDA device available", WGX_ERR_CUDA);
    }
    if (device < 0 || device >= n) fail("device index out of range");
    set_device(device);
    auto *ctx = new wgx_context();
    ctx->device = device;
    cudaError_t e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      delete ctx;
      check_cuda(e, "cudaStreamCreate");
    }
    *out = ctx;
  });
}

int wgx_context_destroy(wgx_context *ctx) {
  return guarded([&] {
    if (!ctx) fail("null context");
    if (ctx->destroyed) return;  // idempotent (context.ts:61-64)
    ctx->destroyed = true;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->invalidate_graph();
    for (auto *b : ctx->owned) {
      if (b->owns_alloc && b->dptr) cudaFree(b->dptr);
      b->dptr = nullptr;
      b->destroyed = true;
    }
    for (void *p : ctx->allocations) cudaFree(p);
    ctx->allocations.clear();
    if (ctx->workspace) cudaFree(ctx->workspace);
    ctx->workspace = nullptr;
    ctx->workspace_bytes = 0;
    ctx->commands.clear();
    cudaStreamDestroy(ctx->stream);
    ctx->stream = nullptr;
  });
}

int wgx_context_release(wgx_context *ctx) {
  return guarded([&] {
    if (!ctx) return;
    if (!ctx->destroyed) wgx_context_destroy(ctx);
    for (auto *b : ctx->owned) delete b;
    ctx->owned.clear();
    delete ctx;
  });
}

int wgx_storage_buffer(wgx_context *ctx, uint64_t size, wgx_buffer **out) {
  return guarded([&] {
    assert_alive(ctx);
    uint64_t aligned = size < 4 ? 4 : (size + 3) / 4 * 4;
    *out = make_buffer(ctx, ctx->device, aligned,
                       WGX_USAGE_STORAGE | WGX_USAGE_COPY_SRC | WGX_USAGE_COPY_DST, true);
  });
}

int wgx_buffer_create(int device, uint64_t size, uint32_t usage, wgx_buffer **out) {
  return guarded([&] {
    if (size == 0) fail("buffer size must be positive");
    *out = make_buffer(nullptr, device, size, usage, false);
  });
}

int wgx_buffer_destroy(wgx_buffer *buf) {
  return guarded([&] {
    if (!buf) return;
    if (buf->ctx) fail("buffer is owned by its context; destroy the context instead");
    if (buf->owns_alloc && buf->dptr) {
      cudaSetDevice(buf->device);
      cudaDeviceSynchronize();
      cudaFree(buf->dptr);
    }
    delete buf;
  });
}

int wgx_buffer_info(const wgx_buffer *buf, uint64_t *size, uint32_t *usage, void **device_ptr) {
  return guarded([&] {
    if (!buf) fail("null buffer");
    if (size) *size = buf->size;
    if (usage) *usage = buf->usage;
    if (device_ptr) *device_ptr = buf->dptr;
  });
}

int wgx_tensor_create(wgx_context *ctx, int dtype, const int64_t *shape, int ndim,
                      wgx_buffer *buffer, wgx_tensor **out) {
  return guarded([&] {
    if (ctx || !buffer) assert_alive(ctx);
    if (ndim < 0) fail("negative rank");
    if (ndim > WGX_MAX_NDIM)
      fail("Tensor rank " + std::to_string(ndim) + " exceeds maximum rank of " +
           std::to_string(WGX_MAX_NDIM));
    int64_t numel = 1;
    for (int i = 0; i < ndim; ++i) {
      if (shape[i] <= 0) fail("Tensor dimensions must be positive integers");
      numel *= shape[i];
    }
    int es = dtype_size(dtype);
    uint64_t required = uint64_t(numel) * es;
    wgx_buffer *buf = buffer;
    if (!buf) {
      uint64_t aligned = required < 4 ? 4 : (required + 3) / 4 * 4;
      buf = make_buffer(ctx, ctx->device, aligned,
                        WGX_USAGE_STORAGE | WGX_USAGE_COPY_SRC | WGX_USAGE_COPY_DST, true);
    } else {
      if (buf->size < required)
        fail("GPUBuffer size (" + std::to_string(buf->size) + "B) < required (" +
             std::to_string(required) + "B)");
      if ((buf->usage & WGX_USAGE_STORAGE) == 0)
        fail("GPUBuffer must have GPUBufferUsage.STORAGE flag");
    }
    auto *t = new wgx_tensor();
    t->buffer = buf;
    t->dtype = dtype;
    t->ndim = ndim;
    for (int i = 0; i < ndim; ++i) t->shape[i] = shape[i];
    t->numel = numel;
    *out = t;
  });
}

int wgx_tensor_release(wgx_tensor *t) {
  delete t;
  return WGX_OK;
}

int wgx_tensor_info(const wgx_tensor *t, int *dtype, int *ndim, int64_t *shape,
                    uint64_t *byte_length, void **device_ptr) {
  return guarded([&] {
    if (!t) fail("null tensor");
    if (dtype) *dtype = t->dtype;
    if (ndim) *ndim = t->ndim;
    if (shape)
      for (int i = 0; i < t->ndim; ++i) shape[i] = t->shape[i];
    if (byte_length) *byte_length = t->byte_length();
    if (device_ptr) *device_ptr = t->buffer->dptr;
  });
}

int wgx_tensor_set_data(wgx_tensor *t, const void *src, uint64_t nbytes) {
  return guarded([&] {
    if (!t) fail("null tensor");
    wgx_buffer *b = t->buffer;
    if (b->ctx && b->ctx->destroyed)
      fail("WgpuExecutionContext is destroyed", WGX_ERR_DESTROYED);
    if ((b->usage & WGX_USAGE_COPY_DST) == 0) fail("setData: buffer missing COPY_DST usage");
    uint64_t bl = t->byte_length();
    if (nbytes > bl)
      fail("setData: source " + std::to_string(nbytes) + "B > tensor " + std::to_string(bl) +
           "B; pass a view");
    set_device(b->device);
    cudaStream_t s = b->ctx ? b->ctx->stream : nullptr;
    if (nbytes)
      check_cuda(cudaMemcpyAsync(b->dptr, src, nbytes, cudaMemcpyHostToDevice, s),
                 "setData cudaMemcpyAsync");
    // pad the write with zeros to a 4-byte boundary, like writeBuffer of
    // the padded staging copy in tensor.ts:125-133
    uint64_t aligned = (nbytes + 3) / 4 * 4;
    if (aligned > nbytes && aligned <= b->size)
      check_cuda(cudaMemsetAsync(static_cast<char *>(b->dptr) + nbytes, 0, aligned - nbytes, s),
                 "setData pad");
    // writeBuffer takes a copy of the source at call time; make the host
    // buffer reusable on return for pinned sources as well
    check_cuda(cudaStreamSynchronize(s), "setData sync");
  });
}

int wgx_tensor_get_data(wgx_tensor *t, void *dst, uint64_t nbytes) {
  return guarded([&] {
    if (!t) fail("null tensor");
    wgx_buffer *b = t->buffer;
    if (b->ctx && b->ctx->destroyed)
      fail("WgpuExecutionContext is destroyed", WGX_ERR_DESTROYED);
    uint64_t bl = t->byte_length();
    if (nbytes < bl) fail("getData: destination smaller than tensor byteLength");
    set_device(b->device);
    // getData sees every submitted command of every context on the device,
    // like a copy submitted to the shared WebGPU queue (tensor.ts:149-152).
    check_cuda(cudaDeviceSynchronize(), "getData sync");
    check_cuda(cudaMemcpy(dst, b->dptr, bl, cudaMemcpyDeviceToHost), "getData cudaMemcpy");
  });
}

int wgx_copy(wgx_context *ctx, wgx_tensor *src, wgx_tensor *dst) {
  return guarded([&] {
    assert_alive(ctx);
    if ((src->buffer->usage & WGX_USAGE_COPY_SRC) == 0)
      fail("copy: source buffer missing COPY_SRC usage");
    if ((dst->buffer->usage & WGX_USAGE_COPY_DST) == 0)
      fail("copy: destination buffer missing COPY_DST usage");
    if (dst->byte_length() < src->byte_length())
      fail("copy: destination (" + std::to_string(dst->byte_length()) + "B) < source (" +
           std::to_string(src->byte_length()) + "B)");
    uint64_t size = (src->byte_length() + 3) / 4 * 4;
    if (size > src->buffer->size) size = src->buffer->size;
    if (size > dst->buffer->size) size = dst->buffer->size;
    void *d = dst->buffer->dptr;
    const void *s = src->buffer->dptr;
    Command c;
    c.name = "copy";
    c.kernel_launches = 0;
    c.run = [d, s, size](const ExecEnv &env) {
      check_cuda(cudaMemcpyAsync(d, s, size, cudaMemcpyDeviceToDevice, env.stream), "copy");
    };
    ctx->commands.push_back(std::move(c));
    ctx->invalidate_graph();
  });
}

int wgx_record_op(wgx_context *ctx, const char *op_name, const wgx_arg *args, int nargs) {
  return guarded([&] {
    assert_alive(ctx);
    const auto &reg = op_registry();
    auto it = reg.find(op_name ? op_name : "");
    if (it == reg.end()) fail(std::string("program: unknown operator '") + op_name + "'");
    std::vector<wgx_arg> a(args, args + nargs);
    set_device(ctx->device);
    size_t before = ctx->commands.size();
    try {
      it->second(ctx, a);
    } catch (...) {
      ctx->commands.resize(before);  // a failed recordIn records nothing
      throw;
    }
    ctx->invalidate_graph();
  });
}

static void replay(wgx_context *ctx, const ExecEnv &env) {
  for (auto &c : ctx->commands) c.run(env);
}

// Grows the context's shared workspace to what the largest command needs.
static ExecEnv ensure_workspace(wgx_context *ctx) {
  uint64_t ws = 0;
  for (auto &c : ctx->commands) ws = std::max(ws, c.workspace_bytes);
  if (ws > ctx->workspace_bytes) {
    check_cuda(cudaStreamSynchronize(ctx->stream), "workspace sync");
    if (ctx->workspace) cudaFree(ctx->workspace);
    ctx->workspace = nullptr;
    ctx->workspace_bytes = 0;
    check_cuda(device_malloc(&ctx->workspace, ws), "cudaMalloc(workspace)");
    ctx->workspace_bytes = ws;
  }
  return ExecEnv{ctx->stream, ctx->workspace, ctx->workspace_bytes};
}

// Kernel launches one replay of a captured graph makes: its kernel nodes
// (copies and memsets are not kernels).
static int64_t kernel_nodes(cudaGraph_t graph) {
  size_t n = 0;
  check_cuda(cudaGraphGetNodes(graph, nullptr, &n), "cudaGraphGetNodes");
  std::vector<cudaGraphNode_t> nodes(n);
  if (n) check_cuda(cudaGraphGetNodes(graph, nodes.data(), &n), "cudaGraphGetNodes");
  int64_t k = 0;
  for (size_t i = 0; i < n; ++i) {
    cudaGraphNodeType t;
    check_cuda(cudaGraphNodeGetType(nodes[i], &t), "cudaGraphNodeGetType");
    if (t == cudaGraphNodeTypeKernel) ++k;
  }
  return k;
}

int wgx_submit(wgx_context *ctx) {
  return guarded([&] {
    assert_alive(ctx);
    if (ctx->commands.empty()) return;  // context.ts:325-327
    set_device(ctx->device);
    if (!ctx->graph_valid) {
      ExecEnv env = ensure_workspace(ctx);
      check_cuda(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal),
                 "cudaStreamBeginCapture");
      try {
        replay(ctx, env);
      } catch (...) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(ctx->stream, &g);
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        throw;
      }
      check_cuda(cudaStreamEndCapture(ctx->stream, &ctx->graph), "cudaStreamEndCapture");
      check_cuda(cudaGraphInstantiate(&ctx->graph_exec, ctx->graph, 0), "cudaGraphInstantiate");
      ctx->graph_valid = true;
      ctx->launches_per_submit = kernel_nodes(ctx->graph);
    }
    check_cuda(cudaGraphLaunch(ctx->graph_exec, ctx->stream), "cudaGraphLaunch");
  });
}

int wgx_sync(wgx_context *ctx) {
  return guarded([&] {
    assert_alive(ctx);
    set_device(ctx->device);
    check_cuda(cudaStreamSynchronize(ctx->stream), "sync");
    uint32_t code = 0;
    uint32_t *w = device_error_word(ctx->device);
    check_cuda(cudaMemcpy(&code, w, 4, cudaMemcpyDeviceToHost), "read device error word");
    if (code) {
      uint32_t zero = 0;
      cudaMemcpy(w, &zero, 4, cudaMemcpyHostToDevice);
      fail("device reported error code " + std::to_string(code) +
               ((code & kErrBounds) ? " (an access outside its buffer was skipped)"
                                    : " (a bounded wait inside a kernel ran out)"),
           WGX_ERR_DEVICE);
    }
  });
}

int wgx_reset(wgx_context *ctx) {
  return guarded([&] {
    assert_alive(ctx);
    set_device(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->commands.clear();
    ctx->invalidate_graph();
  });
}

int wgx_context_stats(const wgx_context *ctx, int64_t *n_commands, int64_t *n_kernel_launches) {
  return guarded([&] {
    if (!ctx) fail("null context");
    // after the first submit: the kernel nodes of the captured graph;
    // before it: the recorders' per-command counts (the tensor-core
    // convolution counts its re-layout launch, which the direct mode skips)
    int64_t launches = 0;
    if (ctx->graph_valid) {
      launches = ctx->launches_per_submit;
    } else {
      for (auto &c : ctx->commands) launches += c.kernel_launches;
    }
    if (n_commands) *n_commands = int64_t(ctx->commands.size());
    if (n_kernel_launches) *n_kernel_launches = launches;
  });
}

// Holds the stream until the host has enqueued what follows: spins until
// the mapped host word *flag reaches `target`, or for at most `limit_ns` of
// %globaltimer (bounded: a host that never writes only costs the limit).
__global__ void hold_stream(const volatile int *flag, int target, uint64_t limit_ns) {
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  do {
    if (*flag >= target) return;
    __nanosleep(500);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  } while (t - t0 < limit_ns);
}

int wgx_context_profile(wgx_context *ctx, int repeats, double *ms, int capacity, int *count) {
  return guarded([&] {
    assert_alive(ctx);
    if (repeats < 1) fail("profile: repeats must be >= 1");
    set_device(ctx->device);
    const int n = int(ctx->commands.size());
    if (count) *count = n;
    if (n == 0) return;
    ExecEnv env = ensure_workspace(ctx);
    std::vector<cudaEvent_t> ev(size_t(n) + 1, nullptr);
    std::vector<double> total(size_t(n), 0.0);
    // The host takes microseconds per launch; if the GPU ran each command as
    // soon as it was enqueued, every event pair would include that wait. A
    // one-thread kernel holds the stream until the host has enqueued the
    // whole replay (a mapped host word it polls, bounded by 1 s), so each
    // pair brackets the command's device time, back to back as in a graph.
    volatile int *flag = nullptr;
    int *dflag = nullptr;
    auto release = [&] {
      if (flag) {
        *flag = 1 << 30;  // frees a hold that is still polling
        cudaStreamSynchronize(ctx->stream);
        cudaFreeHost(const_cast<int *>(flag));
      }
      for (auto e : ev)
        if (e) cudaEventDestroy(e);
    };
    try {
      void *hp = nullptr;
      check_cuda(cudaHostAlloc(&hp, sizeof(int), cudaHostAllocMapped), "profile flag");
      flag = static_cast<volatile int *>(hp);
      *flag = 0;
      check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void **>(&dflag), hp, 0),
                 "profile flag");
      for (auto &e : ev) check_cuda(cudaEventCreate(&e), "profile event");
      for (int r = 0; r < repeats; ++r) {
        hold_stream<<<1, 1, 0, ctx->stream>>>(dflag, r + 1, 1000000000ull);
        check_cuda(cudaGetLastError(), "profile hold");
        check_cuda(cudaEventRecord(ev[0], ctx->stream), "profile record");
        for (int i = 0; i < n; ++i) {
          ctx->commands[size_t(i)].run(env);
          check_cuda(cudaEventRecord(ev[size_t(i) + 1], ctx->stream), "profile record");
        }
        __atomic_store_n(const_cast<int *>(flag), r + 1, __ATOMIC_RELEASE);
        check_cuda(cudaEventSynchronize(ev[size_t(n)]), "profile sync");
        for (int i = 0; i < n; ++i) {
          float t = 0.f;
          check_cuda(cudaEventElapsedTime(&t, ev[size_t(i)], ev[size_t(i) + 1]), "profile time");
          total[size_t(i)] += t;
        }
      }
    } catch (...) {
      release();
      throw;
    }
    release();
    for (int i = 0; i < n && i < capacity; ++i) ms[i] = total[size_t(i)] / repeats;
  });
}

const char *wgx_context_command_name(const wgx_context *ctx, int index) {
  if (!ctx || index < 0 || size_t(index) >= ctx->commands.size()) return nullptr;
  return ctx->commands[size_t(index)].name.c_str();
}

// ------------------------------------------------------------ pipeline
// Pipelined steps (see wgx_pipeline_create in wgx.h). Slot k = step % depth.
// Ordering per slot, with events:
//   upload stream:   wait in_free[k]; H2D host_in -> sin[k]; record uploaded[k]
//   context stream:  wait uploaded[k]; sin[k] -> input; record in_free[k];
//                    graph; wait out_free[k]; output -> sout[k]; record computed[k]
//   download stream: wait computed[k]; D2H sout[k] -> host_out; record out_free[k]
// The host waits for out_free[k] of the slot's previous step before reusing
// slot k (and so before the caller reuses that step's host buffers).
struct wgx_pipeline {
  wgx_context *ctx = nullptr;
  wgx_tensor *input = nullptr, *output = nullptr;
  int depth = 0;
  uint64_t in_bytes = 0, out_bytes = 0;
  cudaStream_t up = nullptr, down = nullptr;
  std::vector<void *> sin, sout;
  std::vector<cudaEvent_t> uploaded, in_free, computed, out_free;
  std::vector<bool> used;  // slot has an issued step
  int64_t steps = 0;
};

static void pipeline_release(wgx_pipeline *p) {
  cudaSetDevice(p->ctx->device);
  if (p->up) cudaStreamSynchronize(p->up);
  if (p->down) cudaStreamSynchronize(p->down);
  for (void *b : p->sin) cudaFree(b);
  for (void *b : p->sout) cudaFree(b);
  for (auto *v : {&p->uploaded, &p->in_free, &p->computed, &p->out_free})
    for (cudaEvent_t e : *v)
      if (e) cudaEventDestroy(e);
  if (p->up) cudaStreamDestroy(p->up);
  if (p->down) cudaStreamDestroy(p->down);
  p->sin.clear();
  p->sout.clear();
  p->up = p->down = nullptr;
}

int wgx_pipeline_create(wgx_context *ctx, wgx_tensor *input, wgx_tensor *output, int depth,
                        wgx_pipeline **out) {
  return guarded([&] {
    assert_alive(ctx);
    if (!input || !output || !out) fail("pipeline: null argument");
    if (depth < 2 || depth > 16) fail("pipeline: depth must be in [2, 16]");
    if (input->buffer->device != ctx->device || output->buffer->device != ctx->device)
      fail("pipeline: tensors must live on the context's device");
    set_device(ctx->device);
    auto p = std::make_unique<wgx_pipeline>();
    p->ctx = ctx;
    p->input = input;
    p->output = output;
    p->depth = depth;
    p->in_bytes = input->byte_length();
    p->out_bytes = output->byte_length();
    try {
      check_cuda(cudaStreamCreateWithFlags(&p->up, cudaStreamNonBlocking), "pipeline stream");
      check_cuda(cudaStreamCreateWithFlags(&p->down, cudaStreamNonBlocking), "pipeline stream");
      p->sin.assign(depth, nullptr);
      p->sout.assign(depth, nullptr);
      for (auto *v : {&p->uploaded, &p->in_free, &p->computed, &p->out_free})
        v->assign(depth, nullptr);
      p->used.assign(depth, false);
      for (int k = 0; k < depth; ++k) {
        check_cuda(device_malloc(&p->sin[k], std::max<uint64_t>(p->in_bytes, 16)),
                   "pipeline staging (input)");
        check_cuda(device_malloc(&p->sout[k], std::max<uint64_t>(p->out_bytes, 16)),
                   "pipeline staging (output)");
        for (auto *v : {&p->uploaded, &p->in_free, &p->computed, &p->out_free})
          check_cuda(cudaEventCreateWithFlags(&(*v)[k], cudaEventDisableTiming),
                     "pipeline event");
      }
    } catch (...) {
      pipeline_release(p.get());
      throw;
    }
    *out = p.release();
  });
}

int wgx_pipeline_step(wgx_pipeline *p, const void *host_in, void *host_out) {
  return guarded([&] {
    if (!p) fail("pipeline: null pipeline");
    assert_alive(p->ctx);
    if ((!host_in && p->in_bytes) || (!host_out && p->out_bytes)) fail("pipeline: null host buffer");
    wgx_context *ctx = p->ctx;
    set_device(ctx->device);
    const int k = int(p->steps % p->depth);
    if (p->used[k]) {
      // the slot's previous step has finished its download: its buffers
      // (device and host) are free
      check_cuda(cudaEventSynchronize(p->out_free[k]), "pipeline wait");
      check_cuda(cudaStreamWaitEvent(p->up, p->in_free[k], 0), "pipeline wait");
    }
    if (p->in_bytes)
      check_cuda(cudaMemcpyAsync(p->sin[k], host_in, p->in_bytes, cudaMemcpyHostToDevice, p->up),
                 "pipeline upload");
    check_cuda(cudaEventRecord(p->uploaded[k], p->up), "pipeline event");
    check_cuda(cudaStreamWaitEvent(ctx->stream, p->uploaded[k], 0), "pipeline wait");
    if (p->in_bytes)
      check_cuda(cudaMemcpyAsync(p->input->data(), p->sin[k], p->in_bytes,
                                 cudaMemcpyDeviceToDevice, ctx->stream),
                 "pipeline input copy");
    check_cuda(cudaEventRecord(p->in_free[k], ctx->stream), "pipeline event");
    if (const int rc = wgx_submit(ctx)) fail(wgx_last_error(), rc);
    if (p->used[k]) check_cuda(cudaStreamWaitEvent(ctx->stream, p->out_free[k], 0), "pipeline wait");
    if (p->out_bytes)
      check_cuda(cudaMemcpyAsync(p->sout[k], p->output->data(), p->out_bytes,
                                 cudaMemcpyDeviceToDevice, ctx->stream),
                 "pipeline output copy");
    check_cuda(cudaEventRecord(p->computed[k], ctx->stream), "pipeline event");
    check_cuda(cudaStreamWaitEvent(p->down, p->computed[k], 0), "pipeline wait");
    if (p->out_bytes)
      check_cuda(cudaMemcpyAsync(host_out, p->sout[k], p->out_bytes, cudaMemcpyDeviceToHost,
                                 p->down),
                 "pipeline download");
    check_cuda(cudaEventRecord(p->out_free[k], p->down), "pipeline event");
    p->used[k] = true;
    ++p->steps;
  });
}

int wgx_pipeline_sync(wgx_pipeline *p) {
  return guarded([&] {
    if (!p) fail("pipeline: null pipeline");
    assert_alive(p->ctx);
    set_device(p->ctx->device);
    check_cuda(cudaStreamSynchronize(p->down), "pipeline sync");
    check_cuda(cudaStreamSynchronize(p->up), "pipeline sync");
    if (const int rc = wgx_sync(p->ctx)) fail(wgx_last_error(), rc);
  });
}

int wgx_pipeline_destroy(wgx_pipeline *p) {
  return guarded([&] {
    if (!p) return;
    std::unique_ptr<wgx_pipeline> owned(p);
    pipeline_release(p);
  });
}

int wgx_context_stream(const wgx_context *ctx, void **stream) {
  return guarded([&] {
    assert_alive(ctx);
    *stream = ctx->stream;
  });
}

int wgx_device_error(int device, uint32_t *code, int clear) {
  return guarded([&] {
    set_device(device);
    uint32_t *w = device_error_word(device);
    uint32_t v = 0;
    check_cuda(cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost), "read device error word");
    if (code) *code = v;
    if (clear) {
      uint32_t zero = 0;
      check_cuda(cudaMemcpy(w, &zero, 4, cudaMemcpyHostToDevice), "clear device error word");
    }
  });
}

int wgx_kernel_timing(int enable) {
  return guarded([&] {
    TimingState &t = timing();
    std::lock_guard<std::mutex> lock(t.mu);
    t.enabled = enable != 0;
  });
}

int wgx_kernel_timing_read(const char *kernel, double *total_ms, int64_t *count, int reset) {
  return guarded([&] {
    TimingState &t = timing();
    std::lock_guard<std::mutex> lock(t.mu);
    for (auto &l : t.pending) {
      if (l.closed) {
        check_cuda(cudaEventSynchronize(l.stop), "timer sync");
        float ms = 0;
        check_cuda(cudaEventElapsedTime(&ms, l.start, l.stop), "timer elapsed");
        auto &tot = t.totals[l.kernel];
        tot.first += ms;
        tot.second += 1;
      }
      cudaEventDestroy(l.start);
      cudaEventDestroy(l.stop);
    }
    t.pending.clear();
    auto it = t.totals.find(kernel ? kernel : "");
    if (total_ms) *total_ms = it == t.totals.end() ? 0.0 : it->second.first;
    if (count) *count = it == t.totals.end() ? 0 : it->second.second;
    if (reset) t.totals.clear();
  });
}

int wgx_mm_scratch_bytes(int64_t M, int64_t N, int64_t K, int dtype, uint64_t *bytes) {
  return guarded([&] { *bytes = mm_scratch_bytes(M, N, K, dtype); });
}

int wgx_mm(const void *a, const void *b, void *out, int64_t M, int64_t N, int64_t K, int dtype,
           void *scratch, uint64_t scratch_bytes, void *stream) {
  return guarded([&] {
    launch_mm(a, b, out, M, N, K, dtype, scratch, scratch_bytes,
              static_cast<cudaStream_t>(stream));
  });
}

int wgx_conv2d_plan_for(const wgx_conv2d_params *p, wgx_conv2d_plan *out) {
  return guarded([&] { *out = plan_conv2d(*p); });
}

int wgx_conv2d_describe(const wgx_conv2d_params *p, char *buf, int32_t len) {
  return guarded([&] {
    if (!p || !buf || len <= 0) fail("conv2d describe: null argument");
    const wgx_conv2d_plan plan = plan_conv2d(*p);
    static const char *names[] = {"?", "umma", "simt-gemm", "depthwise", "direct", "pointwise1"};
    std::string d = plan.variant == WGX_CONV_UMMA
                        ? umma_conv_describe(*p)
                        : std::string(names[(plan.variant >= 1 && plan.variant <= 5) ? plan.variant : 0]);
    std::snprintf(buf, size_t(len), "%s", d.c_str());
  });
}

int wgx_conv2d(const wgx_conv2d_params *p, const void *in, const void *w, const void *bias,
               void *out, void *scratch, uint64_t scratch_bytes, void *stream) {
  return guarded([&] {
    launch_conv2d(*p, in, w, nullptr, bias, out, scratch, scratch_bytes,
                  static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"
