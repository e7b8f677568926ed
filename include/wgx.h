/*
 * wgx.h - C ABI of the B200-native dense-contraction engine behind the
 * wgpu-executorch operator / program API.
 *
 * Every entry point returns an int status (WGX_OK == 0). On failure the
 * calling thread's message is available from wgx_last_error(); the message
 * wording follows the reference's thrown Error strings so that a host shim
 * (Node-API, ctypes) can rethrow them unchanged.
 *
 * Reference interfaces replaced (paths inside barhanc/wgpu-executorch):
 *   src/context.ts  WgpuExecutionContext      -> wgx_context_* / wgx_submit ...
 *   src/tensor.ts   Tensor                    -> wgx_tensor_*
 *   src/program.ts  Program + resolveArgs     -> wgx_record_program
 *   src/shader.ts   Shader.recordIn           -> wgx_record_op
 *   src/command.ts  createComputeBundle       -> (internal: launch records)
 *   src/shaders/mm, convolution, conv-with-clamp (WGSL kernels)
 *                                             -> wgx_mm / wgx_conv2d
 *
 * No torch types appear here: plain pointers, sizes and opaque handles.
 */
#ifndef WGX_H
#define WGX_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WGX_API __attribute__((visibility("default")))
#else
#define WGX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ */
/* status codes                                                        */
/* ------------------------------------------------------------------ */
#define WGX_OK 0
#define WGX_ERR_INVALID 1   /* validation error (the reference throws Error) */
#define WGX_ERR_CUDA 2      /* a CUDA runtime call failed                     */
#define WGX_ERR_DESTROYED 3 /* context used after destroy()                   */
#define WGX_ERR_NOMEM 4     /* device or pinned allocation failed             */
#define WGX_ERR_DEVICE 5    /* a kernel reported an error (bounded wait ran out) */
#define WGX_ERR_UNSUPPORTED 6

/* dtypes, in the order of src/tensor.ts:4-5 (DType) */
#define WGX_FLOAT32 0
#define WGX_FLOAT16 1
#define WGX_INT32 2
#define WGX_INT8 3
#define WGX_UINT8 4
#define WGX_BOOL 5
#define WGX_FLOAT64 6
#define WGX_INT64 7

/* buffer usage bits: the GPUBufferUsage values the reference checks
 * (src/context.ts:10-11, 175-180; src/tensor.ts:67-69, 118-120) */
#define WGX_USAGE_MAP_READ 0x0001u
#define WGX_USAGE_COPY_SRC 0x0004u
#define WGX_USAGE_COPY_DST 0x0008u
#define WGX_USAGE_UNIFORM 0x0040u
#define WGX_USAGE_STORAGE 0x0080u

#define WGX_MAX_NDIM 8 /* src/tensor.ts:23 MAX_NDIM */

typedef struct wgx_context wgx_context;
typedef struct wgx_buffer wgx_buffer;
typedef struct wgx_tensor wgx_tensor;

/* Positional operator argument: the resolved form of one Program value
 * (src/program.ts:188-224 resolveArgs: Tensor | scalar | number[] |
 * Tensor[] | undefined). */
#define WGX_ARG_NULL 0
#define WGX_ARG_TENSOR 1
#define WGX_ARG_NUMBER 2 /* JS number: f64 */
#define WGX_ARG_BOOL 3
#define WGX_ARG_INT_LIST 4
#define WGX_ARG_TENSOR_LIST 5
#define WGX_ARG_STRING 6

typedef struct wgx_arg {
  int32_t kind;
  int32_t count; /* list length */
  union {
    wgx_tensor *tensor;
    double number;
    int32_t boolean;
    const int64_t *ints;
    wgx_tensor *const *tensors;
    const char *string;
  } v;
} wgx_arg;

/* ------------------------------------------------------------------ */
/* errors / library                                                    */
/* ------------------------------------------------------------------ */
WGX_API const char *wgx_last_error(void);
WGX_API int wgx_version(void);
WGX_API int wgx_device_count(int *count);

/* ------------------------------------------------------------------ */
/* context: src/context.ts:17 WgpuExecutionContext                     */
/* ------------------------------------------------------------------ */
/* new WgpuExecutionContext(device)  (src/context.ts:28-30) */
WGX_API int wgx_context_create(int device, wgx_context **out);
/* destroy(): frees owned buffers, idempotent; afterwards every call fails
 * with "WgpuExecutionContext is destroyed" (src/context.ts:52-72). */
WGX_API int wgx_context_destroy(wgx_context *ctx);
/* frees the handle itself (after destroy); the JS object's finaliser */
WGX_API int wgx_context_release(wgx_context *ctx);
/* storageBuffer(size): STORAGE|COPY_SRC|COPY_DST, size rounded up to 4,
 * minimum 4, owned by the context (src/context.ts:86-92). */
WGX_API int wgx_storage_buffer(wgx_context *ctx, uint64_t size, wgx_buffer **out);
/* device.createBuffer({size, usage}) on CUDA device `device`: a buffer no
 * context owns (tests/api/context.test.ts:31-67 build such buffers). */
WGX_API int wgx_buffer_create(int device, uint64_t size, uint32_t usage, wgx_buffer **out);
WGX_API int wgx_buffer_destroy(wgx_buffer *buf);
WGX_API int wgx_buffer_info(const wgx_buffer *buf, uint64_t *size, uint32_t *usage, void **device_ptr);
/* tensor(dtype, shape, buffer?) (src/context.ts:135-147): buffer NULL ->
 * a new storage buffer owned by ctx; else a non-owning view, and ctx may be
 * NULL (new Tensor(dtype, shape, device, buffer), src/tensor.ts:50-71). */
WGX_API int wgx_tensor_create(wgx_context *ctx, int dtype, const int64_t *shape, int ndim,
                      wgx_buffer *buffer_or_null, wgx_tensor **out);
WGX_API int wgx_tensor_release(wgx_tensor *t);
WGX_API int wgx_tensor_info(const wgx_tensor *t, int *dtype, int *ndim, int64_t *shape,
                    uint64_t *byte_length, void **device_ptr);
/* Tensor.setData (src/tensor.ts:115-135): prefix write, padded with zeros
 * to 4 bytes, error if larger than the tensor. */
WGX_API int wgx_tensor_set_data(wgx_tensor *t, const void *src, uint64_t nbytes);
/* Tensor.getData (src/tensor.ts:142-158): waits for submitted work and
 * copies byteLength bytes to dst. */
WGX_API int wgx_tensor_get_data(wgx_tensor *t, void *dst, uint64_t nbytes);
/* copy(src, dst) (src/context.ts:172-192): recorded buffer copy. */
WGX_API int wgx_copy(wgx_context *ctx, wgx_tensor *src, wgx_tensor *dst);
/* recordShader(shader, args) (src/context.ts:201-205) with the shader
 * looked up by ExecuTorch name (src/shaders/index.ts:58-60). */
WGX_API int wgx_record_op(wgx_context *ctx, const char *op_name, const wgx_arg *args, int nargs);
/* recordProgram(program, weights, args) (src/context.ts:219-317); the
 * Program is its JSON text (src/program.ts:150-165). args are the I/O
 * values [in..., out...]. */
WGX_API int wgx_record_program(wgx_context *ctx, const char *json, uint64_t json_len,
                       const void *weights, uint64_t weights_len, const wgx_arg *args,
                       int nargs);
/* submit() (src/context.ts:323-370): first call after recording captures
 * the command list into a CUDA graph, every call launches the graph. */
WGX_API int wgx_submit(wgx_context *ctx);
/* sync() (src/context.ts:377-380) */
WGX_API int wgx_sync(wgx_context *ctx);
/* reset() (src/context.ts:386-389) */
WGX_API int wgx_reset(wgx_context *ctx);
/* number of recorded commands and of kernel launches one submit replays
 * (after the first submit: the kernel nodes of the captured CUDA graph;
 * before it: the recorders' per-command counts, an upper bound) */
WGX_API int wgx_context_stats(const wgx_context *ctx, int64_t *n_commands, int64_t *n_kernel_launches);
/* Replays the recorded commands eagerly (outside the captured graph)
 * `repeats` times with a CUDA event pair around each command and writes the
 * mean milliseconds of command i to ms[i] (at most `capacity` entries).
 * Each replay is held on the device (a one-thread kernel polling a mapped
 * host word, at most 1 s) until the host has enqueued all of it: the pairs
 * time the device work of back-to-back commands, as in a graph replay, not
 * the host's launch rate;
 * *count receives the number of commands. The reference times whole
 * submits only (utils/benchmark/main.ts:60-77); this is the per-command
 * breakdown of that figure. */
WGX_API int wgx_context_profile(wgx_context *ctx, int repeats, double *ms, int capacity, int *count);
/* Pipelined serving steps of a recorded program. No counterpart in the
 * reference: there, writeBuffer (Tensor.setData, src/tensor.ts:115-135),
 * the dispatches of submit() (src/context.ts:323-370) and the readback of
 * getData (src/tensor.ts:142-158) are ordered on the one WebGPU queue, and
 * wgx_tensor_set_data / wgx_submit / wgx_tensor_get_data keep that order.
 * A pipeline runs the same three parts of consecutive steps on three
 * streams so that they overlap: step k uploads host_in into a device
 * staging slot (upload stream) while step k-1 computes; the context stream
 * copies the slot into `input`, replays the recorded commands and copies
 * `output` into an output slot; the download stream copies that slot to
 * host_out while step k+1 computes. Every step still moves all of its input
 * and output across the host link. `input` and `output` are the tensors the
 * recorded program reads and writes (bound by wgx_record_program); depth
 * (>= 2) staging slots of each are allocated on the device. host_in and
 * host_out (pinned memory for the copies to overlap) belong to the step
 * until `depth` further steps have been issued or wgx_pipeline_sync has
 * returned: wgx_pipeline_step first waits for the step issued `depth`
 * steps earlier to finish its download. */
typedef struct wgx_pipeline wgx_pipeline;
WGX_API int wgx_pipeline_create(wgx_context *ctx, wgx_tensor *input, wgx_tensor *output,
                                int depth, wgx_pipeline **out);
WGX_API int wgx_pipeline_step(wgx_pipeline *p, const void *host_in, void *host_out);
/* waits for every issued step (and reports device errors like wgx_sync) */
WGX_API int wgx_pipeline_sync(wgx_pipeline *p);
/* waits for the issued steps and frees the pipeline's streams and slots */
WGX_API int wgx_pipeline_destroy(wgx_pipeline *p);
/* the op name of recorded command `index` (NULL when out of range); the
 * string lives until the context is reset or destroyed */
WGX_API const char *wgx_context_command_name(const wgx_context *ctx, int index);
/* the context's CUDA stream (cudaStream_t) for callers that interleave work */
WGX_API int wgx_context_stream(const wgx_context *ctx, void **stream);

/* ------------------------------------------------------------------ */
/* stateless hot-path kernels                                          */
/* ------------------------------------------------------------------ */
/* out[M,N] = a[M,K] @ b[K,N], row-major, dtype WGX_FLOAT32 or
 * WGX_FLOAT16 (src/shaders/mm/index.ts:32-93; mm-64x64.wgsl.ts:8-115).
 * fp16 accumulates in fp32. scratch: wgx_mm_scratch_bytes(). */
WGX_API int wgx_mm_scratch_bytes(int64_t M, int64_t N, int64_t K, int dtype, uint64_t *bytes);
WGX_API int wgx_mm(const void *a, const void *b, void *out, int64_t M, int64_t N, int64_t K, int dtype,
           void *scratch, uint64_t scratch_bytes, void *stream);

/* epilogue activations */
#define WGX_ACT_NONE 0
#define WGX_ACT_CLAMP 1 /* et_vk.conv_with_clamp: clamp(v, min, max) */
#define WGX_ACT_SILU 2  /* v * sigmoid(v): conv -> sigmoid -> mul      */

/* aten.convolution / et_vk.conv_with_clamp geometry: the 80-byte
 * ConvParams of src/shaders/convolution/index.ts:149-162 plus the clamp
 * words of src/shaders/conv-with-clamp/index.ts:146-164. */
typedef struct wgx_conv2d_params {
  int32_t B, IC, IH, IW;
  int32_t OC, OH, OW;
  int32_t KH, KW;
  int32_t sH, sW, pH, pW, dH, dW;
  int32_t groups;
  int32_t has_bias;
  int32_t dtype;      /* WGX_FLOAT32 / WGX_FLOAT16 */
  int32_t act;        /* WGX_ACT_* */
  float out_min;      /* clamp bounds (-inf/+inf when absent) */
  float out_max;
} wgx_conv2d_params;

/* kernel variant chosen for a convolution (host-only, no GPU needed) */
#define WGX_CONV_UMMA 1       /* tcgen05/TMEM implicit GEMM (fp16) */
#define WGX_CONV_SIMT_GEMM 2  /* FFMA implicit GEMM (fp32, odd shapes) */
#define WGX_CONV_DEPTHWISE 3  /* memory-bound depthwise */
#define WGX_CONV_DIRECT 4     /* grouped direct conv */
#define WGX_CONV_POINTWISE1 5 /* single output channel 1x1 */

typedef struct wgx_conv2d_plan {
  int32_t variant;
  int32_t n_launches;
  uint64_t scratch_bytes;
  uint64_t grid_ctas; /* CTAs of the main kernel */
} wgx_conv2d_plan;

WGX_API int wgx_conv2d_plan_for(const wgx_conv2d_params *p, wgx_conv2d_plan *out);
/* A one-line, NUL-terminated description of the kernel configuration that
 * wgx_conv2d_plan_for selects (variant; for the tensor-core path the tile
 * orientation, N, M blocks per tile, channels per stage, filter rows per
 * stage, pipeline stages, resident weights, skipped taps). No counterpart
 * in the reference (its variant selection is convolution/index.ts:58-310). */
WGX_API int wgx_conv2d_describe(const wgx_conv2d_params *p, char *buf, int32_t len);
/* in: NCHW [B,IC,IH,IW]; w: OIHW [OC,IC/groups,KH,KW]; bias: [OC] or NULL;
 * out: NCHW [B,OC,OH,OW]. The packed-weight cache lives in scratch. */
WGX_API int wgx_conv2d(const wgx_conv2d_params *p, const void *in, const void *w, const void *bias,
               void *out, void *scratch, uint64_t scratch_bytes, void *stream);
/* Same convolution for callers that cannot allocate device memory (inside
 * a stream capture, under a foreign allocator, or in loops that cannot
 * afford cudaFree's synchronisation). No counterpart in the reference.
 * Scratch comes from a fixed 32 MiB buffer built into the library instead
 * of from the caller; the call allocates nothing. Convolutions needing more
 * than 32 MiB of scratch (wgx_conv2d_plan_for: scratch_bytes) are rejected.
 * The first call on a device looks the buffer up (once per device); make
 * that first call before any stream capture. All calls on a device share
 * the buffer: calls that overlap on the GPU race, so order them on one
 * stream. The looked-up address (like the device error word's) is cached
 * for the life of the process: do not use the library across a
 * cudaDeviceReset of a device it has already run on. */
WGX_API int wgx_conv2d_noalloc(const wgx_conv2d_params *p, const void *in, const void *w,
                               const void *bias, void *out, void *stream);

/* ------------------------------------------------------------------ */
/* kernel timing: when enabled, the hot-path kernels launched outside a */
/* CUDA graph record a CUDA-event pair on their own stream around the   */
/* main kernel. read() waits for the recorded pairs and returns the     */
/* summed milliseconds and launch count for `kernel` (e.g.              */
/* "umma_conv_kernel"); reset=1 clears the totals.                      */
/* ------------------------------------------------------------------ */
WGX_API int wgx_kernel_timing(int enable);
WGX_API int wgx_kernel_timing_read(const char *kernel, double *total_ms, int64_t *count, int reset);

/* ------------------------------------------------------------------ */
/* device error word: kernels with bounded waits set it instead of      */
/* hanging; wgx_sync reports it.                                        */
/* ------------------------------------------------------------------ */
WGX_API int wgx_device_error(int device, uint32_t *code, int clear);

/* ------------------------------------------------------------------ */
/* Fault injection for failure-detection tests. No counterpart in the  */
/* reference (whose errors are synchronous throws, context.ts:52-56,   */
/* 226-230, 296-298). Process-wide; wgx_debug_inject(0) clears it.      */
/*  WGX_INJECT_ALLOC_FAIL: the next device allocation of the library    */
/*    fails as cudaMalloc's out-of-memory would (WGX_ERR_NOMEM); one    */
/*    shot, nothing is allocated, the context stays usable.             */
/*  WGX_INJECT_SKIP_LOADS: tensor-core convolution kernels launched     */
/*    while it is set issue none of their copies, so their bounded      */
/*    mbarrier waits run out (after ~2 s); the kernel records the        */
/*    timeout in the device error word and returns, and the next        */
/*    wgx_sync reports WGX_ERR_DEVICE. No trap, no fault.               */
/* ------------------------------------------------------------------ */
#define WGX_INJECT_ALLOC_FAIL 1u
#define WGX_INJECT_SKIP_LOADS 2u
WGX_API int wgx_debug_inject(uint32_t flags);

/* How the loaded library was built (no counterpart in the reference):
 * WGX_BUILD_BOUNDS is set in the bounds-checking debug build
 * (lib/libwgx_bounds.so, `make bounds`), whose hot-path kernels skip any
 * global access outside its buffer and report it as WGX_ERR_DEVICE at the
 * next wgx_sync. */
#define WGX_BUILD_BOUNDS 1u
WGX_API int wgx_build_flags(uint32_t *flags);

#ifdef __cplusplus
}
#endif
#endif /* WGX_H */
