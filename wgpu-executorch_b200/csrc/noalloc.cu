// wgx_conv2d_noalloc: the convolution entry point for callers that must not
// allocate device memory.
//
// wgx_conv2d needs scratch space (the re-laid input and the packed weights
// of the tensor-core path) and leaves it to the caller to provide it. Some
// callers have no way to do that: code recorded inside a CUDA stream
// capture (where cudaMalloc is not allowed), hosts whose device memory is
// owned by an allocator they cannot reach from the call site, and latency-
// critical loops that cannot pay the device-wide synchronisation that
// cudaFree implies. This entry point takes only inputs and outputs and
// uses a fixed scratch buffer compiled into the library instead.
//
// The buffer is a file-scope __device__ array, so every GPU that loads the
// library holds it (NOALLOC_SCRATCH_BYTES) until the process exits. All
// calls on one device share it and it keeps whatever the last call left
// there: two calls that run at the same time on the same GPU (different
// streams, or different host threads) overwrite each other's scratch and
// give wrong results; order them on one stream. Nothing in the buffer has
// to start at zero: every scratch byte a call reads was written earlier in
// that same call (input rows past the last image are read too, but they
// only feed output positions that are discarded).
#include <mutex>

#include "internal.h"

namespace wgx {

static constexpr uint64_t NOALLOC_SCRATCH_BYTES = 32ull << 20;  // 32 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on `device`. In host code the array's
// name only stands in for the symbol; the real address comes from
// cudaGetSymbolAddress, queried once per device with that device current.
static void *noalloc_scratch(int device) {
  static std::mutex mu;
  static void *addr[64] = {};
  if (device < 0 || device >= 64) fail("wgx_conv2d_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    void *p = nullptr;
    check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
               "wgx_conv2d_noalloc: cudaGetSymbolAddress(scratch)");
    addr[device] = p;
  }
  return addr[device];
}

}  // namespace wgx

extern "C" WGX_API int wgx_conv2d_noalloc(const wgx_conv2d_params *p, const void *in,
                                          const void *w, const void *bias, void *out,
                                          void *stream) {
  using namespace wgx;
  try {
    clear_error();
    if (!p) fail("wgx_conv2d_noalloc: null params");
    const uint64_t need = conv2d_scratch_bytes(*p, true);
    if (need > NOALLOC_SCRATCH_BYTES)
      fail("wgx_conv2d_noalloc: this convolution needs " + std::to_string(need) +
           " bytes of scratch but the built-in buffer holds " +
           std::to_string(NOALLOC_SCRATCH_BYTES) +
           "; call wgx_conv2d with caller-provided scratch instead");
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "wgx_conv2d_noalloc: cudaGetDevice");
    void *scratch = need ? noalloc_scratch(dev) : nullptr;
    launch_conv2d(*p, in, w, nullptr, bias, out, scratch, need ? NOALLOC_SCRATCH_BYTES : 0,
                  static_cast<cudaStream_t>(stream));
    return WGX_OK;
  } catch (const Error &e) {
    return set_error(e.code, e.msg);
  } catch (const std::exception &e) {
    return set_error(WGX_ERR_INVALID, e.what());
  }
}
