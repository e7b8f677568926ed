// tcgen05 / TMEM implicit-GEMM convolution for fp16 (sm_100a).
#pragma once
#include "internal.h"

namespace wgx {

// per_image_w: the weights differ per image (a batched GEMM), see
// UmmaLink::per_image_weights
bool umma_conv_supported(const wgx_conv2d_params &p, bool per_image_w = false);
uint64_t umma_conv_grid(const wgx_conv2d_params &p);
std::string umma_conv_describe(const wgx_conv2d_params &p);
// (per image when per_image_w)
uint64_t umma_conv_packed_weight_bytes(const wgx_conv2d_params &p, bool per_image_w = false);
uint64_t umma_conv_input_bytes(const wgx_conv2d_params &p, bool per_image_w = false);
void umma_conv_pack_weights(const wgx_conv2d_params &p, const __half *w, void *packed,
                            cudaStream_t stream);
// How one tensor-core convolution connects to its neighbours in a program.
struct UmmaLink {
  // output: write the consumer convolution's re-laid input (its xs buffer,
  // umma_conv_input_bytes(*consumer) bytes, padding and unused channels
  // zeroed once by the caller) instead of NCHW `out`
  const wgx_conv2d_params *consumer = nullptr;
  void *consumer_xs = nullptr;
  // input: `xs` already holds this convolution's re-laid input (written by
  // its producer), so the re-layout kernel is skipped
  bool xs_ready = false;
  // input: the concatenation along channels of nsrc NCHW sources (channel
  // counts src_ch, each a multiple of 8); 0 = the single tensor `in`
  int nsrc = 0;
  const __half *src[8] = {};
  int src_ch[8] = {};
  // NCHW output: add `resid` (same shape as the output) after the
  // activation; or split the output channels into nout tensors (channel
  // counts out_ch)
  const __half *resid = nullptr;
  // false when an output buffer is also an input buffer: the input must then
  // be staged (re-layout kernel) before the main kernel writes, so the TMA
  // direct mode, which reads the input while writing, is not used
  bool allow_direct = true;
  int nout = 0;
  __half *outp[4] = {};
  int out_ch[4] = {};
  // weights: image b has its own OIHW weights at w_to_pack + b*OC*IC*KH*KW,
  // packed image after image into `packed` (B x the per-image packed bytes):
  // aten.bmm as a 1x1 convolution (A[b] = weights, B[b] = the input image)
  bool per_image_weights = false;
};

// True when `prod` can write its output straight into the re-laid input of
// `cons` (both on the tensor-core path, matching shapes, OC % 8 == 0).
bool umma_conv_link_ok(const wgx_conv2d_params &prod, const wgx_conv2d_params &cons);

// in: NCHW fp16; packed: the operand-layout weights (umma_conv_pack_weights
// output), or, when w_to_pack is not null, the buffer to pack w_to_pack
// (OIHW) into first; xs: input scratch of umma_conv_input_bytes(p) bytes;
// out: NCHW fp16; link: see UmmaLink (null = a standalone convolution).
void umma_conv_run(const wgx_conv2d_params &p, const __half *in, void *packed,
                   const __half *w_to_pack, const __half *bias, __half *out, void *xs,
                   cudaStream_t stream, const UmmaLink *link = nullptr);

// aten.bmm in fp16 on the tensor cores: C[b] = A[b] B[b] (A [batch,M,K],
// B [batch,K,N], C [batch,M,N], row-major), run as a 1x1 convolution with
// per-image weights. scratch: umma_bmm_scratch_bytes bytes.
bool umma_bmm_supported(int64_t batch, int64_t M, int64_t K, int64_t N);
uint64_t umma_bmm_scratch_bytes(int64_t batch, int64_t M, int64_t K, int64_t N);
void umma_bmm_run(const __half *A, const __half *B, __half *C, int64_t batch, int64_t M, int64_t K,
                  int64_t N, void *scratch, uint64_t scratch_bytes, cudaStream_t stream);

}  // namespace wgx
