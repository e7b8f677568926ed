// tcgen05 / TMEM implicit-GEMM convolution for fp16 (sm_100a).
#pragma once
#include "internal.h"

namespace wgx {

bool umma_conv_supported(const wgx_conv2d_params &p);
uint64_t umma_conv_grid(const wgx_conv2d_params &p);
uint64_t umma_conv_packed_weight_bytes(const wgx_conv2d_params &p);
uint64_t umma_conv_input_bytes(const wgx_conv2d_params &p);
void umma_conv_pack_weights(const wgx_conv2d_params &p, const __half *w, void *packed,
                            cudaStream_t stream);
// in: NCHW fp16; packed: the operand-layout weights (umma_conv_pack_weights
// output), or, when w_to_pack is not null, the buffer to pack w_to_pack
// (OIHW) into first; xs: input scratch of umma_conv_input_bytes(p) bytes;
// out: NCHW fp16.
void umma_conv_run(const wgx_conv2d_params &p, const __half *in, void *packed,
                   const __half *w_to_pack, const __half *bias, __half *out, void *xs,
                   cudaStream_t stream);

}  // namespace wgx
