// TMA tensor maps for the tensor-core convolution (sm_100a).
#pragma once
#include <cuda.h>

#include "internal.h"

namespace wgx {

constexpr int kMaxTmaps = 8;

// One tensor map per input source, passed to the kernel as a __grid_constant__
// parameter.
struct TmapSet {
  CUtensorMap m[kMaxTmaps];
};

// 3-D map over an NCHW fp16 tensor viewed as [B][C][HW]: dimension 0 is the
// HW positions of one channel plane (contiguous), 1 the channels, 2 the
// images; box = 64 positions (128 bytes, one 128-byte swizzle row) x box_c
// channels x 1 image, 128-byte swizzle, zero fill outside the tensor.
// Requires HW % 8 == 0 (16-byte plane stride) and a 16-byte aligned base.
void encode_nchw_tmap(CUtensorMap *map, const void *base, int B, int C, int HW, int box_c);

}  // namespace wgx
