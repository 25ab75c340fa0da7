// Internal (non-ABI) declarations shared by the kernel translation units.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/vqb.h"

namespace vqb {

// Validated geometry of one VQ projection.
struct LinearGeometry {
  int E, OUT, IN, D, K, G, bits;
  int row_words;  // 32-bit words per code row (packed WPR, or NSUB*bytes/4 unpacked)
  const void* codes;
  const void* codebook;
  const void* scales;
};

vqb_status validate(const vqb_linear_desc* d, LinearGeometry* out);

vqb_status launch_decode(const LinearGeometry& geo, const void* x, int x_dtype, int T, const uint32_t* idx,
                         int N, int krep, void* y, int y_dtype, bool narrow_x_f16, bool round_f16_first,
                         int wround, int ks, int* err, cudaStream_t stream);

vqb_status launch_unpack(const uint32_t* packed, int64_t rows, int64_t wpr, int nsub, int bits, uint16_t* out,
                         cudaStream_t stream);

}  // namespace vqb
