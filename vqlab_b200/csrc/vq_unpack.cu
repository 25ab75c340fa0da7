// Device vq_pack reader: packed [rows, wpr] uint32 -> uint16 codes [rows, nsub].
// One thread per code; code j of a row sits at bits [j*bits, (j+1)*bits) of
// the row's little-endian word stream (src/vqlab/runtime/vq_pack.py:79-97 and
// the Metal VQ_CODE macro, vq_switch.py:595-603).  Used by the tests to pin
// the in-kernel extraction bit-exactly and by callers that need plain codes.
#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

__global__ void vq_unpack_kernel(const uint32_t* __restrict__ packed, int64_t rows, int64_t wpr, int nsub, int bits,
                                 uint16_t* __restrict__ out) {
  const int64_t total = rows * nsub;
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nsub;
    const int64_t j = i - r * nsub;
    const uint32_t* row = packed + r * wpr;
    const int64_t bit = j * bits;
    const int64_t w = bit >> 5;
    const int sh = static_cast<int>(bit & 31);
    uint64_t v = static_cast<uint64_t>(__ldg(row + w)) >> sh;
    if (sh + bits > 32) v |= static_cast<uint64_t>(__ldg(row + w + 1)) << (32 - sh);
    out[i] = static_cast<uint16_t>(v & mask);
  }
}

vqb_status launch_unpack(const uint32_t* packed, int64_t rows, int64_t wpr, int nsub, int bits, uint16_t* out,
                         cudaStream_t stream) {
  const int64_t total = rows * nsub;
  if (total == 0) return VQB_OK;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  vq_unpack_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(packed, rows, wpr, nsub, bits, out);
  if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

}  // namespace vqb
