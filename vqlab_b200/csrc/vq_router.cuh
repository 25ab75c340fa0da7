// The MoE router for one token, one warp, E <= 32 * VPL experts: the
// reference block's routing (tests/test_qwen3_5_parity.py:180-204, router
// convention family/qwen3_5.py:110-118) -- fp32 softmax over the E logits
// (max-subtracted exp, divided by the sum), the top_k largest probabilities
// by top_k rounds of a warp arg-max (larger probability first, the lower
// expert id on a tie), their weights divided by the selected sum (added in
// selection order).  Each lane keeps its VPL probabilities in registers,
// sorted once; a top-k round is two warp reductions (redux) over the lanes'
// heads, and the winning lane drops its head.  Used by the router kernel and
// by the fused MoE block, so both route identically.
#pragma once

#include "vqb_common.cuh"

namespace vqb {

// Lane j < k receives slot j: its expert (out_i) and renormalised weight
// (out_w).  NaN logits leave no candidate: such a slot gets expert 0, weight 0.
template <int VPL>
__device__ __forceinline__ void route_row_reg(const float* __restrict__ row, int E, int k, int lane, int& out_i,
                                              float& out_w) {
  float p[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? __ldg(row + e) : -INFINITY;
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i)
    if (lane + 32 * i < E) m = fmaxf(m, p[i]);
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (lane + 32 * i < E) {
      p[i] = expf(p[i] - m);
      sum += p[i];
    }
  }
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  // the lane's entries sorted once (bitonic network): larger probability
  // first, the lower expert id among equals; removed entries (-1) and NaN last
  int ix[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float q = lane + 32 * i < E ? __fdiv_rn(p[i], sum) : -1.0f;
    const bool live = q > -1.0f;
    p[i] = live ? q : -1.0f;
    ix[i] = live ? lane + 32 * i : 0x7fffffff;
  }
#pragma unroll
  for (int size = 2; size <= VPL; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const bool i_first = p[i] > p[j] || (p[i] == p[j] && ix[i] < ix[j]);
          const bool swap = ((i & size) == 0) ? !i_first : i_first;
          const float tv = p[i];
          const int ti = ix[i];
          p[i] = swap ? p[j] : p[i];
          ix[i] = swap ? ix[j] : ix[i];
          p[j] = swap ? tv : p[j];
          ix[j] = swap ? ti : ix[j];
        }
      }
    }
  }
  float mine_w = 0.0f, wsum = 0.0f;
  int mine_i = 0;
  for (int j = 0; j < k; ++j) {
    // the warp's best (larger probability, then the lower expert id): one
    // reduction over the lanes' heads as ordered keys (probabilities are >= 0;
    // key 0 = a lane with nothing left), one over the ids holding that key;
    // the winning lane drops its head
    const uint32_t key = p[0] >= 0.0f ? __float_as_uint(p[0]) + 1u : 0u;
    const uint32_t top = __reduce_max_sync(0xffffffffu, key);
    const uint32_t bi = __reduce_min_sync(0xffffffffu, key == top ? static_cast<uint32_t>(ix[0]) : 0xffffffffu);
    float bv = 0.0f;  // no candidate left (NaN logits): expert 0, weight 0
    int sel = 0;
    if (top != 0u) {
      bv = __uint_as_float(top - 1u);
      sel = static_cast<int>(bi);
      const bool pop = static_cast<uint32_t>(ix[0]) == bi;
#pragma unroll
      for (int i = 0; i + 1 < VPL; ++i) {
        p[i] = pop ? p[i + 1] : p[i];
        ix[i] = pop ? ix[i + 1] : ix[i];
      }
      p[VPL - 1] = pop ? -1.0f : p[VPL - 1];
      ix[VPL - 1] = pop ? 0x7fffffff : ix[VPL - 1];
    }
    if (lane == j) {
      mine_w = bv;
      mine_i = sel;
    }
    wsum += bv;
  }
  out_i = mine_i;
  out_w = __fdiv_rn(mine_w, wsum);
}

}  // namespace vqb
