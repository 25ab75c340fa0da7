// The MoE router for one token, one warp, E <= 32 * VPL experts: the
// reference block's routing (tests/test_qwen3_5_parity.py:180-204, router
// convention family/qwen3_5.py:110-118) -- fp32 softmax over the E logits
// (max-subtracted exp, divided by the sum), the top_k largest probabilities
// by top_k rounds of a warp arg-max (larger probability first, the lower
// expert id on a tie), their weights divided by the selected sum (added in
// selection order).  Each lane keeps its VPL probabilities in registers: the
// logit loads are independent, and a top-k round rescans only the winning
// lane's values (every other lane's best is unchanged).  Used by the router
// kernel and by the fused MoE block, so both route identically.
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
#pragma unroll
  for (int i = 0; i < VPL; ++i) p[i] = lane + 32 * i < E ? __fdiv_rn(p[i], sum) : -1.0f;
  // this lane's best remaining entry (strictly larger wins: the lowest index among equals)
  auto local_best = [&](float& bv, int& bi) {
    bv = -1.0f;
    bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (p[i] > bv) {
        bv = p[i];
        bi = lane + 32 * i;
      }
    }
  };
  float lv;
  int li;
  local_best(lv, li);
  float mine_w = 0.0f, wsum = 0.0f;
  int mine_i = 0;
  for (int j = 0; j < k; ++j) {
    float bv = lv;
    int bi = li;
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi >= E) {  // no candidate left (NaN logits): expert 0, weight 0
      bi = 0;
      bv = 0.0f;
    } else if ((bi & 31) == lane) {
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        if (lane + 32 * i == bi) p[i] = -1.0f;
      local_best(lv, li);
    }
    if (lane == j) {
      mine_w = bv;
      mine_i = bi;
    }
    wsum += bv;
  }
  out_i = mine_i;
  out_w = __fdiv_rn(mine_w, wsum);
}

}  // namespace vqb
