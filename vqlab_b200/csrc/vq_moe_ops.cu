// The elementwise work of the MoE block around the three VQ projections, one
// pass each instead of a chain of framework ops (the reference block:
// tests/test_qwen3_5_parity.py:180-204, mlx_lm SwitchGLU):
//   swiglu:  h = dtype( silu(f32(gate)) * f32(up) ),  silu(v) = v / (1 + exp(-v))
//   combine: y[t, :] = dtype( sum_j w[t, j] * f32(d[t, j, :]) ), j = 0 .. k-1 in order, fp32
// Both are HBM-bound streams; 16-byte vectors when the tensors allow it.
#include "vqb_common.cuh"
#include "vqb_internal.h"
#include "vq_router.cuh"

namespace vqb {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// VEC elements of T per thread-step (16 bytes when VEC * sizeof(T) == 16)
template <typename T, int VEC>
__global__ void swiglu_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ h, int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t nv = n / VEC;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    T gv[VEC], uv[VEC], hv[VEC];
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(gv) = __ldg(reinterpret_cast<const uint4*>(g) + i);
      *reinterpret_cast<uint4*>(uv) = __ldg(reinterpret_cast<const uint4*>(u) + i);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) { gv[j] = g[i * VEC + j]; uv[j] = u[i * VEC + j]; }
    }
#pragma unroll
    for (int j = 0; j < VEC; ++j) hv[j] = from_f<T>(__fmul_rn(silu(to_f(gv[j])), to_f(uv[j])));
    if constexpr (VEC * sizeof(T) == 16) {
      reinterpret_cast<uint4*>(h)[i] = *reinterpret_cast<uint4*>(hv);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) h[i * VEC + j] = hv[j];
    }
  }
}

// one thread = VEC consecutive hidden elements of one token
template <typename T, int VEC>
__global__ void combine_kernel(const T* __restrict__ d, const float* __restrict__ w, T* __restrict__ y, int Tn, int k,
                               int H) {
  pdl_wait();
  pdl_trigger();
  const int per_tok = H / VEC;
  const int64_t total = static_cast<int64_t>(Tn) * per_tok;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / per_tok);
    const int c = static_cast<int>(i - static_cast<int64_t>(t) * per_tok);
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;
    for (int j = 0; j < k; ++j) {
      const float wj = __ldg(w + static_cast<int64_t>(t) * k + j);
      const T* row = d + (static_cast<int64_t>(t) * k + j) * H + static_cast<int64_t>(c) * VEC;
      T v[VEC];
      if constexpr (VEC * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(v) = __ldg(reinterpret_cast<const uint4*>(row));
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[e] = row[e];
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(to_f(v[e]), wj));  // product rounded, no fma
    }
    T o[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = from_f<T>(acc[e]);
    T* out = y + static_cast<int64_t>(t) * H + static_cast<int64_t>(c) * VEC;
    if constexpr (VEC * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(out) = *reinterpret_cast<uint4*>(o);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) out[e] = o[e];
    }
  }
}

// Partial combine for expert parallelism: out[t, :] = sum over this rank's
// slots j (skip[t, j] != kSkipExpert) of w[t, j] * f32(d[t, j, :]), in slot
// order, kept in fp32 (the owner of token t adds the ranks' partials).  A
// skipped slot's d row is never read.
template <typename T, int VEC>
__global__ void combine_partial_kernel(const T* __restrict__ d, const float* __restrict__ w,
                                       const uint32_t* __restrict__ skip, float* __restrict__ y, int Tn, int k,
                                       int H) {
  pdl_wait();
  pdl_trigger();
  const int per_tok = H / VEC;
  const int64_t total = static_cast<int64_t>(Tn) * per_tok;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / per_tok);
    const int c = static_cast<int>(i - static_cast<int64_t>(t) * per_tok);
    float acc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] = 0.0f;
    for (int j = 0; j < k; ++j) {
      if (skip && __ldg(skip + static_cast<int64_t>(t) * k + j) == kSkipExpert) continue;
      const float wj = __ldg(w + static_cast<int64_t>(t) * k + j);
      const T* row = d + (static_cast<int64_t>(t) * k + j) * H + static_cast<int64_t>(c) * VEC;
      T v[VEC];
      if constexpr (VEC * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(v) = __ldg(reinterpret_cast<const uint4*>(row));
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[e] = row[e];
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(to_f(v[e]), wj));
    }
    float* out = y + static_cast<int64_t>(t) * H + static_cast<int64_t>(c) * VEC;
#pragma unroll
    for (int e = 0; e < VEC; ++e) out[e] = acc[e];
  }
}

// The router of the MoE block in one pass, one warp per token: fp32 softmax
// over the E logits (max-subtracted exp, divided by the sum), the top_k largest
// probabilities by top_k rounds of a warp arg-max (larger probability first,
// the lower expert id on a tie), their weights divided by the selected sum
// (added in selection order).  The warp keeps its row of probabilities in
// shared memory; a chosen entry is marked -1 (probabilities are >= 0).
__global__ void __launch_bounds__(256) route_topk_kernel(const float* __restrict__ logits, int T, int E, int k,
                                                         int32_t* __restrict__ idx, float* __restrict__ w) {
  extern __shared__ float s_prob[];
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  float* p = s_prob + static_cast<size_t>(warp) * E;
  for (int t = blockIdx.x * nw + warp; t < T; t += gridDim.x * nw) {
    const float* row = logits + static_cast<int64_t>(t) * E;
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) {
      const float v = row[e];
      p[e] = v;
      m = fmaxf(m, v);
    }
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.0f;
    for (int e = lane; e < E; e += 32) {
      const float ex = expf(p[e] - m);
      p[e] = ex;
      sum += ex;
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    for (int e = lane; e < E; e += 32) p[e] = __fdiv_rn(p[e], sum);
    __syncwarp();
    float mine_w = 0.0f, wsum = 0.0f;
    int mine_i = 0;
    for (int j = 0; j < k; ++j) {
      float bv = -1.0f;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        const float v = p[e];
        if (v > bv) {
          bv = v;
          bi = e;
        }
      }
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
        p[bi] = -1.0f;
      }
      __syncwarp();
      if (lane == j) {
        mine_w = bv;
        mine_i = bi;
      }
      wsum += bv;
    }
    if (lane < k) {
      idx[static_cast<int64_t>(t) * k + lane] = mine_i;
      w[static_cast<int64_t>(t) * k + lane] = __fdiv_rn(mine_w, wsum);
    }
    __syncwarp();
  }
}

// The same router for E <= 32 * VPL experts with each lane's VPL
// probabilities in registers (route_row_reg, vq_router.cuh): same arithmetic,
// same order and same tie-breaking as route_topk_kernel, so the results are
// bit-identical.
template <int VPL>
__global__ void __launch_bounds__(256) route_topk_reg_kernel(const float* __restrict__ logits, int T, int E, int k,
                                                             int32_t* __restrict__ idx, float* __restrict__ w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_trigger();
  const int nw = blockDim.x >> 5;
  for (int t = blockIdx.x * nw + warp; t < T; t += gridDim.x * nw) {
    int mine_i;
    float mine_w;
    route_row_reg<VPL>(logits + static_cast<int64_t>(t) * E, E, k, lane, mine_i, mine_w);
    if (lane < k) {
      idx[static_cast<int64_t>(t) * k + lane] = mine_i;
      w[static_cast<int64_t>(t) * k + lane] = mine_w;
    }
  }
}

thread_local int g_sms_ops = 0;  // the current device's SM count, refreshed by ensure_sms()

vqb_status ensure_sms() {
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  g_sms_ops = di.sms;
  return VQB_OK;
}

unsigned grid_for(int64_t work) {
  int64_t b = (work + 255) / 256;
  if (b > 8 * static_cast<int64_t>(g_sms_ops)) b = 8 * static_cast<int64_t>(g_sms_ops);
  return static_cast<unsigned>(b < 1 ? 1 : b);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
vqb_status launch_swiglu(const void* g, const void* u, void* h, int64_t n, cudaStream_t s) {
  cudaError_t ce;
  constexpr int V = 16 / sizeof(T);
  if (n % V == 0 && aligned16(g) && aligned16(u) && aligned16(h)) {
    ce = launch_pdl(swiglu_kernel<T, V>, grid_for(n / V), 256, 0, s, static_cast<const T*>(g), static_cast<const T*>(u),
                                                        static_cast<T*>(h), n);
  } else {
    ce = launch_pdl(swiglu_kernel<T, 1>, grid_for(n), 256, 0, s, static_cast<const T*>(g), static_cast<const T*>(u),
                                                    static_cast<T*>(h), n);
  }
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

template <typename T>
vqb_status launch_combine(const void* d, const float* w, void* y, int Tn, int k, int H, cudaStream_t s) {
  cudaError_t ce;
  constexpr int V = 16 / sizeof(T);
  if (H % V == 0 && aligned16(d) && aligned16(y)) {
    ce = launch_pdl(combine_kernel<T, V>, grid_for(static_cast<int64_t>(Tn) * (H / V)), 256, 0, s,
        static_cast<const T*>(d), w, static_cast<T*>(y), Tn, k, H);
  } else {
    ce = launch_pdl(combine_kernel<T, 1>, grid_for(static_cast<int64_t>(Tn) * H), 256, 0, s, static_cast<const T*>(d), w,
                                                                               static_cast<T*>(y), Tn, k, H);
  }
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

template <typename T>
vqb_status launch_combine_partial(const void* d, const float* w, const uint32_t* skip, float* y, int Tn, int k, int H,
                                  cudaStream_t s) {
  cudaError_t ce;
  constexpr int V = 16 / sizeof(T);
  if (H % V == 0 && aligned16(d)) {
    ce = launch_pdl(combine_partial_kernel<T, V>, grid_for(static_cast<int64_t>(Tn) * (H / V)), 256, 0, s,
        static_cast<const T*>(d), w, skip, y, Tn, k, H);
  } else {
    ce = launch_pdl(combine_partial_kernel<T, 1>, grid_for(static_cast<int64_t>(Tn) * H), 256, 0, s, static_cast<const T*>(d), w,
                                                                                       skip, y, Tn, k, H);
  }
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

}  // namespace

}  // namespace vqb

using namespace vqb;

extern "C" vqb_status vqb_swiglu(const void* gate, const void* up, void* out, int64_t n, vqb_dtype dtype,
                                 vqb_stream_t stream) {
  if (n < 0) return VQB_BAD_SHAPE;
  if (n == 0) return VQB_OK;
  if (!gate || !up || !out) return VQB_NULL_POINTER;
  vqb_status st = ensure_sms();
  if (st != VQB_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == VQB_BF16) return launch_swiglu<__nv_bfloat16>(gate, up, out, n, s);
  if (dtype == VQB_F16) return launch_swiglu<__half>(gate, up, out, n, s);
  if (dtype == VQB_F32) return launch_swiglu<float>(gate, up, out, n, s);
  return VQB_BAD_SHAPE;
}

extern "C" vqb_status vqb_moe_combine(const void* expert_out, const float* weights, void* out, int32_t n_tokens,
                                      int32_t top_k, int32_t hidden, vqb_dtype dtype, vqb_stream_t stream) {
  if (n_tokens < 0 || top_k < 1 || hidden < 1) return VQB_BAD_SHAPE;
  if (n_tokens == 0) return VQB_OK;
  if (!expert_out || !weights || !out) return VQB_NULL_POINTER;
  vqb_status st = ensure_sms();
  if (st != VQB_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == VQB_BF16) return launch_combine<__nv_bfloat16>(expert_out, weights, out, n_tokens, top_k, hidden, s);
  if (dtype == VQB_F16) return launch_combine<__half>(expert_out, weights, out, n_tokens, top_k, hidden, s);
  if (dtype == VQB_F32) return launch_combine<float>(expert_out, weights, out, n_tokens, top_k, hidden, s);
  return VQB_BAD_SHAPE;
}

extern "C" vqb_status vqb_moe_combine_partial(const void* expert_out, const float* weights, const uint32_t* indices,
                                              float* out, int32_t n_tokens, int32_t top_k, int32_t hidden,
                                              vqb_dtype dtype, vqb_stream_t stream) {
  if (n_tokens < 0 || top_k < 1 || hidden < 1) return VQB_BAD_SHAPE;
  if (n_tokens == 0) return VQB_OK;
  if (!expert_out || !weights || !out) return VQB_NULL_POINTER;
  vqb_status st = ensure_sms();
  if (st != VQB_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == VQB_BF16)
    return launch_combine_partial<__nv_bfloat16>(expert_out, weights, indices, out, n_tokens, top_k, hidden, s);
  if (dtype == VQB_F16) return launch_combine_partial<__half>(expert_out, weights, indices, out, n_tokens, top_k, hidden, s);
  if (dtype == VQB_F32) return launch_combine_partial<float>(expert_out, weights, indices, out, n_tokens, top_k, hidden, s);
  return VQB_BAD_SHAPE;
}

extern "C" vqb_status vqb_moe_route(const float* logits, int32_t n_tokens, int32_t num_experts, int32_t top_k,
                                    int32_t* indices, float* weights, vqb_stream_t stream) {
  if (n_tokens < 0 || num_experts < 1 || num_experts > 8192 || top_k < 1 || top_k > 32 || top_k > num_experts)
    return VQB_BAD_SHAPE;
  if (n_tokens == 0) return VQB_OK;
  if (!logits || !indices || !weights) return VQB_NULL_POINTER;
  vqb_status st = ensure_sms();
  if (st != VQB_OK) return st;
  if (num_experts <= 1024) {
    // probabilities in registers: 8 tokens (warps) per 256-thread block
    const int nwr = 8;
    int64_t blocks = (static_cast<int64_t>(n_tokens) + nwr - 1) / nwr;
    if (blocks > 8 * static_cast<int64_t>(g_sms_ops)) blocks = 8 * static_cast<int64_t>(g_sms_ops);
    const unsigned nb = static_cast<unsigned>(blocks);
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t ce;
    if (num_experts <= 128) ce = launch_pdl(route_topk_reg_kernel<4>, nb, 256, 0, cs, logits, n_tokens, num_experts, top_k, indices, weights);
    else if (num_experts <= 256) ce = launch_pdl(route_topk_reg_kernel<8>, nb, 256, 0, cs, logits, n_tokens, num_experts, top_k, indices, weights);
    else if (num_experts <= 512) ce = launch_pdl(route_topk_reg_kernel<16>, nb, 256, 0, cs, logits, n_tokens, num_experts, top_k, indices, weights);
    else ce = launch_pdl(route_topk_reg_kernel<32>, nb, 256, 0, cs, logits, n_tokens, num_experts, top_k, indices, weights);
    if (ce != cudaSuccess) return VQB_CUDA_ERROR;
    note_launch();
    return VQB_OK;
  }
  const size_t row_bytes = sizeof(float) * static_cast<size_t>(num_experts);
  int nw = static_cast<int>((48 * 1024) / row_bytes);
  nw = nw < 1 ? 1 : (nw > 8 ? 8 : nw);
  const size_t smem = row_bytes * nw;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(route_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
          cudaSuccess)
    return VQB_CUDA_ERROR;
  cudaError_t ce;
  int64_t blocks = (static_cast<int64_t>(n_tokens) + nw - 1) / nw;
  if (blocks > 8 * static_cast<int64_t>(g_sms_ops)) blocks = 8 * static_cast<int64_t>(g_sms_ops);
  ce = launch_pdl(route_topk_kernel, static_cast<unsigned>(blocks), nw * 32, smem, reinterpret_cast<cudaStream_t>(stream), 
      logits, n_tokens, num_experts, top_k, indices, weights);
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}
