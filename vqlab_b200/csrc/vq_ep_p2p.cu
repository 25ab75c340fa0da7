// Expert-parallel exchange over peer memory: the fixed-shape decode step of an
// expert-sharded MoE layer without NCCL.  No reference counterpart (the
// reference runs every expert on one device); the layer it serves is the
// reference block of tests/test_qwen3_5_parity.py:180-204.
//
// Each rank owns one region (layout in include/vqb.h) and maps the others'
// through CUDA IPC.  Three kernels per step, one stream:
//   dispatch  every block writes (destination rank, token row) items straight
//             into the destination's region -- the row (16-byte stores over
//             NVLink, skipped when the token has no pair there), the row's
//             expert slots mapped to the destination's local ids, its weights;
//   combine   every thread sums the slots of one gathered token's 8 hidden
//             values that this rank served (fp32, slot order, each product
//             rounded: vqb_moe_combine_partial's arithmetic) and stores them
//             straight into the owning rank's partials block;
//   reduce    the owner adds the ranks' partials in rank order, rounds once.
// Dispatch and combine end the same way: every thread fences its stores at
// system scope, the last block to finish (a counter in the own region)
// release-stores the step's epoch into each rank's signal word for this
// rank, then acquire-polls this rank's signal words until every rank's epoch
// has arrived, for at most the wait limit (%globaltimer); on expiry it records
// VQB_TIMEOUT in the status word and returns.  The epoch (own region) advances
// at the end of combine.  One region per rank suffices: a rank writes step e+1
// rows into a peer only after that peer's step e partials reached it, i.e. after
// the peer finished every kernel that reads its step e rows, and it writes step
// e+1 partials only after the peer's step e+1 rows signal, which the peer
// sends after its step e reduce.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstddef>
#include <cstring>

#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

namespace {

constexpr int kEpMaxWorld = VQB_EP_MAX_WORLD;
constexpr size_t kEpControlBytes = 512;
constexpr uint32_t kEpSkip = 0xFFFFFFFFu;

// control block at the start of every region
struct EpControl {
  uint32_t sig[2][32];   // [dispatch | combine][source rank]: epoch of the source's last signal
  uint32_t epoch;        // steps completed (own rank only)
  uint32_t done[3];      // blocks finished in the running dispatch / combine launch
  int32_t status;        // VQB_TIMEOUT once a wait gave up
};
static_assert(sizeof(EpControl) <= kEpControlBytes, "control block");
static_assert(offsetof(EpControl, status) == VQB_EP_STATUS_OFFSET, "status offset is part of the ABI");

struct EpOffsets {
  size_t x, slots, weights, partials, total;
};

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

EpOffsets ep_offsets(const vqb_ep_layout& L) {
  const size_t rows = static_cast<size_t>(L.world) * L.tokens;
  EpOffsets o;
  o.x = kEpControlBytes;
  o.slots = o.x + round256(rows * L.hidden * 2);
  o.weights = o.slots + round256(rows * L.top_k * 4);
  o.partials = o.weights + round256(rows * L.top_k * 4);
  o.total = o.partials + round256(rows * L.hidden * 4);
  return o;
}

bool layout_ok(const vqb_ep_layout* L) {
  return L && L->world >= 1 && L->world <= kEpMaxWorld && L->rank >= 0 && L->rank < L->world && L->tokens >= 1 &&
         L->top_k >= 1 && L->top_k <= 256 && L->hidden >= 8 && L->hidden % 8 == 0 && L->experts_per_rank >= 1 &&
         static_cast<int64_t>(L->world) * L->tokens * L->hidden <= (int64_t(1) << 31);
}

struct EpArgs {
  char* region[kEpMaxWorld];  // [world]: own at [rank], peers mapped
  int world, rank, C, k, H, el;
  size_t off_x, off_slots, off_weights, off_partials;
  int phases;
  uint64_t limit_ns;
};

__device__ __forceinline__ EpControl* control(char* region) { return reinterpret_cast<EpControl*>(region); }

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ep_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// true once *w has reached epoch e; false when limit_ns elapsed first
__device__ bool wait_epoch(const uint32_t* w, uint32_t e, uint64_t limit_ns) {
  if (static_cast<int32_t>(ld_acquire_sys(w) - e) >= 0) return true;
  const uint64_t t0 = ep_now_ns();
  for (uint32_t i = 1;; ++i) {
    if (static_cast<int32_t>(ld_acquire_sys(w) - e) >= 0) return true;
    if ((i & 15u) == 0u && ep_now_ns() - t0 > limit_ns) return false;
    __nanosleep(100);
  }
}

// Every thread's stores fenced at system scope; true in the last block of the launch to get here.
__device__ bool last_block_done(uint32_t* counter) {
  __shared__ int s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(counter, 1u);
    s_last = prev == gridDim.x - 1;
    if (s_last) atomicExch(counter, 0u);  // ready for the next launch (stream-ordered)
  }
  __syncthreads();
  return s_last != 0;
}

// The last block: signal every rank (phase 1), wait for every rank's signal (phase 2).
__device__ void signal_and_wait(const EpArgs& a, int which, uint32_t e, bool advance_epoch) {
  EpControl* own = control(a.region[a.rank]);
  const int t = threadIdx.x;
  if ((a.phases & 1) && t < a.world) {
    __threadfence_system();
    st_release_sys(&control(a.region[t])->sig[which][a.rank], e);
  }
  if (a.phases & 2) {
    const bool ok = t >= a.world || wait_epoch(&own->sig[which][t], e, a.limit_ns);
    if (!ok) atomicExch(&own->status, static_cast<int32_t>(VQB_TIMEOUT));
    __syncthreads();
    if (advance_epoch && t == 0) *reinterpret_cast<volatile uint32_t*>(&own->epoch) = e;
  }
}

__device__ __forceinline__ uint32_t step_epoch(const EpArgs& a) {
  return *reinterpret_cast<volatile const uint32_t*>(&control(a.region[a.rank])->epoch) + 1u;
}

// one block per (destination, token row) item, grid-strided
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpArgs a, const uint4* __restrict__ x, int n_tokens,
                                                          const int32_t* __restrict__ idx,
                                                          const float* __restrict__ w) {
  const uint32_t e = step_epoch(a);
  if (a.phases & 1) {
    __shared__ int s_any;
    const int vpr = a.H / 8;  // 16-byte vectors per row
    const int items = a.world * a.C;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
      const int p = it / a.C, c = it - p * a.C;
      char* dst = a.region[p];
      const int64_t row = static_cast<int64_t>(a.rank) * a.C + c;
      if (threadIdx.x == 0) s_any = 0;
      __syncthreads();
      if (threadIdx.x < a.k) {
        const int j = threadIdx.x;
        uint32_t id = kEpSkip;
        float wt = 0.0f;
        if (c < n_tokens) {
          const int32_t g = idx[static_cast<int64_t>(c) * a.k + j];
          const int32_t lo = p * a.el;
          if (g >= lo && g - lo < a.el) {
            id = static_cast<uint32_t>(g - lo);
            s_any = 1;  // benign race: every writer stores 1
          }
          wt = w[static_cast<int64_t>(c) * a.k + j];
        }
        reinterpret_cast<uint32_t*>(dst + a.off_slots)[row * a.k + j] = id;
        reinterpret_cast<float*>(dst + a.off_weights)[row * a.k + j] = wt;
      }
      __syncthreads();
      if (s_any) {
        uint4* out = reinterpret_cast<uint4*>(dst + a.off_x) + row * vpr;
        const uint4* in = x + static_cast<int64_t>(c) * vpr;
        for (int v = threadIdx.x; v < vpr; v += blockDim.x) out[v] = __ldg(in + v);
      }
      __syncthreads();  // s_any is rewritten by the next item
    }
  }
  if (!last_block_done(&control(a.region[a.rank])->done[0])) return;
  signal_and_wait(a, 0, e, false);
}

template <typename T>
__device__ __forceinline__ float ep_to_f(T v);
template <>
__device__ __forceinline__ float ep_to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float ep_to_f<__half>(__half v) { return __half2float(v); }

// one thread = 8 hidden values of one gathered token: 16 bytes of each served slot in, 32 bytes out
template <typename T>
__global__ void __launch_bounds__(256) ep_combine_kernel(EpArgs a, const T* __restrict__ d) {
  const uint32_t e = step_epoch(a);
  if (a.phases & 1) {
    const char* own = a.region[a.rank];
    const uint32_t* slots = reinterpret_cast<const uint32_t*>(own + a.off_slots);
    const float* wts = reinterpret_cast<const float*>(own + a.off_weights);
    const int per_tok = a.H / 8;
    const int64_t total = static_cast<int64_t>(a.world) * a.C * per_tok;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int t = static_cast<int>(i / per_tok);
      const int cv = static_cast<int>(i - static_cast<int64_t>(t) * per_tok);
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
      for (int j = 0; j < a.k; ++j) {
        const int64_t pj = static_cast<int64_t>(t) * a.k + j;
        if (slots[pj] == kEpSkip) continue;
        const float wj = wts[pj];
        T v[8];
        *reinterpret_cast<uint4*>(v) = __ldg(reinterpret_cast<const uint4*>(d + pj * a.H) + cv);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(ep_to_f(v[q]), wj));
      }
      const int s = t / a.C, c = t - s * a.C;  // owner rank and its token row
      float4* out = reinterpret_cast<float4*>(a.region[s] + a.off_partials) +
                    ((static_cast<int64_t>(a.rank) * a.C + c) * a.H) / 4 + 2 * cv;
      out[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      out[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
  if (!last_block_done(&control(a.region[a.rank])->done[1])) return;
  signal_and_wait(a, 1, e, true);
}

template <typename T>
__device__ __forceinline__ T ep_from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 ep_from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half ep_from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float ep_from_f<float>(float v) { return v; }

// one thread = 4 hidden values of one token: the ranks' partials in rank order, one rounding
template <typename TY>
__global__ void __launch_bounds__(256) ep_reduce_kernel(const float4* __restrict__ part, TY* __restrict__ y,
                                                        int n_tokens, int C, int H, int world) {
  const int per_tok = H / 4;
  const int64_t total = static_cast<int64_t>(n_tokens) * per_tok;
  const int64_t rank_stride = static_cast<int64_t>(C) * per_tok;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 s = part[i];
    for (int r = 1; r < world; ++r) {
      const float4 v = part[r * rank_stride + i];
      s.x = __fadd_rn(s.x, v.x);
      s.y = __fadd_rn(s.y, v.y);
      s.z = __fadd_rn(s.z, v.z);
      s.w = __fadd_rn(s.w, v.w);
    }
    TY* o = y + i * 4;
    o[0] = ep_from_f<TY>(s.x);
    o[1] = ep_from_f<TY>(s.y);
    o[2] = ep_from_f<TY>(s.z);
    o[3] = ep_from_f<TY>(s.w);
  }
}

thread_local int g_ep_sms = 0;  // the current device's SM count, refreshed by ep_sms()

vqb_status ep_sms() {
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  g_ep_sms = di.sms;
  return VQB_OK;
}

vqb_status make_args(const vqb_ep_layout* L, void* const* regions, const vqb_ep_options* opts, EpArgs* a) {
  if (!layout_ok(L)) return VQB_BAD_SHAPE;
  if (!regions) return VQB_NULL_POINTER;
  const EpOffsets o = ep_offsets(*L);
  *a = EpArgs{};
  for (int r = 0; r < L->world; ++r) {
    if (!regions[r]) return VQB_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(regions[r]) & 255) != 0) return VQB_BAD_ALIGNMENT;
    a->region[r] = static_cast<char*>(regions[r]);
  }
  a->world = L->world;
  a->rank = L->rank;
  a->C = L->tokens;
  a->k = L->top_k;
  a->H = L->hidden;
  a->el = L->experts_per_rank;
  a->off_x = o.x;
  a->off_slots = o.slots;
  a->off_weights = o.weights;
  a->off_partials = o.partials;
  const int ph = opts ? opts->phases : 0;
  if (ph < 0 || ph > 3) return VQB_BAD_SHAPE;
  a->phases = ph == 0 ? 3 : ph;
  const int64_t us = opts && opts->wait_limit_us > 0 ? opts->wait_limit_us : 2000000;
  a->limit_ns = static_cast<uint64_t>(us) * 1000u;
  return ep_sms();
}

unsigned ep_grid(int64_t work, int per_sm) {
  int64_t b = work;
  const int64_t cap = static_cast<int64_t>(per_sm) * g_ep_sms;
  if (b > cap) b = cap;
  return static_cast<unsigned>(b < 1 ? 1 : b);
}

}  // namespace

}  // namespace vqb

using namespace vqb;

extern "C" size_t vqb_ep_region_bytes(const vqb_ep_layout* layout, size_t* offsets) {
  if (!layout_ok(layout)) return 0;
  const EpOffsets o = ep_offsets(*layout);
  if (offsets) {
    offsets[0] = o.x;
    offsets[1] = o.slots;
    offsets[2] = o.weights;
    offsets[3] = o.partials;
  }
  return o.total;
}

extern "C" vqb_status vqb_ep_region_alloc(const vqb_ep_layout* layout, void** region) {
  if (!region) return VQB_NULL_POINTER;
  *region = nullptr;
  const size_t n = vqb_ep_region_bytes(layout, nullptr);
  if (n == 0) return VQB_BAD_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, n) != cudaSuccess) return VQB_CUDA_ERROR;
  if (cudaMemset(p, 0, n) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return VQB_CUDA_ERROR;
  }
  *region = p;
  return VQB_OK;
}

extern "C" vqb_status vqb_ep_region_free(void* region) {
  if (!region) return VQB_OK;
  return cudaFree(region) == cudaSuccess ? VQB_OK : VQB_CUDA_ERROR;
}

extern "C" vqb_status vqb_ep_ipc_handle(void* region, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == VQB_EP_IPC_HANDLE_BYTES, "IPC handle size");
  if (!region || !handle) return VQB_NULL_POINTER;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, region) != cudaSuccess) return VQB_CUDA_ERROR;
  memcpy(handle, &h, sizeof(h));
  return VQB_OK;
}

extern "C" vqb_status vqb_ep_ipc_open(const void* handle, void** peer_region) {
  if (!handle || !peer_region) return VQB_NULL_POINTER;
  *peer_region = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return VQB_CUDA_ERROR;
  *peer_region = p;
  return VQB_OK;
}

extern "C" vqb_status vqb_ep_ipc_close(void* peer_region) {
  if (!peer_region) return VQB_OK;
  return cudaIpcCloseMemHandle(peer_region) == cudaSuccess ? VQB_OK : VQB_CUDA_ERROR;
}

extern "C" vqb_status vqb_ep_dispatch(const vqb_ep_layout* layout, void* const* regions, const void* x,
                                      vqb_dtype x_dtype, int32_t n_tokens, const int32_t* indices,
                                      const float* weights, const vqb_ep_options* opts, vqb_stream_t stream) {
  EpArgs a;
  vqb_status st = make_args(layout, regions, opts, &a);
  if (st != VQB_OK) return st;
  if (x_dtype != VQB_BF16 && x_dtype != VQB_F16) return VQB_UNSUPPORTED_GEOMETRY;
  if (n_tokens < 0 || n_tokens > layout->tokens) return VQB_BAD_SHAPE;
  if (n_tokens > 0 && (!x || !indices || !weights)) return VQB_NULL_POINTER;
  if (n_tokens > 0 && (reinterpret_cast<uintptr_t>(x) & 15) != 0) return VQB_BAD_ALIGNMENT;
  const unsigned grid = ep_grid(static_cast<int64_t>(layout->world) * layout->tokens, 4);
  ep_dispatch_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      a, static_cast<const uint4*>(x), n_tokens, indices, weights);
  if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

extern "C" vqb_status vqb_ep_combine(const vqb_ep_layout* layout, void* const* regions, const void* expert_out,
                                     vqb_dtype dtype, const vqb_ep_options* opts, vqb_stream_t stream) {
  EpArgs a;
  vqb_status st = make_args(layout, regions, opts, &a);
  if (st != VQB_OK) return st;
  if (!expert_out) return VQB_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(expert_out) & 15) != 0) return VQB_BAD_ALIGNMENT;
  const int64_t work = static_cast<int64_t>(layout->world) * layout->tokens * (layout->hidden / 8);
  const unsigned grid = ep_grid((work + 255) / 256, 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == VQB_BF16) {
    ep_combine_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a, static_cast<const __nv_bfloat16*>(expert_out));
  } else if (dtype == VQB_F16) {
    ep_combine_kernel<__half><<<grid, 256, 0, s>>>(a, static_cast<const __half*>(expert_out));
  } else {
    return VQB_UNSUPPORTED_GEOMETRY;
  }
  if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

extern "C" vqb_status vqb_ep_reduce(const vqb_ep_layout* layout, void* region, void* y, vqb_dtype y_dtype,
                                    int32_t n_tokens, vqb_stream_t stream) {
  if (!layout_ok(layout)) return VQB_BAD_SHAPE;
  if (n_tokens < 0 || n_tokens > layout->tokens) return VQB_BAD_SHAPE;
  if (n_tokens == 0) return VQB_OK;
  if (!region || !y) return VQB_NULL_POINTER;
  vqb_status st = ep_sms();
  if (st != VQB_OK) return st;
  const EpOffsets o = ep_offsets(*layout);
  const float4* part = reinterpret_cast<const float4*>(static_cast<const char*>(region) + o.partials);
  const int64_t work = static_cast<int64_t>(n_tokens) * (layout->hidden / 4);
  const unsigned grid = ep_grid((work + 255) / 256, 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int C = layout->tokens, H = layout->hidden, W = layout->world;
  if (y_dtype == VQB_BF16) {
    ep_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(part, static_cast<__nv_bfloat16*>(y), n_tokens, C, H, W);
  } else if (y_dtype == VQB_F16) {
    ep_reduce_kernel<__half><<<grid, 256, 0, s>>>(part, static_cast<__half*>(y), n_tokens, C, H, W);
  } else if (y_dtype == VQB_F32) {
    ep_reduce_kernel<float><<<grid, 256, 0, s>>>(part, static_cast<float*>(y), n_tokens, C, H, W);
  } else {
    return VQB_UNSUPPORTED_GEOMETRY;
  }
  if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}
