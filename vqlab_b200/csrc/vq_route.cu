// Device routing prep: group (token, slot) pairs by expert.
//
// The reference does this on the host after a device sync: a stable argsort of
// the flat expert indices, the inverse permutation and per-expert tiles
// (vq_switch.py:5372-5394, :4585-4610).  Here it stays on the device and
// produces, in the caller's workspace:
//   counts[E]          pairs per expert
//   offsets[E+1]       exclusive prefix of counts
//   sorted[N]          pair ids grouped by expert (order inside an expert is
//                      not fixed; every pair's output is computed on its own,
//                      so results do not depend on it)
//   chunks[*]          (expert, first sorted slot, pair count <= max_pairs)
//   meta[0]            number of chunks; meta[1] error flag (expert id >= E)
// One CTA handles the whole batch (decode sizes: N up to a few thousand).
#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

__global__ void __launch_bounds__(1024) route_small_kernel(const uint32_t* __restrict__ idx, int N, int E,
                                                            int max_pairs, RouteWorkspace ws) {
  extern __shared__ int sh[];
  int* cnt = sh;            // [E]
  int* cur = sh + E;        // [E]
  int* nch = sh + 2 * E;    // [E] chunks per expert, then its exclusive scan
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < N; p += blockDim.x) {
    uint32_t e = idx ? idx[p] : 0u;
    if (e >= static_cast<uint32_t>(E)) {
      ws.meta[1] = VQB_BAD_ROUTING;  // reported; the pair is routed to expert 0 so no read goes out of range
      e = 0;
    }
    atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  {
    // block-wide exclusive scans of the pair counts and of the chunk counts:
    // each thread scans a contiguous run of experts, the run totals are
    // scanned across the block through warp shuffles.
    __shared__ int2 wsum[32];
    const int per = (E + blockDim.x - 1) / blockDim.x;
    const int e0 = threadIdx.x * per, e1 = min(E, e0 + per);
    int a = 0, b = 0;
    for (int e = e0; e < e1; ++e) { a += cnt[e]; b += (cnt[e] + max_pairs - 1) / max_pairs; }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int ia = a, ib = b;
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, ia, o), tb = __shfl_up_sync(0xffffffffu, ib, o);
      if (lane >= o) { ia += ta; ib += tb; }
    }
    if (lane == 31) wsum[wid] = make_int2(ia, ib);
    __syncthreads();
    if (wid == 0) {
      int2 v = lane < static_cast<int>(blockDim.x >> 5) ? wsum[lane] : make_int2(0, 0);
      for (int o = 1; o < 32; o <<= 1) {
        const int ta = __shfl_up_sync(0xffffffffu, v.x, o), tb = __shfl_up_sync(0xffffffffu, v.y, o);
        if (lane >= o) { v.x += ta; v.y += tb; }
      }
      wsum[lane] = v;  // inclusive warp-total prefix
    }
    __syncthreads();
    int run = (wid > 0 ? wsum[wid - 1].x : 0) + ia - a;
    int chunks = (wid > 0 ? wsum[wid - 1].y : 0) + ib - b;
    for (int e = e0; e < e1; ++e) {
      ws.offsets[e] = run;
      cur[e] = run;
      run += cnt[e];
      nch[e] = chunks;
      chunks += (cnt[e] + max_pairs - 1) / max_pairs;
    }
    if (threadIdx.x == blockDim.x - 1) {
      ws.offsets[E] = wsum[(blockDim.x >> 5) - 1].x;
      ws.meta[0] = wsum[(blockDim.x >> 5) - 1].y;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    ws.counts[e] = cnt[e];
    const int n = cnt[e];
    int base = nch[e];
    for (int s = 0; s < n; s += max_pairs) {
      int4 ch;
      ch.x = e;
      ch.y = ws.offsets[e] + s;
      ch.z = min(max_pairs, n - s);
      ch.w = 0;
      ws.chunks[base++] = ch;
    }
  }
  for (int p = threadIdx.x; p < N; p += blockDim.x) {
    uint32_t e = idx ? idx[p] : 0u;
    if (e >= static_cast<uint32_t>(E)) e = 0;
    const int slot = atomicAdd(&cur[e], 1);
    ws.sorted[slot] = p;
  }
}

size_t route_workspace_bytes(int N, int E, int max_pairs) {
  (void)max_pairs;
  size_t b = 0;
  auto add = [&](size_t n) { b += (n + 255) & ~size_t(255); };
  add(sizeof(int) * 4);             // meta
  add(sizeof(int) * E);             // counts
  add(sizeof(int) * (E + 1));       // offsets
  add(sizeof(int) * (N > 0 ? N : 1));  // sorted
  add(sizeof(int4) * (N + E + 1));  // chunks (<= N + E)
  return b;
}

RouteWorkspace carve_route_workspace(void* base, int N, int E) {
  RouteWorkspace w;
  char* p = static_cast<char*>(base);
  auto take = [&](size_t n) { char* r = p; p += (n + 255) & ~size_t(255); return r; };
  w.meta = reinterpret_cast<int*>(take(sizeof(int) * 4));
  w.counts = reinterpret_cast<int*>(take(sizeof(int) * E));
  w.offsets = reinterpret_cast<int*>(take(sizeof(int) * (E + 1)));
  w.sorted = reinterpret_cast<int*>(take(sizeof(int) * (N > 0 ? N : 1)));
  w.chunks = reinterpret_cast<int4*>(take(sizeof(int4) * (N + E + 1)));
  return w;
}

vqb_status launch_route_small(const uint32_t* idx, int N, int E, int max_pairs, const RouteWorkspace& ws,
                              cudaStream_t stream) {
  const size_t smem = sizeof(int) * 3 * static_cast<size_t>(E);
  if (smem > 200 * 1024) return VQB_UNSUPPORTED_GEOMETRY;
  cudaError_t ce = cudaSuccess;
  if (smem > 48 * 1024)
    ce = cudaFuncSetAttribute(route_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(smem));
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  route_small_kernel<<<1, 1024, smem, stream>>>(idx, N, E, max_pairs, ws);
  return cudaGetLastError() == cudaSuccess ? VQB_OK : VQB_CUDA_ERROR;
}

}  // namespace vqb
