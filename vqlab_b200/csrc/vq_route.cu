// Device routing prep: group (token, slot) pairs by expert.
//
// The reference does this on the host after a device sync: a stable argsort of
// the flat expert indices, the inverse permutation and per-expert tiles
// (vq_switch.py:5372-5394, :4585-4610).  Here it stays on the device and
// produces, in the caller's workspace:
//   counts[E]          pairs per expert
//   offsets[E+1]       exclusive prefix of counts
//   sorted[N]          pair ids grouped by expert, ascending inside an expert
//                      (a stable counting sort, like the reference's stable
//                      argsort), so tile contents -- and with them the
//                      GEMM's summation order -- are the same on every call
//   chunks[*]          (expert, first sorted slot, pair count <= max_pairs)
//   meta[0]            number of chunks; meta[1] error flag (expert id >= E,
//                      other than kSkipExpert, which marks a pair to leave out);
//                      the kernel clears meta[0..3] first
// One CTA handles the whole batch.  Warp w owns the contiguous pair range
// [w*per, (w+1)*per): it counts its pairs per expert into its own row of a
// [32][E] shared table (lanes of a warp that share an expert are grouped with
// bit ballots, the lowest lane adds the group's size), the table is
// scanned over warps per expert, and the warp walks its range again placing
// each pair at its expert's running slot.
#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

namespace {

constexpr int kRouteWarpsMax = 32;   // 1024 threads; small batches use 8 warps (less table to clear)

// The pair's expert, kSkipExpert for a pair to leave out (no chunk holds it,
// its output row is not written), else an index >= E is reported and the
// pair routed to expert 0 so no read goes out of range.
__device__ __forceinline__ uint32_t expert_of(const uint32_t* idx, int p, int E, int* meta) {
  uint32_t e = idx ? idx[p] : 0u;
  if (e == kSkipExpert) return e;
  if (e >= static_cast<uint32_t>(E)) {
    meta[1] = VQB_BAD_ROUTING;
    e = 0;
  }
  return e;
}

// Lanes of the warp holding the same key (key < 2^nbits): the AND over the
// key's bits of each bit's ballot or its complement.  nbits ballots replace
// __match_any_sync, which is slow when most lanes hold distinct keys (random
// routing: ~30 distinct experts per 32 pairs).
__device__ __forceinline__ uint32_t same_key_lanes(uint32_t key, int nbits) {
  uint32_t peers = 0xFFFFFFFFu;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (key >> b) & 1u;
    const uint32_t m = __ballot_sync(0xFFFFFFFFu, bit);
    peers &= bit ? m : ~m;
  }
  return peers;
}

}  // namespace

template <int kRouteWarps>
__global__ void __launch_bounds__(kRouteWarps * 32) route_small_kernel(const uint32_t* __restrict__ idx, int N, int E,
                                                                        int max_pairs, RouteWorkspace ws) {
  extern __shared__ int sh[];
  int* cnt = sh;                 // [E]
  int* nch = sh + E;             // [E] chunk-count prefix
  int* tab = sh + 2 * E;         // [kRouteWarps][E] per-warp counts, then per-warp running slots
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int per = (N + kRouteWarps - 1) / kRouteWarps;
  // keys: the expert, or E for a lane with no pair / a skipped pair
  int nbits = 1;
  while ((1 << nbits) <= E) ++nbits;
  const int lo = min(N, wid * per), hi = min(N, lo + per);
  const uint32_t lt = (1u << lane) - 1u;

  for (int i = threadIdx.x; i < kRouteWarps * E; i += blockDim.x) tab[i] = 0;
  pdl_wait();  // the previous kernel may still read this workspace
  pdl_trigger();
  if (threadIdx.x < 4) ws.meta[threadIdx.x] = 0;  // status block, before any thread can report into it
  __syncthreads();
  // 1. per-warp counts (the range's expert ids are read kBatch steps at a
  // time, so the loads of a warp are in flight together)
  int* row = tab + wid * E;
  constexpr int kBatch = 4;
  for (int b0 = lo; b0 < hi; b0 += 32 * kBatch) {
    uint32_t eb[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int p = b0 + 32 * u + lane;
      eb[u] = p < hi ? expert_of(idx, p, E, ws.meta) : kSkipExpert;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const uint32_t e = eb[u];
      const bool valid = e != kSkipExpert;
      const uint32_t peers = same_key_lanes(valid ? e : static_cast<uint32_t>(E), nbits);
      if (valid && (peers & lt) == 0) row[e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  // 2. per expert: total, and exclusive prefix over warps
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = tab[w * E + e];
      tab[w * E + e] = run;
      run += c;
    }
    cnt[e] = run;
  }
  __syncthreads();
  {
    // block-wide exclusive scans of the pair counts and of the chunk counts:
    // each thread scans a contiguous run of experts, the run totals are
    // scanned across the block through warp shuffles.
    __shared__ int2 wsum[32];
    const int pe = (E + blockDim.x - 1) / blockDim.x;
    const int e0 = threadIdx.x * pe, e1 = min(E, e0 + pe);
    int a = 0, b = 0;
    for (int e = e0; e < e1; ++e) { a += cnt[e]; b += (cnt[e] + max_pairs - 1) / max_pairs; }
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
      for (int w = 0; w < kRouteWarps; ++w) tab[w * E + e] += run;  // running slot of warp w in expert e
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
  // 3. stable placement: warp w walks its range again in order
  for (int b0 = lo; b0 < hi; b0 += 32 * kBatch) {
    uint32_t eb[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int p = b0 + 32 * u + lane;
      uint32_t e = kSkipExpert;
      if (p < hi) {
        e = idx ? idx[p] : 0u;
        if (e != kSkipExpert && e >= static_cast<uint32_t>(E)) e = 0;
      }
      eb[u] = e;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int p = b0 + 32 * u + lane;
      const uint32_t e = eb[u];
      const bool valid = e != kSkipExpert;
      const uint32_t peers = same_key_lanes(valid ? e : static_cast<uint32_t>(E), nbits);
      if (valid) ws.sorted[row[e] + __popc(peers & lt)] = p;
      __syncwarp();
      if (valid && (peers & lt) == 0) row[e] += __popc(peers);
      __syncwarp();
    }
  }
}

size_t route_workspace_bytes(int N, int E, int max_pairs, int row_tiles) {
  (void)max_pairs;
  size_t b = 0;
  auto add = [&](size_t n) { b += (n + 255) & ~size_t(255); };
  add(sizeof(int) * 4);             // meta
  add(sizeof(int) * E);             // counts
  add(sizeof(int) * (E + 1));       // offsets
  add(sizeof(int) * (N > 0 ? N : 1));  // sorted
  add(sizeof(int4) * (N + E + 1));  // chunks (<= N + E)
  add(sizeof(int) * static_cast<size_t>(E) * (row_tiles > 0 ? row_tiles : 1));  // tile bases
  return b;
}

RouteWorkspace carve_route_workspace(void* base, int N, int E, int row_tiles) {
  RouteWorkspace w;
  char* p = static_cast<char*>(base);
  auto take = [&](size_t n) { char* r = p; p += (n + 255) & ~size_t(255); return r; };
  w.meta = reinterpret_cast<int*>(take(sizeof(int) * 4));
  w.counts = reinterpret_cast<int*>(take(sizeof(int) * E));
  w.offsets = reinterpret_cast<int*>(take(sizeof(int) * (E + 1)));
  w.sorted = reinterpret_cast<int*>(take(sizeof(int) * (N > 0 ? N : 1)));
  w.chunks = reinterpret_cast<int4*>(take(sizeof(int4) * (N + E + 1)));
  w.tile_base = reinterpret_cast<int*>(take(sizeof(int) * static_cast<size_t>(E) * (row_tiles > 0 ? row_tiles : 1)));
  return w;
}

template <int W>
static vqb_status launch_route_w(const uint32_t* idx, int N, int E, int max_pairs, const RouteWorkspace& ws,
                                 cudaStream_t stream) {
  const size_t smem = sizeof(int) * (2 + W) * static_cast<size_t>(E);
  if (smem > 200 * 1024) return VQB_UNSUPPORTED_GEOMETRY;
  cudaError_t ce = cudaSuccess;
  if (smem > 48 * 1024)
    ce = cudaFuncSetAttribute(route_small_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(smem));
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  if (launch_pdl(route_small_kernel<W>, 1, W * 32, smem, stream, idx, N, E, max_pairs, ws) != cudaSuccess)
    return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

vqb_status launch_route_small(const uint32_t* idx, int N, int E, int max_pairs, const RouteWorkspace& ws,
                              cudaStream_t stream) {
  if (N <= 256) return launch_route_w<8>(idx, N, E, max_pairs, ws, stream);
  return launch_route_w<kRouteWarpsMax>(idx, N, E, max_pairs, ws, stream);
}

}  // namespace vqb
