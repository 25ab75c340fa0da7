// The MoE block of one layer in ONE persistent launch (sm_100a): router
// top-k, routing, the gate and up projections, SwiGLU, the down projection
// and the slot combine -- the reference block of
// tests/test_qwen3_5_parity.py:180-204 (mlx_lm SwitchGLU around
// VQSwitchLinear, vq_switch.py:5284-5423) for decode batches, where the
// library's per-step kernels spend more time starting and draining than
// decoding.
//
// One CTA per SM, cooperative launch (every CTA resident), phases separated by
// grid barriers:
//   0. the CTAs narrow x to fp16 (the MoE host cast) and route the tokens
//      (one warp per token, the arithmetic of the router kernel,
//      vq_router.cuh) into the workspace; after a grid barrier every CTA
//      groups the (token, slot) pairs by expert (a stable counting sort) into
//      chunks of <= 8 tokens of one expert.  Meanwhile the copy thread loads
//      the codebook half the CTA needs first;
//   1. gate and up: CTAs form four groups (gate, up) x (dims 0-3, dims 4-7);
//      a group's CTA keeps that projection's codebook half [K][4] resident in
//      shared memory (128 KB for K = 16384) and computes, for its work items,
//      the partial product of those four dimensions: an item is (chunk, 256
//      output rows, a range of the input windows).  A window is 64 codes
//      (512 inputs) of the item's rows: code words and scales arrive by TMA,
//      the chunk's token rows by bulk copies, double-buffered;
//   2. SwiGLU: the partials of each (pair, row) are summed in a fixed order,
//      rounded as the projection outputs are (fp16, then x's dtype), and
//      h = dtype(silu(g) * u) is stored as the down projection's fp16 input;
//   3. down: two groups (dims 0-3, dims 4-7) over (chunk, 256 rows of H,
//      window range) items;
//   4. combine: y[t] = dtype(sum_j w[t, j] * d[t, j]) in slot order.
//
// The decode engine (consumer warps, 32 output rows each, two MMA row tiles
// of 16): thread (g, t) of a warp extracts four consecutive 14- or 12-bit
// codes of rows g and g + 8 of each tile from the staged code words, looks
// each up in the resident half (one 8-byte shared-memory read), scales it --
// W = fp16(cb * s), one RNE rounding, the reference's non-ACCS weights -- and
// a tile's two rows form the A operand of one mma.sync m16n8k16 per 4 codes
// against the chunk's tokens (B, 8 columns, loaded once for both tiles); the
// k order inside an MMA is permuted identically for A and B.  Partials
// are fp32; a work item's partial goes to its own slot, so every sum runs in
// a fixed order and repeated calls are bit-identical.
//
// Every wait is bounded (2 s of %globaltimer): an mbarrier wait that expires
// stops the CTA's work, a grid barrier that expires stops waiting; every CTA
// still arrives at every grid barrier, waits for its own copies in flight and
// records VQB_TIMEOUT in the workspace status block.
#include <cuda.h>

#include <algorithm>

#include "vqb_common.cuh"
#include "vqb_internal.h"
#include "vqb_tma.cuh"
#include "vq_router.cuh"

namespace vqb {

namespace {

constexpr int kMbWarps = 8;                         // consumer (decode) warps
constexpr int kMbThreads = (kMbWarps + 1) * 32;     // + the copy warp
constexpr int kMbCopyWarp = kMbWarps;
constexpr int kMbRows = 256;                        // output rows of a work item (32 per consumer warp)
constexpr int kMbTok = 8;                           // tokens of a chunk (the MMA's N)
constexpr int kMbWinK = 512;                        // inputs per window (64 d8 codes)
constexpr int kMbStages = 2;
constexpr int kMbXStride = kMbWinK * 2 + 16;        // bytes of a staged token row (padded against bank conflicts)
constexpr int kMbScaleRow = 16;                     // 8 fp16 scales (G = 64) per row per window
constexpr int kMbMaxPairs = 640;
constexpr int kMbMaxExperts = 1024;
constexpr int kMbSlotBudget = 640;                  // split slots x pairs of a partial buffer
constexpr int kMbMaxSplit = 8;

struct MbProj {
  const uint16_t* halves;  // [2][K][4] fp16
  int OUT, IN;
};

struct MbParams {
  const float* logits;     // [T, E] fp32
  const void* x;           // [T, H] bf16 / fp16
  void* y;                 // [T, H] x's dtype
  int32_t* idx_out;        // optional [T, k]
  float* w_out;            // optional [T, k]
  int T, E, k, H, I, K, x_bf16;
  MbProj proj[3];          // gate, up, down
  float* part1;            // [(proj * 2 + half) * S1 + split][pair][I]
  float* part3;            // [half * S3 + split][pair][H]
  uint16_t* h16;           // [pair][I] fp16: the down projection's input
  uint16_t* x16;           // [T][H] fp16: x narrowed once (the MoE host cast)
  int32_t* ridx;           // [T * k] routing: expert of each pair
  float* rw;               // [T * k] routing: weight of each pair
  int* status;             // workspace status block: [1] = VQB_TIMEOUT when a wait expired
  int dense;               // a dense MLP (E = 1, no router): x kept in its dtype, outputs rounded once
  uint64_t wait_ns;        // limit of the bounded mbarrier waits
  int stall_cta;           // tests: this CTA waits for a signal nothing sends (-1: none)
};

struct MbMaps {
  CUtensorMap codes[3];    // uint32 [E * OUT][row words], box (2 * BITS words) x 256 rows
  CUtensorMap scales[3];   // fp16 [E * OUT][IN / 64], box 8 x 256
};

// Shared memory: the resident codebook half, two stages of (code words,
// scales, token rows), the routing results, barriers.  The routing scratch
// (counts, offsets, expert ids) lives in stage 0 before any window is loaded.
struct MbLayout {
  uint32_t cb, codes[kMbStages], scales[kMbStages], xrows[kMbStages], w, sorted, chunks, bars, total;
};

__host__ __device__ inline uint32_t mb_align(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline MbLayout mb_layout(int K, int words) {
  MbLayout L;
  uint32_t off = 0;
  L.cb = off;
  off = mb_align(off + static_cast<uint32_t>(K) * 8u, 128);
  for (int s = 0; s < kMbStages; ++s) {
    L.codes[s] = off;
    off = mb_align(off + kMbRows * static_cast<uint32_t>(words) * 4u, 128);
    L.scales[s] = off;
    off = mb_align(off + kMbRows * kMbScaleRow, 128);
    L.xrows[s] = off;
    off = mb_align(off + kMbTok * kMbXStride, 128);
  }
  L.w = off;
  off = mb_align(off + 4u * kMbMaxPairs, 16);
  L.sorted = off;
  off = mb_align(off + 2u * kMbMaxPairs, 16);
  L.chunks = off;
  off = mb_align(off + 8u * kMbMaxPairs, 16);
  L.bars = off;
  off += 8u * 8u + 4u * 64u;  // 5 mbarriers (+ spare), 64 ints of CTA state
  L.total = off;
  return L;
}

// CTA state words after the barriers
constexpr int kStAbort = 0, kStChunks = 1, kStErr = 4, kStBarOk = 5, kStScan = 8;  // scan: 16 int2 from word 8

// Split of a phase's windows: S pieces per (chunk, row block) minimising the
// busiest CTA's windows (+ 1/8 window per item: its partial store), slots
// S * P within the partial buffer.
__device__ __forceinline__ int mb_split(int nseg, int ng, int nw, int P) {
  // lane S - 1 prices S (32-bit divisions: nseg * S stays far below 2^32), then
  // the warp takes the smallest cost, the smaller S among equal costs; every
  // lane of the calling warp gets the answer
  int smax = nw < kMbMaxSplit ? nw : kMbMaxSplit;
  const int cap = kMbSlotBudget / P > 1 ? kMbSlotBudget / P : 1;
  if (smax > cap) smax = cap;
  const int lane = static_cast<int>(threadIdx.x & 31u);
  int best = lane + 1;
  long long best_cost = 0x7fffffffffffffffLL;
  if (best <= smax) {
    const unsigned items = (static_cast<unsigned>(nseg) * static_cast<unsigned>(best) + static_cast<unsigned>(ng) - 1u) /
                           static_cast<unsigned>(ng);
    best_cost = static_cast<long long>(items) * (8LL * ((nw + best - 1) / best) + 1);
  }
  for (int o = 16; o; o >>= 1) {
    const long long oc = __shfl_xor_sync(0xffffffffu, best_cost, o);
    const int os = __shfl_xor_sync(0xffffffffu, best, o);
    if (oc < best_cost || (oc == best_cost && os < best)) {
      best_cost = oc;
      best = os;
    }
  }
  return best;
}

// slots of a partial buffer for P pairs: S * P for every S mb_split may pick
__host__ __device__ inline int mb_slots(int P) {
  const int a = P > kMbSlotBudget ? P : kMbSlotBudget;
  return a < kMbMaxSplit * P ? a : kMbMaxSplit * P;
}

// ------------------------------------------------------------ device helpers

// Grid-wide arrivals of this device's fused-block launches.  Every CTA of a
// launch arrives exactly once at each of its four barriers -- also after a
// timeout -- so a launch advances the count by 4 * gridDim.x and a barrier's
// round is (count before the arrival) / gridDim.x.  Zero when the module loads.
__device__ unsigned long long g_mb_arrivals;

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Arrive; when `wait`, wait (bounded) until every CTA of the grid arrived.
// Returns false when the wait was skipped or expired.
__device__ bool mb_grid_barrier(bool wait, int* st) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long old = atomicAdd(&g_mb_arrivals, 1ull);
    // round = old / grid, through an fp64 quotient made exact (a 64-bit
    // integer division is a long serial routine)
    const unsigned long long grid = gridDim.x;
    unsigned long long round = static_cast<unsigned long long>(static_cast<double>(old) / static_cast<double>(grid));
    while (round * grid > old) --round;
    while ((round + 1ull) * grid <= old) ++round;
    const unsigned long long target = (round + 1ull) * grid;
    int ok = wait ? 1 : 0;
    if (wait) {
      const uint64_t t0 = global_ns();
      while (ld_acquire_u64(&g_mb_arrivals) < target) {
        if (global_ns() - t0 > kWaitLimitNs) {
          ok = 0;
          st[kStErr] = 1;
          break;
        }
        __nanosleep(32);
      }
    }
    __threadfence();
    st[kStBarOk] = ok;
  }
  __syncthreads();
  return st[kStBarOk] != 0;
}

__device__ __forceinline__ uint32_t sel4(int t, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return (t & 2) ? ((t & 1) ? d : c) : ((t & 1) ? b : a);
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// two bf16 -> two fp16, round to nearest even (the MoE host cast of x)
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) {
  const float lo = __uint_as_float(v << 16), hi = __uint_as_float(v & 0xFFFF0000u);
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_16816_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// two fp16 -> two bf16, round to nearest even (the dense weights' cast to x's dtype)
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t v) {
  const float2 f = __half22float2(*reinterpret_cast<__half2*>(&v));
  __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<uint32_t*>(&b);
}

// the output rounding of a projection: fp16, then x's dtype (the MoE
// projections, vq_switch.py:5423); a dense layer rounds its fp32 accumulator
// to x's dtype once (vq_dense.py:294-312)
__device__ __forceinline__ float round_out(float v, int x_bf16, int dense = 0) {
  if (dense && x_bf16) return __bfloat162float(__float2bfloat16_rn(v));
  const __half h = __float2half_rn(v);
  return x_bf16 ? __bfloat162float(__float2bfloat16_rn(__half2float(h))) : __half2float(h);
}

__device__ __forceinline__ float mb_silu(float v) { return v / (1.0f + expf(-v)); }

// One window (64 codes) of a work item for one consumer warp: output rows
// 32 * warp + 16 * j + g and + 8 for tiles j = 0, 1 of the item's 256, this
// CTA's dimension half h.  Thread t takes codes 4t .. 4t+3 of each group of
// 16; for code c the MMA's k slots (2t, 2t+1, 2t+8, 2t+9) hold dims 4h .. 4h+3
// of W (A) and of x (B).
template <int BITS, bool WBF16>
__device__ __forceinline__ void mb_window(const uint32_t* __restrict__ cw, const uint16_t* __restrict__ sc,
                                          const unsigned char* __restrict__ xr, const uint16_t* __restrict__ cb,
                                          int warp, int g, int t, int n, int h, float (&acc)[2][4]) {
  constexpr int W = 2 * BITS;                     // words of a row's window
  constexpr int QW = BITS / 2;                    // words per 16 codes
  constexpr int o1 = (4 * BITS) >> 5, o2 = (8 * BITS) >> 5, o3 = (12 * BITS) >> 5;  // word of code 4t, t = 1..3
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  // rows: [0] tile 0 row g, [1] tile 0 row g+8, [2] tile 1 row g, [3] tile 1 row g+8
  const uint32_t* rows[4];
  uint4 scl[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int rr = warp * 32 + (r >> 1) * 16 + (r & 1) * 8 + g;
    rows[r] = cw + rr * W;
    scl[r] = *reinterpret_cast<const uint4*>(sc + rr * 8);
  }
  const int sh = (t * 4 * BITS) & 31;
  const bool has_x = g < n;
  const unsigned char* xg = xr + g * kMbXStride + 8 * h;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int wq0 = q * QW;
    const int wq1 = wq0 + o3 + 2 < W - 1 ? wq0 + o3 + 2 : W - 1;
    uint64_t v[4];
    uint32_t s2[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      uint32_t wd[W];  // only the units [wq0 / 4, wq1 / 4] are loaded
#pragma unroll
      for (int u = wq0 / 4; u <= wq1 / 4; ++u) {
        const uint4 x4 = *reinterpret_cast<const uint4*>(rows[r] + 4 * u);
        wd[4 * u] = x4.x;
        wd[4 * u + 1] = x4.y;
        wd[4 * u + 2] = x4.z;
        wd[4 * u + 3] = x4.w;
      }
      // thread t's three words (the third is unused when its four codes end in the second)
      uint32_t w3[3];
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        const int i0 = wq0 + i, i1 = wq0 + o1 + i, i2 = wq0 + o2 + i, i3 = wq0 + o3 + i;
        w3[i] = sel4(t, wd[i0 < W ? i0 : W - 1], wd[i1 < W ? i1 : W - 1], wd[i2 < W ? i2 : W - 1],
                     wd[i3 < W ? i3 : W - 1]);
      }
      v[r] = static_cast<uint64_t>(__funnelshift_r(w3[0], w3[1], sh)) |
             (static_cast<uint64_t>(__funnelshift_r(w3[1], w3[2], sh)) << 32);
      // scale group of codes 16q + 4t .. (G = 64: 8 codes): 2q + t / 2
      const uint32_t qs = q == 0 ? scl[r].x : (q == 1 ? scl[r].y : (q == 2 ? scl[r].z : scl[r].w));
      const uint32_t hs = (t & 2) ? (qs >> 16) : (qs & 0xFFFFu);
      s2[r] = hs | (hs << 16);
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      uint32_t x0 = 0, x1 = 0;
      if (has_x) {
        const uint2 xv = *reinterpret_cast<const uint2*>(xg + 16 * (16 * q + 4 * t + s));
        x0 = xv.x;
        x1 = xv.y;
      }
      uint2 e[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint32_t c = static_cast<uint32_t>(v[r] >> (BITS * s)) & kMask;
        e[r] = *reinterpret_cast<const uint2*>(cb + c * 4);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t w0 = hmul2_bits(e[2 * j].x, s2[2 * j]), w1 = hmul2_bits(e[2 * j + 1].x, s2[2 * j + 1]);
        uint32_t w2 = hmul2_bits(e[2 * j].y, s2[2 * j]), w3 = hmul2_bits(e[2 * j + 1].y, s2[2 * j + 1]);
        if constexpr (WBF16) {
          mma_16816_bf16(acc[j], f16x2_to_bf16x2(w0), f16x2_to_bf16x2(w1), f16x2_to_bf16x2(w2),
                         f16x2_to_bf16x2(w3), x0, x1);
        } else {
          mma_16816(acc[j], w0, w1, w2, w3, x0, x1);
        }
      }
    }
  }
}

// A phase's work: items (chunk, 256-row block, split) of this CTA's group.
struct MbPhase {
  int proj, half, j, ng, S, nseg, rts, nw, OUT;
  float* part;
  int pg;       // partial group: slots [pg * S, pg * S + S)
  bool x_h16;   // token rows from h16 (down) instead of x16 (gate / up)
};

struct MbItem {
  int c, rt, s, w0, w1;
};

__device__ __forceinline__ MbItem mb_item(const MbPhase& ph, int i) {
  MbItem it;
  const int seg = i / ph.S;
  it.s = i - seg * ph.S;
  it.c = seg / ph.rts;
  it.rt = seg - it.c * ph.rts;
  it.w0 = it.s * ph.nw / ph.S;
  it.w1 = (it.s + 1) * ph.nw / ph.S;
  return it;
}

// copy thread: the code window, scales and token rows of every window of the
// phase's items into the stages (gw counts windows over the whole launch)
template <int BITS>
__device__ void mb_produce(const CUtensorMap* cmap, const CUtensorMap* smap, const MbParams& prm, const MbPhase& ph,
                           const uint2* chunks, const uint16_t* sorted, unsigned char* smem, const MbLayout& L,
                           uint64_t* full, uint64_t* empty, uint32_t& gw, volatile int* abort_flag) {
  constexpr int W = 2 * BITS;
  const int items = ph.nseg * ph.S;
  for (int i = ph.j; i < items; i += ph.ng) {
    const MbItem it = mb_item(ph, i);
    const uint2 ch = chunks[it.c];
    const int e = static_cast<int>(ch.x & 0xFFFFu), n = static_cast<int>(ch.x >> 16), start = static_cast<int>(ch.y);
    const int row0 = e * ph.OUT + it.rt * kMbRows;
    for (int w = it.w0; w < it.w1; ++w) {
      const int st = static_cast<int>(gw & 1u);
      if (!mbar_wait(&empty[st], ((gw >> 1) & 1u) ^ 1u, abort_flag, prm.wait_ns)) return;
      mbar_expect_tx(&full[st], kMbRows * W * 4 + kMbRows * kMbScaleRow + n * kMbWinK * 2);
      tma_load_2d(cmap, &full[st], smem + L.codes[st], w * W, row0);
      tma_load_2d(smap, &full[st], smem + L.scales[st], w * (kMbWinK / 64), row0);
      for (int m = 0; m < n; ++m) {
        const int pair = sorted[start + m];
        const unsigned char* src =
            ph.x_h16 ? reinterpret_cast<const unsigned char*>(prm.h16) +
                           (static_cast<size_t>(pair) * prm.I + static_cast<size_t>(w) * kMbWinK) * 2
                     : reinterpret_cast<const unsigned char*>(prm.x16) +
                           (static_cast<size_t>(pair / prm.k) * prm.H + static_cast<size_t>(w) * kMbWinK) * 2;
        bulk_load(smem + L.xrows[st] + m * kMbXStride, src, kMbWinK * 2, &full[st]);
      }
      ++gw;
    }
  }
}

// consumer warps: decode every window of the phase's items, then store the
// item's fp32 partial for its (pair, row) cells into the item's slot
template <int BITS, bool WBF16>
__device__ bool mb_consume(const MbParams& prm, const MbPhase& ph, const uint2* chunks, const uint16_t* sorted,
                           const unsigned char* smem, const MbLayout& L, uint64_t* full, uint64_t* empty,
                           uint32_t& gw, volatile int* abort_flag, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int P = prm.T * prm.k;
  const uint16_t* cb = reinterpret_cast<const uint16_t*>(smem + L.cb);
  const int items = ph.nseg * ph.S;
  for (int i = ph.j; i < items; i += ph.ng) {
    const MbItem it = mb_item(ph, i);
    const uint2 ch = chunks[it.c];
    const int n = static_cast<int>(ch.x >> 16), start = static_cast<int>(ch.y);
    float acc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
    for (int w = it.w0; w < it.w1; ++w) {
      const int st = static_cast<int>(gw & 1u);
      if (!warp_wait(&full[st], (gw >> 1) & 1u, abort_flag, prm.wait_ns)) return false;
      mb_window<BITS, WBF16>(reinterpret_cast<const uint32_t*>(smem + L.codes[st]),
                           reinterpret_cast<const uint16_t*>(smem + L.scales[st]), smem + L.xrows[st], cb, warp, g,
                           t, n, ph.half, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      ++gw;
    }
    // D fragments: rows g and g + 8 of each of the warp's two tiles, tokens 2t and 2t + 1
    const int r = it.rt * kMbRows + warp * 32 + g;
    float* base = ph.part + static_cast<size_t>(ph.pg * ph.S + it.s) * P * ph.OUT;
    if (2 * t < n) {
      float* o = base + static_cast<size_t>(sorted[start + 2 * t]) * ph.OUT + r;
      o[0] = acc[0][0];
      o[8] = acc[0][2];
      o[16] = acc[1][0];
      o[24] = acc[1][2];
    }
    if (2 * t + 1 < n) {
      float* o = base + static_cast<size_t>(sorted[start + 2 * t + 1]) * ph.OUT + r;
      o[0] = acc[0][1];
      o[8] = acc[0][3];
      o[16] = acc[1][1];
      o[24] = acc[1][3];
    }
  }
  return true;
}

__device__ void mb_load_half(const uint16_t* halves, int half, int K, unsigned char* dst, uint64_t* bar) {
  const unsigned char* src = reinterpret_cast<const unsigned char*>(halves + static_cast<size_t>(half) * K * 4);
  const uint32_t bytes = static_cast<uint32_t>(K) * 8u;
  mbar_expect_tx(bar, bytes);
  for (uint32_t off = 0; off < bytes; off += 8192u)
    bulk_load(dst + off, src + off, bytes - off < 8192u ? bytes - off : 8192u, bar);
}

// One token routed by all kMbWarps warps of the CTA (E <= 1024, k <= 32),
// with route_row_reg's arithmetic and result: the same max, the same exps,
// the per-lane sums added in the same order (lane l: entries l, l + 32, ...)
// and combined by the same butterfly, the same divisions; the top_k by
// (probability, then the lower id) as a per-warp top-k of each warp's entries
// merged by warp 0.  scr: >= 1600 floats of shared memory.  Warp 0 lane j < k
// receives slot j.
__device__ void mb_route_one(const float* __restrict__ row, int E, int k, float* scr, int warp, int lane, int& out_i,
                             float& out_w) {
  constexpr int NT = kMbWarps * 32;
  float* ex = scr;                                         // [1024] exp(logit - max)
  float* red = scr + kMbMaxExperts;                        // [kMbWarps] per-warp max, then [0] the sum
  float* cv = red + 32;                                    // [kMbWarps][32] per-warp top-k values
  int* ci = reinterpret_cast<int*>(cv + kMbWarps * 32);    // [kMbWarps][32] their ids
  const int tid = warp * 32 + lane;
  float lg[kMbMaxExperts / NT];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kMbMaxExperts / NT; ++j) {
    const int e = tid + NT * j;
    lg[j] = e < E ? __ldg(row + e) : -INFINITY;
    if (e < E) m = fmaxf(m, lg[j]);
  }
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  asm volatile("bar.sync 1, %0;" :: "r"(NT) : "memory");
#pragma unroll
  for (int w = 0; w < kMbWarps; ++w) m = fmaxf(m, red[w]);
#pragma unroll
  for (int j = 0; j < kMbMaxExperts / NT; ++j) {
    const int e = tid + NT * j;
    if (e < E) ex[e] = expf(lg[j] - m);
  }
  asm volatile("bar.sync 1, %0;" :: "r"(NT) : "memory");
  if (warp == 0) {
    float sum = 0.0f;
    for (int e = lane; e < E; e += 32) sum += ex[e];
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[0] = sum;
  }
  asm volatile("bar.sync 1, %0;" :: "r"(NT) : "memory");
  const float sum = red[0];
  // this thread's entries, sorted: larger probability first, the lower id among equals
  constexpr int J = kMbMaxExperts / NT;
  float p[J];
  int ix[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = tid + NT * j;
    const float q = e < E ? __fdiv_rn(ex[e], sum) : -1.0f;
    const bool live = q > -1.0f;
    p[j] = live ? q : -1.0f;
    ix[j] = live ? e : 0x7fffffff;
  }
#pragma unroll
  for (int size = 2; size <= J; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < J; ++i) {
        const int j2 = i ^ stride;
        if (j2 > i) {
          const bool i_first = p[i] > p[j2] || (p[i] == p[j2] && ix[i] < ix[j2]);
          const bool swap = ((i & size) == 0) ? !i_first : i_first;
          const float tv = p[i];
          const int ti = ix[i];
          p[i] = swap ? p[j2] : p[i];
          ix[i] = swap ? ix[j2] : ix[i];
          p[j2] = swap ? tv : p[j2];
          ix[j2] = swap ? ti : ix[j2];
        }
      }
    }
  }
  // the warp's top k, in order
  for (int r = 0; r < k; ++r) {
    const uint32_t key = p[0] >= 0.0f ? __float_as_uint(p[0]) + 1u : 0u;
    const uint32_t top = __reduce_max_sync(0xffffffffu, key);
    const uint32_t bi = __reduce_min_sync(0xffffffffu, key == top ? static_cast<uint32_t>(ix[0]) : 0xffffffffu);
    if (lane == 0) {
      cv[warp * 32 + r] = top ? __uint_as_float(top - 1u) : -1.0f;
      ci[warp * 32 + r] = top ? static_cast<int>(bi) : 0x7fffffff;
    }
    const bool pop = top != 0u && static_cast<uint32_t>(ix[0]) == bi;
#pragma unroll
    for (int i = 0; i + 1 < J; ++i) {
      p[i] = pop ? p[i + 1] : p[i];
      ix[i] = pop ? ix[i + 1] : ix[i];
    }
    p[J - 1] = pop ? -1.0f : p[J - 1];
    ix[J - 1] = pop ? 0x7fffffff : ix[J - 1];
  }
  asm volatile("bar.sync 1, %0;" :: "r"(NT) : "memory");
  if (warp == 0) {
    // merge the warps' lists: lane q < kMbWarps holds the head of list q
    int h = 0;
    float hv = lane < kMbWarps ? cv[lane * 32] : -1.0f;
    int hi = lane < kMbWarps ? ci[lane * 32] : 0x7fffffff;
    float mine_w = 0.0f, wsum = 0.0f;
    int mine_i = 0;
    for (int j = 0; j < k; ++j) {
      const uint32_t key = hv >= 0.0f ? __float_as_uint(hv) + 1u : 0u;
      const uint32_t top = __reduce_max_sync(0xffffffffu, key);
      const uint32_t bi = __reduce_min_sync(0xffffffffu, key == top ? static_cast<uint32_t>(hi) : 0xffffffffu);
      float bv = 0.0f;  // no candidate left (NaN logits): expert 0, weight 0
      int sel = 0;
      if (top != 0u) {
        bv = __uint_as_float(top - 1u);
        sel = static_cast<int>(bi);
        if (lane < kMbWarps && static_cast<uint32_t>(hi) == bi) {
          ++h;
          hv = h < k ? cv[lane * 32 + h] : -1.0f;
          hi = h < k ? ci[lane * 32 + h] : 0x7fffffff;
        }
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
}

// Phase 0a (all CTAs together): the tokens are routed into prm.ridx / prm.rw
// (and the caller's indices / weights) -- with no more tokens than CTAs, token
// t by all warps of CTA t; else token t by warp (t / nC) % warps of CTA
// t % nC -- and x is narrowed to fp16 into prm.x16, an even share of it per
// CTA.  scr: shared memory no one else uses in this phase.
__device__ void mb_route_tokens(const MbParams& prm, float* scr, int warp, int lane) {
  const int T = prm.T, E = prm.E, k = prm.k;
  const int nC = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  if (prm.dense) {
    // one expert, every token to it with weight 1
    for (int t = cta * blockDim.x + threadIdx.x; t < T; t += nC * blockDim.x) {
      prm.ridx[t] = 0;
      prm.rw[t] = 1.0f;
    }
  } else if (T <= nC) {
    if (cta < T && warp < kMbWarps) {
      int ei = 0;
      float ew = 0.0f;
      mb_route_one(prm.logits + static_cast<size_t>(cta) * E, E, k, scr, warp, lane, ei, ew);
      if (warp == 0 && lane < k) {
        prm.ridx[cta * k + lane] = ei;
        prm.rw[cta * k + lane] = ew;
        if (prm.idx_out) {
          prm.idx_out[cta * k + lane] = ei;
          prm.w_out[cta * k + lane] = ew;
        }
      }
    }
  } else if (warp < kMbWarps) {
    for (int t = cta + nC * warp; t < T; t += nC * kMbWarps) {
      const float* row = prm.logits + static_cast<size_t>(t) * E;
      int ei;
      float ew;
      if (E <= 128) route_row_reg<4>(row, E, k, lane, ei, ew);
      else if (E <= 256) route_row_reg<8>(row, E, k, lane, ei, ew);
      else if (E <= 512) route_row_reg<16>(row, E, k, lane, ei, ew);
      else route_row_reg<32>(row, E, k, lane, ei, ew);
      if (lane < k) {
        prm.ridx[t * k + lane] = ei;
        prm.rw[t * k + lane] = ew;
        if (prm.idx_out) {
          prm.idx_out[t * k + lane] = ei;
          prm.w_out[t * k + lane] = ew;
        }
      }
    }
  }
  // x -> fp16, 8 elements per thread-step (H is a multiple of 512)
  const int nv = T * prm.H / 8;  // the host keeps T * H below 2^31
  const int per = (nv + nC - 1) / nC;
  const int v0 = cta * per, v1 = v0 + per < nv ? v0 + per : nv;
  for (int v = v0 + static_cast<int>(threadIdx.x); v < v1; v += static_cast<int>(blockDim.x)) {
    uint4 u = reinterpret_cast<const uint4*>(prm.x)[v];
    if (prm.x_bf16 && !prm.dense) {
      u.x = bf16x2_to_f16x2(u.x);
      u.y = bf16x2_to_f16x2(u.y);
      u.z = bf16x2_to_f16x2(u.z);
      u.w = bf16x2_to_f16x2(u.w);
    }
    reinterpret_cast<uint4*>(prm.x16)[v] = u;
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");  // x16 is read by bulk copies after the barrier
}

// Phase 0b (consumer warps, every CTA): the routed pairs grouped by expert --
// counts, exclusive scans of pairs and of chunks (<= 8 tokens each), chunk
// records in expert order, and a stable placement (pairs keep their index
// order inside an expert).  Results: w[P] (weights), sorted[P] (pair ids in
// chunk order), chunks[NC] = (expert | n << 16, first sorted slot),
// st[kStChunks] = NC.
__device__ void mb_route(const MbParams& prm, unsigned char* scratch, float* wsm, uint16_t* sorted, uint2* chunks,
                         int* st, int warp, int lane) {
  const int T = prm.T, E = prm.E, k = prm.k, P = T * k;
  const int tid = threadIdx.x;
  int* cnt = reinterpret_cast<int*>(scratch);   // [E]
  int* poff = cnt + kMbMaxExperts;               // [E] pair offset, then the placement cursor
  int* coff = poff + kMbMaxExperts;              // [E] chunk offset
  uint16_t* eid = reinterpret_cast<uint16_t*>(coff + kMbMaxExperts);  // [P] expert of each pair
  for (int q = tid; q < P; q += kMbWarps * 32) {
    const int e = __ldcg(prm.ridx + q);
    eid[q] = static_cast<uint16_t>(e >= 0 && e < E ? e : 0);
    wsm[q] = __ldcg(prm.rw + q);
  }
  for (int e = tid; e < E; e += kMbWarps * 32) cnt[e] = 0;
  asm volatile("bar.sync 1, %0;" :: "r"(kMbWarps * 32) : "memory");
  for (int p = tid; p < P; p += kMbWarps * 32) atomicAdd(&cnt[eid[p]], 1);
  asm volatile("bar.sync 1, %0;" :: "r"(kMbWarps * 32) : "memory");
  // exclusive scans over experts (kEpt consecutive ones per thread) of pairs and of chunks
  constexpr int kEpt = kMbMaxExperts / (kMbWarps * 32);
  int2* wsum = reinterpret_cast<int2*>(st + kStScan);
  const int e0 = kEpt * tid;
  int a = 0, b = 0;
#pragma unroll
  for (int i = 0; i < kEpt; ++i) {
    const int c = e0 + i < E ? cnt[e0 + i] : 0;
    a += c;
    b += (c + kMbTok - 1) / kMbTok;
  }
  int ia = a, ib = b;
  for (int o = 1; o < 32; o <<= 1) {
    const int ta = __shfl_up_sync(0xffffffffu, ia, o), tb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ta;
      ib += tb;
    }
  }
  if (lane == 31) wsum[warp] = make_int2(ia, ib);
  asm volatile("bar.sync 1, %0;" :: "r"(kMbWarps * 32) : "memory");
  if (warp == 0) {
    int2 v = lane < kMbWarps ? wsum[lane] : make_int2(0, 0);
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, v.x, o), tb = __shfl_up_sync(0xffffffffu, v.y, o);
      if (lane >= o) {
        v.x += ta;
        v.y += tb;
      }
    }
    __syncwarp();
    if (lane < kMbWarps) wsum[lane] = v;  // inclusive over warps
  }
  asm volatile("bar.sync 1, %0;" :: "r"(kMbWarps * 32) : "memory");
  {
    int pa = (warp > 0 ? wsum[warp - 1].x : 0) + ia - a;
    int pb = (warp > 0 ? wsum[warp - 1].y : 0) + ib - b;
#pragma unroll
    for (int i = 0; i < kEpt; ++i) {
      if (e0 + i < E) {
        const int c = cnt[e0 + i];
        poff[e0 + i] = pa;
        coff[e0 + i] = pb;
        pa += c;
        pb += (c + kMbTok - 1) / kMbTok;
      }
    }
    if (tid == 0) st[kStChunks] = wsum[kMbWarps - 1].y;
  }
  asm volatile("bar.sync 1, %0;" :: "r"(kMbWarps * 32) : "memory");
  for (int e = tid; e < E; e += kMbWarps * 32) {
    const int c = cnt[e];
    for (int q = 0; q * kMbTok < c; ++q) {
      const int nq = c - q * kMbTok < kMbTok ? c - q * kMbTok : kMbTok;
      chunks[coff[e] + q] = make_uint2(static_cast<uint32_t>(e) | (static_cast<uint32_t>(nq) << 16),
                                       static_cast<uint32_t>(poff[e] + q * kMbTok));
    }
  }
  asm volatile("bar.sync 1, %0;" :: "r"(kMbWarps * 32) : "memory");
  if (warp == 0) {
    // lanes holding the same expert: the AND over its bits of each bit's ballot or its complement
    int nbits = 1;
    while ((1 << nbits) <= E) ++nbits;
    const uint32_t lt = (1u << lane) - 1u;
    for (int b0 = 0; b0 < P; b0 += 32) {
      const int p = b0 + lane;
      const uint32_t key = p < P ? eid[p] : static_cast<uint32_t>(E);
      uint32_t peers = 0xFFFFFFFFu;
      for (int bit = 0; bit < nbits; ++bit) {
        const bool on = (key >> bit) & 1u;
        const uint32_t m = __ballot_sync(0xFFFFFFFFu, on);
        peers &= on ? m : ~m;
      }
      if (p < P) sorted[poff[key] + __popc(peers & lt)] = static_cast<uint16_t>(p);
      __syncwarp();
      if (p < P && (peers & lt) == 0) poff[key] += __popc(peers);
      __syncwarp();
    }
  }
}

// SwiGLU of one element from its gate / up sums, stored as the down
// projection's 16-bit input
__device__ __forceinline__ void mb_store_h(const MbParams& prm, int64_t e, float gs, float us) {
  const float hv = __fmul_rn(mb_silu(round_out(gs, prm.x_bf16, prm.dense)), round_out(us, prm.x_bf16, prm.dense));
  if (prm.dense && prm.x_bf16) {
    prm.h16[e] = __bfloat16_as_ushort(__float2bfloat16_rn(hv));  // the down layer's bf16 input
  } else {
    const float hd = prm.x_bf16 ? __bfloat162float(__float2bfloat16_rn(hv)) : __half2float(__float2half_rn(hv));
    prm.h16[e] = __half_as_ushort(__float2half_rn(hd));
  }
}

template <int BITS, bool WBF16>
__global__ void __launch_bounds__(kMbThreads, 1) moe_block_kernel(const __grid_constant__ MbMaps maps,
                                                                   const __grid_constant__ MbParams prm) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const MbLayout L = mb_layout(prm.K, 2 * BITS);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kMbStages;
  uint64_t* cbar = full + 2 * kMbStages;
  int* st = reinterpret_cast<int*>(smem + L.bars + 64);
  volatile int* abort_flag = st + kStAbort;
  float* wsm = reinterpret_cast<float*>(smem + L.w);
  uint16_t* sorted = reinterpret_cast<uint16_t*>(smem + L.sorted);
  uint2* chunks = reinterpret_cast<uint2*>(smem + L.chunks);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int nC = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  const int P = prm.T * prm.k;
  const bool copier = warp == kMbCopyWarp && lane == 0;

  if (tid == 0) {
    for (int i = 0; i < kMbStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kMbWarps);
    }
    mbar_init(cbar, 1);
    mbar_init(cbar + 1, 1);  // the test stall's signal: nothing arrives on it
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < 64; ++i) st[i] = 0;
    if (cta == 0)
      for (int i = 0; i < 4; ++i) prm.status[i] = 0;
  }
  __syncthreads();

  // groups: phase 1 (gate, up) x (half 0, 1) by cta % 4, phase 3 half by cta % 2
  const int g1 = cta & 3, g3 = cta & 1;
  if (copier) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&maps.codes[g1 >> 1])) : "memory");
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&maps.scales[g1 >> 1])) : "memory");
    mb_load_half(prm.proj[g1 >> 1].halves, g1 & 1, prm.K, smem + L.cb, cbar);
  }
  mb_route_tokens(prm, reinterpret_cast<float*>(smem + L.codes[1]), warp, lane);
  if (!mb_grid_barrier(true, st) && tid == 0) *abort_flag = 1;
  __syncthreads();
  if (warp < kMbWarps && !*abort_flag) {
    mb_route(prm, smem + L.codes[0], wsm, sorted, chunks, st, warp, lane);
    // the routing scratch in stage 0 is overwritten by tensor copies next
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();

  const int NC = st[kStChunks];
  const int rt1 = prm.I / kMbRows, rt3 = prm.H / kMbRows;
  const int S1 = mb_split(NC * rt1, nC >> 2, prm.H / kMbWinK, P);
  const int S3 = mb_split(NC * rt3, nC >> 1, prm.I / kMbWinK, P);
  MbPhase ph1{g1 >> 1, g1 & 1, cta >> 2, (nC - g1 + 3) >> 2, S1, NC * rt1, rt1, prm.H / kMbWinK, prm.I,
              prm.part1, g1, false};
  MbPhase ph3{2, g3, cta >> 1, (nC - g3 + 1) >> 1, S3, NC * rt3, rt3, prm.I / kMbWinK, prm.H, prm.part3, g3, true};
  uint32_t gw = 0;  // windows issued (copy thread) / consumed (each consumer warp) so far
  bool cb3_issued = false;

  // ---------------- phase 1: gate and up partials
  if (cta == prm.stall_cta && warp < kMbWarps) warp_wait(cbar + 1, 0, abort_flag, prm.wait_ns);  // tests only
  if (copier) {
    mb_produce<BITS>(&maps.codes[ph1.proj], &maps.scales[ph1.proj], prm, ph1, chunks, sorted, smem, L, full, empty,
                     gw, abort_flag);
  } else if (warp < kMbWarps && ph1.j < ph1.nseg * ph1.S) {
    if (warp_wait(cbar, 0, abort_flag, prm.wait_ns))
      mb_consume<BITS, WBF16>(prm, ph1, chunks, sorted, smem, L, full, empty, gw, abort_flag, warp, lane);
  }
  __syncthreads();  // every consumer is done with the phase-1 codebook half
  if (copier) {
    mbar_drain(cbar, 0);  // a CTA with no phase-1 items never waited for its half
    if (!*abort_flag) {
      asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&maps.codes[2])) : "memory");
      asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&maps.scales[2])) : "memory");
      mb_load_half(prm.proj[2].halves, g3, prm.K, smem + L.cb, cbar);
      cb3_issued = true;
    }
  }
  bool ok = mb_grid_barrier(*abort_flag == 0, st);

  // ---------------- phase 2: SwiGLU -> the down projection's fp16 input
  // (elements spread evenly over the CTAs; an element's partial loads are
  // issued together, then summed in the fixed order: split, then half)
  if (ok && warp < kMbWarps) {
    const int I = prm.I;
    const int64_t n2 = static_cast<int64_t>(P) * I;
    const int64_t per = (n2 + nC - 1) / nC;
    const int64_t e0 = static_cast<int64_t>(cta) * per, e1 = e0 + per < n2 ? e0 + per : n2;
    const size_t gstride = static_cast<size_t>(S1) * P * I;  // one partial group
    if (S1 == 1) {
      // one split (the large batches): eight elements' partial loads in flight
      // per thread before any store, then the same sums as below
      constexpr int kB = 8;
      for (int64_t eb = e0 + tid; eb < e1; eb += kB * kMbWarps * 32) {
        float v[kB][4];
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          const int64_t e = eb + static_cast<int64_t>(b) * kMbWarps * 32;
#pragma unroll
          for (int q = 0; q < 4; ++q) v[b][q] = e < e1 ? __ldcg(prm.part1 + q * gstride + static_cast<size_t>(e)) : 0.0f;
        }
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          const int64_t e = eb + static_cast<int64_t>(b) * kMbWarps * 32;
          if (e < e1) {
            float gs = 0.0f, us = 0.0f;
            gs += v[b][0];
            gs += v[b][1];
            us += v[b][2];
            us += v[b][3];
            mb_store_h(prm, e, gs, us);
          }
        }
      }
    } else
#pragma unroll 4
    for (int64_t e = e0 + tid; e < e1; e += kMbWarps * 32) {
      float v[4][kMbMaxSplit];
#pragma unroll
      for (int s = 0; s < kMbMaxSplit; ++s) {
        if (s < S1) {
          const size_t o = static_cast<size_t>(s) * P * I + static_cast<size_t>(e);
#pragma unroll
          for (int q = 0; q < 4; ++q) v[q][s] = prm.part1[q * gstride + o];
        }
      }
      float gs = 0.0f, us = 0.0f;
#pragma unroll
      for (int s = 0; s < kMbMaxSplit; ++s) {
        if (s < S1) {
          gs += v[0][s];
          gs += v[1][s];
          us += v[2][s];
          us += v[3][s];
        }
      }
      mb_store_h(prm, e, gs, us);
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");  // h16 is read by bulk copies after the barrier
  }
  ok = mb_grid_barrier(ok && *abort_flag == 0, st);

  // ---------------- phase 3: down partials
  if (ok) {
    if (copier) {
      // h16 rows were written by other CTAs' generic stores; the bulk copies read them
      asm volatile("fence.proxy.async.global;" ::: "memory");
      mb_produce<BITS>(&maps.codes[2], &maps.scales[2], prm, ph3, chunks, sorted, smem, L, full, empty, gw,
                       abort_flag);
    } else if (warp < kMbWarps && ph3.j < ph3.nseg * ph3.S) {
      if (warp_wait(cbar, 1, abort_flag, prm.wait_ns))
        mb_consume<BITS, WBF16>(prm, ph3, chunks, sorted, smem, L, full, empty, gw, abort_flag, warp, lane);
    }
  }
  ok = mb_grid_barrier(ok && *abort_flag == 0, st);

  // ---------------- phase 4: combine over the slots.  The elements are
  // spread evenly over the CTAs; each CTA first forms every (element, slot)
  // product d * w with one thread per product (the slot's partial loads
  // issued together) into its free stage memory, then adds each element's
  // products in slot order.
  if (ok) {
    const int H = prm.H, k = prm.k;
    const int n4 = prm.T * H;  // below 2^31 (host check): 32-bit index math, no 64-bit divisions per product
    const int per = (n4 + nC - 1) / nC;
    const int e0 = cta * per, e1 = e0 + per < n4 ? e0 + per : n4;
    const size_t hstride = static_cast<size_t>(S3) * P * H;
    float* prod = reinterpret_cast<float*>(smem + L.codes[0]);
    const int cap = static_cast<int>((L.w - L.codes[0]) / (4u * static_cast<uint32_t>(k)));  // elements per pass
    for (int sub = e0; sub < e1; sub += cap) {
      const int ne = e1 - sub < cap ? e1 - sub : cap;
      if (S3 == 1) {
        // one split (the large batches): eight products' partial loads in
        // flight per thread before any store, then the same sums as below
        constexpr int kB = 8;
        for (int qb = tid; qb < ne * k; qb += kB * kMbThreads) {
          float v[kB][2];
#pragma unroll
          for (int b = 0; b < kB; ++b) {
            const int q = qb + b * kMbThreads;
            v[b][0] = v[b][1] = 0.0f;
            if (q < ne * k) {
              const int j = q / ne, el = q - j * ne;
              const int e = sub + el;
              const int t = e / H, r = e - t * H;
              const size_t o = static_cast<size_t>(t * k + j) * H + r;
              v[b][0] = __ldcg(prm.part3 + o);
              v[b][1] = __ldcg(prm.part3 + hstride + o);
            }
          }
#pragma unroll
          for (int b = 0; b < kB; ++b) {
            const int q = qb + b * kMbThreads;
            if (q < ne * k) {
              const int j = q / ne, el = q - j * ne;
              const int t = (sub + el) / H;
              float ds = 0.0f;
              ds += v[b][0];
              ds += v[b][1];
              prod[el * k + j] = __fmul_rn(round_out(ds, prm.x_bf16, prm.dense), wsm[t * k + j]);
            }
          }
        }
      } else
#pragma unroll 4
      for (int q = tid; q < ne * k; q += kMbThreads) {
        const int j = q / ne, el = q - j * ne;
        const int e = sub + el;
        const int t = e / H, r = e - t * H;
        float v[2 * kMbMaxSplit];
#pragma unroll
        for (int s = 0; s < kMbMaxSplit; ++s) {
          if (s < S3) {
            const size_t o = (static_cast<size_t>(s) * P + t * k + j) * H + r;
            v[2 * s] = prm.part3[o];
            v[2 * s + 1] = prm.part3[hstride + o];
          }
        }
        float ds = 0.0f;
#pragma unroll
        for (int s = 0; s < kMbMaxSplit; ++s) {
          if (s < S3) {
            ds += v[2 * s];
            ds += v[2 * s + 1];
          }
        }
        prod[el * k + j] = __fmul_rn(round_out(ds, prm.x_bf16, prm.dense), wsm[t * k + j]);
      }
      __syncthreads();
      for (int el = tid; el < ne; el += kMbThreads) {
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) acc = __fadd_rn(acc, prod[el * k + j]);
        const int e = sub + el;
        if (prm.x_bf16) reinterpret_cast<__nv_bfloat16*>(prm.y)[e] = __float2bfloat16_rn(acc);
        else reinterpret_cast<__half*>(prm.y)[e] = __float2half_rn(acc);
      }
      __syncthreads();
    }
  }

  // teardown: the copy thread waits for its copies still in flight
  if (copier) {
    for (uint32_t q = 1; q <= kMbStages && q <= gw; ++q)
      mbar_drain(&full[(gw - q) & 1u], ((gw - q) >> 1) & 1u);
    if (cb3_issued) mbar_drain(cbar, 1);
  }
  __syncthreads();
  if (tid == 0 && (st[kStErr] || st[kStAbort])) atomicExch(prm.status + 1, static_cast<int>(VQB_TIMEOUT));
}

// ------------------------------------------------------------ host

struct MbGeo {
  LinearGeometry p[3];  // gate, up, down
  int E, H, I, K, bits, k;
};

// The shape checks common to the MoE block and the dense MLP once the three
// projections are validated and g's sizes are set (else
// VQB_UNSUPPORTED_GEOMETRY: the caller runs the per-step kernels).
vqb_status mb_check_common(const vqb_linear_desc* const ds[3], int T, int x_dtype, MbGeo* g) {
  if (x_dtype != VQB_BF16 && x_dtype != VQB_F16) return VQB_UNSUPPORTED_GEOMETRY;
  if (g->E > kMbMaxExperts || static_cast<int64_t>(T) * g->k > kMbMaxPairs) return VQB_UNSUPPORTED_GEOMETRY;
  if (g->H % kMbWinK != 0 || g->I % kMbWinK != 0) return VQB_UNSUPPORTED_GEOMETRY;
  if (static_cast<int64_t>(T) * g->H > 0x7fffffff) return VQB_UNSUPPORTED_GEOMETRY;  // 32-bit element indices
  if (g->bits != 12 && g->bits != 14) return VQB_UNSUPPORTED_GEOMETRY;
  for (int i = 0; i < 3; ++i) {
    const LinearGeometry& q = g->p[i];
    if (q.D != 8 || q.G != 64 || q.K != g->K || q.bits != g->bits || ds[i]->pack_bits != g->bits) return VQB_UNSUPPORTED_GEOMETRY;
    if (q.K != (1 << q.bits)) return VQB_UNSUPPORTED_GEOMETRY;  // every code names an entry
    if (q.row_table || !q.codebook_halves) return VQB_UNSUPPORTED_GEOMETRY;
    if ((reinterpret_cast<uintptr_t>(q.codes) & 15) != 0 || (reinterpret_cast<uintptr_t>(q.scales) & 15) != 0)
      return VQB_UNSUPPORTED_GEOMETRY;
  }
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  if (di.sms < 4 || mb_layout(g->K, 2 * g->bits).total > static_cast<uint32_t>(di.smem_optin))
    return VQB_UNSUPPORTED_GEOMETRY;
  return VQB_OK;
}

vqb_status mb_validate3(const vqb_linear_desc* const ds[3], MbGeo* g) {
  for (int i = 0; i < 3; ++i) {
    const vqb_status st = validate(ds[i], &g->p[i]);
    if (st != VQB_OK) return st;
  }
  const LinearGeometry &ga = g->p[0], &gu = g->p[1], &gd = g->p[2];
  if (ga.E != gu.E || ga.E != gd.E || ga.OUT != gu.OUT || ga.IN != gu.IN || gd.IN != ga.OUT || gd.OUT != ga.IN)
    return VQB_BAD_SHAPE;
  g->E = ga.E;
  g->H = ga.IN;
  g->I = ga.OUT;
  g->K = ga.K;
  g->bits = ga.bits;
  return VQB_OK;
}

vqb_status mb_check(const vqb_moe_block_desc* d, int T, int x_dtype, MbGeo* g) {
  if (!d) return VQB_NULL_POINTER;
  const vqb_linear_desc* const ds[3] = {&d->gate, &d->up, &d->down};
  vqb_status st = mb_validate3(ds, g);
  if (st != VQB_OK) return st;
  if (T < 1 || d->top_k < 1 || d->top_k > 32 || d->top_k > g->E) return VQB_BAD_SHAPE;
  g->k = d->top_k;
  return mb_check_common(ds, T, x_dtype, g);
}

vqb_status mb_check_dense(const vqb_dense_mlp_desc* d, int T, int x_dtype, MbGeo* g) {
  if (!d) return VQB_NULL_POINTER;
  const vqb_linear_desc* const ds[3] = {&d->gate, &d->up, &d->down};
  vqb_status st = mb_validate3(ds, g);
  if (st != VQB_OK) return st;
  if (T < 1 || g->E != 1) return VQB_BAD_SHAPE;
  g->k = 1;
  return mb_check_common(ds, T, x_dtype, g);
}

struct MbWorkspace {
  size_t status, part1, part3, h16, x16, ridx, rw, total;
};

MbWorkspace mb_workspace(int T, int k, int H, int I) {
  const int P = T * k;
  const size_t slots = static_cast<size_t>(mb_slots(P));
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  MbWorkspace w;
  w.status = 0;
  w.part1 = 256;
  w.part3 = w.part1 + up(4 * slots * I * sizeof(float));
  w.h16 = w.part3 + up(2 * slots * H * sizeof(float));
  w.x16 = w.h16 + up(static_cast<size_t>(P) * I * 2);
  w.ridx = w.x16 + up(static_cast<size_t>(T) * H * 2);
  w.rw = w.ridx + up(static_cast<size_t>(P) * 4);
  w.total = w.rw + up(static_cast<size_t>(P) * 4);
  return w;
}

// One launch of the block kernel for a checked geometry (dense: no router,
// every token to the one expert with weight 1, the dense layers' numerics).
vqb_status mb_launch(const MbGeo& g, bool dense, const float* logits, const void* x, int x_dtype, int T, void* y,
                     int32_t* indices, float* weights, void* workspace, size_t workspace_bytes,
                     const vqb_moe_block_options* opts, vqb_stream_t stream) {
  if (!x || !y || !workspace) return VQB_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0 || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return VQB_BAD_ALIGNMENT;
  if (opts && opts->wait_limit_us < 0) return VQB_BAD_SHAPE;
  const MbWorkspace ws = mb_workspace(T, g.k, g.H, g.I);
  if (workspace_bytes < ws.total) return VQB_WORKSPACE_TOO_SMALL;
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return VQB_CUDA_ERROR;

  const int W = 2 * g.bits;
  MbMaps maps;
  for (int i = 0; i < 3; ++i) {
    const LinearGeometry& q = g.p[i];
    const uint64_t rows = static_cast<uint64_t>(q.E) * q.OUT;
    if (!encode_2d(enc, &maps.codes[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, q.codes, static_cast<uint64_t>(q.row_words),
                   rows, static_cast<uint32_t>(W), kMbRows, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_2d(enc, &maps.scales[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, q.scales,
                   static_cast<uint64_t>(q.IN / 64), rows, kMbWinK / 64, kMbRows, CU_TENSOR_MAP_SWIZZLE_NONE))
      return VQB_CUDA_ERROR;
  }
  MbParams prm{};
  prm.logits = logits;
  prm.x = x;
  prm.y = y;
  prm.idx_out = indices;
  prm.w_out = weights;
  prm.T = T;
  prm.E = g.E;
  prm.k = g.k;
  prm.H = g.H;
  prm.I = g.I;
  prm.K = g.K;
  prm.x_bf16 = x_dtype == VQB_BF16 ? 1 : 0;
  prm.dense = dense ? 1 : 0;
  prm.wait_ns = opts && opts->wait_limit_us > 0 ? static_cast<uint64_t>(opts->wait_limit_us) * 1000ull : kWaitLimitNs;
  prm.stall_cta = opts ? opts->stall_cta : -1;
  for (int i = 0; i < 3; ++i) {
    prm.proj[i].halves = static_cast<const uint16_t*>(g.p[i].codebook_halves);
    prm.proj[i].OUT = g.p[i].OUT;
    prm.proj[i].IN = g.p[i].IN;
  }
  char* base = static_cast<char*>(workspace);
  prm.status = reinterpret_cast<int*>(base + ws.status);
  prm.part1 = reinterpret_cast<float*>(base + ws.part1);
  prm.part3 = reinterpret_cast<float*>(base + ws.part3);
  prm.h16 = reinterpret_cast<uint16_t*>(base + ws.h16);
  prm.x16 = reinterpret_cast<uint16_t*>(base + ws.x16);
  prm.ridx = reinterpret_cast<int32_t*>(base + ws.ridx);
  prm.rw = reinterpret_cast<float*>(base + ws.rw);

  const MbLayout L = mb_layout(g.K, W);
  // bf16 operands for a dense layer with bf16 x (its weights take x's dtype, vq_dense.py:294)
  const bool wbf16 = dense && x_dtype == VQB_BF16;
  void (*kern)(MbMaps, MbParams) =
      g.bits == 14 ? (wbf16 ? moe_block_kernel<14, true> : moe_block_kernel<14, false>)
                   : (wbf16 ? moe_block_kernel<12, true> : moe_block_kernel<12, false>);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L.total)) !=
      cudaSuccess)
    return VQB_CUDA_ERROR;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(di.sms));
  cfg.blockDim = dim3(kMbThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  timer_before(cfg.stream);
  const cudaError_t ce = cudaLaunchKernelEx(&cfg, kern, maps, prm);
  timer_after(cfg.stream);
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

}  // namespace

}  // namespace vqb

using namespace vqb;

extern "C" vqb_status vqb_moe_block_supported(const vqb_moe_block_desc* desc, int32_t n_tokens, vqb_dtype x_dtype) {
  MbGeo g;
  return mb_check(desc, n_tokens, x_dtype, &g);
}

extern "C" size_t vqb_moe_block_workspace_size(const vqb_moe_block_desc* desc, int32_t n_tokens) {
  if (!desc || n_tokens < 1 || desc->top_k < 1) return 0;
  return mb_workspace(n_tokens, desc->top_k, desc->gate.in_features > 0 ? desc->gate.in_features : 0,
                      desc->gate.out_features > 0 ? desc->gate.out_features : 0)
      .total;
}

extern "C" vqb_status vqb_moe_block_forward(const vqb_moe_block_desc* desc, const float* router_logits,
                                            const void* x, vqb_dtype x_dtype, int32_t n_tokens, void* y,
                                            int32_t* indices, float* weights, void* workspace,
                                            size_t workspace_bytes, const vqb_moe_block_options* opts,
                                            vqb_stream_t stream) {
  MbGeo g;
  vqb_status st = mb_check(desc, n_tokens, x_dtype, &g);
  if (st != VQB_OK) return st;
  if (!router_logits) return VQB_NULL_POINTER;
  if ((indices == nullptr) != (weights == nullptr)) return VQB_NULL_POINTER;
  return mb_launch(g, false, router_logits, x, x_dtype, n_tokens, y, indices, weights, workspace, workspace_bytes,
                   opts, stream);
}

extern "C" vqb_status vqb_dense_mlp_supported(const vqb_dense_mlp_desc* desc, int32_t n_tokens, vqb_dtype x_dtype) {
  MbGeo g;
  return mb_check_dense(desc, n_tokens, x_dtype, &g);
}

extern "C" size_t vqb_dense_mlp_workspace_size(const vqb_dense_mlp_desc* desc, int32_t n_tokens) {
  if (!desc || n_tokens < 1) return 0;
  return mb_workspace(n_tokens, 1, desc->gate.in_features > 0 ? desc->gate.in_features : 0,
                      desc->gate.out_features > 0 ? desc->gate.out_features : 0)
      .total;
}

extern "C" vqb_status vqb_dense_mlp_forward(const vqb_dense_mlp_desc* desc, const void* x, vqb_dtype x_dtype,
                                            int32_t n_tokens, void* y, void* workspace, size_t workspace_bytes,
                                            const vqb_moe_block_options* opts, vqb_stream_t stream) {
  MbGeo g;
  vqb_status st = mb_check_dense(desc, n_tokens, x_dtype, &g);
  if (st != VQB_OK) return st;
  return mb_launch(g, true, nullptr, x, x_dtype, n_tokens, y, nullptr, nullptr, workspace, workspace_bytes, opts,
                   stream);
}
