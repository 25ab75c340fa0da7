// Small-codebook dense decode on the tensor cores (sm_100a): a VQLinear whose
// d2 codebook has at most 256 entries and 8-bit codes (the attention
// projections of a dense model: d2/K256) at decode batches of up to 8 rows,
// in the reference's fused dense arm (vq_switch.py:2319-2327, taken by
// vq_dense.py:401-441 for d2 layers at small N): x narrowed to fp16, the fp32
// partial sum of each 64-input scale group multiplied by the group's scale,
// y stored once in the output dtype.
//
// One launch of 512-thread CTAs (16 warps; thread 0 also issues the copies),
// one CTA per SM at a time:
//   * the codebook is replicated per lane in shared memory: entry e for lane l
//     is the word at byte e * 256 + 4 * l, so the 32 lookups of a warp always
//     hit 32 different banks, and one byte permute (the code byte next to
//     4 * lane) forms the address;
//   * a CTA takes 256 output rows (or 128, warps w and w + 8 then sharing a
//     16-row tile and taking a window's first and last four scale groups)
//     and a range of 512-input windows (split s of S); each window's codes
//     (256 bytes per row: two TMA boxes of 128 bytes x the CTA's rows with
//     the 128-byte swizzle), its scales (8 fp16 per row) and the tokens' x
//     rows (bulk copies) arrive in two stages, refilled once every warp has
//     released the stage;
//   * inside a scale group (32 codes of a row), thread t of a quad takes codes
//     8t .. 8t+7 (one 8-byte read per row) and the inputs they cover (two
//     16-byte reads of x): MMA step m uses codes 8t+2m and 8t+2m+1 as the A
//     slots t and t+4 of an m16n8k16 -- a permutation of k applied to A and B
//     alike, so the sum is the group's dot product; the four steps accumulate
//     the group partial, which is added, times the row's scale, to the row's
//     accumulator;
//   * with one split per row block a CTA stores y itself; otherwise the S
//     CTAs of a row block form a thread-block cluster: each CTA owns a share
//     of the rows, every CTA stores its fp32 partials of those rows into the
//     owner's shared memory (distributed shared memory, into the table's
//     unused upper halves), and after one cluster barrier each owner sums its
//     rows over the S partials in split order and stores y.  No CTA waits on
//     global memory.
//
// Every mbarrier wait is bounded (2 s); a CTA whose wait expires computes
// nothing further, still reaches the cluster barriers, waits for its copies
// in flight and writes VQB_TIMEOUT to the workspace status block (int32 [1]),
// which block 0 clears when it starts (the launch's first CTAs are resident
// long before any wait could expire).
#include <cuda.h>

#include <map>
#include <mutex>
#include <tuple>

#include "vqb_common.cuh"
#include "vqb_internal.h"
#include "vqb_tma.cuh"

namespace vqb {

namespace {

constexpr int kLtWarps = 16;                     // decode warps
constexpr int kLtThreads = kLtWarps * 32;        // thread 0 also issues the copies
constexpr int kLtRows = 256;                     // output rows of a CTA
constexpr int kLtTiles = kLtRows / (16 * kLtWarps);  // 16-row MMA tiles per warp
constexpr int kLtWarpRows = 16 * kLtTiles;
constexpr int kLtWinK = 512;                     // inputs per window: 256 codes, 256 bytes per row
constexpr int kLtStages = 2;
constexpr int kLtTok = 8;                        // tokens (the MMA's N)
constexpr int kLtXStride = kLtWinK * 2 + 16;     // bytes of a staged x row (16 B pad: conflict-free reads)
constexpr int kLtMaxSplit = 8;                   // portable cluster size
constexpr uint32_t kLtTable = 256 * 256;         // 256 entries x (32 lanes x 4 B, 128 B unused)
constexpr uint32_t kLtHalfBox = 128 * kLtRows;   // one 128-byte-wide code box
constexpr uint32_t kLtScaleOff = 2 * kLtHalfBox;
constexpr uint32_t kLtXOff = kLtScaleOff + 16 * kLtRows;
constexpr uint32_t kLtStageBytes = (kLtXOff + kLtTok * kLtXStride + 1023) & ~1023u;
constexpr uint32_t kLtBarOff = kLtStages * kLtStageBytes;  // from the aligned stage base
// the table at the start of dynamic shared memory, then up to 1023 bytes to
// align the stages to 1024 (the 128-byte swizzle's 8-row pattern), stages, barriers
constexpr uint32_t kLtSmem = kLtTable + 1024 + kLtBarOff + 64;
// split-K partials a row's owner receives: float i at byte (i / 32) * 256 +
// 128 + 4 (i % 32) -- the upper halves of the table's 256-byte entries, which
// lookups never read; [source split][token][owned row], at most
// 8 x 8 x 37 floats (< 8192)
__device__ __forceinline__ uint32_t lt_recv_off(int i) {
  return (static_cast<uint32_t>(i >> 5) << 8) + 128u + (static_cast<uint32_t>(i & 31) << 2);
}

struct LtParams {
  const uint32_t* codebook;  // [K] entries of two fp16
  int K;
  const void* x;             // [T][IN] fp16 / bf16
  void* y;                   // [T][OUT]
  int y_dtype;
  int T, OUT, IN;
  int S, nw;                 // CTAs (splits) per row block = cluster size, windows per row
  int* status;               // workspace status block
};

struct LtMaps {
  CUtensorMap codes;   // uint32 [OUT][IN / 8], box 32 words x 256 rows, 128-byte swizzle
  CUtensorMap scales;  // fp16 [OUT][IN / 64], box 8 x 256
};

__device__ __forceinline__ void lt_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];"
               :: "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ void lt_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lt_bf16x2_to_f16x2(uint32_t v) {
  __half2 h = __floats2half2_rn(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
  return *reinterpret_cast<uint32_t*>(&h);
}

// cluster barrier halves, every thread of every CTA in the cluster (a
// hardware barrier; all CTAs of a cluster are co-scheduled)
__device__ __forceinline__ void lt_cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void lt_cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }
__device__ __forceinline__ void lt_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ void lt_st_cluster(uint32_t local_smem, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_smem), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" :: "r"(remote), "f"(v) : "memory");
}

// One staged window for one warp: rows kLtWarpRows * warp + 8 * r + g (MMA
// tile j holds r = 2j and 2j + 1), tokens 2t and 2t + 1 of each tile, scale
// groups qlo .. qlo + NQ - 1 (qlo 0 or 4).  Lanes of tokens >= T read no x
// (their B values are zero).
//   off[qq]: swizzled byte offset of this thread's 8 codes of group 4h + qq
//   inside a 128-byte box row (chunk (2qq + t/2) ^ g, half t & 1).
template <int NQ>
__device__ __forceinline__ void lt_window(const unsigned char* table, const unsigned char* sb, int warp, int qlo, int g,
                                          int t, uint32_t lane4, const uint32_t (&off)[4], bool has_x,
                                          float (&acc)[kLtTiles][4]) {
  const unsigned char* cbase = sb + (warp * kLtWarpRows + g) * 128;
  const unsigned char* xb = sb + kLtXOff + g * kLtXStride + 32 * t;
  const unsigned char* sbase = sb + kLtScaleOff + (warp * kLtWarpRows + g) * 16;
  uint4 sc[2 * kLtTiles];
#pragma unroll
  for (int r = 0; r < 2 * kLtTiles; ++r) sc[r] = *reinterpret_cast<const uint4*>(sbase + r * 8 * 16);
#pragma unroll
  for (int qi = 0; qi < NQ; ++qi) {
    const int q = qlo + qi;            // qlo is 0 or 4: q & 3 == qi & 3
    const int h = q >> 2, qq = qi & 3;
    uint2 cw[2 * kLtTiles];
#pragma unroll
    for (int r = 0; r < 2 * kLtTiles; ++r)
      cw[r] = *reinterpret_cast<const uint2*>(cbase + h * kLtHalfBox + r * 1024 + off[qq]);
    uint4 v0 = make_uint4(0u, 0u, 0u, 0u), v1 = v0;
    if (has_x) {
      v0 = *reinterpret_cast<const uint4*>(xb + 128 * q);
      v1 = *reinterpret_cast<const uint4*>(xb + 128 * q + 16);
    }
    float part[kLtTiles][4];
#pragma unroll
    for (int j = 0; j < kLtTiles; ++j) part[j][0] = part[j][1] = part[j][2] = part[j][3] = 0.0f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t b0 = m == 0 ? v0.x : (m == 1 ? v0.z : (m == 2 ? v1.x : v1.z));
      const uint32_t b1 = m == 0 ? v0.y : (m == 1 ? v0.w : (m == 2 ? v1.y : v1.w));
      // codes 8t + 2m and 8t + 2m + 1 of the row: bytes 2(m & 1), +1 of word m >> 1;
      // the permute puts the code byte above 4 * lane (table byte code * 256 + 4 * lane)
      const uint32_t s_lo = (m & 1) ? 0x5524u : 0x5504u, s_hi = (m & 1) ? 0x5534u : 0x5514u;
#pragma unroll
      for (int j = 0; j < kLtTiles; ++j) {
        const uint32_t w0 = (m >> 1) ? cw[2 * j].y : cw[2 * j].x;
        const uint32_t w1 = (m >> 1) ? cw[2 * j + 1].y : cw[2 * j + 1].x;
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(table + __byte_perm(w0, lane4, s_lo));
        const uint32_t a1 = *reinterpret_cast<const uint32_t*>(table + __byte_perm(w1, lane4, s_lo));
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(table + __byte_perm(w0, lane4, s_hi));
        const uint32_t a3 = *reinterpret_cast<const uint32_t*>(table + __byte_perm(w1, lane4, s_hi));
        lt_mma(part[j], a0, a1, a2, a3, b0, b1);
      }
    }
    // the group's scales: fp16 number q of each row's 8
#pragma unroll
    for (int j = 0; j < kLtTiles; ++j) {
      const uint4& u0 = sc[2 * j];
      const uint4& u1 = sc[2 * j + 1];
      const uint32_t p0 = (q >> 1) == 0 ? u0.x : ((q >> 1) == 1 ? u0.y : ((q >> 1) == 2 ? u0.z : u0.w));
      const uint32_t p1 = (q >> 1) == 0 ? u1.x : ((q >> 1) == 1 ? u1.y : ((q >> 1) == 2 ? u1.z : u1.w));
      const float s0 = __half2float(__ushort_as_half(static_cast<unsigned short>((q & 1) ? (p0 >> 16) : p0)));
      const float s1 = __half2float(__ushort_as_half(static_cast<unsigned short>((q & 1) ? (p1 >> 16) : p1)));
      acc[j][0] = fmaf(s0, part[j][0], acc[j][0]);
      acc[j][1] = fmaf(s0, part[j][1], acc[j][1]);
      acc[j][2] = fmaf(s1, part[j][2], acc[j][2]);
      acc[j][3] = fmaf(s1, part[j][3], acc[j][3]);
    }
  }
}

// Thread 0: the copies of window w into stage st (codes: two swizzled boxes;
// scales; the tokens' x rows).
__device__ __forceinline__ void lt_issue(const LtMaps& maps, const LtParams& p, unsigned char* sb, uint64_t* bar,
                                         int w, int rb, int rows) {
  const unsigned char* xg = static_cast<const unsigned char*>(p.x);
  mbar_expect_tx(bar, 2u * 128u * rows + 16u * rows + static_cast<uint32_t>(p.T) * kLtWinK * 2);
  tma_load_2d(&maps.codes, bar, sb, w * 64, rb * rows);
  tma_load_2d(&maps.codes, bar, sb + kLtHalfBox, w * 64 + 32, rb * rows);
  tma_load_2d(&maps.scales, bar, sb + kLtScaleOff, w * 8, rb * rows);
  for (int j = 0; j < p.T; ++j)
    bulk_load(sb + kLtXOff + j * kLtXStride, xg + (static_cast<size_t>(j) * p.IN + static_cast<size_t>(w) * kLtWinK) * 2,
              kLtWinK * 2, bar);
}

// KQ = 1: 256 rows per CTA, warp w owns tile w and all 8 groups of a window.
// KQ = 2: 128 rows per CTA; warps w and w + 8 share tile w % 8 and take
// groups 0-3 (code box 0) and 4-7 (code box 1), their fp32 partials added in
// that order before the store.
template <bool XBF16, int KQ>
__global__ void __launch_bounds__(kLtThreads, 1) dense_lut_kernel(const __grid_constant__ LtMaps maps,
                                                                  const __grid_constant__ LtParams p) {
  constexpr int kRows = kLtRows / KQ, kTiles = kLtWarps / KQ;
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* stages = smem + kLtTable + ((1024u - ((smem_u32(smem) + kLtTable) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kLtBarOff);
  uint64_t* empty = full + kLtStages;
  int* sflags = reinterpret_cast<int*>(full + 2 * kLtStages);  // [0] abort, [1] windows issued
  volatile int* abort_flag = sflags;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  // 1-d clusters of S CTAs: the split is the CTA's rank in its cluster
  const int rb = blockIdx.x / p.S, split = blockIdx.x - rb * p.S;
  const int w0 = split * p.nw / p.S, w1 = (split + 1) * p.nw / p.S, nwin = w1 - w0;

  if (tid == 0) {
    for (int s = 0; s < kLtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLtWarps);
    }
    sflags[0] = 0;
    sflags[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // this CTA's weights into L2 while the previous kernel finishes (a
    // prefetch returns no data, so it cannot observe a stale value)
    for (int b = 0; b < p.K * 4; b += 128)
      asm volatile("prefetch.global.L2 [%0];" :: "l"(reinterpret_cast<const char*>(p.codebook) + b));
    for (int w = w0; w < w1; ++w) {
      lt_prefetch_2d(&maps.codes, w * 64, rb * kRows);
      lt_prefetch_2d(&maps.codes, w * 64 + 32, rb * kRows);
      lt_prefetch_2d(&maps.scales, w * 8, rb * kRows);
    }
  }
  // tokens T..7 read zeros: their x rows are never copied
  {
    const int per = (kLtTok - p.T) * (kLtXStride / 16);
    for (int i = tid; i < kLtStages * per; i += kLtThreads) {
      const int s = i / per, r = i - s * per;
      *reinterpret_cast<uint4*>(stages + s * kLtStageBytes + kLtXOff + p.T * kLtXStride + r * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __syncthreads();
  // first half of the barrier that tells every CTA of the cluster its peers have started
  if (p.S > 1) lt_cluster_arrive_relaxed();
  pdl_wait();
  pdl_trigger();
  if (tid == 0) {
    if (blockIdx.x == 0) p.status[1] = 0;
    for (int n = 0; n < kLtStages && n < nwin; ++n) lt_issue(maps, p, stages + n * kLtStageBytes, &full[n], w0 + n, rb, kRows);
    sflags[1] = nwin < kLtStages ? nwin : kLtStages;
  }
  // the replicated codebook: entry e for lane l at byte e * 256 + 4 l; codes >= K read zeros.
  // Warp w writes entries w + kLtWarps * k: one global load per lane, then shuffles.
  {
    constexpr int kPer = 256 / kLtWarps;
    const int mine_e = warp + kLtWarps * (lane % kPer);
    const uint32_t mine = mine_e < p.K ? __ldg(p.codebook + mine_e) : 0u;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const uint32_t v = __shfl_sync(0xffffffffu, mine, k);
      *reinterpret_cast<uint32_t*>(smem + (warp + kLtWarps * k) * 256 + lane * 4) = v;
    }
  }
  __syncthreads();

  float acc[kLtTiles][4];
#pragma unroll
  for (int j = 0; j < kLtTiles; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  const int g = lane >> 2, t = lane & 3;
  const int wt = warp % kTiles, kq = warp / kTiles;  // MMA tile, group share
  const uint32_t lane4 = static_cast<uint32_t>(lane) * 4u;
  uint32_t off[4];
#pragma unroll
  for (int qq = 0; qq < 4; ++qq) off[qq] = ((static_cast<uint32_t>(2 * qq + (t >> 1)) ^ g) << 4) | (8u * (t & 1));
  bool alive = true;
  for (int n = 0; n < nwin; ++n) {
    const int st = n & 1;
    unsigned char* sb = stages + st * kLtStageBytes;
    if (alive) alive = warp_wait(&full[st], (n >> 1) & 1, abort_flag);
    if (XBF16) {
      // x narrowed to fp16 in place (each thread a share), then every warp reads it
      if (alive) {
        for (int k = tid; k < p.T * (kLtWinK / 8); k += kLtThreads) {
          uint4* q = reinterpret_cast<uint4*>(sb + kLtXOff + (k >> 6) * kLtXStride + (k & 63) * 16);
          uint4 v = *q;
          v.x = lt_bf16x2_to_f16x2(v.x);
          v.y = lt_bf16x2_to_f16x2(v.y);
          v.z = lt_bf16x2_to_f16x2(v.z);
          v.w = lt_bf16x2_to_f16x2(v.w);
          *q = v;
        }
      }
      __syncthreads();
    }
    if (alive) lt_window<8 / KQ>(smem, sb, wt, kq * (8 / KQ), g, t, lane4, off, g < p.T, acc);
    // the in-place narrowing's writes before the next copy into this stage
    if (XBF16) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (tid == 0 && n + kLtStages < nwin && !*abort_flag) {
      // refill this stage once every warp has released it
      if (mbar_wait(&empty[st], (n >> 1) & 1, abort_flag)) {
        lt_issue(maps, p, sb, &full[st], w0 + n + kLtStages, rb, kRows);
        sflags[1] = n + kLtStages + 1;
      }
    }
  }
  if constexpr (KQ == 2) {
    // every warp is past its last window: stage 0's first 4 KB holds the
    // second group share's partials, added after the first's
    __syncthreads();
    float* red = reinterpret_cast<float*>(stages);
    if (kq == 1)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[(wt * 32 + lane) * 4 + e] = acc[0][e];
    __syncthreads();
    if (kq == 0)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[0][e] = acc[0][e] + red[(wt * 32 + lane) * 4 + e];
  }
  if (p.S == 1 && kq == 0) {
    // rows kLtWarpRows wt + 16 j + g (+ 8), tokens 2t, 2t + 1
    const int row0 = rb * kRows + wt * kLtWarpRows + g;
#pragma unroll
    for (int j = 0; j < kLtTiles; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = row0 + 16 * j + 8 * (e >> 1), tok = 2 * t + (e & 1);
        if (row < p.OUT && tok < p.T)
          store_y(p.y, static_cast<int64_t>(tok) * p.OUT + row, acc[j][e], p.y_dtype, false);
      }
  }
  __syncthreads();
  if (tid == 0) {
    // copies still in flight (only after an expired wait) land before stage 0 is reused or the CTA exits
    const int issued = sflags[1];
    for (int k = issued > kLtStages ? issued - kLtStages : 0; k < issued; ++k) mbar_drain(&full[k & 1], (k >> 1) & 1);
    if (*abort_flag) p.status[1] = static_cast<int>(VQB_TIMEOUT);
  }
  if (p.S == 1) return;
  // ---- split-K over the cluster: the owner of local row lr is rank lr / R
  const int R = (kRows + p.S - 1) / p.S;
  lt_cluster_wait();  // every peer has started: its shared memory may be written
#pragma unroll
  for (int j = 0; j < kLtTiles; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int lr = wt * kLtWarpRows + 16 * j + 8 * (e >> 1) + g, tok = 2 * t + (e & 1);
      if (kq == 0 && tok < p.T) {
        const int owner = lr / R;
        lt_st_cluster(smem_u32(smem) + lt_recv_off((split * kLtTok + tok) * R + (lr - owner * R)),
                      static_cast<uint32_t>(owner), acc[j][e]);
      }
    }
  lt_cluster_sync();
  // this rank's rows, summed over the S partials in split order
  const int r0 = split * R, nr = (r0 + R < kRows ? R : kRows - r0);
  for (int k = tid; k < p.T * nr; k += kLtThreads) {
    const int tok = k / nr, r = k - tok * nr;
    const int row = rb * kRows + r0 + r;
    if (row < p.OUT) {
      float sum = 0.0f;
      for (int q = 0; q < p.S; ++q)
        sum += *reinterpret_cast<const float*>(smem + lt_recv_off((q * kLtTok + tok) * R + r));
      store_y(p.y, static_cast<int64_t>(tok) * p.OUT + row, sum, p.y_dtype, false);
    }
  }
}

// ============================================================================
// d8 variant: a dense d8 projection whose whole codebook fits shared memory
// (K <= 4096 entries of 8 fp16 = 64 KB; benchmark configuration C1:
// 4096 x 4096, K4096, 12-bit codes) at up to 8 rows, in the reference's
// _decode_matmul arithmetic (vq_dense.py:267-312): W = fp16(cb * s), then bf16
// for bf16 x; x as it is; fp32 accumulation; y rounded once.
//   * the codebook (plus a zero entry at index K: codes >= K read zeros) is
//     copied whole into shared memory; a lookup is one 16-byte read;
//   * a window's codes are 64 codes x bits of each of 256 rows (8 * bits bytes
//     per row, one TMA box, even bits only so a row is whole 16-byte units);
//   * inside a 64-input group thread t of a quad owns inputs 16t .. 16t+15,
//     i.e. codes 2t and 2t+1 (one funnel shift of two words holds both), and
//     MMA step m takes inputs 16t+4m .. 16t+4m+3 (a permutation of k applied
//     to A and B alike); W is prescaled per element (HMUL2 by the row's group
//     scale) and accumulated by the MMA directly;
//   * work split, copies, bounded waits, cluster split-K and the status word
//     as in the d2 kernel above.
constexpr int kL8MaxK = 4096;
constexpr uint32_t kL8RecvBytes = 8448;  // [split][token][owned row] floats: S x 8 x ceil(256 / S) <= 2080
constexpr uint32_t kL8ScaleOff(int bits) { return 256u * 8u * static_cast<uint32_t>(bits); }
constexpr uint32_t kL8XOff(int bits) { return kL8ScaleOff(bits) + 16u * kLtRows; }
constexpr uint32_t kL8StageBytes(int bits) { return (kL8XOff(bits) + kLtTok * kLtXStride + 1023u) & ~1023u; }

struct L8Params {
  const uint4* codebook;  // [K] entries of eight fp16
  int K, bits;
  const void* x;          // [T][IN] fp16 / bf16
  void* y;                // [T][OUT]
  int y_dtype;
  int T, OUT, IN;
  int S, nw;
  uint32_t table_bytes;   // (K + 1) * 16 rounded up to 1024
  uint32_t stage_bytes;
  int* status;
};

__device__ __forceinline__ uint32_t l8_scale_word(uint32_t w, uint32_t s2, bool bf16) {
  __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&w), *reinterpret_cast<const __half2*>(&s2));
  uint32_t r = *reinterpret_cast<uint32_t*>(&h);
  if (bf16) {
    const float2 f = __half22float2(h);
    __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
    r = *reinterpret_cast<uint32_t*>(&b);
  }
  return r;
}

__device__ __forceinline__ void l8_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, bool bf16) {
  if (bf16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One staged window for one warp: rows 16 wt + g and + 8, tokens 2t, 2t + 1,
// scale groups qlo .. qlo + NQ - 1 of the window.
template <bool XBF16, int NQ>
__device__ __forceinline__ void l8_window(const unsigned char* table, const unsigned char* sb, const L8Params& p,
                                          int wt, int qlo, int g, int t, bool has_x, float (&acc)[4]) {
  const int warp = wt;
  const int bits = p.bits;
  const uint32_t mask = (1u << bits) - 1u;
  const int rw = 2 * bits;  // code words per row
  const uint32_t* crow0 = reinterpret_cast<const uint32_t*>(sb) + (warp * 16 + g) * rw;
  const uint32_t* crow1 = crow0 + 8 * rw;
  const uint32_t kmax = static_cast<uint32_t>(p.K);
  const uint4 sc0 = *reinterpret_cast<const uint4*>(sb + kL8ScaleOff(bits) + (warp * 16 + g) * 16);
  const uint4 sc1 = *reinterpret_cast<const uint4*>(sb + kL8ScaleOff(bits) + (warp * 16 + g + 8) * 16);
  const unsigned char* xb = sb + kL8XOff(bits) + g * kLtXStride + 32 * t;
  const int tb = 2 * t * bits;  // bit offset of code 2t inside a group's 8 codes
#pragma unroll
  for (int qi = 0; qi < NQ; ++qi) {
    const int q = qlo + qi;
    const int b0 = 8 * q * bits + tb;
    const int wi = b0 >> 5, sh = b0 & 31;
    const uint32_t v0 = __funnelshift_r(crow0[wi], crow0[wi + 1], sh);
    const uint32_t v1 = __funnelshift_r(crow1[wi], crow1[wi + 1], sh);
    const uint32_t c00 = min(v0 & mask, kmax), c01 = min((v0 >> bits) & mask, kmax);
    const uint32_t c10 = min(v1 & mask, kmax), c11 = min((v1 >> bits) & mask, kmax);
    const uint4 e00 = *reinterpret_cast<const uint4*>(table + c00 * 16u);
    const uint4 e01 = *reinterpret_cast<const uint4*>(table + c01 * 16u);
    const uint4 e10 = *reinterpret_cast<const uint4*>(table + c10 * 16u);
    const uint4 e11 = *reinterpret_cast<const uint4*>(table + c11 * 16u);
    uint4 xv0 = make_uint4(0u, 0u, 0u, 0u), xv1 = xv0;
    if (has_x) {
      xv0 = *reinterpret_cast<const uint4*>(xb + 128 * q);
      xv1 = *reinterpret_cast<const uint4*>(xb + 128 * q + 16);
    }
    // the rows' group-q scales as fp16 pairs
    const uint32_t p0 = (q >> 1) == 0 ? sc0.x : ((q >> 1) == 1 ? sc0.y : ((q >> 1) == 2 ? sc0.z : sc0.w));
    const uint32_t p1 = (q >> 1) == 0 ? sc1.x : ((q >> 1) == 1 ? sc1.y : ((q >> 1) == 2 ? sc1.z : sc1.w));
    const uint32_t h0 = (q & 1) ? (p0 >> 16) : (p0 & 0xFFFFu), h1 = (q & 1) ? (p1 >> 16) : (p1 & 0xFFFFu);
    const uint32_t s0 = h0 | (h0 << 16), s1 = h1 | (h1 << 16);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      // step m: code 2t (m < 2) or 2t + 1, dimensions 4 (m & 1) .. + 3
      const uint4& r0 = m < 2 ? e00 : e01;
      const uint4& r1 = m < 2 ? e10 : e11;
      uint32_t a[4];
      a[0] = l8_scale_word((m & 1) ? r0.z : r0.x, s0, XBF16);
      a[2] = l8_scale_word((m & 1) ? r0.w : r0.y, s0, XBF16);
      a[1] = l8_scale_word((m & 1) ? r1.z : r1.x, s1, XBF16);
      a[3] = l8_scale_word((m & 1) ? r1.w : r1.y, s1, XBF16);
      const uint32_t bb0 = m == 0 ? xv0.x : (m == 1 ? xv0.z : (m == 2 ? xv1.x : xv1.z));
      const uint32_t bb1 = m == 0 ? xv0.y : (m == 1 ? xv0.w : (m == 2 ? xv1.y : xv1.w));
      l8_mma(acc, a, bb0, bb1, XBF16);
    }
  }
}

// KQ = 1: 256 rows per CTA, warp w owns tile w and all 8 groups of a window.
// KQ = 2: 128 rows per CTA (twice the CTAs for the same work); warps w and
// w + 8 share tile w % 8 and take groups 0-3 and 4-7, their fp32 partials
// added in that order before the store.
template <bool XBF16, int KQ>
__global__ void __launch_bounds__(kLtThreads, 1) dense_lut8_kernel(const __grid_constant__ LtMaps maps,
                                                                   const __grid_constant__ L8Params p) {
  constexpr int kRows = kLtRows / KQ, kTiles = kLtWarps / KQ;
  extern __shared__ __align__(16) unsigned char smem[];
  // [table (K + 1 entries)][recv][pad to 1024][stages][barriers]
  float* recv = reinterpret_cast<float*>(smem + p.table_bytes);
  const uint32_t pre = p.table_bytes + kL8RecvBytes;
  unsigned char* stages = smem + pre + ((1024u - ((smem_u32(smem) + pre) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + kLtStages * p.stage_bytes);
  uint64_t* empty = full + kLtStages;
  uint64_t* tbar = empty + kLtStages;
  int* sflags = reinterpret_cast<int*>(tbar + 1);  // [0] abort, [1] windows issued
  volatile int* abort_flag = sflags;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int rb = blockIdx.x / p.S, split = blockIdx.x - rb * p.S;
  const int w0 = split * p.nw / p.S, w1 = (split + 1) * p.nw / p.S, nwin = w1 - w0;
  const int rw = 2 * p.bits;  // code words of a row per window

  if (tid == 0) {
    for (int s = 0; s < kLtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kLtWarps);
    }
    mbar_init(tbar, 1);
    sflags[0] = 0;
    sflags[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // this CTA's windows into L2 while the previous kernel finishes (a
    // prefetch returns no data, so it cannot observe a stale value)
    for (int w = w0; w < w1; ++w) {
      lt_prefetch_2d(&maps.codes, w * rw, rb * kRows);
      lt_prefetch_2d(&maps.scales, w * 8, rb * kRows);
    }
    // the zero entry at index K
    *reinterpret_cast<uint4*>(smem + static_cast<uint32_t>(p.K) * 16u) = make_uint4(0u, 0u, 0u, 0u);
  }
  // the codebook's 128-byte lines into L2, one per thread
  for (int b = tid * 128; b < p.K * 16; b += kLtThreads * 128)
    asm volatile("prefetch.global.L2 [%0];" :: "l"(reinterpret_cast<const char*>(p.codebook) + b));
  {
    const int per = (kLtTok - p.T) * (kLtXStride / 16);
    for (int i = tid; i < kLtStages * per; i += kLtThreads) {
      const int s = i / per, r = i - s * per;
      *reinterpret_cast<uint4*>(stages + s * p.stage_bytes + kL8XOff(p.bits) + p.T * kLtXStride + r * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __syncthreads();
  if (p.S > 1) lt_cluster_arrive_relaxed();
  pdl_wait();
  pdl_trigger();
  const unsigned char* xg = static_cast<const unsigned char*>(p.x);
  const uint32_t tx = static_cast<uint32_t>(kRows) * 8u * static_cast<uint32_t>(p.bits) + 16u * kRows +
                      static_cast<uint32_t>(p.T) * kLtWinK * 2u;
  auto issue = [&](int n) {
    unsigned char* sb = stages + (n & 1) * p.stage_bytes;
    const int w = w0 + n;
    mbar_expect_tx(&full[n & 1], tx);
    tma_load_2d(&maps.codes, &full[n & 1], sb, w * rw, rb * kRows);
    tma_load_2d(&maps.scales, &full[n & 1], sb + kL8ScaleOff(p.bits), w * 8, rb * kRows);
    for (int j = 0; j < p.T; ++j)
      bulk_load(sb + kL8XOff(p.bits) + j * kLtXStride,
                xg + (static_cast<size_t>(j) * p.IN + static_cast<size_t>(w) * kLtWinK) * 2, kLtWinK * 2, &full[n & 1]);
  };
  if (tid == 0) {
    if (blockIdx.x == 0) p.status[1] = 0;
    // the codebook, whole (16-byte pieces of up to 16 KB)
    const uint32_t cbytes = static_cast<uint32_t>(p.K) * 16u;
    mbar_expect_tx(tbar, cbytes);
    for (uint32_t off = 0; off < cbytes; off += 16384u)
      bulk_load(smem + off, reinterpret_cast<const unsigned char*>(p.codebook) + off,
                cbytes - off < 16384u ? cbytes - off : 16384u, tbar);
    for (int n = 0; n < kLtStages && n < nwin; ++n) issue(n);
    sflags[1] = nwin < kLtStages ? nwin : kLtStages;
  }
  __syncthreads();

  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const int g = lane >> 2, t = lane & 3;
  const int wt = warp % kTiles, kq = warp / kTiles;  // MMA tile, group share
  bool alive = warp_wait(tbar, 0, abort_flag);
  for (int n = 0; n < nwin; ++n) {
    const int st = n & 1;
    const unsigned char* sb = stages + st * p.stage_bytes;
    if (alive) alive = warp_wait(&full[st], (n >> 1) & 1, abort_flag);
    if (alive) l8_window<XBF16, 8 / KQ>(smem, sb, p, wt, kq * (8 / KQ), g, t, g < p.T, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (tid == 0 && n + kLtStages < nwin && !*abort_flag) {
      if (mbar_wait(&empty[st], (n >> 1) & 1, abort_flag)) {
        issue(n + kLtStages);
        sflags[1] = n + kLtStages + 1;
      }
    }
  }
  if constexpr (KQ == 2) {
    // every warp is past its last window: stage 0's first 4 KB holds the
    // second group share's partials, added after the first's
    __syncthreads();
    float* red = reinterpret_cast<float*>(stages);
    if (kq == 1)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[(wt * 32 + lane) * 4 + e] = acc[e];
    __syncthreads();
    if (kq == 0)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = acc[e] + red[(wt * 32 + lane) * 4 + e];
  }
  if (p.S == 1 && kq == 0) {
    const int row0 = rb * kRows + wt * 16 + g;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = row0 + 8 * (e >> 1), tok = 2 * t + (e & 1);
      if (row < p.OUT && tok < p.T) store_y(p.y, static_cast<int64_t>(tok) * p.OUT + row, acc[e], p.y_dtype, false);
    }
  }
  __syncthreads();
  if (tid == 0) {
    const int issued = sflags[1];
    for (int k = issued > kLtStages ? issued - kLtStages : 0; k < issued; ++k) mbar_drain(&full[k & 1], (k >> 1) & 1);
    mbar_drain(tbar, 0);
    if (*abort_flag) p.status[1] = static_cast<int>(VQB_TIMEOUT);
  }
  if (p.S == 1) return;
  // ---- split-K over the cluster: the owner of local row lr is rank lr / R
  const int R = (kRows + p.S - 1) / p.S;
  lt_cluster_wait();
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int lr = wt * 16 + 8 * (e >> 1) + g, tok = 2 * t + (e & 1);
    if (kq == 0 && tok < p.T) {
      const int owner = lr / R;
      lt_st_cluster(smem_u32(recv + (split * kLtTok + tok) * R + (lr - owner * R)), static_cast<uint32_t>(owner),
                    acc[e]);
    }
  }
  lt_cluster_sync();
  const int r0 = split * R, nr = (r0 + R < kRows ? R : kRows - r0);
  for (int k = tid; k < p.T * nr; k += kLtThreads) {
    const int tok = k / nr, r = k - tok * nr;
    const int row = rb * kRows + r0 + r;
    if (row < p.OUT) {
      float sum = 0.0f;
      for (int q = 0; q < p.S; ++q) sum += recv[(q * kLtTok + tok) * R + r];
      store_y(p.y, static_cast<int64_t>(tok) * p.OUT + row, sum, p.y_dtype, false);
    }
  }
}

}  // namespace

// ------------------------------------------------------------------ host

bool dense_lut_geometry(const LinearGeometry& g) {
  return g.E == 1 && g.row_table == nullptr && g.D == 2 && g.bits == 8 && g.K >= 1 && g.K <= 256 && g.G == 64 &&
         g.OUT >= 1 && g.IN >= kLtWinK && g.IN % kLtWinK == 0 && g.row_words == g.IN / 8;
}

bool dense_lut_eligible(const LinearGeometry& g, const void* x, int x_dtype, int T) {
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return dense_lut_geometry(g) && T >= 1 && T <= kLtTok && (x_dtype == VQB_F16 || x_dtype == VQB_BF16) && a16(x) &&
         a16(g.codes) && a16(g.scales) && (reinterpret_cast<uintptr_t>(g.codebook) & 3) == 0;
}

// Clusters of S CTAs (kLtThreads threads and `smem` bytes each) that fit on
// the current device at once; 0 when the query fails, and that cluster size
// is not used.  Answers are cached per (device, kernel, S, smem) under a lock,
// so a call costs one map lookup after the first.
template <typename... KArgs>
static int lt_cluster_capacity(void (*kern)(KArgs...), int S, uint32_t smem, int sms) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int, uint32_t>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const auto key = std::make_tuple(dev, reinterpret_cast<const void*>(kern), S, smem);
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(S * sms));
  cfg.blockDim = dim3(kLtThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(S);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

vqb_status launch_dense_lut(const LinearGeometry& g, const void* x, int x_dtype, int T, void* y, int y_dtype,
                            int* status, cudaStream_t stream) {
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return VQB_CUDA_ERROR;
  using Kern = void (*)(LtMaps, LtParams);
  const bool bf = x_dtype == VQB_BF16;
  const Kern kerns[2] = {bf ? dense_lut_kernel<true, 1> : dense_lut_kernel<false, 1>,
                         bf ? dense_lut_kernel<true, 2> : dense_lut_kernel<false, 2>};
  for (Kern k : kerns)
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kLtSmem)) !=
        cudaSuccess)
      return VQB_CUDA_ERROR;
  LtParams p{};
  p.codebook = static_cast<const uint32_t*>(g.codebook);
  p.K = g.K;
  p.x = x;
  p.y = y;
  p.y_dtype = y_dtype;
  p.T = T;
  p.OUT = g.OUT;
  p.IN = g.IN;
  p.nw = g.IN / kLtWinK;
  p.status = status;
  // rows per CTA (256, or 128 with the window's groups split over warp pairs)
  // and CTAs per row block: the smallest (waves of clusters) x (windows per
  // CTA) x (rows per CTA), the first found among equals -- 5120 x 5120: 20
  // row blocks of 256 x 5 splits of 2 windows; 1024 x 5120: 8 row blocks of
  // 128 x 5 splits
  const int smax = p.nw < kLtMaxSplit ? p.nw : kLtMaxSplit;
  int best_kq = 1, best_s = 1;
  int64_t best_cost = INT64_MAX;
  for (int kq = 1; kq <= 2; ++kq) {
    const int rows = kLtRows / kq;
    const int nrb = (g.OUT + rows - 1) / rows;
    for (int S = 1; S <= smax; ++S) {
      const int cap = S == 1 ? di.sms : lt_cluster_capacity(kerns[kq - 1], S, kLtSmem, di.sms);
      if (cap <= 0) continue;
      const int64_t cost = ((nrb + cap - 1) / cap) * static_cast<int64_t>((p.nw + S - 1) / S) * rows;
      if (cost < best_cost) {
        best_cost = cost;
        best_kq = kq;
        best_s = S;
      }
    }
  }
  p.S = best_s;
  const int rows = kLtRows / best_kq;
  const int nrb = (g.OUT + rows - 1) / rows;
  LtMaps maps;
  if (!encode_2d(enc, &maps.codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, g.codes, static_cast<uint64_t>(g.row_words),
                 static_cast<uint64_t>(g.OUT), 32, static_cast<uint32_t>(rows), CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(enc, &maps.scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, g.scales, static_cast<uint64_t>(g.IN / 64),
                 static_cast<uint64_t>(g.OUT), kLtWinK / 64, static_cast<uint32_t>(rows), CU_TENSOR_MAP_SWIZZLE_NONE))
    return VQB_CUDA_ERROR;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(best_s);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(nrb * best_s));
  cfg.blockDim = dim3(kLtThreads);
  cfg.dynamicSmemBytes = kLtSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = best_s > 1 ? 2 : 1;
  timer_before(stream);
  const cudaError_t ce = cudaLaunchKernelEx(&cfg, kerns[best_kq - 1], maps, p);
  timer_after(stream);
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

// ------------------------------------------------------------- host: d8

bool dense_lut8_eligible(const LinearGeometry& g, const void* x, int x_dtype, int T) {
  const auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  return g.E == 1 && g.row_table == nullptr && g.D == 8 && g.K >= 1 && g.K <= kL8MaxK && g.bits >= 2 &&
         g.bits <= 16 && (g.bits & 1) == 0 && g.K <= (1 << g.bits) && g.G == 64 && g.OUT >= 1 && g.IN >= kLtWinK &&
         g.IN % kLtWinK == 0 && g.row_words == g.IN / 256 * g.bits && T >= 1 && T <= kLtTok &&
         (x_dtype == VQB_F16 || x_dtype == VQB_BF16) && a16(x) && a16(g.codes) && a16(g.scales) && a16(g.codebook);
}

vqb_status launch_dense_lut8(const LinearGeometry& g, const void* x, int x_dtype, int T, void* y, int y_dtype,
                             int* status, cudaStream_t stream) {
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return VQB_CUDA_ERROR;
  L8Params p{};
  p.codebook = static_cast<const uint4*>(g.codebook);
  p.K = g.K;
  p.bits = g.bits;
  p.x = x;
  p.y = y;
  p.y_dtype = y_dtype;
  p.T = T;
  p.OUT = g.OUT;
  p.IN = g.IN;
  p.nw = g.IN / kLtWinK;
  p.status = status;
  p.table_bytes = (static_cast<uint32_t>(g.K + 1) * 16u + 1023u) & ~1023u;
  p.stage_bytes = kL8StageBytes(g.bits);
  const uint32_t smem = p.table_bytes + kL8RecvBytes + 1024u + kLtStages * p.stage_bytes + 64u;
  if (smem > static_cast<uint32_t>(di.smem_optin)) return VQB_UNSUPPORTED_GEOMETRY;
  using Kern = void (*)(LtMaps, L8Params);
  const bool bf = x_dtype == VQB_BF16;
  const Kern kerns[2] = {bf ? dense_lut8_kernel<true, 1> : dense_lut8_kernel<false, 1>,
                         bf ? dense_lut8_kernel<true, 2> : dense_lut8_kernel<false, 2>};
  for (Kern k : kerns)
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
      return VQB_CUDA_ERROR;
  // rows per CTA (256, or 128 with the window's groups split over warp
  // pairs) and CTAs per row block: the smallest (waves of clusters) x
  // (windows per CTA) x (rows per CTA), the first found among equals -- C1:
  // 32 row blocks of 128 x 4 splits, 128 CTAs in one wave
  const int smax = p.nw < kLtMaxSplit ? p.nw : kLtMaxSplit;
  int best_kq = 1, best_s = 1;
  int64_t best_cost = INT64_MAX;
  for (int kq = 1; kq <= 2; ++kq) {
    const int rows = kLtRows / kq;
    const int nrb = (g.OUT + rows - 1) / rows;
    for (int S = 1; S <= smax; ++S) {
      const int cap = S == 1 ? di.sms : lt_cluster_capacity(kerns[kq - 1], S, smem, di.sms);
      if (cap <= 0) continue;
      const int64_t cost = ((nrb + cap - 1) / cap) * static_cast<int64_t>((p.nw + S - 1) / S) * rows;
      if (cost < best_cost) {
        best_cost = cost;
        best_kq = kq;
        best_s = S;
      }
    }
  }
  p.S = best_s;
  const int rows = kLtRows / best_kq;
  const int nrb = (g.OUT + rows - 1) / rows;
  LtMaps maps;
  if (!encode_2d(enc, &maps.codes, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, g.codes, static_cast<uint64_t>(g.row_words),
                 static_cast<uint64_t>(g.OUT), static_cast<uint32_t>(2 * g.bits), static_cast<uint32_t>(rows),
                 CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(enc, &maps.scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, g.scales, static_cast<uint64_t>(g.IN / 64),
                 static_cast<uint64_t>(g.OUT), kLtWinK / 64, static_cast<uint32_t>(rows), CU_TENSOR_MAP_SWIZZLE_NONE))
    return VQB_CUDA_ERROR;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(best_s);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(nrb * best_s));
  cfg.blockDim = dim3(kLtThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = best_s > 1 ? 2 : 1;
  timer_before(stream);
  const cudaError_t ce = cudaLaunchKernelEx(&cfg, kerns[best_kq - 1], maps, p);
  timer_after(stream);
  if (ce != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  return VQB_OK;
}

}  // namespace vqb
