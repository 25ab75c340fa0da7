// Grouped VQ GEMM for large token counts on the 5th-generation tensor cores
// (sm_100a: tcgen05.mma with the accumulator and the A operand in tensor
// memory, B staged by TMA).  The B200 counterpart of the reference's
// segmented, count-sorted prefill GEMM (gemmseg2, vq_switch.py:3687-4310,
// dispatched by _gemmseg_prefill :4569-4722) and of the dense large-N path
// (_decode_matmul, vq_dense.py:267-312).
//
// Work: pairs are sorted by expert and x is gathered into that order (fp16,
// or bf16 for the dense bf16 arm); a tile is (expert e, 128 output rows,
// up to 256 of e's tokens).  Per tile and K chunk of 64:
//   * 4 decode warps (thread = output row = TMEM lane) walk their row's packed
//     code stream, look each code up in the codebook (shared-memory prefix,
//     rest through L1), scale it -- W = fp16(cb * s), one RNE rounding -- and
//     store the 64 weights of the chunk into a TMEM A buffer (tcgen05.st);
//   * a TMA warp loads the 64-wide token tile of x into shared memory
//     (128-byte swizzle, the canonical K-major UMMA layout);
//   * one elected thread of the MMA warp issues four tcgen05.mma (K = 16 each)
//     D[128 x N] += A_tmem[128 x 16] . B_smem[16 x N] and commits to the
//     barriers that free the A and B buffers.
// After the last chunk the decode warps read D from TMEM (tcgen05.ld) and
// store y[pair, row] with the output rounding.  N is the tile's real token
// count rounded up to 16, so small experts cost only their own columns.
//
// Numerics: the weights take one fp16 rounding of cb*s (the reference's
// non-ACCS / dense arms round the same product; its ACCS arm applies s to
// fp32 group partials instead), x is fp16 (the MoE host cast) or bf16 with
// bf16(fp16(cb*s)) weights (dense bf16, vq_dense.py:294), accumulation fp32.
//
// Every mbarrier wait is bounded: on expiry the CTA records VQB_TIMEOUT in
// the status word, stops issuing, frees its tensor memory and returns.
#include <cuda.h>

#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

namespace {

constexpr int kTileM = 128;
constexpr int kChunkK = 64;          // K per pipeline stage (one 128-byte swizzle row of fp16)
constexpr int kMaxN = 256;           // tokens per tile
constexpr int kBStages = 3;
constexpr int kAStages = 4;         // two chunks decoded per iteration, double-buffered
constexpr int kThreads = 256;        // warp 0: TMA + TMEM alloc, warp 1: MMA, warps 4-7: decode + epilogue
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSpinLimit = 1u << 26;

struct TParams {
  const uint32_t* codes;
  const uint16_t* codebook;
  const uint16_t* scales;
  const int* sorted;       // pair ids grouped by expert
  const int4* chunks;      // (expert, first sorted slot, tokens <= 256, 0)
  const int* meta;         // [0] chunk count
  int* status;             // [1] <- VQB_TIMEOUT on a bounded-wait expiry
  void* y;
  int64_t expert_words;
  int row_words;
  int OUT, IN, G, NGRP, bits;
  int ns;                  // codebook entries staged in shared memory
  int row_tiles;
  int y_dtype;
  int round_f16_first;
  int b_bf16;              // B (x) and A are bf16 (dense bf16 arm)
};

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// bounded wait: false when the limit expired (the caller aborts)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && *abort_flag) return false;
  }
  *abort_flag = 1;
  return false;
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem desc]
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void tc_st_x32(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
         "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
         "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
         "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tc_ld_x16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// K-major, 128-byte swizzle shared-memory matrix descriptor (sm_100 format:
// start >> 4 at [0,14), leading byte offset >> 4 at [16,30) (unused for
// swizzled K-major, set to 1), stride byte offset >> 4 at [32,46) = 1024 B
// between 8-row groups, version 1 at [46,48), layout type 2 (SWIZZLE_128B) at
// [61,64)).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulator, A/B fp16 or bf16, both
// K-major, N >> 3 at [17,23), M >> 4 at [24,29).
__device__ __forceinline__ uint32_t make_idesc(int n, bool bf16) {
  uint32_t d = 0;
  d |= 1u << 4;                                // c_format F32
  d |= (bf16 ? 1u : 0u) << 7;                  // a_format
  d |= (bf16 ? 1u : 0u) << 10;                 // b_format
  d |= static_cast<uint32_t>(n >> 3) << 17;    // n_dim
  d |= static_cast<uint32_t>(kTileM >> 4) << 24;  // m_dim
  return d;
}

// -------------------------------------------------------------- the kernel

template <int D>
__device__ __forceinline__ void decode_chunk(const TParams& prm, const uint16_t* cb_s, PrefetchWalker& wk,
                                             uint32_t mask, __half2 s2, uint32_t* out) {
  // 64 k of one row -> 32 fp16x2 words, W = fp16(cb * s)
  constexpr int CODES = kChunkK / D;
  constexpr int WPC = D / 2;
  uint32_t c[CODES];
#pragma unroll
  for (int i = 0; i < CODES; ++i) c[i] = wk.next(prm.bits, mask);
#pragma unroll
  for (int i = 0; i < CODES; ++i) {
    if constexpr (D == 8) {
      const uint4 v = c[i] < static_cast<uint32_t>(prm.ns) ? reinterpret_cast<const uint4*>(cb_s)[c[i]]
                                                           : __ldg(reinterpret_cast<const uint4*>(prm.codebook) + c[i]);
      out[WPC * i] = v.x; out[WPC * i + 1] = v.y; out[WPC * i + 2] = v.z; out[WPC * i + 3] = v.w;
    } else if constexpr (D == 4) {
      const uint2 v = c[i] < static_cast<uint32_t>(prm.ns) ? reinterpret_cast<const uint2*>(cb_s)[c[i]]
                                                           : __ldg(reinterpret_cast<const uint2*>(prm.codebook) + c[i]);
      out[WPC * i] = v.x; out[WPC * i + 1] = v.y;
    } else {
      out[i] = c[i] < static_cast<uint32_t>(prm.ns) ? reinterpret_cast<const uint32_t*>(cb_s)[c[i]]
                                                    : __ldg(reinterpret_cast<const uint32_t*>(prm.codebook) + c[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    __half2 h = __hmul2(*reinterpret_cast<__half2*>(&out[i]), s2);
    out[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  if (prm.b_bf16) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float2 f = h2x2f(out[i]);
      __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
      out[i] = *reinterpret_cast<uint32_t*>(&b);
    }
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) vq_prefill_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                  const TParams prm) {
  extern __shared__ __align__(16) unsigned char smem_dyn[];
  // layout: [B stages (1024-aligned: the 128-byte swizzle atom)][codebook prefix][barriers][tmem addr][flags]
  unsigned char* smem_raw = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  const size_t b_stage_bytes = static_cast<size_t>(kMaxN) * kChunkK * 2;  // 32 KB
  unsigned char* b_base = smem_raw;
  uint16_t* cb_s = reinterpret_cast<uint16_t*>(smem_raw + kBStages * b_stage_bytes);
  const size_t cb_bytes = (static_cast<size_t>(prm.ns) * D * 2 + 15) & ~size_t(15);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(cb_s) + ((cb_bytes + 7) & ~size_t(7)));
  uint64_t* b_full = bars;                      // [kBStages]
  uint64_t* b_empty = bars + kBStages;          // [kBStages]
  uint64_t* a_full = bars + 2 * kBStages;       // [kAStages]
  uint64_t* a_empty = a_full + kAStages;        // [kAStages]
  uint64_t* acc_full = a_empty + kAStages;      // [1]
  uint64_t* mma_done = acc_full + 1;            // [1] teardown: every issued MMA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBStages; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
    for (int i = 0; i < kAStages; ++i) { mbar_init(&a_full[i], 128); mbar_init(&a_empty[i], 1); }
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // codebook prefix -> shared memory
  {
    const uint4* src = reinterpret_cast<const uint4*>(prm.codebook);
    uint4* dst = reinterpret_cast<uint4*>(cb_s);
    const int n16 = static_cast<int>((static_cast<size_t>(prm.ns) * D * 2) / 16);
    for (int i = threadIdx.x; i < n16; i += kThreads) dst[i] = __ldg(src + i);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // TMEM columns: [0, 256) accumulator D, [256, 256 + 32 * kAStages) A buffers
  const uint32_t tmem_d = tmem_base;
  const uint32_t tmem_a = tmem_base + kMaxN;

  const int nchunks = prm.meta[0];
  const int64_t nitems = static_cast<int64_t>(nchunks) * prm.row_tiles;
  const int n_k = prm.IN / kChunkK;

  if (warp == 0) {
    // ---------------- TMA producer: token tiles of x, kBStages deep
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
      uint32_t stage = 0, phase = 0;
      int filled[kBStages] = {};
      uint32_t fill_phase[kBStages] = {};
      for (int64_t it = blockIdx.x; it < nitems && !*abort_flag; it += gridDim.x) {
        const int chunk = static_cast<int>(it / prm.row_tiles);
        const int4 ch = prm.chunks[chunk];
        for (int kc = 0; kc < n_k; ++kc) {
          if (!mbar_wait(&b_empty[stage], phase ^ 1u, abort_flag)) break;
          mbar_expect_tx(&b_full[stage], static_cast<uint32_t>(b_stage_bytes));
          tma_load_2d(&xmap, &b_full[stage], b_base + stage * b_stage_bytes, kc * kChunkK, ch.y);
          filled[stage] = 1;
          fill_phase[stage] = phase;
          if (++stage == kBStages) { stage = 0; phase ^= 1u; }
        }
      }
      // no copy may still be writing shared memory when the CTA exits
      for (int s2 = 0; s2 < kBStages; ++s2) {
        if (filled[s2]) {
          for (uint32_t i = 0; i < kSpinLimit && !mbar_try_wait(&b_full[s2], fill_phase[s2]); ++i) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one thread)
    if (lane == 0) {
      uint32_t bstage = 0, bphase = 0, astage = 0, aphase = 0;
      for (int64_t it = blockIdx.x; it < nitems && !*abort_flag; it += gridDim.x) {
        const int chunk = static_cast<int>(it / prm.row_tiles);
        const int4 ch = prm.chunks[chunk];
        const int n = (ch.z + 15) & ~15;
        const uint32_t idesc = make_idesc(n, prm.b_bf16 != 0);
        bool ok = true;
        for (int kc = 0; kc < n_k && ok; ++kc) {
          ok = mbar_wait(&a_full[astage], aphase, abort_flag) && mbar_wait(&b_full[bstage], bphase, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t b_addr = smem_u32(b_base + bstage * b_stage_bytes);
#pragma unroll
          for (int kk = 0; kk < kChunkK / 16; ++kk) {
            // A: 16 k = 8 columns of packed fp16 pairs; B: advance 32 bytes inside the swizzle row
            tc_mma_ts(tmem_d, tmem_a + astage * 32 + kk * 8, sw128_desc(b_addr + kk * 32), idesc,
                      (kc > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&b_empty[bstage]);
          tc_commit(&a_empty[astage]);
          if (++bstage == kBStages) { bstage = 0; bphase ^= 1u; }
          if (++astage == kAStages) { astage = 0; aphase ^= 1u; }
        }
        if (ok) tc_commit(acc_full);
      }
      // every MMA this thread issued has completed before TMEM is freed
      tc_commit(mma_done);
      for (uint32_t i = 0; i < kSpinLimit && !mbar_try_wait(mma_done, 0); ++i) {
      }
    }
  } else if (warp >= 4) {
    // ---------------- decode + epilogue (thread = row = TMEM lane)
    const int q = warp & 3;                       // TMEM lane quarter
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t mask = (1u << prm.bits) - 1u;
    uint32_t astage = 0, aphase = 0, accphase = 0;
    for (int64_t it = blockIdx.x; it < nitems && !*abort_flag; it += gridDim.x) {
      const int chunk = static_cast<int>(it / prm.row_tiles);
      const int rt = static_cast<int>(it - static_cast<int64_t>(chunk) * prm.row_tiles);
      const int4 ch = prm.chunks[chunk];
      const int e = ch.x;
      const int r = rt * kTileM + q * 32 + lane;
      const int rr = min(r, prm.OUT - 1);
      const uint32_t* row = prm.codes + static_cast<int64_t>(e) * prm.expert_words +
                            static_cast<int64_t>(rr) * prm.row_words;
      const uint16_t* srow = prm.scales + (static_cast<int64_t>(e) * prm.OUT + rr) * prm.NGRP;
      PrefetchWalker wk;
      wk.init(row, prm.row_words);
      bool ok = true;
      // two chunks per iteration: both chunks' lookups are in flight together
      for (int kc = 0; kc < n_k; kc += 2) {
        const bool two = kc + 1 < n_k;
        uint32_t w0[32], w1[32];
        const __half s0 = __ushort_as_half(__ldg(srow + (kc * kChunkK) / prm.G));
        const __half s1 = two ? __ushort_as_half(__ldg(srow + ((kc + 1) * kChunkK) / prm.G)) : s0;
        decode_chunk<D>(prm, cb_s, wk, mask, __halves2half2(s0, s0), w0);
        if (two) decode_chunk<D>(prm, cb_s, wk, mask, __halves2half2(s1, s1), w1);
        for (int h = 0; h < (two ? 2 : 1); ++h) {
          if (!mbar_wait(&a_empty[astage], aphase ^ 1u, abort_flag)) { ok = false; break; }
          tc_fence_after();
          tc_st_x32(tmem_a + lane_off + astage * 32, h == 0 ? w0 : w1);
          tc_wait_st();
          tc_fence_before();
          mbar_arrive(&a_full[astage]);
          if (++astage == kAStages) { astage = 0; aphase ^= 1u; }
        }
        if (!ok) break;
      }
      if (!ok) break;
      // epilogue: D columns [0, n) of this lane's row
      if (!mbar_wait(acc_full, accphase, abort_flag)) break;
      accphase ^= 1u;
      tc_fence_after();
      const int ntok = ch.z;
      for (int c0 = 0; c0 < ntok; c0 += 16) {
        uint32_t v[16];
        tc_ld_x16(tmem_d + lane_off + c0, v);
        tc_wait_ld();
        if (r < prm.OUT) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c0 + j < ntok) {
              const int pair = prm.sorted[ch.y + c0 + j];
              store_y(prm.y, static_cast<int64_t>(pair) * prm.OUT + r, __uint_as_float(v[j]), prm.y_dtype,
                      prm.round_f16_first != 0);
            }
          }
        }
      }
      tc_fence_before();
    }
  }

  // teardown: everyone done with TMEM before it is freed
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abort_flag && threadIdx.x == 0) atomicExch(prm.status + 1, static_cast<int>(VQB_TIMEOUT));
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(kTmemCols) : "memory");
}

// x rows gathered into expert-sorted order as 16-bit B rows: xs[s] = x[sorted[s] / krep]
__global__ void gather_sorted_kernel(const void* __restrict__ x, int x_dtype, const int* __restrict__ sorted, int N,
                                     int krep, int IN, int to_bf16, uint16_t* __restrict__ xs) {
  const int per_row = IN;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
       i < static_cast<int64_t>(N) * per_row; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(i / per_row);
    const int k = static_cast<int>(i - static_cast<int64_t>(s) * per_row);
    const int t = sorted[s] / krep;
    const float v = load_x(x, static_cast<int64_t>(t) * IN + k, x_dtype, false);
    xs[i] = to_bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int g_sms_tc = 0;

}  // namespace

bool tc_prefill_supported(const LinearGeometry& geo) {
  if (geo.IN % kChunkK != 0) return false;
  if (geo.G % kChunkK != 0) return false;      // one scale per row per 64-k chunk
  if (geo.bits > 16) return false;
  if ((reinterpret_cast<uintptr_t>(geo.codes) & 15) != 0 || geo.row_words % 4 != 0) return false;
  return true;
}

size_t tc_prefill_x_bytes(int64_t N, int IN) { return (static_cast<size_t>(N) * IN * 2 + 1023) & ~size_t(1023); }

vqb_status launch_prefill_tc(const LinearGeometry& geo, const void* x, int x_dtype, int krep, const RouteWorkspace& rw,
                             int N, uint16_t* xs, void* y, int y_dtype, bool round_f16_first, bool bf16_operands,
                             int* status, cudaStream_t stream) {
  if (N <= 0) return VQB_OK;
  if (g_sms_tc == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return VQB_CUDA_ERROR;
    if (cudaDeviceGetAttribute(&g_sms_tc, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return VQB_CUDA_ERROR;
  }
  EncodeTiledFn enc = encode_fn();
  if (!enc) return VQB_CUDA_ERROR;
  // 1. gather x into expert-sorted 16-bit rows
  {
    const int64_t n = static_cast<int64_t>(N) * geo.IN;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 8 * g_sms_tc) blocks = 8 * g_sms_tc;
    gather_sorted_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, x_dtype, rw.sorted, N, krep, geo.IN,
                                                                            bf16_operands ? 1 : 0, xs);
    if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
  }
  // 2. TMA map over xs [N rows, IN] 16-bit: box 64 x 256, 128-byte swizzle
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(geo.IN), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(geo.IN) * 2};
  cuuint32_t box[2] = {kChunkK, kMaxN};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&map, bf16_operands ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xs, dims,
          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return VQB_CUDA_ERROR;

  TParams prm{};
  prm.codes = static_cast<const uint32_t*>(geo.codes);
  prm.codebook = static_cast<const uint16_t*>(geo.codebook);
  prm.scales = static_cast<const uint16_t*>(geo.scales);
  prm.sorted = rw.sorted;
  prm.chunks = rw.chunks;
  prm.meta = rw.meta;
  prm.status = status;
  prm.y = y;
  prm.row_words = geo.row_words;
  prm.expert_words = static_cast<int64_t>(geo.OUT) * geo.row_words;
  prm.OUT = geo.OUT;
  prm.IN = geo.IN;
  prm.G = geo.G;
  prm.NGRP = geo.IN / geo.G;
  prm.bits = geo.bits;
  prm.row_tiles = (geo.OUT + kTileM - 1) / kTileM;
  prm.y_dtype = y_dtype;
  prm.round_f16_first = round_f16_first ? 1 : 0;
  prm.b_bf16 = bf16_operands ? 1 : 0;

  const size_t b_bytes = static_cast<size_t>(kBStages) * kMaxN * kChunkK * 2;
  const size_t tail = 256 + 1024;  // barriers, tmem slot, flags, and the 1024-byte alignment slack
  const size_t budget = 227 * 1024;
  const size_t entry = static_cast<size_t>(geo.D) * 2;
  size_t ns = (budget - b_bytes - tail - 16) / entry;
  ns = ns / 8 * 8;
  if (ns > static_cast<size_t>(geo.K)) ns = geo.K;
  prm.ns = static_cast<int>(ns);
  const size_t smem = b_bytes + ((ns * entry + 15) & ~size_t(15)) + tail + 16;

  cudaError_t ce;
  auto launch = [&](auto kern) {
    ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (ce != cudaSuccess) return;
    kern<<<g_sms_tc, kThreads, smem, stream>>>(map, prm);
    ce = cudaGetLastError();
  };
  if (geo.D == 8) launch(vq_prefill_tc_kernel<8>);
  else if (geo.D == 4) launch(vq_prefill_tc_kernel<4>);
  else launch(vq_prefill_tc_kernel<2>);
  return ce == cudaSuccess ? VQB_OK : VQB_CUDA_ERROR;
}

}  // namespace vqb
