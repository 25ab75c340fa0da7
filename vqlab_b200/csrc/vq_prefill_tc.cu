// Grouped VQ GEMM for large token counts on the 5th-generation tensor cores
// (sm_100a: tcgen05.mma with the accumulator and the A operand in tensor
// memory, B and the code stream staged by TMA).  The B200 counterpart of the
// reference's segmented, count-sorted prefill GEMM (gemmseg2,
// vq_switch.py:3687-4310, dispatched by _gemmseg_prefill :4569-4722) and of
// the dense large-N path (_decode_matmul, vq_dense.py:267-312).
//
// Work: pairs are sorted by expert and x is gathered into that order (fp16,
// or bf16 for the dense bf16 arm).  A tile is (expert e, 128 output rows, up
// to 128 of e's tokens); a CTA runs tiles one after another (persistent grid,
// one CTA per SM).  Per tile and K chunk of 64:
//   * 16 decode warps in 4 sets: set s decodes chunk s of every window of 4
//     chunks.  In a set, thread = output row = TMEM lane; it extracts the
//     chunk's codes from the window of packed rows a TMA warp staged in
//     shared memory, looks each one up in the shared-memory codebook, scales
//     it -- W = fp16(cb * s), one RNE rounding -- and stores the 64 weights of
//     its row into a TMEM A stage (tcgen05.st);
//   * a TMA warp loads the tile's tokens x[:, chunk] (boxes of 32 rows, only
//     as many as the tile has tokens; 128-byte swizzle, the canonical K-major
//     UMMA layout);
//   * one elected thread of the MMA warp issues four tcgen05.mma (K = 16 each)
//     D[128 x N] += A_tmem[128 x 16] . B_smem[16 x N] and commits to the
//     barriers that free the A and B buffers.
// Codebooks larger than the shared-memory slice (d8/K16384 is 256 KB) run in
// passes: pass h keeps entries [h*KP, (h+1)*KP) resident (a bulk copy by a
// loader warp), codes outside the slice contribute zero weights, and the
// accumulator collects every pass -- each weight is non-zero in exactly one
// pass, so the product sum is the single-pass one in another order.  Every
// lookup is a shared-memory read.  Consecutive tiles walk the slices in
// alternating order so one reload serves two passes.
// Two TMEM accumulators let the epilogue of one tile (tcgen05.ld, y[pair, row]
// with the output rounding) overlap the next tile's MMAs.
//
// Numerics: the weights take one fp16 rounding of cb*s (the reference's
// non-ACCS / dense arms round the same product; its ACCS arm applies s to
// fp32 group partials instead), x is fp16 (the MoE host cast) or bf16 with
// bf16(fp16(cb*s)) weights (dense bf16, vq_dense.py:294), accumulation fp32.
//
// Every mbarrier wait is bounded (2 s of %globaltimer): on expiry the CTA records VQB_TIMEOUT in
// the status word, stops issuing, waits for its copies in flight, frees its
// tensor memory and returns.
#include <cuda.h>

#include <algorithm>

#include "vqb_common.cuh"
#include "vqb_internal.h"
#include "vqb_tma.cuh"

namespace vqb {

namespace {

constexpr int kTileM = 128;
constexpr int kChunkK = 64;                          // K per A stage (one 128-byte swizzle row of fp16)
constexpr int kMaxN = kPrefillTileTokens;            // tokens per tile
constexpr int kBoxRows = 32;                         // x rows per TMA box
constexpr int kBStageBytes = kMaxN * kChunkK * 2;    // 16 KB
constexpr int kBStages = 4;                          // position g -> B stage g % 4
constexpr int kAStages = 8;                          // position g -> A stage g % 8 (two per decode set)
constexpr int kWStages = 3;                          // code/scale windows (the dimension-split layout uses 2)
constexpr int kSets = 4;                             // window = kSets chunks, one per set
constexpr int kIssuers = 2;                          // MMA issuing threads, one accumulator each
constexpr int kDecodeWarps = 4 * kSets;              // 4 TMEM lane quarters per set
// warp roles (a warp reaches TMEM lanes 32 * (warp % 4) ...; the issuers sit on different SM sub-partitions)
constexpr int kWarpTmaX = 0, kWarpMma0 = 1, kWarpTmaCode = 2, kWarpMma1 = 3, kWarpCbLoad = 4;
constexpr int kFirstDecodeWarp = 5;
constexpr int kThreads = (kFirstDecodeWarp + kDecodeWarps) * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = kIssuers * kMaxN;        // columns: [0,128) D0, [128,256) D1, then 8 A stages of 32
constexpr int kScaleRowBytes = 16;                   // 8 fp16 scales per row per window
constexpr int kNumBars = 2 * kBStages + 2 + kAStages + 2 * kWStages + 2 + kIssuers + 1 + kIssuers;

struct TParams {
  const uint32_t* codes;
  const uint16_t* codebook;
  const uint16_t* scales;
  const int* sorted;       // pair ids grouped by expert
  const int4* chunks;      // (expert, first sorted slot, tokens <= 128, 0)
  const int* meta;         // [0] chunk count
  int* status;             // [1] <- VQB_TIMEOUT on a bounded-wait expiry
  void* y;
  int OUT, IN, G, NGRP, bits, K;
  int n_k;                 // real K positions per pass (IN / 64; IN / 128 with the dimension split)
  int n_pos;               // A stages per tile per pass (n_k rounded up to whole windows)
  int wst;                 // code/scale window stages in use (<= kWStages)
  int row_tiles;
  int y_dtype;
  int round_f16_first;
  int b_bf16;              // B (x) and A are bf16 (dense bf16 arm)
  int W;                   // code window pitch in words
  int wswz;                // window layout: 0 plain (W / 4 odd), 1 64-byte swizzle (W 16), 2 128-byte swizzle (W 32)
  int wpw;                 // code words per window of the packed row
  int code_stage_bytes;
  int win_stage_bytes;
  int scale_tma;           // scales staged with the codes (else read from global)
  int log2g;
  int kp_log2;             // codebook entries per pass = 1 << kp_log2 (npass > 1)
  int kp;
  int npass;
  int kpos_log2;           // log2 of the original k a position covers (6; 7 with the dimension split)
  int off_win, off_cb, off_bar;
  const int32_t* row_table;  // SKIPZERO [E, OUT] -> compact row (-1 dead), nullptr = plain layout
  const int* tile_base;      // SKIPZERO: first compact row of each (expert, 128-row tile), -1 = all dead
  int64_t nrows;             // rows of codes / scales
  int max_group;             // tiles per group allowed by the L2 budget for re-read code windows
  int cb_early;              // the codebook (slice source) predates the kernel this one depends on
  int ksplit;                // work items per tile: split-K over its windows (1 = whole tiles)
  float* partial;            // ksplit > 1: fp32 partial tiles [item][pcols columns][128 rows]
  int pcols;                 // columns of a partial slot (tokens a chunk can hold, rounded to 16)
};

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

// Token rows a B slot holds for a tile of n tokens, and the K positions that
// share one B stage (a stage holds 128 token rows of 64 k).
__host__ __device__ __forceinline__ int slot_rows(int n) { return n <= 32 ? 32 : (n <= 64 ? 64 : 128); }
__host__ __device__ __forceinline__ int slot_positions(int rows) { return rows <= 32 ? 4 : (rows <= 64 ? 2 : 1); }

// Codebook slice a tile-pass reads: consecutive tiles of a CTA walk the
// slices in alternating order, so the slice resident at the end of one tile is
// the first one the next tile uses.
__device__ __forceinline__ int pass_slice(int npass, int tile_local, int pass) {
  return npass == 1 ? 0 : ((tile_local & 1) ? npass - 1 - pass : pass);
}

// ------------------------------------------------------------ decode side

// Look one code up in the shared-memory codebook slice.  The slice holds
// entries [h * KP, h * KP + KP) at [0, KP) and a zero entry at index `lim`
// (KP, or K with one pass): `c ^ sel` is below KP exactly when the code lies
// in the resident slice (sel = h * KP, KP a power of two), so min(c ^ sel, lim)
// reads either the code's entry or the zero entry -- one unconditional
// shared-memory load per code, and out-of-range codes read zeros too.
template <int D>
__device__ __forceinline__ void lookup(const uint16_t* cb_s, uint32_t c, uint32_t sel, uint32_t lim, uint32_t* out) {
  const uint32_t li = min(c ^ sel, lim);
  if constexpr (D == 8) {
    const uint4 v = reinterpret_cast<const uint4*>(cb_s)[li];
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  } else if constexpr (D == 4) {
    const uint2 v = reinterpret_cast<const uint2*>(cb_s)[li];
    out[0] = v.x; out[1] = v.y;
  } else {
    out[0] = reinterpret_cast<const uint32_t*>(cb_s)[li];
  }
}

// The NC consecutive codes starting at bit b0 of a staged window row, for a
// compile-time width BITS: the bits are read with conflict-free 16-byte loads,
// aligned to bit 0 with a funnel shift, and every code then sits at a fixed
// bit position.  crow: the row in the staged code window (16-byte aligned,
// pitch W words), whose 16-byte units sit at index ^ xr (the TMA swizzle of
// this row; 0 for the plain layout) -- either way 16-byte reads by 32
// consecutive rows hit 32 different bank groups; b0 is the same for every row.
template <int BITS, int NC>
__device__ __forceinline__ void extract_codes(const uint32_t* crow, int xr, int b0, uint32_t* c) {
  constexpr uint32_t MASK = (1u << BITS) - 1u;
  constexpr int NB = NC * BITS;              // bits of the codes
  constexpr int NW = (NB + 31) / 32 + 1;     // words holding them after word alignment (+ straddle)
  constexpr int NQ = (NW + 3 + 3) / 4;       // 16-byte loads that cover a start anywhere in a 16-byte unit
  const int w0 = b0 >> 5, sh = b0 & 31, dw = w0 & 3;
  const uint4* row4 = reinterpret_cast<const uint4*>(crow);
  uint32_t q[4 * NQ];
#pragma unroll
  for (int i = 0; i < NQ; ++i) {
    const uint4 v = row4[((w0 >> 2) + i) ^ xr];
    q[4 * i] = v.x; q[4 * i + 1] = v.y; q[4 * i + 2] = v.z; q[4 * i + 3] = v.w;
  }
  // drop the dw leading words (dw is the same for the whole warp)
  uint32_t t[4 * NQ - 2];
#pragma unroll
  for (int i = 0; i < 4 * NQ - 2; ++i) t[i] = (dw & 2) ? q[i + 2] : q[i];
  uint32_t r[NW];
#pragma unroll
  for (int i = 0; i < NW; ++i) r[i] = (dw & 1) ? t[i + 1] : t[i];
  uint32_t n[NW - 1];
#pragma unroll
  for (int i = 0; i < NW - 1; ++i) n[i] = __funnelshift_r(r[i], r[i + 1], sh);
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int bit = i * BITS, wi = bit >> 5, bs = bit & 31;
    const uint32_t v = (bs + BITS <= 32) ? (n[wi] >> bs) : __funnelshift_r(n[wi], n[wi + 1], bs);
    c[i] = v & MASK;
  }
}

// W = fp16(cb * s) in place over 32 fp16x2 words (words [0, 16) take s_lo,
// [16, 32) s_hi), then bf16 for the bf16 operand arm.
__device__ __forceinline__ void scale_words(uint32_t* out, __half2 s_lo, __half2 s_hi, bool to_bf16) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    __half2 v = __hmul2(*reinterpret_cast<__half2*>(&out[i]), i < 16 ? s_lo : s_hi);
    out[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  if (to_bf16) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float2 f = h2x2f(out[i]);
      __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
      out[i] = *reinterpret_cast<uint32_t*>(&b);
    }
  }
}

// One row's 64 weights of one chunk -> 32 fp16x2 (or bf16x2) words.
// b0: bit offset of the chunk's first code in the staged row.  BITS > 0: the
// fixed-position extraction above; BITS == 0: any width, a sequential bit walk.
template <int D, int BITS>
__device__ __forceinline__ void decode_chunk(const TParams& prm, const uint16_t* cb_s, const uint32_t* crow, int xr,
                                             int b0, __half2 s2, int h, uint32_t* out) {
  constexpr int CPC = kChunkK / D;   // codes per chunk
  constexpr int WPC = D / 2;         // output words per code
  const uint32_t sel = prm.npass > 1 ? static_cast<uint32_t>(h) << prm.kp_log2 : 0u;
  const uint32_t lim = prm.npass > 1 ? static_cast<uint32_t>(prm.kp) : static_cast<uint32_t>(prm.K);
  if constexpr (BITS > 0) {
    uint32_t c[CPC];
    extract_codes<BITS, CPC>(crow, xr, b0, c);
#pragma unroll
    for (int i = 0; i < CPC; ++i) lookup<D>(cb_s, c[i], sel, lim, out + WPC * i);
  } else {
    const int bits = prm.bits;
    const uint32_t mask = (1u << bits) - 1u;
    auto word = [&](int wi) { return crow[(((wi >> 2) ^ xr) << 2) | (wi & 3)]; };
    int wi = b0 >> 5;
    uint64_t buf = static_cast<uint64_t>(word(wi++)) >> (b0 & 31);
    int nb = 32 - (b0 & 31);
#pragma unroll 8
    for (int i = 0; i < CPC; ++i) {
      if (nb < bits) {
        buf |= static_cast<uint64_t>(word(wi++)) << nb;
        nb += 32;
      }
      const uint32_t c = static_cast<uint32_t>(buf) & mask;
      buf >>= bits;
      nb -= bits;
      lookup<D>(cb_s, c, sel, lim, out + WPC * i);
    }
  }
  scale_words(out, s2, s2, prm.b_bf16 != 0);
}

// Dimension split (d8 codebooks larger than shared memory): pass h keeps dims
// [4h, 4h + 4) of every entry resident (8 bytes per entry, a zero entry at
// index K), and a position covers 16 codes x 4 dims = 64 A columns.  Column
// 4i + d of position p holds W[row, 8 (16p + i) + 4h + d]; x was gathered in
// the same permuted order, so every weight is decoded once and enters one MMA.
// Codes 0-7 and 8-15 of a position may sit in different scale groups (G = 64).
// 16 codes of BITS whose stream starts at bit 0 of word DW of q (twelve words
// read from the 16-byte unit holding the first one): constant shifts only.
template <int BITS, int DW>
__device__ __forceinline__ void codes16_at_word(const uint32_t* q, uint32_t* c) {
  constexpr uint32_t MASK = (1u << BITS) - 1u;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    constexpr int dummy = 0;
    (void)dummy;
    const int bit = i * BITS, wi = DW + (bit >> 5), bs = bit & 31;
    const uint32_t v = (bs + BITS <= 32) ? (q[wi] >> bs) : __funnelshift_r(q[wi], q[wi + 1], bs);
    c[i] = v & MASK;
  }
}

template <int BITS>
__device__ __forceinline__ void decode_pos_dsplit(const TParams& prm, const uint16_t* cb_s, const uint32_t* crow,
                                                  int xr, int b0, __half2 s_lo, __half2 s_hi, uint32_t* out) {
  uint32_t c[16];
  if ((b0 & 31) == 0 && 16 * BITS <= 8 * 32) {
    // the position starts on a word (d8/14-bit: 224 bits per position): the
    // warp-uniform word offset inside the first 16-byte unit picks an
    // unrolled extraction, no select tree or funnel alignment
    const int w0 = b0 >> 5;
    const uint4* row4 = reinterpret_cast<const uint4*>(crow);
    uint32_t q[12];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint4 v = row4[((w0 >> 2) + i) ^ xr];
      q[4 * i] = v.x; q[4 * i + 1] = v.y; q[4 * i + 2] = v.z; q[4 * i + 3] = v.w;
    }
    switch (w0 & 3) {
      case 0: codes16_at_word<BITS, 0>(q, c); break;
      case 1: codes16_at_word<BITS, 1>(q, c); break;
      case 2: codes16_at_word<BITS, 2>(q, c); break;
      default: codes16_at_word<BITS, 3>(q, c); break;
    }
  } else {
    extract_codes<BITS, 16>(crow, xr, b0, c);
  }
  if (prm.K == (1 << BITS)) {
    // every code of the width is a codebook entry: no clamp
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint2 v = reinterpret_cast<const uint2*>(cb_s)[c[i]];
      out[2 * i] = v.x;
      out[2 * i + 1] = v.y;
    }
  } else {
    const uint32_t lim = static_cast<uint32_t>(prm.K);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint2 v = reinterpret_cast<const uint2*>(cb_s)[min(c[i], lim)];
      out[2 * i] = v.x;
      out[2 * i + 1] = v.y;
    }
  }
  scale_words(out, s_lo, s_hi, prm.b_bf16 != 0);
}

// Tiles run in groups: up to 8 consecutive tiles of this CTA whose
// accumulators (two per tile, n16 columns each, n16 = tokens rounded up to 16)
// fit the 256 accumulator columns together.  Every pass of a group runs over
// all its tiles before the next pass, so one codebook reload and one
// accumulator drain serve the whole group -- the small-token tiles of decode
// batches are short, and a reload per tile would cost as much as the tile.
// The second pass re-reads the group's code windows, so a group's packed
// codes stay within an L2 budget per CTA (max_group) and come from L2.
struct TileGroup {
  int count;
  int n16;
};
constexpr int kAccCols = kIssuers * kMaxN;  // TMEM columns [0, 256)
constexpr int kMaxGroup = 8;

// Work item it: tile it / ksplit (chunk-major over row tiles), split it % ksplit
// of the tile's npass * nwin windows (contiguous, window-aligned ranges).
__device__ __forceinline__ int item_chunk(const TParams& prm, int64_t it) {
  return static_cast<int>((it / prm.ksplit) / prm.row_tiles);
}
__device__ __forceinline__ int item_row_tile(const TParams& prm, int64_t it) {
  return static_cast<int>((it / prm.ksplit) % prm.row_tiles);
}
// The item's windows of codebook slice h (a pass runs slice pass_slice(...)):
// [lo, hi) of that slice's nwin windows, empty when lo >= hi.  The item's
// range is fixed in slice order, whatever order a group walks the slices in.
__device__ __forceinline__ void item_pass_windows(const TParams& prm, int64_t it, int h, int nwin, int& lo, int& hi) {
  const int S = prm.ksplit, sp = static_cast<int>(it % S), nwt = prm.npass * nwin;
  const int wlo = sp * nwt / S, whi = (sp + 1) * nwt / S;
  lo = max(wlo - h * nwin, 0);
  hi = min(whi - h * nwin, nwin);
}
__device__ __forceinline__ int tile_n16(const TParams& prm, int64_t it) {
  return (prm.chunks[item_chunk(prm, it)].z + 15) & ~15;
}
__device__ __forceinline__ TileGroup form_group(const TParams& prm, int64_t it0, int64_t nitems) {
  TileGroup grp{1, tile_n16(prm, it0)};
  while (grp.count < prm.max_group) {
    const int64_t it = it0 + static_cast<int64_t>(grp.count) * gridDim.x;
    if (it >= nitems) break;
    const int n16 = max(grp.n16, tile_n16(prm, it));
    if ((grp.count + 1) * 2 * n16 > kAccCols) break;
    grp.n16 = n16;
    ++grp.count;
  }
  return grp;
}

// A decode thread's row of tile `it`: r (output row), whether it is live, its
// row in codes / scales (crow) and in the staged windows (woff).  With a row
// table dead rows decode nothing and store +0, and a row whose compact index
// falls outside its tile's window counts as dead.
struct TileRow {
  int r;
  bool live;
  int64_t crow;
  int woff;
};
__device__ __forceinline__ TileRow tile_row(const TParams& prm, int64_t it, int lrow, int e) {
  const int rt = item_row_tile(prm, it);
  TileRow tr;
  tr.r = rt * kTileM + lrow;
  const int rr = min(tr.r, prm.OUT - 1);
  tr.crow = static_cast<int64_t>(e) * prm.OUT + rr;
  tr.woff = lrow;
  tr.live = true;
  if (prm.row_table) {
    const int tb = prm.tile_base[e * prm.row_tiles + rt];
    tr.crow = tr.r < prm.OUT ? static_cast<int64_t>(prm.row_table[static_cast<int64_t>(e) * prm.OUT + tr.r]) : -1;
    const int64_t o = tr.crow - tb;
    tr.live = tr.crow >= 0 && tr.crow < prm.nrows && tb >= 0 && o >= 0 && o < kTileM;
    tr.woff = tr.live ? static_cast<int>(o) : 0;
  }
  return tr;
}

// -------------------------------------------------------------- the kernel

template <int D, int BITS, bool DS>
__global__ void __launch_bounds__(kThreads, 1)
    vq_prefill_tc_kernel(const __grid_constant__ CUtensorMap xmap32, const __grid_constant__ CUtensorMap xmap64,
                         const __grid_constant__ CUtensorMap xmap128, const __grid_constant__ CUtensorMap cmap,
                         const __grid_constant__ CUtensorMap smap, const TParams prm) {
  extern __shared__ __align__(16) unsigned char smem_dyn[];
  // [B stages][2 code/scale windows][codebook slice][barriers][tmem addr][flag]; 1024-aligned (swizzle atom)
  // (pointer arithmetic on the shared array keeps the compiler's knowledge
  // that every access below is a shared-memory access)
  unsigned char* base = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
  unsigned char* b_base = base;
  unsigned char* w_base = base + prm.off_win;
  uint16_t* cb_s = reinterpret_cast<uint16_t*>(base + prm.off_cb);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + prm.off_bar);
  uint64_t* b_full = bars;                         // [kBStages] x slot landed
  uint64_t* b_empty = b_full + kBStages;           // [kBStages] MMAs done with the slot
  uint64_t* a_full = b_empty + kBStages;           // [2] all 16 decode warps stored their window's A stages
                                                   //     (window w -> a_full[w & 1]; one wait per window)
  uint64_t* st_free = a_full + 2;                  // [kAStages] MMAs of position g done: A stage g % 8 free
  uint64_t* w_full = st_free + kAStages;           // [kWStages] code/scale window landed
  uint64_t* w_empty = w_full + kWStages;           // [kWStages] all 16 decode warps read it
  uint64_t* cb_full = w_empty + kWStages;          // [1] codebook slice landed
  uint64_t* cb_empty = cb_full + 1;                // [1] all decode warps done with the slice
  uint64_t* acc_full = cb_empty + 1;               // [kIssuers] issuer i's accumulator complete
  uint64_t* acc_empty = acc_full + kIssuers;       // [1] epilogue read both accumulators
  uint64_t* mma_done = acc_empty + 1;              // [kIssuers] teardown: every issued MMA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBStages; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
    for (int i = 0; i < 2; ++i) mbar_init(&a_full[i], kDecodeWarps);
    for (int i = 0; i < kAStages; ++i) mbar_init(&st_free[i], 1);
    for (int i = 0; i < kWStages; ++i) { mbar_init(&w_full[i], 1); mbar_init(&w_empty[i], kDecodeWarps); }
    mbar_init(cb_full, 1);
    mbar_init(cb_empty, kDecodeWarps);
    for (int i = 0; i < kIssuers; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&mma_done[i], 1); }
    mbar_init(acc_empty, kDecodeWarps);
    *abort_flag = 0;
    // the zero entry after the resident slice (never written by the slice copies)
    constexpr int kEntryHalves = DS ? 4 : D;
    uint16_t* zero = cb_s + static_cast<size_t>(DS ? prm.K : (prm.npass > 1 ? prm.kp : prm.K)) * kEntryHalves;
    for (int i = 0; i < kEntryHalves; ++i) zero[i] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched as a programmatic dependent of the kernel before it (the x
  // gather): the set-up above overlaps that kernel's tail; nothing it wrote
  // (routing tables, gathered x) and nothing it may still read is touched
  // before this wait returns.  The codebook loader thread waits in its own
  // role, after it has started the first codebook slice (prm.cb_early).
  const bool cb_thread = warp == kWarpCbLoad && lane == 0;
  if (!cb_thread) asm volatile("griddepcontrol.wait;" ::: "memory");
  // the split-K reduction after this kernel may be scheduled beside it (it waits for this grid's end)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int nchunks = cb_thread ? 0 : prm.meta[0];
  const int64_t nitems = static_cast<int64_t>(nchunks) * prm.row_tiles * prm.ksplit;
  const int nwin = prm.n_pos / kSets;

  if (warp == kWarpTmaX) {
    // ---------------- TMA producer: x slots (slot_positions(n) consecutive K positions per B stage)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&xmap32)) : "memory");
      asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&xmap64)) : "memory");
      asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&xmap128)) : "memory");
      uint32_t gs = 0;  // slot sequence number
      bool ok = true;
      int jg = 0;
      for (int64_t it0 = blockIdx.x; it0 < nitems && ok; ++jg) {
        const TileGroup grp = form_group(prm, it0, nitems);
        for (int pass = 0; pass < prm.npass && ok; ++pass) {
          // the dimension split reads x's permuted half of the resident codebook dims
          const int cbase = DS ? pass_slice(prm.npass, jg, pass) * prm.n_pos : 0;
          for (int t = 0; t < grp.count && ok; ++t) {
            const int64_t it = it0 + static_cast<int64_t>(t) * gridDim.x;
            int lo, hi;
            item_pass_windows(prm, it, pass_slice(prm.npass, jg, pass), nwin, lo, hi);
            const int4 ch = prm.chunks[item_chunk(prm, it)];
            const int rows = slot_rows(ch.z);
            const int pp = slot_positions(rows);
            // one box per slot: 64 k x rows tokens x pp chunks, laid out [chunk][token][k]
            const CUtensorMap* map = rows == 32 ? &xmap32 : (rows == 64 ? &xmap64 : &xmap128);
            const uint32_t bytes = static_cast<uint32_t>(pp * rows * kChunkK * 2);
            for (int p0 = lo * kSets; p0 < hi * kSets; p0 += pp, ++gs) {
              const uint32_t bs = gs % kBStages;
              if (!mbar_wait(&b_empty[bs], ((gs / kBStages) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
              mbar_expect_tx(&b_full[bs], bytes);
              unsigned char* dst = b_base + bs * kBStageBytes;
              tma_load_3d(map, &b_full[bs], dst, 0, ch.y, cbase + p0);
            }
          }
        }
        it0 += static_cast<int64_t>(grp.count) * gridDim.x;
      }
      // no copy may still be writing shared memory when the CTA exits
      for (uint32_t k = 1; k <= kBStages && k <= gs; ++k) mbar_drain(&b_full[(gs - k) % kBStages], ((gs - k) / kBStages) & 1u);
    }
  } else if (warp == kWarpMma0 || warp == kWarpMma1) {
    // ---------------- MMA issuers.  A tile's K positions come in slots of pp
    // positions sharing one B stage (pp > 1 for tiles of <= 64 tokens).  Slot
    // gs of the CTA's slot sequence goes to issuer gs & 1, which accumulates
    // into its own D_i of the tile; the epilogue adds D_0 + D_1 when both took
    // part.  With an even number of B stages every stage then belongs to one
    // issuer, and a slot is one window (pp = 4) or a window is cut into 2 or 4
    // slots (pp = 2, 1): each issuer waits on b_full[bs] and on a_full[w & 1]
    // for consecutive phases only -- an issuer that skipped a phase could take
    // the previous phase's completion for the one it wants.  Tile t of a group
    // owns accumulator columns [2 t n16, 2 t n16 + 2 n16).
    if (lane == 0) {
      const int iss = warp == kWarpMma0 ? 0 : 1;
      // descriptor of B stage 0; later stages / positions start further on (the start-address field counts 16-byte units)
      const uint64_t bdesc0 = sw128_desc(smem_u32(b_base));
      uint32_t g = 0, gs = 0;
      uint32_t waited = 0xFFFFFFFFu;  // last window whose A stages this issuer has seen complete
      bool ok = true;
      int jg = 0;
      for (int64_t it0 = blockIdx.x; it0 < nitems && ok; ++jg) {
        const TileGroup grp = form_group(prm, it0, nitems);
        if (jg >= 1 && !mbar_wait(acc_empty, static_cast<uint32_t>((jg - 1) & 1), abort_flag)) break;
        tc_fence_after();
        uint32_t started = 0;  // tiles whose accumulator this issuer has written in this group
        for (int pass = 0; pass < prm.npass && ok; ++pass) {
          for (int t = 0; t < grp.count && ok; ++t) {
            const int64_t it = it0 + static_cast<int64_t>(t) * gridDim.x;
            int lo, hi;
            item_pass_windows(prm, it, pass_slice(prm.npass, jg, pass), nwin, lo, hi);
            if (lo >= hi) continue;
            const int4 ch = prm.chunks[item_chunk(prm, it)];
            const uint32_t idesc = make_idesc((ch.z + 15) & ~15, prm.b_bf16 != 0);
            const int rows = slot_rows(ch.z);
            const int pp = slot_positions(rows);
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>((2 * t + iss) * grp.n16);
            for (int p0 = lo * kSets; p0 < hi * kSets; p0 += pp, ++gs) {
              if ((gs & 1u) != static_cast<uint32_t>(iss)) continue;
              const uint32_t bs = gs % kBStages;
              if (!(ok = mbar_wait(&b_full[bs], (gs / kBStages) & 1u, abort_flag))) break;
              for (int q = 0; q < pp; ++q) {
                const uint32_t gp = g + static_cast<uint32_t>(p0 - lo * kSets + q);
                const uint32_t ast = gp % kAStages;
                const uint32_t win = gp >> 2;
                if (win != waited) {
                  if (!(ok = mbar_wait(&a_full[win & 1u], (win >> 1) & 1u, abort_flag))) break;
                  tc_fence_after();
                  waited = win;
                }
                const uint32_t a_tmem = tmem_base + kTmemA + ast * 32;
                const uint64_t bd = bdesc0 + static_cast<uint64_t>((bs * kBStageBytes + q * rows * kChunkK * 2) >> 4);
                tc_mma_ts(d_tmem, a_tmem, bd, idesc, (started >> t) & 1u);
                tc_mma_ts(d_tmem, a_tmem + 8, bd + 2, idesc, 1u);    // +32 bytes: next 16 k of the swizzle row
                tc_mma_ts(d_tmem, a_tmem + 16, bd + 4, idesc, 1u);
                tc_mma_ts(d_tmem, a_tmem + 24, bd + 6, idesc, 1u);
                started |= 1u << t;
                tc_commit(&st_free[ast]);
              }
              if (!ok) break;
              tc_commit(&b_empty[bs]);
            }
            g += static_cast<uint32_t>((hi - lo) * kSets);
          }
        }
        if (ok) tc_commit(&acc_full[iss]);
        it0 += static_cast<int64_t>(grp.count) * gridDim.x;
      }
      // every MMA this thread issued has completed before TMEM is freed
      tc_commit(&mma_done[iss]);
      mbar_drain(&mma_done[iss], 0);
    }
  } else if (warp == kWarpTmaCode) {
    // ---------------- TMA producer: windows of packed code rows (+ scales)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(&cmap)) : "memory");
      uint32_t ws = 0, wp = 0;
      int filled[kWStages] = {};
      uint32_t fill_phase[kWStages] = {};
      const uint32_t bytes = static_cast<uint32_t>(prm.code_stage_bytes + (prm.scale_tma ? kTileM * kScaleRowBytes : 0));
      bool ok = true;
      int jg = 0;
      for (int64_t it0 = blockIdx.x; it0 < nitems && ok; ++jg) {
        const TileGroup grp = form_group(prm, it0, nitems);
        for (int pass = 0; pass < prm.npass && ok; ++pass) {
          for (int t = 0; t < grp.count && ok; ++t) {
            const int64_t it = it0 + static_cast<int64_t>(t) * gridDim.x;
            int lo, hi;
            item_pass_windows(prm, it, pass_slice(prm.npass, jg, pass), nwin, lo, hi);
            const int rt = item_row_tile(prm, it);
            const int4 ch = prm.chunks[item_chunk(prm, it)];
            // the tile's rows in codes / scales: (e, rt*128 ...), or from its first live compact row
            const int yrow = prm.row_table ? max(prm.tile_base[ch.x * prm.row_tiles + rt], 0) : ch.x * prm.OUT + rt * kTileM;
            for (int w = lo; w < hi; ++w) {
              if (!mbar_wait(&w_empty[ws], wp ^ 1u, abort_flag)) { ok = false; break; }
              mbar_expect_tx(&w_full[ws], bytes);
              unsigned char* dst = w_base + ws * prm.win_stage_bytes;
              tma_load_2d(&cmap, &w_full[ws], dst, (w * prm.wpw) & ~3, yrow);
              if (prm.scale_tma) {
                const int g_first = ((w * kSets) << prm.kpos_log2) >> prm.log2g;
                tma_load_2d(&smap, &w_full[ws], dst + prm.code_stage_bytes, g_first & ~7, yrow);
              }
              filled[ws] = 1;
              fill_phase[ws] = wp;
              if (++ws == prm.wst) { ws = 0; wp ^= 1u; }
            }
          }
        }
        it0 += static_cast<int64_t>(grp.count) * gridDim.x;
      }
      for (int s = 0; s < prm.wst; ++s)
        if (filled[s]) mbar_drain(&w_full[s], fill_phase[s]);
    }
  } else if (warp == kWarpCbLoad) {
    // ---------------- codebook slice loader
    if (lane == 0) {
      // slice h: entries [h * kp, ...), or (dimension split) dims [4h, 4h + 4)
      // of all entries from the [2][K][4] copy of the codebook
      auto load_slice = [&](int h) {
        const int64_t first = DS ? 0 : static_cast<int64_t>(h) * prm.kp;
        const int64_t cnt = DS ? static_cast<int64_t>(prm.K)
                               : min(static_cast<int64_t>(prm.kp), static_cast<int64_t>(prm.K) - first);
        const uint32_t bytes = static_cast<uint32_t>(cnt * (DS ? 8 : D * 2));
        mbar_expect_tx(cb_full, bytes);
        const unsigned char* src = reinterpret_cast<const unsigned char*>(prm.codebook) +
                                   (DS ? static_cast<int64_t>(h) * prm.K * 8 : first * D * 2);
        for (uint32_t off = 0; off < bytes; off += 8192u)
          bulk_load(reinterpret_cast<unsigned char*>(cb_s) + off, src + off, min(8192u, bytes - off), cb_full);
      };
      int resident = -1;
      uint32_t loads = 0;
      if (prm.cb_early) {
        // the first group's first pass always reads slice 0, and the codebook
        // (its halves built by an earlier call) is not written by the kernel
        // this one depends on: load it before waiting for that kernel
        load_slice(0);
        resident = 0;
        loads = 1;
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      const int64_t nitems_cb = static_cast<int64_t>(prm.meta[0]) * prm.row_tiles * prm.ksplit;
      bool ok = true;
      int jg = 0;
      for (int64_t it0 = blockIdx.x; it0 < nitems_cb && ok; ++jg) {
        const TileGroup grp = form_group(prm, it0, nitems_cb);
        for (int pass = 0; pass < prm.npass; ++pass) {
          const int h = pass_slice(prm.npass, jg, pass);
          if (h == resident) continue;
          if (loads > 0 && !mbar_wait(cb_empty, (loads - 1) & 1u, abort_flag)) { ok = false; break; }
          load_slice(h);
          resident = h;
          ++loads;
        }
        it0 += static_cast<int64_t>(grp.count) * gridDim.x;
      }
      if (loads > 0) mbar_drain(cb_full, (loads - 1) & 1u);
    }
  } else if (warp >= kFirstDecodeWarp) {
    // ---------------- decode (+ epilogue): set s, TMEM lane quarter q = warp % 4, thread = row
    const int s = (warp - kFirstDecodeWarp) >> 2;
    const int q = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int lrow = q * 32 + lane;                 // row inside the tile
    uint32_t ws = 0, wp = 0;
    uint32_t g = 0;                                 // position sequence number
    uint32_t gsl = 0;                               // B slot sequence number (the issuers' gs)
    int cur = -1;
    uint32_t cb_loads = 0;
    bool ok = true;
    int jg = 0;
    for (int64_t it0 = blockIdx.x; it0 < nitems && ok; ++jg) {
      const TileGroup grp = form_group(prm, it0, nitems);
      // accumulators the issuers wrote, per tile: bit 2t = D_0, bit 2t + 1 = D_1
      uint32_t used = 0;
      for (int pass = 0; pass < prm.npass && ok; ++pass) {
        const int h = pass_slice(prm.npass, jg, pass);
        if (h != cur) {
          if (cur >= 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive(cb_empty);
          }
          if (!warp_wait(cb_full, cb_loads & 1u, abort_flag)) { ok = false; break; }
          ++cb_loads;
          cur = h;
        }
        for (int t = 0; t < grp.count && ok; ++t) {
          const int64_t it = it0 + static_cast<int64_t>(t) * gridDim.x;
          int lo, hi;
          item_pass_windows(prm, it, pass_slice(prm.npass, jg, pass), nwin, lo, hi);
          if (lo >= hi) continue;
          {
            const int nslots = (hi - lo) * kSets / slot_positions(slot_rows(prm.chunks[item_chunk(prm, it)].z));
            used |= (nslots >= 2 ? 3u : (1u << (gsl & 1u))) << (2 * t);
            gsl += static_cast<uint32_t>(nslots);
          }
          const TileRow tr = tile_row(prm, it, lrow, prm.chunks[item_chunk(prm, it)].x);
          const int xr = prm.wswz == 1 ? ((tr.woff >> 1) & 3) : (prm.wswz == 2 ? (tr.woff & 7) : 0);
          const uint16_t* srow = prm.scales + (tr.live ? tr.crow : 0) * prm.NGRP;
          for (int w = lo; w < hi; ++w) {
            if (!warp_wait(&w_full[ws], wp, abort_flag)) { ok = false; break; }
            const unsigned char* wst = w_base + ws * prm.win_stage_bytes;
            const int p = w * kSets + s;
            uint32_t out[32];
            if (p < prm.n_k && tr.live) {
              // scale of the group holding original k = kk (staged with the window, or from global)
              auto scale_at = [&](int kk) -> uint16_t {
                if (prm.scale_tma) {
                  const uint4 sv = reinterpret_cast<const uint4*>(wst + prm.code_stage_bytes)[tr.woff];
                  const int gi = (kk >> prm.log2g) - ((((w * kSets) << prm.kpos_log2) >> prm.log2g) & ~7);
                  const uint32_t sw = (gi & 4) ? ((gi & 2) ? sv.w : sv.z) : ((gi & 2) ? sv.y : sv.x);
                  return static_cast<uint16_t>((gi & 1) ? (sw >> 16) : (sw & 0xFFFFu));
                }
                return __ldg(srow + kk / prm.G);
              };
              const int wstart = w * prm.wpw;
              const uint32_t* crow_s = reinterpret_cast<const uint32_t*>(wst) + tr.woff * prm.W;
              if constexpr (DS) {
                __half slo, shi;
                if (prm.scale_tma && prm.log2g == 6) {
                  // G = 64: the window's 8 staged scales are groups 8w .. 8w+7, this
                  // position's pair (2s, 2s+1) is 32-bit word s of the row's 16 bytes
                  const uint32_t sw = reinterpret_cast<const uint32_t*>(wst + prm.code_stage_bytes)[tr.woff * 4 + s];
                  slo = __ushort_as_half(static_cast<uint16_t>(sw & 0xFFFFu));
                  shi = __ushort_as_half(static_cast<uint16_t>(sw >> 16));
                } else {
                  slo = __ushort_as_half(scale_at(p << 7));
                  shi = __ushort_as_half(scale_at((p << 7) + 64));
                }
                const int b0 = (wstart & 3) * 32 + s * 16 * BITS;
                decode_pos_dsplit<BITS>(prm, cb_s, crow_s, xr, b0, __halves2half2(slo, slo), __halves2half2(shi, shi),
                                        out);
              } else {
                const __half sh = __ushort_as_half(scale_at(p * kChunkK));
                const int b0 = (wstart & 3) * 32 + s * (kChunkK / D) * prm.bits;
                decode_chunk<D, BITS>(prm, cb_s, crow_s, xr, b0, __halves2half2(sh, sh), h, out);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) out[i] = 0u;  // K padding up to a whole window, or a dead row
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_empty[ws]);
            if (++ws == prm.wst) { ws = 0; wp ^= 1u; }
            // position p of this tile-pass has sequence number g + p - 4 lo; its
            // A stage was last read by the position 8 before it
            const uint32_t gp = g + static_cast<uint32_t>(p - lo * kSets);
            const uint32_t ast = gp % kAStages;
            if (!warp_wait(&st_free[ast], ((gp / kAStages) & 1u) ^ 1u, abort_flag)) { ok = false; break; }
            tc_fence_after();
            tc_st_x32(tmem_base + lane_off + kTmemA + ast * 32, out);
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[(gp >> 2) & 1u]);
          }
          g += static_cast<uint32_t>((hi - lo) * kSets);
        }
      }
      if (!ok) break;
      // epilogue: y = D_0 (+ D_1 when both issuers took part) for every tile of
      // the group.  A group of one tile deals its 16-column blocks to the 4
      // sets; a group of several gives tile t to set t % 4, so each set reads
      // the routing records of its own tiles only (those global reads are the
      // epilogue's latency)
      if (!warp_wait(&acc_full[0], static_cast<uint32_t>(jg & 1), abort_flag) ||
          !warp_wait(&acc_full[1], static_cast<uint32_t>(jg & 1), abort_flag))
        break;
      tc_fence_after();
      int blk = 0;
      const bool spread = grp.count == 1;
      for (int t = spread ? 0 : s; t < grp.count; t += spread ? 1 : kSets) {
        const int64_t it = it0 + static_cast<int64_t>(t) * gridDim.x;
        const int4 ch = prm.chunks[item_chunk(prm, it)];
        const TileRow tr = tile_row(prm, it, lrow, ch.x);
        const int ntok = ch.z;
        const int n = (ntok + 15) & ~15;
        const bool u0 = (used >> (2 * t)) & 1u, u1 = (used >> (2 * t + 1)) & 1u;
        // D_0 + D_1 in that order when both issuers wrote the tile
        auto tile_acc = [&](uint32_t a, uint32_t b) {
          return u0 && u1 ? __uint_as_float(a) + __uint_as_float(b) : __uint_as_float(u1 ? b : a);
        };
        float* part = prm.ksplit > 1 ? prm.partial + it * (static_cast<int64_t>(prm.pcols) * kTileM) : nullptr;
        const uint32_t d0 = static_cast<uint32_t>(2 * t * grp.n16), d1 = d0 + static_cast<uint32_t>(grp.n16);
        for (int c0 = 0; c0 < n; c0 += 16, ++blk) {
          if (spread && (blk & (kSets - 1)) != s) continue;
          uint32_t v0[16], v1[16];
          tc_ld_x16(tmem_base + lane_off + d0 + static_cast<uint32_t>(c0), v0);
          tc_ld_x16(tmem_base + lane_off + d1 + static_cast<uint32_t>(c0), v1);
          tc_wait_ld();
          if (part) {
            // split-K: this item's fp32 partial, column-major so a warp's 32 rows are one 128-byte line
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const float v = tile_acc(v0[jj], v1[jj]);
              if (c0 + jj < ntok) part[(c0 + jj) * kTileM + lrow] = v;
            }
          } else if (tr.r < prm.OUT) {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              if (c0 + jj < ntok) {
                const int pair = prm.sorted[ch.y + c0 + jj];
                float acc = tile_acc(v0[jj], v1[jj]);
                if (!tr.live) acc = 0.0f;  // dead row (row table): exact +0
                store_y(prm.y, static_cast<int64_t>(pair) * prm.OUT + tr.r, acc, prm.y_dtype, prm.round_f16_first != 0);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      it0 += static_cast<int64_t>(grp.count) * gridDim.x;
    }
  }

  // teardown: everyone done with TMEM before it is freed
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (*abort_flag && threadIdx.x == 0) atomicExch(prm.status + 1, static_cast<int>(VQB_TIMEOUT));
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem_base), "r"(kTmemCols) : "memory");
}

// SKIPZERO: the first live compact row of every (expert, 128-row tile), or -1
// when the tile has none (a warp per tile; compact rows run in (expert, row)
// order, so a tile's live rows are the next consecutive compact rows).
__global__ void tile_base_kernel(const int32_t* __restrict__ rt, int E, int OUT, int row_tiles, int64_t nrows,
                                 int* __restrict__ tb) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (t >= static_cast<int64_t>(E) * row_tiles) return;
  const int e = static_cast<int>(t / row_tiles), ti = static_cast<int>(t - static_cast<int64_t>(e) * row_tiles);
  int m = 0x7FFFFFFF;
  for (int i = lane; i < kTileM; i += 32) {
    const int r = ti * kTileM + i;
    if (r < OUT) {
      const int v = rt[static_cast<int64_t>(e) * OUT + r];
      if (v >= 0 && v < nrows) m = min(m, v);
    }
  }
  for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) tb[t] = m == 0x7FFFFFFF ? -1 : m;
}

// x rows gathered into expert-sorted order as 16-bit B rows: xs[s] = x[sorted[s] / krep].
// One thread per 16-byte vector (8 elements) of the output, so a few rows
// still spread over many threads; x is fp16 or bf16 with 16-byte aligned rows
// (IN % 64 == 0 and an aligned base).  dsplit: the dimension-split order --
// elements 8j .. 8j+3 go to columns 4j .. 4j+3 and elements 8j+4 .. 8j+7 to
// IN/2 + 4j .. (the x side of decode_pos_dsplit's column order).
__global__ void gather_sorted_kernel(const void* __restrict__ x, int x_dtype, const int* __restrict__ sorted,
                                     const int* __restrict__ n_sorted, int krep, int IN, int to_bf16, int dsplit,
                                     uint16_t* __restrict__ xs) {
  // launched as a programmatic dependent of the routing sort: wait for its
  // tables; the grouped GEMM that follows may start its set-up now (it waits
  // for this grid's end before reading xs)
  pdl_wait();
  pdl_trigger();
  const int vec = IN / 8;
  const bool convert = (x_dtype == VQB_BF16) != (to_bf16 != 0);
  const int64_t total = static_cast<int64_t>(*n_sorted) * vec;  // pairs left out are not in sorted
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < total;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(q / vec), i = static_cast<int>(q - static_cast<int64_t>(s) * vec);
    const int t = sorted[s] / krep;
    uint4 v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + static_cast<int64_t>(t) * IN) + i);
    if (convert) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (to_bf16) {
          const float2 f = __half22float2(*reinterpret_cast<__half2*>(&w[j]));
          __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
          w[j] = *reinterpret_cast<uint32_t*>(&b);
        } else {
          const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[j]));
          __half2 h = __floats2half2_rn(f.x, f.y);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
    }
    if (dsplit) {
      uint2* d2 = reinterpret_cast<uint2*>(xs + static_cast<int64_t>(s) * IN);
      d2[i] = make_uint2(v.x, v.y);
      d2[vec + i] = make_uint2(v.z, v.w);
    } else {
      reinterpret_cast<uint4*>(xs + static_cast<int64_t>(s) * IN)[i] = v;
    }
  }
}

// Split-K: y[pair, row] = the sum of a tile's ksplit fp32 partials in split
// order, with the output rounding (one thread per (tile, column, row), rows
// fastest; cmax = the partial slot's columns, the most tokens a chunk holds).
// With a row table a dead row stores +0 (the GEMM epilogue's rule: no compact
// row, or one outside its tile's staged window).
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, const int* __restrict__ meta,
                                     const int4* __restrict__ chunks, const int* __restrict__ sorted, int row_tiles,
                                     int S, int OUT, int cmax, void* y, int y_dtype, int round_f16_first,
                                     const int32_t* __restrict__ row_table, const int* __restrict__ tile_base,
                                     int64_t nrows) {
  // launched as a programmatic dependent of the GEMM: wait for its partials; the
  // kernel after this one (the next projection's GEMM) may begin its set-up
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t ntiles = static_cast<int64_t>(meta[0]) * row_tiles;
  const int64_t total = ntiles * cmax * kTileM;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int lr = static_cast<int>(i % kTileM);
    const int64_t rest = i / kTileM;
    const int c = static_cast<int>(rest % cmax);
    const int64_t ti = rest / cmax;
    const int4 ch = chunks[static_cast<int>(ti / row_tiles)];
    const int r = static_cast<int>(ti % row_tiles) * kTileM + lr;
    if (c >= ch.z || r >= OUT) continue;
    float v = 0.0f;
    for (int sp = 0; sp < S; ++sp) {
      const float pv = partial[((ti * S + sp) * cmax + c) * kTileM + lr];
      v = sp == 0 ? pv : v + pv;
    }
    if (row_table) {
      const int rt = static_cast<int>(ti % row_tiles);
      const int tb = tile_base[ch.x * row_tiles + rt];
      const int64_t crow = row_table[static_cast<int64_t>(ch.x) * OUT + r];
      const int64_t o = crow - tb;
      if (!(crow >= 0 && crow < nrows && tb >= 0 && o >= 0 && o < kTileM)) v = 0.0f;
    }
    store_y(y, static_cast<int64_t>(sorted[ch.y + c]) * OUT + r, v, y_dtype, round_f16_first != 0);
  }
}

// The d8 codebook [K][8] as two dimension halves [2][K][4] for the
// dimension-split passes (one thread per entry).
__global__ void split_codebook_kernel(const uint16_t* __restrict__ cb, int K, uint16_t* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= K) return;
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(cb) + c);
  reinterpret_cast<uint2*>(out)[c] = make_uint2(v.x, v.y);
  reinterpret_cast<uint2*>(out)[K + c] = make_uint2(v.z, v.w);
}

// xs [N, IN] 16-bit as a 3-d tensor (64 k, N tokens, IN / 64 chunks): a box
// {64, rows, pp} lands as pp consecutive [rows][64] K-major swizzled tiles
bool encode_x3d(EncodeTiledFn enc, CUtensorMap* map, bool bf16, const void* xs, int IN, int N, uint32_t rows,
                uint32_t pp) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kChunkK), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(IN / kChunkK)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(IN) * 2, static_cast<cuuint64_t>(kChunkK) * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kChunkK), rows, pp};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(xs), dims,
             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// the current device's attributes, refreshed by ensure_device_attrs() at the
// start of every host entry that reads them (per thread: no shared state)
thread_local int g_sms_tc = 0;
thread_local int g_smem_optin = 0;

template <int D>
void* pick_kernel(int bits) {
  // code widths of the shipped geometries get the fixed-position extraction
  if constexpr (D == 8) {
    if (bits == 12) return reinterpret_cast<void*>(vq_prefill_tc_kernel<8, 12, false>);
    if (bits == 14) return reinterpret_cast<void*>(vq_prefill_tc_kernel<8, 14, false>);
    if (bits == 16) return reinterpret_cast<void*>(vq_prefill_tc_kernel<8, 16, false>);
    return reinterpret_cast<void*>(vq_prefill_tc_kernel<8, 0, false>);
  } else if constexpr (D == 4) {
    if (bits == 12) return reinterpret_cast<void*>(vq_prefill_tc_kernel<4, 12, false>);
    if (bits == 13) return reinterpret_cast<void*>(vq_prefill_tc_kernel<4, 13, false>);
    return reinterpret_cast<void*>(vq_prefill_tc_kernel<4, 0, false>);
  } else {
    if (bits == 8) return reinterpret_cast<void*>(vq_prefill_tc_kernel<2, 8, false>);
    if (bits == 9) return reinterpret_cast<void*>(vq_prefill_tc_kernel<2, 9, false>);
    return reinterpret_cast<void*>(vq_prefill_tc_kernel<2, 0, false>);
  }
}

// Code widths with a dimension-split kernel (d8 codebooks over the shared-memory budget).
bool dsplit_bits(int bits) { return bits == 14; }


// Shared-memory layout for one mode: [B stages][wst code/scale windows]
// [codebook slice + zero entry][barriers]; returns the total, or 0 when the
// slice does not fit.  ds: dimension split (all K entries, 4 dims, 2 window
// stages); else the largest power-of-two slice of whole entries that fits.
size_t plan_smem(const LinearGeometry& geo, TParams& prm, bool ds) {
  prm.kpos_log2 = ds ? 7 : 6;
  prm.n_k = geo.IN >> prm.kpos_log2;
  prm.n_pos = (prm.n_k + kSets - 1) / kSets * kSets;
  prm.wst = ds ? 2 : kWStages;
  // code window: kSets positions of every row, read from an aligned-down
  // 16-byte boundary (up to o_max extra words); rows of 64 or 128 bytes take
  // the matching TMA swizzle, others an odd number of 16-byte units -- either
  // way conflict-free 16-byte reads across rows
  prm.wpw = ((kSets << prm.kpos_log2) / geo.D) * geo.bits / 32;
  const int o_max = prm.wpw % 4 == 0 ? 0 : (prm.wpw % 2 == 0 ? 2 : 3);
  const int need = o_max + prm.wpw;
  int W;
  if (need <= 16) { W = 16; prm.wswz = 1; }
  else if (need <= 32 && !(need % 4 == 0 && (need / 4) % 2 == 1)) { W = 32; prm.wswz = 2; }
  else {
    W = (need + 3) & ~3;
    if ((W / 4) % 2 == 0) W += 4;
    prm.wswz = 0;
  }
  prm.W = W;
  prm.code_stage_bytes = kTileM * W * 4;
  prm.win_stage_bytes = prm.code_stage_bytes + (prm.scale_tma ? kTileM * kScaleRowBytes : 0);
  const size_t tail = static_cast<size_t>(kNumBars) * 8 + 16;
  const size_t fixed = 1024 + static_cast<size_t>(kBStages) * kBStageBytes +
                       static_cast<size_t>(prm.wst) * prm.win_stage_bytes + tail + 16;
  if (static_cast<size_t>(g_smem_optin) <= fixed + 1024) return 0;
  const size_t avail = static_cast<size_t>(g_smem_optin) - fixed;
  size_t entry = static_cast<size_t>(geo.D) * 2;
  if (ds) {
    entry = 8;
    if (static_cast<size_t>(geo.K + 1) * entry > avail) return 0;
    prm.kp = geo.K;
    prm.kp_log2 = 0;
    prm.npass = 2;
  } else if (static_cast<size_t>(geo.K + 1) * entry <= avail) {
    prm.kp = geo.K;
    prm.kp_log2 = 0;
    prm.npass = 1;
  } else {
    int l = 0;
    while (((static_cast<size_t>(2) << l) + 1) * entry <= avail) ++l;
    prm.kp_log2 = l;
    prm.kp = 1 << l;
    prm.npass = (geo.K + prm.kp - 1) / prm.kp;
  }
  const size_t cb_bytes = (static_cast<size_t>(prm.kp + 1) * entry + 15) & ~size_t(15);  // + the zero entry
  prm.off_win = kBStages * kBStageBytes;
  prm.off_cb = prm.off_win + prm.wst * prm.win_stage_bytes;
  prm.off_bar = static_cast<int>(prm.off_cb + cb_bytes);
  const size_t smem = 1024 + static_cast<size_t>(prm.off_bar) + tail;
  return smem <= static_cast<size_t>(g_smem_optin) ? smem : 0;
}

// The dimension split applies to d8 codebooks too large for one pass, with a
// compiled code width and whole windows of 512 k.
bool dsplit_eligible(const LinearGeometry& geo, const TParams& one_pass_plan) {
  return geo.D == 8 && one_pass_plan.npass > 1 && dsplit_bits(geo.bits) && geo.IN % (kSets * 128) == 0 &&
         geo.K % 2 == 0;
}

vqb_status ensure_device_attrs() {
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  g_sms_tc = di.sms;
  g_smem_optin = di.smem_optin;
  return VQB_OK;
}

}  // namespace

bool tc_prefill_dsplit(const LinearGeometry& geo) {
  if (!tc_prefill_supported(geo) || ensure_device_attrs() != VQB_OK) return false;
  TParams prm{};
  prm.IN = geo.IN;
  prm.K = geo.K;
  prm.NGRP = geo.G > 0 ? geo.IN / geo.G : 0;
  prm.scale_tma = 1;
  plan_smem(geo, prm, false);
  return dsplit_eligible(geo, prm) && plan_smem(geo, prm, true) != 0;
}

bool tc_prefill_supported(const LinearGeometry& geo) {
  if (geo.IN % kChunkK != 0) return false;
  if (geo.G % kChunkK != 0) return false;      // one scale per row per 64-k chunk
  if (geo.bits > 16) return false;
  if ((reinterpret_cast<uintptr_t>(geo.codes) & 15) != 0 || geo.row_words % 4 != 0) return false;
  if ((static_cast<int64_t>(geo.K) * geo.D * 2) % 16 != 0) return false;  // codebook bulk copies
  return true;
}

// Upper bound on the tiles of a call: chunks of <= 128 tokens per expert
// (at most the distinct experts plus N / 128 of them) times the row tiles.
static int64_t tiles_bound(int64_t N, int E, int OUT) {
  const int64_t chunks = E == 1 ? (N + kMaxN - 1) / kMaxN : std::min<int64_t>(N, E) + N / kMaxN;
  return chunks * ((OUT + kTileM - 1) / kTileM);
}
// Columns of a split-K partial slot: the most tokens a chunk can hold.
static int partial_cols(int64_t N) { return static_cast<int>(std::min<int64_t>(kMaxN, (N + 15) & ~int64_t(15))); }

// Split-K for calls whose tiles cannot fill the GPU (a dense layer with few
// row tiles, a decode batch over a few experts): each tile's IN / 256 windows
// are cut into ksplit contiguous ranges, one work item each.  ksplit
// minimises (items per SM, rounded up) x (windows per item + 2, the per-item
// fixed cost), over 1..8 ranges of at least 2 windows, for the tile bound.
int tc_prefill_ksplit(int64_t N, int E, int OUT, int IN) {
  if (N <= 0 || IN <= 0 || ensure_device_attrs() != VQB_OK) return 1;
  const int64_t tiles = tiles_bound(N, E, OUT);
  if (tiles > 2 * static_cast<int64_t>(g_sms_tc)) return 1;
  const int64_t nwt = IN / 256;
  int best = 1;
  int64_t best_cost = -1;
  for (int S = 1; S <= 8 && nwt / S >= 2; ++S) {
    const int64_t cost = ((tiles * S + g_sms_tc - 1) / g_sms_tc) * ((nwt + S - 1) / S + 2);
    if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = S; }
  }
  return best;
}

// Workspace of one grouped-GEMM call after the routing tables: x gathered in
// expert order [N, IN] 16-bit, the [2][K][4] dimension halves of a d8
// codebook, and the split-K partial tiles.
static size_t xs_bytes(int64_t N, int IN) { return (static_cast<size_t>(N) * IN * 2 + 1023) & ~size_t(1023); }
static size_t split_cb_bytes(int K, int D) {
  return D == 8 && K > 0 ? (static_cast<size_t>(K) * 16 + 1023) & ~size_t(1023) : 0;
}
static size_t partial_bytes(int64_t N, int E, int OUT, int IN) {
  const int S = tc_prefill_ksplit(N, E, OUT, IN);
  if (S <= 1) return 0;
  return static_cast<size_t>(tiles_bound(N, E, OUT)) * S * partial_cols(N) * kTileM * sizeof(float);
}

size_t tc_prefill_x_bytes(int64_t N, int IN, int K, int D, int E, int OUT) {
  if (IN <= 0) return 0;
  return xs_bytes(N, IN) + split_cb_bytes(K, D) + partial_bytes(N, E, OUT, IN);
}

vqb_status launch_prefill_tc(const LinearGeometry& geo, const void* x, int x_dtype, int krep, const RouteWorkspace& rw,
                             int N, uint16_t* xs, void* y, int y_dtype, bool round_f16_first, bool bf16_operands,
                             bool gather_x, int* status, cudaStream_t stream) {
  if (N <= 0) return VQB_OK;
  if (ensure_device_attrs() != VQB_OK) return VQB_CUDA_ERROR;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return VQB_CUDA_ERROR;

  TParams prm{};
  prm.codes = static_cast<const uint32_t*>(geo.codes);
  prm.codebook = static_cast<const uint16_t*>(geo.codebook);
  prm.scales = static_cast<const uint16_t*>(geo.scales);
  prm.sorted = rw.sorted;
  prm.chunks = rw.chunks;
  prm.meta = rw.meta;
  prm.status = status;
  prm.y = y;
  prm.OUT = geo.OUT;
  prm.IN = geo.IN;
  prm.G = geo.G;
  prm.NGRP = geo.IN / geo.G;
  prm.bits = geo.bits;
  prm.K = geo.K;
  prm.row_tiles = (geo.OUT + kTileM - 1) / kTileM;
  prm.y_dtype = y_dtype;
  prm.round_f16_first = round_f16_first ? 1 : 0;
  prm.b_bf16 = bf16_operands ? 1 : 0;
  prm.row_table = geo.row_table;
  prm.tile_base = rw.tile_base;
  prm.nrows = geo.nrows;
  const bool g_pow2 = (geo.G & (geo.G - 1)) == 0;
  prm.scale_tma = (prm.NGRP % 8 == 0 && g_pow2 && (reinterpret_cast<uintptr_t>(geo.scales) & 15) == 0) ? 1 : 0;
  int log2g = 0;
  while ((1 << (log2g + 1)) <= geo.G) ++log2g;
  prm.log2g = log2g;
  const size_t tail = static_cast<size_t>(kNumBars) * 8 + 16;
  size_t smem = plan_smem(geo, prm, false);
  bool ds = false;
  if (dsplit_eligible(geo, prm)) {
    const size_t s2 = plan_smem(geo, prm, true);
    if (s2 > 0) {
      smem = s2;
      ds = true;
    } else {
      smem = plan_smem(geo, prm, false);
    }
  }
  if (smem == 0) return VQB_UNSUPPORTED_GEOMETRY;
  uint16_t* cb_split = ds ? reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(xs) + xs_bytes(N, geo.IN)) : nullptr;
  prm.ksplit = tc_prefill_ksplit(N, geo.E, geo.OUT, geo.IN);
  prm.pcols = partial_cols(N);
  {
    // the code bytes of a group read twice stay in L2: 256 KB per CTA (37 MB over 148 SMs)
    constexpr int64_t kGroupCodeBudget = 256 * 1024;
    const int64_t tile_bytes = static_cast<int64_t>(kTileM) * geo.row_words * 4;
    const int64_t g = prm.npass > 1 ? kGroupCodeBudget / std::max<int64_t>(tile_bytes, 1) : kMaxGroup;
    prm.max_group = static_cast<int>(std::min<int64_t>(kMaxGroup, std::max<int64_t>(1, g)));
  }
  prm.partial = prm.ksplit > 1 ? reinterpret_cast<float*>(reinterpret_cast<char*>(xs) + xs_bytes(N, geo.IN) +
                                                          split_cb_bytes(geo.K, geo.D))
                               : nullptr;

  // 1. gather x into expert-sorted 16-bit rows (unless the caller's previous call did)
  if (gather_x) {
    if (x_dtype != VQB_F16 && x_dtype != VQB_BF16) return VQB_UNSUPPORTED_GEOMETRY;
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return VQB_BAD_ALIGNMENT;
    int64_t blocks = (static_cast<int64_t>(N) * (geo.IN / 8) + 255) / 256;
    if (blocks > 16 * g_sms_tc) blocks = 16 * g_sms_tc;
    if (launch_pdl(gather_sorted_kernel, static_cast<unsigned>(blocks), 256, 0, stream, x, x_dtype,
                   static_cast<const int*>(rw.sorted), static_cast<const int*>(rw.offsets + geo.E), krep, geo.IN,
                   bf16_operands ? 1 : 0, ds ? 1 : 0, xs) != cudaSuccess)
      return VQB_CUDA_ERROR;
    note_launch();
  }
  // 1a. dimension halves of the codebook (the caller's, when it built them once)
  // The GEMM may start loading the caller's codebook, or the halves it built
  // once, before its programmatic-dependency wait when the kernel right before
  // it is the x gather: that kernel waited for everything the caller launched
  // earlier, and no kernel of this call writes them.  Halves derived here come
  // from the kernel right before the GEMM, and after a call that reuses the
  // gathered x the kernel before it may be the caller's own.
  prm.cb_early = gather_x && (!ds || geo.codebook_halves) ? 1 : 0;
  if (ds && geo.codebook_halves) {
    prm.codebook = static_cast<const uint16_t*>(geo.codebook_halves);
  } else if (ds) {
    split_codebook_kernel<<<static_cast<unsigned>((geo.K + 255) / 256), 256, 0, stream>>>(prm.codebook, geo.K,
                                                                                          cb_split);
    if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
    note_launch();
    prm.codebook = cb_split;
  }
  // 1b. SKIPZERO tile bases
  if (geo.row_table) {
    const int64_t warps = static_cast<int64_t>(geo.E) * prm.row_tiles;
    tile_base_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(
        geo.row_table, geo.E, geo.OUT, prm.row_tiles, geo.nrows, rw.tile_base);
    if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
    note_launch();
  }
  // 2. TMA maps: xs [N, IN] 16-bit seen as [chunk][token][64 k] (boxes of
  //    32 x 4, 64 x 2 and 128 x 1 tokens x chunks, 128-byte swizzle); codes
  //    [E*OUT, row_words] u32 (box W x 128); scales [E*OUT, NGRP] fp16 (box 8 x 128)
  CUtensorMap xmaps[3], cmap, smap;
  for (int i = 0; i < 3; ++i) {
    const uint32_t rows = 32u << i;
    if (!encode_x3d(enc, &xmaps[i], bf16_operands, xs, geo.IN, N, rows, static_cast<uint32_t>(slot_positions(rows))))
      return VQB_CUDA_ERROR;
  }
  const uint64_t rows = static_cast<uint64_t>(geo.nrows > 0 ? geo.nrows : 1);
  const CUtensorMapSwizzle cswz = prm.wswz == 1 ? CU_TENSOR_MAP_SWIZZLE_64B
                                  : (prm.wswz == 2 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!encode_2d(enc, &cmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, geo.codes, static_cast<uint64_t>(geo.row_words), rows,
                 static_cast<uint32_t>(prm.W), kTileM, cswz))
    return VQB_CUDA_ERROR;
  if (prm.scale_tma) {
    if (!encode_2d(enc, &smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, geo.scales, static_cast<uint64_t>(prm.NGRP), rows, 8,
                   kTileM, CU_TENSOR_MAP_SWIZZLE_NONE))
      return VQB_CUDA_ERROR;
  } else {
    smap = cmap;  // unused
  }

  void* kern = ds ? reinterpret_cast<void*>(vq_prefill_tc_kernel<8, 14, true>)
                  : (geo.D == 8 ? pick_kernel<8>(geo.bits) : (geo.D == 4 ? pick_kernel<4>(geo.bits) : pick_kernel<2>(geo.bits)));
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return VQB_CUDA_ERROR;
  void* args[] = {&xmaps[0], &xmaps[1], &xmaps[2], &cmap, &smap, &prm};
  timer_before(stream);
  // programmatic stream serialization: the GEMM's CTAs may launch while the
  // kernel before it finishes; the kernel waits (griddepcontrol.wait) before
  // touching anything that kernel wrote
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g_sms_tc);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t ce = cudaLaunchKernelExC(&cfg, kern, args);
  timer_after(stream);
  if (ce != cudaSuccess || cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
  note_launch();
  if (prm.ksplit > 1) {
    const int cmax = prm.pcols;
    const int64_t tiles = tiles_bound(N, geo.E, geo.OUT);
    int64_t blocks = (tiles * cmax * kTileM + 255) / 256;
    if (blocks > 8 * g_sms_tc) blocks = 8 * g_sms_tc;
    cudaLaunchConfig_t rcfg = {};
    rcfg.gridDim = dim3(static_cast<unsigned>(blocks));
    rcfg.blockDim = dim3(256);
    rcfg.stream = stream;
    rcfg.attrs = attr;
    rcfg.numAttrs = 1;
    const int rff = round_f16_first ? 1 : 0;
    if (cudaLaunchKernelEx(&rcfg, splitk_reduce_kernel, static_cast<const float*>(prm.partial),
                           static_cast<const int*>(rw.meta), static_cast<const int4*>(rw.chunks),
                           static_cast<const int*>(rw.sorted), prm.row_tiles, prm.ksplit, geo.OUT, cmax, y, y_dtype,
                           rff, geo.row_table, static_cast<const int*>(rw.tile_base), geo.nrows) != cudaSuccess ||
        cudaGetLastError() != cudaSuccess)
      return VQB_CUDA_ERROR;
    note_launch();
  }
  return VQB_OK;
}

}  // namespace vqb

extern "C" vqb_status vqb_codebook_halves(const void* codebook, int32_t num_codes, void* out, vqb_stream_t stream) {
  if (num_codes < 1) return VQB_BAD_SHAPE;
  if (!codebook || !out) return VQB_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(codebook) & 15) != 0 || (reinterpret_cast<uintptr_t>(out) & 15) != 0)
    return VQB_BAD_ALIGNMENT;
  vqb::split_codebook_kernel<<<static_cast<unsigned>((num_codes + 255) / 256), 256, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(static_cast<const uint16_t*>(codebook),
                                                                         num_codes, static_cast<uint16_t*>(out));
  if (cudaGetLastError() != cudaSuccess) return VQB_CUDA_ERROR;
  vqb::note_launch();
  return VQB_OK;
}
