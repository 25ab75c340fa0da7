// Expert-grouped VQ decode kernel on the tensor cores (sm_100a, mma.sync).
//
// The small-N VQ matmul y[p, r] = sum_k W_e[r, k] x_p[k] is bound by codebook
// lookups (one random D*2-byte gather per code), and a CUDA-core dot product
// costs ~40 instructions per code, which makes such a kernel issue-bound
// before it is lookup-bound.  Here each thread gathers its codebook entries
// straight into mma.sync A-fragment registers -- a d8 entry is 16 bytes, i.e.
// the four fp16x2 registers of two m16n8k16 A fragments for one row -- and the
// tensor core does the dot products for up to 8 tokens per MMA:
//
//   * k permutation.  Inside one scale group, thread t (lane & 3) of a quad
//     owns the 16 consecutive k values [16t, 16t+16); MMA m of the group takes
//     k = 16t + 4m .. +3 of that range (A: rows g, g+8; B: tokens g).  Any
//     permutation of k is exact as long as A and B use the same one, and an
//     MMA never mixes two scale groups (G must be a multiple of 16).
//   * codes.  Each warp stages its 16 rows' code stream through shared
//     memory one window (512 k values) at a time with coalesced 16-byte loads,
//     prefetched one window ahead; rows are padded so the per-thread 32-bit
//     reads are bank-conflict free.  The row's scales for the window are staged
//     with them.
//   * codebook.  Staged once per persistent CTA: all of it, or its first NS
//     entries when it is larger than shared memory (d8/K16384 = 256 KB), the
//     rest read through L1.
//   * x.  The chunk's tokens are staged once per chunk as 16-bit rows padded by
//     16 bytes, so the 32-byte B-fragment reads of a quarter warp hit distinct
//     bank groups.
//
// Numerics.  WR == 0 (VQSwitchLinear and the fused dense kernels): A = the
// fp16 codebook entry, B = x narrowed to fp16, fp32 accumulation of each scale
// group's partial, then acc = fma(s, partial, acc) -- the reference's group
// structure (vq_switch.py:1344-1352, gemmseg2 ACCS :4171-4203) with the
// in-group sum order of the tensor core.  WR == 1/2 (dense _decode_matmul,
// vq_dense.py:267-312): A = fp16(cb * s) (one RNE rounding, the fp16 multiply
// of vq_dense.py:136), re-rounded to bf16 for bf16 x (WR == 1), B = x in its
// own dtype, fp32 accumulation over all k.
#include <algorithm>
#include <cmath>

#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kWinK = 512;  // k values per staged code window

struct MParams {
  const uint32_t* codes;
  const uint16_t* codebook;
  const uint16_t* scales;
  const uint16_t* x16;      // [T, IN] 16-bit x (fp16 or bf16 per WR), x_mode 0
  const void* xraw;         // the caller's x [T, IN] (16-byte aligned rows), x_mode 1 / 2
  int x_dtype;              // its vqb_dtype
  int x_mode;               // 0: x16; 1: xraw is already the 16-bit B type; 2: convert xraw while staging
  const int* sorted;
  const int4* chunks;
  const int* meta;
  void* y;
  int64_t expert_words;
  const int32_t* row_table;  // SKIPZERO [E, OUT] -> compact row (-1 dead), nullptr = plain layout
  int64_t nrows;             // rows of codes / scales
  int row_words;
  int OUT, IN, G, NGRP, NSUB, bits, krep, K;
  int ks, mt, tiles, ns;
  int win_k;                // k values per window (kWinK, or 1024 when 512 does not give 16-byte rows)
  int win_words;            // code words of one row per window
  int cs_stride;            // words per staged code row (padded)
  int sc_stride;            // halves per staged scale row
  int x_stride;             // halves per staged x row (padded)
  int pm;                   // token slots staged per chunk (<= 16)
  int y_dtype;
  int round_f16_first;
  int cb_half;              // SPLIT: codebook entries held by each CTA of the pair
  int nbuf;                 // code-window buffers per warp: 2 = the next window's rows copied asynchronously
};

// asynchronous 16-byte global -> shared copy (L2 only), and its group fences
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
               :: "r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

__device__ __forceinline__ void mma_f16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16x2 (fp16(cb*s) pair) -> bf16x2 with one more RNE rounding
__device__ __forceinline__ uint32_t h2_to_bf2(uint32_t h) {
  const float2 f = h2x2f(h);
  __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<uint32_t*>(&b);
}

// The 16/D consecutive codes starting at bit `bit0` of a staged window row
// (LSB-first stream, vq_pack v1): a short bit walk over 32-bit shared-memory
// words that reads only the words it needs.
template <int D>
__device__ __forceinline__ void fetch_codes(const uint32_t* row_words, int bit0, uint32_t mask, int bits,
                                            uint32_t* c) {
  constexpr int CPT = 16 / D;
  if (CPT * bits <= 32) {
    // all CPT codes inside one 32-bit funnel window (d8: 2 codes of <= 16 bits)
    const int wi = bit0 >> 5;
    const uint32_t v = __funnelshift_r(row_words[wi], row_words[wi + 1], bit0 & 31);
#pragma unroll
    for (int i = 0; i < CPT; ++i) c[i] = (v >> (i * bits)) & mask;
    return;
  }
  if (CPT * bits <= 64) {
    // inside one 64-bit window of three words (d2/8-bit, d4/12-bit); the
    // staged rows carry spare words for the read past the last code
    const int wi = bit0 >> 5, sh = bit0 & 31;
    const uint32_t lo = __funnelshift_r(row_words[wi], row_words[wi + 1], sh);
    const uint32_t hi = __funnelshift_r(row_words[wi + 1], row_words[wi + 2], sh);
    const uint64_t v = (static_cast<uint64_t>(hi) << 32) | lo;
#pragma unroll
    for (int i = 0; i < CPT; ++i) c[i] = static_cast<uint32_t>(v >> (i * bits)) & mask;
    return;
  }
  int wi = bit0 >> 5;
  const int sh = bit0 & 31;
  uint64_t buf = row_words[wi++] >> sh;
  int nb = 32 - sh;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    if (nb < bits) {
      buf |= static_cast<uint64_t>(row_words[wi++]) << nb;
      nb += 32;
    }
    c[i] = static_cast<uint32_t>(buf) & mask;
    buf >>= bits;
    nb -= bits;
  }
}

// SPLIT: this CTA holds entries [base, base + half) of the codebook; a code
// outside it contributes zeros (its partner CTA adds the other half).
template <int D>
__device__ __forceinline__ void lookup_split(const uint16_t* cb_s, uint32_t base, uint32_t half, const uint32_t* c,
                                             uint32_t* w) {
  constexpr int CPT = 16 / D;
  constexpr int WPC = D / 2;  // fp16x2 words per entry
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const uint32_t rel = c[i] - base;
    if constexpr (D == 8) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (rel < half) v = reinterpret_cast<const uint4*>(cb_s)[rel];
      w[WPC * i] = v.x; w[WPC * i + 1] = v.y; w[WPC * i + 2] = v.z; w[WPC * i + 3] = v.w;
    } else if constexpr (D == 4) {
      uint2 v = make_uint2(0, 0);
      if (rel < half) v = reinterpret_cast<const uint2*>(cb_s)[rel];
      w[WPC * i] = v.x; w[WPC * i + 1] = v.y;
    } else {
      uint32_t v = 0;
      if (rel < half) v = reinterpret_cast<const uint32_t*>(cb_s)[rel];
      w[i] = v;
    }
  }
}

// Codebook lookups.  CB == kCbFull: shared memory holds all K entries and a
// zero entry at index K, so min(c, K) is one unconditional shared-memory read
// (a code >= K, which no valid stream holds, reads zeros).  CB == kCbPrefix:
// the first ns entries are in shared memory, the rest are read through L1 at
// min(c, K - 1), so no code reads outside the codebook.
constexpr int kCbPrefix = 0, kCbFull = 1, kCbSplit = 2;

template <int D, int CB>
__device__ __forceinline__ void lookup(const uint16_t* cb_s, const uint16_t* __restrict__ cb_g, int ns, int K,
                                       const uint32_t* c, uint32_t* w) {
  constexpr int CPT = 16 / D;
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    if constexpr (D == 8) {
      uint4 v;
      if constexpr (CB == kCbFull) {
        v = reinterpret_cast<const uint4*>(cb_s)[min(c[i], static_cast<uint32_t>(K))];
      } else {
        v = c[i] < static_cast<uint32_t>(ns)
                ? reinterpret_cast<const uint4*>(cb_s)[c[i]]
                : __ldg(reinterpret_cast<const uint4*>(cb_g) + min(c[i], static_cast<uint32_t>(K - 1)));
      }
      w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    } else if constexpr (D == 4) {
      uint2 v;
      if constexpr (CB == kCbFull) {
        v = reinterpret_cast<const uint2*>(cb_s)[min(c[i], static_cast<uint32_t>(K))];
      } else {
        v = c[i] < static_cast<uint32_t>(ns)
                ? reinterpret_cast<const uint2*>(cb_s)[c[i]]
                : __ldg(reinterpret_cast<const uint2*>(cb_g) + min(c[i], static_cast<uint32_t>(K - 1)));
      }
      w[2 * i] = v.x; w[2 * i + 1] = v.y;
    } else {
      uint32_t v;
      if constexpr (CB == kCbFull) {
        v = reinterpret_cast<const uint32_t*>(cb_s)[min(c[i], static_cast<uint32_t>(K))];
      } else {
        v = c[i] < static_cast<uint32_t>(ns)
                ? reinterpret_cast<const uint32_t*>(cb_s)[c[i]]
                : __ldg(reinterpret_cast<const uint32_t*>(cb_g) + min(c[i], static_cast<uint32_t>(K - 1)));
      }
      w[i] = v;
    }
  }
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared-memory address of the same variable in the partner CTA of the pair
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(p)), remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" :: "r"(addr), "f"(v) : "memory");
}

// Eight consecutive x elements from element i (16-byte aligned) as the B
// operand's 16-bit type: fp16 by RNE (the narrowing x_to_16bit_kernel
// applies), or bf16.
__device__ __forceinline__ uint4 x8_to_16bit(const void* x, int dtype, int64_t i, bool to_bf16) {
  float f[8];
  if (dtype == VQB_F32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + i));
    const float4 b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + i) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + i));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 t;
      if (dtype == VQB_BF16) t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
      else t = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (to_bf16) {
      __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
      o[j] = *reinterpret_cast<uint32_t*>(&b);
    } else {
      __half2 h = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
      o[j] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Place of (expert e, output row) in codes / scales: the plain [E, OUT, ...]
// layout, or its SKIPZERO compact row; -1 = dead (reads nothing, writes +0).
__device__ __forceinline__ int64_t code_row(const MParams& prm, int e, int row) {
  const int64_t er = static_cast<int64_t>(e) * prm.OUT + row;
  if (!prm.row_table) return er;
  const int64_t c = prm.row_table[er];
  return c < prm.nrows ? c : -1;
}

template <int D, int WR, int NT, int CB>
__global__ void __launch_bounds__(kThreads, 1) vq_decode_mma_kernel(const MParams prm) {
  constexpr bool SPLIT = CB == kCbSplit;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // layout: [cb prefix][x rows][per-warp code+scale windows][slice partials]
  uint16_t* cb_s = reinterpret_cast<uint16_t*>(smem_raw);
  // the whole codebook is followed by its zero entry at index K (the host sizes (ns + 1) entries)
  size_t off = (static_cast<size_t>(prm.ns + (CB == kCbFull ? 1 : 0)) * D * 2 + 15) & ~size_t(15);
  uint16_t* x_s = reinterpret_cast<uint16_t*>(smem_raw + off);
  off += (static_cast<size_t>(prm.pm) * prm.x_stride * 2 + 15) & ~size_t(15);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // per warp: nbuf code-window buffers, then the window's scales
  const size_t cwin_words = static_cast<size_t>(16) * prm.cs_stride;
  const size_t win_bytes = (prm.nbuf * cwin_words * 4 + 16 * prm.sc_stride * 2 + 15) & ~size_t(15);
  uint32_t* c_base = reinterpret_cast<uint32_t*>(smem_raw + off + warp * win_bytes);
  uint16_t* s_s = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(c_base) + prm.nbuf * cwin_words * 4);
  off += kWarps * win_bytes;
  float* red = reinterpret_cast<float*>(smem_raw + off);

  const uint32_t crank = SPLIT ? cluster_rank() : 0u;
  const uint32_t cb_base = SPLIT ? crank * static_cast<uint32_t>(prm.cb_half) : 0u;
  // codebook prefix (or this CTA's half) -> shared memory, eight 16-byte loads
  // in flight per thread
  {
    const uint4* src = reinterpret_cast<const uint4*>(prm.codebook + static_cast<size_t>(cb_base) * D);
    uint4* dst = reinterpret_cast<uint4*>(cb_s);
    const int n16 = static_cast<int>((static_cast<size_t>(prm.ns) * D * 2) / 16);
    int i = threadIdx.x;
    for (; i + 7 * kThreads < n16; i += 8 * kThreads) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(src + i + u * kThreads);
#pragma unroll
      for (int u = 0; u < 8; ++u) dst[i + u * kThreads] = v[u];
    }
    for (; i < n16; i += kThreads) dst[i] = __ldg(src + i);
    if (CB == kCbFull && threadIdx.x == 0) {
      for (int j = 0; j < D; ++j) cb_s[static_cast<size_t>(prm.K) * D + j] = 0;  // the zero entry at index K
    }
  }

  // Launched as a programmatic dependent of the routing sort (or of the x
  // conversion after it): the codebook load above overlaps that kernel's tail
  // -- the routing sort waited for every kernel launched before this call, and
  // no kernel of this call writes the codebook -- and nothing that kernel
  // writes or may still read is touched before this wait returns.
  pdl_wait();
  pdl_trigger();

  // the partner CTA must be running before its shared memory is written
  if constexpr (SPLIT) cluster_sync_all();

  const int g = lane >> 2, t = lane & 3;
  const int ks = prm.ks, mt = prm.mt;
  const int slice = warp % ks, msub = warp / ks;
  const int rows_per_item = 16 * mt;
  const uint32_t mask = (1u << prm.bits) - 1u;
  const int n_win = prm.IN / prm.win_k;  // windows per row (IN is a multiple of win_k, checked on the host)
  const int wb = (n_win * slice) / ks, we = (n_win * (slice + 1)) / ks;
  const int gk = prm.G;                  // k per scale group
  const int chunks_per_row = prm.win_words / 4;

  // Window loader: lane -> (row slot, 16-byte chunk) with a power-of-two
  // split of the warp, so no division: cpl = 8 or 16 chunk lanes per row.
  const int cpl = chunks_per_row <= 8 ? 8 : 16;
  const int rows_per_pass = 32 / cpl;
  const int l_chunk = lane & (cpl - 1);
  const int l_row = lane / cpl;
  const bool l_chunk_ok = l_chunk < chunks_per_row;
  const int ng_win = prm.win_k >= gk ? prm.win_k / gk : 1;  // scale groups per window (<= 8)
  const int s_gi = lane & 7, s_row = lane >> 3;                // scales: 4 rows x 8 groups per pass
  const bool s_ok = s_gi < ng_win;

  const int nchunks = prm.meta[0];
  const int64_t nitems = static_cast<int64_t>(nchunks) * prm.tiles;
  // a split pair works through the same items in lock step
  const int unit = SPLIT ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int nunits = SPLIT ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int64_t it0 = (nitems * unit) / nunits;
  const int64_t it1 = (nitems * (unit + 1)) / nunits;
  int cur_chunk = -1;
  int4 ch = make_int4(0, 0, 0, 0);

  for (int64_t it = it0; it < it1; ++it) {
    const int chunk = static_cast<int>(it / prm.tiles);
    const int tile = static_cast<int>(it - static_cast<int64_t>(chunk) * prm.tiles);
    if (chunk != cur_chunk) {
      __syncthreads();  // x_s of the previous chunk consumed; codebook prefix visible after the next barrier
      ch = prm.chunks[chunk];
      const int nv = prm.IN / 8;  // 16-byte vectors per x row
      for (int q = threadIdx.x; q < ch.z * nv; q += kThreads) {
        const int p = q / nv, v = q - p * nv;
        const int pair = prm.sorted[ch.y + p];
        const int64_t xrow = static_cast<int64_t>(pair / prm.krep) * prm.IN;
        uint4 val;
        if (prm.x_mode == 0) val = __ldg(reinterpret_cast<const uint4*>(prm.x16 + xrow) + v);
        else if (prm.x_mode == 1) val = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(prm.xraw) + xrow) + v);
        else val = x8_to_16bit(prm.xraw, prm.x_dtype, xrow + v * 8, WR == 1);
        *reinterpret_cast<uint4*>(x_s + p * prm.x_stride + v * 8) = val;
      }
      cur_chunk = chunk;
      __syncthreads();
    }
    const int e = ch.x, P = ch.z;
    const int r0 = tile * rows_per_item + msub * 16;  // this warp's 16 rows
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
    // B rows this thread reads: token g of each n-tile (clamped into the chunk)
    int tok[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) tok[n] = min(g + 8 * n, P - 1);


    float part[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) part[n][0] = part[n][1] = part[n][2] = part[n][3] = 0.0f;
    // this warp's code rows of window w into buffer cs: asynchronous copies
    // when double-buffered (the next window's rows land while this one is
    // decoded), else 16-byte streaming loads; a dead row stages zeros
    auto stage_codes = [&](int w, uint32_t* cs) {
      if (l_chunk_ok) {
        const uint32_t* src = prm.codes + static_cast<int64_t>(w) * prm.win_words + l_chunk * 4;
#pragma unroll 4
        for (int rr = l_row; rr < 16; rr += rows_per_pass) {
          const int64_t cr = code_row(prm, e, min(r0 + rr, prm.OUT - 1));
          uint32_t* dst = cs + rr * prm.cs_stride + l_chunk * 4;
          if (prm.nbuf == 2 && cr >= 0) {
            cp_async16(dst, src + cr * prm.row_words);
          } else {
            uint4 v = make_uint4(0, 0, 0, 0);
            if (cr >= 0) v = ldg_stream_v4(src + cr * prm.row_words);
            *reinterpret_cast<uint4*>(dst) = v;
          }
        }
      }
    };
    // window w's scales, loaded into registers one window ahead
    uint16_t sv[4] = {0, 0, 0, 0};
    auto load_scales = [&](int w) {
      const int g0 = (w * prm.win_k) / gk;
      if (s_ok) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int64_t cr = code_row(prm, e, min(r0 + s_row + 4 * q, prm.OUT - 1));
          sv[q] = cr >= 0 ? __ldg(prm.scales + cr * prm.NGRP + g0 + s_gi) : uint16_t(0);
        }
      }
    };
    __syncwarp();
    if (wb < we) {
      if (prm.nbuf == 2) {
        stage_codes(wb, c_base);
        cp_async_commit();
      }
      load_scales(wb);
    }
    // scale-group tracking: k at which the current group ends, its slot in s_s
    int gend = ((wb * prm.win_k) / gk + 1) * gk;
    for (int w = wb; w < we; ++w) {
      uint32_t* c_s = c_base + (prm.nbuf == 2 ? static_cast<size_t>((w - wb) & 1) * cwin_words : 0);
      __syncwarp();  // every lane is done with the previous window's buffers
      if (s_ok) {
#pragma unroll
        for (int q = 0; q < 4; ++q) s_s[(s_row + 4 * q) * prm.sc_stride + s_gi] = sv[q];
      }
      if (prm.nbuf == 2) {
        if (w + 1 < we) stage_codes(w + 1, c_base + static_cast<size_t>((w + 1 - wb) & 1) * cwin_words);
        cp_async_commit();
        cp_async_wait<1>();  // this window's copies have landed
      } else {
        stage_codes(w, c_s);
      }
      if (w + 1 < we) load_scales(w + 1);
      __syncwarp();
      const int kw0 = w * prm.win_k;
      int bit0 = ((16 / D) * t) * prm.bits;      // this thread's first code in the window row
      const int bit_step = (64 / D) * prm.bits;  // per 64-k block
      const uint32_t* xrow[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) xrow[n] = reinterpret_cast<const uint32_t*>(x_s + tok[n] * prm.x_stride + kw0 + 16 * t);
      int gslot = 0;  // current group's column in s_s
      for (int kg = 0; kg < prm.win_k; kg += 64, bit0 += bit_step) {
        const int k0 = kw0 + kg;
        uint32_t ca[16 / D], cb2[16 / D];
        fetch_codes<D>(c_s + g * prm.cs_stride, bit0, mask, prm.bits, ca);
        fetch_codes<D>(c_s + (g + 8) * prm.cs_stride, bit0, mask, prm.bits, cb2);
        uint32_t wa[8], wb8[8];
        if constexpr (SPLIT) {
          lookup_split<D>(cb_s, cb_base, static_cast<uint32_t>(prm.cb_half), ca, wa);
          lookup_split<D>(cb_s, cb_base, static_cast<uint32_t>(prm.cb_half), cb2, wb8);
        } else {
          lookup<D, CB>(cb_s, prm.codebook, prm.ns, prm.K, ca, wa);
          lookup<D, CB>(cb_s, prm.codebook, prm.ns, prm.K, cb2, wb8);
        }
        if constexpr (WR != 0) {
          const __half sa = __ushort_as_half(s_s[g * prm.sc_stride + gslot]);
          const __half sb = __ushort_as_half(s_s[(g + 8) * prm.sc_stride + gslot]);
          const __half2 sa2 = __halves2half2(sa, sa), sb2 = __halves2half2(sb, sb);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            __half2 va = __hmul2(*reinterpret_cast<__half2*>(&wa[i]), sa2);
            __half2 vb = __hmul2(*reinterpret_cast<__half2*>(&wb8[i]), sb2);
            wa[i] = *reinterpret_cast<uint32_t*>(&va);
            wb8[i] = *reinterpret_cast<uint32_t*>(&vb);
            if (WR == 1) {
              wa[i] = h2_to_bf2(wa[i]);
              wb8[i] = h2_to_bf2(wb8[i]);
            }
          }
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (n > 0 && 8 * n >= P) break;  // token tile beyond this chunk's pairs: no x reads, no MMAs
          const uint4 xv0 = *reinterpret_cast<const uint4*>(xrow[n] + kg / 2);
          const uint4 xv1 = *reinterpret_cast<const uint4*>(xrow[n] + kg / 2 + 4);
          const uint32_t xb[8] = {xv0.x, xv0.y, xv0.z, xv0.w, xv1.x, xv1.y, xv1.z, xv1.w};
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const uint32_t a[4] = {wa[2 * m], wb8[2 * m], wa[2 * m + 1], wb8[2 * m + 1]};
            if (WR == 1) mma_bf16(WR != 0 ? acc[n] : part[n], a, xb[2 * m], xb[2 * m + 1]);
            else mma_f16(WR != 0 ? acc[n] : part[n], a, xb[2 * m], xb[2 * m + 1]);
          }
        }
        if (k0 + 64 == gend) {
          if constexpr (WR == 0) {
            const float sa = h2f(s_s[g * prm.sc_stride + gslot]);
            const float sb = h2f(s_s[(g + 8) * prm.sc_stride + gslot]);
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              acc[n][0] = fmaf(sa, part[n][0], acc[n][0]);
              acc[n][1] = fmaf(sa, part[n][1], acc[n][1]);
              acc[n][2] = fmaf(sb, part[n][2], acc[n][2]);
              acc[n][3] = fmaf(sb, part[n][3], acc[n][3]);
              part[n][0] = part[n][1] = part[n][2] = part[n][3] = 0.0f;
            }
          }
          gend += gk;
          ++gslot;
        }
      }
    }
    if constexpr (WR == 0) {
      // a group cut by the slice end is closed here with its own scale
      if ((static_cast<int64_t>(we) * prm.win_k) % gk != 0 && wb < we) {
        const int grp = (we * prm.win_k - 1) / gk;
        const int64_t ca = code_row(prm, e, min(r0 + g, prm.OUT - 1));
        const int64_t cb = code_row(prm, e, min(r0 + g + 8, prm.OUT - 1));
        const float sa = ca >= 0 ? h2f(prm.scales[ca * prm.NGRP + grp]) : 0.0f;
        const float sb = cb >= 0 ? h2f(prm.scales[cb * prm.NGRP + grp]) : 0.0f;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          acc[n][0] = fmaf(sa, part[n][0], acc[n][0]);
          acc[n][1] = fmaf(sa, part[n][1], acc[n][1]);
          acc[n][2] = fmaf(sb, part[n][2], acc[n][2]);
          acc[n][3] = fmaf(sb, part[n][3], acc[n][3]);
        }
      }
    }
    // D fragment: (row g, tokens 2t, 2t+1), (row g+8, tokens 2t, 2t+1) per n-tile
    if constexpr (SPLIT) {
      // both halves' partials -> rank 0's red[rank][slice][row][token]; rank 0
      // sums them in (rank, slice) order and stores
      const int ntok = 8 * NT;
      const size_t plane = static_cast<size_t>(ks) * rows_per_item * ntok;
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tk = 8 * n + 2 * t + (i & 1);
          const int rl = msub * 16 + g + 8 * (i >> 1);
          float* dst = red + crank * plane + (static_cast<size_t>(slice) * rows_per_item + rl) * ntok + tk;
          if (crank == 0) *dst = acc[n][i];
          else st_cluster_f32(map_to_rank(dst, 0), acc[n][i]);
        }
      cluster_sync_all();
      if (crank == 0) {
        for (int q = threadIdx.x; q < rows_per_item * P; q += kThreads) {
          const int rl = q / P, tk = q - rl * P;
          const int row = tile * rows_per_item + rl;
          if (row < prm.OUT) {
            float v = 0.0f;
            for (int rk = 0; rk < 2; ++rk)
              for (int sl = 0; sl < ks; ++sl)
                v = (rk == 0 && sl == 0) ? red[rl * ntok + tk]
                                         : v + red[rk * plane + (static_cast<size_t>(sl) * rows_per_item + rl) * ntok + tk];
            const int pair = prm.sorted[ch.y + tk];
            if (prm.row_table && code_row(prm, e, row) < 0) v = 0.0f;  // dead row: exact +0
            store_y(prm.y, static_cast<int64_t>(pair) * prm.OUT + row, v, prm.y_dtype, prm.round_f16_first != 0);
          }
        }
      }
      cluster_sync_all();  // rank 0 has read red before either CTA writes it again
    } else if (ks == 1) {
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tk = 8 * n + 2 * t + (i & 1);
          const int row = r0 + g + 8 * (i >> 1);
          if (tk < P && row < prm.OUT) {
            const int pair = prm.sorted[ch.y + tk];
            const float v = (prm.row_table && code_row(prm, e, row) < 0) ? 0.0f : acc[n][i];  // dead: +0
            store_y(prm.y, static_cast<int64_t>(pair) * prm.OUT + row, v, prm.y_dtype, prm.round_f16_first != 0);
          }
        }
    } else {
      // slice partials: red[slice][msub*16 + row][token], summed in slice order
      const int ntok = 8 * NT;
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tk = 8 * n + 2 * t + (i & 1);
          const int rl = msub * 16 + g + 8 * (i >> 1);
          red[(slice * rows_per_item + rl) * ntok + tk] = acc[n][i];
        }
      __syncthreads();
      for (int q = threadIdx.x; q < rows_per_item * P; q += kThreads) {
        const int rl = q / P, tk = q - rl * P;
        const int row = tile * rows_per_item + rl;
        if (row < prm.OUT) {
          float v = red[rl * ntok + tk];
          for (int sl = 1; sl < ks; ++sl) v = v + red[(sl * rows_per_item + rl) * ntok + tk];
          if (prm.row_table && code_row(prm, e, row) < 0) v = 0.0f;  // dead row: exact +0
          const int pair = prm.sorted[ch.y + tk];
          store_y(prm.y, static_cast<int64_t>(pair) * prm.OUT + row, v, prm.y_dtype, prm.round_f16_first != 0);
        }
      }
      __syncthreads();
    }
  }
}

// x -> 16-bit rows for the B operand: fp16 (narrowed, WR 0/2) or the raw
// bf16 (WR 1), for x whose rows the kernel cannot read in place.
__global__ void x_to_16bit_kernel(const void* __restrict__ x, int x_dtype, int64_t n, int to_bf16,
                                  uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = load_x(x, i, x_dtype, false);
    out[i] = to_bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
  }
}

}  // namespace

size_t mma_x16_bytes(int64_t T, int IN) { return (static_cast<size_t>(T) * IN * 2 + 255) & ~size_t(255); }

static int window_k(const LinearGeometry& geo) {
  int win_k = kWinK;
  while (((win_k / geo.D) * geo.bits) % 128 != 0 && win_k < 8192) win_k *= 2;
  return win_k;
}

bool mma_decode_supported(const LinearGeometry& geo, int wround, int x_dtype) {
  if (geo.G % 64 != 0) return false;   // blocks of 64 k never straddle a scale group
  const int win_k = window_k(geo);
  if (geo.IN % win_k != 0) return false;
  if (win_k % geo.G != 0 && geo.G % win_k != 0) return false;
  const int chunks_per_row = (win_k / geo.D) * geo.bits / 128;
  if (chunks_per_row > 16) return false;   // window loader covers <= 16 chunks per row
  if (win_k < geo.G ? false : (win_k / geo.G) > 8) return false;  // <= 8 scale groups per window
  if (geo.bits > 16) return false;
  if (wround == 1 && x_dtype != VQB_BF16) return false;
  if (wround == 2 && x_dtype == VQB_F32) return false;
  if ((reinterpret_cast<uintptr_t>(geo.codes) & 15) != 0 || geo.row_words % 4 != 0) return false;
  return true;
}

vqb_status launch_decode_mma(const LinearGeometry& geo, const GroupedDecodeArgs& a, uint16_t* x16, int T,
                             cudaStream_t stream) {
  if (a.N <= 0) return VQB_OK;
  DeviceInfo di;
  if (device_info(&di) != VQB_OK) return VQB_CUDA_ERROR;
  const int nsm = di.sms;
  const int WR = a.wround;
  // x -> 16-bit B-operand rows (the reference's host cast for the MoE path):
  // converted while the kernel stages x when its rows are 16-byte aligned
  // (IN is a multiple of 512 here), else by a conversion pass
  const bool x_direct = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  const int x_target = WR == 1 ? VQB_BF16 : VQB_F16;
  if (!x_direct) {
    const int64_t n = static_cast<int64_t>(T) * geo.IN;
    int64_t blocks = (n + 255) / 256;
    if (blocks > 4 * nsm) blocks = 4 * nsm;
    if (launch_pdl(x_to_16bit_kernel, static_cast<unsigned>(blocks), 256, 0, stream, a.x, a.x_dtype, n,
                   WR == 1 ? 1 : 0, x16) != cudaSuccess)
      return VQB_CUDA_ERROR;
    note_launch();
  }
  MParams prm{};
  prm.codes = static_cast<const uint32_t*>(geo.codes);
  prm.codebook = static_cast<const uint16_t*>(geo.codebook);
  prm.scales = static_cast<const uint16_t*>(geo.scales);
  prm.x16 = x16;
  prm.xraw = a.x;
  prm.x_dtype = a.x_dtype;
  prm.x_mode = !x_direct ? 0 : (a.x_dtype == x_target ? 1 : 2);
  prm.sorted = a.route->sorted;
  prm.chunks = a.route->chunks;
  prm.meta = a.route->meta;
  prm.y = a.y;
  prm.row_words = geo.row_words;
  prm.expert_words = static_cast<int64_t>(geo.OUT) * geo.row_words;
  prm.row_table = geo.row_table;
  prm.nrows = geo.nrows;
  prm.OUT = geo.OUT;
  prm.IN = geo.IN;
  prm.G = geo.G;
  prm.NGRP = geo.IN / geo.G;
  prm.NSUB = geo.IN / geo.D;
  prm.bits = geo.bits;
  prm.K = geo.K;
  prm.krep = a.krep;
  prm.y_dtype = a.y_dtype;
  prm.round_f16_first = a.round_f16_first ? 1 : 0;
  prm.pm = a.pmax;
  const int NT = (a.pmax + 7) / 8;
  // window: 512 k values, doubled while a row's window is not 16-byte whole
  const int win_k = window_k(geo);
  if (geo.IN % win_k != 0) return VQB_UNSUPPORTED_GEOMETRY;
  prm.win_k = win_k;
  prm.win_words = (win_k / geo.D) * geo.bits / 32;
  // padded row stride: an odd number of 16-byte chunks, plus room for the
  // three-word reads of the last codes
  int cs_chunks = prm.win_words / 4 + 1;
  if ((cs_chunks & 1) == 0) ++cs_chunks;
  prm.cs_stride = cs_chunks * 4;
  const int grp_per_win = (win_k + geo.G - 1) / geo.G + 1;
  prm.sc_stride = (grp_per_win + 7) & ~7;
  prm.x_stride = ((geo.IN + 7) & ~7) + 8;  // +16 bytes
  // K-slices (windows) and M-tiles per item: 16 warps
  int ks = a.ks;
  const int n_win = geo.IN / win_k;
  if (ks <= 0) {
    // K-slices per item.  With eight or more 16-row units per warp at one
    // slice, one slice (no partial reduction, the most shared memory left for
    // the codebook); otherwise the most slices among those that minimise
    // (items per CTA, rounded up) x (windows of the longest slice).  Chunks
    // are estimated as the distinct experts uniform routing would give, or
    // pairs / chunk size if more.  Measured on B200 (us): d8/K16384 switch
    // 1024 x 4096 at 80 pairs: 229 / 200 / 187 / 197 for 1 / 2 / 4 / 8 slices,
    // at 640 pairs 821 / 859 / 895 / 1001; dense d8 17408 x 5120 at N = 1
    // 107 / 65 / 72 / 90; dense d2 5120 x 5120 at N = 1: 89 / 52 / 44 / 44.
    const double de = static_cast<double>(geo.E) * (1.0 - std::exp(-static_cast<double>(a.N) / geo.E));
    const int64_t chunks_est =
        std::max<int64_t>((a.N + a.pmax - 1) / a.pmax, std::max<int64_t>(1, static_cast<int64_t>(de + 0.5)));
    const int64_t units = chunks_est * ((geo.OUT + 15) / 16);
    ks = 1;
    if (units < 8 * static_cast<int64_t>(nsm) * kWarps) {
      int64_t best = -1;
      for (int k = 1; k <= 16 && k <= n_win; k *= 2) {
        const int64_t items = chunks_est * ((geo.OUT + 16 * (kWarps / k) - 1) / (16 * (kWarps / k)));
        const int64_t cost = ((items + nsm - 1) / nsm) * ((n_win + k - 1) / k);
        if (best < 0 || cost <= best) { best = cost; ks = k; }
      }
    }
  }
  if (ks > n_win) ks = n_win;
  if (ks != 1 && ks != 2 && ks != 4 && ks != 8 && ks != 16) return VQB_BAD_SHAPE;
  prm.ks = ks;
  prm.mt = kWarps / ks;
  const int rows_per_item = 16 * prm.mt;
  prm.tiles = (geo.OUT + rows_per_item - 1) / rows_per_item;

  const size_t x_bytes = (static_cast<size_t>(a.pmax) * prm.x_stride * 2 + 15) & ~size_t(15);
  const size_t win_bytes = (static_cast<size_t>(16) * prm.cs_stride * 4 + 16 * prm.sc_stride * 2 + 15) & ~size_t(15);
  // the device's opt-in limit less 1 KB: a launch never asks for the last
  // bytes of shared memory (an ncu launch list once reported LaunchFailed for
  // a launch that left 64 bytes; the margin costs 64 d8 codebook entries)
  const size_t budget = static_cast<size_t>(di.smem_optin) - 1024;
  const size_t entry = static_cast<size_t>(geo.D) * 2;
  // A codebook larger than what one SM can hold next to the staging buffers is
  // split across a CTA pair (d8/K16384: 2 x 128 KB), so no lookup leaves
  // shared memory; smaller ones are held whole by every CTA.
  const size_t red_plain = ks > 1 ? static_cast<size_t>(ks) * rows_per_item * 8 * NT * sizeof(float) : 0;
  const size_t fixed_plain = x_bytes + kWarps * win_bytes + red_plain;
  bool split = false;
  // measured on B200 (C2 shapes): the shared-memory prefix with the rest in
  // L1/L2 beats the pair split, whose doubled per-SM instruction stream costs
  // more than the L2 lookups it removes; the split stays available on request
  const bool may_split = a.stage_codebook == 3;
  if (may_split && fixed_plain + static_cast<size_t>(geo.K) * entry > budget && (geo.K % 16) == 0) {
    const size_t red_split = 2 * static_cast<size_t>(ks) * rows_per_item * 8 * NT * sizeof(float);
    if (x_bytes + kWarps * win_bytes + red_split + static_cast<size_t>(geo.K / 2) * entry <= budget) split = true;
  }
  const size_t red_bytes = split ? 2 * static_cast<size_t>(ks) * rows_per_item * 8 * NT * sizeof(float) : red_plain;
  const size_t fixed = x_bytes + kWarps * win_bytes + red_bytes;
  if (fixed > budget) return VQB_UNSUPPORTED_GEOMETRY;
  size_t ns;
  if (split) {
    ns = static_cast<size_t>(geo.K / 2);
    prm.cb_half = geo.K / 2;
  } else {
    ns = (budget - fixed) / entry;
    ns = ns / 8 * 8;
    if (ns > static_cast<size_t>(geo.K)) ns = geo.K;
    if (a.stage_codebook == 0) ns = 0;
    prm.cb_half = 0;
  }
  // the whole codebook plus its zero entry in shared memory: one unconditional read per code
  const bool full = !split && ns == static_cast<size_t>(geo.K) &&
                    fixed + ((static_cast<size_t>(geo.K + 1) * entry + 15) & ~size_t(15)) <= budget;
  prm.ns = static_cast<int>(ns);
  size_t smem = (((full ? ns + 1 : ns) * entry + 15) & ~size_t(15)) + fixed;
  // a second code-window buffer per warp (the next window copied while this
  // one is decoded) when the whole codebook is resident and it still fits; the
  // prefix and pair-split modes spend that memory on codebook entries
  const size_t cwin = static_cast<size_t>(16) * prm.cs_stride * 4;
  prm.nbuf = 1;
  if (full && smem + kWarps * cwin <= budget) {
    prm.nbuf = 2;
    smem += kWarps * cwin;
  }
  const int grid = split ? (nsm & ~1) : nsm;

  cudaError_t ce = cudaSuccess;
  auto launch = [&](auto kern, bool is_split) {
    ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (ce != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = is_split ? 2 : 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    timer_before(stream);
    ce = cudaLaunchKernelEx(&cfg, kern, prm);
    timer_after(stream);
    if (ce == cudaSuccess) note_launch();
  };
#define VQB_M1(DD, WW, NN)                                                               \
  do {                                                                                   \
    if (split) launch(vq_decode_mma_kernel<DD, WW, NN, kCbSplit>, true);                  \
    else if (full) launch(vq_decode_mma_kernel<DD, WW, NN, kCbFull>, false);              \
    else launch(vq_decode_mma_kernel<DD, WW, NN, kCbPrefix>, false);                      \
  } while (0)
#define VQB_M2(DD, WW) do { if (NT == 1) VQB_M1(DD, WW, 1); else VQB_M1(DD, WW, 2); } while (0)
#define VQB_M3(DD) do { if (WR == 1) VQB_M2(DD, 1); else if (WR == 2) VQB_M2(DD, 2); else VQB_M2(DD, 0); } while (0)
  if (geo.D == 8) VQB_M3(8);
  else if (geo.D == 4) VQB_M3(4);
  else VQB_M3(2);
#undef VQB_M1
#undef VQB_M2
#undef VQB_M3
  return ce == cudaSuccess ? VQB_OK : VQB_CUDA_ERROR;
}

}  // namespace vqb
