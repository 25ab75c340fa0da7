// Small-N fused VQ decode kernel (sm_100a): y[p, r] = sum_k W_{e(p)}[r, k] x[t(p), k]
// with W decoded on the fly from packed codes, the fp16 codebook and the
// per-(row, group) fp16 scales.  This is the B200 kernel behind the
// reference's fused decode dispatch (vq_switch.py:2919-3249; the packed d8
// walk kernel :1316-1392 is the arithmetic it keeps).
//
// Work mapping.  One CTA = 256 threads = 8 warps covers a tile of
// 32 * (8 / ks) output rows of ONE (token, expert) pair and splits each row's
// code stream into ks contiguous slices (one warp per slice).  Lane = row:
// each thread walks its own row's packed bit stream with 16-byte streaming
// loads (L1::no_allocate, so the code stream does not evict the codebook from
// L1), looks each code up in the codebook through the read-only L1 path, and
// takes the dot product with the pair's token row, which the CTA stages once
// in shared memory as fp32 (every lane reads the same x element: a broadcast).
//
// Numerics (per slice, identical to the reference walk): per code the D
// products cb*x are summed left to right (exact fp16*fp16 products, so the
// fma chain equals the sequential sum), a group's partial `gacc` collects its
// codes in order, and `acc = fma(s[g], gacc, acc)` closes each group.  With
// ks == 1 this is the serial order of vq_switch.py:1344-1352 exactly; with
// ks > 1 the slice accumulators are added in slice order at the end.
#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

struct DecodeParams {
  const uint32_t* codes;     // packed words (unpacked u8/u16 rows are read as 8/16-bit streams)
  const uint16_t* codebook;  // [K, D] fp16 bits
  const uint16_t* scales;    // [E, OUT, NGRP] fp16 bits
  const void* x;             // [T, IN]
  const uint32_t* idx;       // [N] expert per pair, or nullptr (dense: expert 0)
  void* y;                   // [N, OUT]
  int* err;                  // device error word (bad expert index), may be nullptr
  int64_t expert_words;      // OUT * row_words
  const int32_t* row_table;  // SKIPZERO [E, OUT] -> compact row (-1 dead), nullptr = plain layout
  int64_t nrows;             // rows of codes / scales
  int row_words;             // words per code row
  int N, krep, E;
  int OUT, IN, G, NGRP, NSUB;
  int bits;
  int ks;                    // K-slices per row (1, 2, 4, 8)
  int x_dtype, y_dtype;
  int narrow_x_f16;          // x takes an fp16 rounding first
  int round_f16_first;       // output: fp16 rounding, then y_dtype
  int wround;                // numerics: 0 = group partials (fused kernels),
                             // 1 = weights rounded fp16 then bf16, 2 = weights rounded fp16
                             //     (dense _decode_matmul, vq_dense.py:267-312)
};

// One code's contribution under the _decode_matmul numerics: each weight is
// W = fp16(cb * s) (one RNE rounding of the exact fp32 product, the fp16
// multiply of vq_dense.py:136), then re-rounded to bf16 when x is bf16
// (`.astype(xf.dtype)`, vq_dense.py:294), and accumulated in ascending k.
template <int D, bool TO_BF16>
__device__ __forceinline__ float code_dot_wround(const uint16_t* __restrict__ cb, uint32_t c, float s,
                                                 const float* xs, float acc) {
  uint32_t w[D / 2];
  if constexpr (D == 8) {
    const uint4 e = __ldg(reinterpret_cast<const uint4*>(cb) + c);
    w[0] = e.x; w[1] = e.y; w[2] = e.z; w[3] = e.w;
  } else if constexpr (D == 4) {
    const uint2 e = __ldg(reinterpret_cast<const uint2*>(cb) + c);
    w[0] = e.x; w[1] = e.y;
  } else {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(cb) + c);
  }
#pragma unroll
  for (int i = 0; i < D / 2; ++i) {
    const float2 f = h2x2f(w[i]);
    float w0 = __half2float(__float2half_rn(f.x * s));
    float w1 = __half2float(__float2half_rn(f.y * s));
    if (TO_BF16) {
      w0 = __bfloat162float(__float2bfloat16_rn(w0));
      w1 = __bfloat162float(__float2bfloat16_rn(w1));
    }
    acc = fmaf(xs[2 * i], w0, acc);
    acc = fmaf(xs[2 * i + 1], w1, acc);
  }
  return acc;
}

template <int D>
__device__ __forceinline__ float code_dot(const uint16_t* __restrict__ cb, uint32_t c, const float* xs) {
  if constexpr (D == 8) {
    const uint4 e = __ldg(reinterpret_cast<const uint4*>(cb) + c);
    const float2 a = h2x2f(e.x), b = h2x2f(e.y), cc = h2x2f(e.z), d = h2x2f(e.w);
    const float4 x0 = *reinterpret_cast<const float4*>(xs);
    const float4 x1 = *reinterpret_cast<const float4*>(xs + 4);
    float d0 = a.x * x0.x;
    d0 = fmaf(a.y, x0.y, d0);
    d0 = fmaf(b.x, x0.z, d0);
    d0 = fmaf(b.y, x0.w, d0);
    float d1 = cc.x * x1.x;
    d1 = fmaf(cc.y, x1.y, d1);
    d1 = fmaf(d.x, x1.z, d1);
    d1 = fmaf(d.y, x1.w, d1);
    return d0 + d1;
  } else if constexpr (D == 4) {
    const uint2 e = __ldg(reinterpret_cast<const uint2*>(cb) + c);
    const float2 a = h2x2f(e.x), b = h2x2f(e.y);
    const float4 x0 = *reinterpret_cast<const float4*>(xs);
    float d0 = a.x * x0.x;
    d0 = fmaf(a.y, x0.y, d0);
    d0 = fmaf(b.x, x0.z, d0);
    d0 = fmaf(b.y, x0.w, d0);
    return d0;
  } else {
    const uint32_t e = __ldg(reinterpret_cast<const uint32_t*>(cb) + c);
    const float2 a = h2x2f(e);
    const float2 x0 = *reinterpret_cast<const float2*>(xs);
    return fmaf(a.y, x0.y, a.x * x0.x);
  }
}

template <int D, bool VEC, int WR>
__global__ void __launch_bounds__(256) vq_decode_kernel(const DecodeParams prm) {
  extern __shared__ float smem[];
  float* xs = smem;                                  // [IN] fp32 token row
  const int ks = prm.ks;
  const int rows_per_cta = 32 * (8 / ks);
  float* red = smem + ((prm.IN + 3) & ~3);           // [ks][rows_per_cta] slice partials

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = warp % ks;
  const int rsub = warp / ks;
  const uint32_t mask = (prm.bits >= 32) ? 0xffffffffu : ((1u << prm.bits) - 1u);
  const int SPG = prm.G / D;

  // slice bounds over the code stream (any boundary; groups may straddle)
  const int jb = static_cast<int>((static_cast<int64_t>(prm.NSUB) * slice) / ks);
  const int je = static_cast<int>((static_cast<int64_t>(prm.NSUB) * (slice + 1)) / ks);

  for (int p = blockIdx.y; p < prm.N; p += gridDim.y) {
    const int t = p / prm.krep;
    uint32_t e = prm.idx ? prm.idx[p] : 0u;
    if (e == kSkipExpert) continue;  // a pair left out: no output row (uniform over the CTA)
    if (e >= static_cast<uint32_t>(prm.E)) {
      // routing error: report once and treat the pair as expert 0 (no OOB read)
      if (prm.err && threadIdx.x == 0) atomicExch(prm.err, static_cast<int>(VQB_BAD_ROUTING));
      e = 0;
    }
    __syncthreads();  // previous pair's xs / red fully consumed
    const int64_t xoff = static_cast<int64_t>(t) * prm.IN;
    for (int i = threadIdx.x; i < prm.IN; i += blockDim.x)
      xs[i] = load_x(prm.x, xoff + i, prm.x_dtype, prm.narrow_x_f16 != 0);
    __syncthreads();

    const int r = blockIdx.x * rows_per_cta + rsub * 32 + lane;
    float acc = 0.0f;
    // the row's place in codes / scales: (e, r), or its compact row (dead -> -1: +0 out, nothing read)
    int64_t crow = static_cast<int64_t>(e) * prm.OUT + r;
    if (prm.row_table && r < prm.OUT) {
      crow = prm.row_table[crow];
      if (crow >= prm.nrows) crow = -1;
    }
    if (r < prm.OUT && jb < je && crow >= 0) {
      const uint32_t* row = prm.codes + crow * prm.row_words;
      const uint16_t* srow = prm.scales + crow * prm.NGRP;
      BitWalker<VEC> wk;
      wk.init(row, static_cast<int64_t>(jb) * prm.bits);
      int g = jb / SPG;
      int gend = (g + 1) * SPG;
      float gacc = 0.0f;
      int j = jb;
      if constexpr (WR != 0) {
        float s = h2f(srow[g]);
        for (; j < je; ++j) {
          if (j == gend) {
            ++g;
            gend += SPG;
            s = h2f(srow[g]);
          }
          const uint32_t c = wk.next(prm.bits, mask);
          acc = code_dot_wround<D, WR == 1>(prm.codebook, c, s, xs + j * D, acc);
        }
        (void)gacc;
      } else if constexpr (D == 2) {
        // reference d2 shape: four dots summed ((d0+d1)+d2)+d3 per 4 codes
        // inside a group (vq_switch.py:1970-1973)
        while (j < je) {
          const int run_end = min(gend, je);
          while (j + 4 <= run_end && ((j - (g * SPG)) & 3) == 0) {
            const uint32_t c0 = wk.next(prm.bits, mask), c1 = wk.next(prm.bits, mask);
            const uint32_t c2 = wk.next(prm.bits, mask), c3 = wk.next(prm.bits, mask);
            const float d0 = code_dot<2>(prm.codebook, c0, xs + j * 2);
            const float d1 = code_dot<2>(prm.codebook, c1, xs + (j + 1) * 2);
            const float d2 = code_dot<2>(prm.codebook, c2, xs + (j + 2) * 2);
            const float d3 = code_dot<2>(prm.codebook, c3, xs + (j + 3) * 2);
            gacc = gacc + (((d0 + d1) + d2) + d3);
            j += 4;
          }
          for (; j < run_end; ++j) gacc = gacc + code_dot<2>(prm.codebook, wk.next(prm.bits, mask), xs + j * 2);
          if (j == gend || j == je) {
            acc = fmaf(h2f(srow[g]), gacc, acc);
            gacc = 0.0f;
            ++g;
            gend += SPG;
          }
        }
      } else {
        for (; j < je; ++j) {
          const uint32_t c = wk.next(prm.bits, mask);
          gacc = gacc + code_dot<D>(prm.codebook, c, xs + j * D);
          if (j + 1 == gend || j + 1 == je) {
            acc = fmaf(h2f(srow[g]), gacc, acc);
            gacc = 0.0f;
            ++g;
            gend += SPG;
          }
        }
      }
    }
    if (ks == 1) {
      if (r < prm.OUT)
        store_y(prm.y, static_cast<int64_t>(p) * prm.OUT + r, acc, prm.y_dtype, prm.round_f16_first != 0);
    } else {
      red[slice * rows_per_cta + rsub * 32 + lane] = acc;
      __syncthreads();
      const int ri = threadIdx.x;
      if (ri < rows_per_cta) {
        const int rr = blockIdx.x * rows_per_cta + ri;
        if (rr < prm.OUT) {
          float s = red[ri];
          for (int q = 1; q < ks; ++q) s = s + red[q * rows_per_cta + ri];
          if (prm.row_table) {
            const int64_t cr = prm.row_table[static_cast<int64_t>(e) * prm.OUT + rr];
            if (cr < 0 || cr >= prm.nrows) s = 0.0f;  // dead row: exact +0
          }
          store_y(prm.y, static_cast<int64_t>(p) * prm.OUT + rr, s, prm.y_dtype, prm.round_f16_first != 0);
        }
      }
    }
  }
}

// Host launcher.  Shapes were validated by the caller (vqb_api.cu).
vqb_status launch_decode(const LinearGeometry& geo, const void* x, int x_dtype, int T, const uint32_t* idx,
                         int N, int krep, void* y, int y_dtype, bool narrow_x_f16, bool round_f16_first,
                         int wround, int ks, int* err, cudaStream_t stream) {
  DecodeParams prm{};
  prm.wround = wround;
  prm.codes = static_cast<const uint32_t*>(geo.codes);
  prm.codebook = static_cast<const uint16_t*>(geo.codebook);
  prm.scales = static_cast<const uint16_t*>(geo.scales);
  prm.x = x;
  prm.idx = idx;
  prm.y = y;
  prm.err = err;
  prm.row_words = geo.row_words;
  prm.expert_words = static_cast<int64_t>(geo.OUT) * geo.row_words;
  prm.row_table = geo.row_table;
  prm.nrows = geo.nrows;
  prm.N = N;
  prm.krep = krep;
  prm.E = geo.E;
  prm.OUT = geo.OUT;
  prm.IN = geo.IN;
  prm.G = geo.G;
  prm.NGRP = geo.IN / geo.G;
  prm.NSUB = geo.IN / geo.D;
  prm.bits = geo.bits;
  prm.x_dtype = x_dtype;
  prm.y_dtype = y_dtype;
  prm.narrow_x_f16 = narrow_x_f16 ? 1 : 0;
  prm.round_f16_first = round_f16_first ? 1 : 0;
  (void)T;
  if (N <= 0) return VQB_OK;

  if (ks <= 0) {
    // enough independent warps to fill 148 SMs: split the row's code stream
    // when the pair count is small
    const int64_t rows_total = static_cast<int64_t>(N) * geo.OUT;
    ks = 1;
    while (ks < 8 && rows_total * ks < 148LL * 32 * 48 && (geo.IN / geo.D) / (ks * 2) >= 32) ks *= 2;
  }
  prm.ks = ks;
  const int rows_per_cta = 32 * (8 / ks);
  const size_t smem = sizeof(float) * (((geo.IN + 3) & ~3) + static_cast<size_t>(ks) * rows_per_cta);
  dim3 grid((geo.OUT + rows_per_cta - 1) / rows_per_cta, N < 65535 ? N : 65535);
  const bool vec = (geo.row_words % 4 == 0) && ((reinterpret_cast<uintptr_t>(geo.codes) & 15) == 0);

  cudaError_t ce = cudaSuccess;
#define VQB_LAUNCH1(DD, VV, WW)                                                                      \
  do {                                                                                              \
    auto kern = vq_decode_kernel<DD, VV, WW>;                                                       \
    if (smem > 48 * 1024) {                                                                         \
      ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,                  \
                                static_cast<int>(smem));                                            \
      if (ce != cudaSuccess) break;                                                                 \
    }                                                                                               \
    timer_before(stream);                                                                           \
    kern<<<grid, 256, smem, stream>>>(prm);                                                         \
    timer_after(stream);                                                                            \
    ce = cudaGetLastError();                                                                        \
    if (ce == cudaSuccess) note_launch();                                                           \
  } while (0)
#define VQB_LAUNCH(DD, VV)                  \
  do {                                      \
    if (wround == 1) VQB_LAUNCH1(DD, VV, 1); \
    else if (wround == 2) VQB_LAUNCH1(DD, VV, 2); \
    else VQB_LAUNCH1(DD, VV, 0);            \
  } while (0)
  if (geo.D == 8) { if (vec) VQB_LAUNCH(8, true); else VQB_LAUNCH(8, false); }
  else if (geo.D == 4) { if (vec) VQB_LAUNCH(4, true); else VQB_LAUNCH(4, false); }
  else { if (vec) VQB_LAUNCH(2, true); else VQB_LAUNCH(2, false); }
#undef VQB_LAUNCH
#undef VQB_LAUNCH1
  return ce == cudaSuccess ? VQB_OK : VQB_CUDA_ERROR;
}

}  // namespace vqb
