/*
 * vq_oracle.c -- CPU restatement of the VQLab VQ expert runtime arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (vqlab_b200/) links,
 * loads or calls this file.  It is used by tests/ as the parity checker,
 * by __graft_entry__.smoke() as the checker of one small GPU call, and by
 * bench.py's CPU-baseline legs as the timed CPU implementation of the path.
 *
 * What it restates (citations are into the reference project, VQLab):
 *   - the vq_pack v1 bit layout reader ............ src/vqlab/runtime/vq_pack.py:79-97
 *     (extraction formula of the Metal VQ_CODE macro, vq_switch.py:595-603)
 *   - the fused small-N decode kernels:
 *       serial-fma "walk" order ................... vq_switch.py:1316-1354, :1373-1392
 *       simd_sum ("ss") 32-group-block order ...... vq_switch.py:1619-1660
 *       dense d2 devx_ss (direct output cast) ..... vq_switch.py:1928-1983, :2495-2524
 *   - gemmseg2 ACCS prefill (per-group fp32 partial, acc += s*partial)
 *                                                   vq_switch.py:4171-4203
 *   - dense _decode_matmul: W16 = fp16(cb*s), W = W16 in x's dtype, y = x @ W^T
 *                                                   vq_dense.py:132-137, :267-312
 *   - float64 exact reconstruction ................ score/kernel_truth_moe.py:37-50
 *
 * The Metal kernels themselves cannot run here (no Apple GPU, no MLX), so the
 * restated orders below are the source's written order; where Metal leaves an
 * order unspecified (dot(float4,float4), simd_sum, the simdgroup MMA) the
 * choice made here is named at the function.  Bit-level agreement with the
 * Metal kernels is therefore UNPINNED for the matmul arithmetic; the vq_pack
 * reader IS pinned by golden vectors produced by the reference's own vq_pack.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- numbers */

static inline float h2f(uint16_t h) { _Float16 v; memcpy(&v, &h, 2); return (float)v; }
static inline uint16_t f2h(float f) { _Float16 v = (_Float16)f; uint16_t h; memcpy(&h, &v, 2); return h; }
static inline float bf2f(uint16_t b) { uint32_t u = (uint32_t)b << 16; float f; memcpy(&f, &u, 4); return f; }
/* IEEE round-to-nearest-even float32 -> bfloat16 (NaN stays a quiet NaN). */
static inline uint16_t f2bf(float f) {
  uint32_t u; memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

void orc_f32_to_f16(const float* in, uint16_t* out, int64_t n) { for (int64_t i = 0; i < n; ++i) out[i] = f2h(in[i]); }
void orc_f32_to_bf16(const float* in, uint16_t* out, int64_t n) { for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]); }
void orc_f16_to_f32(const uint16_t* in, float* out, int64_t n) { for (int64_t i = 0; i < n; ++i) out[i] = h2f(in[i]); }
void orc_bf16_to_f32(const uint16_t* in, float* out, int64_t n) { for (int64_t i = 0; i < n; ++i) out[i] = bf2f(in[i]); }

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* --------------------------------------------------------------- vq_pack */

/* Code j of a packed row: the row is an LSB-first bit stream in which code j
 * occupies bits [j*bits, (j+1)*bits) (32 codes fill exactly `bits` words, so
 * the per-block layout of vq_pack.py:11-27 is this stream cut into blocks).
 * Same two-word read as vq_pack.unpack (vq_pack.py:87-95). */
static inline uint32_t extract_code(const uint32_t* row, int64_t j, int bits) {
  const int64_t bit = j * (int64_t)bits;
  const int64_t w = bit >> 5;
  const int sh = (int)(bit & 31);
  uint64_t v = (uint64_t)row[w] >> sh;
  if (sh + bits > 32) v |= (uint64_t)row[w + 1] << (32 - sh);
  return (uint32_t)(v & ((1u << bits) - 1u));
}

int64_t orc_words_per_row(int64_t nsub, int bits) { return (nsub + 31) / 32 * bits; }

/* packed [rows, wpr] -> codes [rows, nsub] (uint16). */
void orc_unpack(const uint32_t* packed, int64_t rows, int64_t wpr, int64_t nsub, int bits, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t j = 0; j < nsub; ++j)
      out[r * nsub + j] = (uint16_t)extract_code(packed + r * wpr, j, bits);
}

/* codes [rows, nsub] -> packed [rows, wpr]; the inverse of orc_unpack
 * (vq_pack.py:48-76: zero-padded tail block, codes must fit `bits`). */
int orc_pack(const uint16_t* codes, int64_t rows, int64_t nsub, int bits, uint32_t* out) {
  const int64_t wpr = orc_words_per_row(nsub, bits);
  int bad = 0;
#pragma omp parallel for schedule(static) reduction(|:bad)
  for (int64_t r = 0; r < rows; ++r) {
    uint32_t* o = out + r * wpr;
    memset(o, 0, (size_t)wpr * 4);
    for (int64_t j = 0; j < nsub; ++j) {
      uint32_t c = codes[r * nsub + j];
      if (c >> bits) { bad = 1; continue; }
      const int64_t bit = j * (int64_t)bits;
      const int64_t w = bit >> 5;
      const int sh = (int)(bit & 31);
      uint64_t v = (uint64_t)c << sh;
      o[w] |= (uint32_t)v;
      if (sh + bits > 32) o[w + 1] |= (uint32_t)(v >> 32);
    }
  }
  return bad;
}

/* ------------------------------------------------------------ fused decode */

/* One code's contribution to a group partial, in the reference's written
 * order.  d8 (vq_switch.py:1349-1350): gacc += dot4(cb[0:4],x[0:4]) +
 * dot4(cb[4:8],x[4:8]).  d4 (:726-728 family): one dot4 per code.  d2 dense
 * (:1970-1973): four dot2 per 4 codes, summed ((d0+d1)+d2)+d3 then added.
 * dot(floatN, floatN) is taken as the left-to-right sum of exact products
 * (fp16*fp16 products are exact in fp32, so fma-vs-mul does not matter; only
 * the order does, and Metal does not specify it: UNPINNED). */
static inline float dot_n(const float* a, const float* b, int n) {
  float s = a[0] * b[0];
  for (int i = 1; i < n; ++i) s = s + a[i] * b[i];
  return s;
}

/* Group partial over codes [j0, j0+cnt) of one row. */
static float group_partial(const uint16_t* crow, const float* cbf, const float* xs, int64_t j0, int cnt, int D) {
  float gacc = 0.0f;
  if (D == 8) {
    for (int q = 0; q < cnt; ++q) {
      const int64_t j = j0 + q;
      const float* e = cbf + (int64_t)crow[j] * 8;
      const float* xv = xs + j * 8;
      gacc = gacc + (dot_n(e, xv, 4) + dot_n(e + 4, xv + 4, 4));
    }
  } else if (D == 4) {
    for (int q = 0; q < cnt; ++q) {
      const int64_t j = j0 + q;
      gacc = gacc + dot_n(cbf + (int64_t)crow[j] * 4, xs + j * 4, 4);
    }
  } else { /* D == 2: groups of four codes, ((d0+d1)+d2)+d3 */
    int q = 0;
    for (; q + 4 <= cnt; q += 4) {
      const int64_t j = j0 + q;
      float d0 = dot_n(cbf + (int64_t)crow[j] * 2, xs + j * 2, 2);
      float d1 = dot_n(cbf + (int64_t)crow[j + 1] * 2, xs + (j + 1) * 2, 2);
      float d2 = dot_n(cbf + (int64_t)crow[j + 2] * 2, xs + (j + 2) * 2, 2);
      float d3 = dot_n(cbf + (int64_t)crow[j + 3] * 2, xs + (j + 3) * 2, 2);
      gacc = gacc + (((d0 + d1) + d2) + d3);
    }
    for (; q < cnt; ++q) {
      const int64_t j = j0 + q;
      gacc = gacc + dot_n(cbf + (int64_t)crow[j] * 2, xs + j * 2, 2);
    }
  }
  return gacc;
}

/* The reduction across groups.
 *   mode 0 "walk":  acc = fma(s[g], gacc[g], acc), ascending g (vq_switch.py:1351)
 *   mode 1 "ss":    per block of 32 groups, acc += tree_sum(s[g]*gacc[g]); the
 *                   32-lane simd_sum is taken as an xor-butterfly 16,8,4,2,1
 *                   (vq_switch.py:1640-1644; Metal leaves the tree: UNPINNED)
 *   mode 2 "accs":  acc = fma(s[g], partial[g], acc) -- the gemmseg2 ACCS update
 *                   (vq_switch.py:4188-4191; partial order inside the MMA is
 *                   unspecified, taken as the ascending-code sum)
 *   mode 3 "prescaled": the gemmseg2 arm without ACCS (vq_switch.py:3897-3900,
 *                   :3960-3976: the staged weight is (half)(s * cb), one RNE
 *                   rounding of the exact fp32 product), y = sum_k x*W in fp32
 *                   over ascending k (the MMA's order: unspecified); computed by
 *                   prescaled_row below, not by this reduction */
static float reduce_groups(const float* s, const float* gacc, int ngrp, int mode) {
  float acc = 0.0f;
  if (mode == 1) {
    for (int b = 0; b < ngrp; b += 32) {
      float v[32];
      for (int l = 0; l < 32; ++l) v[l] = (b + l < ngrp) ? s[b + l] * gacc[b + l] : 0.0f;
      for (int off = 16; off >= 1; off >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ off];
        memcpy(v, t, sizeof v);
      }
      acc = acc + v[0];
    }
  } else {
    for (int g = 0; g < ngrp; ++g) acc = fmaf(s[g], gacc[g], acc);
  }
  return acc;
}

/* Mode 3: one row of the non-ACCS gemmseg2 arm. */
static float prescaled_row(const uint16_t* crow, const float* cbf, const uint16_t* srow, const float* xs,
                           int NSUB, int D, int G) {
  float acc = 0.0f;
  for (int j = 0; j < NSUB; ++j)
    for (int u = 0; u < D; ++u) {
      const int k = j * D + u;
      const float w = h2f(f2h(cbf[(int64_t)crow[j] * D + u] * h2f(srow[k / G])));
      acc = acc + xs[k] * w;
    }
  return acc;
}

/* Fused expert decode: y32[p, r] = pre-rounding accumulator of pair p, row r.
 *   codes  [E, OUT, NSUB] uint16 (already unpacked)
 *   cb     [K, D] fp16 bits;  scales [E, OUT, NGRP] fp16 bits
 *   xh     [T, IN] fp16 bits (the host cast of vq_switch.py:5301-5308)
 *   idx    [N] expert of each pair; pair p reads token p / krep (xkrep rewrite,
 *          vq_switch.py:4438-4451)
 * The output rounding (fp16 then the caller's dtype, vq_switch.py:5423) is
 * applied by the caller. */
void orc_switch_fused(const uint16_t* codes, const uint16_t* cb, const uint16_t* scales,
                      int E, int OUT, int IN, int D, int G, int K,
                      const uint16_t* xh, int T, const uint32_t* idx, int N, int krep,
                      int mode, float* y32) {
  const int NSUB = IN / D, NGRP = IN / G, SPG = G / D;
  float* cbf = (float*)malloc((size_t)K * D * sizeof(float));
  for (int64_t i = 0; i < (int64_t)K * D; ++i) cbf[i] = h2f(cb[i]);
  float* xf = (float*)malloc((size_t)T * IN * sizeof(float));
  for (int64_t i = 0; i < (int64_t)T * IN; ++i) xf[i] = h2f(xh[i]);
  (void)E;
#pragma omp parallel
  {
    float* gacc = (float*)malloc((size_t)NGRP * sizeof(float));
    float* sv = (float*)malloc((size_t)NGRP * sizeof(float));
#pragma omp for collapse(2) schedule(static)
    for (int p = 0; p < N; ++p)
      for (int r = 0; r < OUT; ++r) {
        const int e = (int)idx[p];
        const float* xs = xf + (int64_t)(p / krep) * IN;
        const uint16_t* crow = codes + ((int64_t)e * OUT + r) * NSUB;
        const uint16_t* srow = scales + ((int64_t)e * OUT + r) * NGRP;
        if (mode == 3) {
          y32[(int64_t)p * OUT + r] = prescaled_row(crow, cbf, srow, xs, NSUB, D, G);
          continue;
        }
        for (int g = 0; g < NGRP; ++g) {
          gacc[g] = group_partial(crow, cbf, xs, (int64_t)g * SPG, SPG, D);
          sv[g] = h2f(srow[g]);
        }
        y32[(int64_t)p * OUT + r] = reduce_groups(sv, gacc, NGRP, mode);
      }
    free(gacc); free(sv);
  }
  free(cbf); free(xf);
}

/* Dense _decode_matmul (vq_dense.py:267-312): W16[o,k] = fp16(cb[c]*s) with one
 * RNE rounding of the exact fp32 product (the fp16 elementwise multiply of
 * vq_dense.py:136), then W in x's dtype (wbf16=1: bf16(W16), the
 * `.astype(xf.dtype)` of vq_dense.py:294), then y32 = sum_k x*W in fp32,
 * ascending k (the GEMM's order is MLX's: UNPINNED).
 *   x [N, IN] float values already in the input dtype. */
void orc_dense_decode_matmul(const uint16_t* codes, const uint16_t* cb, const uint16_t* scales,
                             int OUT, int IN, int D, int G, const float* x, int N, int wbf16, float* y32) {
  const int NSUB = IN / D, NGRP = IN / G;
#pragma omp parallel
  {
    float* w = (float*)malloc((size_t)IN * sizeof(float));
#pragma omp for schedule(static)
    for (int r = 0; r < OUT; ++r) {
      const uint16_t* crow = codes + (int64_t)r * NSUB;
      for (int j = 0; j < NSUB; ++j)
        for (int u = 0; u < D; ++u) {
          const int k = j * D + u;
          const float s = h2f(scales[(int64_t)r * NGRP + k / G]);
          const uint16_t w16 = f2h(h2f(cb[(int64_t)crow[j] * D + u]) * s);
          w[k] = wbf16 ? bf2f(f2bf(h2f(w16))) : h2f(w16);
        }
      for (int n = 0; n < N; ++n) {
        const float* xr = x + (int64_t)n * IN;
        float acc = 0.0f;
        for (int k = 0; k < IN; ++k) acc = acc + xr[k] * w[k];
        y32[(int64_t)n * OUT + r] = acc;
      }
    }
    free(w);
  }
  (void)NGRP;
}

/* float64 exact reference (score/kernel_truth_moe.py:37-50,
 * score/kernel_truth.py:18-24): W64 = cb64[c]*s64, y = x64 @ W64^T, with x
 * given as the already-rounded input values.  Pair p reads token p/krep. */
void orc_exact_f64(const uint16_t* codes, const uint16_t* cb, const uint16_t* scales,
                   int E, int OUT, int IN, int D, int G,
                   const float* x, int T, const uint32_t* idx, int N, int krep, double* y) {
  const int NSUB = IN / D, NGRP = IN / G;
  (void)E; (void)T;
#pragma omp parallel for collapse(2) schedule(static)
  for (int p = 0; p < N; ++p)
    for (int r = 0; r < OUT; ++r) {
      const int e = idx ? (int)idx[p] : 0;
      const float* xr = x + (int64_t)(p / krep) * IN;
      const uint16_t* crow = codes + ((int64_t)e * OUT + r) * NSUB;
      const uint16_t* srow = scales + ((int64_t)e * OUT + r) * NGRP;
      double acc = 0.0;
      for (int j = 0; j < NSUB; ++j)
        for (int u = 0; u < D; ++u) {
          const int k = j * D + u;
          acc += (double)h2f(cb[(int64_t)crow[j] * D + u]) * (double)h2f(srow[k / G]) * (double)xr[k];
        }
      y[(int64_t)p * OUT + r] = acc;
    }
}

/* The same fused decode reading PACKED codes [E, OUT, WPR] directly: each row
 * is unpacked into a per-thread buffer with the vq_pack reader above and then
 * reduced exactly as orc_switch_fused does (the CPU form of the walk kernel,
 * which reads packed words per row, vq_switch.py:1373-1392). */
void orc_switch_fused_packed(const uint32_t* packed, int bits, const uint16_t* cb, const uint16_t* scales,
                             int E, int OUT, int IN, int D, int G, int K,
                             const uint16_t* xh, int T, const uint32_t* idx, int N, int krep,
                             int mode, float* y32) {
  const int NSUB = IN / D, NGRP = IN / G, SPG = G / D;
  const int64_t WPR = orc_words_per_row(NSUB, bits);
  float* cbf = (float*)malloc((size_t)K * D * sizeof(float));
  for (int64_t i = 0; i < (int64_t)K * D; ++i) cbf[i] = h2f(cb[i]);
  float* xf = (float*)malloc((size_t)T * IN * sizeof(float));
  for (int64_t i = 0; i < (int64_t)T * IN; ++i) xf[i] = h2f(xh[i]);
  (void)E;
#pragma omp parallel
  {
    float* gacc = (float*)malloc((size_t)NGRP * sizeof(float));
    float* sv = (float*)malloc((size_t)NGRP * sizeof(float));
    uint16_t* crow = (uint16_t*)malloc((size_t)NSUB * sizeof(uint16_t));
#pragma omp for collapse(2) schedule(static)
    for (int p = 0; p < N; ++p)
      for (int r = 0; r < OUT; ++r) {
        const int e = (int)idx[p];
        const float* xs = xf + (int64_t)(p / krep) * IN;
        const uint32_t* prow = packed + ((int64_t)e * OUT + r) * WPR;
        for (int j = 0; j < NSUB; ++j) crow[j] = (uint16_t)extract_code(prow, j, bits);
        const uint16_t* srow = scales + ((int64_t)e * OUT + r) * NGRP;
        if (mode == 3) {
          y32[(int64_t)p * OUT + r] = prescaled_row(crow, cbf, srow, xs, NSUB, D, G);
          continue;
        }
        for (int g = 0; g < NGRP; ++g) {
          gacc[g] = group_partial(crow, cbf, xs, (int64_t)g * SPG, SPG, D);
          sv[g] = h2f(srow[g]);
        }
        y32[(int64_t)p * OUT + r] = reduce_groups(sv, gacc, NGRP, mode);
      }
    free(gacc); free(sv); free(crow);
  }
  free(cbf); free(xf);
}
