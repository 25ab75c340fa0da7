// C ABI of libvqb200.so (declared in include/vqb.h): argument validation with
// the reference's error classes, path selection, workspace layout, launches.
#include <atomic>
#include <cstdio>

#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {

// Every geometry rule the reference enforces before it dispatches a kernel:
// explicit D (vq_switch.py:3106-3109), the packed row width
// (:3124-3128), IN % G and G % D (the group/subvector structure of
// vq_pack/fit_moe), the codebook sharding guard (:5285-5296).
vqb_status validate(const vqb_linear_desc* d, LinearGeometry* g) {
  if (!d || !d->codes || !d->codebook || !d->scales) return VQB_NULL_POINTER;
  if (d->row_table && d->num_rows < 0) return VQB_BAD_SHAPE;
  if (d->expected_num_codes > 0 && d->num_codes != d->expected_num_codes) return VQB_CODEBOOK_SHARDED;
  if (d->dim != 2 && d->dim != 4 && d->dim != 8) return VQB_UNSUPPORTED_GEOMETRY;
  if (d->num_experts < 1 || d->out_features < 1 || d->in_features < 1 || d->group_size < 1 || d->num_codes < 1)
    return VQB_BAD_SHAPE;
  if (d->in_features % d->group_size != 0 || d->group_size % d->dim != 0) return VQB_BAD_SHAPE;
  const int nsub = d->in_features / d->dim;
  int bits, row_words;
  if (d->pack_bits > 0) {
    if (d->pack_bits > 16) return VQB_UNSUPPORTED_GEOMETRY;
    if ((int64_t(1) << d->pack_bits) < d->num_codes) return VQB_BAD_SHAPE;
    bits = d->pack_bits;
    row_words = (nsub + 31) / 32 * bits;
    if (d->codes_last_dim > 0 && d->codes_last_dim != row_words) return VQB_BAD_WPR;
  } else {
    if (d->code_bytes != 1 && d->code_bytes != 2) return VQB_UNSUPPORTED_GEOMETRY;
    if (d->code_bytes == 1 && d->num_codes > 256) return VQB_BAD_SHAPE;
    const int64_t row_bytes = int64_t(nsub) * d->code_bytes;
    // unpacked rows are read as 8/16-bit code streams (byte-identical to
    // pack_bits 8/16 rows when whole words; vq_switch.py:2975-2996)
    if (row_bytes % 4 != 0) return VQB_UNSUPPORTED_GEOMETRY;
    if ((reinterpret_cast<uintptr_t>(d->codes) & 3) != 0) return VQB_BAD_ALIGNMENT;
    bits = 8 * d->code_bytes;
    row_words = static_cast<int>(row_bytes / 4);
    if (d->codes_last_dim > 0 && d->codes_last_dim != nsub) return VQB_BAD_SHAPE;
  }
  if ((reinterpret_cast<uintptr_t>(d->codebook) & 15) != 0 || (reinterpret_cast<uintptr_t>(d->scales) & 1) != 0)
    return VQB_BAD_ALIGNMENT;
  if (d->codebook_halves) {
    if (d->dim != 8) return VQB_BAD_SHAPE;
    if ((reinterpret_cast<uintptr_t>(d->codebook_halves) & 15) != 0) return VQB_BAD_ALIGNMENT;
  }
  g->E = d->num_experts;
  g->OUT = d->out_features;
  g->IN = d->in_features;
  g->D = d->dim;
  g->K = d->num_codes;
  g->G = d->group_size;
  g->bits = bits;
  g->row_words = row_words;
  g->codes = d->codes;
  g->codebook = d->codebook;
  g->scales = d->scales;
  g->row_table = d->row_table;
  g->nrows = d->row_table ? static_cast<int64_t>(d->num_rows) : static_cast<int64_t>(g->E) * g->OUT;
  g->codebook_halves = d->codebook_halves;
  return VQB_OK;
}

namespace {
std::atomic<uint64_t> g_launches{0};
thread_local cudaEvent_t t_timer_start = nullptr, t_timer_stop = nullptr;
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {
constexpr int kMaxDeviceIndex = 64;
std::atomic<int> g_dev_sms[kMaxDeviceIndex];
std::atomic<int> g_dev_optin[kMaxDeviceIndex];
}  // namespace

// SM count and opt-in shared memory per block of the current device, read
// once per device index (every GPU of a process may differ).
vqb_status device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return VQB_CUDA_ERROR;
  if (dev < kMaxDeviceIndex) {
    const int s = g_dev_sms[dev].load(std::memory_order_relaxed);
    const int o = g_dev_optin[dev].load(std::memory_order_relaxed);
    if (s > 0 && o > 0) {
      out->sms = s;
      out->smem_optin = o;
      return VQB_OK;
    }
  }
  int s = 0, o = 0;
  if (cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&o, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || s <= 0 || o <= 0)
    return VQB_CUDA_ERROR;
  if (dev < kMaxDeviceIndex) {
    g_dev_sms[dev].store(s, std::memory_order_relaxed);
    g_dev_optin[dev].store(o, std::memory_order_relaxed);
  }
  out->sms = s;
  out->smem_optin = o;
  return VQB_OK;
}

void timer_before(cudaStream_t stream) {
  if (t_timer_start) cudaEventRecord(t_timer_start, stream);
}

void timer_after(cudaStream_t stream) {
  if (t_timer_stop) cudaEventRecord(t_timer_stop, stream);
  t_timer_start = t_timer_stop = nullptr;
}

static bool dtype_ok(int t) { return t == VQB_F16 || t == VQB_BF16 || t == VQB_F32; }


// Workspace: [routing (status block first)][x as 16-bit rows: the token rows
// for the decode kernel's B operand, or all pairs' rows in expert order for
// the grouped GEMM -- whichever is larger]
size_t x_region_bytes(int N, int E, int64_t T, int IN, int OUT, int K, int D) {
  const size_t a = mma_x16_bytes(T, IN), b = tc_prefill_x_bytes(N, IN, K, D, E, OUT);
  return a > b ? a : b;
}
size_t linear_workspace_bytes(int N, int E, int64_t T, int IN, int OUT, int K, int D) {
  return route_workspace_bytes(N, E, kDecodeMaxPairs, row_tiles_128(OUT)) + x_region_bytes(N, E, T, IN, OUT, K, D);
}

// Shared body of the switch and dense entry points once shapes are valid.
vqb_status run_linear(const LinearGeometry& geo, const void* x, int x_dtype, int n_tokens,
                             const uint32_t* indices, int krep, int N, void* y, int y_dtype, void* workspace,
                             const vqb_options* opts, bool narrow_x_f16, bool round_f16_first, int wround,
                             bool large, cudaStream_t stream) {
  // the routing kernel clears the status block itself; the per-pair paths, which route nothing, clear it here
  RouteWorkspace rw = carve_route_workspace(workspace, N, geo.E, row_tiles_128(geo.OUT));
  const int ks = opts ? opts->k_split : 0;
  const int variant = opts ? opts->decode_variant : 0;
  uint16_t* xbuf = reinterpret_cast<uint16_t*>(static_cast<char*>(workspace) +
                                               route_workspace_bytes(N, geo.E, kDecodeMaxPairs,
                                                                     row_tiles_128(geo.OUT)));
  if (large && variant == 0 && tc_prefill_supported(geo) && x_dtype != VQB_F32 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // grouped tcgen05 GEMM: tiles of up to 128 of one expert's tokens; routing
    // tables and gathered x reused from the previous call when the caller says so
    const int reuse = opts ? opts->reuse : 0;
    if (!(reuse & (VQB_REUSE_ROUTING | VQB_REUSE_X))) {
      vqb_status st = launch_route_small(indices, N, geo.E, kPrefillTileTokens, rw, stream);
      if (st != VQB_OK) return st;
    }
    return launch_prefill_tc(geo, x, x_dtype, krep, rw, N, xbuf, y, y_dtype, round_f16_first,
                             /*bf16_operands=*/wround == 1, /*gather_x=*/!(reuse & VQB_REUSE_X), rw.meta, stream);
  }
  if (variant == 1 || !mma_decode_supported(geo, wround, x_dtype)) {
    if (cudaMemsetAsync(rw.meta, 0, sizeof(int) * 4, stream) != cudaSuccess) return VQB_CUDA_ERROR;
  }
  if (variant == 1) {
    // one pair per CTA, the reference walk order (kept for exact-order checks)
    return launch_decode(geo, x, x_dtype, n_tokens, indices, N, krep, y, y_dtype, narrow_x_f16, round_f16_first,
                         wround, ks, rw.meta + 1, stream);
  }
  if (!mma_decode_supported(geo, wround, x_dtype)) {
    // geometries outside the tensor-core kernel (group not a multiple of 64,
    // IN not a multiple of 512, unaligned rows) take the per-pair kernel
    return launch_decode(geo, x, x_dtype, n_tokens, indices, N, krep, y, y_dtype, narrow_x_f16, round_f16_first,
                         wround, ks > 8 ? 8 : ks, rw.meta + 1, stream);
  }
  const int pmax = decode_pairs_per_chunk(N, geo.E, geo.K, geo.D, geo.IN, opts ? opts->pairs_per_chunk : 0);
  vqb_status st = launch_route_small(indices, N, geo.E, pmax, rw, stream);
  if (st != VQB_OK) return st;
  GroupedDecodeArgs a{};
  a.x = x;
  a.x_dtype = x_dtype;
  a.krep = krep;
  a.route = &rw;
  a.N = N;
  a.y = y;
  a.y_dtype = y_dtype;
  a.narrow_x_f16 = narrow_x_f16;
  a.round_f16_first = round_f16_first;
  a.wround = wround;
  a.ks = ks;
  const int stage = opts ? opts->stage_codebook : 0;
  a.stage_codebook = stage == 1 ? 1 : (stage == 2 ? 0 : (stage == 3 ? 3 : -1));
  a.pmax = pmax;
  return launch_decode_mma(geo, a, xbuf, n_tokens, stream);
}

}  // namespace vqb

using namespace vqb;

extern "C" {

const char* vqb_version(void) { return "vqb200 0.1 sm_100a"; }

uint64_t vqb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

vqb_status vqb_time_next_kernel(void* start_event, void* stop_event) {
  if ((start_event == nullptr) != (stop_event == nullptr)) return VQB_NULL_POINTER;
  t_timer_start = static_cast<cudaEvent_t>(start_event);
  t_timer_stop = static_cast<cudaEvent_t>(stop_event);
  return VQB_OK;
}

const char* vqb_status_string(vqb_status s) {
  switch (s) {
    case VQB_OK: return "ok";
    case VQB_BAD_SHAPE: return "inconsistent tensor shapes for a VQ projection";
    case VQB_BAD_WPR: return "packed codes row width does not match ceil(NSUB/32)*BITS";
    case VQB_UNSUPPORTED_GEOMETRY: return "unsupported VQ geometry (D must be 2, 4 or 8; BITS <= 16)";
    case VQB_CODEBOOK_SHARDED: return "VQ codebook was sharded: K differs from the K the module was built with";
    case VQB_CUDA_ERROR: return "CUDA launch or runtime error";
    case VQB_TIMEOUT: return "a bounded device wait timed out";
    case VQB_BAD_ROUTING: return "an expert index was out of range";
    case VQB_WORKSPACE_TOO_SMALL: return "workspace too small";
    case VQB_BAD_ALIGNMENT: return "misaligned tensor pointer";
    case VQB_NULL_POINTER: return "null tensor pointer";
  }
  return "unknown status";
}

vqb_status vqb_unpack(const uint32_t* packed, int64_t rows, int64_t wpr, int32_t nsub, int32_t bits, uint16_t* out,
                      vqb_stream_t stream) {
  if (!packed || !out) return VQB_NULL_POINTER;
  if (bits < 1 || bits > 16 || nsub < 0 || rows < 0) return VQB_UNSUPPORTED_GEOMETRY;
  if (wpr != (int64_t(nsub) + 31) / 32 * bits) return VQB_BAD_WPR;
  return launch_unpack(packed, rows, wpr, nsub, bits, out, reinterpret_cast<cudaStream_t>(stream));
}

size_t vqb_switch_workspace_size(const vqb_linear_desc* desc, int32_t n_tokens, int32_t top_k,
                                 const vqb_options* opts) {
  (void)opts;
  const int64_t T = n_tokens > 0 ? n_tokens : 0;
  const int64_t N = T * (top_k > 0 ? top_k : 1);
  const int E = desc ? (desc->num_experts > 0 ? desc->num_experts : 1) : 1;
  const int IN = desc ? (desc->in_features > 0 ? desc->in_features : 0) : 0;
  const int OUT = desc ? (desc->out_features > 0 ? desc->out_features : 0) : 0;
  const int K = desc ? (desc->num_codes > 0 ? desc->num_codes : 0) : 0;
  const int D = desc ? desc->dim : 0;
  return linear_workspace_bytes(static_cast<int>(N), E, T, IN, OUT, K, D);
}

// The switch entry's kernel family for N pairs (the GEMM or the decode
// kernel), before the per-call fallbacks for fp32 or unaligned x.
static bool switch_uses_gemm(const LinearGeometry& geo, int N, const vqb_options* opts) {
  // Path: the reference runs the fused small-N kernel up to VQ_FUSED_MAX_N =
  // 512 pairs and the grouped GEMM above it (vq_switch.py:45, :5313-5315).  The
  // grouped GEMM decodes every routed expert's tile with a fixed cost per
  // tile group (codebook reload, accumulator drain) that the K extent
  // amortises, so on a B200 it pays once pairs * IN exceed ~4608 per expert as
  // well.  A d8 codebook too large for shared memory changes the balance: the
  // decode kernel then reads part of the codebook through L1/L2 while the
  // GEMM keeps half of every entry resident per pass (and splits K over CTAs
  // when a call has few tiles), and the GEMM wins at every batch.  Measured
  // (512 experts, d8/K16384, uniform routing, device time per call, us,
  // GEMM vs decode):
  //   1024 x 4096 gate:  10 pairs 35.7 vs 40.1;  20: 58.7 vs 61.6;  30: 61.5 vs 84.3;
  //                      1.25 pairs/expert 500 vs 790;  10: 680 vs 2810
  //   4096 x 1024 down:  10 pairs 36.5 vs 38.0;  20: 52.6 vs 57.6;  30: 68.1 vs 78.4;
  //                      1.25 pairs/expert 570 vs 710;  10: 820 vs 2620
  constexpr int64_t kGemmPairInPerExpert = 4608;
  constexpr int kDsplitMinPairs = 0;
  const int path = opts ? opts->path : VQB_PATH_AUTO;
  const int max_fused = (opts && opts->max_fused_pairs > 0) ? opts->max_fused_pairs : 512;
  const bool dsplit_gemm = N > kDsplitMinPairs && !(opts && opts->max_fused_pairs > 0) && tc_prefill_dsplit(geo);
  return path == VQB_PATH_PREFILL ||
                     (path == VQB_PATH_AUTO &&
                      (dsplit_gemm || (N > max_fused && static_cast<int64_t>(N) * geo.IN > kGemmPairInPerExpert * geo.E)));
}

vqb_status vqb_switch_forward(const vqb_linear_desc* desc, const void* x, vqb_dtype x_dtype, int32_t n_tokens,
                              const uint32_t* indices, int32_t top_k, void* y, vqb_dtype y_dtype, void* workspace,
                              size_t workspace_bytes, const vqb_options* opts, vqb_stream_t stream) {
  LinearGeometry geo;
  vqb_status st = validate(desc, &geo);
  if (st != VQB_OK) return st;
  if (n_tokens < 0 || top_k < 1) return VQB_BAD_SHAPE;
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return VQB_BAD_SHAPE;
  const int64_t N64 = int64_t(n_tokens) * top_k;
  if (N64 > 0x7fffffff) return VQB_BAD_SHAPE;
  const int N = static_cast<int>(N64);
  if (N == 0) return VQB_OK;
  if (!x || !indices || !y) return VQB_NULL_POINTER;
  if (workspace_bytes < vqb_switch_workspace_size(desc, n_tokens, top_k, opts)) return VQB_WORKSPACE_TOO_SMALL;
  if (!workspace) return VQB_NULL_POINTER;
  const bool large = switch_uses_gemm(geo, N, opts);
  // MoE numerics: x narrowed to fp16, fp32 accumulation, fp16 output rounding
  // then the caller's dtype (vq_switch.py:5301-5308, :5423).
  return run_linear(geo, x, x_dtype, n_tokens, indices, top_k, N, y, y_dtype, workspace, opts,
                    /*narrow_x_f16=*/true, /*round_f16_first=*/true, /*wround=*/0, large,
                    reinterpret_cast<cudaStream_t>(stream));
}

int32_t vqb_switch_path(const vqb_linear_desc* desc, int32_t n_tokens, int32_t top_k, const vqb_options* opts) {
  LinearGeometry geo;
  const vqb_status st = validate(desc, &geo);
  if (st != VQB_OK) return -static_cast<int32_t>(st);
  if (n_tokens < 0 || top_k < 1 || int64_t(n_tokens) * top_k > 0x7fffffff) return -static_cast<int32_t>(VQB_BAD_SHAPE);
  const int N = n_tokens * top_k;
  return switch_uses_gemm(geo, N, opts) && tc_prefill_supported(geo) ? VQB_PATH_PREFILL : VQB_PATH_DECODE;
}

size_t vqb_dense_workspace_size(const vqb_linear_desc* desc, int64_t n_rows, const vqb_options* opts) {
  (void)opts;
  const int n = static_cast<int>(n_rows > 0 ? (n_rows > 0x7fffffff ? 0x7fffffff : n_rows) : 0);
  const int IN = desc ? (desc->in_features > 0 ? desc->in_features : 0) : 0;
  const int OUT = desc ? (desc->out_features > 0 ? desc->out_features : 0) : 0;
  const int K = desc ? (desc->num_codes > 0 ? desc->num_codes : 0) : 0;
  const int D = desc ? desc->dim : 0;
  return linear_workspace_bytes(n, 1, n, IN, OUT, K, D);
}

vqb_status vqb_dense_forward(const vqb_linear_desc* desc, const void* x, vqb_dtype x_dtype, int64_t n_rows, void* y,
                             vqb_dtype y_dtype, void* workspace, size_t workspace_bytes, const vqb_options* opts,
                             vqb_stream_t stream) {
  LinearGeometry geo;
  vqb_status st = validate(desc, &geo);
  if (st != VQB_OK) return st;
  if (geo.E != 1) return VQB_BAD_SHAPE;
  if (geo.row_table) return VQB_UNSUPPORTED_GEOMETRY;  // SKIPZERO is a switch-layer format (vq_switch.py:5205)
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return VQB_BAD_SHAPE;
  if (n_rows < 0 || n_rows > 0x7fffffff) return VQB_BAD_SHAPE;
  if (n_rows == 0) return VQB_OK;
  if (!x || !y) return VQB_NULL_POINTER;
  if (workspace_bytes < vqb_dense_workspace_size(desc, n_rows, opts)) return VQB_WORKSPACE_TOO_SMALL;
  if (!workspace) return VQB_NULL_POINTER;
  const int path = opts ? opts->path : VQB_PATH_AUTO;
  // Which reference path serves this call (vq_dense.py:401-441): the fused
  // dense kernel only for d2/d4 at N <= the per-geometry cutoff
  // (_fused_max_n, vq_dense.py:94-102: unpacked 12, packed d2 72, packed d4
  // 32); everything else, and every d8 layer, is _decode_matmul.
  bool fused;
  if (path == VQB_PATH_DECODE) fused = true;
  else if (path == VQB_PATH_PREFILL) fused = false;
  else {
    int maxn = desc->pack_bits == 0 ? 12 : (geo.D == 2 ? 72 : (geo.D == 4 ? 32 : 0));
    if (opts && opts->max_fused_pairs > 0) maxn = opts->max_fused_pairs;
    fused = geo.D != 8 && n_rows <= maxn;
  }
  // fused numerics: x narrowed to fp16 in-kernel, group partials, y stored
  // directly in the output dtype (vq_switch.py:2319-2327).
  // _decode_matmul numerics: W = fp16(cb*s) in x's dtype, y = x @ W^T.
  if (!fused && x_dtype == VQB_F32) return VQB_UNSUPPORTED_GEOMETRY;
  const int wround = fused ? 0 : (x_dtype == VQB_BF16 ? 1 : 2);
  const int n = static_cast<int>(n_rows);
  // the grouped GEMM once the decode kernel would need more than one pass of
  // 16 tokens over the weights, and at every N for a d8 codebook too large for
  // shared memory (dimension-split passes; split-K fills the GPU when the
  // layer has few row tiles).  Measured on B200, d8/K16384, us, GEMM vs
  // decode: 17408 x 5120 at N = 1 47 vs 57, N = 4 48 vs 59; 5120 x 17408 at
  // N = 4 120 vs 221 before split-K.
  // The fused arm's calls above 8 rows go to the GEMM too, with its fp16
  // operands (x narrowed to fp16, W = fp16(cb*s), fp32 accumulation): d2/K256
  // 5120 x 5120 at N = 16 30 vs 73 us, N = 32 31 vs 118 us.
  const bool large = path == VQB_PATH_PREFILL || (!fused && (n > 16 || tc_prefill_dsplit(geo))) ||
                     (fused && path == VQB_PATH_AUTO && n > 8);
  // a d2 codebook of <= 256 entries at <= 8 rows: the small-codebook kernel
  // (the codebook replicated per lane in shared memory, one launch, no routing
  // step, split-K reduced inside thread-block clusters)
  if (fused && path == VQB_PATH_AUTO && !(opts && (opts->decode_variant != 0 || opts->k_split != 0)) &&
      (reinterpret_cast<uintptr_t>(workspace) & 3) == 0 && dense_lut_eligible(geo, x, x_dtype, n))
    return launch_dense_lut(geo, x, x_dtype, n, y, y_dtype, static_cast<int*>(workspace),
                            reinterpret_cast<cudaStream_t>(stream));
  // a d8 codebook of <= 4096 entries at <= 8 rows (C1's matvec): the same
  // structure with the whole codebook resident, _decode_matmul arithmetic
  if (!fused && path == VQB_PATH_AUTO && n <= 8 && !(opts && (opts->decode_variant != 0 || opts->k_split != 0)) &&
      (reinterpret_cast<uintptr_t>(workspace) & 3) == 0 && dense_lut8_eligible(geo, x, x_dtype, n))
    return launch_dense_lut8(geo, x, x_dtype, n, y, y_dtype, static_cast<int*>(workspace),
                             reinterpret_cast<cudaStream_t>(stream));
  return run_linear(geo, x, x_dtype, n, nullptr, 1, n, y, y_dtype, workspace, opts, /*narrow_x_f16=*/fused,
                    /*round_f16_first=*/false, wround, large, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
