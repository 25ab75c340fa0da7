// Internal (non-ABI) declarations shared by the kernel translation units.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda_runtime.h>

#include "../../include/vqb.h"

namespace vqb {

// Validated geometry of one VQ projection.
struct LinearGeometry {
  int E, OUT, IN, D, K, G, bits;
  int row_words;  // 32-bit words per code row (packed WPR, or NSUB*bytes/4 unpacked)
  const void* codes;
  const void* codebook;
  const void* scales;
  const int32_t* row_table;  // SKIPZERO [E, OUT] -> compact row, -1 dead; nullptr = plain layout
  int64_t nrows;             // rows of codes / scales (E * OUT, or the compact live-row count)
  const void* codebook_halves;  // d8: caller-built [2][K][4] halves, nullptr = derived per call
};

vqb_status validate(const vqb_linear_desc* d, LinearGeometry* out);

// Pairs grouped by expert (vq_route.cu).
struct RouteWorkspace {
  int* meta;      // [0] chunk count, [1] error flag
  int* counts;    // [E]
  int* offsets;   // [E+1]
  int* sorted;    // [N] pair ids grouped by expert
  int4* chunks;   // (expert, first sorted slot, pairs, 0)
  int* tile_base; // [E][row tiles of 128]: first compact row of each tile (SKIPZERO grouped GEMM)
};

// row_tiles: 128-row tiles per expert (room for the SKIPZERO tile bases)
size_t route_workspace_bytes(int N, int E, int max_pairs, int row_tiles);
RouteWorkspace carve_route_workspace(void* base, int N, int E, int row_tiles);
inline int row_tiles_128(int OUT) { return (OUT + 127) / 128; }
vqb_status launch_route_small(const uint32_t* idx, int N, int E, int max_pairs, const RouteWorkspace& ws,
                              cudaStream_t stream);

// One pair per CTA, CUDA-core walk in the reference's order (vq_decode.cu).
vqb_status launch_decode(const LinearGeometry& geo, const void* x, int x_dtype, int T, const uint32_t* idx,
                         int N, int krep, void* y, int y_dtype, bool narrow_x_f16, bool round_f16_first,
                         int wround, int ks, int* err, cudaStream_t stream);

vqb_status launch_unpack(const uint32_t* packed, int64_t rows, int64_t wpr, int nsub, int bits, uint16_t* out,
                         cudaStream_t stream);

constexpr uint32_t kSkipExpert = 0xFFFFFFFFu;  // expert index of a pair to leave out (no output row)
constexpr int kDecodeMaxPairs = 16;  // route workspace sizing bound (chunks <= N + E either way)

// Expert-grouped decode on the tensor cores (vq_decode_mma.cu).
struct GroupedDecodeArgs {
  const void* x;          // token rows [T, IN] (x_dtype)
  int x_dtype;
  int krep;               // pair p reads token p / krep
  const RouteWorkspace* route;
  int N;                  // pairs
  void* y;                // [N, OUT]
  int y_dtype;
  bool narrow_x_f16;
  bool round_f16_first;
  int wround;
  int ks;                 // 0 = auto
  int stage_codebook;     // -1 auto, 0 none, 1 prefix only (no split), 3 split across a CTA pair
  int pmax;               // tokens per chunk the route step used (<= 16)
};
bool mma_decode_supported(const LinearGeometry& geo, int wround, int x_dtype);
size_t mma_x16_bytes(int64_t T, int IN);
vqb_status launch_decode_mma(const LinearGeometry& geo, const GroupedDecodeArgs& a, uint16_t* x16, int T,
                             cudaStream_t stream);

// Small-codebook dense decode (vq_dense_lut.cu): d2, K <= 256, 8-bit codes,
// group 64, IN a multiple of 512, up to 8 rows, fp16/bf16 x; `status` is the
// workspace status block (int32 [1] = VQB_TIMEOUT after an expired wait, else 0).
bool dense_lut_geometry(const LinearGeometry& g);
bool dense_lut_eligible(const LinearGeometry& g, const void* x, int x_dtype, int T);
vqb_status launch_dense_lut(const LinearGeometry& g, const void* x, int x_dtype, int T, void* y, int y_dtype,
                            int* status, cudaStream_t stream);
// The d8 variant (_decode_matmul arithmetic): K <= 4096, even bits, group 64,
// IN a multiple of 512, up to 8 rows, fp16/bf16 x.
bool dense_lut8_eligible(const LinearGeometry& g, const void* x, int x_dtype, int T);
vqb_status launch_dense_lut8(const LinearGeometry& g, const void* x, int x_dtype, int T, void* y, int y_dtype,
                             int* status, cudaStream_t stream);

// Grouped tcgen05 GEMM for large token counts (vq_prefill_tc.cu).
bool tc_prefill_supported(const LinearGeometry& geo);
bool tc_prefill_dsplit(const LinearGeometry& geo);  // the GEMM would run dimension-split passes
size_t tc_prefill_x_bytes(int64_t N, int IN, int K, int D, int E, int OUT);  // gathered x, d8 codebook halves, split-K partials
int tc_prefill_ksplit(int64_t N, int E, int OUT, int IN);
vqb_status launch_prefill_tc(const LinearGeometry& geo, const void* x, int x_dtype, int krep, const RouteWorkspace& rw,
                             int N, uint16_t* xs, void* y, int y_dtype, bool round_f16_first, bool bf16_operands, bool gather_x,
                             int* status, cudaStream_t stream);
constexpr int kPrefillTileTokens = 128;

// Launch `kern` as a programmatic dependent of the kernel before it on the
// stream: its CTAs may start while that kernel finishes, so the kernel must
// execute griddepcontrol.wait (pdl_wait) before it reads or writes memory the
// previous kernel touches; griddepcontrol.launch_dependents (pdl_trigger) lets
// the kernel after it do the same.  Both are no-ops in a kernel launched
// without the attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Launch accounting and the one-shot kernel timer (vqb_api.cu): every kernel
// launch of the library calls note_launch(); the dominant kernel of a call
// (the decode or grouped-GEMM kernel) is bracketed by timer_before/after,
// which record the events armed by vqb_time_next_kernel on its stream.
void note_launch();

// Attributes of the current device (cached per device index).
struct DeviceInfo {
  int sms;
  int smem_optin;
};
vqb_status device_info(DeviceInfo* out);
void timer_before(cudaStream_t stream);
void timer_after(cudaStream_t stream);

// Workspace layout and the shared body of the switch / dense entry points (vqb_api.cu).
size_t linear_workspace_bytes(int N, int E, int64_t T, int IN, int OUT, int K, int D);
vqb_status run_linear(const LinearGeometry& geo, const void* x, int x_dtype, int n_tokens, const uint32_t* indices,
                      int krep, int N, void* y, int y_dtype, void* workspace, const vqb_options* opts,
                      bool narrow_x_f16, bool round_f16_first, int wround, bool large, cudaStream_t stream);

// Tokens that share one pass over an expert's rows (one MMA n-tile holds 8).
inline int decode_pairs_per_chunk(int N, int E, int K, int D, int IN, int override_pairs) {
  int pm;
  if (override_pairs == 1 || override_pairs == 2 || override_pairs == 4 || override_pairs == 8 ||
      override_pairs == 16)
    pm = override_pairs;
  else if (E == 1) pm = N > 8 ? 16 : 8;
  else if (N <= E) pm = 2;
  else if (N <= 4 * static_cast<int64_t>(E)) pm = 4;
  else pm = 8;
  // a codebook that does not fit shared memory keeps the x staging small so
  // more of the table stays resident
  if (E > 1 && static_cast<int64_t>(K) * D * 2 > 160 * 1024 && pm > 4 && override_pairs == 0) pm = 4;
  const int64_t fit = (64 * 1024) / ((static_cast<int64_t>(IN) + 8) * 2);
  if (pm > fit) pm = fit < 1 ? 1 : static_cast<int>(fit >= 16 ? 16 : (fit >= 8 ? 8 : (fit >= 4 ? 4 : (fit >= 2 ? 2 : 1))));
  return pm;
}

}  // namespace vqb
