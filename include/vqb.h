/*
 * vqb.h -- C ABI of the B200 VQ expert runtime (libvqb200.so).
 *
 * The drop-in boundary for the VQLab runtime hot path: the fused
 * codebook-decode matmul behind `VQSwitchLinear` (routed MoE experts) and
 * `VQLinear` (dense projections), reading the vq_pack v1 packed layout.
 *
 * Every pointer is a DEVICE pointer owned by the caller.  The compute entry
 * points (vqb_unpack, vqb_codebook_halves, vqb_switch_forward[_static],
 * vqb_dense_forward, the MoE elementwise calls, vqb_moe_block_forward and
 * vqb_ep_dispatch / combine / reduce) are asynchronous on the given stream and
 * allocate nothing; calls
 * that need scratch memory take a caller-supplied workspace whose size the
 * matching *_workspace_size function returns.  Only the expert-parallel set-up
 * calls (vqb_ep_region_alloc / _free, vqb_ep_ipc_open / _close) allocate,
 * map or free device memory, synchronously.  No torch types cross this
 * boundary.
 *
 * Tensor formats (identical to the reference's safetensors tensors):
 *   codes     packed (pack_bits > 0): uint32 [E, OUT, WPR], WPR = ceil(NSUB/32)*BITS,
 *             code j of a row at bits [j*BITS, (j+1)*BITS) of the row's
 *             little-endian word stream (src/vqlab/runtime/vq_pack.py:11-27)
 *             unpacked (pack_bits == 0): uint8 / uint16 [E, OUT, NSUB]
 *   codebook  fp16 [K, D], D in {2, 4, 8}
 *   scales    fp16 [E, OUT, IN/G]  (one scale per output row and group of G inputs)
 *   x         bf16 / fp16 [T, IN]  (token rows)
 *   indices   uint32 [T, top_k]    (expert of each (token, slot) pair)
 *   y         [T*top_k, OUT] for the switch, [N, OUT] for dense
 */
#ifndef VQB_H_
#define VQB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* vqb_stream_t;

/* Error convention.  The reference raises on every unsupported geometry and
 * never falls through to a wrong-memory read (vq_switch.py:3016-3019,
 * :3106-3109, :3124-3128, :3347-3354, :5285-5296); each raise maps to one
 * status here. */
typedef enum vqb_status {
  VQB_OK = 0,
  VQB_BAD_SHAPE = 1,              /* inconsistent sizes (IN % G, G % D, ...) */
  VQB_BAD_WPR = 2,                /* codes row width != ceil(NSUB/32)*BITS (vq_switch.py:3124-3128) */
  VQB_UNSUPPORTED_GEOMETRY = 3,   /* D not in {2,4,8}, BITS > 16, ... (vq_switch.py:3106-3109) */
  VQB_CODEBOOK_SHARDED = 4,       /* K differs from the K the module was built with (vq_switch.py:5285-5296) */
  VQB_CUDA_ERROR = 5,             /* a launch or runtime call failed */
  VQB_TIMEOUT = 6,                /* a bounded device wait gave up */
  VQB_BAD_ROUTING = 7,            /* an expert index >= E was seen on the device */
  VQB_WORKSPACE_TOO_SMALL = 8,
  VQB_BAD_ALIGNMENT = 9,
  VQB_NULL_POINTER = 10
} vqb_status;

typedef enum vqb_dtype { VQB_F16 = 0, VQB_BF16 = 1, VQB_F32 = 2 } vqb_dtype;

/* Kernel path selection.  AUTO for vqb_switch_forward: the fused small-N
 * kernel up to VQ_FUSED_MAX_N = 512 pairs as in the reference
 * (vq_switch.py:45, :5313); above it the grouped prefill GEMM once also
 * pairs * in_features > 4608 * num_experts (its fixed cost per expert tile
 * needs that much work to pay on a B200), else still the decode kernel.  A d8
 * codebook too large for shared memory (the GEMM's dimension-split passes)
 * sends every call to the GEMM.  AUTO for
 * vqb_dense_forward follows the reference's dense cutoffs. */
typedef enum vqb_path { VQB_PATH_AUTO = 0, VQB_PATH_DECODE = 1, VQB_PATH_PREFILL = 2 } vqb_path;

/* One VQ-coded projection: a VQSwitchLinear (E experts) or a VQLinear (E = 1).
 * Mirrors the module attributes of vq_switch.py:5198-5282 / vq_dense.py:315-344. */
typedef struct vqb_linear_desc {
  int32_t num_experts;        /* E (1 for a dense VQLinear) */
  int32_t out_features;       /* OUT */
  int32_t in_features;        /* IN */
  int32_t dim;                /* D, codebook entry width */
  int32_t num_codes;          /* K, codebook rows */
  int32_t group_size;         /* G */
  int32_t pack_bits;          /* BITS; 0 = unpacked codes */
  int32_t code_bytes;         /* unpacked only: 1 (uint8) or 2 (uint16) */
  int32_t expected_num_codes; /* K at construction (sharding guard); 0 = no check */
  int32_t codes_last_dim;     /* caller's codes.shape[-1] (WPR check, vq_switch.py:3124-3128); 0 = no check */
  const void* codes;
  const void* codebook;
  const void* scales;
  const int32_t* row_table;   /* SKIPZERO (vq_switch.py:5205-5216): int32 [E, OUT] mapping (expert, out
                                 row) to a compact row of codes / scales, -1 = dead; NULL = the plain
                                 [E, OUT, ...] layout.  Dead rows read no bytes and write +0. */
  int32_t num_rows;           /* with row_table: rows of the compact codes [num_rows, WPR] and scales
                                 [num_rows, IN/G]; entries >= num_rows are treated as dead */
  const void* codebook_halves; /* optional, D = 8 only: the codebook's two dimension halves, fp16
                                 [2][K][4] (vqb_codebook_halves), 16-byte aligned; NULL = a call on
                                 the grouped GEMM derives them itself (one more kernel per call) */
} vqb_linear_desc;

/* Optional knobs; pass NULL for defaults. */
typedef struct vqb_options {
  int32_t path;               /* vqb_path */
  int32_t k_split;            /* decode kernel K-slices per row (0 = auto; grouped kernel 1..16, per-pair 1..8) */
  int32_t max_fused_pairs;    /* AUTO cutoff in pairs (0 = 512) */
  int32_t decode_variant;     /* 0 = expert-grouped persistent kernel, 1 = one pair per CTA (reference order) */
  int32_t stage_codebook;     /* grouped kernel: 0 = auto, 1 = shared-memory prefix (no pair split),
                                 2 = none, 3 = split the codebook across a CTA pair */
  int32_t pairs_per_chunk;    /* grouped kernel: tokens sharing one lookup pass (0 = auto, else 1, 2 or 4) */
  int32_t reuse;              /* VQB_REUSE_* flags: the workspace already holds this call's routing tables
                                 (and gathered x) from the previous call on the same stream; honoured on the
                                 grouped-GEMM path only (the decode kernel chunks pairs differently) */
  int32_t reserved;
} vqb_options;

/* vqb_options.reuse: an MoE block's gate, up and down projections share one
 * routing (same indices, n_tokens, top_k and num_experts) and gate / up one
 * x.  With one workspace for the three calls, the first call routes (and
 * gathers x), the others skip that work:
 *   VQB_REUSE_ROUTING  routing tables valid in the workspace (same indices)
 *   VQB_REUSE_X        x gathered for the same x, in_features, codebook
 *                      geometry and dtypes (implies VQB_REUSE_ROUTING) */
#define VQB_REUSE_ROUTING 1
#define VQB_REUSE_X 2

/* Library identity and messages. */
const char* vqb_version(void);
const char* vqb_status_string(vqb_status status);

/* Device-side vq_pack reader: packed [rows, wpr] -> uint16 codes [rows, nsub].
 * Replaces vq_pack.unpack (src/vqlab/runtime/vq_pack.py:79-97) and the MLX
 * reader _unpack_rows (src/vqlab/runtime/vq_dense.py:140-184). */
vqb_status vqb_unpack(const uint32_t* packed, int64_t rows, int64_t wpr, int32_t nsub,
                      int32_t bits, uint16_t* out, vqb_stream_t stream);

/* The two dimension halves of a d8 codebook: out fp16 [2][K][4] = dims 0-3 of
 * every entry, then dims 4-7 (codebook fp16 [K][8], both 16-byte aligned).
 * The grouped GEMM keeps one half of a d8/K16384 codebook in shared memory per
 * pass and reads it in this layout; a caller that builds it once per codebook
 * and passes it as vqb_linear_desc.codebook_halves saves that kernel on every
 * call.  No reference counterpart (the reference's kernels read [K][D]). */
vqb_status vqb_codebook_halves(const void* codebook, int32_t num_codes, void* out, vqb_stream_t stream);

/* Expert index of a pair to leave out: vqb_switch_forward computes nothing
 * for it and does not write its output row (expert parallelism marks the
 * pairs another rank serves this way, with no host-side compaction). */
#define VQB_SKIP_EXPERT 0xFFFFFFFFu

/* Scratch bytes vqb_switch_forward needs for n_tokens x top_k pairs.  The
 * first 16 bytes of the workspace are a status block the call rewrites:
 * int32 [1] is set to VQB_BAD_ROUTING when an expert index >= E (other than
 * VQB_SKIP_EXPERT) was seen (such a pair is computed as expert 0, never read
 * out of range). */
size_t vqb_switch_workspace_size(const vqb_linear_desc* desc, int32_t n_tokens, int32_t top_k,
                                 const vqb_options* opts);

/* y[t*top_k + j, :] = W_{indices[t, j]} x[t, :] for every (token, slot).
 * Replaces VQSwitchLinear.__call__ (src/vqlab/runtime/vq_switch.py:5284-5423):
 * x is narrowed to fp16 (the host cast of :5301-5308), accumulation is fp32,
 * the result is rounded to fp16 and then to y_dtype (:5423). */
vqb_status vqb_switch_forward(const vqb_linear_desc* desc, const void* x, vqb_dtype x_dtype,
                              int32_t n_tokens, const uint32_t* indices, int32_t top_k,
                              void* y, vqb_dtype y_dtype, void* workspace, size_t workspace_bytes,
                              const vqb_options* opts, vqb_stream_t stream);

/* The kernel family vqb_switch_forward selects for this call shape:
 * VQB_PATH_DECODE (fused decode kernel) or VQB_PATH_PREFILL (grouped GEMM),
 * for 16-byte aligned fp16 / bf16 x (fp32 or unaligned x always decode); a
 * negative value is -vqb_status for an invalid descriptor or shape.  No
 * reference counterpart: the reference's dispatch is internal
 * (vq_switch.py:5313-5315); measurement and tests use it to name the kernel. */
int32_t vqb_switch_path(const vqb_linear_desc* desc, int32_t n_tokens, int32_t top_k, const vqb_options* opts);

/* vqb_switch_forward without a workspace argument: the call allocates
 * nothing and takes its scratch from an 8 MiB array inside the library's
 * device image.  No counterpart in the reference (its runtime allocates
 * through MLX).  For callers that cannot hand the library device memory:
 * a host program that reaches the GPU only through this ABI and has no
 * device allocator, or a serving loop that allows no allocation after
 * start-up.  Limits:
 *   - scratch = routing tables for n_tokens*top_k pairs + n_tokens*in_features
 *     fp16 values must fit in 8 MiB, else VQB_WORKSPACE_TOO_SMALL;
 *   - it always runs the decode (small-N) kernel;
 *   - the array is one per GPU and is reused by every call: calls that
 *     overlap on the GPU race on it and must be serialized by the caller;
 *   - the first call on a device looks the array's address up (once per
 *     device and context, that device current: again after the context was
 *     destroyed and created anew); make it before any stream capture.
 * An expert index >= num_experts (other than VQB_SKIP_EXPERT) is not read out
 * of range: such a pair is computed as expert 0, so its y rows hold expert 0's
 * output.  The status block that records it (int32 [1] = VQB_BAD_ROUTING) sits
 * at the start of the library's array and is not readable through this ABI;
 * a caller that must detect bad indices validates them before the call. */
vqb_status vqb_switch_forward_static(const vqb_linear_desc* desc, const void* x, vqb_dtype x_dtype,
                                     int32_t n_tokens, const uint32_t* indices, int32_t top_k,
                                     void* y, vqb_dtype y_dtype, const vqb_options* opts,
                                     vqb_stream_t stream);

/* The MoE block's elementwise work around the projections (the reference's
 * block: tests/test_qwen3_5_parity.py:180-204; mlx_lm SwitchGLU), one pass each.
 *
 * vqb_swiglu: out[i] = dtype( silu(f32(gate[i])) * f32(up[i]) ) for n
 * elements, silu(v) = v / (1 + exp(-v)) in fp32.
 *
 * vqb_moe_combine: out[t, :] = dtype( sum_{j<top_k} w[t, j] * f32(d[t, j, :]) ),
 * expert outputs d [n_tokens, top_k, hidden], weights fp32 [n_tokens, top_k],
 * the slot sum in fp32 in slot order (each product rounded, no fused
 * multiply-add). */
vqb_status vqb_swiglu(const void* gate, const void* up, void* out, int64_t n, vqb_dtype dtype, vqb_stream_t stream);
vqb_status vqb_moe_combine(const void* expert_out, const float* weights, void* out, int32_t n_tokens,
                           int32_t top_k, int32_t hidden, vqb_dtype dtype, vqb_stream_t stream);

/* The block's router in one kernel: for each of n_tokens rows of fp32
 * router logits [n_tokens, num_experts], p = softmax(logits) in fp32, the
 * top_k largest p in descending order (the lower expert id first on a tie)
 * -> indices int32 [n_tokens, top_k], and weights fp32 [n_tokens, top_k] =
 * p / (sum of the selected p), always renormalised -- the router convention
 * of family/qwen3_5.py:110-118 restated by tests/test_qwen3_5_parity.py:180-204.
 * num_experts <= 8192, top_k <= 32. */
vqb_status vqb_moe_route(const float* logits, int32_t n_tokens, int32_t num_experts, int32_t top_k,
                         int32_t* indices, float* weights, vqb_stream_t stream);

/* Expert-parallel partial combine: out[t, :] = sum_j w[t, j] * expert_out[t, j, :]
 * over the slots whose indices[t, j] != VQB_SKIP_EXPERT (indices may be NULL:
 * every slot), slot order, fp32 out [n_tokens, hidden] with no rounding; a
 * skipped slot's expert_out row is never read.  No reference counterpart
 * (the reference runs every expert on one device). */
vqb_status vqb_moe_combine_partial(const void* expert_out, const float* weights, const uint32_t* indices, float* out,
                                   int32_t n_tokens, int32_t top_k, int32_t hidden, vqb_dtype dtype,
                                   vqb_stream_t stream);

/* ---- The whole MoE block in one launch (decode batches) ----
 *
 * y = combine(down(swiglu(gate(x), up(x)))) routed by router_logits: the
 * block of tests/test_qwen3_5_parity.py:180-204 around three VQSwitchLinear
 * projections (vq_switch.py:5284-5423), with the routing of vqb_moe_route
 * (bit-identical indices and weights) and the roundings of the per-step
 * calls -- each projection's output to fp16 and then to x's dtype, h = dtype(
 * silu(g) * u) narrowed to fp16 as the down projection's input, the combine
 * in fp32 in slot order -- in ONE persistent cooperative kernel.  The
 * projections take W = fp16(cb * s) weights with fp32 accumulation (the
 * reference's non-ACCS arm).  No reference counterpart as one call (the
 * reference dispatches each step).
 *
 * gate / up: [E, I, H]; down: [E, H, I]; each descriptor's codebook_halves
 * must be set (vqb_codebook_halves).  Served shapes (else
 * VQB_UNSUPPORTED_GEOMETRY, and the caller runs the per-step calls): d8
 * codebooks with K = 2^BITS, BITS 12 or 14, packed codes, group size 64, the
 * same K for the three projections, H and I multiples of 512, E <= 1024,
 * n_tokens * top_k <= 640, no SKIPZERO row table, bf16 / fp16 x, codes and
 * scales 16-byte aligned.  indices / weights (both or neither) receive the
 * routing [n_tokens, top_k].  The first 16 bytes of the workspace are a status
 * block the call rewrites (int32 [1] = VQB_TIMEOUT when a bounded device wait
 * gave up).  Calls of this kernel on one GPU must not overlap: each holds one
 * CTA on every SM until it ends (a cooperative launch), and their grid
 * barriers share one arrival counter per device. */
typedef struct vqb_moe_block_desc {
  vqb_linear_desc gate;
  vqb_linear_desc up;
  vqb_linear_desc down;
  int32_t top_k;
} vqb_moe_block_desc;

/* Optional knobs of vqb_moe_block_forward (NULL = defaults).  wait_limit_us:
 * the kernel's bounded waits for its own copies give up after this long
 * (0 = 2 s; its grid barriers always wait up to 2 s); stall_cta: tests of the
 * failure path only -- that CTA waits for a signal nothing sends, gives up
 * after wait_limit_us and the call reports VQB_TIMEOUT (-1 = none; 0 is a real
 * CTA, so a zero-filled struct must set it to -1). */
typedef struct vqb_moe_block_options {
  int32_t wait_limit_us;
  int32_t stall_cta;
} vqb_moe_block_options;

/* ---- A dense VQ MLP in one launch (decode batches) ----
 *
 * y = down(swiglu(gate(x), up(x))) for three VQLinear projections (gate / up
 * [I, H], down [H, I], num_experts = 1): the caller-side composition of
 * VQLinear.__call__ (vq_dense.py:346-441) in a dense model's MLP, with the
 * numerics of the per-step calls on the d8 path (_decode_matmul,
 * vq_dense.py:267-312): weights bf16(fp16(cb * s)) for bf16 x (fp16 for fp16
 * x), x kept in its dtype, fp32 accumulation, each projection's output
 * rounded once to x's dtype, h = dtype(silu(g) * u) (vqb_swiglu).  The same
 * persistent kernel as vqb_moe_block_forward with one expert and no router;
 * served shapes as there (d8, K = 2^BITS at 12 / 14 bits, G = 64, H and I
 * multiples of 512, codebook_halves set, n_tokens <= 640), else
 * VQB_UNSUPPORTED_GEOMETRY.  It decodes every weight once per 8 tokens, so it
 * pays at small n_tokens; the Python module takes it up to 8.  The same
 * status block and calls-must-not-overlap rule as the MoE block. */
typedef struct vqb_dense_mlp_desc {
  vqb_linear_desc gate;
  vqb_linear_desc up;
  vqb_linear_desc down;
} vqb_dense_mlp_desc;

vqb_status vqb_dense_mlp_supported(const vqb_dense_mlp_desc* desc, int32_t n_tokens, vqb_dtype x_dtype);
size_t vqb_dense_mlp_workspace_size(const vqb_dense_mlp_desc* desc, int32_t n_tokens);
vqb_status vqb_dense_mlp_forward(const vqb_dense_mlp_desc* desc, const void* x, vqb_dtype x_dtype, int32_t n_tokens,
                                 void* y, void* workspace, size_t workspace_bytes, const vqb_moe_block_options* opts,
                                 vqb_stream_t stream);

vqb_status vqb_moe_block_supported(const vqb_moe_block_desc* desc, int32_t n_tokens, vqb_dtype x_dtype);
size_t vqb_moe_block_workspace_size(const vqb_moe_block_desc* desc, int32_t n_tokens);
vqb_status vqb_moe_block_forward(const vqb_moe_block_desc* desc, const float* router_logits, const void* x,
                                 vqb_dtype x_dtype, int32_t n_tokens, void* y, int32_t* indices, float* weights,
                                 void* workspace, size_t workspace_bytes, const vqb_moe_block_options* opts,
                                 vqb_stream_t stream);

/* ---- Expert-parallel exchange over peer memory (fixed-shape decode path) ----
 *
 * No reference counterpart: the reference runs every expert on one device
 * (its multi-node path pipelines whole layers).  This replaces the NCCL
 * all-gather / all-to-all pair around the expert projections when every rank
 * holds at most `tokens` tokens: each rank WRITES its token rows straight into
 * the other ranks' memory, and each rank's partial expert sums are written
 * straight into the owning rank's memory.
 *
 * One process per GPU; the `world` GPUs must have peer access to one another
 * (NVLink / NVSwitch on one node).  Each rank allocates one exchange region
 * (vqb_ep_region_alloc) and maps every other rank's region through CUDA IPC
 * (vqb_ep_ipc_handle, then vqb_ep_ipc_open of each peer's handle).  One layer
 * step, all on one stream and with no host synchronisation (graph-capturable):
 *   vqb_ep_dispatch   this rank's rows, expert slots and weights into every region
 *   the rank's projections on its region's x_rows / slots (vqb_switch_forward)
 *   vqb_ep_combine    fp32 slot sums of this rank's pairs into the owners' regions
 *   vqb_ep_reduce     the owner sums the ranks' partials (rank order), rounds once
 * Every rank makes the same calls in the same order.  Each dispatch and combine
 * ends in a bounded wait for the other ranks' signals (opts->wait_limit_us,
 * default 2 s): when it gives up, the int32 at VQB_EP_STATUS_OFFSET of the
 * rank's region becomes VQB_TIMEOUT and the exchange is out of step -- free
 * the regions and set them up again.
 *
 * Region layout (byte offsets from vqb_ep_region_bytes; W = world, C = tokens):
 *   [0, 512)  control: signal words the ranks write, epoch, status
 *   x_rows    16-bit [W * C, hidden]: block s = rank s's token rows (x dtype);
 *             a row whose token has no pair on this rank is not sent
 *   slots     int32 [W * C, top_k]: this rank's local expert of each pair,
 *             VQB_SKIP_EXPERT (-1) for pairs of other ranks and padding rows
 *   weights   fp32 [W * C, top_k]
 *   partials  fp32 [W, C, hidden]: block s = rank s's slot sums for this rank's tokens */
#define VQB_EP_MAX_WORLD 8
#define VQB_EP_STATUS_OFFSET 272
#define VQB_EP_IPC_HANDLE_BYTES 64

typedef struct vqb_ep_layout {
  int32_t world;             /* ranks, 1..VQB_EP_MAX_WORLD */
  int32_t rank;              /* this rank */
  int32_t tokens;            /* C: token rows per rank per step (the fixed shape) */
  int32_t top_k;             /* 1..256 */
  int32_t hidden;            /* a multiple of 8 */
  int32_t experts_per_rank;  /* rank r serves global experts [r * E_local, (r + 1) * E_local) */
} vqb_ep_layout;

typedef struct vqb_ep_options {
  int32_t phases;            /* 0 or 3 = both; 1 = write and signal only, 2 = wait only: ranks
                                emulated in one process run every rank's phase 1 before any
                                phase 2, so that no launch waits on a later launch */
  int32_t wait_limit_us;     /* 0 = 2,000,000 */
} vqb_ep_options;

/* Region size; offsets (may be NULL) receives {x_rows, slots, weights, partials}. */
size_t vqb_ep_region_bytes(const vqb_ep_layout* layout, size_t* offsets);
/* cudaMalloc of the region on the current device, zeroed (synchronous; set-up only). */
vqb_status vqb_ep_region_alloc(const vqb_ep_layout* layout, void** region);
vqb_status vqb_ep_region_free(void* region);
/* The region's CUDA IPC handle (VQB_EP_IPC_HANDLE_BYTES bytes) for the other ranks. */
vqb_status vqb_ep_ipc_handle(void* region, void* handle);
/* Map a peer's region into this process (peer access enabled); close with vqb_ep_ipc_close. */
vqb_status vqb_ep_ipc_open(const void* handle, void** peer_region);
vqb_status vqb_ep_ipc_close(void* peer_region);

/* regions: host array of `world` device pointers, regions[rank] = this rank's
 * own region, the others its mappings of the peers' regions.
 * x [n_tokens, hidden] 16-bit (16-byte aligned rows), indices int32
 * [n_tokens, top_k] GLOBAL expert ids, weights fp32 [n_tokens, top_k];
 * n_tokens <= tokens (rows n_tokens..tokens-1 route nowhere). */
vqb_status vqb_ep_dispatch(const vqb_ep_layout* layout, void* const* regions, const void* x, vqb_dtype x_dtype,
                           int32_t n_tokens, const int32_t* indices, const float* weights,
                           const vqb_ep_options* opts, vqb_stream_t stream);
/* expert_out [world * tokens, top_k, hidden] (dtype): the projections' output
 * for this region's x_rows / slots; rows of skipped pairs are never read. */
vqb_status vqb_ep_combine(const vqb_ep_layout* layout, void* const* regions, const void* expert_out,
                          vqb_dtype dtype, const vqb_ep_options* opts, vqb_stream_t stream);
/* y[t, :] = y_dtype(sum over ranks r in order of partials[r, t, :]) for t < n_tokens. */
vqb_status vqb_ep_reduce(const vqb_ep_layout* layout, void* region, void* y, vqb_dtype y_dtype, int32_t n_tokens,
                         vqb_stream_t stream);

/* Measurement aids; neither has a counterpart in the reference, whose Metal
 * runtime exposes no launch accounting or per-kernel timing.
 *
 * vqb_launch_count: kernels this library has launched in the process so far
 * (every route, conversion, decode and GEMM kernel; not graph replays).
 *
 * vqb_time_next_kernel: arm a one-shot timer for the calling host thread.  The
 * next vqb_switch_forward / vqb_dense_forward call on this thread records
 * start_event (a cudaEvent_t) on its stream immediately before its dominant
 * kernel -- the decode or grouped-GEMM kernel -- and stop_event immediately
 * after it, then disarms.  Both NULL disarms; one NULL is VQB_NULL_POINTER. */
uint64_t vqb_launch_count(void);
vqb_status vqb_time_next_kernel(void* start_event, void* stop_event);

/* Scratch bytes vqb_dense_forward needs for n_rows input rows.  The first 16
 * bytes of the workspace are a status block the call rewrites: int32 [1] is
 * VQB_TIMEOUT when a bounded device wait of the call gave up, else 0. */
size_t vqb_dense_workspace_size(const vqb_linear_desc* desc, int64_t n_rows, const vqb_options* opts);

/* y[n, :] = W x[n, :] for a dense VQ projection (E = 1).
 * Replaces VQLinear.__call__ (src/vqlab/runtime/vq_dense.py:346-441): the
 * small-N fused kernel narrows x to fp16 in-kernel and stores y_dtype
 * directly (vq_switch.py:2319-2327); the large-N path materialises
 * W = fp16(cb*s) in x's dtype tile by tile and runs the GEMM
 * (_decode_matmul, vq_dense.py:267-312).  Under VQB_PATH_AUTO a d2 layer with
 * <= 256 codebook entries stored as 8-bit codes (IN a multiple of 512, group
 * 64, 16-byte aligned x / codes / scales) at <= 8 rows runs as one launch with
 * the codebook replicated per lane in shared memory, and a d8 layer with
 * <= 4096 entries and an even code width likewise with the codebook whole in
 * shared memory; same numerics. */
vqb_status vqb_dense_forward(const vqb_linear_desc* desc, const void* x, vqb_dtype x_dtype,
                             int64_t n_rows, void* y, vqb_dtype y_dtype,
                             void* workspace, size_t workspace_bytes,
                             const vqb_options* opts, vqb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VQB_H_ */
