// vqb_switch_forward_static: the expert decode call for callers that cannot
// give the library any device memory of its own.
//
// vqb_switch_forward needs a scratch workspace (the expert routing tables and
// x converted to fp16).  Some callers have no way to provide one: a host
// program that reaches the GPU only through this C ABI and owns no device
// allocator, or a serving loop that forbids device allocation after start-up
// (a cudaMalloc can synchronize the whole device and carve up a memory pool
// that was sized once).  For them this entry point takes its scratch from a
// fixed array in the library's own device image instead.  It serves the
// decode path (the expert-grouped tensor-core kernel) and allocates nothing.
//
// Rules of the shared array (documented in include/vqb.h as well):
//   * it is kStaticScratchBytes (8 MiB) on every GPU that loads the library,
//     held until the process exits;
//   * a call whose scratch would not fit returns VQB_WORKSPACE_TOO_SMALL
//     before touching the GPU;
//   * the first call on a device (and the first call after that device's
//     context was destroyed and created again) resolves the array's device
//     address, with that device current -- make that first call before any
//     stream capture;
//   * every call reuses the same bytes and leaves the previous call's data in
//     them; the call clears the part that must start at zero itself.  Two
//     calls that overlap on the GPU (other streams, other host threads) race
//     on the array: serialize them.
#include <cuda.h>

#include <mutex>

#include "vqb_common.cuh"
#include "vqb_internal.h"

namespace vqb {
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// The resolved address of the array for one device, valid for the context
// whose process-unique id (cuCtxGetId) it was resolved in.
struct ScratchSlot {
  unsigned long long ctx_id;
  void* ptr;
};

std::mutex g_scratch_mu;
ScratchSlot g_scratch[kMaxDevices] = {};
bool g_driver_looked_up = false;
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

void* driver_entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return p;
}

// Process-unique id of the current context, 0 when it cannot be read.
unsigned long long current_ctx_id() {
  if (!g_ctx_get_current || !g_ctx_get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  if (g_ctx_get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_static_scratch in the current context.  The symbol's
// name is only a host-side handle; the address must come from the runtime,
// and it is re-resolved whenever the current context is not the one the
// cached address belongs to (a device reset, or a context destroyed and
// created again, unloads the module the old address pointed into).
vqb_status scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return VQB_CUDA_ERROR;
  if (dev < 0 || dev >= kMaxDevices) return VQB_CUDA_ERROR;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_driver_looked_up) {
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(driver_entry("cuCtxGetCurrent"));
    g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(driver_entry("cuCtxGetId"));
    g_driver_looked_up = true;
  }
  ScratchSlot& slot = g_scratch[dev];
  const unsigned long long id = current_ctx_id();
  if (slot.ptr && id != 0 && slot.ctx_id == id) {
    *out = slot.ptr;
    return VQB_OK;
  }
  // first call in this context (or no context id available: resolve every call)
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return VQB_CUDA_ERROR;
  slot.ptr = p;
  slot.ctx_id = current_ctx_id();  // the lookup above makes the device's primary context current
  *out = p;
  return VQB_OK;
}

}  // namespace
}  // namespace vqb

using namespace vqb;

extern "C" vqb_status vqb_switch_forward_static(const vqb_linear_desc* desc, const void* x, vqb_dtype x_dtype,
                                                int32_t n_tokens, const uint32_t* indices, int32_t top_k, void* y,
                                                vqb_dtype y_dtype, const vqb_options* opts, vqb_stream_t stream) {
  LinearGeometry geo;
  vqb_status st = validate(desc, &geo);
  if (st != VQB_OK) return st;
  if (n_tokens < 0 || top_k < 1) return VQB_BAD_SHAPE;
  if (x_dtype != VQB_F16 && x_dtype != VQB_BF16 && x_dtype != VQB_F32) return VQB_BAD_SHAPE;
  if (y_dtype != VQB_F16 && y_dtype != VQB_BF16 && y_dtype != VQB_F32) return VQB_BAD_SHAPE;
  const int64_t N64 = int64_t(n_tokens) * top_k;
  if (N64 > 0x7fffffff) return VQB_BAD_SHAPE;
  const int N = static_cast<int>(N64);
  if (N == 0) return VQB_OK;
  if (!x || !indices || !y) return VQB_NULL_POINTER;
  // routing tables + x as 16-bit rows, the decode path's scratch
  const size_t need = linear_workspace_bytes(N, geo.E, n_tokens, 0, geo.OUT, 0, 0) + mma_x16_bytes(n_tokens, geo.IN);
  if (need > kStaticScratchBytes) return VQB_WORKSPACE_TOO_SMALL;
  void* scratch = nullptr;
  st = scratch_address(&scratch);
  if (st != VQB_OK) return st;
  // same numerics as vqb_switch_forward's decode path (the status block at the
  // front of the scratch is cleared inside run_linear)
  return run_linear(geo, x, x_dtype, n_tokens, indices, top_k, N, y, y_dtype, scratch, opts,
                    /*narrow_x_f16=*/true, /*round_f16_first=*/true, /*wround=*/0, /*large=*/false,
                    reinterpret_cast<cudaStream_t>(stream));
}
