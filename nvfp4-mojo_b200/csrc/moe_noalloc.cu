// moe_noalloc.cu -- nvfp4_moe_forward_noalloc: the MoE layer for callers
// that cannot allocate device memory.
//
// Who needs it: a caller that holds only the pointers it was given and has no
// device allocator of its own (for example host code that reaches this
// library through a foreign-function call, as the reference's Mojo code would
// with external_call), or a serving loop that must not call cudaMalloc once it
// runs (cudaMalloc synchronises the device and is not allowed while a stream
// is being captured).  Such a caller cannot provide the workspace that
// nvfp4_moe_forward needs.
//
// This entry point uses instead a fixed scratch array in device memory,
// g_moe_scratch, of NVFP4_NOALLOC_SCRATCH_BYTES (16 MiB): every GPU that loads
// the library holds it until the process exits.  It allocates nothing: no
// cudaMalloc, cudaFree, or allocating library routine.  Layers whose
// workspace would exceed the array (nvfp4_moe_workspace_size(desc, T) > 16 MiB)
// are rejected with NVFP4_ERR_WORKSPACE before anything is launched.
//
// Set-up: in host code the name g_moe_scratch is only a host-side stand-in, not
// a device address, so the first call on each device (with that device
// current) asks the runtime for the array's device address with
// cudaGetSymbolAddress and caches it; make that first call before any stream
// capture.  Every call on a device shares the one array, which keeps the last
// call's contents: the layer writes every scratch byte it reads earlier in the
// same call, so nothing has to start at zero, but calls that overlap on the
// GPU (different streams, or different host threads) race on it and must be
// serialised by the caller.
#include <mutex>

#include "../../include/nvfp4.h"
#include "abi_util.h"

namespace nvfp4 {
namespace {

static __device__ __align__(256) uint8_t g_moe_scratch[NVFP4_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void *g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's g_moe_scratch (looked up once per device).
int scratch_for_current_device(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(NVFP4_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_moe_scratch);
    if (e != cudaSuccess || !p)
      return fail(NVFP4_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return NVFP4_OK;
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

extern "C" int nvfp4_moe_forward_noalloc(const nvfp4_moe_desc *desc,
                                         const nvfp4_moe_weights *weights, const void *x,
                                         const void *residual, void *y, int y_dtype, int64_t T,
                                         int32_t *topk_ids, float *topk_w, void *stream) {
  NVFP4_ABI_RANGE();
  if (!desc) return fail(NVFP4_ERR_INVALID_ARG, "null MoE descriptor");
  if (desc->top_k <= 0 || T < 0 || T > (1 << 24) / desc->top_k)
    return fail(NVFP4_ERR_INVALID_ARG, "bad token count or top_k");
  const size_t need = nvfp4_moe_workspace_size(desc, T);
  if (need == 0 && T > 0) return fail(NVFP4_ERR_INVALID_ARG, "invalid MoE descriptor");
  if (need > (size_t)NVFP4_NOALLOC_SCRATCH_BYTES)
    return fail(NVFP4_ERR_WORKSPACE,
                "%lld tokens need %zu bytes of scratch; the static scratch holds %zu bytes "
                "(use nvfp4_moe_forward with a caller workspace, or fewer tokens per call)",
                (long long)T, need, (size_t)NVFP4_NOALLOC_SCRATCH_BYTES);
  void *scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  return nvfp4_moe_forward(desc, weights, x, residual, y, y_dtype, T, topk_ids, topk_w, scratch,
                           (size_t)NVFP4_NOALLOC_SCRATCH_BYTES, stream);
}
