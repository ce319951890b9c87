// Shared-selection prefill for callers that cannot allocate device memory.
//
// Some hosts of this op may not call cudaMalloc (or any allocating routine): plugins running
// inside a runtime that owns every device allocation through its own pool, code that runs
// under a fixed memory budget decided before the process starts, or integrations that only
// hand over the input and output buffers.  sta_shared_forward_static serves them: it is
// sta_shared_forward with its scratch taken from a fixed array in device memory that this
// library holds, so a call allocates nothing.
//
// Contract (also stated in include/sta.h):
//  * the array holds STA_STATIC_SCRATCH_BYTES (64 MiB); every GPU that loads the library keeps
//    it for the life of the process.  The CUDA runtime reserves it when it loads this module
//    on a device: at library load with CUDA_MODULE_LOADING=EAGER, otherwise (the default, lazy
//    loading) on the first call on that device -- so under lazy loading the first call can
//    still fail with out-of-memory (STA_ERR_CUDA) if the device is already full;
//  * when the op's scratch would be larger, the op walks over smaller groups of kv heads; if a
//    single kv head still needs more, the call fails with STA_ERR_WORKSPACE and a message;
//  * the first call on a device looks up the array's device address (cudaGetSymbolAddress) with
//    that device current, so make that first call before any stream capture;
//  * all calls share the one array and it keeps the previous call's contents: nothing in the
//    pipeline reads scratch before writing it, so no clearing is needed, but calls that overlap
//    on the GPU (different streams, or different host threads on one device) race on it.
#include "common.cuh"
#include "sta_internal.h"

#define STA_STATIC_SCRATCH_BYTES_VALUE (64ull << 20)

namespace sta {
namespace {

__device__ __align__(256) uint8_t g_static_scratch[STA_STATIC_SCRATCH_BYTES_VALUE];

// device address of g_static_scratch per device, looked up once per device
void* g_static_scratch_addr[64] = {nullptr};

}  // namespace
}  // namespace sta

extern "C" int sta_shared_forward_static(const sta_forward_args* a, void* stream) {
  using namespace sta;
  if (!a) return fail(STA_ERR_ARG, "sta_shared_forward_static: null arguments");
  const int rc = check_shared_forward(a);
  if (rc != STA_OK) return rc;
  if (a->n <= 0 || a->batch <= 0) return STA_OK;  // nothing to do (as sta_shared_forward)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(STA_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(STA_ERR_UNSUPPORTED, "sta_shared_forward_static: device index >= 64");
  if (!g_static_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(STA_ERR_CUDA, "sta_shared_forward_static: cudaGetSymbolAddress of the static scratch failed");
    g_static_scratch_addr[dev] = p;
  }
  // cap the scratch at the array's size: the op then runs over groups of kv heads
  sta_forward_args b = *a;
  const int64_t cap = (int64_t)STA_STATIC_SCRATCH_BYTES_VALUE;
  if (b.max_workspace_bytes <= 0 || b.max_workspace_bytes > cap) b.max_workspace_bytes = cap;
  const size_t need = sta_shared_workspace_bytes(&b);
  if (need == 0) return fail(STA_ERR_ARG, "sta_shared_forward_static: empty workspace layout");
  if (need > (size_t)STA_STATIC_SCRATCH_BYTES_VALUE)
    return fail(STA_ERR_WORKSPACE,
                "sta_shared_forward_static: one kv head of this problem needs more scratch than "
                "the 64 MiB static array; use sta_shared_forward with a caller workspace");
  return sta_shared_forward(&b, g_static_scratch_addr[dev], (size_t)STA_STATIC_SCRATCH_BYTES_VALUE,
                            stream);
}
