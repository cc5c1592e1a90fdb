// oasis_gemm_static_scratch: the split-K GEMM without a caller workspace.
//
// Some callers of this library cannot allocate device memory: a host runtime
// whose allocator is owned by someone else (a serving framework that hands out
// only its own tensors), code running where cudaMalloc is forbidden or would
// synchronize the device at a bad moment, or a plugin ABI that passes only
// inputs and outputs. For them this entry point takes its split-K scratch
// (the partial tiles of the split-K clusters) from a fixed array in device
// memory that the library owns. It allocates nothing itself.
//
// Costs and limits, stated once here:
//  * every GPU that loads this library holds kStaticScratchBytes (8 MiB) of
//    device memory for this array until the process exits;
//  * problems whose split-K scratch would exceed that are rejected with
//    OASIS_ERR_WORKSPACE (use oasis_gemm with a workspace instead);
//  * all calls share the one array: two calls that overlap on the GPU (different
//    streams, or different host threads on the same device) race on it. Issue them
//    on one stream, one after another. The partials need no clearing (every
//    split overwrites its own before the cluster barrier).
//  * the first call on each device looks the array's device address up (with
//    that device current) and caches it; make that first call before any stream
//    capture. The cache assumes one primary context per device for the life of
//    the process: after cudaDeviceReset the address may change, so do not call
//    this entry point again in that process.
#include <mutex>

#include "../../include/oasis_b200.h"
#include "gemm.cuh"
#include "status.h"

namespace oasis {
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;

// Library-owned split-K scratch. In host code this name is only a host-side
// stand-in for the symbol; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of g_static_scratch on the current device (looked up once per device).
int static_scratch_ptr(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "gemm_static_scratch: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(OASIS_ERR_UNSUPPORTED, "gemm_static_scratch: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return set_error(OASIS_ERR_CUDA, "gemm_static_scratch: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return OASIS_OK;
}

}  // namespace
}  // namespace oasis

extern "C" size_t oasis_gemm_static_scratch_capacity(void) { return oasis::kStaticScratchBytes; }

extern "C" int oasis_gemm_static_scratch(const OasisGemmArgs* a, oasis_stream_t stream) {
  OASIS_REQUIRE(a, "gemm_static_scratch: null args");
  const size_t need = oasis::gemm_splitk_bytes(a->m, a->n, a->k, a->mode, a->block_n, a->splits);
  if (need > oasis::kStaticScratchBytes)
    return oasis::set_error(OASIS_ERR_WORKSPACE,
                            "gemm_static_scratch: %d x %d x %d needs %zu bytes of split-K scratch, more than the "
                            "fixed %zu; call oasis_gemm with a workspace (or splits = 1)",
                            a->m, a->n, a->k, need, oasis::kStaticScratchBytes);
  void* scratch = nullptr;
  OASIS_TRY(oasis::static_scratch_ptr(&scratch));
  OasisGemmArgs b = *a;  // the caller's workspace fields, if any, are ignored
  b.workspace = scratch;
  b.workspace_bytes = oasis::kStaticScratchBytes;
  return oasis_gemm(&b, stream);
}
