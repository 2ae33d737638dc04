// glmaxx_router_compact_launch_static: the device router + stable compaction
// without a caller-provided workspace and without allocating anything.
//
// Some callers cannot hand the library scratch memory: an engine whose HBM is
// carved up front into a fixed arena with no room left for per-call workspace,
// or code that runs while the device must not allocate (cudaMalloc/cudaFree may
// synchronise the device).  For them
// the router's scratch (partial logits, token-in-expert bitmap, word prefixes,
// counts) lives in one file-scope device array of kRouterStaticScratchBytes,
// which every GPU that loads this library holds until the process exits.
//
// Behaviour and limits:
//  - Same results as glmaxx_router_compact_launch; the descriptor's workspace
//    and workspace_bytes fields are ignored.  Inputs and outputs are the
//    caller's, as usual.
//  - Shapes whose scratch would exceed the array are rejected with
//    GLMAXX_ERR_DESCRIPTOR (the limit is GLMAXX_ROUTER_STATIC_SCRATCH_BYTES;
//    glmaxx_router_workspace_bytes() gives a shape's need: 256 experts at top-8
//    fit up to T = 507, 4,190,208 bytes; T = 508 needs 4,198,400).
//  - The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress with that device current) and caches it for the
//    life of the process; cudaDeviceReset, which would reload the module at a
//    possibly different address, is not supported.  Make that first call before
//    any stream capture.
//  - All calls on a device share the one array and leave their scratch in it.
//    Everything that must start at zero is cleared by the call itself (the
//    bitmap by the logits kernel, the status word by a memset).  Two calls whose
//    work overlaps on the GPU (different streams, or concurrent graph replays)
//    race on the array and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/glmaxx_kernel.h"
#include "runtime.h"

namespace glmaxx {
namespace {

constexpr uint64_t kRouterStaticScratchBytes = GLMAXX_ROUTER_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_router_scratch[kRouterStaticScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_router_scratch on the current device (looked up once per
// device; the host-side symbol is a stand-in, never a device pointer).
int32_t scratch_address(void** out) {
  int dev = -1;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return int32_t(st);
  if (dev < 0 || dev >= kMaxDevices) return GLMAXX_ERR_DESCRIPTOR;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    st = cudaGetSymbolAddress(&p, g_router_scratch);
    if (st != cudaSuccess) return int32_t(st);
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace
}  // namespace glmaxx

extern "C" int32_t glmaxx_router_compact_launch_static(const glmaxx_router_descriptor* descriptor,
                                                       void* cuda_stream,
                                                       int32_t* asynchronous_error) {
  using namespace glmaxx;
  if (descriptor == nullptr || asynchronous_error == nullptr) return GLMAXX_ERR_NULL;
  *asynchronous_error = 0;
  const uint64_t need =
      router_workspace_bytes(descriptor->tokens, descriptor->experts, descriptor->top_k);
  if (descriptor->tokens == 0 || descriptor->experts == 0 || descriptor->top_k == 0 ||
      need > kRouterStaticScratchBytes)
    return GLMAXX_ERR_DESCRIPTOR;
  DeviceInfo info;
  const int32_t arch = current_device_info(&info);
  if (arch != 0) return arch;
  void* scratch = nullptr;
  const int32_t st = scratch_address(&scratch);
  if (st != 0) return st;
  glmaxx_router_descriptor d = *descriptor;
  d.workspace = reinterpret_cast<uint64_t>(scratch);
  d.workspace_bytes = kRouterStaticScratchBytes;
  return router_compact_launch(&d, cuda_stream, asynchronous_error);
}
