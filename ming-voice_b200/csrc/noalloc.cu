// mv_block_decode_noalloc: the one-kernel decode block with its scratch in a static device array.
//
// Some callers cannot hand the library a workspace. A host that binds the C-ABI without a device
// allocator of its own (no torch caching allocator, a plain C or FFI caller) would need cudaMalloc,
// which synchronises the device and is not allowed while a stream is being captured into a graph.
// A serving loop that reserved all device memory up front has no room to grow either. This entry point
// serves them: its scratch is a fixed array in the library's own device memory (1 MiB, reserved when the
// module loads), so a call performs no allocation at all.
//
// Set-up: the first call on each device (made with that device current) looks the array's address up
// with cudaGetSymbolAddress and caches it; make that first call before any stream capture starts.
//
// What must start at zero: the 256-byte header at the front of the scratch (the grid-barrier counters and
// the error word). Each call clears it with cudaMemsetAsync on the caller's stream before the launch; the
// rest of the scratch (router logits, activations) is written before it is read.
//
// Races: there is ONE scratch per device. Two calls that can execute at the same time on one device
// (different streams without ordering between them, or two host threads) overwrite each other's
// counters and activations. Issue all calls of a device on one stream, or order them with events.
#include <cuda_runtime.h>

#include <mutex>

#include "mingmoe.h"
#include "mingmoe_internal.h"

namespace mv {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB: M = 16 at H=2048 / I=1408 / top-6 + 2 uses 0.7 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the static scratch on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "mv_block_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MV_ERR_UNSUPPORTED, "mv_block_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "mv_block_decode_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MV_OK;
}

}  // namespace
}  // namespace mv

extern "C" int mv_block_decode_noalloc(const mv_block* b, const void* x, int M, void* out, float* logits_out,
                                       void* ids_out, int ids_dtype, float* wts_out, unsigned int* status_out,
                                       void* stream) {
  using namespace mv;
  if (b == nullptr) return fail(MV_ERR_INVALID, "mv_block_decode_noalloc: null block");
  const size_t need = mv_block_decode_workspace_bytes(M, b->top_k + b->n_shared, b->experts.I, b->E);
  if (need > kNoAllocScratchBytes)
    return fail(MV_ERR_WORKSPACE,
                "mv_block_decode_noalloc: M=%d, %d experts per token, I=%d, E=%d need %zu bytes of scratch; the "
                "static scratch holds %zu (call mv_block_decode with a workspace instead)",
                M, b->top_k + b->n_shared, b->experts.I, b->E, need, kNoAllocScratchBytes);
  void* ws = nullptr;
  int rc = scratch_for_current_device(&ws);
  if (rc != MV_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(ws, 0, kWsHeaderBytes, st);
  if (e != cudaSuccess) return cuda_status(e, "mv_block_decode_noalloc: clearing the scratch header");
  rc = mv_block_decode(b, x, M, out, logits_out, ids_out, ids_dtype, wts_out, ws, kNoAllocScratchBytes, stream);
  if (rc != MV_OK) return rc;
  if (status_out != nullptr) {
    // the header's error word and its location (two 32-bit words) for this call
    e = cudaMemcpyAsync(status_out, static_cast<unsigned char*>(ws) + 4, 2 * sizeof(unsigned int), cudaMemcpyDefault,
                        st);
    if (e != cudaSuccess) return cuda_status(e, "mv_block_decode_noalloc: copying the status words");
  }
  return MV_OK;
}
