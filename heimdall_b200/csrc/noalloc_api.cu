// Allocation-free variant of the fused decode step (bf_bifrost_layer_decode_noalloc).
//
// Some callers cannot allocate device memory at the point where they run a decode step: for example a
// serving runtime whose memory manager reserves almost all of HBM up front for its own pools (so a fresh
// allocation fails or fragments that reservation), or a foreign-language host that binds only a few C entry
// points and has no way to own a device buffer for our workspace.  For them this entry point takes its
// scratch from a fixed array compiled into the library instead of a caller-provided workspace.
//
// The array lives in device global memory, one copy per GPU that loads the library, and stays allocated
// until the process exits.  Its size bounds the batch: the request must fit bf_layer_decode_workspace(...)
// into kNoAllocScratchBytes (16 MiB, enough for 64 sequences of the Bifrost geometry H=24, G=4, D=256,
// W=2048), otherwise the call returns BF_ERR_WORKSPACE before launching anything.
//
// In host code the array's name is only a host-side stand-in, not a device address, so the device address
// is looked up with cudaGetSymbolAddress once per device (with that device current) on the first call and
// cached; that first call should therefore happen before any stream capture begins.
// Every call on a device shares the one array: calls that overlap on the GPU (e.g. on two streams at once)
// race on it.  Nothing in the array needs to start at zero: each byte a call reads was written earlier in
// the same call, and the array keeps the last call's contents afterwards.
#include <mutex>

#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64] = {nullptr};

// device address of this device's scratch array (looked up once per device)
static int noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BF_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return cuda_fail();
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return BF_OK;
}

}  // namespace bfb

using namespace bfb;

extern "C" int bf_bifrost_layer_decode_noalloc(const bf_layer* L, const void* x, const void* q, const void* k,
                                               const void* v, const void* qr, const void* kr, const int64_t* pos,
                                               int B, bf_ring_cache* cache, int memory, float* o, float* lse,
                                               bf_stream_t stream) {
  if (!L || B <= 0) return BF_ERR_INVALID_ARGUMENT;
  const size_t need = bf_layer_decode_workspace(B, L->H, L->G, L->D, L->window);
  if (need == 0 || need > kNoAllocScratchBytes) return BF_ERR_WORKSPACE;
  void* ws = nullptr;
  int rc = noalloc_scratch(&ws);
  if (rc) return rc;
  return bf_bifrost_layer_decode(L, x, q, k, v, qr, kr, pos, B, cache, memory, o, lse, ws, kNoAllocScratchBytes,
                                 stream);
}
