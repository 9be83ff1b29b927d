// Internal declarations shared by the .cu files behind the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define BF_ABI_VERSION 1
#define BF_MAX_STAGES 12

namespace bfb {

struct DeviceState {
  int device;
  unsigned int* err;  // device error word of this device
  int sm_count;
};

int device_state(DeviceState* st);
// non-blocking side streams per device (created on first use, kept for the process) for work that runs
// concurrently inside one call, forked from and joined back into the caller's stream with events before the
// call returns: which = 0 and 2 have the device's least stream priority, which = 1 its greatest
cudaStream_t side_stream(const DeviceState& st, int which);

// per-stage timing hooks (no-ops unless bf_stage_events installed events)
void stage_mark(int stage, int end, cudaStream_t stream);
enum Stage { ST_XPROJ = 0, ST_HEADPROJ, ST_GDN_P1, ST_GDN_P2, ST_GDN_P3, ST_WIN_PREP, ST_WIN, ST_CACHE, ST_DEC_STATE,
             ST_DEC_WIN, ST_DEC_GATHER, ST_DEC_COMBINE };
bool aligned16(const void* p);
// Opts `fn` into `bytes` of dynamic shared memory on the current device.  cudaFuncSetAttribute applies to
// the current device only, so this is done once per (kernel, device), under a lock; later calls only look
// the pair up -- so `bytes` must be the kernel's largest launch size, the same on every call.  Returns BF_OK or
// BF_ERR_CUDA.
int ensure_smem_attr(const void* fn, int bytes);
// BF_ERR_CUDA with the CUDA error recorded for bf_last_cuda_error (e: a failed call's result, or the pending
// launch error when e is cudaSuccess); launch_status() is BF_OK or that
int cuda_fail(cudaError_t e = cudaSuccess);
inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : cuda_fail(e);
}

// max_ctas > 0 caps the persistent grid (to share the GPU with a concurrent kernel); 0 = one CTA per SM
int launch_gdn_decode(const float* q, const float* k, const void* v, int v_bf16, const float* g,
                      const float* beta, const float* s_in, float* s_out, float* o, int B, int G, int R, int D,
                      cudaStream_t stream, int max_ctas = 0);

}  // namespace bfb
