// C ABI entry points: argument validation, status codes, per-device state, launch sequencing.
// Every entry point validates its arguments completely before the first launch and returns a
// BF_* status; nothing here allocates device memory.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "capi_internal.h"

namespace bfb {

// device error word (one per device context); kernels receive its address as an argument
__device__ unsigned int g_bf_error_word[4] = {0u, 0u, 0u, 0u};

static std::mutex g_dev_mu;
static unsigned int* g_err_ptr[64] = {nullptr};
static int g_sm_count[64] = {0};
static int g_cc_major[64] = {0};

int device_state(DeviceState* st) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BF_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bf_error_word) != cudaSuccess) return cuda_fail();
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return cuda_fail();
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return cuda_fail();
    g_err_ptr[dev] = static_cast<unsigned int*>(p);
    g_sm_count[dev] = sms;
    g_cc_major[dev] = major;
  }
  if (g_cc_major[dev] != 10) return BF_ERR_NO_DEVICE;
  st->device = dev;
  st->err = g_err_ptr[dev];
  st->sm_count = g_sm_count[dev];
  return BF_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static thread_local int g_last_cuda_error = 0;

int cuda_fail(cudaError_t e) {
  if (e == cudaSuccess) e = cudaGetLastError();
  g_last_cuda_error = (int)e;
  return BF_ERR_CUDA;
}

// per kernel: bit d set = the shared-memory opt-in was applied on device d
static std::unordered_map<const void*, uint64_t> g_smem_attr;

int ensure_smem_attr(const void* fn, int bytes) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BF_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  uint64_t& done = g_smem_attr[fn];
  if (done & (1ull << dev)) return BF_OK;
  const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e);
  done |= 1ull << dev;
  return BF_OK;
}

static cudaStream_t g_side[3][64] = {{nullptr}};

// which = 0 and 2: the device's least priority (the window, which fills whatever SMs the memory chain leaves;
// two streams so that consecutive window launches overlap); which = 1: its greatest priority (the memory chain,
// whose CTAs are dispatched first as SMs free up)
cudaStream_t side_stream(const DeviceState& st, int which) {
  if (which < 0 || which > 2) return nullptr;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_side[which][st.device]) {
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) return nullptr;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, which == 1 ? greatest : least) != cudaSuccess)
      return nullptr;
    g_side[which][st.device] = s;
  }
  return g_side[which][st.device];
}

// optional per-stage CUDA events (bf_stage_events): recorded on the launching stream around each stage
static cudaEvent_t g_stage_ev[2 * BF_MAX_STAGES];
static int g_stage_n = 0;

void stage_mark(int stage, int end, cudaStream_t stream) {
  if (stage < g_stage_n && g_stage_ev[2 * stage + end]) cudaEventRecord(g_stage_ev[2 * stage + end], stream);
}

}  // namespace bfb

using namespace bfb;

extern "C" {

const char* bf_last_cuda_error(void) {
  return g_last_cuda_error ? cudaGetErrorString((cudaError_t)g_last_cuda_error) : "no CUDA error recorded";
}

const char* bf_strerror(int code) {
  switch (code) {
    case BF_OK: return "ok";
    case BF_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, shape or size)";
    case BF_ERR_UNSUPPORTED: return "unsupported shape or configuration for this build";
    case BF_ERR_ALIGNMENT: return "pointer is not 16-byte aligned";
    case BF_ERR_WORKSPACE: return "workspace too small";
    case BF_ERR_CUDA: return "CUDA runtime error";
    case BF_ERR_TIMEOUT: return "a bounded device-side wait gave up";
    case BF_ERR_NO_DEVICE: return "no sm_100 device is current";
    default: return "unknown status";
  }
}

int bf_abi_version(void) { return BF_ABI_VERSION; }

int bf_device_error(unsigned int* word, bf_stream_t stream) {
  if (!word) return BF_ERR_INVALID_ARGUMENT;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return cuda_fail();
  unsigned int v[4] = {0u, 0u, 0u, 0u};
  if (cudaMemcpy(v, st.err, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return cuda_fail();
  for (int i = 0; i < 4; ++i) word[i] = v[i];
  if (v[0]) {
    const unsigned int zero[4] = {0u, 0u, 0u, 0u};
    if (cudaMemcpy(st.err, zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess) return cuda_fail();
  }
  return BF_OK;
}

int bf_stage_events(void* const* events, int n_stages) {
  if (n_stages < 0 || n_stages > BF_MAX_STAGES || (n_stages > 0 && !events)) return BF_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < 2 * BF_MAX_STAGES; ++i)
    g_stage_ev[i] = (i < 2 * n_stages) ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  g_stage_n = n_stages;
  return BF_OK;
}

int bf_gdn_decode_step(const float* q, const float* k, const void* v, int v_dtype, const float* g,
                       const float* beta, const float* s_in, float* s_out, float* o, int B, int G, int R,
                       int D, bf_stream_t stream) {
  if (!q || !k || !v || !g || !beta || !s_in || !s_out || !o) return BF_ERR_INVALID_ARGUMENT;
  if (B <= 0 || G <= 0 || R <= 0 || R > 8 || D <= 0 || D > 256 || (D % 32) != 0) return BF_ERR_INVALID_ARGUMENT;
  if (v_dtype != BF_F32 && v_dtype != BF_BF16) return BF_ERR_INVALID_ARGUMENT;
  if (!aligned16(s_in) || !aligned16(s_out)) return BF_ERR_ALIGNMENT;
  if ((long long)B * G > 65535) return BF_ERR_UNSUPPORTED;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  return launch_gdn_decode(q, k, v, v_dtype == BF_BF16, g, beta, s_in, s_out, o, B, G, R, D, stream);
}

}  // extern "C"
