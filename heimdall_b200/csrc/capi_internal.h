// Internal declarations shared by the .cu files behind the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define BF_ABI_VERSION 1

namespace bfb {

struct DeviceState {
  int device;
  unsigned int* err;  // device error word of this device
  int sm_count;
};

int device_state(DeviceState* st);
bool aligned16(const void* p);

int launch_gdn_decode(const float* q, const float* k, const void* v, int v_bf16, const float* g,
                      const float* beta, const float* s_in, float* s_out, float* o, int B, int G, int R, int D,
                      cudaStream_t stream);

}  // namespace bfb
