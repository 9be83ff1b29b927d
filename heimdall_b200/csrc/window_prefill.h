// Argument block of the prefill window-attention kernel (window_prefill.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace bfb {

struct WinPreArgs {
  int B, H, G;
  int Tq;               // queries per (b, h); query i has position qpos0 + i
  int Tk;               // keys in the extended sequence; key j has position kpos0 + j
  int Tkp;              // padded key count of V^T (multiple of 64)
  int W;                // window
  long long qpos0, kpos0;
  long long klo;        // smallest position usable as a window key: max(sinks, first valid ring position)
  // sink keys/values (positions 0..ns-1), element strides per batch / KV head / key
  const __nv_bfloat16* sink_k;
  long long sk_b, sk_h, sk_k;
  const __nv_bfloat16* sink_v;
  long long sv_b, sv_h, sv_k;
  int ns;
  // outputs
  float* o;             // [B,Tq,H,D]
  float* lse;           // [B,H,Tq] or null
  // fused gate + mix (o_mem null: plain window output)
  const float* o_mem;   // [B,Tq,H,D]
  const float* mixx;    // [B,Tq,H]
  const float* mix_lse; // [H]
  const float* mem_scale;
  unsigned int* err;
};

}  // namespace bfb
