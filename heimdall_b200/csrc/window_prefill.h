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
  // query tiles that the memory reads will mix (tile perm_tile0 + c, 0 <= c < perm_nch) go to o_perm instead of o:
  // tile (b, c, h) at o_perm + ((b * perm_nch + c) * H + h) * 128 * 256 floats, in the order the memory-read
  // epilogue loads it: [value half][64-column block][32-row group][float4 index][row in group][4]
  float* o_perm;
  int perm_tile0, perm_nch;
  unsigned int* err;
};

}  // namespace bfb
