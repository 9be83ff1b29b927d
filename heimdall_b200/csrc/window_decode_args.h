// Argument block of the decode window kernels (window_decode.cu), filled by layer_api.cu.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace bfb {

struct WinDecArgs {
  const __nv_bfloat16* qr;     // [B,H,D]   roped query of the new token
  const __nv_bfloat16* kr;     // [B,G,D]   roped key of the new token
  const __nv_bfloat16* v;      // [B,G,D]   value of the new token
  const __nv_bfloat16* ring_k; // [B,G,W,D]
  const __nv_bfloat16* ring_v; // [B,G,W,D]
  const int64_t* ring_pos;     // [W] or [B,W]
  long long ring_pos_bstride;  // 0 (shared) or W
  const __nv_bfloat16* sink_k; // [B,G,ns,D] or null
  const __nv_bfloat16* sink_v;
  int ns;
  const int64_t* pos;          // [B] position of the new token
  float* part;                 // workspace: [B*G][nsplit][R*(D+2)]
  int B, G, R, D, W, S, nsplit;
  // combine / epilogue
  const float* o_mem;          // [B,H,D] or null (memory off)
  const float* mixx;           // [B,H]
  const float* mix_lse;        // [H]
  const float* mem_scale;      // [H]
  float* o;                    // [B,H,D]
  float* lse_out;              // [B,H] or null
  // ring write (null ring_km = no write)
  const float* km;             // [B,G,D]
  const float* g_new;          // [B,G]
  const float* beta_new;       // [B,G]
  __nv_bfloat16* ring_k_w;
  __nv_bfloat16* ring_v_w;
  float* ring_km;              // [B,W,G,D]
  float* ring_g;               // [B,W,G]
  float* ring_beta;            // [B,W,G]
  int64_t* ring_pos_w;
};

}  // namespace bfb
