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
  // query tiles that the memory reads will mix (tile perm_tile0 + c, 0 <= c < perm_nch) go to o_perm instead of o,
  // in fp16: tile (b, c, h) at o_perm + ((b * perm_nch + c) * H + h) * 128 * 256 halves, in the order the
  // memory-read epilogue loads it: [value half][64-column block][32-row group][8-column group][row in group][8]
  __half* o_perm;
  int perm_tile0, perm_nch;
  // query tiles qt0 .. qt0 + nqt - 1 only (nqt = 0: all tiles); items of other tiles are not this launch's
  int qt0, nqt;
  unsigned int* err;
};

}  // namespace bfb
