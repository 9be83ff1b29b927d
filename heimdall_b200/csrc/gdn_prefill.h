// Argument blocks of the chunked gated delta-rule prefill kernels (gdn_prefill.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace bfb {

constexpr int kGC = 128;   // chunk length of the GPU scan (tokens)
// parts of launch_gdn_prefill: P1 (per-chunk products), P2 (the recurrence), P3 (the reads; not in transform mode),
// FIX (sequence parallelism, second phase: the chunk-start states and corrected values from the incoming state,
// all chunks at once, from what the map pass stored)
constexpr int kGdnP1 = 1, kGdnP2 = 2, kGdnP3 = 4, kGdnAll = 7, kGdnFix = 8;
constexpr int kGD = 256;   // head dim (Dk == Dv)

// The write stream (step u writes one key/value into memory) and the read stream (step u reads with
// R query heads).  Write step u comes from the ring when u < nring (ring position ring_pos0 + u,
// a no-op when that slot is not valid) and otherwise from new token u - nring; read step u is query
// u + qoff.  Steps >= n_steps are padding (no-ops).
struct GdnStreams {
  int B, G, R, T;              // T = new tokens per sequence
  int n_steps, n_pad, n_chunks;
  int nring, W, qoff;
  long long ring_pos0;
  const float* km;             // [B,T,G,D] fp32
  const __nv_bfloat16* v;      // [B,T,G,D] bf16 values (or null when v32 is set)
  const float* v32;            // [B,T,G,D] fp32 values (optional)
  const float* g;              // [B,T,G]
  const float* beta;           // [B,T,G]
  const float* ring_km;        // [B,W,G,D]
  const __nv_bfloat16* ring_v; // [B,G,W,D]
  const float* ring_g;         // [B,W,G]
  const float* ring_beta;      // [B,W,G]
  const int64_t* ring_pos;     // [W]
  // per-chunk products (workspace)
  __half* kw;                  // [B,G,n_pad,D]   write keys (fp16)
  __half* w;                   // [B,G,n_pad,D]   T (beta e^gc k)
  __half* u;                   // [B,G,n_pad,D]   T (beta v)
  float* gc;                   // [B,G,n_pad]     cumulative log-decay inside the chunk
  __half* ST;                  // [B,G,n_chunks,D(dv),D(dk)]  state at chunk start, transposed
  __half* VT;                  // [B,G,n_chunks,D(dv),kGC]    v_new, transposed
  const float* s0;             // [B,G,D,D] or null
  float* s_out;                // [B,G,D,D]
  const __half* qm;            // [B,T,H,D] fp16 (read queries, unit-norm * D^-1/2)
  float* o;                    // [B,T,H,D] memory read of query u + qoff
  // segment-transform mode (m_out != null): no reads; P2 also runs the recurrence from the identity with
  // zero inputs, whose final value is the segment's state map M (S_out = M S_in + N), and writes it here
  float* m_out;                // [B,G,D,D]
  // sequence parallelism with a fix-up phase (MC != null, with m_out in the map pass): the map pass also keeps,
  // per chunk, the chunk-start state from a zero incoming state (ST) with its corrected values (VT), and the
  // chunk-start transition M_c (state at chunk c = M_c S_in + N_c), fp16 row-major [k][j]; the fix-up (kGdnFix)
  // reads them with the incoming state s0, transposed to fp16 in SinT, and rewrites ST and VT in place
  __half* MC;                  // [B,G,n_chunks,D,D]
  __half* SinT;                // [B,G,D(dv),D(dk)]
  // packed variable-length sequences (chunk_tok0 != null; B = 1, no ring, qoff = 0): global chunk c holds
  // packed tokens chunk_tok0[c] .. + chunk_len[c] - 1 of one sequence; sequence i owns chunks
  // seq_chunk0[i] .. seq_chunk0[i+1] - 1 (seq_chunk0[n_seq] = number of chunks); states are per sequence
  const int* chunk_tok0;
  const int* chunk_len;
  const int* seq_chunk0;
  int n_seq;
  // fused gate and mix (mix != 0; then o is the layer output holding the window result o_win): the memory
  // read of a query at position p >= W becomes o = o_win + gamma (mem_scale o_mem - o_win) in place, with
  // gamma = sigmoid(mixx + mix_lse (lse - ln W)); rows below W keep o_win
  int mix;
  long long pos0;              // position of token 0 of each sequence
  const float* lse;            // [B,H,T] window log-sum-exp
  const float* mixx;           // [B,T,H]
  const float* mix_lse;        // [H]
  const float* mem_scale;      // [H]
  // with mix: the window result of the rows this kernel reads, per (b, chunk, head) tile of 128 x 256 fp16 in
  // the order of the epilogue's loads (null: the window result is read from o itself)
  const __half* owin;
  // P3 over chunks p3_c0 .. p3_c1 - 1 only (p3_c1 = 0: all chunks; not with packed sequences)
  int p3_c0, p3_c1;
  unsigned int* err;
};

}  // namespace bfb
