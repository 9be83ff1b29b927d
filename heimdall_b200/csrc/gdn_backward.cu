// Backward of the GQA gated delta rule: the gradients that torch autograd takes through
// heimdall/motor.py:70-102 (delta_rule_gqa) when seq_loss (motor.py:149-193) trains a converted layer.
//
// Forward, per token t and KV head (state S [Dk, Dv]; the Dv value columns never interact):
//   S~ = a S_{t-1} (a = e^{g_t}),   e = v_t - S~^T k_t,   S_t = S~ + beta_t k_t e^T,   o_{t,r} = S_t^T q_{t,r}.
// Backward, tokens in reverse, dS = dL/dS_t gathered from the later tokens (dL/dS_T at the end):
//   dS += sum_r q_{t,r} do_{t,r}^T                         dq_{t,r} = S_t do_{t,r}
//   kds = dS^T k_t,  de = beta kds,  dv_t = de,             dbeta_t = e . kds
//   dk_t = beta dS e - S~ de,  dS~ = dS - k de^T,           dg_t = <dS~, S~>,   dS_{t-1} = a dS~
// and dL/dS_0 = dS after token 0.  Everything is fp32.
//
// gdn_bwd_kernel: one CTA per (sequence, KV head, kGB_Cols value columns), one warp per kGB_WCols columns, lane l
// holding key rows 4l..4l+3 and 128+4l..128+4l+3 of them.  The token recurrence is sequential, so a warp's
// dependent chain per token is what bounds the kernel: the work splits into as many warps as there are value
// columns (one column per warp), each warp's chain short, the SMs' schedulers given independent warps.  The
// recurrences of S and dS stay inside the warp (their row sums are warp reductions); the outputs that sum over
// value columns (dq, dk, dbeta, dg) leave each token as one partial per CTA, reduced across the CTA's warps in
// shared memory (one barrier per token, double-buffered), and gdn_bwd_reduce_kernel adds the CTAs' partials.
// States: a first forward pass stores the state at every 64-token chunk start (fp32, CTA-private); the backward
// walks the chunks in reverse, recomputes the chunk's states into a CTA-private scratch (L2-resident at training
// sizes), then walks its tokens in reverse.  The forward passes read a whole chunk's k, v, g, beta from shared
// memory (one cp.async batch per chunk); the reverse walk stages each token's q, k, do two tokens ahead in a
// three-slot cp.async ring and loads the next state while it computes.
#include "bifrost_b200.h"
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

constexpr int kGB_D = 256;
constexpr int kGB_Warps = 8;
constexpr int kGB_Threads = 32 * kGB_Warps;
constexpr int kGB_WCols = 1;                        // value columns per warp
constexpr int kGB_Cols = kGB_Warps * kGB_WCols;     // per CTA
constexpr int kGB_Chunk = 64;                       // tokens per checkpoint
constexpr int kGB_MaxR = 8;
constexpr int kGB_LaneF = 8 * kGB_WCols;            // floats of one lane's state block
constexpr int kGB_SliceF = kGB_D * kGB_Cols;        // floats of one CTA's state slice
constexpr int kGB_Emax = (kGB_MaxR + 1) * kGB_D + 4;  // partial row (dq R x D, dk D, dbeta, dg), padded
constexpr int kGB_Stage = kGB_MaxR * kGB_D + kGB_D + kGB_MaxR * kGB_Cols + 4;   // q, k, do slice, (g, beta)
static_assert(kGB_LaneF % 4 == 0 && kGB_Cols % 4 == 0, "whole 16-byte vectors");
static_assert(kGB_Stage % 4 == 0 && kGB_Emax % 4 == 0, "16-byte aligned shared-memory rows");

struct GdnBwdArgs {
  const float* q;      // [B, T, G, R, D]
  const float* k;      // [B, T, G, D]
  const float* v;      // [B, T, G, D]
  const float* g;      // [B, T, G]
  const float* beta;   // [B, T, G]
  const float* s0;     // [B, G, D, D] or null
  const float* dout;   // [B, T, G, R, D]
  const float* dsT;    // [B, G, D, D] or null
  float* dv;           // [B, T, G, D]
  float* ds0;          // [B, G, D, D]
  float* ckpt;         // [B*G, ncta, nchunk, slice]
  float* scr;          // [B*G, ncta, kGB_Chunk, slice]
  float* escr;         // [B*G, ncta, kGB_Chunk, kGB_Cols]
  float* part;         // [B*G, T, ncta, E]
  int B, T, G, R, ncta, nchunk, E;
};

typedef float GbBlock[8][kGB_WCols];   // one lane's 8 rows x the warp's columns

// a lane's block in a CTA slice stored as [warp][lane][8 rows][columns]: contiguous per lane
__device__ __forceinline__ void gb_load_slice(const float* base, int warp, int lane, GbBlock& s) {
  const float4* p = reinterpret_cast<const float4*>(base + (warp * 32 + lane) * kGB_LaneF);
  float f[kGB_LaneF];
#pragma unroll
  for (int i = 0; i < kGB_LaneF / 4; ++i) {
    const float4 x = __ldcg(p + i);
    f[4 * i] = x.x; f[4 * i + 1] = x.y; f[4 * i + 2] = x.z; f[4 * i + 3] = x.w;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c) s[i][c] = f[i * kGB_WCols + c];
}
__device__ __forceinline__ void gb_store_slice(float* base, int warp, int lane, const GbBlock& s) {
  float4* p = reinterpret_cast<float4*>(base + (warp * 32 + lane) * kGB_LaneF);
  float f[kGB_LaneF];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c) f[i * kGB_WCols + c] = s[i][c];
#pragma unroll
  for (int i = 0; i < kGB_LaneF / 4; ++i)
    __stcg(p + i, make_float4(f[4 * i], f[4 * i + 1], f[4 * i + 2], f[4 * i + 3]));
}
// key row of this lane's i-th state row: 4l + j and 128 + 4l + j (j < 4), so that 16-byte accesses to row
// vectors are contiguous across the warp (no shared-memory bank conflicts)
__device__ __forceinline__ int gb_row(int lane, int i) { return 128 * (i >> 2) + 4 * lane + (i & 3); }

// this lane's rows, the warp's columns of a row-major [D, D] state (s0 / dsT)
__device__ __forceinline__ void gb_load_dense(const float* m, int lane, int col, GbBlock& s) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c) s[i][c] = m[(size_t)gb_row(lane, i) * kGB_D + col + c];
}
__device__ __forceinline__ void gb_zero(GbBlock& s) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c) s[i][c] = 0.f;
}

__device__ __forceinline__ float gb_allsum(float x) {
#pragma unroll
  for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// forward inputs of up to 64 tokens in shared memory: k rows, this CTA's v columns, g, beta
struct GbFwdStage {
  float k[kGB_Chunk][kGB_D];
  float v[kGB_Chunk][kGB_Cols];
  float g[kGB_Chunk], beta[kGB_Chunk];
};
// stage tokens t0 .. t0 + n - 1 (all threads; returns after a barrier with the data visible)
__device__ __forceinline__ void gb_stage_forward(const GdnBwdArgs& A, int b, int g, int t0, int n, int col0,
                                                 GbFwdStage* fs) {
  const int tid = threadIdx.x;
  for (int f = tid; f < n * (kGB_D / 4); f += kGB_Threads) {
    const int tt = f / (kGB_D / 4), x = f % (kGB_D / 4);
    cp_async16(&fs->k[tt][4 * x], A.k + (((size_t)b * A.T + t0 + tt) * A.G + g) * kGB_D + 4 * x);
  }
  for (int f = tid; f < n * (kGB_Cols / 4); f += kGB_Threads) {
    const int tt = f / (kGB_Cols / 4), x = f % (kGB_Cols / 4);
    cp_async16(&fs->v[tt][4 * x], A.v + (((size_t)b * A.T + t0 + tt) * A.G + g) * kGB_D + col0 + 4 * x);
  }
  if (tid < n) {
    const size_t tg = ((size_t)b * A.T + t0 + tid) * A.G + g;
    cp_async4(&fs->g[tid], A.g + tg);
    cp_async4(&fs->beta[tid], A.beta + tg);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
}

// one staged forward token on this lane's block: S = a S; e = v - S^T k; S += beta k e^T.  e -> e_out.
__device__ __forceinline__ void gb_forward_staged(GbBlock& s, const GbFwdStage* fs, int tt, int lane, int warp,
                                                  float (&e_out)[kGB_WCols]) {
  const float4 k0 = *reinterpret_cast<const float4*>(&fs->k[tt][4 * lane]);
  const float4 k1 = *reinterpret_cast<const float4*>(&fs->k[tt][128 + 4 * lane]);
  const float kr[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
  const float a = expf(fs->g[tt]), bt = fs->beta[tt];
  float dot[kGB_WCols];
#pragma unroll
  for (int c = 0; c < kGB_WCols; ++c) dot[c] = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c) {
      s[i][c] *= a;
      dot[c] = fmaf(kr[i], s[i][c], dot[c]);
    }
#pragma unroll
  for (int c = 0; c < kGB_WCols; ++c) e_out[c] = fs->v[tt][warp * kGB_WCols + c] - gb_allsum(dot[c]);
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c) s[i][c] = fmaf(bt * kr[i], e_out[c], s[i][c]);
}

// cp.async token t's backward inputs (q rows, k, this CTA's do columns, raw g and beta) into stg
__device__ __forceinline__ void gb_stage_backward(const GdnBwdArgs& A, int b, int g, int t, int col0, float* stg) {
  const int tid = threadIdx.x;
  const size_t tg = ((size_t)b * A.T + t) * A.G + g;
  const int nq = A.R * (kGB_D / 4), nk = kGB_D / 4, nd = A.R * (kGB_Cols / 4);
  for (int f = tid; f < nq + nk + nd; f += kGB_Threads) {
    if (f < nq) {
      cp_async16(stg + 4 * f, A.q + tg * A.R * kGB_D + 4 * f);
    } else if (f < nq + nk) {
      const int x = f - nq;
      cp_async16(stg + kGB_MaxR * kGB_D + 4 * x, A.k + tg * kGB_D + 4 * x);
    } else {
      const int y = f - nq - nk, r = y / (kGB_Cols / 4), x = y % (kGB_Cols / 4);
      cp_async16(stg + kGB_MaxR * kGB_D + kGB_D + r * kGB_Cols + 4 * x,
                 A.dout + (tg * A.R + r) * kGB_D + col0 + 4 * x);
    }
  }
  if (tid == 0) {
    cp_async4(stg + kGB_Stage - 4, A.g + tg);
    cp_async4(stg + kGB_Stage - 3, A.beta + tg);
  }
}

template <int R>
__global__ void __launch_bounds__(kGB_Threads, 1) gdn_bwd_kernel(GdnBwdArgs A) {
  extern __shared__ __align__(16) float gb_smem[];
  float* s_part = gb_smem;                              // [2][warps][Emax]
  float* s_stage = gb_smem + 2 * kGB_Warps * kGB_Emax;  // [3][kGB_Stage]; the forward stage aliases both
  GbFwdStage* fs = reinterpret_cast<GbFwdStage*>(s_part);
  const int bg = blockIdx.x, b = bg / A.G, g = bg % A.G, cta = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col0 = cta * kGB_Cols, col = col0 + warp * kGB_WCols;
  const size_t slice_cta = (size_t)bg * A.ncta + cta;
  float* ckpt = A.ckpt + slice_cta * A.nchunk * kGB_SliceF;
  float* scr = A.scr + slice_cta * kGB_Chunk * kGB_SliceF;
  float* escr = A.escr + slice_cta * kGB_Chunk * kGB_Cols;
  const int T = A.T;
  float e[kGB_WCols];

  // ---- forward: the state at every chunk start
  GbBlock s;
  if (A.s0) gb_load_dense(A.s0 + (size_t)bg * kGB_D * kGB_D, lane, col, s);
  else gb_zero(s);
  for (int ch = 0; ch < A.nchunk; ++ch) {
    const int t0 = ch * kGB_Chunk, n = min(kGB_Chunk, T - t0);
    gb_store_slice(ckpt + (size_t)ch * kGB_SliceF, warp, lane, s);
    __syncthreads();   // the previous chunk's stage is consumed
    gb_stage_forward(A, b, g, t0, n, col0, fs);
    for (int tt = 0; tt < n; ++tt) gb_forward_staged(s, fs, tt, lane, warp, e);
  }

  // ---- backward, chunk by chunk in reverse
  GbBlock ds;
  if (A.dsT) gb_load_dense(A.dsT + (size_t)bg * kGB_D * kGB_D, lane, col, ds);
  else gb_zero(ds);
  const int E = A.E;
  for (int ch = A.nchunk - 1; ch >= 0; --ch) {
    const int t0 = ch * kGB_Chunk, n = min(kGB_Chunk, T - t0);
    const float* ck = ckpt + (size_t)ch * kGB_SliceF;
    // recompute the chunk's states (after each token) and errors e
    __syncthreads();   // the previous chunk's buffers (aliased by the forward stage) are consumed
    gb_stage_forward(A, b, g, t0, n, col0, fs);
    gb_load_slice(ck, warp, lane, s);
    for (int tt = 0; tt < n; ++tt) {
      gb_forward_staged(s, fs, tt, lane, warp, e);
      gb_store_slice(scr + (size_t)tt * kGB_SliceF, warp, lane, s);
      if (lane == 0) {
#pragma unroll
        for (int c = 0; c < kGB_WCols; ++c) __stcg(escr + tt * kGB_Cols + warp * kGB_WCols + c, e[c]);
      }
    }
    // the reverse walk's first two tokens' inputs; iteration it (token t0 + n - 1 - it) reads stage it % 3
    __syncthreads();   // the forward stage (aliasing the ring) is consumed; escr visible to each warp
    gb_stage_backward(A, b, g, t0 + n - 1, col0, s_stage);
    cp_async_commit();
    if (n > 1) gb_stage_backward(A, b, g, t0 + n - 2, col0, s_stage + kGB_Stage);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();   // stage 0 visible
    GbBlock st, sp;
    gb_load_slice(scr + (size_t)(n - 1) * kGB_SliceF, warp, lane, st);
    gb_load_slice(n > 1 ? scr + (size_t)(n - 2) * kGB_SliceF : ck, warp, lane, sp);
    float ecur[kGB_WCols];
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c) ecur[c] = __ldcg(escr + (n - 1) * kGB_Cols + warp * kGB_WCols + c);
    for (int it = 0; it < n; ++it) {
      const int tt = n - 1 - it, t = t0 + tt;
      const float* stg = s_stage + (it % 3) * kGB_Stage;
      float* prt = s_part + (it & 1) * kGB_Warps * kGB_Emax + warp * kGB_Emax;
      // token t - 2's inputs, two iterations ahead (one commit group per iteration, possibly empty)
      if (it + 2 < n) gb_stage_backward(A, b, g, t - 2, col0, s_stage + ((it + 2) % 3) * kGB_Stage);
      cp_async_commit();
      GbBlock nx;
      float enx[kGB_WCols];
      if (tt > 0) {
        gb_load_slice(tt > 1 ? scr + (size_t)(tt - 2) * kGB_SliceF : ck, warp, lane, nx);
#pragma unroll
        for (int c = 0; c < kGB_WCols; ++c) enx[c] = __ldcg(escr + (tt - 1) * kGB_Cols + warp * kGB_WCols + c);
      } else {
        gb_zero(nx);
#pragma unroll
        for (int c = 0; c < kGB_WCols; ++c) enx[c] = 0.f;
      }
      const float a = expf(stg[kGB_Stage - 4]), bt = stg[kGB_Stage - 3];
      const float4 k0 = *reinterpret_cast<const float4*>(stg + kGB_MaxR * kGB_D + 4 * lane);
      const float4 k1 = *reinterpret_cast<const float4*>(stg + kGB_MaxR * kGB_D + 128 + 4 * lane);
      const float kr[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
      // dS += q do^T; dq partial = S_t do
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float4 q0 = *reinterpret_cast<const float4*>(stg + r * kGB_D + 4 * lane);
        const float4 q1 = *reinterpret_cast<const float4*>(stg + r * kGB_D + 128 + 4 * lane);
        const float qr[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float dv[kGB_WCols];
#pragma unroll
        for (int c = 0; c < kGB_WCols; ++c)
          dv[c] = stg[kGB_MaxR * kGB_D + kGB_D + r * kGB_Cols + warp * kGB_WCols + c];
        float dq[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          dq[i] = 0.f;
#pragma unroll
          for (int c = 0; c < kGB_WCols; ++c) {
            ds[i][c] = fmaf(qr[i], dv[c], ds[i][c]);
            dq[i] = fmaf(st[i][c], dv[c], dq[i]);
          }
        }
        *reinterpret_cast<float4*>(prt + r * kGB_D + 4 * lane) = make_float4(dq[0], dq[1], dq[2], dq[3]);
        *reinterpret_cast<float4*>(prt + r * kGB_D + 128 + 4 * lane) = make_float4(dq[4], dq[5], dq[6], dq[7]);
      }
      // kds = dS^T k; de = beta kds; dbeta = e . kds
      float kds[kGB_WCols], de[kGB_WCols], dbeta = 0.f;
#pragma unroll
      for (int c = 0; c < kGB_WCols; ++c) {
        float x = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) x = fmaf(kr[i], ds[i][c], x);
        kds[c] = gb_allsum(x);
        de[c] = bt * kds[c];
        dbeta = fmaf(ecur[c], kds[c], dbeta);
      }
      if (lane == 0) {
#pragma unroll
        for (int c = 0; c < kGB_WCols; ++c) A.dv[(((size_t)b * T + t) * A.G + g) * kGB_D + col + c] = de[c];
      }
      // dk partial = beta dS e - S~ de;  dS~ = dS - k de^T;  dg = <dS~, S~>;  dS_{t-1} = a dS~
      float dk[8], dg = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float x = 0.f, y = 0.f;
#pragma unroll
        for (int c = 0; c < kGB_WCols; ++c) {
          const float stl = a * sp[i][c];
          x = fmaf(ds[i][c], ecur[c], x);
          y = fmaf(stl, de[c], y);
          const float dst = fmaf(-kr[i], de[c], ds[i][c]);
          dg = fmaf(dst, stl, dg);
          ds[i][c] = a * dst;
        }
        dk[i] = bt * x - y;
      }
      dg = gb_allsum(dg);
      *reinterpret_cast<float4*>(prt + R * kGB_D + 4 * lane) = make_float4(dk[0], dk[1], dk[2], dk[3]);
      *reinterpret_cast<float4*>(prt + R * kGB_D + 128 + 4 * lane) = make_float4(dk[4], dk[5], dk[6], dk[7]);
      if (lane == 0) {
        prt[(R + 1) * kGB_D] = dbeta;
        prt[(R + 1) * kGB_D + 1] = dg;
      }
      cp_async_wait<1>();   // the next token's stage (issued an iteration ago) has landed
      __syncthreads();
      {
        const float* pall = s_part + (it & 1) * kGB_Warps * kGB_Emax;
        float* out = A.part + (((size_t)bg * T + t) * A.ncta + cta) * E;
#pragma unroll 2
        for (int x = tid; x < E; x += kGB_Threads) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kGB_Warps; ++w) acc += pall[w * kGB_Emax + x];
          __stcg(out + x, acc);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < kGB_WCols; ++c) {
          st[i][c] = sp[i][c];
          sp[i][c] = nx[i][c];
        }
#pragma unroll
      for (int c = 0; c < kGB_WCols; ++c) ecur[c] = enx[c];
    }
  }
  cp_async_wait<0>();
  // dL/dS_0
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < kGB_WCols; ++c)
      A.ds0[(size_t)bg * kGB_D * kGB_D + (size_t)gb_row(lane, i) * kGB_D + col + c] = ds[i][c];
}

// grid (T, B * G): add the CTAs' partials of one token and scatter them into dq, dk, dbeta, dg
__global__ void __launch_bounds__(256) gdn_bwd_reduce_kernel(GdnBwdArgs A, float* dq, float* dk, float* dg,
                                                             float* dbeta) {
  const int t = blockIdx.x, bg = blockIdx.y, b = bg / A.G, g = bg % A.G;
  const float* src = A.part + ((size_t)bg * A.T + t) * A.ncta * A.E;
  const size_t tg = ((size_t)b * A.T + t) * A.G + g;
  const int RD = A.R * kGB_D;
  for (int x = threadIdx.x; x < A.E; x += 256) {
    float acc = 0.f;
#pragma unroll 8
    for (int c = 0; c < A.ncta; ++c) acc += __ldcs(src + (size_t)c * A.E + x);
    if (x < RD) dq[tg * RD + x] = acc;
    else if (x < RD + kGB_D) dk[tg * kGB_D + (x - RD)] = acc;
    else if (x == RD + kGB_D) dbeta[tg] = acc;
    else if (x == RD + kGB_D + 1) dg[tg] = acc;
  }
}

static int gb_smem_bytes() { return (2 * kGB_Warps * kGB_Emax + 3 * kGB_Stage) * 4; }
static_assert(sizeof(GbFwdStage) <= (2 * kGB_Warps * kGB_Emax + 3 * kGB_Stage) * 4,
              "the forward stage aliases the buffers");

static void gb_sizes(int B, int T, int G, int R, size_t& ckpt, size_t& scr, size_t& escr, size_t& part) {
  const size_t ncta = kGB_D / kGB_Cols, nchunk = (T + kGB_Chunk - 1) / kGB_Chunk, bg = (size_t)B * G;
  const size_t E = (size_t)(R + 1) * kGB_D + 2;
  auto al = [](size_t x) { return (x * 4 + 255) / 256 * 256; };
  ckpt = al(bg * ncta * nchunk * kGB_SliceF);
  scr = al(bg * ncta * kGB_Chunk * kGB_SliceF);
  escr = al(bg * ncta * kGB_Chunk * kGB_Cols);
  part = al(bg * T * ncta * E);
}

}  // namespace bfb

using namespace bfb;

extern "C" {

size_t bf_gdn_bwd_workspace(int B, int T, int G, int R, int D) {
  if (B <= 0 || T <= 0 || G <= 0 || R <= 0 || R > kGB_MaxR || D != kGB_D) return 0;
  size_t a, b, c, d;
  gb_sizes(B, T, G, R, a, b, c, d);
  return a + b + c + d;
}

int bf_gdn_bwd(const float* q, const float* k, const float* v, const float* g, const float* beta, const float* s0,
               const float* dout, const float* dstate, float* dq, float* dk, float* dv, float* dg, float* dbeta,
               float* ds0, int B, int T, int G, int R, int D, void* ws, size_t ws_bytes, bf_stream_t stream) {
  if (!q || !k || !v || !g || !beta || !dout || !dq || !dk || !dv || !dg || !dbeta || !ds0 || !ws || B <= 0 ||
      T <= 0 || G <= 0 || R <= 0)
    return BF_ERR_INVALID_ARGUMENT;
  if (D != kGB_D || R > kGB_MaxR) return BF_ERR_UNSUPPORTED;
  const size_t need = bf_gdn_bwd_workspace(B, T, G, R, D);
  if (ws_bytes < need) return BF_ERR_WORKSPACE;
  const void* al[] = {q, k, v, dout, dq, dk, dv, ds0, ws};
  for (const void* p : al)
    if (!aligned16(p)) return BF_ERR_ALIGNMENT;
  if ((s0 && !aligned16(s0)) || (dstate && !aligned16(dstate))) return BF_ERR_ALIGNMENT;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  size_t c_b, s_b, e_b, p_b;
  gb_sizes(B, T, G, R, c_b, s_b, e_b, p_b);
  GdnBwdArgs A{};
  A.q = q; A.k = k; A.v = v; A.g = g; A.beta = beta; A.s0 = s0; A.dout = dout; A.dsT = dstate;
  A.dv = dv; A.ds0 = ds0;
  char* w = static_cast<char*>(ws);
  A.ckpt = reinterpret_cast<float*>(w);
  A.scr = reinterpret_cast<float*>(w + c_b);
  A.escr = reinterpret_cast<float*>(w + c_b + s_b);
  A.part = reinterpret_cast<float*>(w + c_b + s_b + e_b);
  A.B = B; A.T = T; A.G = G; A.R = R;
  A.ncta = kGB_D / kGB_Cols;
  A.nchunk = (T + kGB_Chunk - 1) / kGB_Chunk;
  A.E = (R + 1) * kGB_D + 2;
  const int smem = gb_smem_bytes();
  switch (R) {
#define GB_CASE(RR)                                                                     \
  case RR:                                                                            \
    if ((rc = ensure_smem_attr((const void*)gdn_bwd_kernel<RR>, smem))) return rc;    \
    gdn_bwd_kernel<RR><<<dim3(B * G, A.ncta), kGB_Threads, smem, stream>>>(A);        \
    break;
    GB_CASE(1) GB_CASE(2) GB_CASE(3) GB_CASE(4) GB_CASE(5) GB_CASE(6) GB_CASE(7) GB_CASE(8)
#undef GB_CASE
    default: return BF_ERR_UNSUPPORTED;
  }
  if ((rc = launch_status())) return rc;
  gdn_bwd_reduce_kernel<<<dim3(T, B * G), 256, 0, stream>>>(A, dq, dk, dg, dbeta);
  return launch_status();
}

}  // extern "C"
