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
// gdn_bwd_kernel: one CTA per (sequence, KV head, 32 value columns), eight warps of four columns, lane l holding
// key rows 8l..8l+7 of them.  The recurrences of S and dS stay inside the CTA (their row sums are warp
// reductions); the outputs that sum over value columns (dq, dk, dbeta, dg) leave each token as one partial per
// CTA, reduced across the CTA's warps in shared memory (one barrier per token, double-buffered), and
// gdn_bwd_reduce_kernel adds the CTAs' partials.  States: a first forward pass stores the state at every 64-token
// chunk start (fp32, CTA-private); the backward walks the chunks in reverse, recomputes the chunk's states into a
// CTA-private scratch (L2-resident at training sizes), then walks its tokens in reverse.  Per token the next
// token's q, k, do are staged in shared memory and the next state loaded while the current token computes.
#include "bifrost_b200.h"
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

constexpr int kGB_D = 256;
constexpr int kGB_Warps = 8;
constexpr int kGB_WCols = 4;                        // value columns per warp
constexpr int kGB_Cols = kGB_Warps * kGB_WCols;     // per CTA
constexpr int kGB_Chunk = 64;                       // tokens per checkpoint
constexpr int kGB_MaxR = 8;
constexpr int kGB_SliceF = kGB_D * kGB_Cols;        // floats of one CTA's state slice
constexpr int kGB_Emax = (kGB_MaxR + 1) * kGB_D + 4;  // partial row (dq R x D, dk D, dbeta, dg), padded
constexpr int kGB_Stage = kGB_MaxR * kGB_D + kGB_D + kGB_MaxR * kGB_Cols + 4;   // q, k, do slice, (a, beta)

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

// this lane's part of a CTA state slice stored as [warp][row][4 columns]: 8 rows x 4 columns, 32 contiguous floats
__device__ __forceinline__ void gb_load_slice(const float* base, int warp, int lane, float (&s)[8][4]) {
  const float4* p = reinterpret_cast<const float4*>(base + warp * (kGB_D * kGB_WCols) + lane * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 x = __ldcg(p + i);
    s[i][0] = x.x; s[i][1] = x.y; s[i][2] = x.z; s[i][3] = x.w;
  }
}
__device__ __forceinline__ void gb_store_slice(float* base, int warp, int lane, const float (&s)[8][4]) {
  float4* p = reinterpret_cast<float4*>(base + warp * (kGB_D * kGB_WCols) + lane * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) __stcg(p + i, make_float4(s[i][0], s[i][1], s[i][2], s[i][3]));
}
// rows 8l..8l+7, columns col..col+3 of a row-major [D, D] state (s0 / dsT / ds0)
__device__ __forceinline__ void gb_load_dense(const float* m, int lane, int col, float (&s)[8][4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 x = *reinterpret_cast<const float4*>(m + (size_t)(8 * lane + i) * kGB_D + col);
    s[i][0] = x.x; s[i][1] = x.y; s[i][2] = x.z; s[i][3] = x.w;
  }
}

__device__ __forceinline__ float gb_allsum(float x) {
#pragma unroll
  for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// one forward token on this lane's 8 x 4 block: S = a S; e = v - S^T k; S += beta k e^T.  Returns e (4 columns).
__device__ __forceinline__ float4 gb_forward_token(float (&s)[8][4], const float4 (&k)[2], float4 v, float a,
                                                   float bt) {
  const float kr[8] = {k[0].x, k[0].y, k[0].z, k[0].w, k[1].x, k[1].y, k[1].z, k[1].w};
  float dot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      s[i][c] *= a;
      dot[c] = fmaf(kr[i], s[i][c], dot[c]);
    }
#pragma unroll
  for (int c = 0; c < 4; ++c) dot[c] = gb_allsum(dot[c]);
  const float e[4] = {v.x - dot[0], v.y - dot[1], v.z - dot[2], v.w - dot[3]};
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) s[i][c] = fmaf(bt * kr[i], e[c], s[i][c]);
  return make_float4(e[0], e[1], e[2], e[3]);
}

struct GbTokIn {   // one token's forward inputs for this lane
  float4 k[2];
  float4 v;
  float a, bt;
};
__device__ __forceinline__ void gb_load_tok(const GdnBwdArgs& A, int b, int g, int t, int lane, int col,
                                            GbTokIn& in) {
  const size_t tg = ((size_t)b * A.T + t) * A.G + g;
  const float4* kp = reinterpret_cast<const float4*>(A.k + tg * kGB_D + 8 * lane);
  in.k[0] = __ldg(kp);
  in.k[1] = __ldg(kp + 1);
  in.v = __ldg(reinterpret_cast<const float4*>(A.v + tg * kGB_D + col));
  in.a = expf(__ldg(A.g + tg));
  in.bt = __ldg(A.beta + tg);
}

// the f-th float4 of token t's staged backward inputs (q rows, k, the CTA's do columns) and where it goes
__device__ __forceinline__ bool gb_stage_src(const GdnBwdArgs& A, int b, int g, int t, int col0, int f,
                                             const float4*& src, int& dst) {
  const size_t tg = ((size_t)b * A.T + t) * A.G + g;
  const int nq = A.R * (kGB_D / 4);
  if (f < nq) {
    src = reinterpret_cast<const float4*>(A.q + tg * A.R * kGB_D) + f;
    dst = 4 * f;
    return true;
  }
  f -= nq;
  if (f < kGB_D / 4) {
    src = reinterpret_cast<const float4*>(A.k + tg * kGB_D) + f;
    dst = kGB_MaxR * kGB_D + 4 * f;
    return true;
  }
  f -= kGB_D / 4;
  if (f < A.R * (kGB_Cols / 4)) {
    const int r = f / (kGB_Cols / 4), x = f % (kGB_Cols / 4);
    src = reinterpret_cast<const float4*>(A.dout + (tg * A.R + r) * kGB_D + col0) + x;
    dst = kGB_MaxR * kGB_D + kGB_D + r * kGB_Cols + 4 * x;
    return true;
  }
  return false;
}

__global__ void __launch_bounds__(256, 1) gdn_bwd_kernel(GdnBwdArgs A) {
  extern __shared__ __align__(16) float gb_smem[];
  float* s_part = gb_smem;                              // [2][8 warps][Emax]
  float* s_stage = gb_smem + 2 * kGB_Warps * kGB_Emax;  // [2][kGB_Stage]
  const int bg = blockIdx.x, b = bg / A.G, g = bg % A.G, cta = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int col0 = cta * kGB_Cols, col = col0 + warp * kGB_WCols;
  const size_t slice_cta = (size_t)bg * A.ncta + cta;
  float* ckpt = A.ckpt + slice_cta * A.nchunk * kGB_SliceF;
  float* scr = A.scr + slice_cta * kGB_Chunk * kGB_SliceF;
  float* escr = A.escr + slice_cta * kGB_Chunk * kGB_Cols;
  const int T = A.T;

  // ---- forward: the state at every chunk start
  float s[8][4];
  if (A.s0) {
    gb_load_dense(A.s0 + (size_t)bg * kGB_D * kGB_D, lane, col, s);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
  }
  {
    GbTokIn cur, nxt;
    gb_load_tok(A, b, g, 0, lane, col, cur);
    nxt = cur;
    for (int t = 0; t < T; ++t) {
      if (t % kGB_Chunk == 0) gb_store_slice(ckpt + (size_t)(t / kGB_Chunk) * kGB_SliceF, warp, lane, s);
      if (t + 1 < T) gb_load_tok(A, b, g, t + 1, lane, col, nxt);
      gb_forward_token(s, cur.k, cur.v, cur.a, cur.bt);
      cur = nxt;
    }
  }

  // ---- backward, chunk by chunk in reverse
  float ds[8][4];
  if (A.dsT) {
    gb_load_dense(A.dsT + (size_t)bg * kGB_D * kGB_D, lane, col, ds);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) ds[i][c] = 0.f;
  }
  const int E = A.E, R = A.R;
  const int nstage = R * (kGB_D / 4) + kGB_D / 4 + R * (kGB_Cols / 4);
  for (int ch = A.nchunk - 1; ch >= 0; --ch) {
    const int t0 = ch * kGB_Chunk, n = min(kGB_Chunk, T - t0);
    const float* ck = ckpt + (size_t)ch * kGB_SliceF;
    // recompute the chunk's states (after each token) and errors e
    gb_load_slice(ck, warp, lane, s);
    {
      GbTokIn cur, nxt;
      gb_load_tok(A, b, g, t0, lane, col, cur);
      nxt = cur;
      for (int tt = 0; tt < n; ++tt) {
        if (tt + 1 < n) gb_load_tok(A, b, g, t0 + tt + 1, lane, col, nxt);
        const float4 e = gb_forward_token(s, cur.k, cur.v, cur.a, cur.bt);
        gb_store_slice(scr + (size_t)tt * kGB_SliceF, warp, lane, s);
        if (lane == 0) __stcg(reinterpret_cast<float4*>(escr + tt * kGB_Cols + warp * kGB_WCols), e);
        cur = nxt;
      }
    }
    // stage the last token's inputs; S_t and S_{t-1}
    {
      const int t = t0 + n - 1;
      for (int f = tid; f < nstage; f += 256) {
        const float4* src;
        int dst;
        if (gb_stage_src(A, b, g, t, col0, f, src, dst))
          *reinterpret_cast<float4*>(s_stage + ((n - 1) & 1) * kGB_Stage + dst) = __ldg(src);
      }
      if (tid == 0) {
        const size_t tg = ((size_t)b * T + t) * A.G + g;
        s_stage[((n - 1) & 1) * kGB_Stage + kGB_Stage - 4] = expf(A.g[tg]);
        s_stage[((n - 1) & 1) * kGB_Stage + kGB_Stage - 3] = A.beta[tg];
      }
    }
    __syncthreads();   // stage visible; escr written by lane 0 of each warp visible to its warp
    float st[8][4], sp[8][4];
    gb_load_slice(scr + (size_t)(n - 1) * kGB_SliceF, warp, lane, st);
    gb_load_slice(n > 1 ? scr + (size_t)(n - 2) * kGB_SliceF : ck, warp, lane, sp);
    float4 ecur = __ldcg(reinterpret_cast<const float4*>(escr + (n - 1) * kGB_Cols + warp * kGB_WCols));
    for (int tt = n - 1; tt >= 0; --tt) {
      const int t = t0 + tt, buf = tt & 1;
      const float* stg = s_stage + buf * kGB_Stage;
      float* prt = s_part + buf * kGB_Warps * kGB_Emax + warp * kGB_Emax;
      // issue the next token's loads first
      float4 pre[3];
      int pdst[3];
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        pdst[u] = -1;
        const float4* src;
        int dst;
        if (tt > 0 && gb_stage_src(A, b, g, t - 1, col0, tid + 256 * u, src, dst)) {
          pre[u] = __ldg(src);
          pdst[u] = dst;
        }
      }
      float pa = 0.f, pb = 0.f;
      if (tt > 0 && tid == 0) {
        const size_t tg = ((size_t)b * T + t - 1) * A.G + g;
        pa = expf(A.g[tg]);
        pb = A.beta[tg];
      }
      float nx[8][4];
      float4 enx = make_float4(0.f, 0.f, 0.f, 0.f);
      if (tt > 0) {
        gb_load_slice(tt > 1 ? scr + (size_t)(tt - 2) * kGB_SliceF : ck, warp, lane, nx);
        enx = __ldcg(reinterpret_cast<const float4*>(escr + (tt - 1) * kGB_Cols + warp * kGB_WCols));
      }
      const float a = stg[kGB_Stage - 4], bt = stg[kGB_Stage - 3];
      const float4 k0 = *reinterpret_cast<const float4*>(stg + kGB_MaxR * kGB_D + 8 * lane);
      const float4 k1 = *reinterpret_cast<const float4*>(stg + kGB_MaxR * kGB_D + 8 * lane + 4);
      const float kr[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
      const float e[4] = {ecur.x, ecur.y, ecur.z, ecur.w};
      // dS += q do^T; dq partial = S_t do
      for (int r = 0; r < R; ++r) {
        const float4 q0 = *reinterpret_cast<const float4*>(stg + r * kGB_D + 8 * lane);
        const float4 q1 = *reinterpret_cast<const float4*>(stg + r * kGB_D + 8 * lane + 4);
        const float4 dd = *reinterpret_cast<const float4*>(stg + kGB_MaxR * kGB_D + kGB_D + r * kGB_Cols +
                                                           warp * kGB_WCols);
        const float qr[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const float dv[4] = {dd.x, dd.y, dd.z, dd.w};
        float dq[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          dq[i] = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            ds[i][c] = fmaf(qr[i], dv[c], ds[i][c]);
            dq[i] = fmaf(st[i][c], dv[c], dq[i]);
          }
        }
        float4* dqp = reinterpret_cast<float4*>(prt + r * kGB_D + 8 * lane);
        dqp[0] = make_float4(dq[0], dq[1], dq[2], dq[3]);
        dqp[1] = make_float4(dq[4], dq[5], dq[6], dq[7]);
      }
      // kds = dS^T k; de = beta kds; dbeta = e . kds
      float kds[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) kds[c] = fmaf(kr[i], ds[i][c], kds[c]);
#pragma unroll
      for (int c = 0; c < 4; ++c) kds[c] = gb_allsum(kds[c]);
      float de[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) de[c] = bt * kds[c];
      const float dbeta = e[0] * kds[0] + e[1] * kds[1] + e[2] * kds[2] + e[3] * kds[3];
      if (lane == 0)
        *reinterpret_cast<float4*>(A.dv + (((size_t)b * T + t) * A.G + g) * kGB_D + col) =
            make_float4(de[0], de[1], de[2], de[3]);
      // dk partial = beta dS e - S~ de;  dS~ = dS - k de^T;  dg = <dS~, S~>;  dS_{t-1} = a dS~
      float dk[8], dg = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float x = 0.f, y = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float stl = a * sp[i][c];
          x = fmaf(ds[i][c], e[c], x);
          y = fmaf(stl, de[c], y);
          const float dst = fmaf(-kr[i], de[c], ds[i][c]);
          dg = fmaf(dst, stl, dg);
          ds[i][c] = a * dst;
        }
        dk[i] = bt * x - y;
      }
      dg = gb_allsum(dg);
      {
        float4* dkp = reinterpret_cast<float4*>(prt + R * kGB_D + 8 * lane);
        dkp[0] = make_float4(dk[0], dk[1], dk[2], dk[3]);
        dkp[1] = make_float4(dk[4], dk[5], dk[6], dk[7]);
        if (lane == 0) {
          prt[(R + 1) * kGB_D] = dbeta;
          prt[(R + 1) * kGB_D + 1] = dg;
        }
      }
      // the next token's stage, then one barrier for both buffers
      float* nst = s_stage + (buf ^ 1) * kGB_Stage;
#pragma unroll
      for (int u = 0; u < 3; ++u)
        if (pdst[u] >= 0) *reinterpret_cast<float4*>(nst + pdst[u]) = pre[u];
      if (tt > 0 && tid == 0) {
        nst[kGB_Stage - 4] = pa;
        nst[kGB_Stage - 3] = pb;
      }
      __syncthreads();
      {
        const float* pall = s_part + buf * kGB_Warps * kGB_Emax;
        float* out = A.part + (((size_t)bg * T + t) * A.ncta + cta) * E;
        for (int x = tid; x < E; x += 256) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kGB_Warps; ++w) acc += pall[w * kGB_Emax + x];
          out[x] = acc;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          st[i][c] = sp[i][c];
          sp[i][c] = nx[i][c];
        }
      ecur = enx;
    }
    __syncthreads();   // the stage and partial buffers are reused by the next chunk
  }
  // dL/dS_0
#pragma unroll
  for (int i = 0; i < 8; ++i)
    *reinterpret_cast<float4*>(A.ds0 + (size_t)bg * kGB_D * kGB_D + (size_t)(8 * lane + i) * kGB_D + col) =
        make_float4(ds[i][0], ds[i][1], ds[i][2], ds[i][3]);
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
    for (int c = 0; c < A.ncta; ++c) acc += src[(size_t)c * A.E + x];
    if (x < RD) dq[tg * RD + x] = acc;
    else if (x < RD + kGB_D) dk[tg * kGB_D + (x - RD)] = acc;
    else if (x == RD + kGB_D) dbeta[tg] = acc;
    else if (x == RD + kGB_D + 1) dg[tg] = acc;
  }
}

static int gb_smem_bytes() { return (2 * kGB_Warps * kGB_Emax + 2 * kGB_Stage) * 4; }

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
  if ((rc = ensure_smem_attr((const void*)gdn_bwd_kernel, smem))) return rc;
  gdn_bwd_kernel<<<dim3(B * G, A.ncta), 256, smem, stream>>>(A);
  if ((rc = launch_status())) return rc;
  gdn_bwd_reduce_kernel<<<dim3(T, B * G), 256, 0, stream>>>(A, dq, dk, dg, dbeta);
  return launch_status();
}

}  // extern "C"
