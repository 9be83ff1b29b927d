// Retrieval attention for the kept (not converted) full-attention layers, single-token decode
// (heimdall/hibrit.py:275-324: HybridAttention._teacher with its retrieval branch and _retrieval_mask).
//
// The query at position p = n - 1 of a KV head group attends, with an exact softmax,
//   the sinks [0, S), the k selected blocks of L keys, and the window [S + nc L, p],
// where nc = min((p - W + 1 - S) / L, nb) candidate blocks end before the window (nb = (n - S) / L full blocks)
// and the k selected ones are those with the largest upper bound of q.k over the block, per KV head: the max
// over the group's R query heads of sum_d (max(q_d, 0) kmax_d + min(q_d, 0) kmin_d), with the block's per-dim key
// minimum and maximum (Quest-style summaries).  Applies when n - S - W >= k L (then nc >= k).
//
// Three kernels, all HBM-bound:
//   ret_summary_kernel: the min / max of each new full block (bf16, exact), one CTA per block and KV head;
//   ret_bounds_kernel:  per (batch, KV head, split of 256 candidate blocks) the bounds from the summaries (four
//                       blocks per warp iteration, loads in flight), then the split's k largest;
//   ret_merge_kernel:   per (batch, KV head) the k largest of the splits' candidates (ascending order);
//   ret_attn_kernel:    split over the attended keys (sinks, selected blocks, window as one virtual sequence), 64 per CTA:
//                       each CTA stages 64 keys and values at a time in shared memory, computes the R query
//                       heads' scores (four threads per key, a quarter of D each), an online softmax per head
//                       and P V (one thread per value column), and writes its partial (max, sum, acc);
//   ret_combine_kernel: merges the partials of the splits, per (batch, query head).
#include "bifrost_b200.h"
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

constexpr int kRA_D = 256;
constexpr int kRA_MaxR = 8;
constexpr int kRA_Chunk = 64;       // keys staged per step
constexpr int kRA_Split = 64;       // keys per CTA of the attention (one staged chunk: CTAs overlap each other's loads)
constexpr int kRA_SelBlocks = 256;  // candidate blocks per CTA of the bounds kernel
constexpr int kRA_MaxCand = 4096;   // candidates merged per (b, g): splits x k

struct RetArgs {
  const __nv_bfloat16* q;     // [B, H, D]
  const __nv_bfloat16* k;     // [B, G, cap, D]
  const __nv_bfloat16* v;     // [B, G, cap, D]
  const __nv_bfloat16* kmin;  // [B, G, nbcap, D]
  const __nv_bfloat16* kmax;
  int* sel;                   // [B, G, K]
  float* cand_v;              // [B, G, nsel, K] per-split candidates (bound, block)
  int* cand_i;
  float* part;                // [B, G, nsplit, R, D + 2]
  float* o;                   // [B, H, D]
  long long cap, nbcap;       // key / block capacity of the cache arrays
  int B, H, G, R, n, S, W, L, K, nc, nk, nsplit, nsel;
};

__global__ void __launch_bounds__(256) ret_summary_kernel(const __nv_bfloat16* __restrict__ k, long long cap,
                                                          int S, int L, int nb0, __nv_bfloat16* __restrict__ kmin,
                                                          __nv_bfloat16* __restrict__ kmax, long long nbcap) {
  const int blk = nb0 + blockIdx.x, bg = blockIdx.y, d = threadIdx.x;
  const __nv_bfloat16* src = k + ((size_t)bg * cap + S + (size_t)blk * L) * kRA_D + d;
  float mn = INFINITY, mx = -INFINITY;
  for (int i = 0; i < L; ++i) {
    const float x = __bfloat162float(src[(size_t)i * kRA_D]);
    mn = fminf(mn, x);
    mx = fmaxf(mx, x);
  }
  kmin[((size_t)bg * nbcap + blk) * kRA_D + d] = __float2bfloat16_rn(mn);   // exact: a bf16 value
  kmax[((size_t)bg * nbcap + blk) * kRA_D + d] = __float2bfloat16_rn(mx);
}

__device__ __forceinline__ void bf16x8_to_f(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}

// bounds of one split of the candidate blocks, then the split's k largest (bound, index) pairs.  Grid
// (B * G, nsel): split s takes candidates [s * kRA_SelBlocks, ...); each warp computes four blocks' bounds per
// iteration with all eight summary loads in flight (lanes over D, one warp reduction per query head)
__global__ void __launch_bounds__(256) ret_bounds_kernel(RetArgs a) {
  __shared__ float s_ub[kRA_SelBlocks];
  __shared__ float s_wv[8];
  __shared__ int s_wi[8];
  const int bg = blockIdx.x, b = bg / a.G, g = bg % a.G, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = split * kRA_SelBlocks, nloc = min(kRA_SelBlocks, a.nc - c0);
  float qv[kRA_MaxR][8];
#pragma unroll
  for (int r = 0; r < kRA_MaxR; ++r) {
    if (r < a.R) {
      bf16x8_to_f(__ldg(reinterpret_cast<const uint4*>(a.q + ((size_t)b * a.H + g * a.R + r) * kRA_D) + lane), qv[r]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[r][e] = 0.f;
    }
  }
  const __nv_bfloat16* mnp = a.kmin + ((size_t)bg * a.nbcap + c0) * kRA_D;
  const __nv_bfloat16* mxp = a.kmax + ((size_t)bg * a.nbcap + c0) * kRA_D;
  for (int c = warp * 4; c < nloc; c += 32) {
    uint4 lo4[4], hi4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      lo4[u] = hi4[u] = make_uint4(0u, 0u, 0u, 0u);
      if (c + u < nloc) {
        lo4[u] = __ldg(reinterpret_cast<const uint4*>(mnp + (size_t)(c + u) * kRA_D) + lane);
        hi4[u] = __ldg(reinterpret_cast<const uint4*>(mxp + (size_t)(c + u) * kRA_D) + lane);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float lo[8], hi[8];
      bf16x8_to_f(lo4[u], lo);
      bf16x8_to_f(hi4[u], hi);
      float best = -INFINITY;
#pragma unroll
      for (int r = 0; r < kRA_MaxR; ++r) {
        if (r >= a.R) break;
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s += fmaxf(qv[r][e], 0.f) * hi[e] + fminf(qv[r][e], 0.f) * lo[e];
        best = fmaxf(best, warp_sum(s));
      }
      if (lane == 0 && c + u < nloc) s_ub[c + u] = best;
    }
  }
  __syncthreads();
  // this split's k largest: k rounds of a block-wide argmax (ties to the smaller index)
  float* out_v = a.cand_v + ((size_t)bg * a.nsel + split) * a.K;
  int* out_i = a.cand_i + ((size_t)bg * a.nsel + split) * a.K;
  for (int kk = 0; kk < a.K; ++kk) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = threadIdx.x; c < nloc; c += 256) {
      const float x = s_ub[c];
      if (x > bv || (x == bv && c < bi)) { bv = x; bi = c; }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { s_wv[warp] = bv; s_wi[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v0 = s_wv[0];
      int i0 = s_wi[0];
      for (int w = 1; w < 8; ++w)
        if (s_wv[w] > v0 || (s_wv[w] == v0 && s_wi[w] < i0)) { v0 = s_wv[w]; i0 = s_wi[w]; }
      const bool ok = i0 >= 0 && i0 < nloc;
      out_v[kk] = ok ? v0 : -INFINITY;
      out_i[kk] = ok ? c0 + i0 : 0x7fffffff;
      if (ok) s_ub[i0] = -INFINITY;
    }
    __syncthreads();
  }
}

// merge the splits' candidates of one (b, g) into the k selected blocks, in ascending order (one warp)
__global__ void __launch_bounds__(32) ret_merge_kernel(RetArgs a) {
  const int bg = blockIdx.x, lane = threadIdx.x;
  const int ncand = a.nsel * a.K;
  const float* cv = a.cand_v + (size_t)bg * ncand;
  const int* ci = a.cand_i + (size_t)bg * ncand;
  __shared__ int s_pick[64];
  __shared__ unsigned char s_used[kRA_MaxCand];
  for (int i = lane; i < ncand; i += 32) s_used[i] = 0;
  __syncwarp();
  for (int kk = 0; kk < a.K; ++kk) {
    float bv = -INFINITY;
    int bi = 0x7fffffff, bj = -1;
    for (int i = lane; i < ncand; i += 32) {
      if (s_used[i]) continue;
      const float x = cv[i];
      const int xi = ci[i];
      if (x > bv || (x == bv && xi < bi)) { bv = x; bi = xi; bj = i; }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; bj = oj; }
    }
    if (lane == 0) {
      s_pick[kk] = bi;
      if (bj >= 0) s_used[bj] = 1;
    }
    __syncwarp();
  }
  if (lane == 0) {   // ascending order (insertion sort of at most 64)
    for (int i = 1; i < a.K; ++i) {
      const int x = s_pick[i];
      int j = i - 1;
      while (j >= 0 && s_pick[j] > x) { s_pick[j + 1] = s_pick[j]; --j; }
      s_pick[j + 1] = x;
    }
    for (int i = 0; i < a.K; ++i) a.sel[(size_t)bg * a.K + i] = s_pick[i];
  }
}

// key position of virtual index i: the sinks, then the selected blocks, then the window
__device__ __forceinline__ int ret_key_pos(const RetArgs& a, const int* sel, int i) {
  if (i < a.S) return i;
  i -= a.S;
  if (i < a.K * a.L) return a.S + sel[i / a.L] * a.L + (i % a.L);
  return a.S + a.nc * a.L + (i - a.K * a.L);
}

// grid (B * G, nsplit); dynamic shared memory: K and V chunks
__global__ void __launch_bounds__(256) ret_attn_kernel(RetArgs a) {
  extern __shared__ __align__(16) uint8_t ra_smem[];
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(ra_smem);            // [64][256 + 8]
  __nv_bfloat16* sv = sk + kRA_Chunk * (kRA_D + 8);                         // [64][256]
  float* sp = reinterpret_cast<float*>(sv + kRA_Chunk * kRA_D);              // [R][64] probabilities
  float* sq = sp + kRA_MaxR * kRA_Chunk;                                     // [R][256] queries (scaled)
  __shared__ int s_sel[64];
  __shared__ float s_m[kRA_MaxR], s_l[kRA_MaxR], s_scale[kRA_MaxR];
  const int bg = blockIdx.x, b = bg / a.G, g = bg % a.G, split = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = split * kRA_Split, i1 = min(i0 + kRA_Split, a.nk);
  const float qs = rsqrtf((float)kRA_D) * kLog2e;   // scores in the log2 domain
  for (int i = tid; i < a.R * kRA_D; i += 256) {
    const int r = i / kRA_D, d = i % kRA_D;
    sq[i] = __bfloat162float(a.q[((size_t)b * a.H + g * a.R + r) * kRA_D + d]) * qs;
  }
  for (int i = tid; i < a.K; i += 256) s_sel[i] = a.sel[(size_t)bg * a.K + i];
  if (tid < kRA_MaxR) { s_m[tid] = -INFINITY; s_l[tid] = 0.f; }
  float acc[kRA_MaxR];
#pragma unroll
  for (int r = 0; r < kRA_MaxR; ++r) acc[r] = 0.f;
  const __nv_bfloat16* kb = a.k + (size_t)bg * a.cap * kRA_D;
  const __nv_bfloat16* vb = a.v + (size_t)bg * a.cap * kRA_D;
  __syncthreads();
  for (int c0 = i0; c0 < i1; c0 += kRA_Chunk) {
    const int nkc = min(kRA_Chunk, i1 - c0);
    // stage: 64 rows of 512 B each for K and V (2048 16-byte chunks each); this thread's eight chunks of each
    // are all loaded before the first store
    uint4 kk[8], vv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = tid + u * 256, row = idx >> 5, col = idx & 31;
      kk[u] = vv[u] = make_uint4(0u, 0u, 0u, 0u);
      if (row < nkc) {
        const int pos = ret_key_pos(a, s_sel, c0 + row);
        kk[u] = __ldg(reinterpret_cast<const uint4*>(kb + (size_t)pos * kRA_D) + col);
        vv[u] = __ldg(reinterpret_cast<const uint4*>(vb + (size_t)pos * kRA_D) + col);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = tid + u * 256, row = idx >> 5, col = idx & 31;
      *reinterpret_cast<uint4*>(sk + row * (kRA_D + 8) + col * 8) = kk[u];
      *reinterpret_cast<uint4*>(sv + row * kRA_D + col * 8) = vv[u];
    }
    __syncthreads();
    // scores: thread (key = tid / 4, quarter = tid % 4) sums 64 dims for every head, then a 4-lane reduction
    {
      const int key = tid >> 2, qq = tid & 3;
      float s[kRA_MaxR];
#pragma unroll
      for (int r = 0; r < kRA_MaxR; ++r) s[r] = 0.f;
      const __nv_bfloat16* krow = sk + key * (kRA_D + 8) + qq * 64;
#pragma unroll 4
      for (int e = 0; e < 64; e += 8) {
        float kf[8];
        bf16x8_to_f(*reinterpret_cast<const uint4*>(krow + e), kf);
#pragma unroll
        for (int r = 0; r < kRA_MaxR; ++r) {
          if (r < a.R) {
            const float* qp = sq + r * kRA_D + qq * 64 + e;
#pragma unroll
            for (int j = 0; j < 8; ++j) s[r] = fmaf(qp[j], kf[j], s[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRA_MaxR; ++r) {
        s[r] += __shfl_xor_sync(0xffffffffu, s[r], 1);
        s[r] += __shfl_xor_sync(0xffffffffu, s[r], 2);
      }
      if (qq == 0) {
#pragma unroll
        for (int r = 0; r < kRA_MaxR; ++r)
          if (r < a.R) sp[r * kRA_Chunk + key] = key < nkc ? s[r] : -INFINITY;
      }
    }
    __syncthreads();
    // online softmax per head: warp r takes head r's 64 scores
    if (warp < a.R) {
      const int r = warp;
      const float x0 = sp[r * kRA_Chunk + lane], x1 = sp[r * kRA_Chunk + 32 + lane];
      float mx = fmaxf(x0, x1);
#pragma unroll
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = s_m[r];
      const float m_new = fmaxf(m_old, mx);
      const float p0 = x0 == -INFINITY ? 0.f : ex2_approx(x0 - m_new);
      const float p1 = x1 == -INFINITY ? 0.f : ex2_approx(x1 - m_new);
      float ls = warp_sum(p0 + p1);
      sp[r * kRA_Chunk + lane] = p0;
      sp[r * kRA_Chunk + 32 + lane] = p1;
      if (lane == 0) {
        const float sc = m_old == -INFINITY ? 0.f : ex2_approx(m_old - m_new);
        s_scale[r] = sc;
        s_l[r] = s_l[r] * sc + ls;
        s_m[r] = m_new;
      }
    }
    __syncthreads();
    // P V: thread = value column
    {
      const int d = tid;
#pragma unroll
      for (int r = 0; r < kRA_MaxR; ++r)
        if (r < a.R) acc[r] *= s_scale[r];
      for (int key = 0; key < nkc; ++key) {
        const float vf = __bfloat162float(sv[key * kRA_D + d]);
#pragma unroll
        for (int r = 0; r < kRA_MaxR; ++r)
          if (r < a.R) acc[r] = fmaf(sp[r * kRA_Chunk + key], vf, acc[r]);
      }
    }
    __syncthreads();
  }
  // partial: [R][D + 2] = acc, max, sum
  float* pp = a.part + ((size_t)bg * a.nsplit + split) * a.R * (kRA_D + 2);
#pragma unroll
  for (int r = 0; r < kRA_MaxR; ++r)
    if (r < a.R) pp[r * (kRA_D + 2) + tid] = acc[r];
  if (tid < a.R) {
    pp[tid * (kRA_D + 2) + kRA_D] = s_m[tid];
    pp[tid * (kRA_D + 2) + kRA_D + 1] = s_l[tid];
  }
}

// grid B * H: merge the splits of one (b, query head)
__global__ void __launch_bounds__(256) ret_combine_kernel(RetArgs a) {
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, g = h / a.R, r = h % a.R;
  const int bg = b * a.G + g;
  const float* pp = a.part + (size_t)bg * a.nsplit * a.R * (kRA_D + 2) + r * (kRA_D + 2);
  const size_t sstride = (size_t)a.R * (kRA_D + 2);
  float M = -INFINITY;
  for (int s = 0; s < a.nsplit; ++s) M = fmaxf(M, pp[s * sstride + kRA_D]);
  float Lsum = 0.f, acc = 0.f;
  for (int s = 0; s < a.nsplit; ++s) {
    const float m = pp[s * sstride + kRA_D];
    const float w = m == -INFINITY ? 0.f : ex2_approx(m - M);
    Lsum += pp[s * sstride + kRA_D + 1] * w;
    acc += pp[s * sstride + threadIdx.x] * w;
  }
  a.o[((size_t)b * a.H + h) * kRA_D + threadIdx.x] = Lsum > 0.f ? acc / Lsum : 0.f;
}

static int ret_smem_attn() {
  return (kRA_Chunk * (kRA_D + 8) + kRA_Chunk * kRA_D) * 2 + (kRA_MaxR * kRA_Chunk + kRA_MaxR * kRA_D) * 4;
}

}  // namespace bfb

using namespace bfb;

extern "C" {

int bf_ret_summarize(const void* k, long long cap, int B, int G, int D, int sinks, int block, int nb0, int nb1,
                     void* kmin, void* kmax, long long nbcap, bf_stream_t stream) {
  if (!k || !kmin || !kmax || B <= 0 || G <= 0 || sinks < 0 || block <= 0 || nb0 < 0 || nb1 < nb0 || nb1 > nbcap)
    return BF_ERR_INVALID_ARGUMENT;
  if (D != kRA_D) return BF_ERR_UNSUPPORTED;
  if ((long long)sinks + (long long)nb1 * block > cap) return BF_ERR_INVALID_ARGUMENT;
  if (nb1 == nb0) return BF_OK;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  ret_summary_kernel<<<dim3(nb1 - nb0, B * G), kRA_D, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(k), cap, sinks, block, nb0, static_cast<__nv_bfloat16*>(kmin),
      static_cast<__nv_bfloat16*>(kmax), nbcap);
  return launch_status();
}

size_t bf_ret_decode_workspace(int B, int H, int G, int D, int n, int sinks, int window, int block, int k) {
  if (B <= 0 || H <= 0 || G <= 0 || H % G || D != kRA_D || block <= 0 || k <= 0 || sinks < 0 || window <= 0)
    return 0;
  const int nb = (n - sinks) / block;
  const int nc = max(0, min((n - 1 - window + 1 - sinks) / block, nb));
  const long long nk = (long long)sinks + (long long)k * block + (n - sinks - (long long)nc * block);
  const long long nsplit = (nk + kRA_Split - 1) / kRA_Split;
  const long long nsel = (nc + kRA_SelBlocks - 1) / kRA_SelBlocks;
  const size_t sel = ((size_t)B * G * k * 4 + 255) / 256 * 256;
  const size_t cand = ((size_t)B * G * (nsel > 0 ? nsel : 1) * k * 4 + 255) / 256 * 256;
  return sel + 2 * cand + (size_t)B * G * nsplit * (H / G) * (kRA_D + 2) * 4;
}

int bf_ret_decode(const void* q, const void* k, const void* v, long long cap, const void* kmin, const void* kmax,
                  long long nbcap, int B, int H, int G, int D, int n, int sinks, int window, int block, int topk,
                  float* o, void* ws, size_t ws_bytes, bf_stream_t stream) {
  if (!q || !k || !v || !kmin || !kmax || !o || !ws || B <= 0 || H <= 0 || G <= 0 || H % G || H / G > kRA_MaxR)
    return BF_ERR_INVALID_ARGUMENT;
  if (D != kRA_D) return BF_ERR_UNSUPPORTED;
  if (block <= 0 || topk <= 0 || topk > 64 || sinks < 0 || window <= 0 || n > cap) return BF_ERR_INVALID_ARGUMENT;
  if ((long long)n - sinks - window < (long long)topk * block) return BF_ERR_INVALID_ARGUMENT;   // no retrieval
  const size_t need = bf_ret_decode_workspace(B, H, G, D, n, sinks, window, block, topk);
  if (need == 0 || ws_bytes < need) return BF_ERR_WORKSPACE;
  const void* ptrs[6] = {q, k, v, kmin, kmax, o};
  for (const void* p : ptrs)
    if (!aligned16(p)) return BF_ERR_ALIGNMENT;
  if (!aligned16(ws)) return BF_ERR_ALIGNMENT;
  RetArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.kmin = static_cast<const __nv_bfloat16*>(kmin);
  a.kmax = static_cast<const __nv_bfloat16*>(kmax);
  a.cap = cap;
  a.nbcap = nbcap;
  a.B = B; a.H = H; a.G = G; a.R = H / G; a.n = n; a.S = sinks; a.W = window; a.L = block; a.K = topk;
  const int nb = (n - sinks) / block;
  a.nc = max(0, min((n - window - sinks) / block, nb));
  if (a.nc > nbcap) return BF_ERR_INVALID_ARGUMENT;
  a.nk = sinks + topk * block + (n - sinks - a.nc * block);
  a.nsplit = (a.nk + kRA_Split - 1) / kRA_Split;
  a.nsel = (a.nc + kRA_SelBlocks - 1) / kRA_SelBlocks;
  if (a.nsel * topk > kRA_MaxCand) return BF_ERR_UNSUPPORTED;
  const size_t sel_b = ((size_t)B * G * topk * 4 + 255) / 256 * 256;
  const size_t cand_b = ((size_t)B * G * a.nsel * topk * 4 + 255) / 256 * 256;
  a.sel = static_cast<int*>(ws);
  a.cand_v = reinterpret_cast<float*>(static_cast<char*>(ws) + sel_b);
  a.cand_i = reinterpret_cast<int*>(static_cast<char*>(ws) + sel_b + cand_b);
  a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + sel_b + 2 * cand_b);
  a.o = o;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  ret_bounds_kernel<<<dim3(B * G, a.nsel), 256, 0, stream>>>(a);
  if ((rc = launch_status())) return rc;
  ret_merge_kernel<<<B * G, 32, 0, stream>>>(a);
  if ((rc = launch_status())) return rc;
  const int asmem = ret_smem_attn();
  if ((rc = ensure_smem_attr((const void*)ret_attn_kernel, asmem))) return rc;
  ret_attn_kernel<<<dim3(B * G, a.nsplit), 256, asmem, stream>>>(a);
  if ((rc = launch_status())) return rc;
  ret_combine_kernel<<<B * H, kRA_D, 0, stream>>>(a);
  return launch_status();
}

}  // extern "C"
