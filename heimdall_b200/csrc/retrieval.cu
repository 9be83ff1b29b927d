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
// Kernels, all HBM-bound (the contractions run on mma.sync tiles fed from registers, see below):
//   ret_summary_kernel: the min / max of each new full block (bf16, exact), one CTA per block and KV head;
//   ret_bounds_kernel:  per warp item of 64 candidate blocks, the bounds of the R query heads from the summaries
//                       ([q+ | q-] against [kmax | kmin]: 32 tensor-core steps per 16 blocks), then the item's k
//                       largest as ordered 64-bit (bound, block) keys;
//   ret_merge_kernel:   per (batch, KV head) the k largest of the items' candidates (ascending block order);
//   ret_attn_kernel:    split over the attended keys (sinks, selected blocks, window as one virtual sequence), 256
//                       per CTA: four warps take 16-key chunks in turn (scores and P V on the tensor cores, P as a
//                       bf16 hi + lo pair; online softmax in registers), merge in shared memory and write the split's partial (acc, max, sum);
//   ret_combine_kernel: merges the partials of the splits, per (batch, query head).
#include "bifrost_b200.h"
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

constexpr int kRA_D = 256;
constexpr int kRA_MaxR = 8;
constexpr int kRA_Split = 256;       // attended keys per CTA of the attention (16 chunks of 16, four warps)
constexpr int kRA_ItemBlocks = 64;   // candidate blocks per warp of the bounds kernel (four 16-block tiles)
constexpr int kRA_MergeSmem = 4096;  // candidates the merge stages in shared memory (larger sets are read from L2)
constexpr int kRA_MergeLanes = 8;    // item lists per merge lane: at most 256 items per (b, g)

struct RetArgs {
  const __nv_bfloat16* q;     // [B, H, D]
  const __nv_bfloat16* k;     // [B, G, cap, D]
  const __nv_bfloat16* v;     // [B, G, cap, D]
  const __nv_bfloat16* kmin;  // [B, G, nbcap, D]
  const __nv_bfloat16* kmax;
  int* sel;                   // [B, G, K]
  unsigned long long* cand;   // [B, G, nitem, K] per-item candidates as ordered (bound, block) keys
  float* part;                // [B, G, nsplit, R, D + 2]
  float* o;                   // [B, H, D]
  long long cap, nbcap;       // key / block capacity of the cache arrays
  int B, H, G, R, n, S, W, L, K, nc, nk, nsplit, nitem;
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

// ---------------------------------------------------------------------------------------------------------------
// Warp-level tensor-core tiles (mma.sync m16n8k16, bf16 in, fp32 accumulate) fed straight from global memory.
//
// Block bounds and attention scores are both  C[row, head] = sum_d A[row, d] B[d, head]  with A = key rows (block
// summaries or keys, 512 B each) and B = the R <= 8 query heads of the group.  A contraction may take the dims in
// any order as long as A and B agree, so lane (g, c) = (lane / 4, lane % 4) loads, per 32-dim slab p, one
// 16-byte vector of dims [32p + 8c, 32p + 8c + 8) of rows g and g + 8 and of query head g, and uses its first
// four dims as the fragment of mma step 2p and its last four as that of step 2p + 1 (fragment k-pairs
// {2c, 2c+1} and {2c+8, 2c+9} <- dims +0,+1 and +2,+3 of the half).  Every access is a 16-byte vector and a warp
// reads 64 contiguous bytes of each of 8 rows per instruction.
//
// P V is  O^T[dim, head] = sum_key V^T[dim, key] P^T[key, head]: lane (g, c) loads dims [64j + 8g, 64j + 8g + 8)
// of keys 2c, 2c+1, 2c+8, 2c+9 and pairs equal dims of two keys with a byte permute (m-tile (j, i) row g <- dim
// 64j + 8g + 2i, row g + 8 <- dim 64j + 8g + 2i + 1).  The probabilities come out of the score tile as
// P[key, head] in the accumulator layout; movmatrix.trans turns each 8x8 half into the P^T operand.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// a 16-byte streaming load kept in program order with the other asm statements, so that a tile's loads are all
// issued before its first tensor-core step
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t bf16x2_max0(uint32_t x) {   // per half max(x, 0) / min(x, 0): exact selections
  uint32_t y;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(y) : "r"(x), "r"(0u));
  return y;
}
__device__ __forceinline__ uint32_t bf16x2_min0(uint32_t x) {
  uint32_t y;
  asm("min.bf16x2 %0, %1, %2;" : "=r"(y) : "r"(x), "r"(0u));
  return y;
}

// (bound, block) as one 64-bit key ordered by bound descending, then block ascending; 0 = no candidate
__device__ __forceinline__ unsigned long long ret_key(float v, int blk) {
  uint32_t u = __float_as_uint(v);
  u ^= (u & 0x80000000u) ? 0xffffffffu : 0x80000000u;
  return ((unsigned long long)u << 32) | (0xffffffffu - (uint32_t)blk);
}
__device__ __forceinline__ int ret_key_block(unsigned long long key) { return (int)(0xffffffffu - (uint32_t)key); }

// warp-wide max of a 64-bit key: the high words' max, then the low words' max among the lanes holding it
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long x) {
  const unsigned hi = (unsigned)(x >> 32), lo = (unsigned)x;
  const unsigned mhi = __reduce_max_sync(0xffffffffu, hi);
  const unsigned mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? lo : 0u);
  return ((unsigned long long)mhi << 32) | mlo;
}

// query heads of group g in the B-operand layout: lane (g, c) holds head g's dims [32p + 8c, +8) for p = 0..7
__device__ __forceinline__ void ret_load_q(const RetArgs& a, int b, int g, int lane, uint4 (&qu)[8]) {
  const int hg = lane >> 2, c = lane & 3;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    qu[p] = make_uint4(0u, 0u, 0u, 0u);
    if (hg < a.R)
      qu[p] = __ldg(reinterpret_cast<const uint4*>(a.q + ((size_t)b * a.H + g * a.R + hg) * kRA_D + 32 * p + 8 * c));
  }
}

// Block bounds of one warp item (kRA_ItemBlocks candidate blocks, four 16-block tiles) on the tensor cores, then
// the item's k largest as 64-bit keys.  Grid (B * G, ceil(items / 4)), four warps = four items per CTA.
__global__ void __launch_bounds__(128, 4) ret_bounds_kernel(RetArgs a) {
  const int bg = blockIdx.x, b = bg / a.G, g = bg % a.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, rg = lane >> 2, c = lane & 3;
  const int item = blockIdx.y * 4 + warp;
  if (item >= a.nitem) return;
  const int c0 = item * kRA_ItemBlocks, nloc = min(kRA_ItemBlocks, a.nc - c0);
  uint4 qu[8];
  ret_load_q(a, b, g, lane, qu);
  const __nv_bfloat16* mnp = a.kmin + ((size_t)bg * a.nbcap + c0) * kRA_D + 8 * c;
  const __nv_bfloat16* mxp = a.kmax + ((size_t)bg * a.nbcap + c0) * kRA_D + 8 * c;
  unsigned long long mine[2] = {0ull, 0ull};     // lane (rg, c) keeps tile c's blocks rg and rg + 8
#pragma unroll 1
  for (int t = 0; t < kRA_ItemBlocks / 16; ++t) {
    const int r0 = min(16 * t + rg, nloc - 1), r1 = min(16 * t + rg + 8, nloc - 1);   // clamped rows: masked below
    uint4 h0[8], h1[8], l0[8], l1[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      h0[p] = ldg_stream(mxp + (size_t)r0 * kRA_D + 32 * p);
      h1[p] = ldg_stream(mxp + (size_t)r1 * kRA_D + 32 * p);
      l0[p] = ldg_stream(mnp + (size_t)r0 * kRA_D + 32 * p);
      l1[p] = ldg_stream(mnp + (size_t)r1 * kRA_D + 32 * p);
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      mma_bf16_16816(acc, h0[p].x, h1[p].x, h0[p].y, h1[p].y, bf16x2_max0(qu[p].x), bf16x2_max0(qu[p].y));
      mma_bf16_16816(acc, h0[p].z, h1[p].z, h0[p].w, h1[p].w, bf16x2_max0(qu[p].z), bf16x2_max0(qu[p].w));
      mma_bf16_16816(acc, l0[p].x, l1[p].x, l0[p].y, l1[p].y, bf16x2_min0(qu[p].x), bf16x2_min0(qu[p].y));
      mma_bf16_16816(acc, l0[p].z, l1[p].z, l0[p].w, l1[p].w, bf16x2_min0(qu[p].z), bf16x2_min0(qu[p].w));
    }
    // acc = UB[block rg | rg + 8][heads 2c, 2c + 1]: max over the group's heads
    const bool h0ok = 2 * c < a.R, h1ok = 2 * c + 1 < a.R;
    float u0 = fmaxf(h0ok ? acc[0] : -INFINITY, h1ok ? acc[1] : -INFINITY);
    float u1 = fmaxf(h0ok ? acc[2] : -INFINITY, h1ok ? acc[3] : -INFINITY);
    u0 = fmaxf(u0, __shfl_xor_sync(0xffffffffu, u0, 1));
    u0 = fmaxf(u0, __shfl_xor_sync(0xffffffffu, u0, 2));
    u1 = fmaxf(u1, __shfl_xor_sync(0xffffffffu, u1, 1));
    u1 = fmaxf(u1, __shfl_xor_sync(0xffffffffu, u1, 2));
    if (c == t) {
      mine[0] = 16 * t + rg < nloc ? ret_key(u0, c0 + 16 * t + rg) : 0ull;
      mine[1] = 16 * t + rg + 8 < nloc ? ret_key(u1, c0 + 16 * t + rg + 8) : 0ull;
    }
  }
  // the item's k largest keys, in descending order (k rounds of a warp max below the previous pick)
  unsigned long long* out = a.cand + ((size_t)bg * a.nitem + item) * a.K;
  unsigned long long prev = ~0ull;
  for (int kk = 0; kk < a.K; ++kk) {
    unsigned long long x = mine[0] < prev ? mine[0] : 0ull;
    if (mine[1] < prev && mine[1] > x) x = mine[1];
    x = warp_max_u64(x);
    if (lane == 0) out[kk] = x;
    prev = x;
    if (x == 0ull) prev = 0ull;   // nothing left: the remaining picks are empty
  }
}

// the k largest of a (b, g)'s item candidates, in ascending block order (one warp).  Every item's list is sorted
// (descending keys), so this is a merge of sorted lists: lane i owns lists i, i + 32, ...; each round the warp
// takes the largest list head and its list advances.  The lists are staged in shared memory first.
__global__ void __launch_bounds__(128) ret_merge_kernel(RetArgs a) {
  const int bg = blockIdx.x, lane = threadIdx.x & 31;
  const int ncand = a.nitem * a.K;
  const unsigned long long* cv = a.cand + (size_t)bg * ncand;
  __shared__ unsigned long long s_c[kRA_MergeSmem];
  __shared__ int s_pick[64];
  const bool staged = ncand <= kRA_MergeSmem;
  if (staged) {   // all four warps stage, eight loads in flight per thread
    for (int base = 0; base < ncand; base += 128 * 8) {
      unsigned long long x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + threadIdx.x + 128 * u;
        x[u] = i < ncand ? cv[i] : 0ull;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + threadIdx.x + 128 * u;
        if (i < ncand) s_c[i] = x[u];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  auto head = [&](int list, int pos) -> unsigned long long {
    if (pos >= a.K) return 0ull;
    const int i = list * a.K + pos;
    return staged ? s_c[i] : cv[i];
  };
  // this lane's best list and its position (a lane owning several lists rescans them after each of its wins)
  int pos[kRA_MergeLanes];
#pragma unroll
  for (int u = 0; u < kRA_MergeLanes; ++u) pos[u] = 0;
  auto lane_best = [&](int& which) -> unsigned long long {
    unsigned long long best = 0ull;
    which = -1;
#pragma unroll
    for (int u = 0; u < kRA_MergeLanes; ++u) {
      const int list = lane + 32 * u;
      if (list < a.nitem) {
        const unsigned long long h = head(list, pos[u]);
        if (h > best) { best = h; which = u; }
      }
    }
    return best;
  };
  int which;
  unsigned long long mine = lane_best(which);
  for (int kk = 0; kk < a.K; ++kk) {
    const unsigned long long x = warp_max_u64(mine);
    if (lane == 0) s_pick[kk] = x ? ret_key_block(x) : 0;
    if (x != 0ull && mine == x) {   // keys are unique: exactly one lane advances
#pragma unroll
      for (int u = 0; u < kRA_MergeLanes; ++u)
        if (u == which) ++pos[u];
      mine = lane_best(which);
    }
  }
  __syncwarp();
  for (int i = lane; i < a.K; i += 32) {   // ascending order: each pick goes to its rank (the blocks are distinct)
    const int x = s_pick[i];
    int rank = 0;
    for (int j = 0; j < a.K; ++j) rank += s_pick[j] < x;
    a.sel[(size_t)bg * a.K + rank] = x;
  }
}

// key position of virtual index i: the sinks, then the selected blocks, then the window
__device__ __forceinline__ int ret_key_pos(const RetArgs& a, const int* sel, int i) {
  if (i < a.S) return i;
  i -= a.S;
  if (i < a.K * a.L) return a.S + sel[i / a.L] * a.L + (i % a.L);
  return a.S + a.nc * a.L + (i - a.K * a.L);
}

// Attention over one split of kRA_Split attended keys (sinks, selected blocks, window as one virtual sequence) of
// one (b, KV head): four warps take 16-key chunks in turn (online softmax per warp in registers, tensor-core
// tiles as above), merge in shared memory and write the split's partial (acc, max, sum) per query head.
__global__ void __launch_bounds__(128, 2) ret_attn_kernel(RetArgs a) {
  __shared__ __align__(16) float s_o[4][kRA_MaxR][kRA_D];
  __shared__ float s_m[4][kRA_MaxR], s_l[4][kRA_MaxR];
  __shared__ int s_pos[kRA_Split];
  __shared__ int s_sel[64];
  const int bg = blockIdx.x, b = bg / a.G, g = bg % a.G, split = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, rg = lane >> 2, c = lane & 3;
  const int i0 = split * kRA_Split, cnt = min(kRA_Split, a.nk - i0);
  for (int i = tid; i < a.K; i += 128) s_sel[i] = a.sel[(size_t)bg * a.K + i];
  __syncthreads();
  for (int i = tid; i < kRA_Split; i += 128) s_pos[i] = ret_key_pos(a, s_sel, i0 + min(i, cnt - 1));
  uint4 qu[8];
  ret_load_q(a, b, g, lane, qu);
  __syncthreads();
  const float qs = rsqrtf((float)kRA_D) * kLog2e;   // scores in the log2 domain
  const __nv_bfloat16* kb = a.k + (size_t)bg * a.cap * kRA_D;
  const __nv_bfloat16* vb = a.v + (size_t)bg * a.cap * kRA_D;
  float o[4][4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[j][i][e] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
#pragma unroll 1
  for (int ch = warp; ch * 16 < cnt; ch += 4) {
    const int k0 = ch * 16;
    const int pk0 = s_pos[k0 + rg], pk1 = s_pos[k0 + rg + 8];
    const int pv0 = s_pos[k0 + 2 * c], pv1 = s_pos[k0 + 2 * c + 1], pv2 = s_pos[k0 + 2 * c + 8],
              pv3 = s_pos[k0 + 2 * c + 9];
    uint4 ka[8], kc[8], v0[4], v1[4], v2[4], v3[4];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      ka[p] = ldg_stream(kb + (size_t)pk0 * kRA_D + 32 * p + 8 * c);
      kc[p] = ldg_stream(kb + (size_t)pk1 * kRA_D + 32 * p + 8 * c);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v0[j] = ldg_stream(vb + (size_t)pv0 * kRA_D + 64 * j + 8 * rg);
      v1[j] = ldg_stream(vb + (size_t)pv1 * kRA_D + 64 * j + 8 * rg);
      v2[j] = ldg_stream(vb + (size_t)pv2 * kRA_D + 64 * j + 8 * rg);
      v3[j] = ldg_stream(vb + (size_t)pv3 * kRA_D + 64 * j + 8 * rg);
    }
    // S[key rg | rg + 8][heads 2c, 2c + 1], accumulated in four independent tiles (short dependent chains)
    float sp4[4][4] = {};
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      mma_bf16_16816(sp4[(2 * p) & 3], ka[p].x, kc[p].x, ka[p].y, kc[p].y, qu[p].x, qu[p].y);
      mma_bf16_16816(sp4[(2 * p + 1) & 3], ka[p].z, kc[p].z, ka[p].w, kc[p].w, qu[p].z, qu[p].w);
    }
    float s[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) s[e] = (sp4[0][e] + sp4[1][e]) + (sp4[2][e] + sp4[3][e]);
    const bool ok0 = k0 + rg < cnt, ok1 = k0 + rg + 8 < cnt;
    s[0] = ok0 ? s[0] * qs : -INFINITY;
    s[1] = ok0 ? s[1] * qs : -INFINITY;
    s[2] = ok1 ? s[2] * qs : -INFINITY;
    s[3] = ok1 ? s[3] * qs : -INFINITY;
    float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    // every chunk holds at least one valid key, so the new maxima are finite
    const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
    const float al0 = ex2_approx(m_run[0] - mn0), al1 = ex2_approx(m_run[1] - mn1);   // 0 while m_run = -inf
    m_run[0] = mn0;
    m_run[1] = mn1;
    // P = P_hi + P_lo, both bf16 (P V takes two tensor-core steps: bf16 alone would add 2^-9 relative noise
    // to every weight, as much again as the bf16 output rounding)
    const float e0 = ex2_approx(s[0] - mn0), e1 = ex2_approx(s[1] - mn1);
    const float e2 = ex2_approx(s[2] - mn0), e3 = ex2_approx(s[3] - mn1);
    l_run[0] = l_run[0] * al0 + (e0 + e2);
    l_run[1] = l_run[1] * al1 + (e1 + e3);
    const uint32_t h01 = pack_bf16x2(e0, e1), h23 = pack_bf16x2(e2, e3);
    const uint32_t l01 = pack_bf16x2(e0 - __uint_as_float(h01 << 16), e1 - __uint_as_float(h01 & 0xffff0000u));
    const uint32_t l23 = pack_bf16x2(e2 - __uint_as_float(h23 << 16), e3 - __uint_as_float(h23 & 0xffff0000u));
    const uint32_t pb0 = movmatrix_trans(h01), pb1 = movmatrix_trans(h23);
    const uint32_t pl0 = movmatrix_trans(l01), pl1 = movmatrix_trans(l23);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w0[4] = {v0[j].x, v0[j].y, v0[j].z, v0[j].w}, w1[4] = {v1[j].x, v1[j].y, v1[j].z, v1[j].w};
      const uint32_t w2[4] = {v2[j].x, v2[j].y, v2[j].z, v2[j].w}, w3[4] = {v3[j].x, v3[j].y, v3[j].z, v3[j].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o[j][i][0] *= al0;
        o[j][i][1] *= al1;
        o[j][i][2] *= al0;
        o[j][i][3] *= al1;
        const uint32_t a0 = __byte_perm(w0[i], w1[i], 0x5410), a1 = __byte_perm(w0[i], w1[i], 0x7632);
        const uint32_t a2 = __byte_perm(w2[i], w3[i], 0x5410), a3 = __byte_perm(w2[i], w3[i], 0x7632);
        mma_bf16_16816(o[j][i], a0, a1, a2, a3, pb0, pb1);
        mma_bf16_16816(o[j][i], a0, a1, a2, a3, pl0, pl1);
      }
    }
  }
  // this warp's partial: sums over its lanes' keys; o[j][i] = O[heads 2c, 2c+1][dims 64j + 8rg + 2i (+1)]
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], off);
    l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], off);
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int h = 2 * c + hh;
    if (h < a.R) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          *reinterpret_cast<float2*>(&s_o[warp][h][64 * j + 8 * rg + 2 * i]) = make_float2(o[j][i][hh], o[j][i][2 + hh]);
        }
      if (rg == 0) {
        s_m[warp][h] = m_run[hh];
        s_l[warp][h] = l_run[hh];
      }
    }
  }
  __syncthreads();
  float* pp = a.part + ((size_t)bg * a.nsplit + split) * a.R * (kRA_D + 2);
  for (int idx = tid; idx < a.R * kRA_D; idx += 128) {
    const int h = idx / kRA_D, d = idx % kRA_D;
    const float M = fmaxf(fmaxf(s_m[0][h], s_m[1][h]), fmaxf(s_m[2][h], s_m[3][h]));
    float acc = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float wt = s_m[w][h] == -INFINITY ? 0.f : ex2_approx(s_m[w][h] - M);
      acc += s_o[w][h][d] * wt;
      L += s_l[w][h] * wt;
    }
    pp[h * (kRA_D + 2) + d] = acc;
    if (d == 0) {
      pp[h * (kRA_D + 2) + kRA_D] = M;
      pp[h * (kRA_D + 2) + kRA_D + 1] = L;
    }
  }
}

// grid (B * H, 2): merge the splits of one (b, query head) for 128 of its dims in one pass (running max; loads
// issued eight splits at a time)
__global__ void __launch_bounds__(128) ret_combine_kernel(RetArgs a) {
  const int bh = blockIdx.x, b = bh / a.H, h = bh % a.H, g = h / a.R, r = h % a.R;
  const int bg = b * a.G + g, d = blockIdx.y * 128 + threadIdx.x;
  const float* pp = a.part + (size_t)bg * a.nsplit * a.R * (kRA_D + 2) + r * (kRA_D + 2);
  const size_t sstride = (size_t)a.R * (kRA_D + 2);
  float M = -INFINITY, Lsum = 0.f, acc = 0.f;
  for (int s0 = 0; s0 < a.nsplit; s0 += 8) {
    float mv[8], lv[8], xv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int s = s0 + u;
      mv[u] = s < a.nsplit ? pp[s * sstride + kRA_D] : -INFINITY;
      lv[u] = s < a.nsplit ? pp[s * sstride + kRA_D + 1] : 0.f;
      xv[u] = s < a.nsplit ? pp[s * sstride + d] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (mv[u] > M) {
        const float sc = M == -INFINITY ? 0.f : ex2_approx(M - mv[u]);
        acc *= sc;
        Lsum *= sc;
        M = mv[u];
      }
      const float w = mv[u] == -INFINITY ? 0.f : ex2_approx(mv[u] - M);
      acc += xv[u] * w;
      Lsum += lv[u] * w;
    }
  }
  a.o[((size_t)b * a.H + h) * kRA_D + d] = Lsum > 0.f ? acc / Lsum : 0.f;
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
  const long long nitem = (nc + kRA_ItemBlocks - 1) / kRA_ItemBlocks;
  const size_t sel = ((size_t)B * G * k * 4 + 255) / 256 * 256;
  const size_t cand = ((size_t)B * G * (nitem > 0 ? nitem : 1) * k * 8 + 255) / 256 * 256;
  return sel + cand + (size_t)B * G * nsplit * (H / G) * (kRA_D + 2) * 4;
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
  a.nitem = (a.nc + kRA_ItemBlocks - 1) / kRA_ItemBlocks;
  if (a.nitem > 32 * kRA_MergeLanes) return BF_ERR_UNSUPPORTED;   // > 16384 candidate blocks
  const size_t sel_b = ((size_t)B * G * topk * 4 + 255) / 256 * 256;
  const size_t cand_b = ((size_t)B * G * a.nitem * topk * 8 + 255) / 256 * 256;
  a.sel = static_cast<int*>(ws);
  a.cand = reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + sel_b);
  a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + sel_b + cand_b);
  a.o = o;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  ret_bounds_kernel<<<dim3(B * G, (a.nitem + 3) / 4), 128, 0, stream>>>(a);
  if ((rc = launch_status())) return rc;
  ret_merge_kernel<<<B * G, 128, 0, stream>>>(a);
  if ((rc = launch_status())) return rc;
  ret_attn_kernel<<<dim3(B * G, a.nsplit), 128, 0, stream>>>(a);
  if ((rc = launch_status())) return rc;
  ret_combine_kernel<<<dim3(B * H, kRA_D / 128), 128, 0, stream>>>(a);
  return launch_status();
}

}  // extern "C"
