// Chunked gated delta rule (prefill), GQA-native: one 256x256 fp32 state per KV head, read by R query heads.
//
// Math (heimdall/kernels.py:94-129, delta_rule_reference; GQA form heimdall/motor.py:70-102), per chunk of
// C = 128 steps with c_i = cumulative log-decay inside the chunk:
//   A = strict_lower(beta_i k_i.k_j e^{c_i - c_j}),  T = (I + A)^-1,  u = T (beta v),  w = T (beta e^{c} k)
//   v' = u - w S,   o_i = e^{c_i} q_i S + sum_{j<=i} (q_i.k_j) e^{c_i - c_j} v'_j,   S <- e^{c_C} S + (e^{c_C - c} k)^T v'
// The chunk length is an implementation choice (the result is the same recurrence); 128 makes every
// tensor-core tile M = 128.  MMA operands are fp16 (11 significant bits; bf16 is too coarse for the state
// budget), accumulation and the state are fp32.
//
// P1 (parallel, CTA = chunk x (b, KV head)): K K^T on tcgen05, A masked/decayed in the epilogue, T by blocked
//     inversion of the 16x16 diagonal blocks then recursive doubling of the block-triangular inverse in
//     shared memory, u = (T diag beta) V and w = (T diag(beta e^c)) K on tcgen05 with the value and key tiles
//     in token-row order; also writes the fp16 keys and the cumulative decays.
// P2 (sequential over chunks, CTA = (b, KV head, kP2_NB state columns)): the state block lives in registers (fp32),
//     v' = u - w S and dS = K^T (e^{c_C - c} v') run on tcgen05 with fp16 copies of S^T / v'^T staged in shared
//     memory and the fp16 key tile as P1 wrote it;
//     the state at each chunk start and v' are written (fp16, transposed) for P3.
// P3 (parallel, CTA = chunk x (b, query head)): Q K^T (-> decayed causal P in fp16), then per half of the value
//     columns o = e^{c} (Q S_chunk) + P v' with the two products in separate TMEM accumulators.
#include "capi_internal.h"
#include "common.cuh"
#include "gdn_prefill.h"
#include "tmap.h"

namespace bfb {

// ------------------------------------------------------------------------------------------ helpers
struct RowSrc {
  const float* k;               // fp32 key row (256)
  const __nv_bfloat16* v;       // bf16 value row (256), or
  const float* v32;             // fp32 value row
  float g, beta;
  bool zero;
};

__device__ __forceinline__ RowSrc write_row(const GdnStreams& s, int b, int gg, int u) {
  RowSrc r{nullptr, nullptr, nullptr, 0.f, 0.f, true};
  if (s.chunk_tok0) {   // packed sequences: row u % kGC of global chunk u / kGC
    const int c = u / kGC, rr = u % kGC;
    if (rr >= s.chunk_len[c]) return r;
    const size_t tok = (size_t)s.chunk_tok0[c] + rr;
    r.k = s.km + (tok * s.G + gg) * kGD;
    if (s.v32) r.v32 = s.v32 + (tok * s.G + gg) * kGD;
    else r.v = s.v + (tok * s.G + gg) * kGD;
    r.g = s.g[tok * s.G + gg];
    r.beta = s.beta[tok * s.G + gg];
    r.zero = false;
    return r;
  }
  if (u >= s.n_steps) return r;
  if (u < s.nring) {
    const long long kp = s.ring_pos0 + u;
    if (kp < 0) return r;
    const int slot = (int)(kp % s.W);
    if (s.ring_pos[slot] != kp) return r;
    r.k = s.ring_km + (((size_t)b * s.W + slot) * s.G + gg) * kGD;
    r.v = s.ring_v + (((size_t)b * s.G + gg) * s.W + slot) * kGD;
    r.g = s.ring_g[((size_t)b * s.W + slot) * s.G + gg];
    r.beta = s.ring_beta[((size_t)b * s.W + slot) * s.G + gg];
  } else {
    const int tok = u - s.nring;
    r.k = s.km + (((size_t)b * s.T + tok) * s.G + gg) * kGD;
    if (s.v32) r.v32 = s.v32 + (((size_t)b * s.T + tok) * s.G + gg) * kGD;
    else r.v = s.v + (((size_t)b * s.T + tok) * s.G + gg) * kGD;
    r.g = s.g[((size_t)b * s.T + tok) * s.G + gg];
    r.beta = s.beta[((size_t)b * s.T + tok) * s.G + gg];
  }
  r.zero = false;
  return r;
}

__device__ __forceinline__ void st_half_sw128(uint8_t* tile, int rows, int row, int col, float x) {
  // element (row, col) of a K-major SW128 tile with `rows` rows; col in 16-bit elements
  const int atom = col >> 6, c = col & 63;
  uint8_t* p = tile + atom * rows * 128 + row * 128 + ((((c >> 3) ^ (row & 7)) << 4)) + (c & 7) * 2;
  *reinterpret_cast<__half*>(p) = __float2half_rn(x);
}

__device__ __forceinline__ void tmem_ld16_wait(uint32_t taddr, float (&f)[16]) {
  uint32_t r[16];
  tmem_ld16(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(r[i]);
}

// ============================================================================================ P1
constexpr int kP1_Threads = 256;
constexpr int kP1_RegK = 0;                   // fp16 key tile [128 tokens][256] (64 KB) -> w staging
constexpr int kP1_RegA = 65536;               // A fp32 [128][kAS] (67.6 KB) -> T_u, T_w fp16 (2 x 32 KB)
constexpr int kP1_RegT = kP1_RegA + 69632;    // T fp32 [128][kAS] -> fp16 value tile [128 tokens][256] -> u staging
constexpr int kP1_RegX = kP1_RegT + 69632;    // doubling scratch (17 KB)
constexpr int kP1_Small = kP1_RegX + 17408;   // gc/g/beta (3 x 512 B) + barriers + row pointers (3 KB) + factors (1 KB)
constexpr int kP1_Smem = kP1_Small + 2048 + 3072 + 1024 + 1024;
constexpr int kAS = 132;                    // row stride (floats) of A and T in shared memory

// rows of zeros that invalid write steps point at, so P1's staging loads need no branches
__device__ __align__(16) float g_zero_row[kGD];

// O = (NEG ? -1 : 1) * L R for M x M blocks of row-major fp32 matrices in shared memory (leading dims in
// floats, multiples of 4; block origins 16-byte aligned); thread tile TR rows x TC columns, the reduction
// reads four columns of L and TC-wide rows of R at a time.  TRI says which factor is lower triangular, so
// that the reduction skips its zero part:
//   TRI = 1: R (O[i][c] needs j >= c).  Threads of a warp share their columns and take rows g + a * M / TR
//            (rows 16 bytes apart in the bank map for a leading dimension of 4 mod 32), so the sum starts
//            at the warp's first column;
//   TRI = 2: L (O[i][c] needs j <= i).  Threads of a warp share their rows, so the sum ends after the
//            warp's last row.
template <int M, int TR, int TC, bool NEG, int TRI>
__device__ __forceinline__ void block_mm(const float* L, int ldl, const float* R, int ldr, float* O, int ldo,
                                         int tt) {
  constexpr int NTC = M / TC, NTR = M / TR, NT = NTR * NTC;
  if (tt >= NT) return;
  int rows[TR], c0;
  if constexpr (TRI == 1) {
    c0 = (tt / NTR) * TC;
#pragma unroll
    for (int a = 0; a < TR; ++a) rows[a] = tt % NTR + a * NTR;
  } else {
    c0 = (tt % NTC) * TC;
#pragma unroll
    for (int a = 0; a < TR; ++a) rows[a] = (tt / NTC) * TR + a;
  }
  const int j0 = TRI == 1 ? (c0 & ~3) : 0;
  const int j1 = TRI == 2 ? ((rows[TR - 1] + 4) & ~3) : M;
  float acc[TR][TC];
#pragma unroll
  for (int a = 0; a < TR; ++a)
#pragma unroll
    for (int b = 0; b < TC; ++b) acc[a][b] = 0.f;
#pragma unroll 2
  for (int j = j0; j < j1; j += 4) {
    float4 av[TR];
#pragma unroll
    for (int a = 0; a < TR; ++a) av[a] = *reinterpret_cast<const float4*>(L + rows[a] * ldl + j);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      float bv[TC];
      if constexpr (TC == 4) {
        const float4 r4 = *reinterpret_cast<const float4*>(R + (j + jj) * ldr + c0);
        bv[0] = r4.x; bv[1] = r4.y; bv[2] = r4.z; bv[3] = r4.w;
      } else if constexpr (TC == 2) {
        const float2 r2 = *reinterpret_cast<const float2*>(R + (j + jj) * ldr + c0);
        bv[0] = r2.x; bv[1] = r2.y;
      } else {
#pragma unroll
        for (int b = 0; b < TC; ++b) bv[b] = R[(j + jj) * ldr + c0 + b];
      }
#pragma unroll
      for (int a = 0; a < TR; ++a) {
        const float x = jj == 0 ? av[a].x : jj == 1 ? av[a].y : jj == 2 ? av[a].z : av[a].w;
#pragma unroll
        for (int b = 0; b < TC; ++b) acc[a][b] = fmaf(x, bv[b], acc[a][b]);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < TR; ++a) {
    float* o = O + rows[a] * ldo + c0;
    const float sg = NEG ? -1.f : 1.f;
    if constexpr (TC == 4) {
      *reinterpret_cast<float4*>(o) = make_float4(sg * acc[a][0], sg * acc[a][1], sg * acc[a][2], sg * acc[a][3]);
    } else if constexpr (TC == 2) {
      *reinterpret_cast<float2*>(o) = make_float2(sg * acc[a][0], sg * acc[a][1]);
    } else {
#pragma unroll
      for (int b = 0; b < TC; ++b) o[b] = sg * acc[a][b];
    }
  }
}

// one doubling level of the block-triangular inverse: for each block pair (rows r1.., r2 = r1 + M)
// T21 = -T22 (A21 T11), with X (the products A21 T11) in scratch; `tt` = thread index, threads split by pair.
// T11 and T22 are lower triangular: the first product skips T11's upper part, the second T22's.
template <int M, int TR, int TC, int TRI1, int TRI2>
__device__ __forceinline__ void inverse_doubling_level(const float* A, float* Tm, float* X, int tt) {
  constexpr int NT = (M / TR) * (M / TC), NPAIR = 128 / (2 * M);
  static_assert(NT * NPAIR <= kP1_Threads, "one tile per thread");
  constexpr int LDX = M + 4;   // X rows 16 bytes apart in the bank map
  const int k = tt / NT, lt = tt % NT;
  const int r1 = k * 2 * M, r2 = r1 + M;
  if (k < NPAIR)
    block_mm<M, TR, TC, false, TRI1>(A + r2 * kAS + r1, kAS, Tm + r1 * kAS + r1, kAS, X + k * M * LDX, LDX, lt);
  __syncthreads();
  if (k < NPAIR)
    block_mm<M, TR, TC, true, TRI2>(Tm + r2 * kAS + r2, kAS, X + k * M * LDX, LDX, Tm + r2 * kAS + r1, kAS, lt);
  __syncthreads();
}

__global__ void __launch_bounds__(kP1_Threads, 1)
    gdn_p1_kernel(const __grid_constant__ CUtensorMap kwmap, const __grid_constant__ CUtensorMap umap,
                  const __grid_constant__ CUtensorMap wmap, GdnStreams s) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* regK = smem + kP1_RegK;
  uint8_t* regA = smem + kP1_RegA;
  uint8_t* regT = smem + kP1_RegT;
  float* s_gc = reinterpret_cast<float*>(smem + kP1_Small);
  float* s_g = s_gc + 128;
  float* s_beta = s_g + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_beta + 128);
  uint64_t* bar_kk = bars + 0;
  uint64_t* bar_uw = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const float** s_kp = reinterpret_cast<const float**>(smem + kP1_Small + 2048);   // [128] key row (or null)
  const __nv_bfloat16** s_vp = reinterpret_cast<const __nv_bfloat16**>(s_kp + 128);  // [128] bf16 value row
  const float** s_vp32 = reinterpret_cast<const float**>(s_vp + 128);             // [128] fp32 value row
  float* A = reinterpret_cast<float*>(regA);   // [128][kAS]
  float* Tm = reinterpret_cast<float*>(regT);  // [128][kAS]

  const int c = blockIdx.x, bg = blockIdx.y, b = bg / s.G, gg = bg % s.G;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const size_t rowbase = (size_t)bg * s.n_pad + (size_t)c * kGC;
  if (s.chunk_tok0 && c >= s.seq_chunk0[s.n_seq]) return;   // grid sized for the most chunks possible

  if (t == 0) {
    mbar_init(bar_kk, 1);
    mbar_init(bar_uw, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // ---- (a) the chunk's write steps: gates and row pointers (thread r < 128; invalid steps point at a zero
  //      row and have beta = 0, so they contribute nothing)
  if (t < 128) {
    const RowSrc src = write_row(s, b, gg, c * kGC + t);
    s_g[t] = src.zero ? 0.f : src.g;
    s_beta[t] = src.zero ? 0.f : src.beta;
    s_kp[t] = src.zero ? g_zero_row : src.k;
    s_vp[t] = src.zero ? reinterpret_cast<const __nv_bfloat16*>(g_zero_row) : src.v;
    s_vp32[t] = src.zero ? g_zero_row : src.v32;
  }
  __syncthreads();
  //      key rows -> fp16 K tile (SW128, 4 atoms), which is also the chunk's tile of fp16 write keys.  Warp w
  //      takes rows w + 8 i; each load covers 512 contiguous bytes of a row (lane l: columns 4 l .. 4 l + 3 of
  //      each half), all 32 in flight at once
  {
    float4 kx[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float* kp = s_kp[warp + 8 * i] + 4 * lane;
      kx[2 * i] = *reinterpret_cast<const float4*>(kp);
      kx[2 * i + 1] = *reinterpret_cast<const float4*>(kp + 128);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int r = warp + 8 * i;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float4 x = kx[2 * i + hh];
        const int col = hh * 128 + 4 * lane;
        *reinterpret_cast<uint2*>(regK + (col >> 6) * (128 * 128) + sw128_offset(r, col & 63)) =
            make_uint2(pack_half2(x.x, x.y), pack_half2(x.z, x.w));
      }
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (t == 0) {
    tma_prefetch(&umap);
    tma_prefetch(&wmap);
    tma_store_3d(&kwmap, regK, 0, (int)rowbase, 0);   // the write keys (fp16)
    tma_store_commit();
    const uint32_t aK = smem_u32(regK);
    constexpr uint32_t idesc = idesc_f16(128, 128, 0);
#pragma unroll
    for (int ks = 0; ks < kGD / 16; ++ks)
      umma_f16_ss(tmem, sdesc_kstep(aK, 128, ks), sdesc_kstep(aK, 128, ks), idesc, ks > 0);
    umma_commit(bar_kk);
  }
  // cumulative decay inside the chunk (thread r < 128): inclusive scans of the four warps, then the totals of
  // the warps before
  float* s_wsum = reinterpret_cast<float*>(smem + kP1_Small + 1600);   // [4], after the barriers
  float gacc = 0.f;
  if (t < 128) {
    gacc = s_g[t];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, gacc, o);
      if (lane >= o) gacc += y;
    }
    if (lane == 31) s_wsum[warp] = gacc;
  }
  __syncthreads();
  if (t < 128) {
    for (int w2 = 0; w2 < warp; ++w2) gacc += s_wsum[w2];
    s_gc[t] = gacc;
    s.gc[rowbase + t] = gacc;
  }
  __syncthreads();
  // per-step factor of w's operand: beta e^{c} (<= 1)
  float* s_bec = reinterpret_cast<float*>(smem + kP1_Small + 2048 + 3072);   // [128], after the row pointers
  if (t < 128) s_bec[t] = s_beta[t] * __expf(s_gc[t]);
  // ---- (b) A = strict_lower(beta_i e^{c_i - c_j} (k_i . k_j)) from TMEM (all warps: row = lane quarter of
  //      the warp, columns 64 * (warp / 4) .. + 63)
  bool alive = true;
  {
    const int r = (warp & 3) * 32 + lane;
    const int cbase = (warp >> 2) * 64;
    alive = mbar_wait_warp(bar_kk, 0, nullptr, s.err, 0x41);
    tc_fence_after();
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const float br = s_beta[r], cr = s_gc[r];
#pragma unroll 1
    for (int c1 = cbase; c1 < cbase + 64; c1 += 32) {   // 32 columns per TMEM read
      uint32_t fa[32];
      tmem_ld32(trow + c1, fa);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int j = c1 + e;
        fa[e] = __float_as_uint((j < r && alive) ? br * __expf(cr - s_gc[j]) * __uint_as_float(fa[e]) : 0.f);
      }
#pragma unroll
      for (int e = 0; e < 32; e += 4)   // rows 528 bytes apart: the 16-byte stores of 8 lanes hit 8 bank groups
        *reinterpret_cast<uint4*>(A + r * kAS + c1 + e) = make_uint4(fa[e], fa[e + 1], fa[e + 2], fa[e + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();  // A complete
  {   // the value rows are read after the inverse: bring them into L2 while it runs
    const int r = t & 127, part = t >> 7;
    const uint8_t* vb = s.v32 ? reinterpret_cast<const uint8_t*>(s_vp32[r]) + part * 512
                              : reinterpret_cast<const uint8_t*>(s_vp[r]) + part * 256;
    prefetch_l2(vb);
    prefetch_l2(vb + 128);
    if (s.v32) {
      prefetch_l2(vb + 256);
      prefetch_l2(vb + 384);
    }
  }
  // ---- (c) T = (I + A)^-1: invert the eight 16x16 diagonal blocks (one column chain per thread), then
  //      double the solved block size 16 -> 32 -> 64 -> 128 with T21 = -T22 (A21 T11)
  for (int i = t; i < 128 * kAS; i += kP1_Threads) Tm[i] = 0.f;
  __syncthreads();
  if (t < 128) {
    // column cl of the inverse of diagonal block r0: x_m = -sum_{j<m} A[m][j] x_j below the unit diagonal;
    // the entries above it are zero, so the sums run over all j < m (rows of A read four at a time)
    const int r0 = (t >> 4) * 16, cl = t & 15;
    float x[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      float acc = 0.f;
      const float* ar = A + (r0 + m) * kAS + r0;
#pragma unroll
      for (int j4 = 0; j4 < m; j4 += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(ar + j4);
        acc = fmaf(a4.x, x[j4], acc);
        if (j4 + 1 < m) acc = fmaf(a4.y, x[j4 + 1], acc);
        if (j4 + 2 < m) acc = fmaf(a4.z, x[j4 + 2], acc);
        if (j4 + 3 < m) acc = fmaf(a4.w, x[j4 + 3], acc);
      }
      x[m] = m < cl ? 0.f : m == cl ? 1.f : -acc;
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) Tm[(r0 + m) * kAS + r0 + cl] = x[m];
  }
  __syncthreads();
  // (T stays zero above its diagonal and T11, T22 are lower triangular, so both products are plain block
  // products: X = A21 T11, T21 = -T22 X)
  float* X = reinterpret_cast<float*>(smem + kP1_RegX);  // scratch: A21 T11 for every block pair of a level
  inverse_doubling_level<16, 2, 2, 0, 0>(A, Tm, X, t);
  inverse_doubling_level<32, 4, 2, 1, 2>(A, Tm, X, t);
  inverse_doubling_level<64, 4, 4, 1, 2>(A, Tm, X, t);
  // ---- T -> T_u = T diag(beta) and T_w = T diag(beta e^c), fp16 SW128 tiles (rows i, K = j) over A: then
  //      u = T_u V and w = T_w K take the value and key tiles as they lie (token rows, MN-major B operands)
#pragma unroll 2
  for (int ch = t >> 7; ch < 16; ch += kP1_Threads / 128) {   // chunk of 8 columns
    // thread = row i: rows 528 bytes apart read distinct banks, the factors of the chunk are broadcasts
    const int i = t & 127;
    const float4* tr = reinterpret_cast<const float4*>(Tm + i * kAS + ch * 8);
    const float4* bj = reinterpret_cast<const float4*>(s_beta + ch * 8);
    const float4* ej = reinterpret_cast<const float4*>(s_bec + ch * 8);
    const float4 t0 = tr[0], t1 = tr[1], b0 = bj[0], b1 = bj[1], e0 = ej[0], e1 = ej[1];
    const uint32_t pu[4] = {pack_half2(t0.x * b0.x, t0.y * b0.y), pack_half2(t0.z * b0.z, t0.w * b0.w),
                            pack_half2(t1.x * b1.x, t1.y * b1.y), pack_half2(t1.z * b1.z, t1.w * b1.w)};
    const uint32_t pw[4] = {pack_half2(t0.x * e0.x, t0.y * e0.y), pack_half2(t0.z * e0.z, t0.w * e0.w),
                            pack_half2(t1.x * e1.x, t1.y * e1.y), pack_half2(t1.z * e1.z, t1.w * e1.w)};
    const uint32_t off = (uint32_t)(ch >> 3) * (128 * 128) + sw128_offset(i, (ch & 7) * 8);
    *reinterpret_cast<uint4*>(regA + off) = make_uint4(pu[0], pu[1], pu[2], pu[3]);
    *reinterpret_cast<uint4*>(regA + 32768 + off) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
  }
  __syncthreads();  // T (fp32) is free: the value tile goes there
  // ---- (d) value rows -> fp16 value tile [128 tokens][256] (SW128 atoms of 64 columns): warp w takes rows
  //      w + 8 i, each load covering 512 contiguous bytes of a row
  if (s.v32) {   // uniform for the launch
    float4 x[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float* vp = s_vp32[warp + 8 * i] + 4 * lane;
      x[2 * i] = *reinterpret_cast<const float4*>(vp);
      x[2 * i + 1] = *reinterpret_cast<const float4*>(vp + 128);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int r = warp + 8 * i;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float4 y = x[2 * i + hh];
        const int col = hh * 128 + 4 * lane;
        *reinterpret_cast<uint2*>(regT + (col >> 6) * (128 * 128) + sw128_offset(r, col & 63)) =
            make_uint2(pack_half2(y.x, y.y), pack_half2(y.z, y.w));
      }
    }
  } else {
    uint4 x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = *reinterpret_cast<const uint4*>(s_vp[warp + 8 * i] + 8 * lane);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int r = warp + 8 * i;
      const uint32_t w4[4] = {x[i].x, x[i].y, x[i].z, x[i].w};
      uint32_t o4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[e]));
        o4[e] = pack_half2(f.x, f.y);
      }
      *reinterpret_cast<uint4*>(regT + (lane >> 3) * (128 * 128) + sw128_offset(r, (lane & 7) * 8)) =
          make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  }
  if (t == 0) tma_store_wait_read();   // the key tile has been stored (w is staged over it at the end)
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (t == 0) {
    constexpr uint32_t idesc = idesc_f16(128, 256, 0) | kIdescBMn;
    const uint32_t aTu = smem_u32(regA), aTw = smem_u32(regA + 32768), bV = smem_u32(regT), bK = smem_u32(regK);
    // B operands: K index = token (8-token groups 1024 bytes apart), N = the 256 columns in four 64-column
    // atoms 16 KB apart; one K step of 16 tokens = two groups
#pragma unroll
    for (int ks = 0; ks < kGC / 16; ++ks)
      umma_f16_ss(tmem, sdesc_kstep(aTu, 128, ks), sdesc_sw128_mn(bV + ks * 2048, 128 * 128), idesc, ks > 0);
#pragma unroll
    for (int ks = 0; ks < kGC / 16; ++ks)
      umma_f16_ss(tmem + 256, sdesc_kstep(aTw, 128, ks), sdesc_sw128_mn(bK + ks * 2048, 128 * 128), idesc, ks > 0);
    umma_commit(bar_uw);
  }
  // ---- (e) u rows (warps 0-3) and w rows (warps 4-7) -> fp16 SW128 tiles over the operands the products
  //      have consumed (u over the value tile, w over the key tile; the 16-byte stores of 8 consecutive rows
  //      hit distinct bank groups), then one TMA store each
  {
    const int r = (warp & 3) * 32 + lane;
    const bool is_w = warp >= 4;
    alive = mbar_wait_warp(bar_uw, 0, nullptr, s.err, 0x42) && alive;
    tc_fence_after();
    const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (is_w ? 256u : 0u);
    uint8_t* tile = is_w ? regK : regT;
#pragma unroll 1
    for (int c1 = 0; c1 < 256; c1 += 64) {   // 64 columns (one atom) per TMEM wait
      uint32_t fa[64];
      tmem_ld32(trow + c1, *reinterpret_cast<uint32_t(*)[32]>(fa));
      tmem_ld32(trow + c1 + 32, *reinterpret_cast<uint32_t(*)[32]>(fa + 32));
      tmem_wait_ld();
      uint8_t* at = tile + (c1 >> 6) * (128 * 128);
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const uint32_t* f = fa + ch * 8;
        *reinterpret_cast<uint4*>(at + sw128_offset(r, ch * 8)) =
            make_uint4(pack_half2(__uint_as_float(f[0]), __uint_as_float(f[1])),
                       pack_half2(__uint_as_float(f[2]), __uint_as_float(f[3])),
                       pack_half2(__uint_as_float(f[4]), __uint_as_float(f[5])),
                       pack_half2(__uint_as_float(f[6]), __uint_as_float(f[7])));
      }
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (t == 0) {
    tma_store_3d(&umap, regT, 0, (int)rowbase, 0);
    tma_store_3d(&wmap, regK, 0, (int)rowbase, 0);
    tma_store_commit();
    tma_store_wait_read();   // shared memory may be released once the stores have read it
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================================ P2
constexpr int kP2_NB = 32;               // state columns per CTA
constexpr int kP2_Threads = 192;         // warps 0-3 state/epilogue, warp 4 TMA, warp 5 MMA
constexpr int kP2_SmemW = kGC * kGD * 2;          // 64 KB
constexpr int kP2_SmemKT = kGD * kGC * 2;         // 64 KB: the chunk's fp16 key tile [128 tokens][256]
constexpr int kP2_SmemST = kP2_NB * kGD * 2;      // 8 KB
constexpr int kP2_SmemVT = kP2_NB * kGC * 2;      // 4 KB
constexpr int kP2_Smem = kP2_SmemW + kP2_SmemKT + kP2_SmemST + kP2_SmemVT + 1024 + 256;
constexpr int kP2_Tmem = 3 * kP2_NB <= 64 ? 64 : 128;   // v' product, then the two halves of the state product

__global__ void __launch_bounds__(kP2_Threads, 1)
    gdn_p2_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap kmap, GdnStreams s) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sKT = sW + kP2_SmemW;
  uint8_t* sST = sKT + kP2_SmemKT;
  uint8_t* sVT = sST + kP2_SmemST;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sVT + kP2_SmemVT);
  uint64_t* bar_w = bars + 0;      // w tile landed
  uint64_t* bar_kt = bars + 1;     // key tile landed
  uint64_t* bar_st = bars + 2;     // S^T staged (128)
  uint64_t* bar_vt = bars + 3;     // v'^T staged (128)
  uint64_t* bar_m1 = bars + 4;     // v' product done
  uint64_t* bar_m2 = bars + 5;     // state product done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 7);

  // per-chunk arrays are indexed by bg = (batch, KV head); with packed sequences (B = 1) bg is the KV head and
  // this CTA walks the chunks of sequence blockIdx.y / G; the states are per (sequence or batch, KV head)
  int bg = blockIdx.y, sidx = blockIdx.y, c_begin = 0, c_end = s.n_chunks;
  if (s.chunk_tok0) {
    const int i = blockIdx.y / s.G;
    bg = blockIdx.y % s.G;
    c_begin = s.seq_chunk0[i];
    c_end = s.seq_chunk0[i + 1];
  }
  const int ncl = c_end - c_begin;          // chunks of this CTA; barrier phases count from its first
  // column blocks beyond the state's (transform mode only) run the map path: start at the identity, no inputs
  const bool mpath = blockIdx.x >= kGD / kP2_NB;
  const int col0 = (mpath ? blockIdx.x - kGD / kP2_NB : blockIdx.x) * kP2_NB;
  // chunk-start states and v' are kept for P3 (also by the map pass of a fix-up run, on the path from zero)
  const bool keep = (s.m_out == nullptr || s.MC != nullptr) && !mpath;
  const bool keep_map = mpath && s.MC != nullptr;   // the transition path keeps its chunk-start maps
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nch = s.n_chunks;
  if (t == 0) {
    mbar_init(bar_w, 1);
    mbar_init(bar_kt, 1);
    mbar_init(bar_st, 128);
    mbar_init(bar_vt, 128);
    mbar_init(bar_m1, 1);
    mbar_init(bar_m2, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kP2_Tmem);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch(&wmap);
      tma_prefetch(&kmap);
      int iw = 0, ik = 0;
      for (int j = 0; j < ncl; ++j) {
        const int c = c_begin + j;
        if (j >= 1 && !mbar_wait(bar_m1, (j - 1) & 1, abort_flag, s.err, 0x51)) break;
        mbar_expect_tx(bar_w, kP2_SmemW);
        tma_load_3d(sW, &wmap, bar_w, 0, bg * s.n_pad + c * kGC, 0);
        iw = j + 1;
        if (j >= 1 && !mbar_wait(bar_m2, (j - 1) & 1, abort_flag, s.err, 0x52)) break;
        mbar_expect_tx(bar_kt, kP2_SmemKT);
        tma_load_3d(sKT, &kmap, bar_kt, 0, bg * s.n_pad + c * kGC, 0);   // the chunk's fp16 keys
        ik = j + 1;
      }
      if (iw > 0) mbar_wait(bar_w, (iw - 1) & 1, nullptr, s.err, 0x53);
      if (ik > 0) mbar_wait(bar_kt, (ik - 1) & 1, nullptr, s.err, 0x54);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t id1 = idesc_f16(128, kP2_NB, 0);
      const uint32_t aW = smem_u32(sW), bST = smem_u32(sST), aKT = smem_u32(sKT), bVT = smem_u32(sVT);
      for (int j = 0; j < ncl; ++j) {
        if (!mbar_wait(bar_w, j & 1, abort_flag, s.err, 0x55)) break;
        if (!mbar_wait(bar_st, j & 1, abort_flag, s.err, 0x56)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kGD / 16; ++ks)
          umma_f16_ss(tmem, sdesc_kstep(aW, 128, ks), sdesc_kstep(bST, kP2_NB, ks), id1, ks > 0);
        umma_commit(bar_m1);
        if (!mbar_wait(bar_kt, j & 1, abort_flag, s.err, 0x57)) break;
        if (!mbar_wait(bar_vt, j & 1, abort_flag, s.err, 0x58)) break;
        tc_fence_after();
        // dS = K^T (e^{c_C - c} v'): A = the key tile as it lies (token rows: M = dimensions in 64-column
        // atoms 16 KB apart, MN-major), rows mt * 128 .. of the state in atoms 2 mt, 2 mt + 1
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
          for (int ks = 0; ks < kGC / 16; ++ks) {
            const uint32_t a = aKT + (uint32_t)mt * (2 * 128 * 128) + (uint32_t)ks * 2048u;
            umma_f16_ss(tmem + kP2_NB * (1 + mt), sdesc_sw128_mn(a, 128 * 128), sdesc_kstep(bVT, kP2_NB, ks),
                        id1 | kIdescAMn, ks > 0);
          }
        }
        umma_commit(bar_m2);
      }
    }
  } else {
    // warps 0-3: thread r owns state rows r and r + 128 (columns col0 .. col0 + kP2_NB - 1) and token row r
    const int r = t;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    float S0[kP2_NB], S1[kP2_NB];
    if (mpath) {
#pragma unroll
      for (int e = 0; e < kP2_NB; ++e) {
        S0[e] = (r == col0 + e) ? 1.f : 0.f;
        S1[e] = (r + 128 == col0 + e) ? 1.f : 0.f;
      }
    } else if (s.s0) {
      const float* sp = s.s0 + (size_t)sidx * kGD * kGD;
#pragma unroll
      for (int e = 0; e < kP2_NB; e += 4) {
        const float4 x0 = *reinterpret_cast<const float4*>(sp + (size_t)r * kGD + col0 + e);
        const float4 x1 = *reinterpret_cast<const float4*>(sp + (size_t)(r + 128) * kGD + col0 + e);
        S0[e] = x0.x; S0[e + 1] = x0.y; S0[e + 2] = x0.z; S0[e + 3] = x0.w;
        S1[e] = x1.x; S1[e + 1] = x1.y; S1[e + 2] = x1.z; S1[e + 3] = x1.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < kP2_NB; ++e) S0[e] = S1[e] = 0.f;
    }
    bool alive = true;
    float lsum = 0.f;   // map path: log of the cumulative decay
    for (int j = 0; j < ncl && alive; ++j) {
      const int c = c_begin + j;
      // the chunk's decays, read first so that they are in registers when the products need them
      const float* gcc = s.gc + (size_t)bg * s.n_pad + (size_t)c * kGC;
      const float lgc = gcc[kGC - 1], gcr = gcc[r];
      // stage S^T (fp16) as the B operand of v' = u - w S, and store it for P3
#pragma unroll
      for (int e = 0; e < kP2_NB; ++e) {
        st_half_sw128(sST, kP2_NB, e, r, S0[e]);
        st_half_sw128(sST, kP2_NB, e, r + 128, S1[e]);
      }
      if (keep) {
        __half* stg = s.ST + (((size_t)bg * nch + c) * kGD + col0) * kGD;
#pragma unroll
        for (int e = 0; e < kP2_NB; ++e) {
          stg[(size_t)e * kGD + r] = __float2half_rn(S0[e]);
          stg[(size_t)e * kGD + r + 128] = __float2half_rn(S1[e]);
        }
      }
      if (keep_map) {   // M_c, row-major fp16 at its true scale (the path keeps it divided by the decay so far)
        const float f = __expf(lsum);
        __half* mc = s.MC + (((size_t)bg * nch + c) * kGD + r) * kGD + col0;
#pragma unroll
        for (int e = 0; e < kP2_NB; e += 8) {
          *reinterpret_cast<uint4*>(mc + e) =
              make_uint4(pack_half2(S0[e] * f, S0[e + 1] * f), pack_half2(S0[e + 2] * f, S0[e + 3] * f),
                         pack_half2(S0[e + 4] * f, S0[e + 5] * f), pack_half2(S0[e + 6] * f, S0[e + 7] * f));
          *reinterpret_cast<uint4*>(mc + (size_t)128 * kGD + e) =
              make_uint4(pack_half2(S1[e] * f, S1[e + 1] * f), pack_half2(S1[e + 2] * f, S1[e + 3] * f),
                         pack_half2(S1[e + 4] * f, S1[e + 5] * f), pack_half2(S1[e + 6] * f, S1[e + 7] * f));
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(bar_st);
      // u row r (this chunk), columns col0 .. col0 + kP2_NB - 1
      const __half* up = s.u + ((size_t)bg * s.n_pad + (size_t)c * kGC + r) * kGD + col0;
      float uu[kP2_NB];
      if (mpath) {
#pragma unroll
        for (int e = 0; e < kP2_NB; ++e) uu[e] = 0.f;
      } else {
#pragma unroll
        for (int h8 = 0; h8 < kP2_NB / 8; ++h8) {
          const uint4 a0 = *reinterpret_cast<const uint4*>(up + 8 * h8);
          const uint32_t w[4] = {a0.x, a0.y, a0.z, a0.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
            uu[8 * h8 + 2 * e] = f2.x;
            uu[8 * h8 + 2 * e + 1] = f2.y;
          }
        }
      }
      // the state update's B operand carries the decay to the chunk end: (e^{c_C - c_r} v'_r)^T
      const float ect = __expf(lgc - gcr);
      if (!mbar_wait_warp(bar_m1, j & 1, abort_flag, s.err, 0x59)) { alive = false; break; }
      tc_fence_after();
      float dv[kP2_NB];
#pragma unroll
      for (int q = 0; q < kP2_NB; q += 16) tmem_ld16_wait(trow + q, *reinterpret_cast<float(*)[16]>(dv + q));
#pragma unroll
      for (int e = 0; e < kP2_NB; ++e) st_half_sw128(sVT, kP2_NB, e, r, (uu[e] - dv[e]) * ect);
      if (keep) {
        __half* vtg = s.VT + (((size_t)bg * nch + c) * kGD + col0) * kGC;
#pragma unroll
        for (int e = 0; e < kP2_NB; ++e) vtg[(size_t)e * kGC + r] = __float2half_rn(uu[e] - dv[e]);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(bar_vt);
      const float decay = __expf(lgc);
      if (!mbar_wait_warp(bar_m2, j & 1, abort_flag, s.err, 0x5a)) { alive = false; break; }
      tc_fence_after();
      float d0[kP2_NB], d1[kP2_NB];
#pragma unroll
      for (int q = 0; q < kP2_NB; q += 16) {
        tmem_ld16_wait(trow + kP2_NB + q, *reinterpret_cast<float(*)[16]>(d0 + q));
        tmem_ld16_wait(trow + 2 * kP2_NB + q, *reinterpret_cast<float(*)[16]>(d1 + q));
      }
      if (mpath) {
        // the map path keeps its state divided by the cumulative decay (the recurrence is homogeneous), so the
        // fp16 operand copies stay in range however far the segment decays; the factor is applied at the end
        const float inv = __expf(-lgc);
        lsum += lgc;
#pragma unroll
        for (int e = 0; e < kP2_NB; ++e) {
          S0[e] = fmaf(d0[e], inv, S0[e]);
          S1[e] = fmaf(d1[e], inv, S1[e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < kP2_NB; ++e) {
          S0[e] = decay * S0[e] + d0[e];
          S1[e] = decay * S1[e] + d1[e];
        }
      }
      tc_fence_before();
    }
    if (alive && mpath) {
      const float f = __expf(lsum);
#pragma unroll
      for (int e = 0; e < kP2_NB; ++e) {
        S0[e] *= f;
        S1[e] *= f;
      }
    }
    if (alive) {
      float* so = (mpath ? s.m_out : s.s_out) + (size_t)sidx * kGD * kGD;
#pragma unroll
      for (int e = 0; e < kP2_NB; e += 4) {
        *reinterpret_cast<float4*>(so + (size_t)r * kGD + col0 + e) = make_float4(S0[e], S0[e + 1], S0[e + 2], S0[e + 3]);
        *reinterpret_cast<float4*>(so + (size_t)(r + 128) * kGD + col0 + e) =
            make_float4(S1[e], S1[e + 1], S1[e + 2], S1[e + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kP2_Tmem);
  }
}

// ============================================================================================ SP fix-up
// Sequence parallelism, second phase.  The map pass kept, per chunk c of this segment, the chunk-start state from a
// zero incoming state (N_c^T in ST) with its corrected values (v'^N_c^T in VT), and the chunk-start transition
// M_c (MC, fp16 row-major [k][j]).  From an incoming state S_in the chunk starts at S_c = M_c S_in + N_c, and its
// corrected values are v'_c = u_c - w_c S_c = v'^N_c - w_c (M_c S_in).  With Z = M_c S_in on the tensor core,
// one CTA per (batch x KV head, chunk, value half) rewrites in place
//   ST <- N_c^T + Z^T              (128 value rows x 256 key columns, fp16)
//   VT <- v'^N_c^T - Z^T w_c^T      (128 value rows x 128 tokens, fp16)
// so the memory reads (P3) run unchanged.  All chunks at once: this replaces a second sequential scan.
constexpr int kFX_Threads = 192;            // warps 0-3 epilogue (thread = value row), warp 4 TMA, warp 5 MMA
constexpr int kFX_SmemA = 128 * kGD * 2;    // 64 KB: S_in^T half (A of Z^T), then Z^T (A of the value product)
constexpr int kFX_SmemB = kGD * kGD * 2;    // 128 KB: M_c [k][j] (B of Z^T), then w_c [t][k] in its first half
constexpr int kFX_Smem = kFX_SmemA + kFX_SmemB + 1024 + 256;

// SinT[bg][v][j] = fp16(S[bg][j][v]) for the fix-up's A operand (32 x 32 tiles through shared memory)
__global__ void sp_sin_transpose_kernel(const float* __restrict__ S, __half* __restrict__ SinT) {
  __shared__ float tile[32][33];
  const size_t off = (size_t)blockIdx.z * kGD * kGD;
  const int j0 = blockIdx.y * 32, v0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) tile[i][threadIdx.x] = S[off + (size_t)(j0 + i) * kGD + v0 + threadIdx.x];
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y)
    SinT[off + (size_t)(v0 + i) * kGD + j0 + threadIdx.x] = __float2half_rn(tile[threadIdx.x][i]);
}

__global__ void __launch_bounds__(kFX_Threads, 1)
    gdn_sp_fixup_kernel(const __grid_constant__ CUtensorMap sinmap, const __grid_constant__ CUtensorMap mcmap,
                        const __grid_constant__ CUtensorMap wmap, GdnStreams s) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + kFX_SmemA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kFX_SmemB);
  uint64_t* bar_a = bars + 0;    // S_in^T half landed
  uint64_t* bar_b = bars + 1;    // M_c landed
  uint64_t* bar_m1 = bars + 2;   // Z^T product done (A and B free)
  uint64_t* bar_z = bars + 3;    // Z^T staged in fp16 (128 arrivals)
  uint64_t* bar_w = bars + 4;    // w_c landed
  uint64_t* bar_m2 = bars + 5;   // value product done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 7);
  const int c = blockIdx.x, bg = blockIdx.y, vh = blockIdx.z;
  const int nch = s.n_chunks;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if (t == 0) {
    mbar_init(bar_a, 1);
    mbar_init(bar_b, 1);
    mbar_init(bar_m1, 1);
    mbar_init(bar_z, 128);
    mbar_init(bar_w, 1);
    mbar_init(bar_m2, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);   // Z^T at columns 0..255, the value product at 256..383
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch(&sinmap);
      tma_prefetch(&mcmap);
      tma_prefetch(&wmap);
      mbar_expect_tx(bar_a, kFX_SmemA);
      tma_load_3d(sA, &sinmap, bar_a, 0, bg * kGD + vh * 128, 0);
      mbar_expect_tx(bar_b, kFX_SmemB);
      tma_load_3d(sB, &mcmap, bar_b, 0, (bg * nch + c) * kGD, 0);
      bool got_w = false;
      if (mbar_wait(bar_m1, 0, abort_flag, s.err, 0xB1)) {   // M_c consumed: w_c goes over it
        mbar_expect_tx(bar_w, kGC * kGD * 2);
        tma_load_3d(sB, &wmap, bar_w, 0, bg * s.n_pad + c * kGC, 0);
        got_w = true;
      }
      // the CTA ends only after its loads landed
      mbar_wait(bar_a, 0, nullptr, s.err, 0xB2);
      mbar_wait(bar_b, 0, nullptr, s.err, 0xB2);
      if (got_w) mbar_wait(bar_w, 0, nullptr, s.err, 0xB2);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t aA = smem_u32(sA), aB = smem_u32(sB);
      if (mbar_wait(bar_a, 0, abort_flag, s.err, 0xB3) && mbar_wait(bar_b, 0, abort_flag, s.err, 0xB4)) {
        tc_fence_after();
        constexpr uint32_t id1 = idesc_f16(128, 256, 0);
#pragma unroll
        for (int ks = 0; ks < kGD / 16; ++ks)
          umma_f16_ss(tmem, sdesc_kstep(aA, 128, ks), sdesc_kstep(aB, kGD, ks), id1, ks > 0);
        umma_commit(bar_m1);
        if (mbar_wait(bar_z, 0, abort_flag, s.err, 0xB5) && mbar_wait(bar_w, 0, abort_flag, s.err, 0xB6)) {
          tc_fence_after();
          constexpr uint32_t id2 = idesc_f16(128, kGC, 0);
#pragma unroll
          for (int ks = 0; ks < kGD / 16; ++ks)
            umma_f16_ss(tmem + 256, sdesc_kstep(aA, 128, ks), sdesc_kstep(aB, kGC, ks), id2, ks > 0);
          umma_commit(bar_m2);
        }
      }
    }
  } else {
    // warps 0-3: thread r = value row vh * 128 + r
    const int r = t;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    const size_t vrow = ((size_t)bg * nch + c) * kGD + (size_t)vh * 128 + r;
    __half* st = s.ST + vrow * kGD;     // [k] of this value row
    __half* vt = s.VT + vrow * kGC;     // [t] of this value row
    bool ok = mbar_wait_warp(bar_m1, 0, abort_flag, s.err, 0xB7);
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c1 = 0; c1 < kGD; c1 += 32) {
        uint32_t z[32];
        tmem_ld32(trow + c1, z);
        tmem_wait_ld();
        // S_c^T row = N_c^T row + Z^T row (in place), and Z^T (fp16) staged as the next product's A operand
        uint4* sp4 = reinterpret_cast<uint4*>(st + c1);
        uint8_t* atom = sA + (c1 >> 6) * (128 * 128);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 nv = sp4[q];
          const uint32_t nw[4] = {nv.x, nv.y, nv.z, nv.w};
          uint32_t ow[4], zw[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float z0 = __uint_as_float(z[8 * q + 2 * e]), z1 = __uint_as_float(z[8 * q + 2 * e + 1]);
            const float2 n2 = __half22float2(*reinterpret_cast<const __half2*>(&nw[e]));
            ow[e] = pack_half2(n2.x + z0, n2.y + z1);
            zw[e] = pack_half2(z0, z1);
          }
          sp4[q] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
          *reinterpret_cast<uint4*>(atom + sw128_offset(r, (c1 & 63) + 8 * q)) = make_uint4(zw[0], zw[1], zw[2], zw[3]);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    mbar_arrive(bar_z);
    ok = ok && mbar_wait_warp(bar_m2, 0, abort_flag, s.err, 0xB8);
    if (ok) {
      tc_fence_after();
#pragma unroll 1
      for (int c1 = 0; c1 < kGC; c1 += 32) {
        uint32_t y[32];
        tmem_ld32(trow + 256 + c1, y);
        tmem_wait_ld();
        uint4* vp4 = reinterpret_cast<uint4*>(vt + c1);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 vv = vp4[q];
          const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
          uint32_t ow[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(&vw[e]));
            ow[e] = pack_half2(v2.x - __uint_as_float(y[8 * q + 2 * e]), v2.y - __uint_as_float(y[8 * q + 2 * e + 1]));
          }
          vp4[q] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================================ P3
// Persistent: a CTA walks work items (b, chunk, KV head g, value half vh) round-robin and, per item, the R
// query heads of g.  The chunk's keys K, the state half S_vh^T and v'_vh^T stay in shared memory for the
// item; each head's queries Q (fp16) stream through one buffer.  Per head:
//   A = Q K^T (TMEM, one of two buffers) -> P = decayed causal A, fp16, written by the epilogue warps over
//   the first half of their own A columns (the TMEM A operand of the next product) ->
//   inter = Q S_vh^T, intra = P v'_vh (TMEM) -> o[:, vh half] = e^c inter + intra (+ gate and mix).
// TMEM holds one A / P buffer and three output buffers X: inter is computed into X, the epilogue scales each
// row by e^{c} in place while it stages P, and intra accumulates on top, so X = o_mem when the head's
// products are done.  While the epilogue mixes and stores head m-1 from its X, the tensor core computes
// intra of head m and Q K^T / inter of head m+1 into the other buffers; the stores stream HBM continuously.
constexpr int kP3_Threads = 320;   // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue (two per TMEM lane quarter)
constexpr int kP3_Epi = 256;       // epilogue threads: row (warp & 3) * 32 + lane, columns ((warp - 2) >> 2) * 64 .. + 63
constexpr int kP3_SmemK = kGC * kGD * 2;      // 64 KB: k tile [128 tokens][256]
constexpr int kP3_SmemS = 128 * kGD * 2;      // 64 KB: S^T half [128 dv][256 dk]
constexpr int kP3_SmemV = 128 * kGC * 2;      // 32 KB: v'^T half [128 dv][128 tokens]
constexpr int kP3_SmemQ = kGC * kGD * 2;      // 64 KB: queries of one head [128][256]
constexpr int kP3_Smem = kP3_SmemK + kP3_SmemS + kP3_SmemV + kP3_SmemQ + 1024 + 256;
constexpr uint32_t kP3_TA = 0;     // A / P
constexpr uint32_t kP3_TX = 128;   // output buffers at 128, 256, 384 (head index mod 3)

struct P3Item {
  int b, c, g, vh;
};
__device__ __forceinline__ P3Item p3_item(const GdnStreams& s, long long u) {
  P3Item it;
  it.vh = (int)(u & 1);
  const long long t = u >> 1;
  it.g = (int)(t % s.G);
  const long long bc = t / s.G;
  const int c0 = s.p3_c1 > 0 ? s.p3_c0 : 0;
  const int nr = s.p3_c1 > 0 ? s.p3_c1 - s.p3_c0 : s.n_chunks;
  it.c = c0 + (int)(bc % nr);
  it.b = (int)(bc / nr);
  return it;
}
__device__ __forceinline__ long long p3_qrow0(const GdnStreams& s, const P3Item& it) {
  return s.chunk_tok0 ? (long long)s.chunk_tok0[it.c] : (long long)it.b * s.T + s.qoff + (long long)it.c * kGC;
}

// per (head, row) epilogue context of one epilogue thread
struct P3Ctx {
  float* orow;        // output row, this thread's 64 columns
  const __half* owp;  // its window result in the workspace: 8 fp16 of column group e8 at owp + e8 * 256
  const float* gcc;   // cumulative log-decay of the chunk
  float ci, eci, gam, rho;
  bool row_ok, gate_on, need_ow;   // need_ow: the output is the window result (mixed when gate_on)
};
// the window result of this thread's 8-column group e8 (fp16): from the workspace, or from o itself
__device__ __forceinline__ uint4 p3_load_ow(const P3Ctx& x, int e8) {
  if (x.owp) return *reinterpret_cast<const uint4*>(x.owp + e8 * 256);
  const float4 lo = *reinterpret_cast<const float4*>(x.orow + 8 * e8);
  const float4 hi = *reinterpret_cast<const float4*>(x.orow + 8 * e8 + 4);
  return make_uint4(pack_half2(lo.x, lo.y), pack_half2(lo.z, lo.w), pack_half2(hi.x, hi.y), pack_half2(hi.z, hi.w));
}
__device__ __forceinline__ float4 p3_ow4(const uint4& u, int half) {   // columns 4 half .. 4 half + 3 of a group
  const uint32_t a = half ? u.z : u.x, b = half ? u.w : u.y;
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&a));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&b));
  return make_float4(f0.x, f0.y, f1.x, f1.y);
}

__device__ __forceinline__ P3Ctx p3_ctx(const GdnStreams& s, const P3Item& it, int rh, int r, int cb) {
  const int H = s.G * s.R, h = it.g * s.R + rh, bg = it.b * s.G + it.g;
  const long long qrow0 = p3_qrow0(s, it);
  const int nvalid = s.chunk_tok0 ? s.chunk_len[it.c] : s.n_steps - it.c * kGC;
  P3Ctx x;
  x.gcc = s.gc + (size_t)bg * s.n_pad + (size_t)it.c * kGC;
  x.ci = x.gcc[r];
  x.eci = __expf(x.ci);
  x.row_ok = r < nvalid;
  x.orow = s.o + (((size_t)qrow0 + r) * H + h) * kGD + it.vh * 128 + cb * 64;
  // tile order [value half][column block][row group][8-column group][row in group][8]
  x.owp = s.owin ? s.owin + (((size_t)it.b * s.n_chunks + it.c) * H + h) * (size_t)(kGC * kGD) +
                       ((size_t)(((it.vh * 2 + cb) * 4 + (r >> 5)) * 8) * 32 + (r & 31)) * 8
                 : nullptr;
  x.need_ow = s.mix && x.row_ok && s.owin != nullptr;
  x.gate_on = false;
  x.gam = x.rho = 0.f;
  if (s.mix && x.row_ok) {
    const long long tq = qrow0 + r - (long long)it.b * s.T;   // token index within its sequence
    x.gate_on = s.pos0 + tq >= s.W;
    x.need_ow = x.need_ow || x.gate_on;
    if (x.gate_on) {
      const float lse = s.lse[((size_t)it.b * H + h) * s.T + tq];
      const float z = s.mixx[((size_t)it.b * s.T + tq) * H + h] + s.mix_lse[h] * (lse - logf((float)s.W));
      x.gam = 1.f / (1.f + __expf(-z));
      x.rho = s.mem_scale[h];
    }
  }
  return x;
}

// TMEM column of the fp16 P operand for key step ks (16 keys): the epilogue thread of column block cb writes
// the probabilities of keys cb*64 .. cb*64+63 into the first 32 columns of its own 64 A columns
__device__ __forceinline__ uint32_t p3_pcol(int ks) { return (uint32_t)((ks >> 2) * 64 + (ks & 3) * 8); }

__global__ void __launch_bounds__(kP3_Threads, 1)
    gdn_p3_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap vmap, GdnStreams s) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sS = sK + kP3_SmemK;
  uint8_t* sV = sS + kP3_SmemS;
  uint8_t* sQ = sV + kP3_SmemV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQ + kP3_SmemQ);
  uint64_t* bar_k = bars + 0;      // K landed (per item)
  uint64_t* bar_s = bars + 1;      // S^T half landed (per item)
  uint64_t* bar_v = bars + 2;      // v'^T half landed (per item)
  uint64_t* bar_kf = bars + 3;     // the item's last Q K^T done: K buffer free
  uint64_t* bar_sf = bars + 4;     // the item's last inter done: S buffer free
  uint64_t* bar_vf = bars + 5;     // the item's last intra done: v' buffer free
  uint64_t* bar_q = bars + 6;      // Q landed (per head)
  uint64_t* bar_qf = bars + 7;     // inter done: Q buffer free (per head)
  uint64_t* bar_a = bars + 8;      // A ready (per head)
  uint64_t* bar_i = bars + 9;      // inter done: X readable for the scaling (per head)
  uint64_t* bar_p = bars + 10;     // P staged and X scaled (kP3_Epi arrivals, per head)
  uint64_t* bar_paf = bars + 11;   // intra done: A / P buffer free (per head)
  uint64_t* bar_o = bars + 12;     // intra done: X = o_mem (per head)
  uint64_t* bar_xf = bars + 13;    // [3] X buffer drained (kP3_Epi arrivals; buffer = head mod 3)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 17);

  const int R = s.R, G = s.G, H = G * R;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nch = s.n_chunks;
  // packed sequences: chunks beyond the last sequence's are not work (B = 1, so they are the trailing items)
  const long long nitems =
      2LL * G * (s.chunk_tok0 ? (long long)s.seq_chunk0[s.n_seq] : (long long)s.B * (s.p3_c1 > 0 ? s.p3_c1 - s.p3_c0 : nch));
  if (t == 0) {
    for (int i = 0; i < 16; ++i)
      mbar_init(bars + i, (i == 10 || i >= 13) ? kP3_Epi : 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&qmap);
      tma_prefetch(&kmap);
      tma_prefetch(&smap);
      tma_prefetch(&vmap);
      int n = 0, m = 0;
      bool ok = true;
      for (long long u = blockIdx.x; u < nitems && ok; u += gridDim.x, ++n) {
        const P3Item it = p3_item(s, u);
        const int bg = it.b * G + it.g;
        const long long qrow0 = p3_qrow0(s, it);
        const int row_st = (bg * nch + it.c) * kGD + it.vh * 128;
        if (n > 0) ok = mbar_wait(bar_kf, (n - 1) & 1, abort_flag, s.err, 0x61);
        if (!ok) break;
        mbar_expect_tx(bar_k, kP3_SmemK);
        tma_load_3d(sK, &kmap, bar_k, 0, bg * s.n_pad + it.c * kGC, 0);
        for (int rh = 0; rh < R && ok; ++rh, ++m) {
          if (m > 0) ok = mbar_wait(bar_qf, (m - 1) & 1, abort_flag, s.err, 0x62);
          if (!ok) break;
          mbar_expect_tx(bar_q, kP3_SmemQ);
          tma_load_4d(sQ, &qmap, bar_q, 0, (int)qrow0, 0, it.g * R + rh);
          if (rh == 0) {
            if (n > 0) ok = mbar_wait(bar_sf, (n - 1) & 1, abort_flag, s.err, 0x63);
            if (!ok) break;
            mbar_expect_tx(bar_s, kP3_SmemS);
            tma_load_3d(sS, &smap, bar_s, 0, row_st, 0);
            if (n > 0) ok = mbar_wait(bar_vf, (n - 1) & 1, abort_flag, s.err, 0x64);
            if (!ok) break;
            mbar_expect_tx(bar_v, kP3_SmemV);
            tma_load_3d(sV, &vmap, bar_v, 0, row_st, 0);
          }
        }
      }
      // drain: every TMA issued has landed before the CTA may exit
      if (n > 0) {
        mbar_wait(bar_k, (n - 1) & 1, nullptr, s.err, 0x65);
        mbar_wait(bar_s, (n - 1) & 1, nullptr, s.err, 0x65);
        mbar_wait(bar_v, (n - 1) & 1, nullptr, s.err, 0x65);
      }
      if (m > 0) mbar_wait(bar_q, (m - 1) & 1, nullptr, s.err, 0x60);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id128 = idesc_f16(128, 128, 0);
      const uint32_t aQ = smem_u32(sQ), bK = smem_u32(sK), bS = smem_u32(sS), bV = smem_u32(sV);
      int n = 0, m = 0;
      bool ok = true;
      for (long long u = blockIdx.x; u < nitems && ok; u += gridDim.x, ++n) {
        for (int rh = 0; rh < R; ++rh, ++m) {
          const int xb = m % 3;
          const uint32_t X = tmem + kP3_TX + 128u * (uint32_t)xb;
          // A = Q K^T (the A / P buffer is free once intra of head m-1 has read its P)
          ok = mbar_wait(bar_q, m & 1, abort_flag, s.err, 0x66) &&
               (rh > 0 || mbar_wait(bar_k, n & 1, abort_flag, s.err, 0x67)) &&
               (m < 1 || mbar_wait(bar_paf, (m - 1) & 1, abort_flag, s.err, 0x68));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kGD / 16; ++ks)
            umma_f16_ss(tmem + kP3_TA, sdesc_kstep(aQ, 128, ks), sdesc_kstep(bK, 128, ks), id128, ks > 0);
          umma_commit(bar_a);
          if (rh == R - 1) umma_commit(bar_kf);
          // inter = Q S^T into X (free once head m-3's output has been stored)
          ok = (m < 3 || mbar_wait(&bar_xf[xb], ((m / 3) - 1) & 1, abort_flag, s.err, 0x69)) &&
               (rh > 0 || mbar_wait(bar_s, n & 1, abort_flag, s.err, 0x6a));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kGD / 16; ++ks)
            umma_f16_ss(X, sdesc_kstep(aQ, 128, ks), sdesc_kstep(bS, 128, ks), id128, ks > 0);
          umma_commit(bar_i);
          umma_commit(bar_qf);
          if (rh == R - 1) umma_commit(bar_sf);
          // X (scaled by e^c) += P v' with P from TMEM
          ok = mbar_wait(bar_p, m & 1, abort_flag, s.err, 0x6d) &&
               (rh > 0 || mbar_wait(bar_v, n & 1, abort_flag, s.err, 0x6e));
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kGC / 16; ++ks)
            umma_f16_ts(X, tmem + kP3_TA + p3_pcol(ks), sdesc_kstep(bV, 128, ks), id128, 1u);
          umma_commit(bar_o);
          umma_commit(bar_paf);
          if (rh == R - 1) umma_commit(bar_vf);
        }
      }
    }
  } else {
    const int q4 = warp & 3;
    const int cb = (warp - 2) >> 2;   // column block (64 keys of A, 64 value columns of the half)
    const int r = q4 * 32 + lane;     // row of the chunk
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    uint4 ow[8];       // window result (fp16) of the head whose output is written next
    P3Ctx pc{};
    bool have_prev = false, alive = true;
    long long u = blockIdx.x;
    int rh = 0, m = 0;
    P3Item it{};
    if (u < nitems) it = p3_item(s, u);
    for (;;) {
      const bool has_cur = u < nitems;
      P3Ctx cc{};
      if (has_cur) cc = p3_ctx(s, it, rh, r, cb);
      if (m == 0 && cc.need_ow) {
#pragma unroll
        for (int e8 = 0; e8 < 8; ++e8) ow[e8] = p3_load_ow(cc, e8);
      }
      if (has_cur) {
        // 1. P of this head over the first half of this thread's A columns: the 64 scores in one TMEM read, the
        //    decays of the keys (the same for every lane: broadcast loads) 16 at a time
        const uint32_t pa = trow + kP3_TA + cb * 64;
        const float4* g4 = reinterpret_cast<const float4*>(cc.gcc + cb * 64);
        const float ci2 = cc.ci * kLog2e;
        alive = mbar_wait_warp(bar_a, m & 1, abort_flag, s.err, 0x6c);
        if (!alive) break;
        tc_fence_after();
#pragma unroll 1
        for (int h2 = 0; h2 < 2; ++h2) {   // 32 keys per TMEM read (P of a half lands behind its reads)
          uint32_t av[32];
          tmem_ld32(pa + h2 * 32, av);
          tmem_wait_ld();
#pragma unroll
          for (int q2 = 0; q2 < 2; ++q2) {   // 16 keys per step: A columns q*16.., P columns q*8..
            const int q = h2 * 2 + q2, j0 = cb * 64 + q * 16;
            uint32_t pk[8];
            if (j0 > q4 * 32 + 31) {   // every key after every row of this warp (warp-uniform)
#pragma unroll
              for (int e = 0; e < 8; ++e) pk[e] = 0u;
            } else if (q4 * 32 >= j0 + 15) {
              // every row of the warp at or after every key: with l = j0 + 15, e^{c_i - c_j} = e^{c_i - c_l} e^{c_l - c_j},
              // both factors <= 1; lane l's column factor is that of key j0 + (l & 15), passed round by shuffles
              const float cl = cc.gcc[j0 + 15];
              const float rowf = ex2_approx((cc.ci - cl) * kLog2e);
              const float colf = ex2_approx((cl - cc.gcc[j0 + (lane & 15)]) * kLog2e);
#pragma unroll
              for (int e = 0; e < 16; e += 2) {
                const int jj = q2 * 16 + e;
                const float f0 = __shfl_sync(0xffffffffu, colf, e), f1 = __shfl_sync(0xffffffffu, colf, e + 1);
                pk[e / 2] = pack_half2(__uint_as_float(av[jj]) * rowf * f0, __uint_as_float(av[jj + 1]) * rowf * f1);
              }
            } else {   // the keys around the diagonal: one exponential per element, masked causally
              float4 gk[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) gk[i] = g4[q * 4 + i];
#pragma unroll
              for (int e = 0; e < 16; e += 2) {
                const int jj = q2 * 16 + e, j = j0 + e;
                const float4 g = gk[e >> 2];
                const float g0 = (e & 2) ? g.z : g.x, g1 = (e & 2) ? g.w : g.y;
                const float p0 = (j <= r) ? __uint_as_float(av[jj]) * ex2_approx(fmaf(-g0, kLog2e, ci2)) : 0.f;
                const float p1 =
                    (j + 1 <= r) ? __uint_as_float(av[jj + 1]) * ex2_approx(fmaf(-g1, kLog2e, ci2)) : 0.f;
                pk[e / 2] = pack_half2(p0, p1);
              }
            }
            tmem_st8(pa + q * 8, pk);
          }
        }
        // 2. inter * e^c in place (intra accumulates on top)
        alive = mbar_wait_warp(bar_i, m & 1, abort_flag, s.err, 0x5e);
        if (!alive) break;
        tc_fence_after();
        const uint32_t xr = trow + kP3_TX + 128u * (uint32_t)(m % 3) + cb * 64;
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
          uint32_t w[16];
          tmem_ld16(xr + q * 16, w);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) w[e] = __float_as_uint(__uint_as_float(w[e]) * cc.eci);
          tmem_st16(xr + q * 16, w);
        }
        tmem_wait_st();
      }
      // the previous head's products are complete before this head's intra may start (keeps bar_o one phase
      // ahead at most)
      if (have_prev) {
        alive = mbar_wait_warp(bar_o, (m - 1) & 1, abort_flag, s.err, 0x6b);
        if (!alive) break;
      }
      if (has_cur) {
        tc_fence_before();
        mbar_arrive(bar_p);
      }
      // 3. the previous head's output: mixed in row order (thread = row) and written back over its X, then
      //    stored from X in 16-row blocks, four threads per 32 contiguous bytes of a row (full sectors); this
      //    head's window result is read into the registers as they are used
      if (have_prev) {
        tc_fence_after();
        const bool refill = has_cur && cc.need_ow;
        const uint32_t xcol = kP3_TX + 128u * (uint32_t)((m - 1) % 3) + cb * 64;
        const uint32_t xr = trow + xcol;
#pragma unroll
        for (int sub2 = 0; sub2 < 2; ++sub2) {
          uint32_t o32[32];
          tmem_ld32(xr + sub2 * 32, o32);
          tmem_wait_ld();
#pragma unroll
          for (int sh = 0; sh < 2; ++sh) {
          const int sub = sub2 * 2 + sh;
          const float* om = reinterpret_cast<const float*>(o32) + sh * 16;
          uint32_t w[16];
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const int e = sub * 4 + e4;
            float4 res;
            if (pc.gate_on) {
              const float4 v = p3_ow4(ow[e >> 1], e & 1);
              res.x = v.x + pc.gam * (pc.rho * om[4 * e4] - v.x);
              res.y = v.y + pc.gam * (pc.rho * om[4 * e4 + 1] - v.y);
              res.z = v.z + pc.gam * (pc.rho * om[4 * e4 + 2] - v.z);
              res.w = v.w + pc.gam * (pc.rho * om[4 * e4 + 3] - v.w);
            } else if (pc.need_ow) {   // rows below the window: the window result as it is
              res = p3_ow4(ow[e >> 1], e & 1);
            } else {
              res = make_float4(om[4 * e4], om[4 * e4 + 1], om[4 * e4 + 2], om[4 * e4 + 3]);
            }
            w[4 * e4] = __float_as_uint(res.x);
            w[4 * e4 + 1] = __float_as_uint(res.y);
            w[4 * e4 + 2] = __float_as_uint(res.z);
            w[4 * e4 + 3] = __float_as_uint(res.w);
            if (refill && (e & 1)) ow[e >> 1] = p3_load_ow(cc, e >> 1);
          }
          tmem_st16(xr + sub * 16, w);
          }
        }
        tmem_wait_st();
        __syncwarp();
        const bool wr = pc.gate_on || pc.need_ow || (pc.row_ok && !s.mix);
        const size_t rstride = (size_t)H * kGD;
#pragma unroll
        for (int sg = 0; sg < 2; ++sg) {
          uint32_t v[32];
          tmem_ld_16x256b_x8(tmem + ((uint32_t)(q4 * 32 + sg * 16) << 16) + xcol, v);
          tmem_wait_ld();
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int rl = sg * 16 + hf * 8 + (lane >> 2);   // row (within this warp's 32) of this half block
            const bool wrow = __shfl_sync(0xffffffffu, wr, rl) != 0;
            float* op = pc.orow + (long long)(rl - lane) * (long long)rstride + 2 * (lane & 3);
            if (wrow) {
#pragma unroll
              for (int k = 0; k < 8; ++k)
                *reinterpret_cast<float2*>(op + 8 * k) =
                    make_float2(__uint_as_float(v[4 * k + 2 * hf]), __uint_as_float(v[4 * k + 2 * hf + 1]));
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&bar_xf[(m - 1) % 3]);
      }
      if (!has_cur) break;
      pc = cc;
      have_prev = true;
      ++m;
      if (++rh == R) {
        rh = 0;
        u += gridDim.x;
        if (u < nitems) it = p3_item(s, u);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================================ launch
// chunk table of packed sequences (one CTA): sequence i has ceil(len_i / kGC) chunks, the last one partial
__global__ void __launch_bounds__(1024) build_chunk_table_kernel(const int* __restrict__ cu_seqlens, int n_seq,
                                                                 int max_chunks, int* __restrict__ seq_chunk0,
                                                                 int* __restrict__ chunk_tok0,
                                                                 int* __restrict__ chunk_len, unsigned int* err) {
  __shared__ int total;
  if (threadIdx.x == 0) {
    int acc = 0;
    seq_chunk0[0] = 0;
    for (int i = 0; i < n_seq; ++i) {
      const int len = cu_seqlens[i + 1] - cu_seqlens[i];
      acc += len > 0 ? (len + kGC - 1) / kGC : 0;
      seq_chunk0[i + 1] = acc;
    }
    if (acc > max_chunks) {   // cu_seqlens inconsistent with T: no chunks at all rather than out-of-range work
      record_error(err, 0x4f);
      for (int i = 0; i <= n_seq; ++i) seq_chunk0[i] = 0;
      acc = 0;
    }
    total = acc;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < total; c += blockDim.x) {
    int lo = 0, hi = n_seq - 1;          // the sequence i with seq_chunk0[i] <= c < seq_chunk0[i + 1]
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seq_chunk0[mid] <= c) lo = mid;
      else hi = mid - 1;
    }
    const int tok0 = cu_seqlens[lo] + (c - seq_chunk0[lo]) * kGC;
    chunk_tok0[c] = tok0;
    chunk_len[c] = min(kGC, cu_seqlens[lo + 1] - tok0);
  }
}

int launch_chunk_table(const int* cu_seqlens, int n_seq, int max_chunks, int* seq_chunk0, int* chunk_tok0,
                       int* chunk_len, unsigned int* err, cudaStream_t stream) {
  build_chunk_table_kernel<<<1, 1024, 0, stream>>>(cu_seqlens, n_seq, max_chunks, seq_chunk0, chunk_tok0, chunk_len,
                                                   err);
  return launch_status();
}

size_t gdn_prefill_workspace(int B, int G, int T_steps, bool transform) {
  const size_t n_pad = (size_t)((T_steps + kGC - 1) / kGC) * kGC;
  const size_t nch = n_pad / kGC;
  auto al = [](size_t x) { return (x + 1023) & ~size_t(1023); };
  size_t n = 0;
  n += al((size_t)B * G * n_pad * kGD * 2) * 3;       // kw, w, u
  n += al((size_t)B * G * n_pad * 4);                 // gc
  if (transform) return n;                            // no P3: the chunk states are not kept
  n += al((size_t)B * G * nch * kGD * kGD * 2);       // ST
  n += al((size_t)B * G * nch * kGD * kGC * 2);       // VT
  return n;
}

// the fix-up phase's extra buffers: per-chunk transitions MC, the incoming state transposed (SinT)
size_t gdn_prefill_fix_workspace(int B, int G, int T_steps) {
  const size_t nch = (size_t)((T_steps + kGC - 1) / kGC);
  auto al = [](size_t x) { return (x + 1023) & ~size_t(1023); };
  return al((size_t)B * G * nch * kGD * kGD * 2) + al((size_t)B * G * kGD * kGD * 2);
}

void gdn_prefill_carve_fix(GdnStreams& s, void* ws) {
  auto al = [](size_t x) { return (x + 1023) & ~size_t(1023); };
  uint8_t* p = static_cast<uint8_t*>(ws);
  s.MC = reinterpret_cast<__half*>(p); p += al((size_t)s.B * s.G * s.n_chunks * kGD * kGD * 2);
  s.SinT = reinterpret_cast<__half*>(p);
}

int gdn_prefill_carve(GdnStreams& s, void* ws) {
  auto al = [](size_t x) { return (x + 1023) & ~size_t(1023); };
  uint8_t* p = static_cast<uint8_t*>(ws);
  const size_t n_pad = (size_t)s.n_pad, nch = (size_t)s.n_chunks;
  s.kw = reinterpret_cast<__half*>(p); p += al((size_t)s.B * s.G * n_pad * kGD * 2);
  s.w = reinterpret_cast<__half*>(p); p += al((size_t)s.B * s.G * n_pad * kGD * 2);
  s.u = reinterpret_cast<__half*>(p); p += al((size_t)s.B * s.G * n_pad * kGD * 2);
  s.gc = reinterpret_cast<float*>(p); p += al((size_t)s.B * s.G * n_pad * 4);
  if (s.m_out && !s.MC) {
    s.ST = s.VT = nullptr;
    return BF_OK;
  }
  s.ST = reinterpret_cast<__half*>(p); p += al((size_t)s.B * s.G * nch * kGD * kGD * 2);
  s.VT = reinterpret_cast<__half*>(p); p += al((size_t)s.B * s.G * nch * kGD * kGC * 2);
  return BF_OK;
}

int launch_gdn_prefill(GdnStreams s, cudaStream_t stream, int parts) {
  if (s.n_steps <= 0) return BF_OK;
  const int H = s.G * s.R;
  {
    int rc0 = ensure_smem_attr((const void*)gdn_p1_kernel, kP1_Smem);
    if (!rc0) rc0 = ensure_smem_attr((const void*)gdn_p2_kernel, kP2_Smem);
    if (!rc0) rc0 = ensure_smem_attr((const void*)gdn_p3_kernel, kP3_Smem);
    if (rc0) return rc0;
  }
  if (parts & kGdnP1) {
    CUtensorMap kwmap, umap, wmap1;
    const uint64_t nrows = (uint64_t)s.B * s.G * s.n_pad;
    int rc1 = make_tmap_kmajor(&kwmap, s.kw, BF_F16, nrows, kGD, kGD, kGC, 4);
    if (!rc1) rc1 = make_tmap_kmajor(&umap, s.u, BF_F16, nrows, kGD, kGD, kGC, 4);
    if (!rc1) rc1 = make_tmap_kmajor(&wmap1, s.w, BF_F16, nrows, kGD, kGD, kGC, 4);
    if (rc1) return rc1;
    stage_mark(ST_GDN_P1, 0, stream);
    gdn_p1_kernel<<<dim3(s.n_chunks, s.B * s.G), kP1_Threads, kP1_Smem, stream>>>(kwmap, umap, wmap1, s);
    if (int e_ = launch_status()) return e_;
    stage_mark(ST_GDN_P1, 1, stream);
  }
  if (parts & kGdnFix) {
    if (!s.MC || !s.SinT || !s.s0 || !s.ST || !s.VT) return BF_ERR_INVALID_ARGUMENT;
    int rcf = ensure_smem_attr((const void*)gdn_sp_fixup_kernel, kFX_Smem);
    if (rcf) return rcf;
    sp_sin_transpose_kernel<<<dim3(kGD / 32, kGD / 32, s.B * s.G), dim3(32, 8), 0, stream>>>(s.s0, s.SinT);
    if (int e_ = launch_status()) return e_;
    CUtensorMap sinmap, mcmap, wmapf;
    rcf = make_tmap_kmajor(&sinmap, s.SinT, BF_F16, (uint64_t)s.B * s.G * kGD, kGD, kGD, 128, 4);
    if (!rcf) rcf = make_tmap_kmajor(&mcmap, s.MC, BF_F16, (uint64_t)s.B * s.G * s.n_chunks * kGD, kGD, kGD, kGD, 4);
    if (!rcf) rcf = make_tmap_kmajor(&wmapf, s.w, BF_F16, (uint64_t)s.B * s.G * s.n_pad, kGD, kGD, kGC, 4);
    if (rcf) return rcf;
    stage_mark(ST_GDN_P2, 0, stream);
    gdn_sp_fixup_kernel<<<dim3(s.n_chunks, s.B * s.G, 2), kFX_Threads, kFX_Smem, stream>>>(sinmap, mcmap, wmapf, s);
    if (int e_ = launch_status()) return e_;
    stage_mark(ST_GDN_P2, 1, stream);
  }
  if (!(parts & (kGdnP2 | kGdnP3))) return BF_OK;
  CUtensorMap wmap, kmap;
  int rc = make_tmap_kmajor(&wmap, s.w, BF_F16, (uint64_t)s.B * s.G * s.n_pad, kGD, kGD, kGC, 4);
  if (!rc) rc = make_tmap_kmajor(&kmap, s.kw, BF_F16, (uint64_t)s.B * s.G * s.n_pad, kGD, kGD, kGC, 4);
  if (rc) return rc;
  if (parts & kGdnP2) {
  stage_mark(ST_GDN_P2, 0, stream);
  gdn_p2_kernel<<<dim3((s.m_out ? 2 : 1) * (kGD / kP2_NB), s.chunk_tok0 ? s.G * s.n_seq : s.B * s.G), kP2_Threads,
                  kP2_Smem, stream>>>(wmap, kmap, s);
  if (int e_ = launch_status()) return e_;
  stage_mark(ST_GDN_P2, 1, stream);
  }
  if (s.m_out || !(parts & kGdnP3)) return BF_OK;   // segment transform: no reads
  // P3 maps: q [B,T,H,D] fp16 as (d, token, atom, head); k/kw; S^T; v'^T
  CUtensorMap qmap, smap, vmap;   // (and kmap, the keys)
  {
    const uint64_t dims[4] = {64, (uint64_t)s.B * s.T, 4, (uint64_t)H};
    const uint64_t strides[3] = {(uint64_t)H * kGD * 2, 128, (uint64_t)kGD * 2};
    const uint32_t box[4] = {64, (uint32_t)kGC, 4, 1};
    rc = make_tmap(&qmap, s.qm, BF_F16, 4, dims, strides, box, true);
    if (rc) return rc;
  }
  rc = make_tmap_kmajor(&smap, s.ST, BF_F16, (uint64_t)s.B * s.G * s.n_chunks * kGD, kGD, kGD, 128, 4);
  if (rc) return rc;
  rc = make_tmap_kmajor(&vmap, s.VT, BF_F16, (uint64_t)s.B * s.G * s.n_chunks * kGD, kGC, kGC, 128, 2);
  if (rc) return rc;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return cuda_fail();
  const long long nitems = 2LL * s.B * s.G * (s.p3_c1 > 0 ? s.p3_c1 - s.p3_c0 : s.n_chunks);   // (b, chunk, KV head, value half)
  if (nitems <= 0) return BF_OK;
  (void)H;
  stage_mark(ST_GDN_P3, 0, stream);
  gdn_p3_kernel<<<(unsigned)(nitems < sms ? nitems : sms), kP3_Threads, kP3_Smem, stream>>>(qmap, kmap, smap, vmap, s);
  stage_mark(ST_GDN_P3, 1, stream);
  return launch_status();
}

}  // namespace bfb
