// Sliding-window + sink attention over a block of queries (prefill), on the 5th-gen tensor core.
//
// Semantics: HybridAttention._window_fp32 (heimdall/hibrit.py:341-361).  A query at position p sees a key
// at position kp when kp <= p and either kp is a sink (kp < S, taken from the sink buffer) or
// (p - kp < W and kp >= S).  Scores use q . k / sqrt(D).  Returns o and lse = log sum exp.
// The fused-layer epilogue also applies the LSE gate and the mix of heimdall/hibrit.py:409-411.
//
// Keys come as one "extended" sequence (ring in time order, then the new tokens; key j has position
// kpos0 + j; positions below `klo` are not valid window keys).  K is bf16 [B,G,Tk,D]; V is pre-transposed
// to fp16 [B,G,D,Tkp] so that it is a K-major B operand.
//
// CTA = (128-query tile, query head, batch), key tiles of 128:
//   S_j = Q K_j^T   (M128 N128 K256; A = Q and B = K_j in shared memory)        -> TMEM S buffer j%2
//   O  += P_j V_j   (M128 N256 K128; A = P_j in TMEM over S_j, B = V_j^T in shared memory)
//   TMEM: S/P buffers at columns 0 and 128, O at 256..511.
// Warp roles (384 threads): warp 0 TMA for Q and K; warp 2 TMA for V^T; warp 1 issues the MMAs (S_{j+1}
// before O += P_j V_j, so the tensor core works while the softmax warps work); warps 4-11 are two softmax
// warpgroups: half hh owns keys [64 hh, 64 hh + 64) of every tile and O columns [128 hh, 128 hh + 128) of
// every row; both halves scan the whole score row for the max (identical decisions), scores in the log2
// domain (FFMA + ex2), O rescaled only when the row max grows by more than 2^8 (P stays in fp16 range).
// The sink keys (<= 8) are exact in fp32: their scores are computed from Q and the sink keys in shared
// memory while the first product runs, their values join in the epilogue.  The epilogue stages the output
// tile in shared memory (128-byte swizzle, the memory read for the fused mix arrives there by TMA) and
// writes it with TMA stores.
#include "capi_internal.h"
#include "common.cuh"
#include "tmap.h"
#include "window_prefill.h"

namespace bfb {

constexpr int kWP_M = 128;       // queries per tile
constexpr int kWP_N = 128;       // keys per tile
constexpr int kWP_D = 256;
constexpr int kWP_Threads = 384;
constexpr int kWP_MaxSinks = 8;
constexpr int kWP_SinkRows = 16;                  // sink keys padded to the smallest MMA N
constexpr int kWP_SmemQ = kWP_M * kWP_D * 2;      // 64 KB
constexpr int kWP_SmemK = kWP_N * kWP_D * 2;      // 64 KB
constexpr int kWP_SmemV = kWP_D * kWP_N * 2;      // 64 KB
constexpr int kWP_SmemSK = kWP_SinkRows * kWP_D * 2;      // 8 KB: sink keys, K-major 128-byte swizzle
constexpr int kWP_SmemSV = kWP_MaxSinks * kWP_D * 4;      // 8 KB: sink values in fp32
constexpr int kWP_Tiles = kWP_SmemQ + kWP_SmemK + kWP_SmemV + kWP_SmemSK + kWP_SmemSV;
constexpr int kWP_Smem = kWP_Tiles + 256 + 4096 + 1024;   // + barriers + row exchanges (3 KB) + alignment
constexpr float kRescaleLog2 = 8.0f;              // rescale O when the max grows by more than 2^8
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kTmO = 256;                    // TMEM column of O

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3f(float x, float y, float z) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
  return r;
}

__device__ __forceinline__ uint32_t cvt_half2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// byte offset of fp32 element (row, col) in the epilogue staging tile: 8 sub-tiles of 32 columns,
// each [128 rows][128 B] with the 128-byte swizzle (the layout of a SWIZZLE_128B TMA box {32, 1, 128, 1})
__device__ __forceinline__ uint32_t stage_off(uint32_t row, uint32_t col) {
  return (col >> 5) * (128u * 128u) + row * 128u + ((((col & 31u) >> 2) ^ (row & 7u)) << 4) + (col & 3u) * 4u;
}

// byte offset of (row, col) of a 128 x 256 fp32 output tile in the memory-read epilogue's order: warp (row group
// row / 32, column block) loads float4 e of its 32 rows as 512 contiguous bytes
__device__ __forceinline__ uint32_t perm_off(uint32_t row, uint32_t col) {
  return (((((col >> 7) * 2 + ((col >> 6) & 1)) * 4 + (row >> 5)) * 16 + ((col & 63) >> 2)) * 32 + (row & 31)) * 16 +
         (col & 3) * 4;
}

// TMEM column of the fp16 P operand for key-step ks (16 keys) of an S buffer: each softmax half writes the
// probabilities of its 64 keys into the first 32 columns of its own 64 score columns.
__device__ __forceinline__ uint32_t p_col(int ks) { return (uint32_t)((ks >> 2) * 64 + (ks & 3) * 8); }

__global__ void __launch_bounds__(kWP_Threads, 1)
    window_prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap,
                          const __grid_constant__ CUtensorMap mmap, WinPreArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kWP_SmemQ;
  uint8_t* sV = sK + kWP_SmemK;
  uint8_t* sO = sK;                        // epilogue staging (128 KB) over the K and V tiles
  uint8_t* sSK = sV + kWP_SmemV;           // [4 atoms][16 rows][128 B]
  float* sSV = reinterpret_cast<float*>(sSK + kWP_SmemSK);                   // [8][256]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWP_Tiles);
  uint64_t* bar_q = bars + 0;      // Q landed
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 2;    // S_j = Q K_j^T finished reading K
  uint64_t* v_full = bars + 3;
  uint64_t* v_empty = bars + 4;    // O += P_j V_j finished (V free, O stable)
  uint64_t* s_full = bars + 5;     // [2]
  uint64_t* p_full = bars + 7;     // [2] P_j in TMEM (one arrival per softmax warp)
  uint64_t* bar_om = bars + 9;     // memory read tile landed in the staging buffer
  uint64_t* bar_st = bars + 10;    // staging tile complete (one arrival per softmax warp)
  uint64_t* bar_sk = bars + 11;    // sink keys staged (one arrival per softmax warp)
  uint64_t* bar_sink = bars + 12;  // sink scores in TMEM
  uint64_t* pair = bars + 13;      // [4] sync of the two softmax warps on a lane quarter (one arrival per warp)
  uint64_t* o_fin = bars + 17;     // the last O += P V finished (once per CTA; a parity wait on v_empty could
                                   // alias: nothing orders the next-to-last product before the last softmax)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 19);
  // row exchange: [2 tile parities][2 halves][128] running maxima, then [2 halves][128] final sums
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = blockIdx.x * kWP_M;
  const int h = blockIdx.y, b = blockIdx.z;
  const int R = a.H / a.G, g = h / R;
  const long long P0 = a.qpos0 + i0;
  const long long Plast = a.qpos0 + min(i0 + kWP_M, a.Tq) - 1;
  // key tiles covering positions [max(klo, P0 - W + 1), Plast] of the extended key sequence
  const long long kp_lo = max(a.klo, P0 - a.W + 1);
  long long jlo = kp_lo - a.kpos0, jhi = min(Plast - a.kpos0, (long long)a.Tk - 1);
  int jt0 = 0, n = 0;
  if (kp_lo <= Plast && jhi >= 0 && jlo <= jhi) {
    if (jlo < 0) jlo = 0;
    jt0 = (int)(jlo / kWP_N);
    n = (int)(jhi / kWP_N) - jt0 + 1;
  }
  const int ns = a.ns;
  const bool mixing = a.o_mem != nullptr;
  const int pc = blockIdx.x - a.perm_tile0;   // chunk of the memory reads this tile belongs to
  float* const perm_dst = (a.o_perm && pc >= 0 && pc < a.perm_nch)
                              ? a.o_perm + (((size_t)b * a.perm_nch + pc) * a.H + h) * (size_t)(kWP_M * kWP_D)
                              : nullptr;

  if (tid == 0) {
    for (int i = 0; i < 13; ++i) mbar_init(bars + i, (i == 7 || i == 8 || i == 10 || i == 11) ? 8 : 1);
    for (int i = 0; i < 4; ++i) mbar_init(pair + i, 2);
    mbar_init(o_fin, 1);
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
      mbar_expect_tx(bar_q, kWP_SmemQ);
      tma_load_3d(sQ, &qmap, bar_q, 0, (b * a.H + h) * a.Tq + i0, 0);
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        if (j >= 1 && !mbar_wait(k_empty, (j - 1) & 1, abort_flag, a.err, 0x31)) break;
        mbar_expect_tx(k_full, kWP_SmemK);
        tma_load_3d(sK, &kmap, k_full, 0, (b * a.G + g) * a.Tk + (jt0 + j) * kWP_N, 0);
        issued = j + 1;
      }
      mbar_wait(bar_q, 0, nullptr, a.err, 0x32);
      if (issued > 0) mbar_wait(k_full, (issued - 1) & 1, nullptr, a.err, 0x33);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      tma_prefetch(&vmap);
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        if (j >= 1 && !mbar_wait(v_empty, (j - 1) & 1, abort_flag, a.err, 0x34)) break;
        mbar_expect_tx(v_full, kWP_SmemV);
        tma_load_3d(sV, &vmap, v_full, 0, (b * a.G + g) * kWP_D, 2 * (jt0 + j));
        issued = j + 1;
      }
      if (issued > 0) mbar_wait(v_full, (issued - 1) & 1, nullptr, a.err, 0x35);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kWP_M, kWP_N, 1);
      constexpr uint32_t idesc_sk = idesc_f16(kWP_M, kWP_SinkRows, 1);
      constexpr uint32_t idesc_pv = idesc_f16(kWP_M, kWP_D, 0);
      const uint32_t aQ = smem_u32(sQ), bK = smem_u32(sK), bV = smem_u32(sV), bSK = smem_u32(sSK);
      bool ok = mbar_wait(bar_q, 0, abort_flag, a.err, 0x36);
      // sink scores Q . sink_k -> O columns (read by the softmax warps before the first O += P V)
      if (ok && ns > 0) {
        ok = mbar_wait(bar_sk, 0, abort_flag, a.err, 0x3c);
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kWP_D / 16; ++ks)
            umma_f16_ss(tmem + kTmO, sdesc_kstep(aQ, kWP_M, ks), sdesc_kstep(bSK, kWP_SinkRows, ks), idesc_sk,
                        ks > 0);
          umma_commit(bar_sink);
        }
      }
      auto issue_pv = [&](int jj) -> bool {
        const int s = jj & 1;
        if (!mbar_wait(&p_full[s], (jj >> 1) & 1, abort_flag, a.err, 0x37)) return false;
        if (!mbar_wait(v_full, jj & 1, abort_flag, a.err, 0x38)) return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kWP_N / 16; ++ks)
          umma_f16_ts(tmem + kTmO, tmem + s * kWP_N + p_col(ks), sdesc_kstep(bV, kWP_D, ks), idesc_pv, (jj | ks) > 0);
        umma_commit(v_empty);
        if (jj == n - 1) umma_commit(o_fin);
        return true;
      };
      for (int j = 0; j < n && ok; ++j) {
        const int s = j & 1;
        ok = mbar_wait(k_full, j & 1, abort_flag, a.err, 0x39);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kWP_D / 16; ++ks)
          umma_f16_ss(tmem + s * kWP_N, sdesc_kstep(aQ, kWP_M, ks), sdesc_kstep(bK, kWP_N, ks), idesc_qk, ks > 0);
        umma_commit(k_empty);
        umma_commit(&s_full[s]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok && n > 0) issue_pv(n - 1);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax + epilogue (warps 4..11)
    const int q4 = warp & 3;
    const int hh = (warp - 4) >> 2;
    const int r = q4 * 32 + lane;                // query row in the tile == TMEM lane
    const int st = tid - 128;                    // 0..255 over the softmax warps
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    const long long p = P0 + r;                  // position of this query
    const float c2 = rsqrtf((float)kWP_D) * kLog2e;   // score -> log2 domain
    uint32_t pair_phase = 0;
    auto pair_sync = [&](unsigned int site) -> bool {  // bounded sync of the two warps on these lanes
      __syncwarp();
      if (lane == 0) mbar_arrive(&pair[q4]);
      const bool ok = mbar_wait_warp(&pair[q4], pair_phase & 1, abort_flag, a.err, site);
      ++pair_phase;
      return ok;
    };
    bool alive = true;
    // sink keys -> K-major swizzled B operand (rows >= ns zero); sink values -> fp32
    for (int i = st; i < kWP_SinkRows * (kWP_D / 8); i += 256) {
      const int e = i / (kWP_D / 8), c = i % (kWP_D / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (e < ns)
        v = __ldg(reinterpret_cast<const uint4*>(a.sink_k + (size_t)b * a.sk_b + (size_t)g * a.sk_h +
                                                 (size_t)e * a.sk_k) + c);
      *reinterpret_cast<uint4*>(sSK + (c >> 3) * (kWP_SinkRows * 128) + e * 128 + (((c & 7) ^ (e & 7)) << 4)) = v;
    }
    for (int i = st; i < ns * (kWP_D / 8); i += 256) {
      const int e = i / (kWP_D / 8), c = i % (kWP_D / 8);
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.sink_v + (size_t)b * a.sv_b + (size_t)g * a.sv_h +
                                                           (size_t)e * a.sv_k) + c);
      float4* d = reinterpret_cast<float4*>(sSV + e * kWP_D + c * 8);
      d[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                         __uint_as_float(v.y & 0xffff0000u));
      d[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xffff0000u), __uint_as_float(v.w << 16),
                         __uint_as_float(v.w & 0xffff0000u));
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_sk);
    float se[kWP_MaxSinks];   // sink scores in the log2 domain (-inf: not visible from this row)
#pragma unroll
    for (int e = 0; e < kWP_MaxSinks; ++e) se[e] = -INFINITY;
    if (ns > 0) {
      alive = mbar_wait_warp(bar_sink, 0, abort_flag, a.err, 0x3a);
      if (alive) {
        tc_fence_after();
        uint32_t w[16];
        tmem_ld16(trow + kTmO, w);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < kWP_MaxSinks; ++e)
          se[e] = (e < ns && e <= p) ? __uint_as_float(w[e]) * c2 : -INFINITY;
      }
    }
    // all sink rows are read (and their values staged) before this CTA's first p_full arrival
    asm volatile("bar.sync 1, 256;" ::: "memory");

    float m_ref = -INFINITY, l = 0.f;            // running max (log2 domain) and this half's sum
    constexpr int NH = kWP_N / 2;                 // 64 keys per half
    for (int j = 0; j < n && alive; ++j) {
      const int s = j & 1;
      if (!mbar_wait_warp(&s_full[s], (j >> 1) & 1, abort_flag, a.err, 0x3b)) { alive = false; break; }
      tc_fence_after();
      // key kt + c is a window key for this row when c_lo <= c <= c_hi (keys past Tk are never valid)
      const long long tile0 = (long long)(jt0 + j) * kWP_N;
      const long long kt = a.kpos0 + tile0;
      const bool full = kt >= a.klo && kt + kWP_N - 1 <= P0 && (Plast - kt) < a.W && tile0 + kWP_N <= a.Tk;
      float u[NH];
      {
        uint32_t w0[32], w1[32];
        tmem_ld32(trow + s * kWP_N + hh * NH, w0);
        tmem_ld32(trow + s * kWP_N + hh * NH + 32, w1);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          u[e] = __uint_as_float(w0[e]);
          u[e + 32] = __uint_as_float(w1[e]);
        }
      }
      if (!full) {
        const long long lo = max(max(a.klo - kt, p - a.W + 1 - kt), 0LL);
        const long long hi = min(min(p - kt, (long long)kWP_N - 1), (long long)a.Tk - 1 - tile0);
        const int c_lo = (int)min(lo, (long long)kWP_N) - hh * NH, c_hi = (int)max(hi, -1LL) - hh * NH;
#pragma unroll
        for (int e = 0; e < NH; ++e) u[e] = (e >= c_lo && e <= c_hi) ? u[e] : -INFINITY;
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int e = 0; e < NH; e += 8) {
        mx0 = max3f(mx0, u[e], u[e + 1]);
        mx1 = max3f(mx1, u[e + 2], u[e + 3]);
        mx2 = max3f(mx2, u[e + 4], u[e + 5]);
        mx3 = max3f(mx3, u[e + 6], u[e + 7]);
      }
      const float mown = max3f(mx0, mx1, fmaxf(mx2, mx3));
      float* xm = xch + (j & 1) * 256;
      xm[hh * 128 + r] = mown;
      if (!pair_sync(0x40)) { alive = false; break; }
      const float mt = fmaxf(mown, xm[(1 - hh) * 128 + r]) * c2;
      float factor = 1.f;
      bool rescale = false;
      if (m_ref == -INFINITY) {
        m_ref = mt;  // O holds nothing yet (or only zeros)
      } else if (mt > m_ref + kRescaleLog2) {
        factor = ex2_approx(m_ref - mt);
        rescale = true;
        m_ref = mt;
        l *= factor;
      }
      uint32_t pk[NH / 2];
      if (m_ref == -INFINITY) {
#pragma unroll
        for (int c = 0; c < NH / 2; ++c) pk[c] = 0u;
      } else {
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
        const float nm = -m_ref;
#pragma unroll
        for (int c = 0; c < NH; c += 2) {
          const float e0 = ex2_approx(fmaf(u[c], c2, nm)), e1 = ex2_approx(fmaf(u[c + 1], c2, nm));
          ls[(c >> 1) & 3] += e0 + e1;
          pk[c / 2] = cvt_half2(e0, e1);
        }
        l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      }
      // O rescale (warp-collective): after O += P_{j-1} V_{j-1} has finished
      if (__any_sync(0xffffffffu, rescale)) {
        if (j >= 1 && !mbar_wait_warp(v_empty, (j - 1) & 1, abort_flag, a.err, 0x3e)) {
          alive = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = hh * 128; c < hh * 128 + 128; c += 32) {
          uint32_t w[32];
          tmem_ld32(trow + kTmO + c, w);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(__uint_as_float(w[e]) * factor);
          tmem_st32(trow + kTmO + c, w);
        }
      }
      // P of this half over the first half of its own score columns
      tmem_st32(trow + s * kWP_N + hh * NH, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    // ------------------------------------------------------------------ epilogue
    if (alive && n > 0) alive = mbar_wait_warp(o_fin, 0, abort_flag, a.err, 0x3d);
    tc_fence_after();
    // the memory read of the fused mix lands in the staging buffer (K/V are free once the last product ended)
    if (mixing && st == 0 && alive) {
      mbar_expect_tx(bar_om, kWP_M * kWP_D * 4);
      for (int c = 0; c < 8; ++c)
        tma_load_4d(sO + c * (kWP_M * 128), &mmap, bar_om, c * 32, h, i0, b);
    }
    xch[512 + hh * 128 + r] = l;
    if (alive) alive = pair_sync(0x43);
    l += xch[512 + (1 - hh) * 128 + r];
    if (alive && mixing) alive = mbar_wait_warp(bar_om, 0, abort_flag, a.err, 0x41);
    if (alive) {
      float mf = m_ref;
#pragma unroll
      for (int e = 0; e < kWP_MaxSinks; ++e) mf = fmaxf(mf, se[e]);
      const float fo = (m_ref == -INFINITY) ? 0.f : ex2_approx(m_ref - mf);
      float lf = l * fo;
      float we[kWP_MaxSinks];
#pragma unroll
      for (int e = 0; e < kWP_MaxSinks; ++e) {
        we[e] = (se[e] == -INFINITY) ? 0.f : ex2_approx(se[e] - mf);
        lf += we[e];
      }
      const float inv = lf > 0.f ? 1.f / lf : 0.f;
      const float lse = lf > 0.f ? (mf + log2f(lf)) * kLn2 : -INFINITY;
      const int qi = i0 + r;
      const bool row_ok = qi < a.Tq;
      const bool gate_on = mixing && p >= a.W;
      float gam = 0.f;
      if (row_ok) {
        if (a.lse && hh == 0) a.lse[((size_t)b * a.H + h) * a.Tq + qi] = lse;
        if (gate_on) {
          const float z = a.mixx[((size_t)b * a.Tq + qi) * a.H + h] + a.mix_lse[h] * (lse - logf((float)a.W));
          gam = 1.f / (1.f + __expf(-z));
        }
      }
      const float rho = mixing ? a.mem_scale[h] : 0.f;
#pragma unroll 1
      for (int c = hh * 128; c < hh * 128 + 128; c += 32) {
        uint32_t w[32];
        if (n > 0) {
          tmem_ld32(trow + kTmO + c, w);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = 0u;
        }
        float ov[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) ov[e] = __uint_as_float(w[e]) * fo;
#pragma unroll
        for (int e2 = 0; e2 < kWP_MaxSinks; ++e2) {
          if (e2 < ns && we[e2] != 0.f) {
            const float4* vw = reinterpret_cast<const float4*>(sSV + e2 * kWP_D + c);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float4 vv = vw[e];
              ov[4 * e] = fmaf(we[e2], vv.x, ov[4 * e]);
              ov[4 * e + 1] = fmaf(we[e2], vv.y, ov[4 * e + 1]);
              ov[4 * e + 2] = fmaf(we[e2], vv.z, ov[4 * e + 2]);
              ov[4 * e + 3] = fmaf(we[e2], vv.w, ov[4 * e + 3]);
            }
          }
        }
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          float4* sp4 = reinterpret_cast<float4*>(sO + (perm_dst ? perm_off(r, c + e) : stage_off(r, c + e)));
          float4 res = make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv, ov[e + 3] * inv);
          if (gate_on) {
            const float4 mv = *sp4;
            res.x += gam * (rho * mv.x - res.x);
            res.y += gam * (rho * mv.y - res.y);
            res.z += gam * (rho * mv.z - res.z);
            res.w += gam * (rho * mv.w - res.w);
          }
          *sp4 = res;
        }
      }
    }
    // all rows staged -> TMA stores of the tile (rows beyond Tq fall outside the map and are dropped)
    fence_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_st);
    if (st == 0) {
      if (alive && mbar_wait(bar_st, 0, abort_flag, a.err, 0x42)) {
        if (perm_dst) {
          for (int c = 0; c < 8; ++c) bulk_store_1d(perm_dst + c * (kWP_M * 32), sO + c * (kWP_M * 128), kWP_M * 128);
        } else {
          for (int c = 0; c < 8; ++c) tma_store_4d(&omap, sO + c * (kWP_M * 128), c * 32, h, i0, b);
        }
        tma_store_commit();
        tma_store_wait_read();
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

// V (time-major [B,T,G,D] bf16, optionally preceded by a ring [B,G,W,D] read in time order) ->
// V^T fp16 [B,G,D,Tkp], keys beyond Tk zero.  One CTA = 64 keys x 256 columns of one (b, g).
__global__ void __launch_bounds__(256) vt_prep_kernel(const __nv_bfloat16* __restrict__ v, long long vb, long long vg,
                                                      long long vj, const __nv_bfloat16* __restrict__ ring_v, int nring,
                                                      long long ring_pos0, int W, int G, int Tk, int Tkp,
                                                      __half* __restrict__ vt) {
  __shared__ __half tile[64][256 + 8];
  const int jb = blockIdx.x * 64, bg = blockIdx.y, b = bg / G, g = bg % G;
  const int t = threadIdx.x;
  // load 64 key rows (8 threads per row, 32 columns each)
  for (int rr = t >> 3; rr < 64; rr += 32) {
    const int j = jb + rr;
    const int c0 = (t & 7) * 32;
    const __nv_bfloat16* src = nullptr;
    if (j < nring) {
      const long long kp = ring_pos0 + j;
      const int slot = (int)(((kp % W) + W) % W);
      src = ring_v + (((size_t)b * G + g) * W + slot) * 256 + c0;
    } else if (j < Tk) {
      src = v + (size_t)b * vb + (size_t)g * vg + (size_t)(j - nring) * vj + c0;
    }
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      uint4 u = src ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        tile[rr][c0 + c + 2 * e] = __float2half_rn(__uint_as_float(w[e] << 16));
        tile[rr][c0 + c + 2 * e + 1] = __float2half_rn(__uint_as_float(w[e] & 0xffff0000u));
      }
    }
  }
  __syncthreads();
  // write 256 rows (columns of V) x 64 keys: each thread one column, 64 keys = 128 bytes
  const int d = t;
  __half* dst = vt + (((size_t)b * G + g) * 256 + d) * Tkp + jb;
  uint32_t w[32];
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    __half2 h2 = __halves2half2(tile[2 * e][d], tile[2 * e + 1][d]);
    w[e] = *reinterpret_cast<uint32_t*>(&h2);
  }
#pragma unroll
  for (int e = 0; e < 32; e += 4) *reinterpret_cast<uint4*>(dst + 2 * e) = make_uint4(w[e], w[e + 1], w[e + 2], w[e + 3]);
}

// K of the extended sequence: ring (time order) then kr [B,G,T,D] -> kext [B,G,W+T,D] (only with a ring)
__global__ void kext_prep_kernel(const __nv_bfloat16* __restrict__ kr, const __nv_bfloat16* __restrict__ ring_k,
                                 int nring, long long ring_pos0, int W, int T, int G, __nv_bfloat16* __restrict__ kext) {
  const int j = blockIdx.x, bg = blockIdx.y, b = bg / G, g = bg % G;
  const int Tk = nring + T;
  const __nv_bfloat16* src;
  if (j < nring) {
    const long long kp = ring_pos0 + j;
    const int slot = (int)(((kp % W) + W) % W);
    src = ring_k + (((size_t)b * G + g) * W + slot) * 256;
  } else {
    src = kr + (((size_t)b * G + g) * T + (j - nring)) * 256;
  }
  const int c = threadIdx.x * 8;
  *reinterpret_cast<uint4*>(kext + (((size_t)b * G + g) * Tk + j) * 256 + c) = *reinterpret_cast<const uint4*>(src + c);
}

int window_prefill_smem() { return kWP_Smem; }

int launch_vt_prep(const __nv_bfloat16* v, long long vb, long long vg, long long vj, const __nv_bfloat16* ring_v,
                   int nring, long long ring_pos0, int W, int B, int G, int Tk, int Tkp, __half* vt,
                   cudaStream_t stream) {
  vt_prep_kernel<<<dim3(Tkp / 64, B * G), 256, 0, stream>>>(v, vb, vg, vj, ring_v, nring, ring_pos0, W, G, Tk, Tkp, vt);
  return launch_status();
}

int launch_kext_prep(const __nv_bfloat16* kr, const __nv_bfloat16* ring_k, int nring, long long ring_pos0, int W, int B,
                     int T, int G, __nv_bfloat16* kext, cudaStream_t stream) {
  kext_prep_kernel<<<dim3(nring + T, B * G), 32, 0, stream>>>(kr, ring_k, nring, ring_pos0, W, T, G, kext);
  return launch_status();
}

int launch_window_prefill(const void* qr, const void* kext, const __half* vt, WinPreArgs a, cudaStream_t stream) {
  CUtensorMap qmap, kmap, vmap, omap, mmap;
  int rc = make_tmap_kmajor(&qmap, qr, BF_BF16, (uint64_t)a.B * a.H * a.Tq, kWP_D, kWP_D, kWP_M, 4);
  if (rc) return rc;
  rc = make_tmap_kmajor(&kmap, kext, BF_BF16, (uint64_t)a.B * a.G * a.Tk, kWP_D, kWP_D, kWP_N, 4);
  if (rc) return rc;
  rc = make_tmap_kmajor(&vmap, vt, BF_F16, (uint64_t)a.B * a.G * kWP_D, a.Tkp, a.Tkp, kWP_D, 2);
  if (rc) return rc;
  // o / o_mem [B,Tq,H,D] fp32 as (d, head, query, batch), boxes of 32 x 1 x 128 x 1 with the 128-byte swizzle
  {
    const uint64_t dims[4] = {(uint64_t)kWP_D, (uint64_t)a.H, (uint64_t)a.Tq, (uint64_t)a.B};
    const uint64_t strides[3] = {(uint64_t)kWP_D * 4, (uint64_t)a.H * kWP_D * 4, (uint64_t)a.Tq * a.H * kWP_D * 4};
    const uint32_t box[4] = {32, 1, (uint32_t)kWP_M, 1};
    rc = make_tmap(&omap, a.o, BF_F32, 4, dims, strides, box, true);
    if (rc) return rc;
    rc = make_tmap(&mmap, a.o_mem ? (const void*)a.o_mem : (const void*)a.o, BF_F32, 4, dims, strides, box, true);
    if (rc) return rc;
  }
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(window_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWP_Smem) !=
        cudaSuccess)
      return cuda_fail();
    attr = true;
  }
  dim3 grid((a.Tq + kWP_M - 1) / kWP_M, a.H, a.B);
  window_prefill_kernel<<<grid, kWP_Threads, kWP_Smem, stream>>>(qmap, kmap, vmap, omap, mmap, a);
  return launch_status();
}

}  // namespace bfb
