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
// CTA = (128-query tile, query head, batch), key tiles of 64.  Both products read their A operand from
// tensor memory, so shared memory only streams K and V^T:
//   TMEM: S/P buffers at columns 0 and 64 (fp32 scores, then fp16 probabilities written over them),
//         Q (bf16, 2 per column) at 128..255, O (fp32) at 256..511.
//   S_j = Q K_j^T   (M128 N64 K256, A = Q in TMEM, B = K_j in shared memory)
//   O  += P_j V_j   (M128 N256 K64, A = P_j in TMEM, B = V_j^T in shared memory)
// Warp roles (384 threads): warp 0 TMA for Q and K (two stages); warp 2 TMA for V^T (two stages); warp 1
// issues the MMAs (S_{j+1} before O += P_j V_j); warps 4-11 are two softmax warpgroups: half hh owns score
// columns [32 hh, 32 hh + 32) and O columns [128 hh, 128 hh + 128) of every row, both halves read the whole
// score row for the max (identical decisions, no exchange), scores in the log2 domain (FFMA + ex2), O is
// rescaled only when the row max grows by more than 2^8 (so P stays within fp16 range).
// The sink keys (<= 8) are folded in exactly in fp32: their scores are computed before the main loop from
// Q and the sink keys staged in shared memory, their values join in the epilogue.
#include "capi_internal.h"
#include "common.cuh"
#include "tmap.h"
#include "window_prefill.h"

namespace bfb {

constexpr int kWP_M = 128;       // queries per tile
constexpr int kWP_N = 64;        // keys per tile
constexpr int kWP_D = 256;
constexpr int kWP_Threads = 384;
constexpr int kWP_MaxSinks = 8;
constexpr int kWP_SmemQ = kWP_M * kWP_D * 2;      // 64 KB (TMA landing buffer; Q is then copied to TMEM)
constexpr int kWP_SmemK = kWP_N * kWP_D * 2;      // 32 KB per stage
constexpr int kWP_SmemV = kWP_D * kWP_N * 2;      // 32 KB per stage
constexpr int kWP_SmemSink = kWP_MaxSinks * kWP_D * 2;   // 4 KB each for sink K and V
constexpr int kWP_SmemXs = 2 * kWP_MaxSinks * kWP_M * 4;  // 8 KB: partial sink scores of the two halves
constexpr int kWP_Tiles = kWP_SmemQ + 2 * (kWP_SmemK + kWP_SmemV) + 2 * kWP_SmemSink + kWP_SmemXs;
constexpr int kWP_Smem = kWP_Tiles + 256 + 1024 + 1024;   // + barriers + row exchange + alignment
constexpr float kRescaleLog2 = 8.0f;              // rescale O when the max grows by more than 2^8
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kTmQ = 128, kTmO = 256;        // TMEM column bases

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t cvt_half2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__global__ void __launch_bounds__(kWP_Threads, 1)
    window_prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap vmap, WinPreArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kWP_SmemQ;            // [2]
  uint8_t* sV = sK + 2 * kWP_SmemK;        // [2]
  __nv_bfloat16* sSK = reinterpret_cast<__nv_bfloat16*>(sV + 2 * kWP_SmemV);   // [8][256]
  __nv_bfloat16* sSV = sSK + kWP_MaxSinks * kWP_D;                              // [8][256]
  float* xs = reinterpret_cast<float*>(sSV + kWP_MaxSinks * kWP_D);              // [2][8][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWP_Tiles);
  uint64_t* bar_q = bars + 0;      // Q landed in shared memory
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* k_empty = bars + 3;    // [2] S_j = Q K_j^T finished with the K stage
  uint64_t* v_full = bars + 5;     // [2]
  uint64_t* v_empty = bars + 7;    // [2] O += P_j V_j finished (V stage free, O stable)
  uint64_t* s_full = bars + 9;     // [2]
  uint64_t* p_full = bars + 11;    // [2] P_j in TMEM (one arrival per softmax warp)
  uint64_t* q_tmem = bars + 13;    // Q copied into TMEM (one arrival per softmax warp)
  uint64_t* pair = bars + 14;      // [4] sync of the two softmax warps on a lane quarter (one arrival per warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 19);
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);   // [2][128] row exchange

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

  if (tid == 0) {
    for (int i = 0; i < 14; ++i) mbar_init(bars + i, (i >= 11) ? 8 : 1);
    for (int i = 0; i < 4; ++i) mbar_init(pair + i, 2);
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
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[s], ((j >> 1) - 1) & 1, abort_flag, a.err, 0x31)) break;
        mbar_expect_tx(&k_full[s], kWP_SmemK);
        tma_load_3d(sK + s * kWP_SmemK, &kmap, &k_full[s], 0, (b * a.G + g) * a.Tk + (jt0 + j) * kWP_N, 0);
        issued = j + 1;
      }
      // drain our copies before the CTA can exit
      mbar_wait(bar_q, 0, nullptr, a.err, 0x32);
      for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, a.err, 0x33);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      tma_prefetch(&vmap);
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&v_empty[s], ((j >> 1) - 1) & 1, abort_flag, a.err, 0x34)) break;
        mbar_expect_tx(&v_full[s], kWP_SmemV);
        tma_load_3d(sV + s * kWP_SmemV, &vmap, &v_full[s], 0, (b * a.G + g) * kWP_D, jt0 + j);
        issued = j + 1;
      }
      for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr, a.err, 0x35);
    }
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {
      constexpr uint32_t idesc_qk = idesc_f16(kWP_M, kWP_N, 1);
      constexpr uint32_t idesc_pv = idesc_f16(kWP_M, kWP_D, 0);
      const uint32_t bK0 = smem_u32(sK), bV0 = smem_u32(sV);
      bool ok = mbar_wait(q_tmem, 0, abort_flag, a.err, 0x36);
      auto issue_pv = [&](int jj) -> bool {
        const int s = jj & 1;
        if (!mbar_wait(&p_full[s], (jj >> 1) & 1, abort_flag, a.err, 0x37)) return false;
        if (!mbar_wait(&v_full[s], (jj >> 1) & 1, abort_flag, a.err, 0x38)) return false;
        tc_fence_after();
        const uint32_t bV = bV0 + s * kWP_SmemV;
#pragma unroll
        for (int ks = 0; ks < kWP_N / 16; ++ks)
          umma_f16_ts(tmem + kTmO, tmem + s * kWP_N + ks * 8, sdesc_sw128(bV + ks * 32), idesc_pv, (jj | ks) > 0);
        umma_commit(&v_empty[s]);
        return true;
      };
      for (int j = 0; j < n && ok; ++j) {
        const int s = j & 1;
        ok = mbar_wait(&k_full[s], (j >> 1) & 1, abort_flag, a.err, 0x39);
        if (!ok) break;
        tc_fence_after();
        const uint32_t bK = bK0 + s * kWP_SmemK;
#pragma unroll
        for (int ks = 0; ks < kWP_D / 16; ++ks)
          umma_f16_ts(tmem + s * kWP_N, tmem + kTmQ + ks * 8, sdesc_kstep(bK, kWP_N, ks), idesc_qk, ks > 0);
        umma_commit(&k_empty[s]);
        umma_commit(&s_full[s]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(n - 1);
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
    // sink keys and values -> shared memory (ns <= 8 rows of 256)
    for (int i = st; i < ns * (kWP_D / 8); i += 256) {
      const int e = i / (kWP_D / 8), c = i % (kWP_D / 8);
      reinterpret_cast<uint4*>(sSK)[i] =
          __ldg(reinterpret_cast<const uint4*>(a.sink_k + (size_t)b * a.sk_b + (size_t)g * a.sk_h + (size_t)e * a.sk_k) + c);
      reinterpret_cast<uint4*>(sSV)[i] =
          __ldg(reinterpret_cast<const uint4*>(a.sink_v + (size_t)b * a.sv_b + (size_t)g * a.sv_h + (size_t)e * a.sv_k) + c);
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");  // all softmax threads reach this point unconditionally
    // Q -> TMEM (this half's 128 dims = 64 columns), and partial sink scores from the same registers
    alive = mbar_wait_warp(bar_q, 0, abort_flag, a.err, 0x3a);
    float sp[kWP_MaxSinks];
#pragma unroll
    for (int e = 0; e < kWP_MaxSinks; ++e) sp[e] = 0.f;
    if (alive) {
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const int atom = 2 * hh + part;          // 64 dims per atom
        uint32_t w[32];
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint4 v = *reinterpret_cast<const uint4*>(sQ + atom * (kWP_M * 128) + sw128_offset(r, ch * 8));
          w[4 * ch] = v.x; w[4 * ch + 1] = v.y; w[4 * ch + 2] = v.z; w[4 * ch + 3] = v.w;
        }
        tmem_st32(trow + kTmQ + atom * 32, w);
#pragma unroll
        for (int e = 0; e < kWP_MaxSinks; ++e) {
          if (e < ns) {
            const uint32_t* kw = reinterpret_cast<const uint32_t*>(sSK + e * kWP_D + atom * 64);
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const uint32_t kk = kw[c];
              acc += __uint_as_float(w[c] << 16) * __uint_as_float(kk << 16);
              acc += __uint_as_float(w[c] & 0xffff0000u) * __uint_as_float(kk & 0xffff0000u);
            }
            sp[e] += acc;
          }
        }
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_tmem);
#pragma unroll
    for (int e = 0; e < kWP_MaxSinks; ++e) xs[(hh * kWP_MaxSinks + e) * kWP_M + r] = sp[e];
    if (alive) alive = pair_sync(0x3f);
    float se[kWP_MaxSinks];   // sink scores in the log2 domain (-inf: not visible from this row)
#pragma unroll
    for (int e = 0; e < kWP_MaxSinks; ++e)
      se[e] = (e < ns && e <= p) ? (xs[e * kWP_M + r] + xs[(kWP_MaxSinks + e) * kWP_M + r]) * c2 : -INFINITY;

    float m_ref = -INFINITY, l = 0.f;            // running max (log2 domain) and this half's sum
    constexpr int NH = kWP_N / 2;
    for (int j = 0; j < n && alive; ++j) {
      const int s = j & 1;
      if (!mbar_wait_warp(&s_full[s], (j >> 1) & 1, abort_flag, a.err, 0x3b)) { alive = false; break; }
      tc_fence_after();
      float u[NH], uo[NH];
      {
        uint32_t w0[32], w1[32];
        tmem_ld32(trow + s * kWP_N + hh * NH, w0);
        tmem_ld32(trow + s * kWP_N + (1 - hh) * NH, w1);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < NH; ++e) {
          u[e] = __uint_as_float(w0[e]);
          uo[e] = __uint_as_float(w1[e]);
        }
      }
      // mask: key position kt + c is a window key for this row when c_lo <= c <= c_hi
      const long long kt = a.kpos0 + (long long)(jt0 + j) * kWP_N;
      const bool full = kt >= a.klo && kt + kWP_N - 1 <= P0 && (Plast - kt) < a.W;
      if (!full) {
        const long long lo = max(max(a.klo - kt, p - a.W + 1 - kt), 0LL);
        const long long hi = min(p - kt, (long long)kWP_N - 1);
        const int c_lo = (int)min(lo, (long long)kWP_N), c_hi = (int)max(hi, -1LL);
        const int my0 = hh * NH, ot0 = (1 - hh) * NH;
#pragma unroll
        for (int c = 0; c < NH; ++c) {
          u[c] = (c + my0 >= c_lo && c + my0 <= c_hi) ? u[c] : -INFINITY;
          uo[c] = (c + ot0 >= c_lo && c + ot0 <= c_hi) ? uo[c] : -INFINITY;
        }
      }
      float mx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx[e] = fmaxf(u[e], uo[e]);
#pragma unroll
      for (int c = 8; c < NH; c += 8)
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = fmaxf(mx[e], fmaxf(u[c + e], uo[c + e]));
      const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * c2;
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
        if (j >= 1 && !mbar_wait_warp(&v_empty[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, a.err, 0x3e)) {
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
      // both halves must have read S_j before P_j is written over it
      tc_fence_before();
      if (!pair_sync(0x40)) { alive = false; break; }
      tc_fence_after();
      tmem_st16(trow + s * kWP_N + hh * (NH / 2), reinterpret_cast<const uint32_t(&)[16]>(pk));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[s]);
    }
    // ------------------------------------------------------------------ epilogue
    if (alive && n > 0) alive = mbar_wait_warp(&v_empty[(n - 1) & 1], ((n - 1) >> 1) & 1, abort_flag, a.err, 0x3d);
    tc_fence_after();
    xch[hh * 128 + r] = l;
    if (alive) alive = pair_sync(0x43);
    l += xch[(1 - hh) * 128 + r];
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
      const bool mixing = a.o_mem != nullptr && p >= a.W;
      float gam = 0.f;
      const size_t orow = (((size_t)b * a.Tq + qi) * a.H + h) * kWP_D;
      if (row_ok) {
        if (a.lse && hh == 0) a.lse[((size_t)b * a.H + h) * a.Tq + qi] = lse;
        if (mixing) {
          const float z = a.mixx[((size_t)b * a.Tq + qi) * a.H + h] + a.mix_lse[h] * (lse - logf((float)a.W));
          gam = 1.f / (1.f + __expf(-z));
        }
      }
      const float rho = a.o_mem ? a.mem_scale[h] : 0.f;
#pragma unroll 1
      for (int c = hh * 128; c < hh * 128 + 128; c += 32) {
        float mv[32];
        if (row_ok && mixing) {   // issue the memory-read loads before the TMEM load
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 t4 = *reinterpret_cast<const float4*>(a.o_mem + orow + c + e);
            mv[e] = t4.x; mv[e + 1] = t4.y; mv[e + 2] = t4.z; mv[e + 3] = t4.w;
          }
        }
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
            const uint32_t* vw = reinterpret_cast<const uint32_t*>(sSV + e2 * kWP_D + c);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const uint32_t vv = vw[e];
              ov[2 * e] += we[e2] * __uint_as_float(vv << 16);
              ov[2 * e + 1] += we[e2] * __uint_as_float(vv & 0xffff0000u);
            }
          }
        }
        if (row_ok) {
          float* op = a.o + orow + c;
          if (mixing) {
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              const float w0 = ov[e] * inv, w1 = ov[e + 1] * inv, w2 = ov[e + 2] * inv, w3 = ov[e + 3] * inv;
              *reinterpret_cast<float4*>(op + e) =
                  make_float4(w0 + gam * (rho * mv[e] - w0), w1 + gam * (rho * mv[e + 1] - w1),
                              w2 + gam * (rho * mv[e + 2] - w2), w3 + gam * (rho * mv[e + 3] - w3));
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; e += 4)
              *reinterpret_cast<float4*>(op + e) =
                  make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv, ov[e + 3] * inv);
          }
        }
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
  return cudaGetLastError() == cudaSuccess ? BF_OK : BF_ERR_CUDA;
}

int launch_kext_prep(const __nv_bfloat16* kr, const __nv_bfloat16* ring_k, int nring, long long ring_pos0, int W, int B,
                     int T, int G, __nv_bfloat16* kext, cudaStream_t stream) {
  kext_prep_kernel<<<dim3(nring + T, B * G), 32, 0, stream>>>(kr, ring_k, nring, ring_pos0, W, T, G, kext);
  return cudaGetLastError() == cudaSuccess ? BF_OK : BF_ERR_CUDA;
}

int launch_window_prefill(const void* qr, const void* kext, const __half* vt, WinPreArgs a, cudaStream_t stream) {
  CUtensorMap qmap, kmap, vmap;
  int rc = make_tmap_kmajor(&qmap, qr, BF_BF16, (uint64_t)a.B * a.H * a.Tq, kWP_D, kWP_D, kWP_M, 4);
  if (rc) return rc;
  rc = make_tmap_kmajor(&kmap, kext, BF_BF16, (uint64_t)a.B * a.G * a.Tk, kWP_D, kWP_D, kWP_N, 4);
  if (rc) return rc;
  rc = make_tmap_kmajor(&vmap, vt, BF_F16, (uint64_t)a.B * a.G * kWP_D, a.Tkp, a.Tkp, kWP_D, 1);
  if (rc) return rc;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(window_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWP_Smem) !=
        cudaSuccess)
      return BF_ERR_CUDA;
    attr = true;
  }
  dim3 grid((a.Tq + kWP_M - 1) / kWP_M, a.H, a.B);
  window_prefill_kernel<<<grid, kWP_Threads, kWP_Smem, stream>>>(qmap, kmap, vmap, a);
  return cudaGetLastError() == cudaSuccess ? BF_OK : BF_ERR_CUDA;
}

}  // namespace bfb
