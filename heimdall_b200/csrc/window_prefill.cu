// Sliding-window + sink attention over a block of queries (prefill), on the 5th-gen tensor core.
//
// Semantics: HybridAttention._window_fp32 (heimdall/hibrit.py:341-361).  A query at position p sees a key
// at position kp when kp <= p and either kp is a sink (kp < S, taken from the sink buffer) or
// (p - kp < W and kp >= S).  Scores use q . k / sqrt(D).  Returns o and lse = log sum exp.
//
// Keys come as one "extended" sequence (ring in time order, then the new tokens; key j has position
// kpos0 + j; positions below `klo` are not valid window keys).  K is bf16 [B,G,Tk,D]; V is pre-transposed
// to fp16 [B,G,D,Tkp] so that it is a K-major B operand.
//
// Work items (b, query tile of 128, query head), walked by persistent CTAs (one per SM) or one item per CTA;
// the R heads of a KV group on one query tile are consecutive items, so concurrently running CTAs share their
// keys and values in L2.
// Per item, key tiles of 128:
//   S_j = Q K_j^T   (M128 N128 K256; A = Q and B = K_j in shared memory)        -> TMEM S buffer (tile parity)
//   O  += P_j V_j   (M128 N256 K128; A = P_j in TMEM over S_j, B = V_j^T in shared memory)
//   TMEM: S/P buffers at columns 0 and 128, O at 256..511.
// Warp roles (384 threads): warp 0 TMA for Q and K; warp 2 TMA for V^T; warp 1 issues the MMAs (S_{j+1}
// before O += P_j V_j, so the tensor core works while the softmax warps work); warps 4-11 are two softmax
// warpgroups: half hh owns keys [64 hh, 64 hh + 64) of every tile and O columns [128 hh, 128 hh + 128) of
// every row; both halves scan the whole score row for the max (identical decisions), scores in the log2
// domain (FFMA + ex2), O rescaled only when the row max grows by more than 2^8 (P stays in fp16 range).
// The sink keys (<= 8) start the online softmax: their scores are one M128 N16 MMA into the item's second
// score buffer, issued as soon as the queries land; they give each row its initial max and weights, and one
// softmax half stages P_sink (fp16) so that O = P_sink V_sink is a single M128 N256 K16 MMA (sink values in
// an 8 KB non-swizzled K-major tile) ahead of the first window tile.  In the persistent launch the next item's
// queries and first key tile load under this item's last products; its sink products and first softmax
// still wait for this item's epilogue (items do not otherwise overlap).  The epilogue scales O by 1/l and
// stores: rows that the memory reads mix go to a workspace in the reads' load order as fp16, others leave
// through a 16-lane TMEM read as 32-byte row segments.
#include "capi_internal.h"
#include "common.cuh"
#include "tmap.h"
#include "window_prefill.h"

namespace bfb {

constexpr int kWP_M = 128;       // queries per tile
constexpr int kWP_N = 128;       // keys per tile
constexpr int kWP_D = 256;
constexpr int kWP_Threads = 512;
// register split (setmaxnreg) of the 128 per thread at launch: warpgroup 0 (loaders, MMA issue) 96, the two
// softmax warpgroups 168, the epilogue warpgroup 80 (128 x 96 + 256 x 168 + 128 x 80 = 512 x 128)
constexpr uint32_t kWP_RegsCtl = 96, kWP_RegsSoftmax = 168, kWP_RegsEpi = 80;
static_assert(128 * kWP_RegsCtl + 256 * kWP_RegsSoftmax + 128 * kWP_RegsEpi == kWP_Threads * 128, "register split");
constexpr int kWP_MaxSinks = 8;
constexpr int kWP_SinkRows = 16;                  // sink keys padded to the smallest MMA N
constexpr int kWP_SmemQ = kWP_M * kWP_D * 2;      // 64 KB
constexpr int kWP_SmemK = kWP_N * kWP_D * 2;      // 64 KB
constexpr int kWP_SmemV = kWP_D * kWP_N * 2;      // 64 KB
constexpr int kWP_SmemSK = kWP_SinkRows * kWP_D * 2;      // 8 KB: sink keys, K-major 128-byte swizzle
constexpr int kWP_SmemSV = kWP_D * kWP_SinkRows * 2;     // 8 KB: sink values^T fp16 [256][16], no swizzle
constexpr int kWP_Tiles = kWP_SmemQ + kWP_SmemK + kWP_SmemV + kWP_SmemSK + kWP_SmemSV;
constexpr int kWP_Smem = kWP_Tiles + 256 + 5120 + 1024;   // + barriers + row exchanges (5 KB) + alignment
constexpr float kRescaleLog2 = 8.0f;              // rescale O when the max grows by more than 2^8
constexpr uint32_t kTmO = 256;                    // TMEM column of O

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

// TMEM column of the fp16 P operand for key-step ks (16 keys) of an S buffer: each softmax half writes the
// probabilities of its 64 keys into the first 32 columns of its own 64 score columns.
__device__ __forceinline__ uint32_t p_col(int ks) { return (uint32_t)((ks >> 2) * 64 + (ks & 3) * 8); }

// The sink values^T as the B operand of one K = 16 product: K-major without swizzle, core matrices of 8 rows x
// 16 bytes; element (d, e) at (d / 8) * 256 + (e / 8) * 128 + (d % 8) * 16 + (e % 8) * 2 (8-row groups 256 B
// apart, the two 8-key halves 128 B apart)
__device__ __forceinline__ uint32_t sv_off(uint32_t d, uint32_t e) {
  return (d >> 3) * 256u + (e >> 3) * 128u + (d & 7u) * 16u + (e & 7u) * 2u;
}
__device__ __forceinline__ uint64_t sdesc_sinkv(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)(128 >> 4) << 16;               // leading byte offset: between the two 8-key core matrices
  d |= (uint64_t)(256 >> 4) << 32;               // stride byte offset: between 8-row groups
  d |= (uint64_t)1 << 46;                        // descriptor version (sm_100); swizzle mode 0 (none)
  return d;
}

// one work item: (b, query tile, query head); a CTA runs the R items of one (b, query tile, KV group) group
struct WItem {
  int b, h, g, i0, qt;
  long long P0, Plast;
  int jt0, n;   // key tiles jt0 .. jt0 + n - 1 of the extended sequence
};
__device__ __forceinline__ WItem win_item(const WinPreArgs& a, long long u, int ntq) {
  // u = ((b * ntq + qt) * G + g) * R + rr
  const int R = a.H / a.G;
  WItem it;
  const int rr = (int)(u % R);
  long long t = u / R;
  it.g = (int)(t % a.G);
  t /= a.G;
  it.qt = a.qt0 + (int)(t % ntq);
  it.b = (int)(t / ntq);
  it.h = it.g * R + rr;
  it.i0 = it.qt * kWP_M;
  it.P0 = a.qpos0 + it.i0;
  it.Plast = a.qpos0 + min(it.i0 + kWP_M, a.Tq) - 1;
  // key tiles covering positions [max(klo, P0 - W + 1), Plast] of the extended key sequence
  const long long kp_lo = max(a.klo, it.P0 - a.W + 1);
  long long jlo = kp_lo - a.kpos0;
  const long long jhi = min(it.Plast - a.kpos0, (long long)a.Tk - 1);
  it.jt0 = 0;
  it.n = 0;
  if (kp_lo <= it.Plast && jhi >= 0 && jlo <= jhi) {
    if (jlo < 0) jlo = 0;
    it.jt0 = (int)(jlo / kWP_N);
    it.n = (int)(jhi / kWP_N) - it.jt0 + 1;
  }
  return it;
}

template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

__global__ void __launch_bounds__(kWP_Threads, 1)
    window_prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap vmap, WinPreArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kWP_SmemQ;
  uint8_t* sV = sK + kWP_SmemK;
  uint8_t* sSK = sV + kWP_SmemV;           // [4 atoms][16 rows][128 B]
  uint8_t* sSV = sSK + kWP_SmemSK;         // sink values^T, fp16 (sv_off layout)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWP_Tiles);
  uint64_t* bar_q = bars + 0;      // Q landed (per item)
  uint64_t* q_free = bars + 1;     // the item's last product reading Q finished (per item)
  uint64_t* k_full = bars + 2;     // (per tile)
  uint64_t* k_empty = bars + 3;    // S_t = Q K_t^T finished reading K
  uint64_t* v_full = bars + 4;
  uint64_t* v_empty = bars + 5;    // O += P_t V_t finished (V free, O stable)
  uint64_t* s_full = bars + 6;     // [2]
  uint64_t* p_full = bars + 8;     // [2] P_t in TMEM (one arrival per softmax warp)
  uint64_t* bar_sk = bars + 10;    // sink keys and values staged (one arrival per softmax warp, once)
  uint64_t* bar_sink = bars + 11;  // the item's sink scores in TMEM (per item, with sinks)
  uint64_t* o_fin = bars + 12;     // the item's O is complete (per item)
  uint64_t* o_free = bars + 13;    // O drained by the epilogue (one arrival per epilogue warp, per item)
  uint64_t* psink = bars + 14;     // P_sink staged (one arrival per half-0 softmax warp, per item, with sinks)
  uint64_t* sread = bars + 15;     // the sink scores read (one arrival per softmax warp, per item, with sinks)
  uint64_t* pair = bars + 16;      // [4] sync of the two softmax warps on a lane quarter (one arrival per warp)
  // per stats slot (item parity): the slot's row sums and max written (one arrival per softmax warp) / read by
  // the epilogue (one arrival per epilogue warp); one barrier pair per slot, so neither side runs two uses ahead
  uint64_t* stats = bars + 20;     // [2]
  uint64_t* sfree = bars + 22;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);
  // [2 tile parities][2 halves][128] running maxima; [2 item slots][2 halves][128] row sums; [2 slots][128] max
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);
  float* xl = xch + 512;
  float* xmx = xl + 512;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntq = a.nqt > 0 ? a.nqt : (a.Tq + kWP_M - 1) / kWP_M;   // query tiles of this launch
  const int R = a.H / a.G;
  const long long u0 = (long long)blockIdx.x * R;                   // this CTA's items u0 .. u0 + R - 1
  const int ns = a.ns;

  if (tid == 0) {
    mbar_init(bar_q, 1);
    mbar_init(q_free, 1);
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&sfree[i], 4);
      mbar_init(&stats[i], 8);
    }
    mbar_init(bar_sk, 8);
    mbar_init(bar_sink, 1);
    mbar_init(o_fin, 1);
    mbar_init(o_free, 4);
    mbar_init(psink, 4);
    mbar_init(sread, 8);
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

  if (warp < 4) {
    setmaxnreg_dec<kWP_RegsCtl>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------------- Q and K tiles
      tma_prefetch(&qmap);
      tma_prefetch(&kmap);
      int t = 0;
      bool ok = true;
      for (int it = 0; it < R && ok; ++it) {
        const WItem w = win_item(a, u0 + it, ntq);
        // Q of the previous item is free once its last score product (or sink product) has finished
        if (it >= 1 && !(ok = mbar_wait(q_free, (it - 1) & 1, abort_flag, a.err, 0x30))) break;
        mbar_expect_tx(bar_q, kWP_SmemQ);
        tma_load_3d(sQ, &qmap, bar_q, 0, (w.b * a.H + w.h) * a.Tq + w.i0, 0);
        if (it + 1 < R) {   // the next head's queries into L2 behind this one's
          const WItem wn = win_item(a, u0 + it + 1, ntq);
          tma_prefetch_tile_3d(&qmap, 0, (wn.b * a.H + wn.h) * a.Tq + wn.i0, 0);
        }
        for (int j = 0; j < w.n; ++j, ++t) {
          if (t >= 1 && !(ok = mbar_wait(k_empty, (t - 1) & 1, abort_flag, a.err, 0x31))) break;
          mbar_expect_tx(k_full, kWP_SmemK);
          tma_load_3d(sK, &kmap, k_full, 0, (w.b * a.G + w.g) * a.Tk + (w.jt0 + j) * kWP_N, 0);
        }
      }
      // drain: every load issued has landed before the CTA may exit
      mbar_wait(bar_q, (R - 1) & 1, nullptr, a.err, 0x32);
      if (t > 0) mbar_wait(k_full, (t - 1) & 1, nullptr, a.err, 0x33);
    } else if (warp == 2 && lane == 0) {
      // ---------------------------------------------------------------- V^T tiles
      tma_prefetch(&vmap);
      int t = 0;
      bool ok = true;
      for (int it = 0; it < R && ok; ++it) {
        const WItem w = win_item(a, u0 + it, ntq);
        for (int j = 0; j < w.n; ++j, ++t) {
          if (t >= 1 && !(ok = mbar_wait(v_empty, (t - 1) & 1, abort_flag, a.err, 0x34))) break;
          mbar_expect_tx(v_full, kWP_SmemV);
          tma_load_3d(sV, &vmap, v_full, 0, (w.b * a.G + w.g) * kWP_D, 2 * (w.jt0 + j));
        }
      }
      if (t > 0) mbar_wait(v_full, (t - 1) & 1, nullptr, a.err, 0x35);
    } else if (warp == 1 && lane == 0) {
      // ---------------------------------------------------------------- MMA issue
      constexpr uint32_t idesc_qk = idesc_f16(kWP_M, kWP_N, 1);
      constexpr uint32_t idesc_sk = idesc_f16(kWP_M, kWP_SinkRows, 1);
      constexpr uint32_t idesc_pv = idesc_f16(kWP_M, kWP_D, 0);
      const uint32_t aQ = smem_u32(sQ), bK = smem_u32(sK), bV = smem_u32(sV), bSK = smem_u32(sSK);
      const uint64_t dSV = sdesc_sinkv(smem_u32(sSV));
      int t = 0;
      bool ok = true;
      for (int it = 0; it < R && ok; ++it) {
        const WItem w = win_item(a, u0 + it, ntq);
        if (!(ok = mbar_wait(bar_q, it & 1, abort_flag, a.err, 0x36))) break;
        // sink scores into columns 0..15 of the S buffer of the item's second tile (its earlier contents were read
        // by products issued before this one); the softmax warps read them before that buffer is written again
        const uint32_t sb = tmem + (uint32_t)((t + 1) & 1) * kWP_N;
        if (ns > 0) {
          if (it == 0 && !(ok = mbar_wait(bar_sk, 0, abort_flag, a.err, 0x3c))) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kWP_D / 16; ++ks)
            umma_f16_ss(sb, sdesc_kstep(aQ, kWP_M, ks), sdesc_kstep(bSK, kWP_SinkRows, ks), idesc_sk, ks > 0);
          umma_commit(bar_sink);
        }
        // O += P_jj V_jj; the item's first product into O waits until the previous item's O is drained
        auto issue_pv = [&](int jj, int tt) -> bool {
          const int s = tt & 1;
          if (!mbar_wait(&p_full[s], (tt >> 1) & 1, abort_flag, a.err, 0x37)) return false;
          if (!mbar_wait(v_full, tt & 1, abort_flag, a.err, 0x38)) return false;
          if (jj == 0 && it >= 1 && !mbar_wait(o_free, (it - 1) & 1, abort_flag, a.err, 0x3f)) return false;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kWP_N / 16; ++ks)
            umma_f16_ts(tmem + kTmO, tmem + s * kWP_N + p_col(ks), sdesc_kstep(bV, kWP_D, ks), idesc_pv,
                        (jj | ks) > 0 ? 1u : 0u);
          umma_commit(v_empty);
          return true;
        };
        for (int j = 0; j < w.n && ok; ++j) {
          const int tt = t + j, s = tt & 1;
          if (!(ok = mbar_wait(k_full, tt & 1, abort_flag, a.err, 0x39))) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kWP_D / 16; ++ks)
            umma_f16_ss(tmem + s * kWP_N, sdesc_kstep(aQ, kWP_M, ks), sdesc_kstep(bK, kWP_N, ks), idesc_qk, ks > 0);
          umma_commit(k_empty);
          umma_commit(&s_full[s]);
          if (j == w.n - 1) umma_commit(q_free);
          // nothing writes the sink scores' buffer again before they are read
          if (j == 0 && ns > 0 && !(ok = mbar_wait(sread, it & 1, abort_flag, a.err, 0x44))) break;
          if (j >= 1 && !(ok = issue_pv(j - 1, tt - 1))) break;
        }
        if (!ok) break;
        if (w.n > 0) {
          if (!(ok = issue_pv(w.n - 1, t + w.n - 1))) break;
        } else {
          if (ns > 0 && !(ok = mbar_wait(sread, it & 1, abort_flag, a.err, 0x44))) break;
          umma_commit(q_free);
        }
        // the sinks' product closes the item: O += P_sink V_sink (the item's only product when it has no tiles).
        // O of an item is complete only after the previous item's O was drained, even with no product at all
        if (ns > 0 && !(ok = mbar_wait(psink, it & 1, abort_flag, a.err, 0x45))) break;
        if (w.n == 0 && it >= 1 && !(ok = mbar_wait(o_free, (it - 1) & 1, abort_flag, a.err, 0x3f))) break;
        if (ns > 0) {
          tc_fence_after();
          const uint32_t psb = (uint32_t)((w.n > 0 ? t + w.n - 1 : t + 1) & 1) * kWP_N;
          umma_f16_ts(tmem + kTmO, tmem + psb + 32, dSV, idesc_pv, w.n > 0 ? 1u : 0u);
        }
        umma_commit(o_fin);
        t += w.n;
      }
    }
  } else if (warp < 12) {
    setmaxnreg_inc<kWP_RegsSoftmax>();
    // ------------------------------------------------------------------ softmax (warps 4..11)
    const int q4 = warp & 3;
    const int hh = (warp - 4) >> 2;
    const int r = q4 * 32 + lane;                // query row in the tile == TMEM lane
    const int st = tid - 128;                    // 0..255 over the softmax warps
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    const float c2 = rsqrtf((float)kWP_D) * kLog2e;   // score -> log2 domain
    constexpr int NH = kWP_N / 2;                 // 64 keys per half
    uint32_t pair_phase = 0;
    auto pair_sync = [&](unsigned int site) -> bool {  // bounded sync of the two warps on these lanes
      __syncwarp();
      if (lane == 0) mbar_arrive(&pair[q4]);
      const bool ok = mbar_wait_warp(&pair[q4], pair_phase & 1, abort_flag, a.err, site);
      ++pair_phase;
      return ok;
    };
    // sink keys -> K-major swizzled B operand (rows >= ns zero); sink values^T -> fp16 B operand (keys >= ns
    // zero): once per CTA, as all its items share (b, g).  Every load is issued before the first store
    {
      const WItem w = win_item(a, u0, ntq);
      static_assert(kWP_SinkRows * (kWP_D / 8) == 2 * 256, "two 16-byte sink-key chunks per thread");
      uint4 skc[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int i = st + q * 256, e = i / (kWP_D / 8), c = i % (kWP_D / 8);
        skc[q] = make_uint4(0u, 0u, 0u, 0u);
        if (e < ns)
          skc[q] = __ldg(reinterpret_cast<const uint4*>(a.sink_k + (size_t)w.b * a.sk_b + (size_t)w.g * a.sk_h +
                                                        (size_t)e * a.sk_k) + c);
      }
      float svl[kWP_SinkRows];   // the sink values of value column st
#pragma unroll
      for (int e = 0; e < kWP_SinkRows; ++e)
        svl[e] = (e < ns) ? __bfloat162float(a.sink_v[(size_t)w.b * a.sv_b + (size_t)w.g * a.sv_h + (size_t)e * a.sv_k + st])
                          : 0.f;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int i = st + q * 256, e = i / (kWP_D / 8), c = i % (kWP_D / 8);
        *reinterpret_cast<uint4*>(sSK + (c >> 3) * (kWP_SinkRows * 128) + e * 128 + (((c & 7) ^ (e & 7)) << 4)) = skc[q];
      }
      uint32_t hv[8];
#pragma unroll
      for (int e2 = 0; e2 < 8; ++e2) hv[e2] = pack_half2(svl[2 * e2], svl[2 * e2 + 1]);
      *reinterpret_cast<uint4*>(sSV + sv_off(st, 0)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
      *reinterpret_cast<uint4*>(sSV + sv_off(st, 8)) = make_uint4(hv[4], hv[5], hv[6], hv[7]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sk);
    }
    bool alive = true;
    int t = 0;
    for (int it = 0; it < R && alive; ++it) {
      const WItem w = win_item(a, u0 + it, ntq);
      const long long p = w.P0 + r;              // position of this query
      const uint32_t sbc = (uint32_t)((t + 1) & 1) * kWP_N;   // S buffer of the sink scores
      // sinks start the online softmax: m_ref = the row's largest visible sink score, l (half 0) = the sum of
      // their weights; half 0 keeps the weights (rescaled with O) for the product that closes the item
      float m_ref = -INFINITY, l = 0.f;            // running max (log2 domain) and this half's sum
      float wsk[kWP_MaxSinks];
#pragma unroll
      for (int e = 0; e < kWP_MaxSinks; ++e) wsk[e] = 0.f;
      if (ns > 0) {
        if (!(alive = mbar_wait_warp(bar_sink, it & 1, abort_flag, a.err, 0x3a))) break;
        tc_fence_after();
        uint32_t sw[16];
        tmem_ld16(trow + sbc, sw);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sread);
#pragma unroll
        for (int e = 0; e < kWP_MaxSinks; ++e) {
          wsk[e] = (e < ns && e <= p) ? __uint_as_float(sw[e]) * c2 : -INFINITY;
          m_ref = fmaxf(m_ref, wsk[e]);
        }
#pragma unroll
        for (int e = 0; e < kWP_MaxSinks; ++e) {
          wsk[e] = (hh == 0 && wsk[e] != -INFINITY) ? ex2_approx(wsk[e] - m_ref) : 0.f;
          l += wsk[e];
        }
      }

      for (int j = 0; j < w.n && alive; ++j) {
        const int tt = t + j, s = tt & 1;
        if (!mbar_wait_warp(&s_full[s], (tt >> 1) & 1, abort_flag, a.err, 0x3b)) { alive = false; break; }
        tc_fence_after();
        // key kt + c is a window key for this row when c_lo <= c <= c_hi (keys past Tk are never valid)
        const long long tile0 = (long long)(w.jt0 + j) * kWP_N;
        const long long kt = a.kpos0 + tile0;
        const bool full = kt >= a.klo && kt + kWP_N - 1 <= w.P0 && (w.Plast - kt) < a.W && tile0 + kWP_N <= a.Tk;
        float uu[NH];
        {
          uint32_t w0[32], w1[32];
          tmem_ld32(trow + s * kWP_N + hh * NH, w0);
          tmem_ld32(trow + s * kWP_N + hh * NH + 32, w1);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            uu[e] = __uint_as_float(w0[e]);
            uu[e + 32] = __uint_as_float(w1[e]);
          }
        }
        if (!full) {
          const long long lo = max(max(a.klo - kt, p - a.W + 1 - kt), 0LL);
          const long long hi = min(min(p - kt, (long long)kWP_N - 1), (long long)a.Tk - 1 - tile0);
          const int c_lo = (int)min(lo, (long long)kWP_N) - hh * NH, c_hi = (int)max(hi, -1LL) - hh * NH;
#pragma unroll
          for (int e = 0; e < NH; ++e) uu[e] = (e >= c_lo && e <= c_hi) ? uu[e] : -INFINITY;
        }
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int e = 0; e < NH; e += 8) {
          mx0 = max3f(mx0, uu[e], uu[e + 1]);
          mx1 = max3f(mx1, uu[e + 2], uu[e + 3]);
          mx2 = max3f(mx2, uu[e + 4], uu[e + 5]);
          mx3 = max3f(mx3, uu[e + 6], uu[e + 7]);
        }
        const float mown = max3f(mx0, mx1, fmaxf(mx2, mx3));
        float* xm = xch + (tt & 1) * 256;
        xm[hh * 128 + r] = mown;
        if (!pair_sync(0x40)) { alive = false; break; }
        const float mt = fmaxf(mown, xm[(1 - hh) * 128 + r]) * c2;
        float factor = 1.f;
        bool rescale = false;
        if (m_ref == -INFINITY) {
          m_ref = mt;  // nothing accumulated yet
        } else if (mt > m_ref + kRescaleLog2) {
          factor = ex2_approx(m_ref - mt);
          rescale = true;
          m_ref = mt;
          l *= factor;
#pragma unroll
          for (int e = 0; e < kWP_MaxSinks; ++e) wsk[e] *= factor;
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
            const float e0 = ex2_approx(fmaf(uu[c], c2, nm)), e1 = ex2_approx(fmaf(uu[c + 1], c2, nm));
            ls[(c >> 1) & 3] += e0 + e1;
            pk[c / 2] = cvt_half2(e0, e1);
          }
          l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        }
        // O rescale (warp-collective), from the item's second tile on: after O += P_{j-1} V_{j-1} has finished
        // (O += P_{j-2} V_{j-2} was issued before S_j, so this parity wait cannot pass early); at the first tile
        // the item has no O yet
        if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
          if (!mbar_wait_warp(v_empty, (tt - 1) & 1, abort_flag, a.err, 0x3e)) {
            alive = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = hh * 128; c < hh * 128 + 128; c += 32) {
            uint32_t ow[32];
            tmem_ld32(trow + kTmO + c, ow);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ow[e] = __float_as_uint(__uint_as_float(ow[e]) * factor);
            tmem_st32(trow + kTmO + c, ow);
          }
        }
        // P of this half over the first half of its own score columns
        tmem_st32(trow + s * kWP_N + hh * NH, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s]);
      }
      if (!alive) break;
      // P_sink (half 0) beside the last P it wrote, or beside the sink scores when the item has no tiles
      if (ns > 0 && hh == 0) {
        const uint32_t psb = (uint32_t)((w.n > 0 ? t + w.n - 1 : t + 1) & 1) * kWP_N;
        uint32_t pk8[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) pk8[e] = cvt_half2(wsk[2 * e], wsk[2 * e + 1]);
#pragma unroll
        for (int e = 4; e < 8; ++e) pk8[e] = 0u;
        tmem_st8(trow + psb + 32, pk8);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(psink);
      }
      t += w.n;
      // the row statistics for the epilogue (slot it & 1, free once the epilogue read item it - 2's)
      const int slot = it & 1;
      if (it >= 2 && !(alive = mbar_wait_warp(&sfree[slot], ((it >> 1) - 1) & 1, abort_flag, a.err, 0x46))) break;
      xl[slot * 256 + hh * 128 + r] = l;
      if (hh == 0) xmx[slot * 128 + r] = m_ref;
      __syncwarp();
      if (lane == 0) mbar_arrive(&stats[slot]);
    }
  } else {
    setmaxnreg_dec<kWP_RegsEpi>();
    // ------------------------------------------------------------------ epilogue (warps 12..15)
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    for (int it = 0; it < R; ++it) {
      const WItem w = win_item(a, u0 + it, ntq);
      const bool has_o = w.n > 0 || ns > 0;
      if (!mbar_wait_warp(o_fin, it & 1, abort_flag, a.err, 0x3d)) break;
      const int slot = it & 1;
      if (!mbar_wait_warp(&stats[slot], (it >> 1) & 1, abort_flag, a.err, 0x43)) break;
      const float l = xl[slot * 256 + r] + xl[slot * 256 + 128 + r];
      const float m_ref = xmx[slot * 128 + r];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[slot]);
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const float lse = l > 0.f ? (m_ref + log2f(l)) * kLn2 : -INFINITY;
      const int qi = w.i0 + r;
      if (qi < a.Tq && a.lse) a.lse[((size_t)w.b * a.H + w.h) * a.Tq + qi] = lse;
      // rows that the memory reads mix go to the workspace tile in their load order
      const int pcn = w.qt - a.perm_tile0;
      __half* const perm_dst = (a.o_perm && pcn >= 0 && pcn < a.perm_nch)
                                   ? a.o_perm + (((size_t)w.b * a.perm_nch + pcn) * a.H + w.h) * (size_t)(kWP_M * kWP_D)
                                   : nullptr;
#pragma unroll 1
      for (int c8 = 0; c8 < 8; ++c8) {
        const int hh = c8 >> 2, c4 = c8 & 3;
        const int c = hh * 128 + c4 * 32;
        uint32_t ow[32];
        if (has_o) {
          tmem_ld32(trow + kTmO + c, ow);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) ow[e] = 0u;
        }
        if (perm_dst) {
          // 8-column group e8 of column block cb = c4 / 2 as fp16: [half][cb][row group][e8][row in group][8],
          // 512 contiguous bytes per warp store
          __half* dst = perm_dst + ((size_t)(((hh * 2 + (c4 >> 1)) * 4 + q4) * 8 + (c4 & 1) * 4) * 32 + lane) * 8;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float* ov = reinterpret_cast<const float*>(ow) + 8 * k;
            *reinterpret_cast<uint4*>(dst + k * 256) =
                make_uint4(cvt_half2(ov[0] * inv, ov[1] * inv), cvt_half2(ov[2] * inv, ov[3] * inv),
                           cvt_half2(ov[4] * inv, ov[5] * inv), cvt_half2(ov[6] * inv, ov[7] * inv));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) ow[e] = __float_as_uint(__uint_as_float(ow[e]) * inv);
          tmem_st32(trow + kTmO + c, ow);
        }
      }
      if (!perm_dst) {
        // the output rows from O in 16-lane blocks: four threads write 32 contiguous bytes of a row
        tmem_wait_st();
        __syncwarp();
#pragma unroll 1
        for (int sg = 0; sg < 2; ++sg) {
#pragma unroll 1
          for (int c64 = 0; c64 < 4; ++c64) {
            uint32_t v[32];
            tmem_ld_16x256b_x8(tmem + ((uint32_t)(q4 * 32 + sg * 16) << 16) + kTmO + c64 * 64, v);
            tmem_wait_ld();
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              const int row = q4 * 32 + sg * 16 + hf * 8 + (lane >> 2);
              if (w.i0 + row < a.Tq) {
                float* op = a.o + (((size_t)w.b * a.Tq + w.i0 + row) * a.H + w.h) * kWP_D + c64 * 64 + 2 * (lane & 3);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                  *reinterpret_cast<float2*>(op + 8 * k) =
                      make_float2(__uint_as_float(v[4 * k + 2 * hf]), __uint_as_float(v[4 * k + 2 * hf + 1]));
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
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
// V^T fp16 [B,G,D,Tkp], keys beyond Tk zero.  One CTA = 64 keys x 256 columns of one (b, g): lane kp of every
// warp holds the key pair (2 kp, 2 kp + 1), warp w the 8-column chunks w, w + 8, w + 16, w + 24 (all eight
// 16-byte loads in flight); the fp16 pairs go through shared memory as [column][key pair] words (odd row pitch:
// conflict-free both ways) and leave as one 128-byte row segment per warp store.
__global__ void __launch_bounds__(256) vt_prep_kernel(const __nv_bfloat16* __restrict__ v, long long vb, long long vg,
                                                      long long vj, const __nv_bfloat16* __restrict__ ring_v, int nring,
                                                      long long ring_pos0, int W, int G, int Tk, int Tkp,
                                                      __half* __restrict__ vt) {
  __shared__ uint32_t tile[256][33];
  const int jb = blockIdx.x * 64, bg = blockIdx.y, b = bg / G, g = bg % G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto row_src = [&](int j) -> const __nv_bfloat16* {
    if (j < nring) {
      const long long kp = ring_pos0 + j;
      const int slot = (int)(((kp % W) + W) % W);
      return ring_v + (((size_t)b * G + g) * W + slot) * 256;
    }
    if (j < Tk) return v + (size_t)b * vb + (size_t)g * vg + (size_t)(j - nring) * vj;
    return nullptr;
  };
  const __nv_bfloat16* s0 = row_src(jb + 2 * lane);
  const __nv_bfloat16* s1 = row_src(jb + 2 * lane + 1);
  uint4 r0[4], r1[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int c = (warp + 8 * q) * 8;
    r0[q] = s0 ? __ldg(reinterpret_cast<const uint4*>(s0 + c)) : make_uint4(0u, 0u, 0u, 0u);
    r1[q] = s1 ? __ldg(reinterpret_cast<const uint4*>(s1 + c)) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int c = (warp + 8 * q) * 8;
    const uint32_t a0[4] = {r0[q].x, r0[q].y, r0[q].z, r0[q].w}, a1[4] = {r1[q].x, r1[q].y, r1[q].z, r1[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      // columns c + 2e (low halves) and c + 2e + 1 (high halves) of keys 2 lane and 2 lane + 1
      tile[c + 2 * e][lane] = pack_half2(__uint_as_float(a0[e] << 16), __uint_as_float(a1[e] << 16));
      tile[c + 2 * e + 1][lane] = pack_half2(__uint_as_float(a0[e] & 0xffff0000u), __uint_as_float(a1[e] & 0xffff0000u));
    }
  }
  __syncthreads();
  __half* dst = vt + ((size_t)b * G + g) * 256 * (size_t)Tkp + jb + 2 * lane;
#pragma unroll 8
  for (int d = warp; d < 256; d += 8) *reinterpret_cast<uint32_t*>(dst + (size_t)d * Tkp) = tile[d][lane];
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
  CUtensorMap qmap, kmap, vmap;
  int rc = make_tmap_kmajor(&qmap, qr, BF_BF16, (uint64_t)a.B * a.H * a.Tq, kWP_D, kWP_D, kWP_M, 4);
  if (rc) return rc;
  rc = make_tmap_kmajor(&kmap, kext, BF_BF16, (uint64_t)a.B * a.G * a.Tk, kWP_D, kWP_D, kWP_N, 4);
  if (rc) return rc;
  rc = make_tmap_kmajor(&vmap, vt, BF_F16, (uint64_t)a.B * a.G * kWP_D, a.Tkp, a.Tkp, kWP_D, 2);
  if (rc) return rc;
  if ((rc = ensure_smem_attr((const void*)window_prefill_kernel, kWP_Smem)) != BF_OK) return rc;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return cuda_fail();
  // one CTA per (b, query tile, KV group): its R query heads run back to back in the CTA
  const long long ngroups = (long long)a.B * (a.nqt > 0 ? a.nqt : (a.Tq + kWP_M - 1) / kWP_M) * a.G;
  if (ngroups == 0) return BF_OK;
  window_prefill_kernel<<<(unsigned)ngroups, kWP_Threads, kWP_Smem, stream>>>(qmap, kmap, vmap, a);
  return launch_status();
}

}  // namespace bfb
