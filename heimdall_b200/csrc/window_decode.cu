// Decode (one new token per sequence) of the sliding-window + sink attention and the LSE-gated mix.
//
// Semantics follow heimdall/hibrit.py:363-424 with t == 1 (the window of _window_fp32,
// hibrit.py:341-361; the gate and mix, hibrit.py:409-411; the ring/sink write, hibrit.py:414-423):
// the new token at position p attends the sinks (positions < S), the ring entries at positions
// p-W+1 .. p-1 that are valid (ring_pos matches) and >= S, and itself.  Then
//   gamma = sigmoid(mixx + mix_lse (lse - ln W)) [p >= W],  o = o_win + gamma (mem_scale o_mem - o_win).
//
// Ring layout is the reference cache layout: ring_k/ring_v [B,G,W,D] bf16 in slot order (slot = pos % W),
// ring_km [B,W,G,D] fp32, ring_g/ring_beta [B,W,G] fp32, ring_pos [W] (or [B,W]) int64.
//
// Kernel 1 (split): persistent CTAs over (sequence, KV head, 256-slot split); TMA streams the ring K/V rows,
// the scores run on the tensor core, the weighted sum of V in fp32 SIMT; per-split (max, sum, acc) partials
// go to the workspace.  K/V are read once per (sequence, KV head).
// Kernel 2 (combine): CTA = (sequence, KV head): merges the splits, adds the sinks and the new token, forms
// lse, applies the gate and mix, and writes the new token into its ring slot.
#include "capi_internal.h"
#include "common.cuh"
#include "tmap.h"
#include "window_decode_args.h"

namespace bfb {

constexpr int kWD_Keys = 512;     // ring slots per split (one work item of the split kernel)
constexpr int kWD_Threads = 256;
constexpr int kWD_MaxR = 8;



__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}

// ------------------------------------------------------------------------------------------------ split kernel
// Persistent CTA (one per SM) over items = (sequence, KV head, split of 512 ring slots), each split as four
// tiles of 128 slots.  Per tile: TMA brings the K and V rows (K-major, 128-byte swizzle); the scores of the
// R query heads are S^T = K_tile Q^T on the tensor core (M128 N16 K256, Q staged as a 16-row K-major
// operand, rows >= R zero) into one of two 16-column TMEM buffers; the softmax warps (one thread per slot)
// mask by the slot's ring position, keep a running max per head and write the probabilities; the PV warps
// (four value columns and a quarter of the tile's slots per thread) accumulate P V in fp32 from the
// swizzled V tile with packed fp32 FMAs over head pairs.  The partial (sum of p v, max, sum of p) per (item, head) goes to the workspace in the
// layout the combine kernel reads.  Slot j is a window key for the token at position p when its ring
// position kp satisfies p - W < kp < p, kp >= S and j == kp mod W (the token at p - W leaves the window at
// this step; the new token and the sinks are added by the combine kernel).

constexpr int kWT_N = 128;                        // ring slots per tile
constexpr int kWT_TilesPerItem = kWD_Keys / kWT_N;
constexpr int kWT_Threads = 512;  // warp 0 K TMA, warp 1 MMA, warp 2 Q staging, warp 3 V TMA, 4-7 softmax, 8-15 PV
constexpr int kWT_SmemK = kWT_N * 256 * 2;        // 64 KB
constexpr int kWT_SmemV = kWT_N * 256 * 2;        // 64 KB, two buffers
constexpr int kWT_SmemQ = 16 * 256 * 2;           // 8 KB, two buffers
constexpr int kWT_SmemP = kWT_N * 8 * 4;          // 4 KB, two buffers
constexpr int kWT_SmemRed = kWD_MaxR * 256 * 4;   // 8 KB
constexpr int kWT_Tiles = kWT_SmemK + 2 * kWT_SmemV + 2 * kWT_SmemQ + 2 * kWT_SmemP + kWT_SmemRed;
constexpr int kWT_Smem = kWT_Tiles + 1024 + 1024; // + barriers/statistics + alignment

template <int R>
__global__ void __launch_bounds__(kWT_Threads, 1)
    win_dec_split_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                         WinDecArgs a, unsigned int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kWT_SmemK;                                   // [2][4 atoms][128 rows][128 B]
  uint8_t* sQ = sV + 2 * kWT_SmemV;                               // [2][4 atoms][16 rows][128 B]
  float* sP = reinterpret_cast<float*>(sQ + 2 * kWT_SmemQ);       // [2][128 slots][8 heads]
  float* red = sP + 2 * kWT_N * 8;                                // [8 heads][256]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWT_Tiles);
  uint64_t* v_full = bars + 2;     // [2]
  uint64_t* pv_done = bars + 4;    // [2] PV of the tile finished (V buffer and P buffer free); 8 warps
  uint64_t* q_full = bars + 6;     // [2] Q of an item staged (warp 2)
  uint64_t* q_empty = bars + 8;    // [2] last QK of the item finished reading its Q buffer
  uint64_t* s_full = bars + 10;    // [2]
  uint64_t* s_empty = bars + 12;   // [2] softmax warps read the scores; 4 warps
  uint64_t* p_full = bars + 14;    // [2] probabilities + rescale factors written; 4 warps
  uint64_t* sync4 = bars + 16;     // softmax warps among themselves; 4 warps
  uint64_t* sync8 = bars + 17;     // PV warps among themselves; 8 warps
  uint64_t* k_full = bars + 18;    // [4] one per 64-column atom of the K tile
  uint64_t* k_empty = bars + 22;   // [4] the four k-steps of an atom finished reading it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 26);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 27);
  float* wmax = reinterpret_cast<float*>(bars + 28);             // [2][4 warps][8]
  float* wsum = wmax + 64;                                       // [4 warps][8]
  float* alpha = wsum + 32;                                      // [2][8]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int D = 256, W = a.W, G = a.G;
  const int nitems = a.B * G * a.nsplit;

  if (tid == 0) {
    for (int i = 0; i < 26; ++i)
      mbar_init(bars + i, (i == 4 || i == 5 || i == 17) ? 8 : (i >= 12 && i <= 16) ? 4 : 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- K producer: the four 64-column atoms of a
    // tile load separately, each as soon as the product of the previous tile has read that atom
    if (lane == 0) {
      tma_prefetch(&kmap);
      int n = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
        const int bg = item / a.nsplit, split = item % a.nsplit;
        for (int tt = 0; tt < kWT_TilesPerItem && ok; ++tt, ++n) {
          const int row = bg * W + (split * kWT_TilesPerItem + tt) * kWT_N;
          for (int at = 0; at < 4; ++at) {
            if (n >= 1 && !(ok = mbar_wait(&k_empty[at], (n - 1) & 1, abort_flag, err, 0x51))) break;
            mbar_expect_tx(&k_full[at], kWT_SmemK / 4);
            tma_load_3d(sK + at * (kWT_SmemK / 4), &kmap, &k_full[at], 0, row, at);
          }
        }
      }
      if (ok && n >= 1)
        for (int at = 0; at < 4; ++at) mbar_wait(&k_full[at], (n - 1) & 1, nullptr, err, 0x53);
    }
  } else if (warp == 3) {
    // ---------------------------------------------------------------- V producer (two tile buffers)
    if (lane == 0) {
      tma_prefetch(&vmap);
      int n = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
        const int bg = item / a.nsplit, split = item % a.nsplit;
        for (int tt = 0; tt < kWT_TilesPerItem && ok; ++tt, ++n) {
          const int row = bg * W + (split * kWT_TilesPerItem + tt) * kWT_N;
          if (n >= 2 && !(ok = mbar_wait(&pv_done[n & 1], ((n - 2) >> 1) & 1, abort_flag, err, 0x52))) break;
          mbar_expect_tx(&v_full[n & 1], kWT_SmemV);
          tma_load_3d(sV + (n & 1) * kWT_SmemV, &vmap, &v_full[n & 1], 0, row, 0);
        }
      }
      // drain: the last loads land before the CTA ends
      if (ok && n >= 1) {
        mbar_wait(&v_full[(n - 1) & 1], ((n - 1) >> 1) & 1, nullptr, err, 0x54);
        if (n >= 2) mbar_wait(&v_full[n & 1], ((n - 2) >> 1) & 1, nullptr, err, 0x55);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kWT_N, 16, 1);
      const uint32_t aK = smem_u32(sK), bQ = smem_u32(sQ);
      int n = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
        if (!(ok = mbar_wait(&q_full[it & 1], (it >> 1) & 1, abort_flag, err, 0x56))) break;
        const uint32_t bQi = bQ + (uint32_t)((it & 1) * kWT_SmemQ);
        for (int tt = 0; tt < kWT_TilesPerItem && ok; ++tt, ++n) {
          if (n >= 2 && !(ok = mbar_wait(&s_empty[n & 1], ((n - 2) >> 1) & 1, abort_flag, err, 0x58))) break;
          for (int at = 0; at < 4; ++at) {
            if (!(ok = mbar_wait(&k_full[at], n & 1, abort_flag, err, 0x57))) break;
            tc_fence_after();
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) {
              const int ks = at * 4 + k4;
              umma_f16_ss(tmem + (n & 1) * 16, sdesc_kstep(aK, kWT_N, ks), sdesc_kstep(bQi, 16, ks), idesc, ks > 0);
            }
            umma_commit(&k_empty[at]);
          }
          if (!ok) break;
          umma_commit(&s_full[n & 1]);
          if (tt == kWT_TilesPerItem - 1) umma_commit(&q_empty[it & 1]);
        }
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- Q staging, one item ahead (rows R..15 zero)
    int it = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++it) {
      const int bg = item / a.nsplit;
      const int b = bg / G, g = bg % G;
      if (it >= 2 && !mbar_wait_warp(&q_empty[it & 1], ((it - 2) >> 1) & 1, abort_flag, err, 0x59)) break;
      uint8_t* q = sQ + (it & 1) * kWT_SmemQ;
      for (int i = lane; i < 16 * 32; i += 32) {
        const int h = i >> 5, c = i & 31;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (h < R) v = __ldg(reinterpret_cast<const uint4*>(a.qr + ((size_t)b * G * R + g * R + h) * D) + c);
        *reinterpret_cast<uint4*>(q + (c >> 3) * (16 * 128) + h * 128 + (((c & 7) ^ (h & 7)) << 4)) = v;
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_full[it & 1]);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------------- softmax warps: thread = slot of the tile
    const int q4 = warp - 4;
    const int r = q4 * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    const float scale = rsqrtf((float)D);
    uint32_t ph4 = 0;
    auto sync_sm = [&](unsigned int site) -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(sync4);
      const bool ok = mbar_wait_warp(sync4, ph4 & 1, abort_flag, err, site);
      ++ph4;
      return ok;
    };
    int n = 0, it = 0;
    bool alive = true;
    for (int item = blockIdx.x; item < nitems && alive; item += gridDim.x, ++it) {
      const int bg = item / a.nsplit, split = item % a.nsplit;
      const int b = bg / G, g = bg % G;
      const long long p = a.pos[b];
      const long long pm = ((p + 1) % W + W) % W;      // slot of position p - W + 1
      float m[R], l[R];
#pragma unroll
      for (int h = 0; h < R; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
      }
      for (int tt = 0; tt < kWT_TilesPerItem; ++tt, ++n) {
        const int s = n & 1;
        // the slot's ring position is loaded before the wait for the scores and tested after it
        const int slot = (split * kWT_TilesPerItem + tt) * kWT_N + r;
        const long long kp = slot < W ? __ldg(a.ring_pos + (size_t)b * a.ring_pos_bstride + slot) : -1;
        if (!(alive = mbar_wait_warp(&s_full[s], (n >> 1) & 1, abort_flag, err, 0x5a))) break;
        bool valid = false;
        const long long off = kp - (p - W + 1);         // 0 .. W-2 for window keys
        if (kp >= a.S && off >= 0 && off < W - 1) {
          long long want = pm + off;
          if (want >= W) want -= W;
          valid = want == slot;
        }
        tc_fence_after();
        uint32_t w[16];
        tmem_ld16(trow + s * 16, w);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[s]);
        float sc[R];
#pragma unroll
        for (int h = 0; h < R; ++h) {
          sc[h] = valid ? __uint_as_float(w[h]) * scale : -INFINITY;
          const float mx = warp_max(sc[h]);
          if (lane == 0) wmax[(s * 4 + q4) * 8 + h] = mx;
        }
        if (!(alive = sync_sm(0x5b))) break;
        float pr[8], alh[R];
#pragma unroll
        for (int h = 0; h < 8; ++h) pr[h] = 0.f;
#pragma unroll
        for (int h = 0; h < R; ++h) {
          const float mt = fmaxf(fmaxf(wmax[(s * 4 + 0) * 8 + h], wmax[(s * 4 + 1) * 8 + h]),
                                 fmaxf(wmax[(s * 4 + 2) * 8 + h], wmax[(s * 4 + 3) * 8 + h]));
          const float mn = fmaxf(m[h], mt);
          const float al = (mn == -INFINITY) ? 1.f : __expf(m[h] - mn);
          pr[h] = (sc[h] == -INFINITY) ? 0.f : __expf(sc[h] - mn);
          l[h] = l[h] * al + pr[h];
          m[h] = mn;
          alh[h] = al;
        }
        // the P buffer and the rescale factors are free once the product of tile n - 2 is done
        if (n >= 2 && !(alive = mbar_wait_warp(&pv_done[s], ((n - 2) >> 1) & 1, abort_flag, err, 0x5c))) break;
        if (r == 0) {
#pragma unroll
          for (int h = 0; h < R; ++h) alpha[s * 8 + h] = alh[h];
        }
        float4* dst = reinterpret_cast<float4*>(sP + (s * kWT_N + r) * 8);
        dst[0] = make_float4(pr[0], pr[1], pr[2], pr[3]);
        dst[1] = make_float4(pr[4], pr[5], pr[6], pr[7]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s]);
      }
      if (!alive) break;
      // item end: sum of p per head over the 128 slot threads; one thread per head writes (max, sum)
#pragma unroll
      for (int h = 0; h < R; ++h) {
        const float sum = warp_sum(l[h]);
        if (lane == 0) wsum[q4 * 8 + h] = sum;
      }
      if (!(alive = sync_sm(0x5d))) break;
      if (r < R) {
        float* out = a.part + (((size_t)bg * a.nsplit + split) * R + r) * (D + 2);
        out[D] = m[r];
        out[D + 1] = wsum[r] + wsum[8 + r] + wsum[16 + r] + wsum[24 + r];
      }
      if (!(alive = sync_sm(0x5e))) break;     // wsum is rewritten at the next item end
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------------- PV warps: value columns 4dq..4dq+3 over a
    // quarter of the slots; accumulators are (head 2i, head 2i+1) pairs updated with packed fp32 FMAs
    constexpr int HP = (R + 1) / 2;
    const int u = tid - 256;
    const int dq = u & 63, kq = u >> 6;
    const uint32_t voff = (uint32_t)(dq >> 4) * (kWT_N * 128) + (uint32_t)((dq & 1) * 8);
    const uint32_t vchunk = (uint32_t)((dq & 15) >> 1);
    uint32_t ph8 = 0;
    auto sync_pv = [&](unsigned int site) -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(sync8);
      const bool ok = mbar_wait_warp(sync8, ph8 & 1, abort_flag, err, site);
      ++ph8;
      return ok;
    };
    int n = 0;
    bool alive = true;
    for (int item = blockIdx.x; item < nitems && alive; item += gridDim.x) {
      const int bg = item / a.nsplit, split = item % a.nsplit;
      uint64_t acc[HP][4];
#pragma unroll
      for (int h = 0; h < HP; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[h][c] = 0ull;
      for (int tt = 0; tt < kWT_TilesPerItem; ++tt, ++n) {
        const int s = n & 1;
        if (!(alive = mbar_wait_warp(&p_full[s], (n >> 1) & 1, abort_flag, err, 0x60))) break;
        if (!(alive = mbar_wait_warp(&v_full[s], (n >> 1) & 1, abort_flag, err, 0x61))) break;
        {
          const uint64_t* al2 = reinterpret_cast<const uint64_t*>(alpha + s * 8);
#pragma unroll
          for (int h = 0; h < HP; ++h) {
            const uint64_t al = al2[h];
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[h][c] = fma2(al, acc[h][c], 0ull);
          }
        }
        const uint8_t* vb = sV + s * kWT_SmemV + voff;
        const float* pb = sP + s * kWT_N * 8;
#pragma unroll 4
        for (int kk = 0; kk < kWT_N / 4; ++kk) {
          const int key = kq * (kWT_N / 4) + kk;
          const ulonglong2 p01 = *reinterpret_cast<const ulonglong2*>(pb + key * 8);
          const ulonglong2 p23 = *reinterpret_cast<const ulonglong2*>(pb + key * 8 + 4);
          const uint64_t pp[4] = {p01.x, p01.y, p23.x, p23.y};
          const uint2 vv = *reinterpret_cast<const uint2*>(vb + key * 128 + ((vchunk ^ (uint32_t)(key & 7)) << 4));
          const uint64_t vd[4] = {dup2(vv.x << 16), dup2(vv.x & 0xffff0000u), dup2(vv.y << 16),
                                  dup2(vv.y & 0xffff0000u)};
#pragma unroll
          for (int h = 0; h < HP; ++h)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[h][c] = fma2(pp[h], vd[c], acc[h][c]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&pv_done[s]);
      }
      if (!alive) break;
      // item end: the four slot quarters are summed through `red` ([head][256] fp32), quarter 0 writes out
      float* rp = red + 4 * dq;
      for (int step = 3; step >= 0 && alive; --step) {
        if (kq == step) {
#pragma unroll
          for (int h = 0; h < HP; ++h) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int hh = 2 * h + e;
              if (hh < R) {
                float4 v = make_float4(lo_hi(acc[h][0], e), lo_hi(acc[h][1], e), lo_hi(acc[h][2], e),
                                       lo_hi(acc[h][3], e));
                if (step < 3) {
                  const float4 o = *reinterpret_cast<const float4*>(rp + hh * 256);
                  v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
                }
                if (step > 0) {
                  *reinterpret_cast<float4*>(rp + hh * 256) = v;
                } else {
                  float* out = a.part + (((size_t)bg * a.nsplit + split) * R + hh) * (D + 2) + 4 * dq;
                  out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
                }
              }
            }
          }
        }
        alive = sync_pv(0x62 + step);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

// Combine: CTA = (sequence, KV head, query head), thread = value column (D = 256).  Every load is issued before
// the arithmetic that needs it: the split statistics and the extra-key scores first, then the split partial
// sums, the extra keys' values and the memory read of the mix, so a CTA costs about two DRAM round trips.
constexpr int kWD_MaxSplits = 16;
constexpr int kWD_MaxExtra = 8;

__global__ void __launch_bounds__(kWD_Threads) win_dec_combine_kernel(WinDecArgs a) {
  const int bg = blockIdx.x, h = blockIdx.y;
  const int b = bg / a.G, g = bg % a.G;
  const int D = a.D, R = a.R, ns = a.nsplit;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long long p = a.pos[b];
  const int hh = g * R + h;
  const size_t qrow = (size_t)b * a.G * R + hh;
  __shared__ float s_ms[kWD_MaxSplits], s_ls[kWD_MaxSplits], s_extra[kWD_MaxExtra];
  const int nx = a.ns + (p >= a.S ? 1 : 0);  // extra keys: the sinks and, once past them, the new token
  const float* part = a.part + ((size_t)bg * ns * R + h) * (D + 2);   // split s at + s * R * (D + 2)
  if (t < ns) {
    s_ms[t] = part[(size_t)t * R * (D + 2) + D];
    s_ls[t] = part[(size_t)t * R * (D + 2) + D + 1];
  }
  if (warp < nx) {   // extra key e = warp: one 16-byte load of q and k per lane
    const int e = warp;
    const __nv_bfloat16* kp = (e < a.ns) ? a.sink_k + (((size_t)b * a.G + g) * a.ns + e) * D
                                         : a.kr + ((size_t)b * a.G + g) * D;
    const uint4 qv = __ldg(reinterpret_cast<const uint4*>(a.qr + qrow * D) + lane);
    const uint4 kv = __ldg(reinterpret_cast<const uint4*>(kp) + lane);
    const uint32_t q4[4] = {qv.x, qv.y, qv.z, qv.w}, k4[4] = {kv.x, kv.y, kv.z, kv.w};
    float sdot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sdot = fmaf(__uint_as_float(q4[i] << 16), __uint_as_float(k4[i] << 16), sdot);
      sdot = fmaf(__uint_as_float(q4[i] & 0xffff0000u), __uint_as_float(k4[i] & 0xffff0000u), sdot);
    }
    sdot = warp_sum(sdot) * rsqrtf((float)D);
    if (lane == 0) s_extra[e] = sdot;
  }
  // this column's loads, all in flight together
  float pv[kWD_MaxSplits], ev[kWD_MaxExtra];
#pragma unroll
  for (int s2 = 0; s2 < kWD_MaxSplits; ++s2) pv[s2] = s2 < ns ? part[(size_t)s2 * R * (D + 2) + t] : 0.f;
#pragma unroll
  for (int e = 0; e < kWD_MaxExtra; ++e) {
    ev[e] = 0.f;
    if (e < nx) {
      const __nv_bfloat16* vp = (e < a.ns) ? a.sink_v + (((size_t)b * a.G + g) * a.ns + e) * D
                                           : a.v + ((size_t)b * a.G + g) * D;
      ev[e] = __bfloat162float(vp[t]);
    }
  }
  const bool gate_on = a.o_mem && p >= a.W;
  const float om = gate_on ? a.o_mem[qrow * D + t] : 0.f;
  const float mx = gate_on ? a.mixx[qrow] : 0.f;
  __syncthreads();
  float m = -INFINITY;
  for (int s2 = 0; s2 < ns; ++s2) m = fmaxf(m, s_ms[s2]);
  for (int e = 0; e < nx; ++e) m = fmaxf(m, s_extra[e]);
  float l = 0.f, acc = 0.f;
#pragma unroll
  for (int s2 = 0; s2 < kWD_MaxSplits; ++s2) {
    if (s2 < ns && s_ms[s2] != -INFINITY) {
      const float f = __expf(s_ms[s2] - m);
      l = fmaf(s_ls[s2], f, l);
      acc = fmaf(pv[s2], f, acc);
    }
  }
#pragma unroll
  for (int e = 0; e < kWD_MaxExtra; ++e) {
    if (e < nx) {
      const float f = __expf(s_extra[e] - m);
      l += f;
      acc = fmaf(f, ev[e], acc);
    }
  }
  const float lse = m + logf(l);
  const float ow = acc / l;
  float res = ow;
  if (gate_on) {
    const float z = mx + a.mix_lse[hh] * (lse - logf((float)a.W));
    const float gam = 1.f / (1.f + __expf(-z));
    res = ow + gam * (a.mem_scale[hh] * om - ow);
  }
  a.o[qrow * D + t] = res;
  if (t == 0 && a.lse_out) a.lse_out[qrow] = lse;
  // ring write of the new token (once per sequence and KV head)
  if (a.ring_km && h == 0) {
    const int slot = (int)(p % a.W);
    const size_t kv = (((size_t)b * a.G + g) * a.W + slot) * D;
    a.ring_k_w[kv + t] = a.kr[((size_t)b * a.G + g) * D + t];
    a.ring_v_w[kv + t] = a.v[((size_t)b * a.G + g) * D + t];
    a.ring_km[(((size_t)b * a.W + slot) * a.G + g) * D + t] = a.km[((size_t)b * a.G + g) * D + t];
    if (t == 0) {
      a.ring_g[((size_t)b * a.W + slot) * a.G + g] = a.g_new[(size_t)b * a.G + g];
      a.ring_beta[((size_t)b * a.W + slot) * a.G + g] = a.beta_new[(size_t)b * a.G + g];
      if (g == 0) a.ring_pos_w[(size_t)b * a.ring_pos_bstride + slot] = p;
    }
  }
}

// Combine, one CTA per (sequence, KV head) for up to kWD_FastSplits splits: thread = value column, the R query
// heads in turn.  Every load of the CTA is issued before the arithmetic: the split statistics and partial sums
// of all R heads, the extra keys' values (shared by the heads of the KV group) and the memory reads; the R x nx
// extra-key scores are warp dot products spread over the eight warps.  One wave of B*G CTAs instead of
// B*G*R CTAs of the per-head kernel above.
constexpr int kWD_FastSplits = 4;

template <int R>
__global__ void __launch_bounds__(kWD_Threads) win_dec_combine_bg_kernel(WinDecArgs a) {
  const int bg = blockIdx.x;
  const int b = bg / a.G, g = bg % a.G;
  constexpr int D = 256;
  const int ns = a.nsplit;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long long p = a.pos[b];
  __shared__ float s_ms[R][kWD_FastSplits], s_ls[R][kWD_FastSplits], s_extra[R][kWD_MaxExtra];
  const int nx = a.ns + (p >= a.S ? 1 : 0);   // extra keys: the sinks and, once past them, the new token
  const float* part = a.part + (size_t)bg * ns * R * (D + 2);   // [split][head][D + 2]
  if (t < ns * R) {
    const int s2 = t / R, h = t % R;
    s_ms[h][s2] = part[(size_t)(s2 * R + h) * (D + 2) + D];
    s_ls[h][s2] = part[(size_t)(s2 * R + h) * (D + 2) + D + 1];
  }
  const size_t qrow0 = (size_t)b * a.G * R + (size_t)g * R;
  for (int j = warp; j < R * nx; j += kWD_Threads / 32) {
    const int h = j / nx, e = j % nx;
    const __nv_bfloat16* kp = (e < a.ns) ? a.sink_k + (((size_t)b * a.G + g) * a.ns + e) * D
                                         : a.kr + ((size_t)b * a.G + g) * D;
    const uint4 qv = __ldg(reinterpret_cast<const uint4*>(a.qr + (qrow0 + h) * D) + lane);
    const uint4 kv = __ldg(reinterpret_cast<const uint4*>(kp) + lane);
    const uint32_t q4[4] = {qv.x, qv.y, qv.z, qv.w}, k4[4] = {kv.x, kv.y, kv.z, kv.w};
    float sdot = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sdot = fmaf(__uint_as_float(q4[i] << 16), __uint_as_float(k4[i] << 16), sdot);
      sdot = fmaf(__uint_as_float(q4[i] & 0xffff0000u), __uint_as_float(k4[i] & 0xffff0000u), sdot);
    }
    sdot = warp_sum(sdot) * rsqrtf((float)D);
    if (lane == 0) s_extra[h][e] = sdot;
  }
  float pv[R][kWD_FastSplits], ev[kWD_MaxExtra], om[R], mx[R];
#pragma unroll
  for (int h = 0; h < R; ++h)
#pragma unroll
    for (int s2 = 0; s2 < kWD_FastSplits; ++s2) pv[h][s2] = s2 < ns ? part[(size_t)(s2 * R + h) * (D + 2) + t] : 0.f;
#pragma unroll
  for (int e = 0; e < kWD_MaxExtra; ++e) {
    ev[e] = 0.f;
    if (e < nx) {
      const __nv_bfloat16* vp = (e < a.ns) ? a.sink_v + (((size_t)b * a.G + g) * a.ns + e) * D
                                           : a.v + ((size_t)b * a.G + g) * D;
      ev[e] = __bfloat162float(vp[t]);
    }
  }
  const bool gate_on = a.o_mem && p >= a.W;
#pragma unroll
  for (int h = 0; h < R; ++h) {
    om[h] = gate_on ? a.o_mem[(qrow0 + h) * D + t] : 0.f;
    mx[h] = gate_on ? a.mixx[qrow0 + h] : 0.f;
  }
  __syncthreads();
  const float lnW = logf((float)a.W);
#pragma unroll
  for (int h = 0; h < R; ++h) {
    float m = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < kWD_FastSplits; ++s2)
      if (s2 < ns) m = fmaxf(m, s_ms[h][s2]);
#pragma unroll
    for (int e = 0; e < kWD_MaxExtra; ++e)
      if (e < nx) m = fmaxf(m, s_extra[h][e]);
    float l = 0.f, acc = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < kWD_FastSplits; ++s2) {
      if (s2 < ns && s_ms[h][s2] != -INFINITY) {
        const float f = __expf(s_ms[h][s2] - m);
        l = fmaf(s_ls[h][s2], f, l);
        acc = fmaf(pv[h][s2], f, acc);
      }
    }
#pragma unroll
    for (int e = 0; e < kWD_MaxExtra; ++e) {
      if (e < nx) {
        const float f = __expf(s_extra[h][e] - m);
        l += f;
        acc = fmaf(f, ev[e], acc);
      }
    }
    const float lse = m + logf(l);
    const float ow = acc / l;
    float res = ow;
    const int hh = g * R + h;
    if (gate_on) {
      const float z = mx[h] + a.mix_lse[hh] * (lse - lnW);
      const float gam = 1.f / (1.f + __expf(-z));
      res = ow + gam * (a.mem_scale[hh] * om[h] - ow);
    }
    a.o[(qrow0 + h) * D + t] = res;
    if (t == 0 && a.lse_out) a.lse_out[qrow0 + h] = lse;
  }
  // ring write of the new token
  if (a.ring_km) {
    const int slot = (int)(p % a.W);
    const size_t kv = (((size_t)b * a.G + g) * a.W + slot) * D;
    a.ring_k_w[kv + t] = a.kr[((size_t)b * a.G + g) * D + t];
    a.ring_v_w[kv + t] = a.v[((size_t)b * a.G + g) * D + t];
    a.ring_km[(((size_t)b * a.W + slot) * a.G + g) * D + t] = a.km[((size_t)b * a.G + g) * D + t];
    if (t == 0) {
      a.ring_g[((size_t)b * a.W + slot) * a.G + g] = a.g_new[(size_t)b * a.G + g];
      a.ring_beta[((size_t)b * a.W + slot) * a.G + g] = a.beta_new[(size_t)b * a.G + g];
      if (g == 0) a.ring_pos_w[(size_t)b * a.ring_pos_bstride + slot] = p;
    }
  }
}

// gather the evicted ring entry (position p - W) for the state update; invalid entries become no-ops
__global__ void decode_gather_evicted_kernel(const float* __restrict__ ring_km, const __nv_bfloat16* __restrict__ ring_v,
                                             const float* __restrict__ ring_g, const float* __restrict__ ring_beta,
                                             const int64_t* __restrict__ ring_pos, long long ring_pos_bstride,
                                             const int64_t* __restrict__ pos, int G, int W, int D, float* __restrict__ k_e,
                                             float* __restrict__ v_e, float* __restrict__ g_e, float* __restrict__ b_e) {
  const int bg = blockIdx.x, b = bg / G, g = bg % G;
  const long long kp = pos[b] - W;
  const int slot = (int)(((kp % W) + W) % W);
  const bool valid = kp >= 0 && ring_pos[(size_t)b * ring_pos_bstride + slot] == kp;
  for (int dd = threadIdx.x; dd < D; dd += blockDim.x) {
    k_e[(size_t)bg * D + dd] = valid ? ring_km[(((size_t)b * W + slot) * G + g) * D + dd] : 0.f;
    v_e[(size_t)bg * D + dd] = valid ? __bfloat162float(ring_v[(((size_t)b * G + g) * W + slot) * D + dd]) : 0.f;
  }
  if (threadIdx.x == 0) {
    g_e[bg] = valid ? ring_g[((size_t)b * W + slot) * G + g] : 0.f;
    b_e[bg] = valid ? ring_beta[((size_t)b * W + slot) * G + g] : 0.f;
  }
}

size_t win_dec_workspace(int B, int G, int R, int D, int W) {
  const int nsplit = (W + kWD_Keys - 1) / kWD_Keys;
  return (size_t)B * G * nsplit * R * (D + 2) * sizeof(float);
}

template <int R>
static int launch_split(const CUtensorMap& kmap, const CUtensorMap& vmap, const WinDecArgs& a, int grid,
                        unsigned int* err, cudaStream_t stream) {
  const int rc = ensure_smem_attr((const void*)win_dec_split_kernel<R>, kWT_Smem);
  if (rc) return rc;
  win_dec_split_kernel<R><<<grid, kWT_Threads, kWT_Smem, stream>>>(kmap, vmap, a, err);
  return BF_OK;
}

int win_dec_check(WinDecArgs& a) {
  a.nsplit = (a.W + kWD_Keys - 1) / kWD_Keys;
  if (a.D != 256 || a.R < 1 || a.R > kWD_MaxR || a.nsplit > kWD_MaxSplits || a.ns + 1 > kWD_MaxExtra)
    return BF_ERR_UNSUPPORTED;
  if (!aligned16(a.qr) || !aligned16(a.kr) || (a.ns && !aligned16(a.sink_k))) return BF_ERR_ALIGNMENT;
  return BF_OK;
}

int win_dec_split_items(const WinDecArgs& a) { return a.B * a.G * ((a.W + kWD_Keys - 1) / kWD_Keys); }

int launch_win_dec_split(WinDecArgs a, cudaStream_t stream, int max_ctas) {
  int rc = win_dec_check(a);
  if (rc) return rc;
  DeviceState st;
  rc = device_state(&st);
  if (rc) return rc;
  CUtensorMap kmap, vmap;
  const uint64_t rows = (uint64_t)a.B * a.G * a.W;
  rc = make_tmap_kmajor(&kmap, a.ring_k, BF_BF16, rows, 256, 256, kWT_N, 1);   // one 64-column atom per load
  if (rc) return rc;
  rc = make_tmap_kmajor(&vmap, a.ring_v, BF_BF16, rows, 256, 256, kWT_N, 4);
  if (rc) return rc;
  const int nitems = a.B * a.G * a.nsplit;
  const int cap = (max_ctas > 0 && max_ctas < st.sm_count) ? max_ctas : st.sm_count;
  const int grid = nitems < cap ? nitems : cap;
  switch (a.R) {
    case 1: rc = launch_split<1>(kmap, vmap, a, grid, st.err, stream); break;
    case 2: rc = launch_split<2>(kmap, vmap, a, grid, st.err, stream); break;
    case 3: rc = launch_split<3>(kmap, vmap, a, grid, st.err, stream); break;
    case 4: rc = launch_split<4>(kmap, vmap, a, grid, st.err, stream); break;
    case 5: rc = launch_split<5>(kmap, vmap, a, grid, st.err, stream); break;
    case 6: rc = launch_split<6>(kmap, vmap, a, grid, st.err, stream); break;
    case 7: rc = launch_split<7>(kmap, vmap, a, grid, st.err, stream); break;
    default: rc = launch_split<8>(kmap, vmap, a, grid, st.err, stream); break;
  }
  if (rc) return rc;
  return launch_status();
}

int launch_win_dec_combine(WinDecArgs a, cudaStream_t stream) {
  int rc = win_dec_check(a);
  if (rc) return rc;
  if (a.nsplit <= kWD_FastSplits) {
    const dim3 grid(a.B * a.G);
    switch (a.R) {
      case 1: win_dec_combine_bg_kernel<1><<<grid, kWD_Threads, 0, stream>>>(a); break;
      case 2: win_dec_combine_bg_kernel<2><<<grid, kWD_Threads, 0, stream>>>(a); break;
      case 3: win_dec_combine_bg_kernel<3><<<grid, kWD_Threads, 0, stream>>>(a); break;
      case 4: win_dec_combine_bg_kernel<4><<<grid, kWD_Threads, 0, stream>>>(a); break;
      case 5: win_dec_combine_bg_kernel<5><<<grid, kWD_Threads, 0, stream>>>(a); break;
      case 6: win_dec_combine_bg_kernel<6><<<grid, kWD_Threads, 0, stream>>>(a); break;
      case 7: win_dec_combine_bg_kernel<7><<<grid, kWD_Threads, 0, stream>>>(a); break;
      default: win_dec_combine_bg_kernel<8><<<grid, kWD_Threads, 0, stream>>>(a); break;
    }
  } else {
    win_dec_combine_kernel<<<dim3(a.B * a.G, a.R), kWD_Threads, 0, stream>>>(a);
  }
  return launch_status();
}

int launch_win_dec(WinDecArgs a, cudaStream_t stream) {
  int rc = launch_win_dec_split(a, stream, 0);
  if (rc) return rc;
  return launch_win_dec_combine(a, stream);
}

int launch_gather_evicted(const float* ring_km, const __nv_bfloat16* ring_v, const float* ring_g,
                          const float* ring_beta, const int64_t* ring_pos, long long ring_pos_bstride,
                          const int64_t* pos, int B, int G, int W, int D, float* k_e, float* v_e, float* g_e,
                          float* b_e, cudaStream_t stream) {
  decode_gather_evicted_kernel<<<B * G, 256, 0, stream>>>(ring_km, ring_v, ring_g, ring_beta, ring_pos,
                                                          ring_pos_bstride, pos, G, W, D, k_e, v_e, g_e, b_e);
  return launch_status();
}

}  // namespace bfb
