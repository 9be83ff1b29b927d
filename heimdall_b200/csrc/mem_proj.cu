// Memory-path input projections (heimdall/hibrit.py:327-334, _mem_inputs) on the 5th-gen tensor core.
//
//  head_proj: qm = unit(q_h fq_h) D^-1/2 (h < H) and km = unit(k_g fk_g) (g < G).  Per head a GEMM
//             [tokens x 256] x [256 x 256]; the weights are pre-transposed to fp16 (K-major B operand)
//             and stay resident in shared memory while a CTA walks its token tiles; q/k arrive in
//             bf16 and are converted to fp16 while being staged (both MMA operands must share a type,
//             and fp16 keeps the weights to 11 significant bits).  The L2 normalisation is the
//             epilogue: one thread owns one accumulator row (one TMEM lane).
//  x_proj:    [a | b | mix] = x [ab_w; mix_w]^T (+ bias), d = hidden size.  x is bf16, the fp32 weights
//             are split into bf16 hi + lo rows (x*hi + x*lo carries ~16 significant bits), so one
//             N=64 GEMM produces both halves; the epilogue forms g, beta and the gate logit.
#include "capi_internal.h"
#include "common.cuh"
#include "tmap.h"

namespace bfb {

// ============================================================================ weight preparation
// fq [nh][D][D] fp32 (d, e) -> wt [nh][D][D] fp16 (e, d) : B operand rows = output feature e
__global__ void prep_head_weights_kernel(const float* __restrict__ w, __half* __restrict__ wt, int D) {
  __shared__ float tile[32][33];
  const int h = blockIdx.z;
  const int d0 = blockIdx.y * 32, e0 = blockIdx.x * 32;
  const float* src = w + (size_t)h * D * D;
  __half* dst = wt + (size_t)h * D * D;
  for (int i = threadIdx.y; i < 32; i += 8) tile[i][threadIdx.x] = src[(size_t)(d0 + i) * D + e0 + threadIdx.x];
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8)
    dst[(size_t)(e0 + i) * D + d0 + threadIdx.x] = __float2half_rn(tile[threadIdx.x][i]);
}

// [ab_w; mix_w] (nout rows x d) fp32 -> hi/lo bf16 [64][d] (rows 0..31 hi, 32..63 lo, zero padded)
__global__ void prep_x_weights_kernel(const float* __restrict__ ab_w, const float* __restrict__ mix_w, int n_ab,
                                      int n_mix, int d, __nv_bfloat16* __restrict__ out) {
  const int row = blockIdx.y;  // 0..31
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < d; c += gridDim.x * blockDim.x) {
    float w = 0.f;
    if (row < n_ab) w = ab_w[(size_t)row * d + c];
    else if (row < n_ab + n_mix) w = mix_w[(size_t)(row - n_ab) * d + c];
    const __nv_bfloat16 hi = __float2bfloat16_rn(w);
    const __nv_bfloat16 lo = __float2bfloat16_rn(w - __bfloat162float(hi));
    out[(size_t)row * d + c] = hi;
    out[(size_t)(row + 32) * d + c] = lo;
  }
}

// ============================================================================ head projection
// Work items are (b, head, 128-token tile), ordered head-major; a persistent CTA walks one contiguous run of
// items, so its weights (the B operand, 128 KB) change at most once or twice.  The A operand streams through
// a ring of 64-column K atoms: the loader warp keeps up to kHP_Slots atoms in flight, four converter warps
// turn each landed atom from bf16 to fp16 in place, the MMA warp issues the atom's four K steps, and the
// epilogue warps drain one of two TMEM accumulators while the tensor core fills the other.
constexpr int kHP_M = 128;                  // tokens per tile
constexpr int kHP_D = 256;                  // head dim (K and N)
constexpr int kHP_Threads = 320;            // warps 0-3 epilogue, 4-7 convert, 8 loads, 9 MMA issue
constexpr int kHP_Slots = 6;                // A atoms in flight
constexpr int kHP_Atom = kHP_M * 64 * 2;            // 16 KB: 128 rows x 64 K (bf16 or fp16), SW128
constexpr int kHP_SmemB = kHP_D * kHP_D * 2;        // 128 KB
constexpr int kHP_Smem = kHP_SmemB + kHP_Slots * kHP_Atom + 1024 + 256;

struct HeadProjArgs {
  const __nv_bfloat16* q;  // [B,T,H,D]
  const __nv_bfloat16* k;  // [B,T,G,D]
  float* qm;               // [B,T,H,D] fp32 (or null when qm16 is set)
  __half* qm16;            // [B,T,H,D] fp16 (optional)
  float* km;               // [B,T,G,D]
  int B, T, H, G;
  int ntiles;              // token tiles per (b, head)
  long long nitems;        // B * (H + G) * ntiles
  unsigned int* err;
};

struct HPItem {
  int b, head, tile;
};
__device__ __forceinline__ HPItem hp_item(const HeadProjArgs& a, long long u) {
  HPItem it;
  it.tile = (int)(u % a.ntiles);
  const long long bh = u / a.ntiles;
  it.head = (int)(bh % (a.H + a.G));
  it.b = (int)(bh / (a.H + a.G));
  return it;
}

__global__ void __launch_bounds__(kHP_Threads, 1)
    head_proj_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap qmap,
                     const __grid_constant__ CUtensorMap kmap, HeadProjArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sA = smem + kHP_SmemB;                     // kHP_Slots atoms
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA + kHP_Slots * kHP_Atom);
  uint64_t* bar_b = bars + 0;                // weights landed (TMA)
  uint64_t* bar_bfree = bars + 1;            // MMAs on the previous weights finished
  uint64_t* full = bars + 2;                 // [kHP_Slots] atom landed (TMA)
  uint64_t* conv = full + kHP_Slots;         // [kHP_Slots] atom converted (128 arrivals)
  uint64_t* empty = conv + kHP_Slots;        // [kHP_Slots] MMA finished reading the atom
  uint64_t* acc_full = empty + kHP_Slots;    // [2] accumulator ready
  uint64_t* acc_free = acc_full + 2;         // [2] accumulator drained (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(acc_free + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long u0 = (long long)blockIdx.x * a.nitems / gridDim.x;
  const long long u1 = (long long)(blockIdx.x + 1) * a.nitems / gridDim.x;
  const int nloc = (int)(u1 - u0);

  if (tid == 0) {
    mbar_init(bar_b, 1);
    mbar_init(bar_bfree, 1);
    for (int i = 0; i < kHP_Slots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&conv[i], 128);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_free[i], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------------------------- loads: weights per head, A atoms
    if (lane == 0) {
      tma_prefetch(&wmap);
      tma_prefetch(&qmap);
      tma_prefetch(&kmap);
      int cur_head = -1, nb = 0, issued = 0;
      bool ok = true;
      for (int li = 0; li < nloc && ok; ++li) {
        const HPItem it = hp_item(a, u0 + li);
        if (it.head != cur_head) {
          if (nb > 0) ok = mbar_wait(bar_bfree, (nb - 1) & 1, abort_flag, a.err, 0x18);
          if (!ok) break;
          mbar_expect_tx(bar_b, kHP_SmemB);
          tma_load_3d(sB, &wmap, bar_b, 0, it.head * kHP_D, 0);
          ++nb;
          cur_head = it.head;
        }
        const bool is_q = it.head < a.H;
        const int hsrc = is_q ? it.head : it.head - a.H;
        for (int at = 0; at < 4; ++at) {
          const int n = li * 4 + at, slot = n % kHP_Slots;
          if (n >= kHP_Slots) ok = mbar_wait(&empty[slot], ((n / kHP_Slots) - 1) & 1, abort_flag, a.err, 0x11);
          if (!ok) break;
          mbar_expect_tx(&full[slot], kHP_Atom);
          tma_load_4d(sA + slot * kHP_Atom, is_q ? (const void*)&qmap : (const void*)&kmap, &full[slot], 0,
                      it.b * a.T + it.tile * kHP_M, at, hsrc);
          issued = n + 1;
        }
      }
      // drain: every TMA issued must have landed before the CTA may exit
      if (nb > 0) mbar_wait(bar_b, (nb - 1) & 1, nullptr, a.err, 0x14);
      for (int n = issued - 1; n >= 0 && n >= issued - kHP_Slots; --n)
        mbar_wait(&full[n % kHP_Slots], (n / kHP_Slots) & 1, nullptr, a.err, 0x17);
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kHP_M, kHP_D, 0);
      const uint32_t bB = smem_u32(sB);
      int cur_head = -1, nb = 0;
      bool ok = true;
      for (int li = 0; li < nloc && ok; ++li) {
        const HPItem it = hp_item(a, u0 + li);
        if (it.head != cur_head) {
          ok = mbar_wait(bar_b, nb & 1, abort_flag, a.err, 0x12);
          ++nb;
          cur_head = it.head;
        }
        const int buf = li & 1;
        if (ok && li >= 2) ok = mbar_wait(&acc_free[buf], ((li >> 1) - 1) & 1, abort_flag, a.err, 0x13);
        const uint32_t d = tmem + buf * 256;
        for (int at = 0; at < 4 && ok; ++at) {
          const int n = li * 4 + at, slot = n % kHP_Slots;
          ok = mbar_wait(&conv[slot], (n / kHP_Slots) & 1, abort_flag, a.err, 0x16);
          if (!ok) break;
          tc_fence_after();
          const uint32_t aA = smem_u32(sA + slot * kHP_Atom);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ss(d, sdesc_kstep(aA, kHP_M, kk), sdesc_kstep(bB, kHP_D, at * 4 + kk), idesc, (at | kk) > 0);
          umma_commit(&empty[slot]);
        }
        if (!ok) break;
        umma_commit(&acc_full[buf]);
        if (li + 1 < nloc && hp_item(a, u0 + li + 1).head != cur_head) umma_commit(bar_bfree);
      }
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- bf16 -> fp16, in place, per atom
    const int st = tid - 128;  // 0..127
    for (int n = 0; n < nloc * 4; ++n) {
      const int slot = n % kHP_Slots;
      if (!mbar_wait(&full[slot], (n / kHP_Slots) & 1, abort_flag, a.err, 0x19)) break;
      uint4* atom = reinterpret_cast<uint4*>(sA + slot * kHP_Atom);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint4 v = atom[st + 128 * j];
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w[e] = pack_half2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xffff0000u));
        atom[st + 128 * j] = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_async_smem();
      mbar_arrive(&conv[slot]);
    }
  } else {
    // ---------------------------------------------------------------- epilogue: one row per thread
    const int row = tid;  // TMEM lane
    for (int li = 0; li < nloc; ++li) {
      const int buf = li & 1;
      if (!mbar_wait_warp(&acc_full[buf], (li >> 1) & 1, abort_flag, a.err, 0x15)) break;
      tc_fence_after();
      const HPItem it = hp_item(a, u0 + li);
      const bool is_q = it.head < a.H;
      const int nheads_src = is_q ? a.H : a.G;
      const int hsrc = is_q ? it.head : it.head - a.H;
      float* dst = is_q ? a.qm : a.km;
      const float out_scale = is_q ? rsqrtf((float)kHP_D) : 1.f;
      const uint32_t base = tmem + ((uint32_t)(warp * 32) << 16) + buf * 256;
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < kHP_D; c += 64) {   // 64 columns per TMEM wait
        uint32_t r[64];
        tmem_ld32(base + c, *reinterpret_cast<uint32_t(*)[32]>(r));
        tmem_ld32(base + c + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float x = __uint_as_float(r[j]);
          ss += x * x;
        }
      }
      const float inv = out_scale / fmaxf(sqrtf(ss), 1e-12f);
      const bool row_ok = it.tile * kHP_M + row < a.T;
      const bool half_out = is_q && a.qm16 != nullptr;
      // scaled in place (for fp16 output packed two per column into columns 0..127: the 64 columns read at c
      // land at c / 2, which the earlier reads have consumed), then stored from TMEM in 16-row blocks: four
      // threads write 32 contiguous bytes of a row
#pragma unroll 1
      for (int c = 0; c < kHP_D; c += 64) {
        uint32_t r[64];
        tmem_ld32(base + c, *reinterpret_cast<uint32_t(*)[32]>(r));
        tmem_ld32(base + c + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
        tmem_wait_ld();
        if (half_out) {
          uint32_t pk[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) pk[j] = pack_half2(__uint_as_float(r[2 * j]) * inv, __uint_as_float(r[2 * j + 1]) * inv);
          tmem_st32(base + c / 2, pk);
        } else {
#pragma unroll
          for (int j = 0; j < 64; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * inv);
          tmem_st32(base + c, *reinterpret_cast<uint32_t(*)[32]>(r));
          tmem_st32(base + c + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
        }
      }
      tmem_wait_st();
      __syncwarp();
      const size_t row0 = ((size_t)it.b * a.T + (size_t)it.tile * kHP_M + warp * 32) * nheads_src + hsrc;   // row 0 of the warp
      const int q = lane & 3;
#pragma unroll 1
      for (int sg = 0; sg < 2; ++sg) {
        const uint32_t lb = tmem + ((uint32_t)(warp * 32 + sg * 16) << 16) + buf * 256;
        bool ok[2];
        size_t off[2];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int rl = sg * 16 + hf * 8 + (lane >> 2);
          ok[hf] = __shfl_sync(0xffffffffu, row_ok, rl) != 0;
          off[hf] = (row0 + (size_t)rl * nheads_src) * kHP_D;
        }
        if (half_out) {
#pragma unroll 1
          for (int cc = 0; cc < kHP_D / 2; cc += 64) {   // packed column j holds fp16 elements 2j, 2j + 1
            uint32_t v[32];
            tmem_ld_16x256b_x8(lb + cc, v);
            tmem_wait_ld();
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              if (ok[hf]) {
                __half* op = a.qm16 + off[hf] + 2 * cc + 4 * q;
#pragma unroll
                for (int k = 0; k < 8; ++k)
                  *reinterpret_cast<uint2*>(op + 16 * k) = make_uint2(v[4 * k + 2 * hf], v[4 * k + 2 * hf + 1]);
              }
            }
          }
        } else {
#pragma unroll 1
          for (int c = 0; c < kHP_D; c += 64) {
            uint32_t v[32];
            tmem_ld_16x256b_x8(lb + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              if (ok[hf]) {
                float* op = dst + off[hf] + c + 2 * q;
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
      mbar_arrive(&acc_free[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================ x projection
constexpr int kXP_M = 128;
constexpr int kXP_N = 64;        // 32 hi + 32 lo
constexpr int kXP_Stages = 4;
constexpr int kXP_StageA = kXP_M * 64 * 2;   // 16 KB
constexpr int kXP_StageB = kXP_N * 64 * 2;   // 8 KB
constexpr int kXP_Smem = kXP_Stages * (kXP_StageA + kXP_StageB) + 1024 + 256;

struct XProjArgs {
  const float* ab_b;      // [2G]
  const float* mix_b;     // [H]
  const float* A_log;     // [G]
  const float* dt_bias;   // [G]
  const float* decay_mask;// [G]
  const float* mix_lse;   // unused here
  float* g;               // [M, G]
  float* beta;            // [M, G]
  float* mixx;            // [M, H]
  const int64_t* pos;     // [M] or null
  long long pos0;         // position of row 0 of each batch when pos == null
  int M, T, d, G, H, sinks;
  unsigned int* err;
};

__global__ void __launch_bounds__(192, 1)
    x_proj_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap, XProjArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kXP_Stages * kXP_StageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kXP_Stages * kXP_StageB);
  uint64_t* full = bars;                 // [stages]
  uint64_t* empty = bars + kXP_Stages;   // [stages]
  uint64_t* done = bars + 2 * kXP_Stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kXP_Stages + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kXP_Stages + 2);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int m0 = blockIdx.x * kXP_M;
  const int nk = (a.d + 63) / 64;
  if (tid == 0) {
    for (int s = 0; s < kXP_Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (tid == 0) {
      tma_prefetch(&xmap);
      tma_prefetch(&wmap);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kXP_Stages;
        if (kb >= kXP_Stages && !mbar_wait(&empty[s], ((kb / kXP_Stages) - 1) & 1, abort_flag, a.err, 0x21)) break;
        mbar_expect_tx(&full[s], kXP_StageA + kXP_StageB);
        tma_load_3d(sA + s * kXP_StageA, &xmap, &full[s], 0, m0, kb);
        tma_load_3d(sB + s * kXP_StageB, &wmap, &full[s], 0, 0, kb);
      }
      // drain: every issued load must have landed before exit
      const int last = nk - 1;
      for (int kb = (last - kXP_Stages + 1 > 0 ? last - kXP_Stages + 1 : 0); kb <= last; ++kb)
        mbar_wait(&full[kb % kXP_Stages], (kb / kXP_Stages) & 1, nullptr, a.err, 0x22);
    }
  } else if (warp == 1) {
    if (tid == 32) {
      constexpr uint32_t idesc = idesc_f16(kXP_M, kXP_N, 1);
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % kXP_Stages;
        ok = mbar_wait(&full[s], (kb / kXP_Stages) & 1, abort_flag, a.err, 0x23);
        if (!ok) break;
        tc_fence_after();
        const uint32_t aB = smem_u32(sA + s * kXP_StageA), bB = smem_u32(sB + s * kXP_StageB);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_f16_ss(tmem, sdesc_kstep(aB, kXP_M, ks), sdesc_kstep(bB, kXP_N, ks), idesc, (kb | ks) > 0);
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(done);
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quarter (warp % 4)
    const int q4 = warp & 3;
    const int row = q4 * 32 + (tid & 31);
    if (mbar_wait_warp(done, 0, abort_flag, a.err, 0x24)) {
      tc_fence_after();
      uint32_t ra[32], rb[32];  // columns 0..31: x*hi, 32..63: x*lo
      const uint32_t base = tmem + ((uint32_t)(q4 * 32) << 16);
      tmem_ld32(base, ra);
      tmem_ld32(base + 32, rb);
      tmem_wait_ld();
      float r[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = __uint_as_float(ra[j]) + __uint_as_float(rb[j]);
      const int m = m0 + row;
      if (m < a.M) {
        const int G = a.G, H = a.H;
        const long long p = a.pos ? (long long)a.pos[m] : a.pos0 + (m % a.T);
        for (int gi = 0; gi < G; ++gi) {
          const float av = r[gi] + a.ab_b[gi];
          const float bv = r[G + gi] + a.ab_b[G + gi];
          const float z = av + a.dt_bias[gi];
          const float sp = z > 20.f ? z : log1pf(__expf(z));
          a.g[(size_t)m * G + gi] = -__expf(a.A_log[gi]) * sp * a.decay_mask[gi];
          a.beta[(size_t)m * G + gi] = (p >= a.sinks) ? 1.f / (1.f + __expf(-bv)) : 0.f;
        }
        for (int h = 0; h < H; ++h)
          a.mixx[(size_t)m * H + h] = r[2 * G + h] + a.mix_b[h];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// x_proj for few rows (decode) as split-K: CTA = (slice of 128 columns of d, block of 32 rows).  The x and
// weight slices are staged in shared memory as fp32 (weights = hi + lo, the same values the tensor-core path
// multiplies), each thread forms 4 outputs of one row over the slice, and the partial sums go to a scratch
// array [slice][row][32]; x_proj_finish_kernel adds the slices and applies the epilogue.  A 128-row
// tensor-core tile would instead walk all d columns in one CTA for a handful of rows.
constexpr int kXS_C = 128;           // columns per slice
constexpr int kXS_Rows = 32;         // rows per CTA
constexpr int kXS_MaxRows = 256;     // the split-K path serves up to this many rows

__global__ void __launch_bounds__(256) x_proj_split_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ w_x, int M, int d,
                                                           float* __restrict__ part) {
  __shared__ __align__(16) float xs[kXS_Rows][kXS_C + 4];   // padded rows: conflict-free 16-byte reads
  __shared__ __align__(16) float ws[32][kXS_C + 4];
  const int t = threadIdx.x;
  const int c0 = blockIdx.x * kXS_C, m0 = blockIdx.y * kXS_Rows;
  const int nc = min(kXS_C, d - c0);
  // stage x (bf16 -> fp32) and w = hi + lo: 8 columns per 16-byte load
  for (int i = t; i < kXS_Rows * (kXS_C / 8); i += 256) {
    const int r = i / (kXS_C / 8), c8 = (i % (kXS_C / 8)) * 8;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (m0 + r < M && c8 < nc) u = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(m0 + r) * d + c0 + c8));
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      xs[r][c8 + 2 * e] = __uint_as_float(w4[e] << 16);
      xs[r][c8 + 2 * e + 1] = __uint_as_float(w4[e] & 0xffff0000u);
    }
  }
  for (int i = t; i < 32 * (kXS_C / 8); i += 256) {
    const int j = i / (kXS_C / 8), c8 = (i % (kXS_C / 8)) * 8;
    uint4 hi = make_uint4(0u, 0u, 0u, 0u), lo = hi;
    if (c8 < nc) {
      hi = __ldg(reinterpret_cast<const uint4*>(w_x + (size_t)j * d + c0 + c8));
      lo = __ldg(reinterpret_cast<const uint4*>(w_x + (size_t)(32 + j) * d + c0 + c8));
    }
    const uint32_t h4[4] = {hi.x, hi.y, hi.z, hi.w}, l4[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ws[j][c8 + 2 * e] = __uint_as_float(h4[e] << 16) + __uint_as_float(l4[e] << 16);
      ws[j][c8 + 2 * e + 1] = __uint_as_float(h4[e] & 0xffff0000u) + __uint_as_float(l4[e] & 0xffff0000u);
    }
  }
  __syncthreads();
  // thread = (row t / 8, outputs 4 (t % 8) .. + 3)
  const int r = t >> 3, j0 = (t & 7) * 4;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int c = 0; c < kXS_C; c += 4) {
    const float4 xv = *reinterpret_cast<const float4*>(&xs[r][c]);
#pragma unroll
    for (int o = 0; o < 4; ++o) {
      const float4 wv = *reinterpret_cast<const float4*>(&ws[j0 + o][c]);
      acc[o] = fmaf(xv.x, wv.x, fmaf(xv.y, wv.y, fmaf(xv.z, wv.z, fmaf(xv.w, wv.w, acc[o]))));
    }
  }
  if (m0 + r < M)
    *reinterpret_cast<float4*>(part + ((size_t)blockIdx.x * M + m0 + r) * 32 + j0) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// sums the slices of x_proj_split_kernel and applies the x_proj epilogue; 8 rows per CTA, thread = (row, output)
__global__ void __launch_bounds__(256) x_proj_finish_kernel(const float* __restrict__ part, int nslices, XProjArgs a) {
  __shared__ float rs[8][33];
  const int t = threadIdx.x, rl = t >> 5, j = t & 31;
  const int m = blockIdx.x * 8 + rl;
  if (m < a.M) {
    float acc = 0.f;
#pragma unroll 8
    for (int sl = 0; sl < nslices; ++sl) acc += part[((size_t)sl * a.M + m) * 32 + j];
    rs[rl][j] = acc;
  }
  __syncwarp();
  if (m >= a.M) return;
  const int G = a.G, H = a.H;
  if (j < G) {
    const long long p = a.pos ? (long long)a.pos[m] : a.pos0 + (m % a.T);
    const float av = rs[rl][j] + a.ab_b[j];
    const float bv = rs[rl][G + j] + a.ab_b[G + j];
    const float z = av + a.dt_bias[j];
    const float sp = z > 20.f ? z : log1pf(__expf(z));
    a.g[(size_t)m * G + j] = -__expf(a.A_log[j]) * sp * a.decay_mask[j];
    a.beta[(size_t)m * G + j] = (p >= a.sinks) ? 1.f / (1.f + __expf(-bv)) : 0.f;
  } else if (j < G + H) {
    a.mixx[(size_t)m * H + (j - G)] = rs[rl][2 * G + (j - G)] + a.mix_b[j - G];
  }
}

size_t x_proj_scratch_bytes(int M, int d) {
  return M <= kXS_MaxRows ? (size_t)((d + kXS_C - 1) / kXS_C) * M * 32 * sizeof(float) : 0;
}

// ============================================================================ launchers
int launch_prep_weights(const float* fq, const float* fk, const float* ab_w, const float* mix_w, int H, int G,
                        int D, int d, __half* w_heads, __nv_bfloat16* w_x, cudaStream_t stream) {
  dim3 blk(32, 8);
  prep_head_weights_kernel<<<dim3(D / 32, D / 32, H), blk, 0, stream>>>(fq, w_heads, D);
  prep_head_weights_kernel<<<dim3(D / 32, D / 32, G), blk, 0, stream>>>(fk, w_heads + (size_t)H * D * D, D);
  prep_x_weights_kernel<<<dim3((d + 255) / 256, 32), 256, 0, stream>>>(ab_w, mix_w, 2 * G, H, d, w_x);
  return launch_status();
}

int launch_head_proj(const __nv_bfloat16* q, const __nv_bfloat16* k, const __half* w_heads, float* qm, __half* qm16,
                     float* km, int B, int T, int H, int G, int sm_count, unsigned int* err, cudaStream_t stream) {
  CUtensorMap wmap, qmap, kmap;
  int rc = make_tmap_kmajor(&wmap, w_heads, BF_F16, (uint64_t)(H + G) * kHP_D, kHP_D, kHP_D, kHP_D, 4);
  if (rc) return rc;
  // q [B,T,H,D] / k [B,T,G,D] bf16 as (d, token, atom, head): one 128-token x 64 atom of one head per TMA
  for (int which = 0; which < 2; ++which) {
    const int nh = which == 0 ? H : G;
    const uint64_t dims[4] = {64, (uint64_t)B * T, 4, (uint64_t)nh};
    const uint64_t strides[3] = {(uint64_t)nh * kHP_D * 2, 128, (uint64_t)kHP_D * 2};
    const uint32_t box[4] = {64, (uint32_t)kHP_M, 1, 1};
    rc = make_tmap(which == 0 ? &qmap : &kmap, which == 0 ? (const void*)q : (const void*)k, BF_BF16, 4, dims, strides,
                   box, true);
    if (rc) return rc;
  }
  if ((rc = ensure_smem_attr((const void*)head_proj_kernel, kHP_Smem)) != BF_OK) return rc;
  const int ntiles = (T + kHP_M - 1) / kHP_M;
  const long long nitems = (long long)B * (H + G) * ntiles;
  if (nitems == 0) return BF_OK;
  // one persistent CTA per SM, each walking a contiguous run of (b, head, tile) items
  const int grid = (int)(nitems < sm_count ? nitems : sm_count);
  HeadProjArgs a{q, k, qm, qm16, km, B, T, H, G, ntiles, nitems, err};
  head_proj_kernel<<<grid, kHP_Threads, kHP_Smem, stream>>>(wmap, qmap, kmap, a);
  return launch_status();
}

int launch_x_proj(const __nv_bfloat16* x, const __nv_bfloat16* w_x, const float* ab_b, const float* mix_b,
                  const float* A_log, const float* dt_bias, const float* decay_mask, float* g, float* beta,
                  float* mixx, const int64_t* pos, long long pos0, int M, int T, int d, int G, int H, int sinks,
                  float* scratch, size_t scratch_bytes, unsigned int* err, cudaStream_t stream) {
  const size_t need = x_proj_scratch_bytes(M, d);
  if (need && scratch && scratch_bytes >= need && d % 8 == 0) {
    const int nslices = (d + kXS_C - 1) / kXS_C;
    x_proj_split_kernel<<<dim3(nslices, (M + kXS_Rows - 1) / kXS_Rows), 256, 0, stream>>>(x, w_x, M, d, scratch);
    XProjArgs a{ab_b, mix_b, A_log, dt_bias, decay_mask, nullptr, g, beta, mixx, pos, pos0, M, T, d, G, H, sinks, err};
    x_proj_finish_kernel<<<(M + 7) / 8, 256, 0, stream>>>(scratch, nslices, a);
    return launch_status();
  }
  CUtensorMap xmap, wmap;
  int rc = make_tmap_kmajor(&xmap, x, BF_BF16, (uint64_t)M, d, d, kXP_M, 1);
  if (rc) return rc;
  rc = make_tmap_kmajor(&wmap, w_x, BF_BF16, 64, d, d, kXP_N, 1);
  if (rc) return rc;
  if ((rc = ensure_smem_attr((const void*)x_proj_kernel, kXP_Smem)) != BF_OK) return rc;
  XProjArgs a{ab_b, mix_b, A_log, dt_bias, decay_mask, nullptr, g, beta, mixx, pos, pos0, M, T, d, G, H, sinks, err};
  x_proj_kernel<<<(M + kXP_M - 1) / kXP_M, 192, kXP_Smem, stream>>>(xmap, wmap, a);
  return launch_status();
}

}  // namespace bfb
