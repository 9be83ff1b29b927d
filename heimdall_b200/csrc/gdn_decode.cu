// Recurrent gated delta-rule step (decode), GQA-native: one state per KV head, read by R query heads.
//
// Replaces heimdall/kernels.py:132-138 (delta_rule_step) and the inline decode update at
// heimdall/hibrit.py:398-403:
//   S <- a S (a = e^g);  delta = (v - S^T k) beta;  S <- S + k delta^T;  o_r = S^T q_r.
// Because o_r = (aS)^T q_r + delta (k . q_r), the state is read once and written once:
// one pass computes (aS)^T k and (aS)^T q_r together, the rank-1 update follows, and the new state is
// stored.  HBM traffic per (sequence, KV head) = 2 * D*D*4 bytes (+ vectors).
//
// Work split: columns of S (the Dv axis) are independent.  An item is one 32-column block of one
// (sequence, KV head) state, a [D rows][32] fp32 tile.  Persistent CTAs (one per SM) stream items
// through a ring of shared-memory stages: warp 8 issues one TMA per tile plus bulk copies of the item's
// q_r and k vectors (and stages v and the gates), warp 10 computes the item's k . q_r dot products from the
// copied vectors, so several tiles are in flight per SM; compute warp w owns column quad w over
// all rows (lane = rows lane + 32 i, so every column sum reduces inside the warp with one reduce-scatter
// of the R x 4 query sums and the 4 key sums), writes the updated tile back over the stage, and warp 9
// stores it with one TMA.
#include "capi_internal.h"
#include "common.cuh"
#include "tmap.h"

namespace bfb {

constexpr int kDecCols = 32;          // columns of S per item
constexpr int kDecMaxR = 8;
constexpr int kDecStages = 5;
constexpr int kDecThreads = 352;      // warps 0-7 compute (one column quad each), 8 loads, 9 stores, 10 k . q_r
constexpr int kDecTile = 256 * kDecCols * 4;           // 32 KB (D = 256), 128-byte swizzled rows
constexpr int kDecVec = (kDecMaxR + 1) * 256 * 4;      // q_r rows + k: 9 KB
constexpr int kDecAux = 1024;                          // v slice (32 floats), a, beta, k . q_r (at 40)
constexpr int kDecStage = kDecTile + kDecVec + kDecAux;  // 42 KB, a multiple of 1024
constexpr int kDecSmem = kDecStages * kDecStage + 256 + 1024;   // + barriers (4 per stage, abort flag)

// Warp reduce-scatter by recursive halving: 32 per-lane partial values in, lane l holds the warp total of
// quantity l (31 shuffles instead of 32 butterflies of 5).
__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int lvl = 16; lvl >= 1; lvl >>= 1) {
    const bool up = (lane & lvl) != 0;
#pragma unroll
    for (int i = 0; i < lvl; ++i) {
      const float send = up ? v[i] : v[i + lvl];
      const float keep = up ? v[i + lvl] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, lvl);
    }
  }
  return v[0];
}
// 16 quantities: lane l holds the total of quantity l >> 1
__device__ __forceinline__ float reduce_scatter16(float (&v)[16], int lane) {
#pragma unroll
  for (int lvl = 16; lvl >= 2; lvl >>= 1) {
    const bool up = (lane & lvl) != 0;
    const int h = lvl >> 1;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = up ? v[i] : v[i + h];
      const float keep = up ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, lvl);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// RT > 0: R == RT and D == 256 at compile time (the Bifrost geometry); RT == 0: R and D from the arguments
template <int RT>
__global__ void __launch_bounds__(kDecThreads, 1) gdn_decode_kernel(
    const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap omap, const float* __restrict__ q,
    const float* __restrict__ k, const void* __restrict__ v, int v_bf16, const float* __restrict__ g,
    const float* __restrict__ beta, float* __restrict__ o, int BG, int R, int D, unsigned int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDecStages * kDecStage);
  uint64_t* full = bars;                       // [stages] TMA bytes + the loader warp's arrival
  uint64_t* done = bars + kDecStages;          // [stages] 8 compute warps wrote the updated tile
  uint64_t* empty = bars + 2 * kDecStages;     // [stages] the store of the stage has read it
  uint64_t* vec = bars + 3 * kDecStages;       // [stages] the q_r and k copies landed
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 4 * kDecStages);

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int ncb = D / kDecCols, nitems = BG * ncb;
  const uint32_t tile_bytes = (uint32_t)D * kDecCols * 4;
  if (t == 0) {
    for (int i = 0; i < kDecStages; ++i) {
      mbar_init(&full[i], 3);
      mbar_init(&done[i], 8);
      mbar_init(&empty[i], 1);
      mbar_init(&vec[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 8) {
    // ------------------------------------------------------------------ loads: tile + q_r + k by TMA / bulk copy,
    // the v slice and the gates with plain loads (all into the stage)
    if (lane == 0) {
      tma_prefetch(&smap);
    }
    int n = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++n) {
      const int s = n % kDecStages;
      if (n >= kDecStages && !mbar_wait_warp(&empty[s], ((n / kDecStages) - 1) & 1, abort_flag, err, 0x71)) break;
      const int bg = item / ncb, col0 = (item % ncb) * kDecCols;
      uint8_t* st = smem + s * kDecStage;
      if (lane == 0) {
        mbar_expect_tx(&vec[s], (uint32_t)(R + 1) * D * 4);
        bulk_load_1d(st + kDecTile, q + (size_t)bg * R * D, (uint32_t)R * D * 4, &vec[s]);
        bulk_load_1d(st + kDecTile + kDecMaxR * 256 * 4, k + (size_t)bg * D, (uint32_t)D * 4, &vec[s]);
        mbar_expect_tx(&full[s], tile_bytes);
        tma_load_2d(st, &smap, &full[s], col0, bg * D);
      }
      float* aux = reinterpret_cast<float*>(st + kDecTile + kDecVec);
      aux[lane] = v_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(v)[(size_t)bg * D + col0 + lane])
                         : reinterpret_cast<const float*>(v)[(size_t)bg * D + col0 + lane];
      if (lane == 0) {
        aux[32] = __expf(g[bg]);
        aux[33] = beta[bg];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
    // drain: the last TMA loads land before the CTA ends
    if (lane == 0) {
      const int last = n - 1;
      for (int j = last; j >= 0 && j > last - kDecStages; --j) {
        mbar_wait(&vec[j % kDecStages], (j / kDecStages) & 1, nullptr, err, 0x72);
        mbar_wait(&full[j % kDecStages], (j / kDecStages) & 1, nullptr, err, 0x72);
      }
    }
  } else if (warp == 10) {
    // ------------------------------------------------------------------ k . q_r of the item (the same for every
    // column block of a state) from the stage's vector copies, into the stage's aux area
    const int Rr = RT > 0 ? RT : R;
    const int Dd = RT > 0 ? 256 : D;
    int n = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++n) {
      const int s = n % kDecStages;
      if (!mbar_wait_warp(&vec[s], (n / kDecStages) & 1, abort_flag, err, 0x77)) break;
      const uint8_t* st = smem + s * kDecStage;
      const float* sq = reinterpret_cast<const float*>(st + kDecTile);
      const float* sk = sq + kDecMaxR * 256;
      float kv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) kv[i] = (lane + 32 * i < Dd) ? sk[lane + 32 * i] : 0.f;
      float acc[kDecMaxR];
#pragma unroll
      for (int r = 0; r < kDecMaxR; ++r) {
        acc[r] = 0.f;
        if (r < Rr) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (lane + 32 * i < Dd) acc[r] = fmaf(sq[r * Dd + lane + 32 * i], kv[i], acc[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < kDecMaxR; ++r)
#pragma unroll
        for (int o2 = 16; o2 >= 1; o2 >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o2);
      float* aux = reinterpret_cast<float*>(smem + s * kDecStage + kDecTile + kDecVec);
      if (lane < kDecMaxR) {
        float val = acc[0];
#pragma unroll
        for (int r = 1; r < kDecMaxR; ++r) val = (lane == r) ? acc[r] : val;
        aux[40 + lane] = val;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ stores: the updated tile by TMA
    // two stores in flight: after issuing item n's store, wait until item n-1's has read its stage, then free it
    if (lane == 0) {
      tma_prefetch(&omap);
      int n = 0;
      for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++n) {
        const int s = n % kDecStages;
        if (!mbar_wait(&done[s], (n / kDecStages) & 1, abort_flag, err, 0x76)) break;
        const int bg = item / ncb, col0 = (item % ncb) * kDecCols;
        tma_store_2d(&omap, smem + s * kDecStage, col0, bg * D);
        tma_store_commit();
        if (n >= 1) {
          tma_store_wait_read_pending<1>();
          mbar_arrive(&empty[(n - 1) % kDecStages]);
        }
      }
      tma_store_wait_read();
      if (n >= 1) mbar_arrive(&empty[(n - 1) % kDecStages]);
      tma_store_wait_all();
    }
  } else {
    // ------------------------------------------------------------------ compute: warp w = column quad w,
    // lane = rows lane + 32 i; column sums reduce inside the warp
    const int Rr = RT > 0 ? RT : R;
    const int Dd = RT > 0 ? 256 : D;
    const int nrow = Dd >> 5;
    int n = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++n) {
      const int s = n % kDecStages;
      // (the vector copies completed before the k . q_r warp's arrival on full; their own barrier is
      // observed here too, so the copies are visible to this warp directly)
      if (!mbar_wait_warp(&full[s], (n / kDecStages) & 1, abort_flag, err, 0x73) ||
          !mbar_wait_warp(&vec[s], (n / kDecStages) & 1, abort_flag, err, 0x78))
        break;
      const int bg = item / ncb, col0 = (item % ncb) * kDecCols;
      uint8_t* tile = smem + s * kDecStage;
      const float* sq = reinterpret_cast<const float*>(tile + kDecTile);      // [R][D]
      const float* sk = sq + kDecMaxR * 256;                                   // [D]
      const float* aux = reinterpret_cast<const float*>(tile + kDecTile + kDecVec);
      const float a = aux[32], bt = aux[33];
      float4 x[8];
      float kr[8];
      float pk[4] = {0.f, 0.f, 0.f, 0.f};
      float pq[kDecMaxR][4];
#pragma unroll
      for (int r = 0; r < kDecMaxR; ++r) pq[r][0] = pq[r][1] = pq[r][2] = pq[r][3] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < nrow) {
          const int row = lane + 32 * i;
          float4 y = *reinterpret_cast<const float4*>(tile + row * 128 + ((warp ^ (row & 7)) << 4));
          y.x *= a; y.y *= a; y.z *= a; y.w *= a;
          x[i] = y;
          kr[i] = sk[row];
          pk[0] = fmaf(kr[i], y.x, pk[0]); pk[1] = fmaf(kr[i], y.y, pk[1]);
          pk[2] = fmaf(kr[i], y.z, pk[2]); pk[3] = fmaf(kr[i], y.w, pk[3]);
#pragma unroll
          for (int r = 0; r < kDecMaxR; ++r) {
            if (r < Rr) {
              const float qv = sq[r * Dd + row];
              pq[r][0] = fmaf(qv, y.x, pq[r][0]); pq[r][1] = fmaf(qv, y.y, pq[r][1]);
              pq[r][2] = fmaf(qv, y.z, pq[r][2]); pq[r][3] = fmaf(qv, y.w, pq[r][3]);
            }
          }
        }
      }
      // column totals by one reduce-scatter: quantity 4r + c = q_r . (aS)[:, c]; with R <= 7 the key sums
      // k . (aS)[:, c] ride in quantities 28 + c, with R = 8 they take a second, 16-quantity pass
      float va[32];
#pragma unroll
      for (int r = 0; r < kDecMaxR; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) va[4 * r + c] = pq[r][c];
      if (Rr <= 7) {
#pragma unroll
        for (int c = 0; c < 4; ++c) va[28 + c] = pk[c];
      }
      const float ta = reduce_scatter32(va, lane);
      float ks4[4];
      if (Rr <= 7) {
#pragma unroll
        for (int c = 0; c < 4; ++c) ks4[c] = __shfl_sync(0xffffffffu, ta, 28 + c);
      } else {
        float vb[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) vb[c] = pk[c];
#pragma unroll
        for (int i = 4; i < 16; ++i) vb[i] = 0.f;
        const float tb = reduce_scatter16(vb, lane);
#pragma unroll
        for (int c = 0; c < 4; ++c) ks4[c] = __shfl_sync(0xffffffffu, tb, 2 * c);
      }
      float d4[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) d4[c] = (aux[warp * 4 + c] - ks4[c]) * bt;
      // outputs o_r[col] = (aS)^T q_r + delta * (k . q_r): lane 4r + c holds head r, column 4w + c
      {
        const int r = lane >> 2, c = lane & 3;
        const float dc = (c == 0) ? d4[0] : (c == 1) ? d4[1] : (c == 2) ? d4[2] : d4[3];
        if (r < Rr) o[((size_t)bg * Rr + r) * Dd + col0 + warp * 4 + c] = ta + dc * aux[40 + r];
      }
      // rank-1 update written back over the tile (the store warp copies it out)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < nrow) {
          const int row = lane + 32 * i;
          float4 y = x[i];
          y.x = fmaf(kr[i], d4[0], y.x);
          y.y = fmaf(kr[i], d4[1], y.y);
          y.z = fmaf(kr[i], d4[2], y.z);
          y.w = fmaf(kr[i], d4[3], y.w);
          *reinterpret_cast<float4*>(tile + row * 128 + ((warp ^ (row & 7)) << 4)) = y;
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&done[s]);
    }
  }
}

int launch_gdn_decode(const float* q, const float* k, const void* v, int v_bf16, const float* g,
                      const float* beta, const float* s_in, float* s_out, float* o, int B, int G, int R, int D,
                      cudaStream_t stream, int max_ctas) {
  if (D % kDecCols || D > 256 || R < 1 || R > kDecMaxR) return BF_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(s_in) || !aligned16(s_out)) return BF_ERR_ALIGNMENT;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  // S as [B*G*D rows][D] fp32; an item is a [D][32] box (128-byte rows, 128-byte swizzle)
  CUtensorMap smap, omap;
  const uint64_t dims[2] = {(uint64_t)D, (uint64_t)B * G * D};
  const uint64_t strides[1] = {(uint64_t)D * 4};
  const uint32_t box[2] = {(uint32_t)kDecCols, (uint32_t)D};
  rc = make_tmap(&smap, s_in, BF_F32, 2, dims, strides, box, true);
  if (rc) return rc;
  rc = make_tmap(&omap, s_out, BF_F32, 2, dims, strides, box, true);
  if (rc) return rc;
  if ((rc = ensure_smem_attr((const void*)gdn_decode_kernel<6>, kDecSmem)) != BF_OK) return rc;
  if ((rc = ensure_smem_attr((const void*)gdn_decode_kernel<0>, kDecSmem)) != BF_OK) return rc;
  const int nitems = B * G * (D / kDecCols);
  const int cap = (max_ctas > 0 && max_ctas < st.sm_count) ? max_ctas : st.sm_count;
  const int grid = nitems < cap ? nitems : cap;
  if (R == 6 && D == 256)
    gdn_decode_kernel<6><<<grid, kDecThreads, kDecSmem, stream>>>(smap, omap, q, k, v, v_bf16, g, beta, o, B * G, R, D,
                                                                 st.err);
  else
    gdn_decode_kernel<0><<<grid, kDecThreads, kDecSmem, stream>>>(smap, omap, q, k, v, v_bf16, g, beta, o, B * G, R, D,
                                                                 st.err);
  return launch_status();
}

}  // namespace bfb
