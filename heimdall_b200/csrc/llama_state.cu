// Interchange with the llama.cpp port's per-sequence Bifrost state row (reference project Heimdall,
// llamacpp/bifrost.patch).  One fp32 row per sequence and converted layer, ggml order (ne0 fastest):
//
//   region   [C, LR]     slot rows [k_rope (G D) | v (G D) | k_mem (G D) | g (G) | beta (G)], C = 3 G D + 2 G
//                        (llama_hparams::bifrost_ring_ch, bifrost.patch:221-224; row assembly :990-996)
//   K plane  [D, LR, G]  k_rope of every slot, (d, l, g) at off_kp + (g LR + l) D + d
//   V plane  [LR, D, G]  v of every slot, transposed: (l, d, g) at off_vp + (g D + d) LR + l
//   delta    [D, D, G]   the memory state, (key k, value v, g) at off_delta + (g D + v) D + k
//
// with LR = round_up(S + W + 2, 32) slots: sink slot l < S holds position l; ring slot S + pos mod (W + 1)
// holds position pos; S + W + 1 is a scratch slot, the rest padding (bifrost_region / bifrost_state,
// :226-239; slot rule :848; offsets :1010-1013).  The delta state's key index is ne0 because the port's decode
// reads it as ggml_mul_mat(s_new, qm), a contraction over ne0 (:1129), so the row holds the transpose of the
// reference cache's S[b, g, k, v].
//
// The reference cache (heimdall/hibrit.py:414-423) keeps the last W positions at slot pos mod W and the sinks
// separately; the row keeps W + 1 ring slots so a decode's read and write never collide.  Pack writes every
// element of the row exactly once: a ring slot gets the cache row of the position any later step reads there
// (one of next_pos - W .. next_pos - 1, when the cache's ring_pos holds that position), sink slot l the sink
// row l (k_rope and v; the port writes only those there in a prefill, :1074-1076), and every other element
// zero (negative positions, the stale (W+1)-th ring slot, scratch, padding: nothing the port reads again).
// Unpack is the inverse for the slots the cache keeps, rounding k_rope and v to bf16 (round to nearest even).
//
// Both are HBM-bound layout copies: one CTA per 32 slots of one sequence writes those slots' region rows
// (one warp per slot row, coalesced), their K-plane rows, and, through shared memory, the 32-slot-wide
// column segments of the transposed V plane; the delta state is a 32 x 32 tiled transpose.
#include "bifrost_b200.h"
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

struct LsGeom {
  int G, D, W, S, LR, C, GD;
  long long off_kp, off_vp, off_dl, nfloats;
};

static LsGeom ls_geom(int G, int D, int W, int S) {
  LsGeom g;
  g.G = G; g.D = D; g.W = W; g.S = S;
  g.GD = G * D;
  g.C = 3 * g.GD + 2 * G;
  g.LR = (S + W + 2 + 31) / 32 * 32;
  g.off_kp = (long long)g.LR * g.C;
  g.off_vp = g.off_kp + (long long)g.LR * g.GD;
  g.off_dl = g.off_vp + (long long)g.LR * g.GD;
  g.nfloats = g.off_dl + (long long)D * D * G;
  return g;
}

struct LsArgs {
  LsGeom m;
  const int64_t* next_pos;     // [B]
  __nv_bfloat16* ring_k;       // [B,G,W,D]
  __nv_bfloat16* ring_v;
  float* ring_km;              // [B,W,G,D]
  float* ring_g;               // [B,W,G]
  float* ring_beta;
  int64_t* ring_pos;           // [W] or [B,W]
  long long pos_bstride;
  __nv_bfloat16* sink_k;       // [B,G,ns,D] or null
  __nv_bfloat16* sink_v;
  int ns;
  float* S;                    // [B,G,D,D] or null (pack: zero state)
  float* rows;
  long long row_stride;
};

__device__ __forceinline__ long long pmod(long long a, long long m) { return ((a % m) + m) % m; }

constexpr int kLS_Slots = 32;     // slots per CTA
constexpr int kLS_Threads = 256;
constexpr int kLS_D = 256;        // head dim (float4 chunk i of a lane: head i / 2, dims ((i & 1) 32 + lane) 4 ..)

__host__ __device__ inline int ls_vpitch(int GD) { return GD + 4; }   // bf16 per slot row of the V staging

__device__ __forceinline__ float4 bf16x4_to_f4(uint2 u) {
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xffff0000u));
}
__device__ __forceinline__ uint2 f4_to_bf16x4(float4 f) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(f.x, f.y), hi = __floats2bfloat162_rn(f.z, f.w);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}
__device__ __forceinline__ int ls_chunk_d(int i, int lane) { return (((i & 1) << 5) + lane) << 2; }

// One warp per slot row: k_rope and v (bf16 -> fp32, into the region and the K plane; v also staged in shared
// memory), k_mem, g, beta; loads are issued four chunks at a time ahead of their stores.  Then the CTA writes
// the transposed V plane from the staging: channel row e holds slots l0 .. l0 + 31 (eight float4 per row).
__global__ void __launch_bounds__(kLS_Threads) llama_pack_slots_kernel(LsArgs a) {
  const LsGeom& m = a.m;
  const int b = blockIdx.y;
  const int l0 = blockIdx.x * kLS_Slots;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int s_kind[kLS_Slots], s_idx[kLS_Slots];
  extern __shared__ __align__(16) unsigned char ls_smem[];
  __nv_bfloat16* s_v = reinterpret_cast<__nv_bfloat16*>(ls_smem);   // [32][GD + 4]
  const long long P = a.next_pos[b];
  if (threadIdx.x < kLS_Slots) {
    const int l = l0 + threadIdx.x;
    int kind = 0, idx = 0;                       // 0: zero, 1: sink row idx, 2: ring row idx
    if (l < m.S) {
      if (l < a.ns && l < P) { kind = 1; idx = l; }
    } else if (l <= m.S + m.W) {
      const long long r = l - m.S;                                   // ring slot r holds positions == r mod W+1
      const long long p = P - 1 - pmod(P - 1 - r, m.W + 1);          // the latest such position before P
      if (p >= 0 && p >= P - m.W) {
        const int j = (int)(p % m.W);
        if (a.ring_pos[(long long)b * a.pos_bstride + j] == p) { kind = 2; idx = j; }
      }
    }
    s_kind[threadIdx.x] = kind;
    s_idx[threadIdx.x] = idx;
  }
  __syncthreads();
  float* row = a.rows + (long long)b * a.row_stride;
  const int vp = ls_vpitch(m.GD);
  const int n4 = 2 * m.G;                      // float4 chunks per lane in a G*D part
  for (int s = warp; s < kLS_Slots; s += kLS_Threads / 32) {
    const int l = l0 + s;                      // LR is a multiple of 32: every slot of the tile exists
    const int kind = s_kind[s], idx = s_idx[s];
    float* rr = row + (long long)l * m.C;
    const __nv_bfloat16 *kb = nullptr, *vb = nullptr;
    long long hs = 0;                          // head stride of the source
    if (kind == 2) {
      kb = a.ring_k + ((long long)b * m.G * m.W + idx) * kLS_D;
      vb = a.ring_v + ((long long)b * m.G * m.W + idx) * kLS_D;
      hs = (long long)m.W * kLS_D;
    } else if (kind == 1) {
      kb = a.sink_k + ((long long)b * m.G * a.ns + idx) * kLS_D;
      vb = a.sink_v + ((long long)b * m.G * a.ns + idx) * kLS_D;
      hs = (long long)a.ns * kLS_D;
    }
    for (int i0 = 0; i0 < n4; i0 += 4) {
      uint2 kr[4], vr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u;
        const long long o = (i >> 1) * hs + ls_chunk_d(i, lane);
        kr[u] = kb ? __ldg(reinterpret_cast<const uint2*>(kb + o)) : make_uint2(0u, 0u);
        vr[u] = vb ? __ldg(reinterpret_cast<const uint2*>(vb + o)) : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u, g = i >> 1, e = g * kLS_D + ls_chunk_d(i, lane);
        const float4 kf = bf16x4_to_f4(kr[u]);
        *reinterpret_cast<float4*>(rr + e) = kf;
        *reinterpret_cast<float4*>(row + m.off_kp + ((long long)g * m.LR + l) * kLS_D + ls_chunk_d(i, lane)) = kf;
        *reinterpret_cast<float4*>(rr + m.GD + e) = bf16x4_to_f4(vr[u]);
        *reinterpret_cast<uint2*>(s_v + s * vp + e) = vr[u];
      }
    }
    const float* km = kind == 2 ? a.ring_km + ((long long)b * m.W + idx) * m.GD : nullptr;
    for (int i0 = 0; i0 < n4; i0 += 4) {
      float4 r4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        r4[u] = km ? __ldg(reinterpret_cast<const float4*>(km) + (i0 + u) * 32 + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 4; ++u) reinterpret_cast<float4*>(rr + 2 * m.GD)[(i0 + u) * 32 + lane] = r4[u];
    }
    if (lane < 2 * m.G) {
      float x = 0.f;
      if (kind == 2) {
        const long long o = ((long long)b * m.W + idx) * m.G;
        x = lane < m.G ? a.ring_g[o + lane] : a.ring_beta[o + lane - m.G];
      }
      rr[3 * m.GD + lane] = x;
    }
  }
  __syncthreads();
  float* vpl = row + m.off_vp + l0;
  for (int t = threadIdx.x; t < m.GD * 8; t += kLS_Threads) {
    const int e = t >> 3, q = (t & 7) << 2;
    const float4 o = make_float4(__bfloat162float(s_v[q * vp + e]), __bfloat162float(s_v[(q + 1) * vp + e]),
                                 __bfloat162float(s_v[(q + 2) * vp + e]), __bfloat162float(s_v[(q + 3) * vp + e]));
    *reinterpret_cast<float4*>(vpl + (long long)e * m.LR + q) = o;
  }
}

// delta state: rows[b] off_dl + (g D + v) D + k  <->  S[b, g, k, v]; one 32 x 32 tile per CTA, blockDim (32, 8)
template <bool kPack>
__global__ void __launch_bounds__(256) llama_state_delta_kernel(LsArgs a) {
  const LsGeom& m = a.m;
  __shared__ float tile[32][33];
  const int bg = blockIdx.z, b = bg / m.G, g = bg % m.G;
  const int tx = threadIdx.x, ty = threadIdx.y;
  float* Sg = a.S ? a.S + (long long)bg * m.D * m.D : nullptr;
  float* dl = a.rows + (long long)b * a.row_stride + m.off_dl + (long long)g * m.D * m.D;
  if (kPack) {
    const int k0 = blockIdx.y * 32, v0 = blockIdx.x * 32;
    for (int i = ty; i < 32; i += 8) tile[i][tx] = Sg ? Sg[(long long)(k0 + i) * m.D + v0 + tx] : 0.f;
    __syncthreads();
    for (int i = ty; i < 32; i += 8) dl[(long long)(v0 + i) * m.D + k0 + tx] = tile[tx][i];
  } else {
    const int v0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
    for (int i = ty; i < 32; i += 8) tile[i][tx] = dl[(long long)(v0 + i) * m.D + k0 + tx];
    __syncthreads();
    for (int i = ty; i < 32; i += 8) Sg[(long long)(k0 + i) * m.D + v0 + tx] = tile[tx][i];
  }
}

// unpack: item i < W is the cache's ring slot j = i, item W + l its sink row l; one warp per item, loads four
// float4 chunks ahead of their stores
__global__ void __launch_bounds__(kLS_Threads) llama_unpack_slots_kernel(LsArgs a) {
  const LsGeom& m = a.m;
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long P = a.next_pos[b];
  const float* row = a.rows + (long long)b * a.row_stride;
  const int n4 = 2 * m.G;
  for (int s = warp; s < kLS_Slots; s += kLS_Threads / 32) {
    const int i = blockIdx.x * kLS_Slots + s;
    if (i >= m.W + a.ns) break;
    const bool ring = i < m.W;
    long long p = 0;
    const float* rr;
    __nv_bfloat16 *kb, *vb;
    long long hs;
    if (ring) {
      p = P - m.W + pmod(i - (P - m.W), m.W);                       // the position of [P - W, P) at slot i
      rr = p >= 0 ? row + (long long)(m.S + pmod(p, m.W + 1)) * m.C : nullptr;
      kb = a.ring_k + ((long long)b * m.G * m.W + i) * kLS_D;
      vb = a.ring_v + ((long long)b * m.G * m.W + i) * kLS_D;
      hs = (long long)m.W * kLS_D;
    } else {
      const int l = i - m.W;
      rr = row + (long long)l * m.C;
      kb = a.sink_k + ((long long)b * m.G * a.ns + l) * kLS_D;
      vb = a.sink_v + ((long long)b * m.G * a.ns + l) * kLS_D;
      hs = (long long)a.ns * kLS_D;
    }
    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = 0; i0 < n4; i0 += 4) {
      float4 kr[4], vr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = i0 + u, e = (c >> 1) * kLS_D + ls_chunk_d(c, lane);
        kr[u] = rr ? *reinterpret_cast<const float4*>(rr + e) : z4;
        vr[u] = rr ? *reinterpret_cast<const float4*>(rr + m.GD + e) : z4;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = i0 + u;
        const long long o = (c >> 1) * hs + ls_chunk_d(c, lane);
        *reinterpret_cast<uint2*>(kb + o) = f4_to_bf16x4(kr[u]);
        *reinterpret_cast<uint2*>(vb + o) = f4_to_bf16x4(vr[u]);
      }
    }
    if (!ring) continue;
    float4* km = reinterpret_cast<float4*>(a.ring_km + ((long long)b * m.W + i) * m.GD);
    for (int i0 = 0; i0 < n4; i0 += 4) {
      float4 r4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) r4[u] = rr ? reinterpret_cast<const float4*>(rr + 2 * m.GD)[(i0 + u) * 32 + lane] : z4;
#pragma unroll
      for (int u = 0; u < 4; ++u) km[(i0 + u) * 32 + lane] = r4[u];
    }
    const long long o = ((long long)b * m.W + i) * m.G;
    if (lane < m.G) {
      a.ring_g[o + lane] = rr ? rr[3 * m.GD + lane] : 0.f;
      a.ring_beta[o + lane] = rr ? rr[3 * m.GD + m.G + lane] : 0.f;
    }
    if (lane == 0 && (a.pos_bstride != 0 || b == 0)) a.ring_pos[(long long)b * a.pos_bstride + i] = rr ? p : -1;
  }
}

static int ls_check(const bf_ring_cache* c, const int64_t* next_pos, int B, int G, int D, int W, int S,
                    const float* rows, long long row_stride, bool pack, LsArgs* out) {
  if (!c || !next_pos || !rows || B <= 0 || G <= 0 || D <= 0 || W <= 0 || S < 0) return BF_ERR_INVALID_ARGUMENT;
  if (!c->ring_k || !c->ring_v || !c->ring_km || !c->ring_g || !c->ring_beta || !c->ring_pos)
    return BF_ERR_INVALID_ARGUMENT;
  if (c->ns < 0 || c->ns > S || (c->ns > 0 && (!c->sink_k || !c->sink_v))) return BF_ERR_INVALID_ARGUMENT;
  if (c->ring_pos_bstride != 0 && c->ring_pos_bstride != W) return BF_ERR_INVALID_ARGUMENT;
  if (!pack && !c->S) return BF_ERR_INVALID_ARGUMENT;
  if (D != kLS_D || G % 2 || G > 8) return BF_ERR_UNSUPPORTED;
  if (!aligned16(rows) || row_stride % 4 || !aligned16(c->ring_km) || ((uintptr_t)c->ring_k & 7) ||
      ((uintptr_t)c->ring_v & 7) || ((uintptr_t)c->sink_k & 7) || ((uintptr_t)c->sink_v & 7))
    return BF_ERR_ALIGNMENT;
  const LsGeom m = ls_geom(G, D, W, S);
  if (row_stride < m.nfloats) return BF_ERR_INVALID_ARGUMENT;
  LsArgs& a = *out;
  a.m = m;
  a.next_pos = next_pos;
  a.ring_k = static_cast<__nv_bfloat16*>(c->ring_k);
  a.ring_v = static_cast<__nv_bfloat16*>(c->ring_v);
  a.ring_km = c->ring_km;
  a.ring_g = c->ring_g;
  a.ring_beta = c->ring_beta;
  a.ring_pos = c->ring_pos;
  a.pos_bstride = c->ring_pos_bstride;
  a.sink_k = static_cast<__nv_bfloat16*>(const_cast<void*>(c->sink_k));
  a.sink_v = static_cast<__nv_bfloat16*>(const_cast<void*>(c->sink_v));
  a.ns = c->ns;
  a.S = c->S;
  a.rows = const_cast<float*>(rows);
  a.row_stride = row_stride;
  return BF_OK;
}

}  // namespace bfb

using namespace bfb;

extern "C" {

size_t bf_llama_state_floats(int G, int D, int window, int sinks) {
  if (G <= 0 || D <= 0 || window <= 0 || sinks < 0) return 0;
  return (size_t)ls_geom(G, D, window, sinks).nfloats;
}

int bf_llama_state_pack(const bf_ring_cache* cache, const int64_t* next_pos, int B, int G, int D, int window,
                        int sinks, float* rows, long long row_stride, bf_stream_t stream) {
  LsArgs a;
  int rc = ls_check(cache, next_pos, B, G, D, window, sinks, rows, row_stride, true, &a);
  if (rc) return rc;
  DeviceState st;
  if ((rc = device_state(&st))) return rc;
  const int smem = kLS_Slots * ls_vpitch(a.m.GD) * 2;
  // the attribute is set once per device, to the largest staging (G = 8)
  if ((rc = ensure_smem_attr((const void*)llama_pack_slots_kernel, kLS_Slots * ls_vpitch(8 * kLS_D) * 2))) return rc;
  llama_pack_slots_kernel<<<dim3(a.m.LR / kLS_Slots, B), kLS_Threads, smem, stream>>>(a);
  if ((rc = launch_status())) return rc;
  llama_state_delta_kernel<true><<<dim3(D / 32, D / 32, B * G), dim3(32, 8), 0, stream>>>(a);
  return launch_status();
}

int bf_llama_state_unpack(const float* rows, long long row_stride, const int64_t* next_pos, int B, int G, int D,
                          int window, int sinks, bf_ring_cache* cache, bf_stream_t stream) {
  LsArgs a;
  int rc = ls_check(cache, next_pos, B, G, D, window, sinks, rows, row_stride, false, &a);
  if (rc) return rc;
  DeviceState st;
  if ((rc = device_state(&st))) return rc;
  const int items = window + a.ns;
  llama_unpack_slots_kernel<<<dim3((items + kLS_Slots - 1) / kLS_Slots, B), kLS_Threads, 0, stream>>>(a);
  if ((rc = launch_status())) return rc;
  llama_state_delta_kernel<false><<<dim3(D / 32, D / 32, B * G), dim3(32, 8), 0, stream>>>(a);
  return launch_status();
}

}  // extern "C"
