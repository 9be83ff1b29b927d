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
// Kernel 1 (split): CTA = (key split of 256 ring entries, sequence, KV head).  Thread t owns one key for
// the scores (R query heads at once), then one 8-column slice of V for the weighted sum over the split's
// keys; per-split (max, sum, acc) partials go to the workspace.  K/V are read once per (sequence, KV head).
// Kernel 2 (combine): CTA = (sequence, KV head): merges the splits, adds the sinks and the new token, forms
// lse, applies the gate and mix, and writes the new token into its ring slot.
#include "capi_internal.h"
#include "common.cuh"
#include "window_decode_args.h"

namespace bfb {

constexpr int kWD_Keys = 256;     // ring entries per split CTA
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

__global__ void __launch_bounds__(kWD_Threads) win_dec_split_kernel(WinDecArgs a) {
  extern __shared__ float sm[];
  const int D = a.D, R = a.R;
  float* sq = sm;                          // [R][D]
  float* sp = sq + kWD_MaxR * 256;         // [R][kWD_Keys] scores, then probabilities
  float* red = sp + kWD_MaxR * kWD_Keys;   // [8][R][D] per-warp partial sums
  __shared__ float s_m[kWD_MaxR], s_l[kWD_MaxR];

  const int split = blockIdx.x, bg = blockIdx.y;
  const int b = bg / a.G, g = bg % a.G;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long long p = a.pos[b];
  const float scale = rsqrtf((float)D);

  for (int i = t; i < R * D; i += kWD_Threads) {
    const int h = i / D, dd = i % D;
    sq[h * 256 + dd] = __bfloat162float(a.qr[((size_t)b * a.G * R + g * R + h) * D + dd]) * scale;
  }
  __syncthreads();

  // ---- scores: thread t <-> ring time index j (position p - W + j)
  const int j = split * kWD_Keys + t;
  bool valid = false;
  size_t rowoff = 0;
  if (j < a.W && j > 0) {
    const long long kp = p - a.W + j;
    const int slot = (int)(((kp % a.W) + a.W) % a.W);
    valid = kp >= a.S && a.ring_pos[(size_t)b * a.ring_pos_bstride + slot] == kp;
    rowoff = (((size_t)b * a.G + g) * a.W + slot) * D;
  }
  float sc[kWD_MaxR];
#pragma unroll
  for (int h = 0; h < kWD_MaxR; ++h) sc[h] = 0.f;
  if (valid) {
    const uint4* kp4 = reinterpret_cast<const uint4*>(a.ring_k + rowoff);
    for (int c = 0; c < D / 8; ++c) {
      float kf[8];
      bf16x8_to_f32(__ldg(kp4 + c), kf);
#pragma unroll
      for (int h = 0; h < kWD_MaxR; ++h) {
        if (h < R) {
          const float4 q0 = *reinterpret_cast<const float4*>(sq + h * 256 + c * 8);
          const float4 q1 = *reinterpret_cast<const float4*>(sq + h * 256 + c * 8 + 4);
          sc[h] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] + q1.y * kf[5] +
                   q1.z * kf[6] + q1.w * kf[7];
        }
      }
    }
  }
  for (int h = 0; h < R; ++h) sp[h * kWD_Keys + t] = valid ? sc[h] : -INFINITY;
  __syncthreads();
  // ---- softmax statistics per head (warp h)
  if (warp < R) {
    float m = -INFINITY;
    for (int i = lane; i < kWD_Keys; i += 32) m = fmaxf(m, sp[warp * kWD_Keys + i]);
    m = warp_max(m);
    float l = 0.f;
    for (int i = lane; i < kWD_Keys; i += 32) {
      const float s = sp[warp * kWD_Keys + i];
      const float e = (m == -INFINITY) ? 0.f : __expf(s - m);
      sp[warp * kWD_Keys + i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_m[warp] = m;
      s_l[warp] = l;
    }
  }
  __syncthreads();
  // ---- weighted V: warp w takes keys [32w, 32w+32) of the split, lane owns columns [8 lane, 8 lane + 8)
  float acc[kWD_MaxR][8];
#pragma unroll
  for (int h = 0; h < kWD_MaxR; ++h)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[h][c] = 0.f;
  const int c0 = lane * 8;
  if (c0 < D) {
    for (int kk = 0; kk < 32; ++kk) {
      const int key = warp * 32 + kk;
      const int jj = split * kWD_Keys + key;
      if (jj >= a.W || jj == 0) continue;
      bool any = false;
      for (int h = 0; h < R; ++h) any |= sp[h * kWD_Keys + key] != 0.f;
      if (!any) continue;
      const long long kp = p - a.W + jj;
      const int slot = (int)(((kp % a.W) + a.W) % a.W);
      float vf[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(a.ring_v + (((size_t)b * a.G + g) * a.W + slot) * D + c0)), vf);
#pragma unroll
      for (int h = 0; h < kWD_MaxR; ++h) {
        if (h < R) {
          const float pr = sp[h * kWD_Keys + key];
#pragma unroll
          for (int c = 0; c < 8; ++c) acc[h][c] += pr * vf[c];
        }
      }
    }
  }
  for (int h = 0; h < R; ++h)
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (c0 + c < D) red[(warp * kWD_MaxR + h) * 256 + c0 + c] = acc[h][c];
  __syncthreads();
  float* out = a.part + ((size_t)bg * a.nsplit + split) * R * (D + 2);
  for (int i = t; i < R * D; i += kWD_Threads) {
    const int h = i / D, dd = i % D;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[(w * kWD_MaxR + h) * 256 + dd];
    out[h * (D + 2) + dd] = s;
  }
  if (t < R) {
    out[t * (D + 2) + D] = s_m[t];
    out[t * (D + 2) + D + 1] = s_l[t];
  }
}

__global__ void __launch_bounds__(kWD_Threads) win_dec_combine_kernel(WinDecArgs a) {
  const int bg = blockIdx.x;
  const int b = bg / a.G, g = bg % a.G;
  const int D = a.D, R = a.R;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long long p = a.pos[b];
  const float scale = rsqrtf((float)D);
  __shared__ float s_extra[kWD_MaxR][8];   // scores of the extra keys: sinks (<= 4..7) + the new token
  __shared__ float s_stat[kWD_MaxR][2];
  const int nx = a.ns + (p >= a.S ? 1 : 0);  // extra keys
  // ---- scores of the extra keys: pair (h, key) per warp iteration
  for (int pr = warp; pr < R * nx; pr += 8) {
    const int h = pr / nx, e = pr % nx;
    const __nv_bfloat16* kp = (e < a.ns) ? a.sink_k + (((size_t)b * a.G + g) * a.ns + e) * D
                                         : a.kr + ((size_t)b * a.G + g) * D;
    const __nv_bfloat16* qp = a.qr + ((size_t)b * a.G * R + g * R + h) * D;
    float s = 0.f;
    for (int dd = lane; dd < D; dd += 32) s += __bfloat162float(qp[dd]) * __bfloat162float(kp[dd]);
    s = warp_sum(s) * scale;
    if (lane == 0) s_extra[h][e] = s;
  }
  __syncthreads();
  // ---- merge split partials + extra keys (thread t = column)
  const float* part = a.part + (size_t)bg * a.nsplit * R * (D + 2);
  for (int h = 0; h < R; ++h) {
    float m = -INFINITY;
    for (int s = 0; s < a.nsplit; ++s) m = fmaxf(m, part[(s * R + h) * (D + 2) + D]);
    for (int e = 0; e < nx; ++e) m = fmaxf(m, s_extra[h][e]);
    float l = 0.f, acc = 0.f;
    for (int s = 0; s < a.nsplit; ++s) {
      const float* ps = part + (s * R + h) * (D + 2);
      const float ms = ps[D];
      if (ms == -INFINITY) continue;
      const float f = __expf(ms - m);
      l += ps[D + 1] * f;
      if (t < D) acc += ps[t] * f;
    }
    for (int e = 0; e < nx; ++e) {
      const float f = __expf(s_extra[h][e] - m);
      l += f;
      if (t < D) {
        const __nv_bfloat16* vp = (e < a.ns) ? a.sink_v + (((size_t)b * a.G + g) * a.ns + e) * D
                                             : a.v + ((size_t)b * a.G + g) * D;
        acc += f * __bfloat162float(vp[t]);
      }
    }
    const int hh = g * R + h;
    const float lse = m + logf(l);
    if (t < D) {
      const float ow = acc / l;
      float res = ow;
      if (a.o_mem && p >= a.W) {
        const float z = a.mixx[(size_t)b * a.G * R + hh] + a.mix_lse[hh] * (lse - logf((float)a.W));
        const float gam = 1.f / (1.f + __expf(-z));
        res = ow + gam * (a.mem_scale[hh] * a.o_mem[((size_t)b * a.G * R + hh) * D + t] - ow);
      }
      a.o[((size_t)b * a.G * R + hh) * D + t] = res;
    }
    if (t == 0 && a.lse_out) a.lse_out[(size_t)b * a.G * R + hh] = lse;
    (void)s_stat;
  }
  // ---- ring write of the new token
  if (a.ring_km) {
    const int slot = (int)(p % a.W);
    const size_t kv = (((size_t)b * a.G + g) * a.W + slot) * D;
    for (int dd = t; dd < D; dd += kWD_Threads) {
      a.ring_k_w[kv + dd] = a.kr[((size_t)b * a.G + g) * D + dd];
      a.ring_v_w[kv + dd] = a.v[((size_t)b * a.G + g) * D + dd];
      a.ring_km[(((size_t)b * a.W + slot) * a.G + g) * D + dd] = a.km[((size_t)b * a.G + g) * D + dd];
    }
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

int launch_win_dec(WinDecArgs a, cudaStream_t stream) {
  a.nsplit = (a.W + kWD_Keys - 1) / kWD_Keys;
  const size_t smem = (size_t)(kWD_MaxR * 256 + kWD_MaxR * kWD_Keys + 8 * kWD_MaxR * 256) * sizeof(float);
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(win_dec_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return BF_ERR_CUDA;
    attr = true;
  }
  win_dec_split_kernel<<<dim3(a.nsplit, a.B * a.G), kWD_Threads, smem, stream>>>(a);
  win_dec_combine_kernel<<<a.B * a.G, kWD_Threads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? BF_OK : BF_ERR_CUDA;
}

int launch_gather_evicted(const float* ring_km, const __nv_bfloat16* ring_v, const float* ring_g,
                          const float* ring_beta, const int64_t* ring_pos, long long ring_pos_bstride,
                          const int64_t* pos, int B, int G, int W, int D, float* k_e, float* v_e, float* g_e,
                          float* b_e, cudaStream_t stream) {
  decode_gather_evicted_kernel<<<B * G, 256, 0, stream>>>(ring_km, ring_v, ring_g, ring_beta, ring_pos,
                                                          ring_pos_bstride, pos, G, W, D, k_e, v_e, g_e, b_e);
  return cudaGetLastError() == cudaSuccess ? BF_OK : BF_ERR_CUDA;
}

}  // namespace bfb
