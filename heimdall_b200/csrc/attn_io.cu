// The converted attention layer's prologue and epilogue around the layer core (fused elementwise passes).
//
// Prologue (heimdall/hibrit.py:254-268, HybridAttention._proj, with heimdall/kernels.py:40-49, rope): from the
// query projection (the output gate interleaved per head when the layer is gated) and the key projection, one
// pass per (token, head) computes the ZNorm (x rsqrt(mean x^2 + eps) (1 + w), fp32, rounded to bf16 as the
// reference rounds it), writes the normalised head token-major (q, k: the memory path's inputs) and, with the
// half-rotation RoPE on its first `rot` dimensions computed from those bf16 values in fp32, head-major (qr, kr:
// the window's inputs).  One warp per (token, head): lane l holds elements 8l .. 8l + 7 (D = 256), the row
// sum of squares is one warp reduction and the rotation partner of an element sits rot/16 lanes away.
// Epilogue (heimdall/hibrit.py:270-272, _out before o_proj): y = bf16(o) * bf16(sigmoid(gate)), rounded to bf16,
// the input of the output projection.
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

constexpr int kAP_D = 256;

__device__ __forceinline__ void bf16x8_unpack(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(w[j] << 16);
    f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 bf16x8_pack(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    w[j] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

struct PrologueArgs {
  const __nv_bfloat16* qg;   // [B,T,H,(1 + gated) D]
  const __nv_bfloat16* kl;   // [B,T,G,D]
  const float* q_norm_w;     // [D]
  const float* k_norm_w;     // [D]
  const float* inv_freq;     // [rot / 2]
  const int64_t* pos;        // [B*T] or null
  long long start;
  float eps;
  int rot, B, T, H, G, gated;
  __nv_bfloat16 *q, *k, *qr, *kr;
};

__global__ void __launch_bounds__(256) attn_prologue_kernel(PrologueArgs a) {
  const int lane = threadIdx.x & 31;
  const long long nheads = (long long)a.B * a.T * (a.H + a.G);
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  const int half = a.rot >> 1, lane_off = half >> 3;   // rotation partner of lane l: l +- half/8
  for (long long u = gw; u < nheads; u += nw) {
    const long long n = u / (a.H + a.G);                // token (b * T + t)
    const int j = (int)(u % (a.H + a.G));
    const bool isq = j < a.H;
    const int hj = isq ? j : j - a.H;
    const __nv_bfloat16* src = isq ? a.qg + (n * a.H + hj) * (size_t)((1 + a.gated) * kAP_D)
                                   : a.kl + (n * a.G + hj) * (size_t)kAP_D;
    const float* nw8 = (isq ? a.q_norm_w : a.k_norm_w) + 8 * lane;
    float x[8];
    bf16x8_unpack(__ldg(reinterpret_cast<const uint4*>(src) + lane), x);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss * (1.f / kAP_D) + a.eps);
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(nw8)), w1 = __ldg(reinterpret_cast<const float4*>(nw8 + 4));
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = bf16_round(x[e] * inv * (1.f + wv[e]));
    const int b = (int)(n / a.T), t = (int)(n % a.T);
    __nv_bfloat16* dst = isq ? a.q + (n * a.H + hj) * (size_t)kAP_D : a.k + (n * a.G + hj) * (size_t)kAP_D;
    reinterpret_cast<uint4*>(dst)[lane] = bf16x8_pack(y);
    // partial RoPE: element i < half pairs with i + half, both from the rounded values
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = y[e];
    const bool rot_lane = 8 * lane < a.rot;
    const int partner = lane < lane_off ? lane + lane_off : lane - lane_off;
    float o8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o8[e] = __shfl_sync(0xffffffffu, y[e], rot_lane ? partner : lane);
    if (rot_lane) {
      const long long p = a.pos ? a.pos[n] : a.start + t;
      const bool first = lane < lane_off;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int f = (first ? 8 * lane : 8 * lane - half) + e;   // frequency index
        const float ang = (float)p * __ldg(a.inv_freq + f);
        float sn, cs;
        sincosf(ang, &sn, &cs);
        // first half: x1 cos - x2 sin (x2 = the partner); second half: x1 sin + x2 cos (x1 = the partner)
        r[e] = first ? y[e] * cs - o8[e] * sn : o8[e] * sn + y[e] * cs;
      }
    }
    __nv_bfloat16* rdst = isq ? a.qr + (((size_t)b * a.H + hj) * a.T + t) * kAP_D
                              : a.kr + (((size_t)b * a.G + hj) * a.T + t) * kAP_D;
    reinterpret_cast<uint4*>(rdst)[lane] = bf16x8_pack(r);
  }
}

__global__ void __launch_bounds__(256) attn_epilogue_kernel(const float* __restrict__ o, const __nv_bfloat16* __restrict__ qg,
                                                            int gated, long long nrows, int H,
                                                            __nv_bfloat16* __restrict__ y) {
  // one thread per 8 elements of a head row: o fp32 [rows = B*T*H][D], gate the second half of qg's head row
  const long long n8 = nrows * (kAP_D / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / (kAP_D / 8);
    const int c8 = (int)(i % (kAP_D / 8));
    const float4 o0 = __ldg(reinterpret_cast<const float4*>(o + row * kAP_D) + 2 * c8);
    const float4 o1 = __ldg(reinterpret_cast<const float4*>(o + row * kAP_D) + 2 * c8 + 1);
    float v[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = bf16_round(v[e]);
    if (gated) {
      float gt[8];
      bf16x8_unpack(__ldg(reinterpret_cast<const uint4*>(qg + row * (2 * kAP_D) + kAP_D) + c8), gt);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = v[e] * bf16_round(1.f / (1.f + expf(-gt[e])));
    }
    reinterpret_cast<uint4*>(y + row * kAP_D)[c8] = bf16x8_pack(v);
  }
  (void)H;
}

}  // namespace bfb

using namespace bfb;

extern "C" {

int bf_attn_prologue(const void* qg, const void* kl, const float* q_norm_w, const float* k_norm_w,
                     const float* inv_freq, int rot, float eps, long long start, const int64_t* pos, int B, int T, int H,
                     int G, int D, int gated, void* q, void* k, void* qr, void* kr, bf_stream_t stream) {
  if (!qg || !kl || !q_norm_w || !k_norm_w || !q || !k || !qr || !kr || B <= 0 || T <= 0 || H <= 0 || G <= 0)
    return BF_ERR_INVALID_ARGUMENT;
  if (rot < 0 || rot > D || (rot > 0 && (!inv_freq || rot % 16)) || !(eps >= 0.f)) return BF_ERR_INVALID_ARGUMENT;
  if (D != kAP_D) return BF_ERR_UNSUPPORTED;
  const void* ptrs[8] = {qg, kl, q_norm_w, k_norm_w, q, k, qr, kr};
  for (const void* p : ptrs)
    if (!aligned16(p)) return BF_ERR_ALIGNMENT;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  PrologueArgs a{static_cast<const __nv_bfloat16*>(qg), static_cast<const __nv_bfloat16*>(kl), q_norm_w, k_norm_w,
                 inv_freq, pos, start, eps, rot, B, T, H, G, gated ? 1 : 0,
                 static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(qr),
                 static_cast<__nv_bfloat16*>(kr)};
  const long long nheads = (long long)B * T * (H + G);
  const long long blocks = (nheads + 7) / 8;
  const int grid = (int)(blocks < 16LL * st.sm_count ? blocks : 16LL * st.sm_count);
  attn_prologue_kernel<<<grid, 256, 0, stream>>>(a);
  return launch_status();
}

int bf_attn_epilogue(const float* o, const void* qg, int gated, int B, int T, int H, int D, void* y,
                     bf_stream_t stream) {
  if (!o || !y || (gated && !qg) || B <= 0 || T <= 0 || H <= 0) return BF_ERR_INVALID_ARGUMENT;
  if (D != kAP_D) return BF_ERR_UNSUPPORTED;
  if (!aligned16(o) || !aligned16(y) || (gated && !aligned16(qg))) return BF_ERR_ALIGNMENT;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  const long long rows = (long long)B * T * H;
  const long long n8 = rows * (kAP_D / 8);
  const long long blocks = (n8 + 255) / 256;
  const int grid = (int)(blocks < 8LL * st.sm_count ? blocks : 8LL * st.sm_count);
  attn_epilogue_kernel<<<grid, 256, 0, stream>>>(o, static_cast<const __nv_bfloat16*>(qg), gated ? 1 : 0, rows, H,
                                                 static_cast<__nv_bfloat16*>(y));
  return launch_status();
}

}  // extern "C"
