// C ABI: the sequence-parallel pieces of the chunked delta rule.
//
// A segment of the write stream (keys k, values v, gates g, beta) maps any initial state S to
//   S_out = M (S - s0) + N,
// where N is the final state from s0 (zero when s0 is null) and M = prod_c (gamma_c I - K~_c^T W_c) is the
// product of the per-chunk state maps (the UT/WY form of heimdall/kernels.py:94-129).
// bf_gdn_segment_transform computes (M, N) for a segment on one GPU: P1 as in the chunked forward, then P2
// over twice the state columns -- the usual recurrence from s0 for N, and the same recurrence from the
// identity with zero inputs for M (each column of the state evolves independently, and the homogeneous
// recurrence applied to I is exactly the product of the maps).  Both run in the forward pass's fp32
// arithmetic.  bf_gdn_apply_prefix folds the segments in order: S_in[0] = s0, S_in[j+1] = M_j S_in[j] + N_j.
// Ranks that own consecutive segments exchange their (M, N) and each computes its own S_in (see
// heimdall_b200/sp.py); the segments then run their outputs from the true incoming state.
#include "bifrost_b200.h"
#include "capi_internal.h"
#include "common.cuh"
#include "gdn_prefill.h"

namespace bfb {
size_t gdn_prefill_workspace(int B, int G, int T_steps, bool transform);
int gdn_prefill_carve(GdnStreams& s, void* ws);
int launch_gdn_prefill(GdnStreams s, cudaStream_t stream, int parts);

static size_t al1k_sp(size_t x) { return (x + 1023) & ~size_t(1023); }

__global__ void sp_bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

// out = A @ S + N for one (b, g) matrix of a batch: 64 x 64 output tile per CTA, 4 x 4 per thread, fp32; k in
// slabs of 64 (four load rounds for D = 256, each thread's 16 + 16 loads issued before its stores): the fold of
// the segment maps runs these one after another on the critical path, so each launch is latency-bound
constexpr int kSM_T = 64, kSM_K = 64;
__global__ void __launch_bounds__(256) state_map_kernel(const float* __restrict__ A, const float* __restrict__ S,
                                                        const float* __restrict__ N, float* __restrict__ out,
                                                        int D) {
  __shared__ float As[kSM_K][kSM_T + 4];   // A tile transposed: As[k][i]
  __shared__ float Ss[kSM_K][kSM_T + 4];   // S tile: Ss[k][j]
  const size_t off = (size_t)blockIdx.z * D * D;
  A += off; S += off; out += off;
  const float* Nz = N ? N + off : nullptr;
  const int i0 = blockIdx.y * kSM_T, j0 = blockIdx.x * kSM_T;
  const int t = threadIdx.x, ti = (t >> 4) * 4, tj = (t & 15) * 4;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < D; k0 += kSM_K) {
    constexpr int kPer = kSM_T * kSM_K / 256;
    float av_[kPer], sv_[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = t + 256 * u;
      const int r = e / kSM_K, c = e % kSM_K;        // A[i0 + r][k0 + c]
      av_[u] = A[(size_t)(i0 + r) * D + k0 + c];
      const int r2 = e / kSM_T, c2 = e % kSM_T;      // S[k0 + r2][j0 + c2]
      sv_[u] = S[(size_t)(k0 + r2) * D + j0 + c2];
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = t + 256 * u;
      As[e % kSM_K][e / kSM_K] = av_[u];
      Ss[e / kSM_T][e % kSM_T] = sv_[u];
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSM_K; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ti]);
      const float4 b = *reinterpret_cast<const float4*>(&Ss[kk][tj]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(av[x], bv[y], acc[x][y]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const size_t row = (size_t)(i0 + ti + x) * D + j0 + tj;
    float4 r = make_float4(acc[x][0], acc[x][1], acc[x][2], acc[x][3]);
    if (Nz) {
      const float4 n = *reinterpret_cast<const float4*>(Nz + row);
      r.x += n.x; r.y += n.y; r.z += n.z; r.w += n.w;
    }
    *reinterpret_cast<float4*>(out + row) = r;
  }
}

// out = A @ S + N per (b, g) matrix (fp32), out distinct from S
int launch_state_map(const float* A, const float* S, const float* N, float* out, int BG, int D, cudaStream_t stream) {
  state_map_kernel<<<dim3(D / kSM_T, D / kSM_T, BG), 256, 0, stream>>>(A, S, N, out, D);
  return launch_status();
}

}  // namespace bfb

using namespace bfb;

extern "C" {

size_t bf_gdn_segment_workspace(int B, int T, int G, int D) {
  if (B <= 0 || T <= 0 || G <= 0 || D != 256) return 0;
  return al1k_sp((size_t)B * T * G * D * 4) + gdn_prefill_workspace(B, G, T, true);
}

int bf_gdn_segment_transform(const void* k, int k_dtype, const void* v, int v_dtype, const float* g,
                             const float* beta, const float* s0, float* m_out, float* n_out, int B, int T, int G,
                             int D, void* ws, size_t ws_bytes, bf_stream_t stream) {
  if (!k || !v || !g || !beta || !m_out || !n_out || !ws) return BF_ERR_INVALID_ARGUMENT;
  if (B <= 0 || T <= 0 || G <= 0) return BF_ERR_INVALID_ARGUMENT;
  if (D != 256) return BF_ERR_UNSUPPORTED;
  if ((k_dtype != BF_F32 && k_dtype != BF_BF16) || (v_dtype != BF_F32 && v_dtype != BF_BF16))
    return BF_ERR_INVALID_ARGUMENT;
  if (ws_bytes < bf_gdn_segment_workspace(B, T, G, D)) return BF_ERR_WORKSPACE;
  if (!aligned16(k) || !aligned16(v) || !aligned16(m_out) || !aligned16(n_out) || !aligned16(ws) ||
      (s0 && !aligned16(s0)))
    return BF_ERR_ALIGNMENT;
  if ((long long)B * G > 65535) return BF_ERR_UNSUPPORTED;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  uint8_t* p = static_cast<uint8_t*>(ws);
  const float* kf = static_cast<const float*>(k);
  if (k_dtype == BF_BF16) {
    float* k32 = reinterpret_cast<float*>(p);
    const size_t nk = (size_t)B * T * G * D;
    sp_bf16_to_f32_kernel<<<1184, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(k), k32, nk);
    if (int e_ = launch_status()) return e_;
    kf = k32;
  }
  p += al1k_sp((size_t)B * T * G * D * 4);
  GdnStreams s{};
  s.B = B; s.G = G; s.R = 1; s.T = T;
  s.n_steps = T;
  s.n_chunks = (T + kGC - 1) / kGC;
  s.n_pad = s.n_chunks * kGC;
  s.nring = 0; s.W = 1; s.qoff = 0; s.ring_pos0 = 0;
  s.km = kf;
  if (v_dtype == BF_BF16) s.v = static_cast<const __nv_bfloat16*>(v);
  else s.v32 = static_cast<const float*>(v);
  s.g = g; s.beta = beta;
  s.s0 = s0; s.s_out = n_out; s.m_out = m_out;
  s.err = st.err;
  gdn_prefill_carve(s, p);
  return launch_gdn_prefill(s, stream, kGdnAll);
}

int bf_gdn_apply_prefix(const float* M, const float* N, int n_seg, const float* s0, float* s_in, int B, int G, int D,
                        bf_stream_t stream) {
  if (!s_in || n_seg < 0 || (n_seg > 0 && (!M || !N)) || B <= 0 || G <= 0) return BF_ERR_INVALID_ARGUMENT;
  if (D <= 0 || D % kSM_T) return BF_ERR_UNSUPPORTED;
  if ((n_seg > 0 && (!aligned16(M) || !aligned16(N))) || !aligned16(s_in) || (s0 && !aligned16(s0)))
    return BF_ERR_ALIGNMENT;
  if ((long long)B * G > 65535) return BF_ERR_UNSUPPORTED;
  const size_t mat = (size_t)B * G * D * D;
  if (s0) {
    if (cudaMemcpyAsync(s_in, s0, mat * 4, cudaMemcpyDeviceToDevice, stream) != cudaSuccess) return cuda_fail();
  } else {
    if (cudaMemsetAsync(s_in, 0, mat * 4, stream) != cudaSuccess) return cuda_fail();
  }
  for (int j = 0; j < n_seg; ++j)
    state_map_kernel<<<dim3(D / kSM_T, D / kSM_T, B * G), 256, 0, stream>>>(M + j * mat, s_in + j * mat, N + j * mat,
                                                                          s_in + (j + 1) * mat, D);
  return launch_status();
}

}  // extern "C"
