// Recurrent gated delta-rule step (decode), GQA-native: one state per KV head, read by R query heads.
//
// Replaces heimdall/kernels.py:132-138 (delta_rule_step) and the inline decode update at
// heimdall/hibrit.py:398-403:
//   S <- a S (a = e^g);  delta = (v - S^T k) beta;  S <- S + k delta^T;  o_r = S^T q_r.
// Because o_r = (aS)^T q_r + delta (k . q_r), the state is read once and written once:
// one pass computes (aS)^T k and (aS)^T q_r together, the rank-1 update is applied in registers and
// the new state is stored.  HBM traffic per (sequence, KV head) = 2 * D*D*4 bytes (+ vectors).
//
// Work split: columns of S (the Dv axis) are independent, so a CTA owns a 32-column block of one
// (sequence, KV head) state; 256 threads = 8 column quads x 32 row groups; each thread keeps
// D/32 rows x 4 columns of S in registers.  Loads/stores are float4 and each warp touches 4 full
// 128-byte row segments per instruction.
#include "common.cuh"

namespace bfb {

constexpr int kDecCols = 32;     // columns of S per CTA
constexpr int kDecThreads = 256;
constexpr int kDecMaxR = 8;

__global__ void __launch_bounds__(kDecThreads) gdn_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const void* __restrict__ v, int v_bf16,
    const float* __restrict__ g, const float* __restrict__ beta, const float* s_in, float* s_out,
    float* __restrict__ o, int G, int R, int D) {
  const int bg = blockIdx.y;             // (sequence, KV head)
  const int col0 = blockIdx.x * kDecCols;
  const int t = threadIdx.x;
  const int cq = t & 7;                  // column quad within the block
  const int rg = t >> 3;                 // row group 0..31
  const int lane = t & 31, warp = t >> 5;
  const int nrow = D >> 5;               // rows per thread

  __shared__ float sk[256];
  __shared__ float sq[kDecMaxR][256];
  __shared__ float red[8][kDecMaxR + 1][kDecCols];   // per-warp partial column sums
  __shared__ float kq[kDecMaxR];
  __shared__ float delta_s[kDecCols];

  const float* kp = k + (size_t)bg * D;
  const float* qp = q + (size_t)bg * R * D;
  for (int i = t; i < D; i += kDecThreads) sk[i] = kp[i];
  for (int i = t; i < R * D; i += kDecThreads) sq[i / D][i % D] = qp[i];
  __syncthreads();

  const float a = __expf(g[bg]);
  const float bt = beta[bg];
  const float* S = s_in + (size_t)bg * D * D;
  float* So = s_out + (size_t)bg * D * D;

  float4 s[8];
  float pk[4] = {0.f, 0.f, 0.f, 0.f};
  float pq[kDecMaxR][4];
#pragma unroll
  for (int r = 0; r < kDecMaxR; ++r) pq[r][0] = pq[r][1] = pq[r][2] = pq[r][3] = 0.f;

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < nrow) {
      const int row = rg + 32 * i;
      float4 x = *reinterpret_cast<const float4*>(S + (size_t)row * D + col0 + cq * 4);
      x.x *= a; x.y *= a; x.z *= a; x.w *= a;
      s[i] = x;
      const float kr = sk[row];
      pk[0] += kr * x.x; pk[1] += kr * x.y; pk[2] += kr * x.z; pk[3] += kr * x.w;
#pragma unroll
      for (int r = 0; r < kDecMaxR; ++r) {
        if (r < R) {
          const float qr = sq[r][row];
          pq[r][0] += qr * x.x; pq[r][1] += qr * x.y; pq[r][2] += qr * x.z; pq[r][3] += qr * x.w;
        }
      }
    }
  }
  // reduce over the 4 row groups sharing this column quad inside the warp (lanes l, l^8, l^16, l^24)
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    pk[c] += __shfl_xor_sync(0xffffffffu, pk[c], 8);
    pk[c] += __shfl_xor_sync(0xffffffffu, pk[c], 16);
#pragma unroll
    for (int r = 0; r < kDecMaxR; ++r) {
      pq[r][c] += __shfl_xor_sync(0xffffffffu, pq[r][c], 8);
      pq[r][c] += __shfl_xor_sync(0xffffffffu, pq[r][c], 16);
    }
  }
  if (lane < 8) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      red[warp][0][cq * 4 + c] = pk[c];
#pragma unroll
      for (int r = 0; r < kDecMaxR; ++r)
        if (r < R) red[warp][r + 1][cq * 4 + c] = pq[r][c];
    }
  }
  // k . q_r (same for every column block; warp r computes head r)
  if (warp < R) {
    float acc = 0.f;
    for (int i = lane; i < D; i += 32) acc += sk[i] * sq[warp][i];
    acc = warp_sum(acc);
    if (lane == 0) kq[warp] = acc;
  }
  __syncthreads();
  // finish the column sums: thread (quantity j, column c) over the 8 warps
  for (int idx = t; idx < (R + 1) * kDecCols; idx += kDecThreads) {
    const int j = idx / kDecCols, c = idx % kDecCols;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) acc += red[w][j][c];
    red[0][j][c] = acc;
  }
  __syncthreads();
  if (t < kDecCols) {
    const int col = col0 + t;
    float vv;
    if (v_bf16) {
      vv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(v)[(size_t)bg * D + col]);
    } else {
      vv = reinterpret_cast<const float*>(v)[(size_t)bg * D + col];
    }
    delta_s[t] = (vv - red[0][0][t]) * bt;
  }
  __syncthreads();
  // outputs o_r[col] = (aS)^T q_r + delta * (k . q_r)
  for (int idx = t; idx < R * kDecCols; idx += kDecThreads) {
    const int r = idx / kDecCols, c = idx % kDecCols;
    o[((size_t)bg * R + r) * D + col0 + c] = red[0][r + 1][c] + delta_s[c] * kq[r];
  }
  // rank-1 update in registers and store
  float d4[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) d4[c] = delta_s[cq * 4 + c];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < nrow) {
      const int row = rg + 32 * i;
      const float kr = sk[row];
      float4 x = s[i];
      x.x += kr * d4[0]; x.y += kr * d4[1]; x.z += kr * d4[2]; x.w += kr * d4[3];
      *reinterpret_cast<float4*>(So + (size_t)row * D + col0 + cq * 4) = x;
    }
  }
}

int launch_gdn_decode(const float* q, const float* k, const void* v, int v_bf16, const float* g,
                      const float* beta, const float* s_in, float* s_out, float* o, int B, int G, int R, int D,
                      cudaStream_t stream) {
  dim3 grid(D / kDecCols, B * G);
  gdn_decode_kernel<<<grid, kDecThreads, 0, stream>>>(q, k, v, v_bf16, g, beta, s_in, s_out, o, G, R, D);
  return cudaGetLastError() == cudaSuccess ? BF_OK : BF_ERR_CUDA;
}

}  // namespace bfb
