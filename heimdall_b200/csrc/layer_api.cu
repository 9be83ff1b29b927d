// C ABI: layer-level entry points (weight preparation, memory inputs, fused decode step).
// Host-side orchestration only: validation, workspace carving, launch order on the caller's stream.
#include "capi_internal.h"
#include "common.cuh"

namespace bfb {

int launch_prep_weights(const float* fq, const float* fk, const float* ab_w, const float* mix_w, int H, int G,
                        int D, int d, __half* w_heads, __nv_bfloat16* w_x, cudaStream_t stream);
int launch_head_proj(const __nv_bfloat16* q, const __nv_bfloat16* k, const __half* w_heads, float* qm, __half* qm16,
                     float* km, int B, int T, int H, int G, int sm_count, unsigned int* err, cudaStream_t stream);
int launch_x_proj(const __nv_bfloat16* x, const __nv_bfloat16* w_x, const float* ab_b, const float* mix_b,
                  const float* A_log, const float* dt_bias, const float* decay_mask, float* g, float* beta,
                  float* mixx, const int64_t* pos, long long pos0, int M, int T, int d, int G, int H, int sinks,
                  float* scratch, size_t scratch_bytes, unsigned int* err, cudaStream_t stream);

size_t win_dec_workspace(int B, int G, int R, int D, int W);
size_t x_proj_scratch_bytes(int M, int d);
int launch_gather_evicted(const float* ring_km, const __nv_bfloat16* ring_v, const float* ring_g,
                          const float* ring_beta, const int64_t* ring_pos, long long ring_pos_bstride,
                          const int64_t* pos, int B, int G, int W, int D, float* k_e, float* v_e, float* g_e,
                          float* b_e, cudaStream_t stream);

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t weights_heads_bytes(int H, int G, int D) { return align_up((size_t)(H + G) * D * D * 2, 1024); }

const __half* weights_heads(const void* wbuf) { return static_cast<const __half*>(wbuf); }
const __nv_bfloat16* weights_x(const void* wbuf, int H, int G, int D) {
  return reinterpret_cast<const __nv_bfloat16*>(static_cast<const uint8_t*>(wbuf) + weights_heads_bytes(H, G, D));
}

int check_layer(const bf_layer* L) {
  if (!L || !L->wbuf || !L->ab_b || !L->mix_b || !L->mix_lse || !L->mem_scale || !L->A_log || !L->dt_bias ||
      !L->decay_mask)
    return BF_ERR_INVALID_ARGUMENT;
  if (L->H <= 0 || L->G <= 0 || L->H % L->G || L->H / L->G > 8 || L->window <= 0 || L->sinks < 0)
    return BF_ERR_INVALID_ARGUMENT;
  if (L->D != 256) return BF_ERR_UNSUPPORTED;
  if (L->d <= 0 || L->d % 64) return BF_ERR_UNSUPPORTED;
  if (2 * L->G + L->H > 32) return BF_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(L->wbuf) & 1023u) != 0) return BF_ERR_ALIGNMENT;
  return BF_OK;
}

// `scratch` (nullable): device memory the small-row x projection may use for its split-K partials
int mem_inputs_impl(const DeviceState& st, const bf_layer* L, const void* x, const void* q, const void* k,
                    const int64_t* pos, long long pos0, int B, int T, float* qm, float* km, float* g, float* beta,
                    float* mixx, cudaStream_t stream, __half* qm16, float* scratch, size_t scratch_bytes) {
  stage_mark(ST_XPROJ, 0, stream);
  int rc = launch_x_proj(static_cast<const __nv_bfloat16*>(x), weights_x(L->wbuf, L->H, L->G, L->D), L->ab_b,
                         L->mix_b, L->A_log, L->dt_bias, L->decay_mask, g, beta, mixx, pos, pos0, B * T, T, L->d,
                         L->G, L->H, L->sinks, scratch, scratch_bytes, st.err, stream);
  if (rc) return rc;
  stage_mark(ST_XPROJ, 1, stream);
  stage_mark(ST_HEADPROJ, 0, stream);
  // the projection is per token and [B,T,heads,D] is token-contiguous: one flat run of B*T tokens
  rc = launch_head_proj(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                        weights_heads(L->wbuf), qm, qm16, km, 1, B * T, L->H, L->G, st.sm_count, st.err, stream);
  stage_mark(ST_HEADPROJ, 1, stream);
  return rc;
}

}  // namespace bfb

// the argument block of the decode window kernels (definition shared with window_decode.cu)
#include "window_decode_args.h"

namespace bfb {
int launch_win_dec(WinDecArgs a, cudaStream_t stream);
int launch_win_dec_split(WinDecArgs a, cudaStream_t stream, int max_ctas);
int launch_win_dec_combine(WinDecArgs a, cudaStream_t stream);
int win_dec_check(WinDecArgs& a);
int win_dec_split_items(const WinDecArgs& a);
}

using namespace bfb;

extern "C" {

size_t bf_layer_weights_bytes(int H, int G, int D, int d) {
  return weights_heads_bytes(H, G, D) + align_up((size_t)64 * d * 2, 1024);
}

int bf_prepare_layer_weights(const float* fq, const float* fk, const float* ab_w, const float* mix_w, int H, int G,
                             int D, int d, void* wbuf, size_t wbytes, bf_stream_t stream) {
  if (!fq || !fk || !ab_w || !mix_w || !wbuf) return BF_ERR_INVALID_ARGUMENT;
  if (H <= 0 || G <= 0 || d <= 0) return BF_ERR_INVALID_ARGUMENT;
  if (D != 256) return BF_ERR_UNSUPPORTED;
  if (2 * G + H > 32 || d % 64) return BF_ERR_UNSUPPORTED;
  if (wbytes < bf_layer_weights_bytes(H, G, D, d)) return BF_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(wbuf) & 1023u) != 0) return BF_ERR_ALIGNMENT;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  return launch_prep_weights(fq, fk, ab_w, mix_w, H, G, D, d, static_cast<__half*>(wbuf),
                             const_cast<__nv_bfloat16*>(weights_x(wbuf, H, G, D)), stream);
}

int bf_mem_inputs(const bf_layer* L, const void* x, const void* q, const void* k, const int64_t* pos,
                  long long pos0, int B, int T, float* qm, float* km, float* g, float* beta, float* mixx,
                  bf_stream_t stream) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (!x || !q || !k || !qm || !km || !g || !beta || !mixx || B <= 0 || T <= 0) return BF_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(q) || !aligned16(k) || !aligned16(qm) || !aligned16(km)) return BF_ERR_ALIGNMENT;
  if ((long long)B * (L->H + L->G) > 65535 || B > 65535) return BF_ERR_UNSUPPORTED;
  DeviceState st;
  rc = device_state(&st);
  if (rc) return rc;
  return mem_inputs_impl(st, L, x, q, k, pos, pos0, B, T, qm, km, g, beta, mixx, stream, nullptr, nullptr, 0);
}

size_t bf_layer_decode_workspace(int B, int H, int G, int D, int window) {
  const int R = G > 0 ? H / G : 1;
  size_t n = 0;
  n += align_up((size_t)B * H * D * 4, 256);      // qm
  n += align_up((size_t)B * G * D * 4, 256);      // km
  n += align_up((size_t)B * G * 4, 256) * 2;      // g, beta
  n += align_up((size_t)B * H * 4, 256);          // mixx
  n += align_up((size_t)B * G * D * 4, 256) * 2;  // k_e, v_e
  n += align_up((size_t)B * G * 4, 256) * 2;      // g_e, b_e
  n += align_up((size_t)B * H * D * 4, 256);      // o_mem
  n += align_up(win_dec_workspace(B, G, R, D, window), 256);
  n += align_up(x_proj_scratch_bytes(B, 1 << 14), 256);   // split-K partials of the gate projections (d <= 16384)
  return n;
}

int bf_bifrost_layer_decode(const bf_layer* L, const void* x, const void* q, const void* k, const void* v,
                            const void* qr, const void* kr, const int64_t* pos, int B, bf_ring_cache* C,
                            int memory, float* o, float* lse, void* ws, size_t ws_bytes, bf_stream_t stream) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (!x || !q || !k || !v || !qr || !kr || !pos || !C || !o || !ws || B <= 0) return BF_ERR_INVALID_ARGUMENT;
  if (!C->ring_k || !C->ring_v || !C->ring_km || !C->ring_g || !C->ring_beta || !C->ring_pos || !C->S)
    return BF_ERR_INVALID_ARGUMENT;
  if (C->ns < 0 || C->ns > 7 || (C->ns > 0 && (!C->sink_k || !C->sink_v))) return BF_ERR_INVALID_ARGUMENT;
  if (C->ring_pos_bstride != 0 && C->ring_pos_bstride != L->window) return BF_ERR_INVALID_ARGUMENT;
  const int H = L->H, G = L->G, D = L->D, W = L->window, R = H / G;
  if (ws_bytes < bf_layer_decode_workspace(B, H, G, D, W)) return BF_ERR_WORKSPACE;
  if (!aligned16(ws) || !aligned16(C->S) || !aligned16(C->ring_k) || !aligned16(C->ring_v) || !aligned16(x) ||
      !aligned16(q) || !aligned16(k))
    return BF_ERR_ALIGNMENT;
  if ((long long)B * G > 65535) return BF_ERR_UNSUPPORTED;
  DeviceState st;
  rc = device_state(&st);
  if (rc) return rc;

  uint8_t* w = static_cast<uint8_t*>(ws);
  auto take = [&](size_t bytes) {
    uint8_t* p = w;
    w += align_up(bytes, 256);
    return p;
  };
  float* qm = reinterpret_cast<float*>(take((size_t)B * H * D * 4));
  float* km = reinterpret_cast<float*>(take((size_t)B * G * D * 4));
  float* g = reinterpret_cast<float*>(take((size_t)B * G * 4));
  float* beta = reinterpret_cast<float*>(take((size_t)B * G * 4));
  float* mixx = reinterpret_cast<float*>(take((size_t)B * H * 4));
  float* k_e = reinterpret_cast<float*>(take((size_t)B * G * D * 4));
  float* v_e = reinterpret_cast<float*>(take((size_t)B * G * D * 4));
  float* g_e = reinterpret_cast<float*>(take((size_t)B * G * 4));
  float* b_e = reinterpret_cast<float*>(take((size_t)B * G * 4));
  float* o_mem = reinterpret_cast<float*>(take((size_t)B * H * D * 4));
  float* part = reinterpret_cast<float*>(take(win_dec_workspace(B, G, R, D, W)));
  const size_t xs_bytes = x_proj_scratch_bytes(B, 1 << 14);
  float* xs = reinterpret_cast<float*>(take(xs_bytes));

  WinDecArgs a{};
  a.qr = static_cast<const __nv_bfloat16*>(qr);
  a.kr = static_cast<const __nv_bfloat16*>(kr);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.ring_k = static_cast<const __nv_bfloat16*>(C->ring_k);
  a.ring_v = static_cast<const __nv_bfloat16*>(C->ring_v);
  a.ring_pos = C->ring_pos;
  a.ring_pos_bstride = C->ring_pos_bstride;
  a.sink_k = static_cast<const __nv_bfloat16*>(C->sink_k);
  a.sink_v = static_cast<const __nv_bfloat16*>(C->sink_v);
  a.ns = C->ns;
  a.pos = pos;
  a.part = part;
  a.B = B;
  a.G = G;
  a.R = R;
  a.D = D;
  a.W = W;
  a.S = L->sinks;
  a.o_mem = memory ? o_mem : nullptr;
  a.mixx = mixx;
  a.mix_lse = L->mix_lse;
  a.mem_scale = L->mem_scale;
  a.o = o;
  a.lse_out = lse;
  a.km = km;
  a.g_new = g;
  a.beta_new = beta;
  a.ring_k_w = static_cast<__nv_bfloat16*>(C->ring_k);
  a.ring_v_w = static_cast<__nv_bfloat16*>(C->ring_v);
  a.ring_km = C->ring_km;
  a.ring_g = C->ring_g;
  a.ring_beta = C->ring_beta;
  a.ring_pos_w = C->ring_pos;
  if ((rc = win_dec_check(a)) != BF_OK) return rc;

  // The evicted ring entry (read only by the state update) and the gate projections (g, beta and the mix logit
  // of the new tokens, read only by the combine kernel) run on the greatest-priority side stream, the gate
  // projections over their own split-K scratch, beside the head projections.  On the caller's stream: the head
  // projections (qm, km) and the state update (o_mem, S), then the window split over the ring and the combine,
  // which also writes the new token into its ring slot (the slot of the evicted entry, read before by the
  // gather).  The state update and the window
  // split are both HBM-bound persistent kernels that each need the whole GPU to reach their bandwidth (a
  // concurrent run on disjoint SM shares measured slower), so they run one after the other.
  cudaStream_t sx = side_stream(st, 1);
  if (!sx) return cuda_fail();
  struct Events {
    cudaEvent_t e[3] = {nullptr, nullptr, nullptr};
    ~Events() {
      for (cudaEvent_t x : e)
        if (x) cudaEventDestroy(x);
    }
  } evs;
  cudaEvent_t &ev_fork = evs.e[0], &ev_x = evs.e[1], &ev_g = evs.e[2];
  for (cudaEvent_t* e : {&ev_fork, &ev_x, &ev_g})
    if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return cuda_fail();
  if (cudaEventRecord(ev_fork, stream) != cudaSuccess || cudaStreamWaitEvent(sx, ev_fork, 0) != cudaSuccess)
    return cuda_fail();
  if (memory) {
    // the token leaving the window (position p - W) is written into memory before the read; gathered on the
    // side stream, beside the head projections
    stage_mark(ST_DEC_GATHER, 0, sx);
    rc = launch_gather_evicted(C->ring_km, static_cast<const __nv_bfloat16*>(C->ring_v), C->ring_g, C->ring_beta,
                               C->ring_pos, C->ring_pos_bstride, pos, B, G, W, D, k_e, v_e, g_e, b_e, sx);
    if (rc) return rc;
    stage_mark(ST_DEC_GATHER, 1, sx);
    if (cudaEventRecord(ev_g, sx) != cudaSuccess) return cuda_fail();
  }
  stage_mark(ST_XPROJ, 0, sx);
  rc = launch_x_proj(static_cast<const __nv_bfloat16*>(x), weights_x(L->wbuf, L->H, L->G, L->D), L->ab_b, L->mix_b,
                     L->A_log, L->dt_bias, L->decay_mask, g, beta, mixx, pos, 0, B, 1, L->d, L->G, L->H, L->sinks, xs,
                     xs_bytes, st.err, sx);
  if (rc) return rc;
  stage_mark(ST_XPROJ, 1, sx);
  if (cudaEventRecord(ev_x, sx) != cudaSuccess) return cuda_fail();
  stage_mark(ST_HEADPROJ, 0, stream);
  rc = launch_head_proj(static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                        weights_heads(L->wbuf), qm, nullptr, km, 1, B, L->H, L->G, st.sm_count, st.err, stream);
  if (rc) return rc;
  stage_mark(ST_HEADPROJ, 1, stream);
  if (memory) {
    if (cudaStreamWaitEvent(stream, ev_g, 0) != cudaSuccess) return cuda_fail();
    stage_mark(ST_DEC_STATE, 0, stream);
    rc = launch_gdn_decode(qm, k_e, v_e, 0, g_e, b_e, C->S, C->S, o_mem, B, G, R, D, stream);
    if (rc) return rc;
    stage_mark(ST_DEC_STATE, 1, stream);
  }
  stage_mark(ST_DEC_WIN, 0, stream);
  rc = launch_win_dec_split(a, stream, 0);
  if (rc) return rc;
  stage_mark(ST_DEC_WIN, 1, stream);
  if (cudaStreamWaitEvent(stream, ev_x, 0) != cudaSuccess) return cuda_fail();
  stage_mark(ST_DEC_COMBINE, 0, stream);
  rc = launch_win_dec_combine(a, stream);
  stage_mark(ST_DEC_COMBINE, 1, stream);
  return rc;
}

}  // extern "C"
