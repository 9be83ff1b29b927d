// C ABI: chunked delta-rule op, window-attention op and the fused layer prefill.
// Host-side orchestration only: validation, workspace carving, launch order on the caller's stream.
#include "capi_internal.h"
#include "common.cuh"
#include "gdn_prefill.h"
#include "window_prefill.h"

namespace bfb {
size_t gdn_prefill_fix_workspace(int B, int G, int T_steps);
void gdn_prefill_carve_fix(GdnStreams& s, void* ws);
int launch_state_map(const float* A, const float* S, const float* N, float* out, int BG, int D, cudaStream_t stream);

int launch_head_proj(const __nv_bfloat16* q, const __nv_bfloat16* k, const __half* w_heads, float* qm, __half* qm16,
                     float* km, int B, int T, int H, int G, int sm_count, unsigned int* err, cudaStream_t stream);
int mem_inputs_impl(const DeviceState& st, const bf_layer* L, const void* x, const void* q, const void* k,
                    const int64_t* pos, long long pos0, int B, int T, float* qm, float* km, float* g, float* beta,
                    float* mixx, cudaStream_t stream, __half* qm16, float* scratch, size_t scratch_bytes);
int check_layer(const bf_layer* L);
size_t gdn_prefill_workspace(int B, int G, int T_steps, bool transform);
int gdn_prefill_carve(GdnStreams& s, void* ws);
int launch_gdn_prefill(GdnStreams s, cudaStream_t stream, int parts);
int launch_chunk_table(const int* cu_seqlens, int n_seq, int max_chunks, int* seq_chunk0, int* chunk_tok0,
                       int* chunk_len, unsigned int* err, cudaStream_t stream);
int launch_vt_prep(const __nv_bfloat16* v, long long vb, long long vg, long long vj, const __nv_bfloat16* ring_v,
                   int nring, long long ring_pos0, int W, int B, int G, int Tk, int Tkp, __half* vt,
                   cudaStream_t stream);
int launch_kext_prep(const __nv_bfloat16* kr, const __nv_bfloat16* ring_k, int nring, long long ring_pos0, int W, int B,
                     int T, int G, __nv_bfloat16* kext, cudaStream_t stream);
int launch_window_prefill(const void* qr, const void* kext, const __half* vt, WinPreArgs a, cudaStream_t stream);

static size_t al1k(size_t x) { return (x + 1023) & ~size_t(1023); }

// ---------------------------------------------------------------------------------------- small kernels
// q [B,T,H,D] (fp32 or bf16) -> fp16; k bf16 -> fp32
__global__ void to_half_kernel(const void* __restrict__ src, int src_bf16, __half* __restrict__ dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float x = src_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[i])
                             : reinterpret_cast<const float*>(src)[i];
    dst[i] = __float2half_rn(x);
  }
}
__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ src, float* __restrict__ dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __bfloat162float(src[i]);
}
// write the last m new tokens into their ring slots (heimdall/hibrit.py:414-422)
__global__ void ring_write_kernel(const __nv_bfloat16* __restrict__ kr, const __nv_bfloat16* __restrict__ v,
                                  const float* __restrict__ km, const float* __restrict__ g, const float* __restrict__ beta,
                                  long long start, int T, int m, int G, int W, __nv_bfloat16* ring_k, __nv_bfloat16* ring_v,
                                  float* ring_km, float* ring_g, float* ring_beta, int64_t* ring_pos) {
  const int i = T - m + blockIdx.x;
  const int bg = blockIdx.y, b = bg / G, gg = bg % G;
  const long long p = start + i;
  const int slot = (int)(p % W);
  const int c = threadIdx.x * 8;
  *reinterpret_cast<uint4*>(ring_k + (((size_t)b * G + gg) * W + slot) * 256 + c) =
      *reinterpret_cast<const uint4*>(kr + (((size_t)b * G + gg) * T + i) * 256 + c);
  *reinterpret_cast<uint4*>(ring_v + (((size_t)b * G + gg) * W + slot) * 256 + c) =
      *reinterpret_cast<const uint4*>(v + (((size_t)b * T + i) * G + gg) * 256 + c);
  float* kmd = ring_km + (((size_t)b * W + slot) * G + gg) * 256 + c;
  const float* kms = km + (((size_t)b * T + i) * G + gg) * 256 + c;
  *reinterpret_cast<float4*>(kmd) = *reinterpret_cast<const float4*>(kms);
  *reinterpret_cast<float4*>(kmd + 4) = *reinterpret_cast<const float4*>(kms + 4);
  if (threadIdx.x == 0) {
    ring_g[((size_t)b * W + slot) * G + gg] = g[((size_t)b * T + i) * G + gg];
    ring_beta[((size_t)b * W + slot) * G + gg] = beta[((size_t)b * T + i) * G + gg];
    if (bg == 0) ring_pos[slot] = p;
  }
}

static int grid_for(size_t n) {
  size_t g = (n + 255) / 256;
  return (int)(g > 4096 ? 4096 : (g < 1 ? 1 : g));
}

}  // namespace bfb

using namespace bfb;

extern "C" {

// ================================================================================ delta rule op
// packed sequences: at most T / kGC + n_seq chunks (each sequence adds at most one partial chunk)
static int max_chunks_for(int T, int n_seq) { return (T + kGC - 1) / kGC + n_seq; }

size_t bf_gdn_chunk_workspace(int B, int T, int G, int R, int D, int n_seq) {
  if (B <= 0 || T <= 0 || G <= 0 || R <= 0 || D != 256 || n_seq < 0) return 0;
  size_t n = al1k((size_t)B * T * G * R * D * 2) + al1k((size_t)B * T * G * D * 4);
  if (n_seq > 0) {
    const int mc = max_chunks_for(T, n_seq);
    n += al1k((size_t)(n_seq + 1) * 4) + 2 * al1k((size_t)mc * 4);
    return n + gdn_prefill_workspace(1, G, mc * kGC, false);
  }
  return n + gdn_prefill_workspace(B, G, T, false);
}

int bf_gdn_chunk_fwd(const void* q, int q_dtype, const void* k, int k_dtype, const void* v, int v_dtype,
                     const float* g, const float* beta, const float* s0, float* o, float* s_out,
                     const int* cu_seqlens, int n_seq, int B, int T, int G, int R, int D, void* ws, size_t ws_bytes,
                     bf_stream_t stream) {
  if (!q || !k || !v || !g || !beta || !o || !s_out || !ws) return BF_ERR_INVALID_ARGUMENT;
  if (B <= 0 || T <= 0 || G <= 0 || R <= 0 || R > 8) return BF_ERR_INVALID_ARGUMENT;
  if (cu_seqlens ? (n_seq <= 0 || B != 1) : n_seq != 0) return BF_ERR_INVALID_ARGUMENT;
  if (D != 256) return BF_ERR_UNSUPPORTED;
  for (int dt : {q_dtype, k_dtype, v_dtype})
    if (dt != BF_F32 && dt != BF_BF16) return BF_ERR_INVALID_ARGUMENT;
  if (ws_bytes < bf_gdn_chunk_workspace(B, T, G, R, D, n_seq)) return BF_ERR_WORKSPACE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(s_out) || !aligned16(ws) ||
      (s0 && !aligned16(s0)))
    return BF_ERR_ALIGNMENT;
  if ((long long)B * G > 65535 || (long long)G * n_seq > 65535 || (long long)B * T * G * R > (1LL << 40))
    return BF_ERR_UNSUPPORTED;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  uint8_t* p = static_cast<uint8_t*>(ws);
  __half* q16 = reinterpret_cast<__half*>(p);
  p += al1k((size_t)B * T * G * R * D * 2);
  float* k32 = reinterpret_cast<float*>(p);
  p += al1k((size_t)B * T * G * D * 4);
  const size_t nq = (size_t)B * T * G * R * D;
  to_half_kernel<<<grid_for(nq), 256, 0, stream>>>(q, q_dtype == BF_BF16, q16, nq);
  const float* kf = static_cast<const float*>(k);
  if (k_dtype == BF_BF16) {
    const size_t nk = (size_t)B * T * G * D;
    bf16_to_f32_kernel<<<grid_for(nk), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(k), k32, nk);
    kf = k32;
  }
  if (int e_ = launch_status()) return e_;
  GdnStreams s{};
  s.B = B; s.G = G; s.R = R; s.T = T;
  s.n_steps = T;
  s.n_chunks = (T + kGC - 1) / kGC;
  if (cu_seqlens) {
    const int mc = max_chunks_for(T, n_seq);
    int* seq_chunk0 = reinterpret_cast<int*>(p);
    p += al1k((size_t)(n_seq + 1) * 4);
    int* chunk_tok0 = reinterpret_cast<int*>(p);
    p += al1k((size_t)mc * 4);
    int* chunk_len = reinterpret_cast<int*>(p);
    p += al1k((size_t)mc * 4);
    rc = launch_chunk_table(cu_seqlens, n_seq, mc, seq_chunk0, chunk_tok0, chunk_len, st.err, stream);
    if (rc) return rc;
    s.n_chunks = mc;
    s.chunk_tok0 = chunk_tok0;
    s.chunk_len = chunk_len;
    s.seq_chunk0 = seq_chunk0;
    s.n_seq = n_seq;
  }
  s.n_pad = s.n_chunks * kGC;
  s.nring = 0; s.W = 1; s.qoff = 0; s.ring_pos0 = 0;
  s.km = kf;
  if (v_dtype == BF_BF16) s.v = static_cast<const __nv_bfloat16*>(v);
  else s.v32 = static_cast<const float*>(v);
  s.g = g; s.beta = beta;
  s.s0 = s0; s.s_out = s_out;
  s.qm = q16; s.o = o;
  s.err = st.err;
  gdn_prefill_carve(s, p);
  return launch_gdn_prefill(s, stream, kGdnAll);
}

// ================================================================================ window op
size_t bf_window_workspace(int B, int G, int Tk, int D) {
  if (B <= 0 || G <= 0 || Tk <= 0 || D != 256) return 0;
  const size_t Tkp = (size_t)((Tk + 63) / 64) * 64;
  return al1k((size_t)B * G * D * Tkp * 2);
}

static int window_common(const void* qr, const void* k_ext, const __half* vt, const void* sink_k, const void* sink_v,
                         int ns, long long qpos0, long long kpos0, long long klo, int B, int H, int G, int Tq, int Tk,
                         int window, float* o, float* lse, unsigned int* err, cudaStream_t stream,
                         __half* o_perm = nullptr, int perm_tile0 = 0, int perm_nch = 0, int qt0 = 0, int nqt = 0) {
  WinPreArgs a{};
  a.B = B; a.H = H; a.G = G; a.Tq = Tq; a.Tk = Tk; a.Tkp = ((Tk + 63) / 64) * 64; a.W = window;
  a.qpos0 = qpos0; a.kpos0 = kpos0; a.klo = klo;
  a.sink_k = static_cast<const __nv_bfloat16*>(sink_k);
  a.sink_v = static_cast<const __nv_bfloat16*>(sink_v);
  a.ns = ns;
  a.sk_b = (long long)G * ns * 256; a.sk_h = (long long)ns * 256; a.sk_k = 256;
  a.sv_b = a.sk_b; a.sv_h = a.sk_h; a.sv_k = 256;
  a.o = o; a.lse = lse;
  a.o_perm = o_perm; a.perm_tile0 = perm_tile0; a.perm_nch = perm_nch;
  a.qt0 = qt0; a.nqt = nqt;
  a.err = err;
  return launch_window_prefill(qr, k_ext, vt, a, stream);
}

int bf_window_attn_fwd(const void* qr, const void* k_ext, const void* v_ext, long long vb, long long vg, long long vj,
                       const void* sink_k, const void* sink_v, int ns, long long qpos0, long long kpos0, long long klo,
                       int B, int H, int G, int Tq, int Tk, int D, int window, float* o, float* lse, void* ws,
                       size_t ws_bytes, bf_stream_t stream) {
  if (!qr || !k_ext || !v_ext || !o || !ws) return BF_ERR_INVALID_ARGUMENT;
  if (B <= 0 || H <= 0 || G <= 0 || H % G || H / G > 8 || Tq <= 0 || Tk <= 0 || window <= 0 || ns < 0 || ns > 8)
    return BF_ERR_INVALID_ARGUMENT;
  if (ns > 0 && (!sink_k || !sink_v)) return BF_ERR_INVALID_ARGUMENT;
  if (D != 256) return BF_ERR_UNSUPPORTED;
  if (ws_bytes < bf_window_workspace(B, G, Tk, D)) return BF_ERR_WORKSPACE;
  if (!aligned16(qr) || !aligned16(k_ext) || !aligned16(v_ext) || !aligned16(o) || !aligned16(ws) ||
      (ns && (!aligned16(sink_k) || !aligned16(sink_v))) || (vj % 8) || (vg % 8) || (vb % 8))
    return BF_ERR_ALIGNMENT;
  if ((long long)B * H > 65535 || B > 65535) return BF_ERR_UNSUPPORTED;
  DeviceState st;
  int rc = device_state(&st);
  if (rc) return rc;
  const int Tkp = ((Tk + 63) / 64) * 64;
  __half* vt = static_cast<__half*>(ws);
  rc = launch_vt_prep(static_cast<const __nv_bfloat16*>(v_ext), vb, vg, vj, nullptr, 0, 0, 1, B, G, Tk, Tkp, vt, stream);
  if (rc) return rc;
  return window_common(qr, k_ext, vt, sink_k, sink_v, ns, qpos0, kpos0, klo, B, H, G, Tq, Tk, window, o, lse, st.err,
                       stream);
}

// ================================================================================ fused layer prefill
size_t bf_layer_prefill_workspace(int B, int T, int H, int G, int D, int window, int with_ring) {
  if (B <= 0 || T <= 0 || H <= 0 || G <= 0 || D != 256 || window <= 0) return 0;
  const size_t Tk = (size_t)T + (with_ring ? window : 0);
  const size_t Tkp = (Tk + 63) / 64 * 64;
  const int steps = with_ring ? T : (T > window ? T - window : 1);
  size_t n = 0;
  n += al1k((size_t)B * T * H * D * 2);     // qm16
  n += al1k((size_t)B * T * G * D * 4);     // km
  n += al1k((size_t)B * T * G * 4) * 2;     // g, beta
  n += al1k((size_t)B * T * H * 4);         // mixx
  n += al1k((size_t)B * H * T * 4);         // window lse (for the gate) when the caller does not keep it
  n += al1k((size_t)B * G * D * D * 4);     // state when there is no cache
  n += al1k((size_t)B * G * D * Tkp * 2);   // V^T
  if (with_ring) n += al1k((size_t)B * G * Tk * D * 2);  // K of the extended sequence
  n += gdn_prefill_workspace(B, G, steps, false);
  n += al1k((size_t)B * ((steps + 127) / 128) * H * 128 * D * 2);   // window results of the mixed rows (fp16), tile order
  return n;
}

// the two-phase (sequence-parallel) prefill's extra workspace: the fix-up buffers and a state for the final
// state M S_in + N
static size_t sp_extra_bytes(int B, int T, int G, int D, int window, int with_ring) {
  const int steps = with_ring ? T : (T > window ? T - window : 1);
  return gdn_prefill_fix_workspace(B, G, steps) + al1k((size_t)B * G * D * D * 4);
}

// The window of a whole-layer prefill with memory reads runs as up to kWinPieces launches over consecutive ranges of
// query tiles, alternating between two least-priority streams so that each launch's CTAs fill the previous one's
// tail; the memory reads of the chunks a piece covers start as soon as that piece (and the state scan) is done,
// beside the next pieces, so only the last piece's reads remain after the window.
constexpr int kWinPieces = 4;
constexpr int kWinPieceMinChunks = 16;   // fewer chunks per piece than this: fewer pieces

// phase: kPhaseAll (the whole layer), kPhaseBegin (memory inputs, P1 and the segment state map -> m_out, n_out),
// kPhaseFinish (the rest, from C->S, reusing the workspace of the begin phase)
constexpr int kPhaseAll = 0, kPhaseBegin = 1, kPhaseFinish = 2;

__global__ void identity_maps_kernel(float* m, float* n, int BG, int D) {
  const size_t total = (size_t)BG * D * D;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e = i % ((size_t)D * D);
    m[i] = (e / D == e % D) ? 1.f : 0.f;
    n[i] = 0.f;
  }
}

static int layer_prefill_impl(const bf_layer* L, const void* x, const void* q, const void* k, const void* v,
                              const void* qr, const void* kr, long long start, int B, int T, bf_ring_cache* C,
                              const void* sink_k, const void* sink_v, int ns, int memory, float* o, float* lse,
                              void* ws, size_t ws_bytes, cudaStream_t stream, int phase, float* m_out,
                              float* n_out) {
  int rc = check_layer(L);
  if (rc) return rc;
  if (!x || !q || !k || !v || !qr || !kr || !o || !ws || B <= 0 || T <= 0 || start < 0) return BF_ERR_INVALID_ARGUMENT;
  if (ns < 0 || ns > 8 || (ns > 0 && (!sink_k || !sink_v))) return BF_ERR_INVALID_ARGUMENT;
  const int H = L->H, G = L->G, D = L->D, W = L->window, R = H / G;
  const bool ring_case = C != nullptr && start > 0;
  if (C && (!C->ring_k || !C->ring_v || !C->ring_km || !C->ring_g || !C->ring_beta || !C->ring_pos || !C->S))
    return BF_ERR_INVALID_ARGUMENT;
  if (C && C->ring_pos_bstride != 0) return BF_ERR_UNSUPPORTED;
  const size_t ws_base = bf_layer_prefill_workspace(B, T, H, G, D, W, ring_case ? 1 : 0);
  const bool two_phase = phase != kPhaseAll;
  if (ws_bytes < ws_base + (two_phase ? sp_extra_bytes(B, T, G, D, W, ring_case ? 1 : 0) : 0)) return BF_ERR_WORKSPACE;
  if (phase == kPhaseFinish && (!m_out || !n_out)) return BF_ERR_INVALID_ARGUMENT;
  for (const void* pp : {x, q, k, v, qr, kr, (const void*)o, (const void*)ws})
    if (!aligned16(pp)) return BF_ERR_ALIGNMENT;
  if (ns && (!aligned16(sink_k) || !aligned16(sink_v))) return BF_ERR_ALIGNMENT;
  if ((long long)B * (H + G) > 65535) return BF_ERR_UNSUPPORTED;
  DeviceState st;
  rc = device_state(&st);
  if (rc) return rc;

  const bool use_mem = memory && start + T > W;
  const int Tk = T + (ring_case ? W : 0);
  const int Tkp = ((Tk + 63) / 64) * 64;
  uint8_t* p = static_cast<uint8_t*>(ws);
  auto take = [&](size_t bytes) {
    uint8_t* r = p;
    p += al1k(bytes);
    return r;
  };
  __half* qm16 = reinterpret_cast<__half*>(take((size_t)B * T * H * D * 2));
  float* km = reinterpret_cast<float*>(take((size_t)B * T * G * D * 4));
  float* g = reinterpret_cast<float*>(take((size_t)B * T * G * 4));
  float* beta = reinterpret_cast<float*>(take((size_t)B * T * G * 4));
  float* mixx = reinterpret_cast<float*>(take((size_t)B * T * H * 4));
  float* lse_ws = reinterpret_cast<float*>(take((size_t)B * H * T * 4));
  float* s_tmp = reinterpret_cast<float*>(take((size_t)B * G * D * D * 4));
  __half* vt = reinterpret_cast<__half*>(take((size_t)B * G * D * Tkp * 2));
  __nv_bfloat16* kext = ring_case ? reinterpret_cast<__nv_bfloat16*>(take((size_t)B * G * Tk * D * 2)) : nullptr;
  void* gws = p;
  float* lse_w = lse ? lse : lse_ws;   // the window's lse, needed by the gate

  // the window (step 3) depends only on the inputs: when there are memory reads to overlap with, the window
  // and the memory chain (steps 1-2) run on two side streams forked here and joined before the reads mix
  // into o.  The chain's stream has the greater priority, so its CTAs (the sequential scan among them, which
  // fills only part of the GPU) are dispatched first and the window's CTAs fill the remaining SMs.
  // Sequence-parallel phases: the window is launched in the first phase and left running on its side stream
  // (it overlaps the state-map scan and the caller's exchange of the maps); the second phase joins it before
  // the reads.  The buffers it uses are the caller's inputs, output and workspace, held until that phase.
  const bool reads_later = use_mem && (ring_case ? T : T - W) > 0;
  const bool will_read = reads_later && phase != kPhaseFinish;   // fork the window and the chain here
  const bool win_here = phase == kPhaseAll || (phase == kPhaseBegin) == reads_later;
  cudaStream_t ws2 = stream;   // (a null handle is the legacy default stream, a valid stream)
  cudaStream_t wsm = stream;   // the memory chain
  // the fork/join events are released when the call returns, on every path (an event recorded for work still
  // in flight may be destroyed: the release is deferred until that work completes)
  struct Events {
    cudaEvent_t fork = nullptr, win = nullptr, mem = nullptr, vt = nullptr, p1 = nullptr, piece[kWinPieces] = {};
    ~Events() {
      for (cudaEvent_t e : {fork, win, mem, vt, p1})
        if (e) cudaEventDestroy(e);
      for (cudaEvent_t e : piece)
        if (e) cudaEventDestroy(e);
    }
  } evs;
  cudaEvent_t& ev_fork = evs.fork;
  cudaEvent_t& ev_win = evs.win;
  cudaEvent_t& ev_mem = evs.mem;
  if (reads_later && phase == kPhaseFinish) {
    // the scan from the incoming state goes on the high-priority stream too, ahead of the window's CTAs
    // still waiting for SMs; it is joined before the reads
    wsm = side_stream(st, 1);
    if (!wsm || cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_mem, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventRecord(ev_fork, stream) != cudaSuccess || cudaStreamWaitEvent(wsm, ev_fork, 0) != cudaSuccess)
      return cuda_fail();
  }
  if (will_read) {
    ws2 = side_stream(st, 0);
    wsm = side_stream(st, 1);
    if (!ws2 || !wsm) return cuda_fail();
    if (cudaEventCreateWithFlags(&ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_win, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_mem, cudaEventDisableTiming) != cudaSuccess)
      return cuda_fail();
    if (cudaEventRecord(ev_fork, stream) != cudaSuccess || cudaStreamWaitEvent(wsm, ev_fork, 0) != cudaSuccess ||
        cudaStreamWaitEvent(ws2, ev_fork, 0) != cudaSuccess)
      return cuda_fail();
  }
  // 1. memory inputs (projections on tcgen05)
  if ((use_mem || C) && phase != kPhaseFinish) {
    rc = mem_inputs_impl(st, L, x, q, k, nullptr, start, B, T, nullptr, km, g, beta, mixx, wsm, qm16, nullptr, 0);
    if (rc) return rc;
  }
  // 2. memory: the write stream is delayed by W (token i enters memory when it leaves the window)
  GdnStreams s{};
  bool reads = false;
  if (use_mem) {
    s.B = B; s.G = G; s.R = R; s.T = T; s.W = W;
    if (ring_case) {
      s.nring = W; s.qoff = 0; s.n_steps = T; s.ring_pos0 = start - W;
      s.ring_km = C->ring_km;
      s.ring_v = static_cast<const __nv_bfloat16*>(C->ring_v);
      s.ring_g = C->ring_g; s.ring_beta = C->ring_beta; s.ring_pos = C->ring_pos;
      s.s0 = C->S;
    } else {
      // no history: the first W write steps are no-ops, so queries before W read the zero state (their gate
      // is off: they keep the window result)
      s.nring = 0; s.qoff = W; s.n_steps = T - W; s.ring_pos0 = 0;
      s.s0 = nullptr;
    }
    s.n_chunks = (s.n_steps + kGC - 1) / kGC;
    s.n_pad = s.n_chunks * kGC;
    s.km = km; s.v = static_cast<const __nv_bfloat16*>(v); s.g = g; s.beta = beta;
    s.s_out = C ? C->S : s_tmp;
    s.qm = qm16; s.err = st.err;
    // the memory reads go straight into the layer output, mixed with the window result there
    s.o = o; s.mix = 1; s.pos0 = start; s.lse = lse_w; s.mixx = mixx; s.mix_lse = L->mix_lse;
    s.mem_scale = L->mem_scale;
    if (phase == kPhaseBegin) {   // the state map of this segment's write stream, from a zero state
      s.s0 = nullptr;
      s.s_out = n_out;
      s.m_out = m_out;
    }
    if (s.n_steps > 0) {
      uint8_t* extra = static_cast<uint8_t*>(ws) + ws_base;   // the two-phase buffers follow the layer's workspace
      if (two_phase) gdn_prefill_carve_fix(s, extra);
      gdn_prefill_carve(s, gws);
      // the window writes the rows the reads cover in tile order when its query tiles line up with the chunks
      if (s.qoff % kGC == 0 && reads_later) {
        s.owin = reinterpret_cast<__half*>(static_cast<uint8_t*>(gws) + al1k(gdn_prefill_workspace(B, G, s.n_steps, false)));
      }
      reads = phase != kPhaseBegin;
      // the second phase does not scan again: the fix-up turns the map pass's per-chunk states from a zero
      // incoming state and per-chunk transitions into the states from C->S (all chunks at once), and the
      // cache's final state is M S_in + N in fp32
      // (without an incoming state, as on the first segment, the map pass's values are final already)
      const int parts = phase == kPhaseBegin ? (kGdnP1 | kGdnP2)
                        : phase == kPhaseFinish ? (s.s0 ? kGdnFix : 0)
                                                : (kGdnP1 | kGdnP2);
      if (phase == kPhaseBegin && will_read && win_here && (parts & kGdnP1)) {
        // sequence-parallel first phase: the window starts once P1 is done, so the projections and P1 have the
        // whole GPU and the window's CTAs fill the SMs that the latency-bound map scan leaves idle
        rc = launch_gdn_prefill(s, wsm, kGdnP1);
        if (rc) return rc;
        if (cudaEventCreateWithFlags(&evs.p1, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventRecord(evs.p1, wsm) != cudaSuccess || cudaStreamWaitEvent(ws2, evs.p1, 0) != cudaSuccess)
          return cuda_fail();
        rc = launch_gdn_prefill(s, wsm, parts & ~kGdnP1);
      } else {
        rc = launch_gdn_prefill(s, wsm, parts);
      }
      if (rc) return rc;
      if (phase == kPhaseFinish) {
        float* s_fin = reinterpret_cast<float*>(extra + gdn_prefill_fix_workspace(B, G, s.n_steps));
        rc = launch_state_map(m_out, C->S, n_out, s_fin, B * G, D, wsm);
        if (!rc && cudaMemcpyAsync(C->S, s_fin, (size_t)B * G * D * D * 4, cudaMemcpyDeviceToDevice, wsm) != cudaSuccess)
          rc = cuda_fail();
        if (rc) return rc;
      }
    } else if (phase == kPhaseBegin) {
      identity_maps_kernel<<<grid_for((size_t)B * G * D * D), 256, 0, stream>>>(m_out, n_out, B * G, D);
      if (int e_ = launch_status()) return e_;
    }
  } else if (phase == kPhaseBegin) {
    identity_maps_kernel<<<grid_for((size_t)B * G * D * D), 256, 0, stream>>>(m_out, n_out, B * G, D);
    if (int e_ = launch_status()) return e_;
  }
  if (phase == kPhaseBegin && will_read) {   // the maps are complete when this call returns, the window not
    if (cudaEventRecord(ev_mem, wsm) != cudaSuccess || cudaStreamWaitEvent(stream, ev_mem, 0) != cudaSuccess)
      return cuda_fail();
  }
  if (!win_here) {
    if (phase == kPhaseFinish && reads_later) {   // join the scan and the window launched by the first phase
      cudaStream_t wsw = side_stream(st, 0);
      if (!wsw || cudaEventCreateWithFlags(&ev_win, cudaEventDisableTiming) != cudaSuccess ||
          cudaEventRecord(ev_win, wsw) != cudaSuccess || cudaStreamWaitEvent(stream, ev_win, 0) != cudaSuccess ||
          cudaEventRecord(ev_mem, wsm) != cudaSuccess || cudaStreamWaitEvent(stream, ev_mem, 0) != cudaSuccess)
        return cuda_fail();
    }
    if (phase == kPhaseBegin) return BF_OK;
  }
  // 3. window attention over the extended keys (o = window result, lse), on the side stream when forked
  const void* kx = kr;
  int n_pieces = 1, piece_c0[kWinPieces] = {}, piece_c1[kWinPieces] = {};
  if (win_here) {
    stage_mark(ST_WIN_PREP, 0, ws2);
    if (ring_case) {
      rc = launch_kext_prep(static_cast<const __nv_bfloat16*>(kr), static_cast<const __nv_bfloat16*>(C->ring_k), W,
                            start - W, W, B, T, G, kext, ws2);
      if (rc) return rc;
      kx = kext;
    }
    rc = launch_vt_prep(static_cast<const __nv_bfloat16*>(v), (long long)T * G * D, D, (long long)G * D,
                        ring_case ? static_cast<const __nv_bfloat16*>(C->ring_v) : nullptr, ring_case ? W : 0,
                        start - W, W, B, G, Tk, Tkp, vt, ws2);
    if (rc) return rc;
    stage_mark(ST_WIN_PREP, 1, ws2);
    stage_mark(ST_WIN, 0, ws2);
    const long long kpos0 = ring_case ? start - W : start;
    __half* owp = reads_later ? const_cast<__half*>(s.owin) : nullptr;
    const int ptile0 = s.qoff / kGC, ntq = (T + kGC - 1) / kGC;
    n_pieces = (phase == kPhaseAll && will_read && owp) ? s.n_chunks / kWinPieceMinChunks : 1;
    n_pieces = n_pieces < 1 ? 1 : (n_pieces > kWinPieces ? kWinPieces : n_pieces);
    if (n_pieces == 1) {
      rc = window_common(qr, kx, vt, sink_k, sink_v, ns, start, kpos0, L->sinks, B, H, G, T, Tk, W, o, lse_w, st.err,
                         ws2, owp, ptile0, s.n_chunks);
      if (rc) return rc;
    } else {
      // the second least-priority stream starts after the V^T staging on ws2
      cudaStream_t ws3 = side_stream(st, 2);
      if (!ws3) return cuda_fail();
      if (cudaEventCreateWithFlags(&evs.vt, cudaEventDisableTiming) != cudaSuccess ||
          cudaEventRecord(evs.vt, ws2) != cudaSuccess || cudaStreamWaitEvent(ws3, evs.vt, 0) != cudaSuccess)
        return cuda_fail();
      for (int k = 0; k < n_pieces; ++k) {
        // piece k: the tiles of chunks [k n / K, (k+1) n / K) (the first also the tiles before the reads)
        piece_c0[k] = (int)((long long)s.n_chunks * k / n_pieces);
        piece_c1[k] = (int)((long long)s.n_chunks * (k + 1) / n_pieces);
        const int tb = k == 0 ? 0 : ptile0 + piece_c0[k];
        const int te = k == n_pieces - 1 ? ntq : ptile0 + piece_c1[k];
        cudaStream_t sk = (k & 1) ? ws3 : ws2;
        if (te > tb) {
          rc = window_common(qr, kx, vt, sink_k, sink_v, ns, start, kpos0, L->sinks, B, H, G, T, Tk, W, o, lse_w,
                             st.err, sk, owp, ptile0, s.n_chunks, tb, te - tb);
          if (rc) return rc;
        }
        if (cudaEventCreateWithFlags(&evs.piece[k], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventRecord(evs.piece[k], sk) != cudaSuccess)
          return cuda_fail();
      }
      // ws2 ends after every piece (the join below and the stage mark wait for all of them)
      for (int k = 1; k < n_pieces; k += 2)
        if (cudaStreamWaitEvent(ws2, evs.piece[k], 0) != cudaSuccess) return cuda_fail();
    }
    stage_mark(ST_WIN, 1, ws2);
  }
  if (phase == kPhaseBegin) return BF_OK;   // the window stays on its stream until the second phase
  if (will_read) {
    // join the memory chain; the window is joined as a whole, or piece by piece by the reads below (their waits
    // then cover every piece before anything else runs on the caller's stream)
    if (cudaEventRecord(ev_mem, wsm) != cudaSuccess || cudaStreamWaitEvent(stream, ev_mem, 0) != cudaSuccess)
      return cuda_fail();
    if (n_pieces == 1 && (cudaEventRecord(ev_win, ws2) != cudaSuccess || cudaStreamWaitEvent(stream, ev_win, 0) != cudaSuccess))
      return cuda_fail();
  }
  // 4. memory reads, mixed into o by the gate (per window piece when the window was split)
  if (reads && n_pieces > 1) {
    for (int k = 0; k < n_pieces; ++k) {
      if (cudaStreamWaitEvent(stream, evs.piece[k], 0) != cudaSuccess) return cuda_fail();
      GdnStreams sp3 = s;
      sp3.p3_c0 = piece_c0[k];
      sp3.p3_c1 = piece_c1[k];
      if (sp3.p3_c1 > sp3.p3_c0) {
        rc = launch_gdn_prefill(sp3, stream, kGdnP3);
        if (rc) return rc;
      }
    }
  } else if (reads) {
    rc = launch_gdn_prefill(s, stream, kGdnP3);
    if (rc) return rc;
  }
  // 5. cache: the last min(T, W) tokens go to their ring slots (the state was updated in place)
  if (C) {
    stage_mark(ST_CACHE, 0, stream);
    const int m = T < W ? T : W;
    ring_write_kernel<<<dim3(m, B * G), 32, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(kr), static_cast<const __nv_bfloat16*>(v), km, g, beta, start, T, m, G, W,
        static_cast<__nv_bfloat16*>(C->ring_k), static_cast<__nv_bfloat16*>(C->ring_v), C->ring_km, C->ring_g,
        C->ring_beta, C->ring_pos);
    if (int e_ = launch_status()) return e_;
    stage_mark(ST_CACHE, 1, stream);
  }
  return BF_OK;
}

int bf_bifrost_layer_prefill(const bf_layer* L, const void* x, const void* q, const void* k, const void* v,
                             const void* qr, const void* kr, long long start, int B, int T, bf_ring_cache* C,
                             const void* sink_k, const void* sink_v, int ns, int memory, float* o, float* lse,
                             void* ws, size_t ws_bytes, bf_stream_t stream) {
  return layer_prefill_impl(L, x, q, k, v, qr, kr, start, B, T, C, sink_k, sink_v, ns, memory, o, lse, ws, ws_bytes,
                            stream, kPhaseAll, nullptr, nullptr);
}

size_t bf_layer_prefill_sp_workspace(int B, int T, int H, int G, int D, int window, int with_ring) {
  const size_t base = bf_layer_prefill_workspace(B, T, H, G, D, window, with_ring);
  return base ? base + sp_extra_bytes(B, T, G, D, window, with_ring) : 0;
}

int bf_bifrost_layer_prefill_sp(const bf_layer* L, const void* x, const void* q, const void* k, const void* v,
                                const void* qr, const void* kr, long long start, int B, int T, bf_ring_cache* C,
                                const void* sink_k, const void* sink_v, int ns, int phase, float* m_out,
                                float* n_out, float* o, float* lse, void* ws, size_t ws_bytes, bf_stream_t stream) {
  if (phase != 0 && phase != 1) return BF_ERR_INVALID_ARGUMENT;
  if (phase == 0 && (!m_out || !n_out || !aligned16(m_out) || !aligned16(n_out))) return BF_ERR_INVALID_ARGUMENT;
  if (start > 0 && !C) return BF_ERR_INVALID_ARGUMENT;
  return layer_prefill_impl(L, x, q, k, v, qr, kr, start, B, T, C, sink_k, sink_v, ns, 1, o, lse, ws, ws_bytes,
                            stream, phase == 0 ? kPhaseBegin : kPhaseFinish, m_out, n_out);
}

}  // extern "C"
