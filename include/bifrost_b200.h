/*
 * bifrost_b200.h -- C ABI of the B200 (sm_100a) implementation of Heimdall's Bifrost
 * converted-layer hot path.
 *
 * Conventions (every entry point):
 *   - all tensor arguments are device pointers to contiguous row-major arrays in the layouts
 *     written beside each argument; sizes are plain ints;
 *   - work is enqueued on the caller's `stream` (NULL = legacy default stream); nothing blocks
 *     except bf_device_error();
 *   - outputs and scratch (`ws`, `ws_bytes`) are allocated by the caller; the matching
 *     *_workspace() call returns the scratch bytes needed; no entry point allocates memory;
 *   - return value: BF_OK (0) or a BF_ERR_* code; bf_strerror() names it; arguments are
 *     validated (shapes, alignment, sizes) before anything is launched;
 *   - outputs are fp32, as in the reference (o, state, lse).
 * Element-type codes: BF_F32, BF_BF16 (and BF_F16 where stated).
 *
 * Reference interfaces each entry point replaces are cited as path:line inside the reference
 * project ValeroisAI/Heimdall.
 */
#ifndef BIFROST_B200_H
#define BIFROST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef BF_STREAM_T_DEFINED
#define BF_STREAM_T_DEFINED
typedef struct CUstream_st* bf_stream_t; /* == cudaStream_t */
#endif

enum {
  BF_OK = 0,
  BF_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape or size */
  BF_ERR_UNSUPPORTED = 2,      /* a shape this build does not implement (e.g. D != 256 on a tensor-core path) */
  BF_ERR_ALIGNMENT = 3,        /* pointer not 16-byte aligned */
  BF_ERR_WORKSPACE = 4,        /* ws_bytes smaller than the *_workspace() size */
  BF_ERR_CUDA = 5,             /* a CUDA runtime call failed (launch, attribute, tensor map) */
  BF_ERR_TIMEOUT = 6,          /* a bounded device-side wait gave up (see bf_device_error) */
  BF_ERR_NO_DEVICE = 7         /* no sm_100 device is current */
};

enum { BF_F32 = 0, BF_BF16 = 1, BF_F16 = 2 };

/* Human-readable name of a status code. */
const char* bf_strerror(int code);
/* Text of the CUDA error behind the calling thread's last BF_ERR_CUDA status. */
const char* bf_last_cuda_error(void);

/* ABI version of this library (bumped on any signature change). */
int bf_abi_version(void);

/* Synchronises `stream`, then reads and clears this device's error record into word[0..3]:
 * word[0] = 0 when no kernel gave up a wait, else (site << 8) | BF_ERR_TIMEOUT of the first one;
 * word[1] = its blockIdx.x, word[2] = blockIdx.y | blockIdx.z << 16, word[3] = its threadIdx.x.
 * Returns BF_OK or BF_ERR_CUDA. */
int bf_device_error(unsigned int* word, bf_stream_t stream);

/* Self-test of the device-side failure path.  Launches one small kernel (tensor memory allocated as the
 * production kernels do) whose bounded mbarrier wait can never complete and gives up after `limit_us`
 * microseconds (1 .. 1000000): it records the timeout in this device's error record (site 0xF1), frees its
 * tensor memory and returns; nothing faults, traps or hangs, and the context stays usable.  The next
 * bf_device_error() on the device reports word[0] = (0xF1 << 8) | BF_ERR_TIMEOUT.  Follows the
 * reference's self-test convention for candidate kernels (heimdall/kernels.py:168-188), applied to the
 * error path rather than to the numerics. */
int bf_selftest_wait_timeout(unsigned int limit_us, bf_stream_t stream);

/* Per-stage timing: `events` holds 2*n_stages cudaEvent_t handles (begin/end per stage); each
 * layer entry point records them on its stream around its stages (0 x-projection, 1 head
 * projection, 2-4 delta-rule phases P1/P2/P3, 5 window key/value prep, 6 window attention,
 * 7 cache write, 8 decode state update, 9 decode window split, 10 decode evicted-entry gather, 11 decode
 * combine; at most 12).  n_stages = 0 turns this off.
 * Process-wide; not for concurrent use from several threads.  No counterpart in the reference
 * (its only timing is wall-clock logging, heimdall/motor.py:292-297). */
int bf_stage_events(void* const* events, int n_stages);

/* ------------------------------------------------------------------------------------------
 * Gated delta rule, recurrent decode step (one token), GQA-native.
 * Replaces heimdall/kernels.py:132-138 (delta_rule_step) and the inline decode update of
 * heimdall/hibrit.py:398-403.
 *   S <- e^{g} S;  delta = (v - S^T k) * beta;  S <- S + k delta^T;  o_r = S^T q_r  (r < R)
 * q    [B,G,R,D] fp32          k [B,G,D] fp32        v [B,G,D] (v_dtype: BF_F32 or BF_BF16)
 * g, beta [B,G] fp32           s_in, s_out [B,G,D,D] fp32 (may alias)      o [B,G,R,D] fp32
 * D must be 256 or a multiple of 32 not above 256.
 */
int bf_gdn_decode_step(const float* q, const float* k, const void* v, int v_dtype, const float* g,
                       const float* beta, const float* s_in, float* s_out, float* o, int B, int G, int R,
                       int D, bf_stream_t stream);


/* ------------------------------------------------------------------------------------------
 * Per-layer parameters (device pointers; fp32 unless stated).  Shapes follow
 * HybridAttention.convert (heimdall/hibrit.py:211-240).
 */
typedef struct bf_layer {
  const void* wbuf;          /* prepared operand weights (bf_prepare_layer_weights) */
  const float* ab_b;         /* [2G]  bias of ab = Linear(d, 2G) */
  const float* mix_b;        /* [H]   bias of mix = Linear(d, H) */
  const float* mix_lse;      /* [H] */
  const float* mem_scale;    /* [H] */
  const float* A_log;        /* [G] */
  const float* dt_bias;      /* [G] */
  const float* decay_mask;   /* [G]   0 = archival (never-forgetting) head */
  int H, G, D, d, window, sinks;
} bf_layer;

/* Decode cache in the reference's per-layer cache-dict layout (heimdall/hibrit.py:414-423). */
typedef struct bf_ring_cache {
  void* ring_k;              /* [B,G,W,D] bf16, slot = position % W */
  void* ring_v;              /* [B,G,W,D] bf16 */
  float* ring_km;            /* [B,W,G,D] */
  float* ring_g;             /* [B,W,G] */
  float* ring_beta;          /* [B,W,G] */
  int64_t* ring_pos;         /* [W] (ring_pos_bstride 0) or [B,W] (ring_pos_bstride W); -1 = empty */
  long long ring_pos_bstride;
  const void* sink_k;        /* [B,G,ns,D] bf16 (positions 0..ns-1) or NULL */
  const void* sink_v;
  int ns;
  float* S;                  /* [B,G,D,D] memory state, updated in place */
} bf_ring_cache;

/* Bytes of the prepared weight buffer of one layer. */
size_t bf_layer_weights_bytes(int H, int G, int D, int d);

/* Convert the fp32 parameters fq [H,D,D], fk [G,D,D], ab_w [2G,d], mix_w [H,d] into the operand
 * layouts of the tensor-core kernels (fp16 transposed head maps, bf16 hi/lo split of the x maps).
 * Call once per layer (and again after the parameters change). */
int bf_prepare_layer_weights(const float* fq, const float* fk, const float* ab_w, const float* mix_w, int H,
                             int G, int D, int d, void* wbuf, size_t wbytes, bf_stream_t stream);

/* Memory inputs and gate logit, replacing heimdall/hibrit.py:327-334 (_mem_inputs) and the
 * mix(x) term of heimdall/hibrit.py:409:
 *   qm = unit(q_h fq_h) D^-1/2 [B,T,H,D]; km = unit(k_g fk_g) [B,T,G,D];
 *   g = -e^{A_log} softplus(a + dt_bias) decay_mask, beta = sigmoid(b) [pos >= sinks]  [B,T,G];
 *   mixx = x mix_w^T + mix_b [B,T,H]   where [a | b] = x ab_w^T + ab_b.
 * x [B,T,d], q [B,T,H,D], k [B,T,G,D] are bf16.  pos [B*T] int64 or NULL (then pos0 + t).
 * D must be 256; d a multiple of 64. */
int bf_mem_inputs(const bf_layer* L, const void* x, const void* q, const void* k, const int64_t* pos,
                  long long pos0, int B, int T, float* qm, float* km, float* g, float* beta, float* mixx,
                  bf_stream_t stream);

/* Scratch bytes of bf_bifrost_layer_decode. */
size_t bf_layer_decode_workspace(int B, int H, int G, int D, int window);

/* One decode step (one new token per sequence) of the converted layer core, replacing
 * HybridAttention._student with t == 1 (heimdall/hibrit.py:363-424): memory inputs, the state update
 * with the token leaving the window, sliding-window + sink attention, LSE gate and mix, and the
 * write of the new token into the ring.  Each sequence b has its own position pos[b] (int64, device);
 * the reference's batched decode is the case of equal positions.  The sinks buffer must already hold
 * the new token when pos < sinks (the reference appends it before attending).
 * x [B,d], q/qr [B,H,D], k/kr/v [B,G,D] bf16.  memory = 0 is the reference's "window" mode.
 * o [B,H,D] fp32, lse [B,H] fp32 or NULL. */
int bf_bifrost_layer_decode(const bf_layer* L, const void* x, const void* q, const void* k, const void* v,
                            const void* qr, const void* kr, const int64_t* pos, int B, bf_ring_cache* cache,
                            int memory, float* o, float* lse, void* ws, size_t ws_bytes, bf_stream_t stream);

/* The same decode step for callers that cannot allocate device memory (for instance a runtime whose
 * memory manager has reserved nearly all of HBM for its own pools, or a host that binds only these C
 * entry points and cannot own a device workspace).  No counterpart in the reference: Heimdall's
 * decode allocates freely through PyTorch.  It allocates nothing: its scratch is a fixed 16 MiB array
 * compiled into the library (one per GPU that loads it, held until the process exits), enough for
 * bf_layer_decode_workspace() of up to 64 sequences of the Bifrost geometry; larger requests return
 * BF_ERR_WORKSPACE before any launch.  The first call on each device looks the array's device address
 * up (cudaGetSymbolAddress) and should come before any stream capture.  All calls on a device share
 * the array, so calls that overlap on the GPU race; nothing in it needs to start at zero. */
int bf_bifrost_layer_decode_noalloc(const bf_layer* L, const void* x, const void* q, const void* k,
                                    const void* v, const void* qr, const void* kr, const int64_t* pos, int B,
                                    bf_ring_cache* cache, int memory, float* o, float* lse, bf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Chunked gated delta rule, forward (prefill), GQA-native.
 * Replaces heimdall/kernels.py:94-129 (delta_rule_reference, reached through delta_rule at
 * heimdall/kernels.py:152-155) and heimdall/motor.py:70-102 (delta_rule_gqa).
 * q [B,T,G*R,D] (q_dtype), k [B,T,G,D] (k_dtype), v [B,T,G,D] (v_dtype): BF_F32 or BF_BF16;
 * g, beta [B,T,G] fp32; s0 [B,G,D,D] fp32 or NULL (zero state); o [B,T,G*R,D] fp32;
 * s_out [B,G,D,D] fp32 (may alias s0).  D must be 256.  The GPU scan uses 128-token chunks and
 * fp16 tensor-core operands with fp32 accumulation and an fp32 state.
 * Packed variable-length sequences: cu_seqlens (device int32 [n_seq + 1], cu_seqlens[0] = 0,
 * non-decreasing, cu_seqlens[n_seq] = T) with B = 1; sequence i is tokens cu_seqlens[i] ..
 * cu_seqlens[i+1] - 1, runs its own recurrence, and s0 / s_out are [n_seq,G,D,D].  cu_seqlens NULL
 * and n_seq = 0: B sequences of T tokens.
 */
size_t bf_gdn_chunk_workspace(int B, int T, int G, int R, int D, int n_seq);
int bf_gdn_chunk_fwd(const void* q, int q_dtype, const void* k, int k_dtype, const void* v, int v_dtype,
                     const float* g, const float* beta, const float* s0, float* o, float* s_out,
                     const int* cu_seqlens, int n_seq, int B, int T, int G, int R, int D, void* ws, size_t ws_bytes,
                     bf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Chunked gated delta rule, backward (GQA-native): the gradients that torch autograd takes through
 * heimdall/motor.py:70-102 (delta_rule_gqa) when seq_loss (heimdall/motor.py:149-193) trains a layer.
 * Inputs as the forward, all fp32: q [B,T,G*R,D], k [B,T,G,D], v [B,T,G,D], g, beta [B,T,G],
 * s0 [B,G,D,D] or NULL (zero initial state); dout [B,T,G*R,D] = dL/do; dstate [B,G,D,D] = dL/d(final
 * state) or NULL (zero).  Outputs fp32, same shapes as the inputs: dq, dk, dv, dg, dbeta and ds0
 * (dL/ds0, written also when s0 is NULL).  D must be 256, R <= 8.  The recurrence runs token by token
 * in fp32 (states recomputed from 64-token checkpoints); see bf_gdn_bwd_workspace for the scratch.
 */
size_t bf_gdn_bwd_workspace(int B, int T, int G, int R, int D);
int bf_gdn_bwd(const float* q, const float* k, const float* v, const float* g, const float* beta, const float* s0,
               const float* dout, const float* dstate, float* dq, float* dk, float* dv, float* dg, float* dbeta,
               float* ds0, int B, int T, int G, int R, int D, void* ws, size_t ws_bytes, bf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Sliding-window + sink attention with log-sum-exp (fp32 softmax), replacing
 * heimdall/hibrit.py:336-361 (_window / _window_fp32).
 * qr [B,H,Tq,D] bf16, query i at position qpos0 + i.  k_ext [B,G,Tk,D] bf16, key j at position
 * kpos0 + j; v_ext bf16 addressed as v_ext[b*vb + g*vg + j*vj + d] (element strides).  Keys with
 * position < klo are not window keys (the reference's kp >= sinks rule, and empty ring slots).
 * sink_k/sink_v [B,G,ns,D] bf16 contiguous, positions 0..ns-1 (ns <= 8), or NULL.
 * A query at p sees window keys p-window < kp <= p and sinks kp <= p.
 * o [B,Tq,H,D] fp32; lse [B,H,Tq] fp32 or NULL.  D must be 256.
 */
size_t bf_window_workspace(int B, int G, int Tk, int D);
int bf_window_attn_fwd(const void* qr, const void* k_ext, const void* v_ext, long long vb, long long vg,
                       long long vj, const void* sink_k, const void* sink_v, int ns, long long qpos0,
                       long long kpos0, long long klo, int B, int H, int G, int Tq, int Tk, int D, int window,
                       float* o, float* lse, void* ws, size_t ws_bytes, bf_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Fused layer prefill of T new tokens at positions start .. start+T-1, replacing
 * HybridAttention._student for any t (heimdall/hibrit.py:363-424): memory inputs, the delayed
 * memory write stream (token j is written at step j + W; earlier steps come from the ring),
 * the chunked delta rule, the window + sink attention, the LSE gate and mix, and (with a cache)
 * the ring write of the last min(T, W) tokens and the in-place state update.
 * x [B,T,d], q [B,T,H,D], k/v [B,T,G,D], qr [B,H,T,D], kr [B,G,T,D]: bf16.
 * cache: NULL (no cache) or the ring cache (ring_pos shared by the batch, ring_pos_bstride 0; S
 * must point at a zero state when the cache holds none yet).  The sinks (positions 0..ns-1,
 * including any of this call's tokens) are passed separately, contiguous [B,G,ns,D] bf16.
 * memory = 0 is the reference's "window" mode.  o [B,T,H,D] fp32; lse [B,H,T] fp32 or NULL.
 */
size_t bf_layer_prefill_workspace(int B, int T, int H, int G, int D, int window, int with_ring);
int bf_bifrost_layer_prefill(const bf_layer* L, const void* x, const void* q, const void* k, const void* v,
                             const void* qr, const void* kr, long long start, int B, int T, bf_ring_cache* cache,
                             const void* sink_k, const void* sink_v, int ns, int memory, float* o, float* lse,
                             void* ws, size_t ws_bytes, bf_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * The converted attention layer around the core: fused prologue and epilogue.  The plain projection GEMMs
 * (q/gate, k, v, o) are left to the caller's GEMM library; these two passes replace the elementwise work
 * between them.
 *
 * bf_attn_prologue replaces the per-head split, the ZNorm and the partial RoPE of HybridAttention._proj
 * (heimdall/hibrit.py:254-268; rope heimdall/kernels.py:40-49) in one pass:
 *   qg [B,T,H,(gated ? 2 : 1)*D] bf16 (query projection, the output gate interleaved per head), kl [B,T,G,D]
 *   bf16 (key projection), q_norm_w / k_norm_w [D] fp32 (zero-centred ZNorm weights, eps), inv_freq [rot/2]
 *   fp32 (1 / theta^(2i/rot), as the reference computes it), pos [B*T] int64 or NULL (then start + t)
 *   -> q [B,T,H,D], k [B,T,G,D] (normalised, before RoPE), qr [B,H,T,D], kr [B,G,T,D] (half-rotation RoPE on
 *   the first rot dimensions), all bf16.  D must be 256; rot a multiple of 16, at most D.
 * bf_attn_epilogue replaces the gating of HybridAttention._out (heimdall/hibrit.py:270-272) ahead of o_proj:
 *   o [B,T,H,D] fp32 (the layer core's output), qg as above -> y [B,T,H*D] bf16 = bf16(o) * sigmoid(gate)
 *   (y = bf16(o) when gated = 0).
 */
int bf_attn_prologue(const void* qg, const void* kl, const float* q_norm_w, const float* k_norm_w,
                     const float* inv_freq, int rot, float eps, long long start, const int64_t* pos, int B, int T, int H,
                     int G, int D, int gated, void* q, void* k, void* qr, void* kr, bf_stream_t stream);
int bf_attn_epilogue(const float* o, const void* qg, int gated, int B, int T, int H, int D, void* y,
                     bf_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Sequence parallelism of the delta rule (a long sequence split into consecutive segments, one per
 * GPU).  A segment of the write stream maps any incoming state S to S_out = M (S - s0) + N, where N
 * is the final state from s0 (zero state when s0 is NULL).  These two entry points replace the
 * reference's single sequential scan over chunks (heimdall/kernels.py:118-129, the loop of
 * delta_rule_reference) when the chunks are spread over several devices.
 *
 * bf_gdn_segment_transform: k, v [B,T,G,D] (fp32 or bf16), g, beta [B,T,G] fp32, s0 [B,G,D,D] or
 * NULL -> m_out, n_out [B,G,D,D] fp32.  D = 256.
 * bf_gdn_apply_prefix: M, N [n_seg][B,G,D,D] (segments in order; NULL allowed when n_seg = 0), s0
 * [B,G,D,D] or NULL ->
 * s_in [n_seg + 1][B,G,D,D]: s_in[0] = s0, s_in[j+1] = M[j] s_in[j] + N[j] (fp32).
 */
size_t bf_gdn_segment_workspace(int B, int T, int G, int D);
int bf_gdn_segment_transform(const void* k, int k_dtype, const void* v, int v_dtype, const float* g,
                             const float* beta, const float* s0, float* m_out, float* n_out, int B, int T, int G,
                             int D, void* ws, size_t ws_bytes, bf_stream_t stream);
int bf_gdn_apply_prefix(const float* M, const float* N, int n_seg, const float* s0, float* s_in, int B, int G,
                        int D, bf_stream_t stream);

/*
 * The fused layer prefill in two phases for sequence parallelism (same arguments and workspace for both; the
 * workspace is bf_layer_prefill_sp_workspace() bytes): phase 0 computes the memory inputs, the per-chunk
 * products and the state map of this segment's write stream (m_out, n_out [B,G,D,D] fp32: S_out = M S_in + N,
 * N from a zero state), keeping each chunk's start state from a zero state and its start transition; phase 1
 * (given phase 0's m_out and n_out again) turns those into the chunk states from the incoming state cache->S
 * all at once (no second sequential scan), runs the memory reads, the window, the gate and mix and the cache
 * write, and leaves cache->S = M S_in + N (fp32).  memory is on; o/lse as in bf_bifrost_layer_prefill
 * (written by phase 1).  Replaces the single scan over chunks of heimdall/kernels.py:118-129 for one layer
 * prefill split over devices.
 */
size_t bf_layer_prefill_sp_workspace(int B, int T, int H, int G, int D, int window, int with_ring);
int bf_bifrost_layer_prefill_sp(const bf_layer* L, const void* x, const void* q, const void* k, const void* v,
                                const void* qr, const void* kr, long long start, int B, int T, bf_ring_cache* cache,
                                const void* sink_k, const void* sink_v, int ns, int phase, float* m_out,
                                float* n_out, float* o, float* lse, void* ws, size_t ws_bytes, bf_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Interchange with the llama.cpp port's per-sequence state row of one converted layer (reference
 * llamacpp/bifrost.patch), so a sequence can move between this library's cache and a llama.cpp server.
 * The row is fp32, ggml order: region [C, LR] (slot rows [k_rope | v | k_mem | g | beta], C = 3 G D + 2 G),
 * K plane [D, LR, G], transposed V plane [LR, D, G], delta state [D, D, G] (key index fastest), with
 * LR = round_up(sinks + window + 2, 32) slots: sinks | ring of window + 1 slots (slot = sinks + pos mod
 * (window + 1)) | scratch + padding.
 *
 * bf_llama_state_floats replaces llama_hparams::bifrost_state (bifrost.patch:221-239): floats per row.
 * bf_llama_state_pack: cache (ring_k/ring_v bf16; ring_pos [W] or [B,W]; sinks [B,G,ns,D] bf16 or ns = 0;
 *   S [B,G,D,D] or NULL = zero state) of B sequences whose next positions are next_pos [B] (device int64) ->
 *   rows (row b at rows + b * row_stride floats; row_stride >= bf_llama_state_floats).  Writes every float of
 *   the rows: the ring rows of positions next_pos - W .. next_pos - 1 that the cache holds, the sink rows,
 *   the delta state; zero elsewhere (what the port writes there is never read again).  Replaces the port's
 *   writes of a prefill / decode into the row (bifrost.patch:1040-1085) for a sequence the library advanced.
 * bf_llama_state_unpack: rows -> cache for sequences at next_pos (ring slot j <- the position of
 *   [next_pos - W, next_pos) that is j mod W, ring_pos set, -1 and zeros for negative positions; sink rows
 *   0 .. ns-1; S).  k_rope and v are rounded to bf16 (nearest even).  With ring_pos [W] (bstride 0) every
 *   sequence must be at the same position.  S is required.
 * D = 256, G even and at most 8; rows 16-byte aligned with row_stride a multiple of 4, ring_km 16-byte and the
 * bf16 arrays 8-byte aligned (else BF_ERR_ALIGNMENT).  Both are layout copies on `stream` (HBM-bound).
 */
/* ---------------------------------------------------------------------------------------------
 * Retrieval attention of the kept (not converted) full-attention layers, single-token decode: replaces the
 * retrieval branch of HybridAttention._teacher (heimdall/hibrit.py:275-290) and _retrieval_mask (:301-324).
 * The query at position n - 1 attends the sinks [0, sinks), the `topk` blocks of `block` keys with the largest
 * upper bound of q.k (max over the group's query heads of sum_d max(q_d, 0) kmax_d + min(q_d, 0) kmin_d) among
 * the nc = (n - window - sinks) / block blocks that end before the window, and the window
 * [sinks + nc * block, n - 1]; exact softmax, scale D^-1/2.  Requires n - sinks - window >= topk * block.
 *
 * bf_ret_summarize: per-dim key min / max of full blocks nb0 .. nb1 - 1 after the sinks:
 *   k [B,G,cap,D] bf16 -> kmin, kmax [B,G,nbcap,D] bf16 (exact).
 * bf_ret_decode: q [B,H,D] bf16 (RoPE'd), k / v [B,G,cap,D] bf16 (the cache, n keys valid, the new token's at
 *   n - 1), kmin / kmax of the first nc blocks -> o [B,H,D] fp32.  Workspace: bf_ret_decode_workspace().
 * D = 256, H / G <= 8, topk <= 64.
 */
int bf_ret_summarize(const void* k, long long cap, int B, int G, int D, int sinks, int block, int nb0, int nb1,
                     void* kmin, void* kmax, long long nbcap, bf_stream_t stream);
size_t bf_ret_decode_workspace(int B, int H, int G, int D, int n, int sinks, int window, int block, int topk);
int bf_ret_decode(const void* q, const void* k, const void* v, long long cap, const void* kmin, const void* kmax,
                  long long nbcap, int B, int H, int G, int D, int n, int sinks, int window, int block, int topk,
                  float* o, void* ws, size_t ws_bytes, bf_stream_t stream);

size_t bf_llama_state_floats(int G, int D, int window, int sinks);
int bf_llama_state_pack(const bf_ring_cache* cache, const int64_t* next_pos, int B, int G, int D, int window,
                        int sinks, float* rows, long long row_stride, bf_stream_t stream);
int bf_llama_state_unpack(const float* rows, long long row_stride, const int64_t* next_pos, int B, int G, int D,
                          int window, int sinks, bf_ring_cache* cache, bf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BIFROST_B200_H */
