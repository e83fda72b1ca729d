/*
 * laguna_b200.h — C ABI of the B200 (sm_100a) kernels for the Laguna MoE decoder hot path.
 *
 * Conventions
 *  - Every pointer is a DEVICE pointer unless stated otherwise. The caller allocates every
 *    input, output and workspace; the library never allocates on these paths and keeps no
 *    pointer past the call.
 *  - bf16 tensors are passed as `const void*` / `void*` (IEEE bfloat16 bit patterns).
 *  - MLX packed layouts: a quantized matrix [rows, cols] is `uint32 weight[rows, cols*bits/32]`
 *    (32/bits codes per word, low bits first) plus bf16 `scales`/`biases` [rows, cols/group];
 *    value = scale * code + bias.  A stacked expert tensor adds a leading [E] axis.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are asynchronous,
 *    stateless and re-entrant per stream.
 *  - Return value: LG_OK (0) or an LG_ERR_* code; lg_last_error() then holds a message
 *    (thread-local).  Argument checks happen on the host before any launch.
 *
 * Each entry point names the lagunaLab interface (file:line) whose computation it replaces.
 */
#ifndef LAGUNA_B200_H
#define LAGUNA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LG_OK = 0,
  LG_ERR_INVALID = 1,     /* bad shape / unsupported configuration (reference ValueError / assert) */
  LG_ERR_UNSUPPORTED = 2, /* valid request this build does not implement */
  LG_ERR_CUDA = 3,        /* CUDA runtime error (launch, memset) */
  LG_ERR_WORKSPACE = 4    /* workspace pointer NULL, misaligned or smaller than required */
};

enum { LG_SCORE_SIGMOID = 0, LG_SCORE_SOFTMAX = 1 };

enum { LG_PATH_AUTO = 0, LG_PATH_GEMV = 1, LG_PATH_TENSOR = 2 };
/* LG_PATH_AUTO's crossover: the GEMV kernels up to this many expert rows (routed picks plus the
 * shared expert's rows), the tcgen05 grouped GEMM above it. */
enum { LG_MOE_GEMV_MAX_ROWS = 768 };

/* ABI version of this library (bumped on any signature change). */
int lg_abi_version(void);

/* Message for the last failing call on this thread ("" if none). */
const char* lg_last_error(void);

/* Number of kernels this library has launched so far (all threads). */
long long lg_launch_count(void);

/*
 * Measurement hook: on this thread, record cudaEvent_t ev_start / ev_end on the launching
 * stream immediately before / after every launch of the named stage ("router_logits",
 * "router_topk", "plan", "experts_gateup", "experts_down", "finalize", "q8_decode").
 * stage == NULL turns it off.  No effect on results.  Inside a stream capture the records
 * become external event-record nodes, so each graph replay re-times the stage.
 */
int lg_profile_stage(const char* stage, void* ev_start, void* ev_end);

/*
 * Programmatic dependent launch for the decode-chain kernels (RMSNorm, GEMVs, embedding,
 * attention prologue, bf16 decode attention, router, plan, MoE GEMVs, finalize, argmax):
 * with on != 0 they are launched so that each may start while the previous kernel in the
 * stream is still running; it waits for that kernel's completion before reading any input
 * the previous kernel could write, and streams only static data (weights, and K/V rows and
 * device-side lengths written by earlier kernels) before.  Contract while on: the kernel
 * launched immediately before one of these must not write its weights, the K/V rows it reads
 * other than the newest, or its device-side length.  Process-wide; returns the previous
 * setting.  Off by default.
 */
int lg_set_pdl(int on);

/* Milliseconds between two recorded cudaEvent_t (waits for ev_end). */
int lg_event_elapsed_ms(void* ev_start, void* ev_end, float* ms);

/*
 * Router: laguna_mlx/laguna.py:137-145 (SparseMoeBlock.route).
 *   logits = x @ Wg^T (fp32), scores = sigmoid(logits), sel = scores + e_bias,
 *   inds = top-k of sel (larger first; equal sel -> lower expert index first),
 *   w = scores[inds], w /= sum(w) if norm_topk_prob, w -> bf16.
 * x bf16 [T, H].  Router weight: gate_bits == 0 -> gate_w fp32 [E, H] (scales/biases NULL);
 * gate_bits == 8 -> MLX 8-bit group-64 (laguna.py:236-238): gate_w uint32 [E, H/4],
 * scales/biases bf16 [E, H/64]; the quantized matmul's bf16 output is what the sigmoid sees.
 * e_bias fp32 [E] or NULL (zeros).  Outputs: inds int32 [T, k], weights bf16 [T, k],
 * logits fp32 [T, E] (required: the top-k reads the logits from it), counts int32 [E]
 * (optional histogram of picks, NULL to skip).
 * Limits: E <= 256, 1 <= k <= min(E, 32), H % 64 == 0.
 */
int lg_router_topk(const void* x, int T, int H,
                   const void* gate_w, const void* gate_scales, const void* gate_biases, int gate_bits,
                   const float* e_bias, int E, int k, int norm_topk_prob, int score_fn,
                   int32_t* inds, void* weights, float* logits, int32_t* counts,
                   void* stream);

/*
 * Routing plan (the token->expert dispatch order used by SwitchGLU's sorted path,
 * mlx-lm switch_layers, called at laguna_mlx/laguna.py:149): per-expert pick counts and an
 * expert-contiguous permutation of the T*k picks.  With with_shared != 0 a last group E
 * holds the T tokens of the shared expert (laguna.py:150), pick ids T*k + t.
 * counts int32 [E+1], offsets int32 [E+2] (exclusive prefix sums), perm int32 [T*k + T]
 * (pick ids ordered by expert, then by pick id).  Deterministic.
 */
int lg_moe_plan(const int32_t* inds, int T, int k, int E, int with_shared,
                int32_t* counts, int32_t* offsets, int32_t* perm, void* stream);

/* Workspace bytes for lg_moe_experts / lg_switch_glu / lg_qmlp at these sizes. */
size_t lg_moe_workspace_bytes(int T, int H, int I, int E, int k, int I_shared);

/*
 * Routed experts + combine: laguna_mlx/laguna.py:147-150 after route():
 *   out = (SwitchGLU(x, inds) * w[..., None]).sum(-2) * routed_scaling_factor + shared_expert(x)
 * SwitchGLU (mlx-lm 0.31.3 switch_layers, laguna.py:134, :149): per pick
 *   y = down(silu(gate(x)) * up(x)) on the picked expert's MLX-layout quantized weights,
 *   gate/up: weight [E, I, H*bits/32], scales/biases [E, I, H/group];
 *   down:    weight [E, H, I*bits/32], scales/biases [E, H, I/group].
 * Shared expert (laguna.py:114-122, :135): same layout without the E axis, intermediate
 * I_shared (0 = no shared expert, all sh_* may then be NULL).
 * x bf16 [T, H]; inds int32 [T, k]; weights bf16 [T, k]; out bf16 [T, H].
 * path: LG_PATH_AUTO picks the split-K GEMV kernels for few picks (<= LG_MOE_GEMV_MAX_ROWS rows
 * including the shared expert's) and the tcgen05 grouped GEMM otherwise; LG_PATH_TENSOR forces the latter
 * (needs H % 256 == 0, I % 128 == 0, I_shared % 128 == 0).  bits == 4, group_size == 64 (the
 * MLX default the reference converts with, scripts/convert.py:14); H, I, I_shared % 64 == 0.
 */
int lg_moe_experts(const void* x, int T, int H, int I, int E, int k,
                   const int32_t* inds, const void* weights, float routed_scaling_factor,
                   const uint32_t* gate_q, const void* gate_s, const void* gate_b,
                   const uint32_t* up_q, const void* up_s, const void* up_b,
                   const uint32_t* down_q, const void* down_s, const void* down_b,
                   int I_shared,
                   const uint32_t* sh_gate_q, const void* sh_gate_s, const void* sh_gate_b,
                   const uint32_t* sh_up_q, const void* sh_up_s, const void* sh_up_b,
                   const uint32_t* sh_down_q, const void* sh_down_s, const void* sh_down_b,
                   int group_size, int bits, int path,
                   void* out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Status word of the last tensor-core expert launch that used this workspace (same sizes as
 * that call): 0 = ok, otherwise the code of the pipeline role whose bounded wait expired (the
 * kernel then stopped instead of hanging).  Synchronous (copies 4 bytes to the host).
 */
int lg_moe_status(const void* workspace, int T, int H, int I, int E, int k, int I_shared,
                  int* status);

/*
 * SwitchGLU call surface (mlx-lm switch_layers.SwitchGLU.__call__(x, indices), used at
 * laguna_mlx/laguna.py:149 and streaming.py:95): per-pick, unweighted outputs
 * y bf16 [T, k, H].  Same weights and limits as lg_moe_experts.
 */
int lg_switch_glu(const void* x, int T, int H, int I, int E, int k, const int32_t* inds,
                  const uint32_t* gate_q, const void* gate_s, const void* gate_b,
                  const uint32_t* up_q, const void* up_s, const void* up_b,
                  const uint32_t* down_q, const void* down_s, const void* down_b,
                  int group_size, int bits, int path,
                  void* y, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Dense quantized SwiGLU MLP: laguna_mlx/laguna.py:114-122 (MLP.__call__; the shared
 * expert and the dense layer-0 MLP).  x bf16 [T, H] -> out bf16 [T, H], intermediate I.
 */
int lg_qmlp(const void* x, int T, int H, int I,
            const uint32_t* gate_q, const void* gate_s, const void* gate_b,
            const uint32_t* up_q, const void* up_s, const void* up_b,
            const uint32_t* down_q, const void* down_s, const void* down_b,
            int group_size, int bits, int path,
            void* out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Affine quantize rows (the append side of mlx-lm's QuantizedKVCache, laguna_mlx/cache.py:90,
 * and MLX-layout weight conversion, scripts/convert.py:14) with this library's rule:
 *   per group: scale = bf16((max - min) / (2^bits - 1)), bias = bf16(min),
 *   code = clamp(rint((x - bias) / scale), 0, 2^bits - 1)  (0 where scale == 0).
 * Source rows: x (bf16 if x_is_f32 == 0, else fp32) [B, H, L, D] with element strides
 * (sb, sh, sl) and unit stride on D.  Destination: packed uint32 [B, H, cap, D*bits/32],
 * scales/biases bf16 [B, H, cap, D/group], rows [offset, offset + L) written.
 * bits in {4, 8}, group_size in {32, 64, 128}, D % group_size == 0.
 */
int lg_quantize_rows(const void* x, int x_is_f32, int B, int H, int L, int D,
                     long long sb, long long sh, long long sl,
                     int bits, int group_size,
                     uint32_t* dst_q, void* dst_s, void* dst_b, int cap, int offset,
                     void* stream);

/*
 * Dequantize rows [0, n) of a packed [B, H, cap, *] buffer to bf16 [B, H, n, D]
 * (laguna_mlx/cache.py:99-100, the DequantKVCache path for multi-token steps).
 */
int lg_dequantize_rows(const uint32_t* q, const void* s, const void* b, int B, int H, int cap,
                       int n, int D, int bits, int group_size, void* out, void* stream);

/* Workspace bytes for lg_q8_decode_attention. */
size_t lg_q8_decode_workspace_bytes(int B, int Hq, int Hkv, int n);

/*
 * Fused single-token attention over an 8-bit group-64 quantized KV cache:
 * laguna_mlx/q8_attn.py:102-130 (q8_decode_attention) and the Metal kernel at :17-92.
 *   out = softmax((q * scale) . K[:n]^T) . V[:n]   per query head, GQA group Hq/Hkv.
 * q bf16 [B, Hq, D]; K/V: packed uint32 [B, Hkv, cap, D/4], scales/biases bf16
 * [B, Hkv, cap, D/64] (full-capacity buffers; only rows < n are read).  out bf16 [B, Hq, D].
 * D == 128, Hq % Hkv == 0, Hq/Hkv <= 16, 1 <= n <= cap.
 * The workspace's first 16 KiB hold completion counters that must be zero before the first
 * call; every completed call leaves them zero again, whatever its sizes, so one zeroed
 * workspace of the largest size needed serves calls of any shapes.
 */
int lg_q8_decode_attention(const void* q, int B, int Hq, int Hkv, int D,
                           const uint32_t* k_q, const void* k_s, const void* k_b,
                           const uint32_t* v_q, const void* v_s, const void* v_b,
                           int cap, int n, float scale,
                           void* out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * lg_q8_decode_attention_noalloc: no counterpart in the reference.  The same fused q8 decode
 * attention as lg_q8_decode_attention, for callers that cannot allocate device memory at the
 * moment they call (a plugin host that only hands over input and output pointers, or a
 * latency-critical path that cannot afford cudaMalloc's implicit device synchronisation).
 * It issues a memset and a kernel launch on `stream`, so it must not be called from a stream
 * callback (cudaLaunchHostFunc), where CUDA forbids every CUDA API call.
 * It allocates nothing: its scratch (split partials and completion counters) lives in a fixed
 * 1 MiB array inside this library, which every GPU that loads the library holds until the
 * process exits (lg_q8_decode_fixed_scratch_bytes() returns the size).  A call whose scratch
 * (lg_q8_decode_workspace_bytes of the same sizes) exceeds it is rejected with LG_ERR_INVALID.
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress)
 * for the current device; make that first call before any stream capture.  Every call clears
 * the counters it needs on `stream`; all calls on a device share the one array, so calls that
 * overlap on the GPU (different streams, or threads without ordering) race and must not be
 * issued.  Inputs, outputs and limits are those of lg_q8_decode_attention.
 */
size_t lg_q8_decode_fixed_scratch_bytes(void);
int lg_q8_decode_attention_noalloc(const void* q, int B, int Hq, int Hkv, int D,
                                   const uint32_t* k_q, const void* k_s, const void* k_b,
                                   const uint32_t* v_q, const void* v_s, const void* v_b,
                                   int cap, int n, float scale, void* out, void* stream);

/* ---------------------------------------------------------------------------------------
 * Full decoder (laguna_mlx/laguna.py:75-206) around the MoE block and the decode attention.
 * Rounding follows the MLX graph: each op's output is materialised in bf16.
 * ------------------------------------------------------------------------------------- */

/*
 * RMSNorm, nn.RMSNorm / mx.fast.rms_norm (laguna.py:158-160, :189):
 *   y = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w), statistics in fp32.
 * With residual != NULL, h = bf16(x + residual) is the decoder's residual stream
 * (laguna.py:163-164) and is also written to sum_out (may be NULL); else h = x.
 * x, residual, sum_out, out bf16 [T, H]; w bf16 [H]; H % 8 == 0; 16-byte aligned.
 */
int lg_rmsnorm(const void* x, const void* residual, const void* w, int T, int H, float eps,
               void* sum_out, void* out, void* stream);

/*
 * 4-bit group-64 dense linear at decode sizes, nn.QuantizedLinear (laguna.py:84-92, :197):
 *   out = bf16(x . W^T) [+ residual, in bf16], W = scale * code + bias per 64-group.
 * x bf16 [T, K] (T <= 64), W uint32 [N, K/8] with bf16 scales/biases [N, K/64], residual
 * and out bf16 [T, N].  K % 64 == 0.  Larger T: dequantize (lg_dequantize_rows) and use a
 * dense GEMM.
 */
int lg_qlinear(const void* x, int T, int K, int N, const uint32_t* w_q, const void* w_s,
               const void* w_b, int group_size, int bits, const void* residual, void* out,
               void* stream);

/*
 * Token embedding, nn.QuantizedEmbedding (laguna.py:174, :183): out[t] = bf16(scale * code
 * + bias) of row ids[t] (device int32 [T]) of a 4-bit group-64 table [V, H].  An id outside
 * [0, V) yields a NaN row.
 */
int lg_embed(const int32_t* ids, int T, const uint32_t* w_q, const void* w_s, const void* w_b,
             int V, int H, int group_size, int bits, void* out, void* stream);

/*
 * Attention prologue, Attention.__call__ (laguna.py:94-106) for one sequence:
 * from qkvg bf16 [T, Hq*D + 2*Hkv*D + (gate_per_head ? Hq : Hq*D)] (the q, k, v and g
 * projections of T tokens at positions p = pos + t, pos = *pos_dev if pos_dev else pos_host):
 *   q_out  bf16 [Hq, T, D]    = rope(bf16(rmsnorm(q_h, qn_w)), p)
 *   k_cache bf16 [Hkv, cap, D] row p = rope(bf16(rmsnorm(k_h, kn_w)), p)
 *   v_cache bf16 [Hkv, cap, D] row p = v_h
 *   gate_out bf16 [T, Hq or Hq*D]     = bf16(softplus(float(g)))
 * RoPE: non-interleaved pairs (i, i + R/2) over the first R dims (laguna.py:62-72). rot_dims 0
 * (inv_freq NULL, mscale 1): R = D and inv_freq_i = theta^(-2i/D), the default rope.
 * Otherwise R = rot_dims (a multiple of 64, <= D) with the caller's frequency table
 * inv_freq fp32 [R/2] (partial rotary, YaRN) and, for mscale != 1 (YaRN's attention factor),
 * the rotated dims scaled by mscale and rounded to bf16 first; dims past R pass through.
 * Cache rows: ring > 0 (a sliding window's ring buffer, ring == cap): row = p mod ring;
 * else row = p - row0.  D % 64 == 0, D <= 256.  Rows outside [0, cap) are not written.
 */
int lg_attn_prep(const void* qkvg, int T, int Hq, int Hkv, int D, const void* qn_w,
                 const void* kn_w, float eps, float rope_theta, const int32_t* pos_dev,
                 int pos_host, int gate_per_head, void* q_out, void* k_cache, void* v_cache,
                 int cap, void* gate_out, const float* inv_freq, int rot_dims, float mscale,
                 int ring, int row0, void* stream);

/*
 * lg_attn_prep with an 8-bit group-64 KV cache (DequantKVCache, laguna_mlx/cache.py:66-106):
 * the new k/v rows are quantized straight into the packed cache rows pos + t (words
 * [Hkv, cap, D/4], bf16 scales/biases [Hkv, cap, D/64]) with the arithmetic of
 * lg_quantize_rows (bit-identical to lg_attn_prep followed by lg_quantize_rows). D <= 256.
 */
int lg_attn_prep_q8(const void* qkvg, int T, int Hq, int Hkv, int D, const void* qn_w,
                    const void* kn_w, float eps, float rope_theta, const int32_t* pos_dev,
                    int pos_host, int gate_per_head, void* q_out, uint32_t* k_q, void* k_s,
                    void* k_b, uint32_t* v_q, void* v_s, void* v_b, int cap, void* gate_out,
                    const float* inv_freq, int rot_dims, float mscale, int ring, int row0,
                    void* stream);

/*
 * lg_attn_prep for one decode step of B independent streams (batched decode, BASELINE config
 * 5; the reference's caches hold one sequence: laguna_mlx/cache.py:66-157 has no batch merge,
 * docs/architecture.md:347-349). Token t of qkvg [B, .] is the newest token of stream t, at
 * position pos_dev[t] (device int32 [B]); its k/v rows go to row pos_dev[t] of stream t's
 * caches (k_cache, v_cache bf16 [B, Hkv, cap, D]; ring > 0: row = position mod ring) and q_out
 * is [B, Hq, D] (the layout lg_bf16_decode_attention_streams reads). Same arithmetic as
 * lg_attn_prep.
 */
int lg_attn_prep_streams(const void* qkvg, int B, int Hq, int Hkv, int D, const void* qn_w,
                         const void* kn_w, float eps, float rope_theta, const int32_t* pos_dev,
                         int gate_per_head, void* q_out, void* k_cache, void* v_cache, int cap,
                         void* gate_out, const float* inv_freq, int rot_dims, float mscale,
                         int ring, void* stream);

/*
 * One token's q/k/v/g projection (lg_decode_gemv with the layer's input RMSNorm fused in,
 * laguna.py:94-99) followed by its attention prologue (lg_attn_prep / lg_attn_prep_q8,
 * laguna.py:100-106) in one launch: qkvg_out = the projection row [q | k | v | g] (bf16,
 * N = (Hq + 2 Hkv) D + (gate_per_head ? Hq : Hq D)), q_out [Hq, 1, D], gate_out [1, Hq or
 * Hq D], and the new k/v rows written into row pos of the cache: the bf16 cache (k_cache,
 * v_cache [Hkv, cap, D]) or the 8-bit cache (k_q, k_s, k_b, v_q, v_s, v_b as in
 * lg_attn_prep_q8; the other pointers NULL). The same bits as lg_decode_gemv followed by the
 * prologue: every 16-row tile of the projection is one CTA; gate rows are finished by their
 * own CTA and the last CTA of each head to finish runs that head's prologue. The workspace
 * (lg_decode_qkv_prep_workspace_bytes) holds one counter per head; it must start zeroed and
 * completed calls leave it so. D % 64 == 0, D <= 256; LG_ERR_UNSUPPORTED when the projection's
 * tiles do not all fit on the GPU at once. inv_freq .. row0: RoPE and cache rows as in
 * lg_attn_prep.
 */
int lg_decode_qkv_prep(const void* x, int K, const uint32_t* w_q, const void* w_s,
                       const void* w_b, const void* norm_w, float eps, int Hq, int Hkv, int D,
                       const void* qn_w, const void* kn_w, float qk_eps, float rope_theta,
                       const int32_t* pos_dev, int pos_host, int gate_per_head, void* qkvg_out,
                       void* q_out, void* gate_out, void* k_cache, void* v_cache, uint32_t* k_q,
                       void* k_s, void* k_b, uint32_t* v_q, void* v_s, void* v_b, int cap,
                       const float* inv_freq, int rot_dims, float mscale, int ring, int row0,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes of lg_decode_qkv_prep (one counter per head slot). */
size_t lg_decode_qkv_prep_workspace_bytes(int Hq, int Hkv);

/* Workspace bytes for lg_bf16_decode_attention planned for n_plan keys. */
size_t lg_bf16_decode_workspace_bytes(int B, int Hq, int Hkv, int n_plan);

/*
 * Single-token attention over a bf16 KV cache: the SDPA branch of Attention.__call__
 * (laguna.py:102-107) with mlx-lm's KVCache, followed by the output gate (laguna.py:105-106):
 *   out = bf16(bf16(softmax(q . K[:n]^T * scale) . V[:n]) * gate)   per query head.
 * q bf16 [B, Hq, 128]; k, v bf16 [B, Hkv, cap, 128]; gate bf16 [B, Hq] (per-head) or NULL;
 * out bf16 [B, Hq, 128].  n = *n_dev + n_add when n_dev != NULL (a device-side length, for
 * decode steps that run without the host), else n.  The work split is planned for n_plan
 * (1 <= n_plan <= cap; an upper bound of n).  Hq % Hkv == 0, Hq / Hkv <= 16.  The workspace's
 * first 16 KiB hold completion counters that must start zeroed; completed calls leave them so.
 */
int lg_bf16_decode_attention(const void* q, int B, int Hq, int Hkv, int D, const void* k,
                             const void* v, int cap, int n, const int32_t* n_dev, int n_add,
                             int n_plan, float scale, const void* gate, void* out,
                             void* workspace, size_t workspace_bytes, void* stream);

/*
 * lg_bf16_decode_attention for B independent streams of different lengths (batched decode,
 * BASELINE config 5): stream b attends over n_dev[b] + n_add keys of its own cache
 * (n_dev: device int32 [B]); n_plan bounds every stream's length.
 */
int lg_bf16_decode_attention_streams(const void* q, int B, int Hq, int Hkv, int D,
                                     const void* k, const void* v, int cap,
                                     const int32_t* n_dev, int n_add, int n_plan, float scale,
                                     const void* gate, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream);

/*
 * Greedy token: ids[t] = argmax of bf16 logits row t of [T, V] (first index among equal
 * maxima, mx.argmax); if pos != NULL, *pos += inc afterwards (advances a device-side cache
 * position so consecutive decode steps need no host round trip).
 */
int lg_argmax(const void* logits, int T, int V, int32_t* ids, int32_t* pos, int inc,
              void* stream);

/* ---- one-token (bs1 decode) kernels -------------------------------------------------------
 * Each streams its weights into shared memory with bulk copies; with lg_set_pdl on, those of
 * the static weights are issued before the kernel waits for its predecessor. They have no
 * separate counterparts in the reference: they are the decode-size forms of the linears
 * (nn.QuantizedLinear, laguna.py:84-92, :197), the decoder layer's RMSNorms (laguna.py:158-161,
 * :189), SparseMoeBlock.__call__ (laguna.py:137-150) and MLP (laguna.py:114-122), fused the way
 * one decode step of the decoder (laguna.py:169-206) chains them.
 */

/*
 * One token through a 4-bit g64 linear [N, K] (w_q/w_s/w_b): out[n] = bf16(W x)[n]
 * (+ residual[n], bf16 add). norm_w != NULL: x is the residual stream and is first
 * RMS-normalised, bf16(bf16(x * rsqrt(mean(x^2) + eps)) * norm_w), bit-identical to
 * lg_rmsnorm. u_q != NULL (with u_s/u_b, same shape): gate/up pair, out = SwiGLU(W_g x, W_u x)
 * with the MLX rounding points (no residual then). K % 64 == 0, K <= 16384; x, weights,
 * scales, biases and norm_w 16-byte aligned.
 */
int lg_decode_gemv(const void* x, int K, int N, const uint32_t* w_q, const void* w_s,
                   const void* w_b, const uint32_t* u_q, const void* u_s, const void* u_b,
                   const void* norm_w, float eps, const void* residual, void* out, void* stream);

/*
 * One token's post-attention RMSNorm and router (laguna.py:137-145) in one launch: xn_out =
 * rmsnorm(h) (bf16 [H], bit-identical to lg_rmsnorm), logits = bf16(xn . W^T) for the 8-bit g64
 * router W [E, H] (bit-identical to lg_router_topk's), then the same sigmoid/softmax, bias,
 * top-k and weights as lg_router_topk: inds int32 [k], weights bf16 [k], logits fp32 [E]
 * (optional). CTAs of 8 experts each; the last one to finish selects. The workspace
 * (lg_router_decode_workspace_bytes) must start with 16 zero bytes; completed calls leave them
 * so. k <= 32; LG_ERR_UNSUPPORTED unless lg_router_decode_supported(H, E).
 */
int lg_router_decode(const void* h, const void* norm_w, float eps, int H, const uint32_t* gate_q,
                     const void* gate_s, const void* gate_b, const float* e_bias, int E, int k,
                     int norm_topk_prob, int score_fn, void* xn_out, int32_t* inds,
                     void* weights, float* logits, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Workspace bytes of lg_router_decode for E experts. */
size_t lg_router_decode_workspace_bytes(int E);

/* 1 if lg_router_decode takes an E x H router (E <= 256, H % 64 == 0, H <= 16384, and
 * H % 512 == 0 or E % 8 == 0), else 0. */
int lg_router_decode_supported(int H, int E);

/* Workspace bytes of lg_moe_decode: a 4 KiB block of completion counters first (must start
 * zeroed; completed calls of any size leave it so), then the groups' down outputs and SwiGLU
 * outputs. */
size_t lg_moe_decode_workspace_bytes(int H, int I, int I_shared, int k);

/* 1 if lg_moe_decode takes these sizes (its shared-memory tiles fit), else 0. */
int lg_moe_decode_supported(int H, int I, int I_shared, int k);

/*
 * One token through the MoE experts (laguna.py:147-150 after route): out = bf16(
 * sum_j bf16(w[j]) * routed_scale * y_j + y_shared) (+ residual, bf16 add), where y_j =
 * bf16(down_e(SwiGLU(gate_e xn, up_e xn))) for e = inds[j] (picks outside [0, E) contribute
 * nothing), y_shared the shared expert's output (I_shared = 0: none). Fixed summation order
 * (fp32, one rounding), two launches (gate/up + SwiGLU; down per (16-row slice, group), the
 * last group of a slice combining the slice and adding the residual).
 * Weights as lg_moe_experts, 16-byte aligned; H, I, I_shared multiples of 64.
 */
int lg_moe_decode(const void* xn, const int32_t* inds, const void* weights, int H, int I, int E,
                  int k, float routed_scale, const uint32_t* g_q, const void* g_s,
                  const void* g_b, const uint32_t* u_q, const void* u_s, const void* u_b,
                  const uint32_t* d_q, const void* d_s, const void* d_b, int I_shared,
                  const uint32_t* sg_q, const void* sg_s, const void* sg_b,
                  const uint32_t* su_q, const void* su_s, const void* su_b,
                  const uint32_t* sd_q, const void* sd_s, const void* sd_b,
                  const void* residual, void* out, void* workspace, size_t workspace_bytes,
                  void* stream);


/*
 * lg_q8_decode_attention for decode steps that run without the host (a CUDA graph replayed per
 * token): the valid length is *n_dev + n_add, read on the device (n_dev: the cache position
 * before the step); the work split is planned for n_plan >= that length (<= cap) and the
 * workspace sized by lg_q8_decode_workspace_bytes(B, Hq, Hkv, n_plan). gate: bf16 [B, Hq]
 * per-head output gate (laguna.py:105-106), out = bf16(bf16(attention) * gate), or NULL.
 * With lg_set_pdl on, the kernel may start while its predecessor runs and streams the K/V
 * tiles before waiting for it, except the tile holding row *n_dev + n_add - 1: the kernel
 * launched just before may write that row (the new key of the step), no other.
 */
int lg_q8_decode_attention_dev(const void* q, int B, int Hq, int Hkv, int D, const uint32_t* k_q,
                               const void* k_s, const void* k_b, const uint32_t* v_q,
                               const void* v_s, const void* v_b, int cap, int n_plan,
                               const int32_t* n_dev, int n_add, float scale, const void* gate,
                               void* out, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Check word of the one-token kernels' shared-memory staging: every 16-byte asynchronous copy
 * verifies that both addresses are 16-byte aligned and that its destination lies inside the
 * CTA's dynamic shared memory; a copy that fails is skipped (its tile's results are then
 * wrong) and the first failure is recorded here: check[0] = 1, check[1] = the destination's
 * shared-memory offset, check[2] = the source address, check[3] = blockIdx.y << 48 |
 * blockIdx.x << 16 | threadIdx.x. All zero when no check failed. Synchronous; reset != 0
 * clears it.
 */
int lg_decode_status(unsigned long long check[4], int reset);

/* ---------------------------------------------------------------------------------------
 * Expert parallelism over the GPUs of one node (no counterpart in the reference, which runs
 * on one device; BASELINE config 5 defines the sharding). W <= 8 ranks, one process per GPU;
 * rank r owns experts [r*E/W, (r+1)*E/W). Each rank allocates an arena of
 * lg_ep_arena_bytes(W, Tr, k, H) zeroed device bytes (Tr: the most tokens a rank routes in
 * one forward, the same on every rank), exports it with lg_ep_ipc_handle, maps every peer's
 * with lg_ep_ipc_open, and passes the W arena pointers (its own at index r) to every call.
 * A forward is, on every rank with the same epoch (1, 2, ... one per forward):
 *   lg_router_topk -> lg_ep_dispatch -> lg_qmlp (shared expert, into the arena's shared rows,
 *   lg_ep_arena_offsets) -> lg_ep_experts -> lg_ep_combine.
 * Epoch 0 in every call of a forward selects the device-held epoch instead: one past the
 * forwards this rank has completed, counted in its arena by lg_ep_advance (launched after
 * each forward's lg_ep_combine), so that forwards can be captured in a CUDA graph and
 * replayed. An arena uses one kind of epoch for its whole life.
 * The exchanges are peer stores issued by the kernels over NVLink (plain peer pointers); ranks
 * synchronise through epoch flags in the arenas with waits bounded by timeout_s (<= 0: 2 s).
 * An expired wait records (code | source << 8) in the arena's status word (lg_ep_status;
 * code 1: dispatch, 2: combine) and the forward completes with NaN outputs instead of
 * hanging. The output equals the one-GPU lg_moe_experts of the same tokens bit for bit.
 * --------------------------------------------------------------------------------------- */
size_t lg_ep_arena_bytes(int W, int Tr, int k, int H);
int lg_ep_arena_offsets(int W, int Tr, int k, int H, size_t* shared_rows, size_t* combine_rows);
size_t lg_ep_ipc_handle_bytes(void);
/* handle: lg_ep_ipc_handle_bytes() bytes; offset: ptr minus the start of its allocation. */
int lg_ep_ipc_handle(const void* ptr, void* handle, size_t* offset);
/* Maps a peer's allocation; *ptr = its start + offset, *base is what lg_ep_ipc_close takes. */
int lg_ep_ipc_open(const void* handle, size_t offset, void** ptr, void** base);
int lg_ep_ipc_close(void* base);
/* Sends this rank's T <= Tr tokens (x bf16 [T, H], inds int32 [T, k], weights bf16 [T, k]) to
 * the owners of their picks: two launches on `stream`. */
int lg_ep_dispatch(const void* x, const int32_t* inds, const void* weights, int T, int Tr,
                   int H, int k, int E, int W, int rank, void* const* arenas, unsigned epoch,
                   void* stream);
/* lg_ep_dispatch with a placement of the experts over the ranks: rank owner_of[e] holds
 * expert e as its local expert local_of[e] (int32 [E] device tables, each rank holding E/W
 * experts; both NULL: the contiguous ranges). Lets a caller balance the experts' load. */
int lg_ep_dispatch_mapped(const void* x, const int32_t* inds, const void* weights, int T, int Tr,
                          int H, int k, int E, int W, int rank, void* const* arenas,
                          unsigned epoch, const int32_t* owner_of, const int32_t* local_of,
                          void* stream);
size_t lg_ep_experts_workspace_bytes(int W, int Tr, int H, int I, int El, int k);
/* Waits for every source's dispatch, runs this rank's El experts (MLX 4-bit g64 weights
 * [El, I, H/8] / [El, H, I/8] with bf16 scales and biases) over the received rows and stores
 * every pick's bf16(bf16(y) * w) into its source's arena; then flags every source. */
int lg_ep_experts(int W, int Tr, int H, int I, int El, int k, const uint32_t* gate_q,
                  const void* gate_s, const void* gate_b, const uint32_t* up_q, const void* up_s,
                  const void* up_b, const uint32_t* down_q, const void* down_s,
                  const void* down_b, int rank, void* const* arenas, unsigned epoch,
                  double timeout_s, int path, void* workspace, size_t workspace_bytes,
                  void* stream);
/* Waits for every owner's rows, then out[t] = bf16(bf16(bf16(sum_j rows) * scale) + shared). */
int lg_ep_combine(const int32_t* inds, int T, int Tr, int H, int k, int E, float routed_scale,
                  int has_shared, int W, int rank, void* const* arenas, unsigned epoch,
                  double timeout_s, void* out, void* stream);
/* After a forward with device-held epochs (epoch 0): one launch on `stream` that counts the
 * forward as completed in this rank's arena. */
int lg_ep_advance(void* arena, void* stream);
/* Status word of an arena (0 = ok). Synchronous; reset != 0 clears it. */
int lg_ep_status(const void* arena, int reset, int* status);

#ifdef __cplusplus
}
#endif

#endif /* LAGUNA_B200_H */
