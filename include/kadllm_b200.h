/*
 * kadllm_b200 -- C ABI of the B200-native GRBeam library (sm_100a).
 *
 * Every entry point takes plain device pointers, element counts / strides
 * (in elements, not bytes), dtype codes and a cudaStream_t passed as void*.
 * None allocates device memory: callers (the Python host layer, through torch)
 * own every buffer.  Calls are asynchronous on `stream`; argument errors are
 * reported synchronously through the return code, with a message available
 * from kadllm_last_error() on the calling thread.
 *
 * Reference interfaces each entry point replaces are cited per function
 * (paths relative to the Kadllm project, Greek-Guardian/Kadllm).
 */
#ifndef KADLLM_B200_H_
#define KADLLM_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define KADLLM_API __attribute__((visibility("default")))
#else
#define KADLLM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
enum { KADLLM_F32 = 0, KADLLM_F16 = 1, KADLLM_BF16 = 2 };

/* status codes: mapped by the Python layer to ValueError / TypeError /
 * NotImplementedError / RuntimeError, the reference's error conventions
 * (src/kadllm/ops.py:17-67, src/kadllm/kernels/flash_attention.py:20-23). */
enum {
  KADLLM_OK = 0,
  KADLLM_EINVAL = 1,      /* bad shape / argument        -> ValueError          */
  KADLLM_EDTYPE = 2,      /* unsupported dtype           -> TypeError           */
  KADLLM_EUNSUPPORTED = 3,/* valid but not implemented   -> NotImplementedError */
  KADLLM_ECUDA = 4        /* CUDA launch / runtime error -> RuntimeError        */
};

/* Message of the last failed call on this thread ("" if none). */
KADLLM_API const char* kadllm_last_error(void);
/* Library ABI version. */
KADLLM_API int kadllm_abi_version(void);

/* ------------------------------------------------------------------------
 * Gated delta rule replay from a shared, request-sized state.
 * Replaces src/kadllm/kernels/gated_delta.py:145 beam_fused_recurrent_gdn
 * (the Triton path of src/kadllm/ops.py:70 gated_delta).
 *   q, k  [BW, T, H, K]   contiguous, dtype x_dtype (f32/f16/bf16)
 *   v     [BW, T, HV, V]  contiguous, x_dtype
 *   log_decay, beta [BW, T, HV] contiguous, any float dtype
 *   state [B, HV, K, V]   contiguous, any float dtype; never written
 *   out   [BW, T, HV, V]  contiguous, x_dtype
 * BW = batch * beam_width; beams of request b are rows b*W .. b*W+W-1.
 * K == V in {32, 64, 128}; 1 <= T <= 8; HV % H == 0.  scale <= 0 -> K^-0.5.
 * status: device uint32, bit 0 set when a tensor-core wait timed out (read it
 * after the stream synchronises; the output is then invalid).
 * ------------------------------------------------------------------------ */
KADLLM_API int kadllm_gated_delta_replay(const void* q, const void* k, const void* v, int x_dtype,
                              const void* log_decay, int decay_dtype, const void* beta,
                              int beta_dtype, const void* state, int state_dtype, void* out,
                              int64_t batch, int64_t beam_width, int64_t steps, int64_t heads,
                              int64_t v_heads, int64_t k_dim, int64_t v_dim, float scale,
                              uint32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Fused GDN token mixer for beam decode (BF16): causal conv1d replay + SiLU,
 * gates, gated delta replay from the shared state and the gated RMSNorm, i.e.
 * src/kadllm/adapters/qwen3_5.py:144-177 (_linear) from the packed input
 * projection up to (not including) out_proj.
 *   proj        [BW*T, ld_proj] bf16, row = beam_row*T + t; columns
 *               [q (H*K) | k (H*K) | v (HV*V) | z (HV*V) | b (HV) | a (HV)]
 *   conv_state  [B, conv_dim, conv_hist] bf16 contiguous (last 3 taps used)
 *   conv_weight [conv_dim, 4] bf16 contiguous
 *   rec_state   [B, HV, K, V] bf16 contiguous
 *   a_log, dt_bias [HV] f32; norm_weight [V] f32 (values of the BF16 params)
 *   out         [BW*T, HV*V] bf16
 *   records     null, or (steps == 1, K == V in {64, 128}) kadllm_gdn_mixer_record_bytes
 *               bytes, 16-byte aligned: per (beam row, value head) the row's delta
 *               beta (v - S^T k) (V fp32 values), from which kadllm_gdn_mixer_continue
 *               runs the next step on the new tokens only
 *   status      device uint32: bit 0 set when a tensor-core wait timed out
 *               (read it after the stream synchronises; the output is then invalid)
 * ------------------------------------------------------------------------ */
KADLLM_API int kadllm_gdn_mixer_replay(const void* proj, int64_t ld_proj, const void* conv_state,
                            int64_t conv_hist, const void* conv_weight, const void* rec_state,
                            const float* a_log, const float* dt_bias, const float* norm_weight,
                            float norm_eps, void* out, int64_t batch, int64_t beam_width,
                            int64_t steps, int64_t heads, int64_t v_heads, int64_t k_dim,
                            int64_t v_dim, void* records, uint32_t* status, void* stream);
KADLLM_API int64_t kadllm_gdn_mixer_record_bytes(int64_t batch, int64_t beam_width, int64_t v_heads,
                                                 int64_t v_dim);

/* ------------------------------------------------------------------------
 * Depthwise causal conv1d replay from a shared prefix state (+ SiLU).
 * Replaces src/kadllm/kernels/causal_conv1d.py:59 beam_causal_conv1d_update
 * (the Triton path of src/kadllm/ops.py:166 causal_conv1d).
 *   x      [BW, C, T] with element strides (xs0, xs1, xs2)  (may be a view)
 *   state  [B, C, hist] with strides (ss0, ss1, ss2); the last width-1 taps
 *          are used; never written
 *   weight [C, width] contiguous; bias [C] or NULL
 *   out    [BW, C, T] contiguous.  x/state/weight/bias/out share `dtype`.
 * width <= 8; silu != 0 applies SiLU.
 * ------------------------------------------------------------------------ */
KADLLM_API int kadllm_causal_conv1d_replay(const void* x, int64_t xs0, int64_t xs1, int64_t xs2,
                                const void* state, int64_t ss0, int64_t ss1, int64_t ss2,
                                int64_t hist, const void* weight, const void* bias, void* out,
                                int dtype, int64_t batch, int64_t beam_width, int64_t channels,
                                int64_t steps, int64_t width, int silu, void* stream);

/* ------------------------------------------------------------------------
 * Shared-prefix + causal-suffix GQA attention for beam decode (BF16).
 * Replaces src/kadllm/kernels/flash_attention.py:11 prefix_attention_flash
 * (the accelerated path of src/kadllm/ops.py:252 prefix_attention).
 *   q        [BW, T, H, D]   strides (sq_bw, sq_t, sq_h), D contiguous
 *   prefix_k [B, L, HK, D]   strides (spk_b, spk_l, spk_h); prefix_v likewise
 *   suffix_k [BW, T, HK, D]  strides (ssk_bw, ssk_t, ssk_h); suffix_v likewise
 *   prefix_mask [B, L] uint8 (nonzero = valid key) or NULL
 *   gate     [BW, T, H, D] strides (sg_bw, sg_t, sg_h) or NULL: out = o * sigmoid(gate)
 *   out      [BW, T, H, D]   strides (so_bw, so_t, so_h)
 * Fully masked or empty (L = 0) prefixes contribute nothing; T <= 8;
 * D in {32, 64, 128, 256}.  q and prefix rows must be 16-byte aligned.
 * ------------------------------------------------------------------------ */
KADLLM_API int kadllm_prefix_attention(
    const void* q, int64_t sq_bw, int64_t sq_t, int64_t sq_h, const void* prefix_k, int64_t spk_b,
    int64_t spk_l, int64_t spk_h, const void* prefix_v, int64_t spv_b, int64_t spv_l, int64_t spv_h,
    const void* suffix_k, int64_t ssk_bw, int64_t ssk_t, int64_t ssk_h, const void* suffix_v,
    int64_t ssv_bw, int64_t ssv_t, int64_t ssv_h, const void* prefix_mask, const void* gate,
    int64_t sg_bw, int64_t sg_t, int64_t sg_h, void* out, int64_t so_bw, int64_t so_t, int64_t so_h, int dtype,
    int64_t batch, int64_t beam_width, int64_t steps, int64_t heads, int64_t kv_heads,
    int64_t prefix_len, int64_t head_dim, float scale, void* stream);

/* ------------------------------------------------------------------------
 * One GRBeam selection step for a whole batch: fp32 log-softmax of every row
 * (full vocabulary), optional mask (-inf, no renormalisation), + parent score,
 * top-`width` of the prev_width*vocab candidates per request, sorted by score
 * (ties: lower flat index first), and the gathered history.
 * Replaces the per-request loop of src/kadllm/grbeam.py:87-104.
 *   logits        [B*Wp rows, V] with row stride ld_row, dtype logits_dtype
 *   parent_scores [B, Wp] f32 or NULL (all zero, first step)
 *   mask          [B*Wp, V] uint8 (nonzero = allowed) or NULL
 *   old_history   [B, Wp, depth] int64 or NULL when depth == 0
 *   out_scores    [B, width] f32;  out_history [B, width, depth+1] int64
 *   out_parent    [B, width] int32 or NULL: each selected beam's previous beam
 *                 (index in 0..Wp-1; 0 for unfilled slots)
 *   workspace     >= kadllm_beam_select_workspace(B, Wp) bytes, 256-byte
 *                 aligned, caller-owned.  Its flag word (offset 0, the same for
 *                 every Wp) is cleared by each depth-0 call, the first step of
 *                 a search, and OR-ed into by every later step.
 * At most 16384 candidates above the per-request threshold are kept; an
 * overflow sets a flag read by kadllm_beam_select_status.
 * ------------------------------------------------------------------------ */
KADLLM_API int64_t kadllm_beam_select_workspace(int64_t batch, int64_t prev_width);
KADLLM_API int kadllm_beam_select(const void* logits, int logits_dtype, int64_t ld_row,
                                  const float* parent_scores, const void* mask,
                                  const int64_t* old_history, float* out_scores,
                                  int64_t* out_history, int32_t* out_parent, void* workspace,
                                  int64_t workspace_bytes, int64_t batch, int64_t prev_width,
                                  int64_t vocab, int64_t width, int64_t depth, void* stream);
/* Fused LM head and selection (the reference's lm_head(norm(x)) then per-request
 * log_softmax + topk, src/kadllm/adapters/qwen3_5.py:235 and
 * src/kadllm/grbeam.py:87-104): kadllm_gemm_logits computes the BF16 logits of
 * the B*Wp decode rows and, in its epilogue, every row's per-256-column-chunk
 * maximum and sum of exp(x - maximum) into the selection workspace (sized by
 * kadllm_beam_select_workspace_fused); kadllm_beam_select_fused then selects
 * without another pass over the logits: row statistics and the threshold come
 * from the chunk statistics, and only the chunks that can hold candidates are
 * read.  Same outputs and tie rule as kadllm_beam_select (BF16, no mask). */
KADLLM_API int64_t kadllm_beam_select_workspace_fused(int64_t batch, int64_t prev_width);
KADLLM_API int kadllm_beam_select_fused(const void* logits, int64_t ld_row, const float* parent_scores,
                                        const int64_t* old_history, float* out_scores, int64_t* out_history,
                                        int32_t* out_parent, void* workspace, int64_t workspace_bytes,
                                        int64_t batch, int64_t prev_width, int64_t vocab, int64_t width,
                                        int64_t depth, void* stream);

/* Copies the workspace's flag word to *flags_out (bit 0: candidate overflow)
 * after synchronising `stream`.  The word is at offset 0 whatever the widths;
 * batch and prev_width are those the workspace was sized for. */
KADLLM_API int kadllm_beam_select_status(const void* workspace, int64_t batch, int64_t prev_width,
                                         uint32_t* flags_out, void* stream);

/* Allocation-free variant of kadllm_beam_select (no counterpart in the
 * reference).  For callers that cannot allocate device memory where they
 * select beams -- a host that hands the library only the tensors it owns, a
 * serving runtime whose memory budget is fixed when the model loads, an
 * allocator that may not grow on the decode path.  Its scratch is one 9 MiB array in the
 * library's device image, reserved on every GPU that loads the library until
 * the process exits; limits: batch <= 32 and batch * prev_width <= 512 (larger
 * sizes return KADLLM_EINVAL).  The first call on a device resolves the
 * array's address (do it before any stream capture).  All calls share the
 * array: calls whose work overlaps on the GPU race and must be serialised.
 * out_flags (device, one word) receives bit 0 = candidate overflow; the other
 * arguments and results are those of kadllm_beam_select. */
KADLLM_API int kadllm_beam_select_noalloc(const void* logits, int logits_dtype, int64_t ld_row,
                                          const float* parent_scores, const void* mask,
                                          const int64_t* old_history, float* out_scores,
                                          int64_t* out_history, uint32_t* out_flags, int64_t batch,
                                          int64_t prev_width, int64_t vocab, int64_t width,
                                          int64_t depth, void* stream);

/* ========================================================================
 * Model building blocks of the native Qwen3.5 hybrid pipeline (BF16).  Each
 * replaces a Transformers module on the reference's prefill / decode path
 * (transformers/models/qwen3_5/modeling_qwen3_5.py, called from
 * src/kadllm/adapters/qwen3_5.py:106-235).
 * ====================================================================== */

/* x = embed[ids] and normed = RMSNorm(x) * (1 + weight) (Qwen3_5RMSNorm);
 * ids [rows] int64, table [vocab, hidden], x / normed [rows, hidden]. */
KADLLM_API int kadllm_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab,
                                    const float* weight, float eps, void* x, void* normed,
                                    int64_t rows, int64_t hidden, void* stream);

/* Residual add + RMSNorm (1 + w): for i < rows, r = i*row_step + row_offset:
 * x[r] = bf16(x[r] + delta[r]) (skipped when delta is NULL), normed[i] = RMSNorm(x[r]).
 * hidden in {128, 256, 512, 1024, 2048}. */
KADLLM_API int kadllm_add_rmsnorm(void* x, const void* delta, int64_t ld_delta, const float* weight,
                                  float eps, void* normed, int64_t rows, int64_t row_step,
                                  int64_t row_offset, int64_t hidden, void* stream);

/* act[r, :] = bf16(bf16(silu(gate_up[r, :inter])) * gate_up[r, inter:2*inter]) (Qwen3_5MLP). */
KADLLM_API int kadllm_silu_mul(const void* gate_up, int64_t ld, int64_t inter, void* out,
                               int64_t rows, void* stream);

/* Attention input path: from the packed projection row [q0|gate0|q1|gate1|...|k|v]
 * (ld_proj per row) apply q_norm / k_norm (RMSNorm 1+w over head_dim) and partial
 * RoPE (cos/sin tables [positions, rotary_dim] bf16) at position
 * pos_base + (pos_of_row ? pos_of_row[r] : r % rows_per_seq), and scatter:
 * q -> q_out[r*sq_row + h*sq_h], k / v -> (k|v)_out[s*s?_seq + p*s?_pos + hk*s?_h]
 * with s = r / rows_per_seq, p = r % rows_per_seq (prefill: the prefix cache
 * [B, HK, L, D]; decode: the per-beam suffix). */
KADLLM_API int kadllm_qk_norm_rope(const void* proj, int64_t ld_proj, int64_t q_heads,
                                   int64_t kv_heads, int64_t head_dim, const float* q_weight,
                                   const float* k_weight, float eps, const void* cos_tab,
                                   const void* sin_tab, int64_t rotary_dim,
                                   const int64_t* pos_of_row, int64_t pos_base,
                                   int64_t rows_per_seq, void* q_out, int64_t sq_row, int64_t sq_h,
                                   void* k_out, int64_t sk_seq, int64_t sk_pos, int64_t sk_h,
                                   void* v_out, int64_t sv_seq, int64_t sv_pos, int64_t sv_h,
                                   int64_t rows, void* stream);

/* Prompt Gated-DeltaNet layer from the packed projection (BF16) in the WY
 * form of the chunked rule, two launches: a parallel per-(request, head,
 * 64-token chunk) preparation (causal conv + SiLU, gates, q/k L2 norm, K K^T and
 * Q K^T on the tensor cores, T = (I + L)^-1, then W = T diag(beta e^G) K and
 * U = T diag(beta) V on the tensor cores) and a sequential per-(request, head)
 * state scan (Vn = U - W S, O = e^G Q S + Aqk Vn, S <- e^{G_last} S + K'^T Vn on
 * the tensor cores, gated RMSNorm fused on the output).
 * Replaces Qwen3_5GatedDeltaNet.forward on the prompt (TF:422-533 with the
 * chunked rule TF:234-311).  proj [B*L, ld_proj] = q | k | v | z | b | a;
 * conv_weight [conv_dim, 4]; writes conv_state [B, conv_dim, 4] (last 4
 * pre-conv columns), out [B*L, ld_out] and state [B, HV, K, V] (bf16).
 * workspace >= kadllm_gdn_prefill_workspace(...) bytes, 256-byte aligned. */
KADLLM_API int64_t kadllm_gdn_prefill_workspace(int64_t batch, int64_t length, int64_t v_heads,
                                               int64_t k_dim, int64_t v_dim);
KADLLM_API int kadllm_gdn_prefill_split(const void* proj, int64_t ld_proj, const void* conv_weight,
                                        void* conv_state, const float* a_log, const float* dt_bias,
                                        const float* norm_weight, float norm_eps, void* out,
                                        int64_t ld_out, void* state, void* workspace,
                                        int64_t workspace_bytes, int64_t batch, int64_t length,
                                        int64_t heads, int64_t v_heads, int64_t k_dim, int64_t v_dim,
                                        void* stream);
/* The same over packed requests of their own lengths: request b is rows
 * [cu_seqlens[b], cu_seqlens[b+1]) of proj / out (device int32 [batch + 1],
 * total_rows = cu_seqlens[batch]); max_length sizes the workspace like
 * length above.  128-dim heads (the tensor-core scan) only. */
KADLLM_API int kadllm_gdn_prefill_split_varlen(const void* proj, int64_t ld_proj, const void* conv_weight,
                                               void* conv_state, const float* a_log, const float* dt_bias,
                                               const float* norm_weight, float norm_eps, void* out,
                                               int64_t ld_out, void* state, void* workspace,
                                               int64_t workspace_bytes, const int32_t* cu_seqlens,
                                               int64_t total_rows, int64_t batch, int64_t max_length,
                                               int64_t heads, int64_t v_heads, int64_t k_dim, int64_t v_dim,
                                               void* stream);

/* Tiled K / V prefix for the tensor-core attention (head_dim 256): per
 * (sequence, kv head) blocks of 64 positions, each a 32 KB core-matrix image
 * [8-position group][32 dim chunks][8 positions][16 bytes], zero past length.
 * src [S][HK][L][D] via element strides (seq, pos, head). */
KADLLM_API int64_t kadllm_kv_tile_bytes(int64_t seqs, int64_t kv_heads, int64_t length, int64_t head_dim);
KADLLM_API int kadllm_kv_tile(const void* src, int64_t s_seq, int64_t s_pos, int64_t s_head, int64_t seqs,
                              int64_t kv_heads, int64_t length, int64_t head_dim, void* tiles,
                              int64_t tile_bytes, void* stream);
/* Packed sequences: sequence s is positions [cu_seqlens[s], cu_seqlens[s+1])
 * of src [positions][HK][D] (strides s_pos, s_head); tiles sized for
 * max_length (kadllm_kv_tile_bytes(seqs, kv_heads, max_length, head_dim)). */
KADLLM_API int kadllm_kv_tile_varlen(const void* src, int64_t s_pos, int64_t s_head, const int32_t* cu_seqlens,
                                     int64_t seqs, int64_t kv_heads, int64_t max_length, int64_t head_dim,
                                     void* tiles, int64_t tile_bytes, void* stream);

/* Attention over a tiled prefix on tcgen05 tensor cores (head_dim 256, BF16):
 * 128 query rows per CTA, S and O in tensor memory, bulk-copied K / V blocks.
 * causal = 0: beam decode -- rows (beam, t, g) of q [B*W rows][T][Hq][D]
 *   attend to the request's prefix and their beam's suffix keys s <= t
 *   (src/kadllm/ops.py:252-341); suffix_k / suffix_v [B*W][T][HK][D]; only the
 *   suffix steps t >= first_step have query rows (and outputs): first_step =
 *   T - 1 attends the newest token alone while the earlier ones stay keys.
 * causal = 1: prompt prefill -- q rows = tokens b*L + pos, keys <= pos (SDPA in
 *   Qwen3_5Attention, TF:620-692); suffix and steps unused.
 * gate (optional): out = bf16(bf16(o) * bf16(sigmoid(gate))).  All strides in
 * elements, multiples of 8; status: device word, bit 0 = a bounded wait of the
 * kernel timed out (results invalid). */
KADLLM_API int kadllm_attention_tiled(const void* q, int64_t sq_row, int64_t sq_t, int64_t sq_h,
                                      const void* k_tiles, const void* v_tiles, int64_t blocks_per_head,
                                      const void* suffix_k, int64_t ssk_row, int64_t ssk_t, int64_t ssk_h,
                                      const void* suffix_v, int64_t ssv_row, int64_t ssv_t, int64_t ssv_h,
                                      const void* gate, int64_t sg_row, int64_t sg_t, int64_t sg_h, void* out,
                                      int64_t so_row, int64_t so_t, int64_t so_h, uint32_t* status,
                                      int64_t batch, int64_t beam_width, int64_t steps, int64_t first_step,
                                      int64_t q_heads, int64_t kv_heads, int64_t prefix_len, int64_t head_dim,
                                      float scale, int causal, void* stream);
/* The same with prompts of their own lengths: request b's prefix has
 * cu_seqlens[b+1] - cu_seqlens[b] tokens (tiles from kadllm_kv_tile_varlen with
 * max_prefix_len); causal = 1: q / gate / out rows are the packed prompt rows
 * cu_seqlens[b] + pos.  Decode rows stay (beam, t, g) per request. */
KADLLM_API int kadllm_attention_tiled_varlen(
    const void* q, int64_t sq_row, int64_t sq_t, int64_t sq_h, const void* k_tiles, const void* v_tiles,
    int64_t blocks_per_head, const void* suffix_k, int64_t ssk_row, int64_t ssk_t, int64_t ssk_h,
    const void* suffix_v, int64_t ssv_row, int64_t ssv_t, int64_t ssv_h, const void* gate, int64_t sg_row,
    int64_t sg_t, int64_t sg_h, void* out, int64_t so_row, int64_t so_t, int64_t so_h, uint32_t* status,
    const int32_t* cu_seqlens, int64_t batch, int64_t beam_width, int64_t steps, int64_t first_step,
    int64_t q_heads, int64_t kv_heads, int64_t max_prefix_len, int64_t head_dim, float scale, int causal,
    void* stream);

/* Decode attention split over the prefix's key blocks, for launches with fewer
 * CTAs than SMs (a few requests, long prefixes: the kernel microbenchmark's one
 * request x 256 beams against 4096 keys): `splits` CTAs per row tile each take a
 * run of key blocks and write their unnormalised output and (maximum, sum) to
 * `workspace` (>= kadllm_attention_split_workspace(...) bytes, 16-byte
 * aligned); a combine kernel merges the runs, the beam's suffix keys and the
 * output gate.  Arguments as kadllm_attention_tiled (decode, causal = 0). */
KADLLM_API int64_t kadllm_attention_split_workspace(int64_t batch, int64_t beam_width, int64_t steps,
                                                    int64_t first_step, int64_t q_heads, int64_t splits);
KADLLM_API int kadllm_attention_tiled_split(const void* q, int64_t sq_row, int64_t sq_t, int64_t sq_h,
                                            const void* k_tiles, const void* v_tiles, int64_t blocks_per_head,
                                            const void* suffix_k, int64_t ssk_row, int64_t ssk_t, int64_t ssk_h,
                                            const void* suffix_v, int64_t ssv_row, int64_t ssv_t, int64_t ssv_h,
                                            const void* gate, int64_t sg_row, int64_t sg_t, int64_t sg_h, void* out,
                                            int64_t so_row, int64_t so_t, int64_t so_h, uint32_t* status,
                                            int64_t batch, int64_t beam_width, int64_t steps, int64_t first_step,
                                            int64_t q_heads, int64_t kv_heads, int64_t prefix_len, int64_t head_dim,
                                            float scale, int64_t splits, void* workspace, int64_t workspace_bytes,
                                            void* stream);

/* Prompt causal GQA attention (flash loop on the tensor cores) with the fused
 * output gate out = bf16(o) * bf16(sigmoid(gate)) (gate may be NULL).
 * q [B*L rows, H, D] (sq_row, sq_h); k / v [B, HK, L, D] via (s?_b, s?_l, s?_h);
 * gate rows / heads (sg_row, sg_h); out (so_row, so_h). */
KADLLM_API int kadllm_causal_attention(const void* q, int64_t sq_row, int64_t sq_h, const void* k,
                                       int64_t sk_b, int64_t sk_l, int64_t sk_h, const void* v,
                                       int64_t sv_b, int64_t sv_l, int64_t sv_h, const void* gate,
                                       int64_t sg_row, int64_t sg_h, void* out, int64_t so_row,
                                       int64_t so_h, int64_t batch, int64_t length, int64_t heads,
                                       int64_t kv_heads, int64_t head_dim, float scale,
                                       void* stream);

/* Projection GEMM on tcgen05 tensor cores (CTA pairs, tensor-map copies, FP32
 * accumulation in tensor memory): the product C = A . B^T of
 * torch.nn.functional.linear(A, B) for every nn.Linear of the decoder and the
 * LM head (Qwen3_5GatedDeltaNet / Qwen3_5Attention / Qwen3_5MLP projections and
 * lm_head, as src/kadllm/adapters/qwen3_5.py:144-202,226-235 calls them).
 *   A [M, K] bf16, row stride lda;  B [N, K] bf16, row stride ldb;  strides
 *   multiples of 8 elements, pointers 16-byte aligned.  The output row width
 *   (N, or n_out for epilogue 1) is a multiple of 8: C is written in 16-byte
 *   granules, and nothing past the row end inside a padded row is touched.
 * epilogue 0: C [M, N] = bf16(A . B^T)                                   (ldc)
 * epilogue 1: B's rows are 128-row blocks [gate block j | up block j] (N a
 *   multiple of 256); C [M, n_out] = bf16(bf16(silu(gate)) * up), gate and up
 *   rounded to bf16 first -- Qwen3_5MLP's act_fn(gate_proj(x)) * up_proj(x)
 * epilogue 2: C = bf16(resid + bf16(A . B^T)), resid [M, N] (ld_resid) may be C:
 *   the decoder's residual update x = x + f(x)
 * status: device word, bit 0 = a bounded wait of the kernel timed out. */
KADLLM_API int kadllm_gemm(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                           const void* resid, int64_t ld_resid, int64_t M, int64_t N, int64_t K, int64_t n_out,
                           int epilogue, uint32_t* status, void* stream);
/* The LM head of a decode step for the fused selection: logits [M = batch *
 * prev_width, N = vocabulary] = A . B^T (BF16), plus each row's chunk statistics
 * into `workspace` (>= kadllm_beam_select_workspace_fused(batch, prev_width)
 * bytes, 256-byte aligned); N a multiple of 8, at most 393216. */
KADLLM_API int kadllm_gemm_logits(const void* a, int64_t lda, const void* b, int64_t ldb, void* logits,
                                  int64_t ld_logits, int64_t M, int64_t N, int64_t K, void* workspace,
                                  int64_t workspace_bytes, int64_t batch, int64_t prev_width, uint32_t* status,
                                  void* stream);

/* Beam reorder as index work: dst row i = src row (i / group) * src_group + index[i]
 * (index clamped to [0, src_group)), row_bytes per row; strides in BYTES, multiples
 * of 16.  Gathers a previous decode step's per-beam rows (projections, suffix K / V)
 * by parent beam, as the reference's history.gather does for the tokens
 * (src/kadllm/grbeam.py:102-104). */
KADLLM_API int kadllm_gather_rows(const void* src, int64_t ld_src, const int32_t* index, int64_t group,
                                  int64_t src_group, int64_t rows, int64_t row_bytes, void* dst, int64_t ld_dst,
                                  void* stream);

/* GDN decode mixer continuing a beam's suffix from the previous decode step (step
 * reuse at T = 2; no separate counterpart in the reference, which replays both
 * suffix tokens from the prefix, src/kadllm/adapters/qwen3_5.py:144-177): beam j
 * of request b has the suffix [token of previous-step beam parent[b*W + j], new
 * token]; proj_prev [B*prev_width, ld_proj] holds the previous step's projection
 * rows (as kadllm_gdn_mixer_replay takes them at T = 1), proj [B*W, ld_proj] the
 * new tokens' rows, out [B*W, HV*V] the new token's mixer output -- the same
 * values kadllm_gdn_mixer_replay gives for that token at T = 2 without
 * recomputing the first token's projection.  Head dims 64 / 128 (K == V).
 * records: null (the first token is replayed from proj_prev), or the previous
 * step's records (kadllm_gdn_mixer_replay, indexed like proj_prev): the first
 * token's delta comes from them (its k and decay are recomputed from proj_prev)
 * and only the new token runs against the state. */
KADLLM_API int kadllm_gdn_mixer_continue(const void* proj_prev, const int32_t* parent, int64_t prev_width,
                                         const void* proj, int64_t ld_proj, const void* conv_state,
                                         int64_t conv_hist, const void* conv_weight, const void* rec_state,
                                         const float* a_log, const float* dt_bias, const float* norm_weight,
                                         float norm_eps, void* out, int64_t batch, int64_t beam_width,
                                         int64_t heads, int64_t v_heads, int64_t k_dim, int64_t v_dim,
                                         const void* records, uint32_t* status, void* stream);

/* Diagnostics: one CTA runs the tensor-core kernels' bounded mbarrier wait on a
 * barrier nothing completes, giving up after max_cycles SM clocks (1 .. 2^32)
 * and setting bit 0 of *status, as those kernels report a timed-out wait. */
KADLLM_API int kadllm_diag_wait_timeout(uint32_t* status, int64_t max_cycles, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KADLLM_B200_H_ */
