/*
 * qwen_fused.h -- C ABI of libqwen_fused.so, the sm_100a (B200) drop-in for
 * the reference's fused_kernels library.
 *
 * The reference loader opens it through QWEN_FUSED_DLL (main.py:113-118) and
 * binds the reference-named symbols with the argtypes of main.py:119-240, so
 * those keep the reference's exact signatures and `void` return.  Cited lines
 * are in qwen3_infer/csrc/fused_kernels.cu unless a file is named.
 *
 * Conventions (unchanged from the reference): every pointer is a device
 * pointer owned by the caller; bf16 = __nv_bfloat16 passed as void*; weights
 * are E4M3 bytes [N, K] row-major; the int K_blk encodes the scale layout
 * (>1: block scales [ceil(N/128), K_blk]; 1: per-row [N, 1]; <0: per-row
 * per-128-K-block [N, -K_blk]; main.py:249-251).  Launches are asynchronous
 * on `stream`; nothing synchronises.
 *
 * Differences: arguments are validated; on invalid input nothing is launched
 * and the error is kept for qwen_last_error().  The new entry points return
 * an int status (0 = success, otherwise a cudaError_t value).
 */
#ifndef QWEN_FUSED_H
#define QWEN_FUSED_H

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference-named exports ------------------------------------------ */

/* y[N] = bf16(x . dequant(W)^T).  Replaces launch_gemv_v4_extern (1328-1336). */
void launch_gemv_v4_extern(const void* x, const void* w, const void* s, void* y, int N, int K, int K_blk,
                           cudaStream_t stream);
/* Same math; replaces launch_gemv_v3_extern (981-989). */
void launch_gemv_v3_extern(const void* x, const void* w, const void* s, void* y, int N, int K, int K_blk,
                           cudaStream_t stream);
/* Four GEMVs sharing x, one launch.  Replaces launch_linear_in_proj4 (1338-1354). */
void launch_linear_in_proj4(const void* x, const void* w0, const void* s0, void* y0, int n0, int kb0,
                            const void* w1, const void* s1, void* y1, int n1, int kb1, const void* w2,
                            const void* s2, void* y2, int n2, int kb2, const void* w3, const void* s3, void* y3,
                            int n3, int kb3, int K, cudaStream_t stream);
/* q/k/v GEMVs sharing x (N_*_blk unused, as in the reference).  Replaces launch_fused_qkv (991-1007). */
void launch_fused_qkv(const void* x, const void* w_q, const void* w_k, const void* w_v, const void* s_q,
                      const void* s_k, const void* s_v, void* q_out, void* k_out, void* v_out, int K, int N_q,
                      int N_k, int N_v, int K_blk, int N_q_blk, int N_k_blk, int N_v_blk, cudaStream_t stream);
/* gate/up GEMVs sharing x.  Replaces launch_fused_gate_up (1009-1025). */
void launch_fused_gate_up(const void* x, const void* w_gate, const void* w_up, const void* s_gate, const void* s_up,
                          void* gate_out, void* up_out, int K, int N_gate, int N_up, int K_blk, int N_gate_blk,
                          int N_up_blk, cudaStream_t stream);
/* In-place RMSNorm(1+w), FP32 weight, N rows of D.  Replaces launch_rmsnorm_ip (1055-1062). */
void launch_rmsnorm_ip(void* x, const void* weight, int N, int D, float eps, cudaStream_t stream);
/* Out-of-place RMSNorm(1+w).  Replaces launch_rmsnorm_out (1045-1053). */
void launch_rmsnorm_out(const void* x, const void* weight, void* out, int N, int D, float eps,
                        cudaStream_t stream);
/* norm_ws = RMSNorm(hidden); q/k/v GEMVs of norm_ws.  Replaces layer_pre_attn (1066-1091). */
void layer_pre_attn(const void* hidden, const float* norm_weight, const void* w_q, const void* s_q, int N_q,
                    int N_q_blk, const void* w_k, const void* s_k, int N_k, int N_k_blk, const void* w_v,
                    const void* s_v, int N_v, int N_v_blk, void* q_out, void* k_out, void* v_out, void* norm_ws,
                    int h_dim, int K_blk, cudaStream_t stream);
/* output = hidden + O(attn); MLP with residual.  Replaces layer_post_attn (1102-1150). */
void layer_post_attn(const void* hidden, const void* attn_out, const void* w_o, const void* s_o, int N_o,
                     int N_o_blk, const float* norm_weight, const void* w_g, const void* s_g, int N_g, int N_g_blk,
                     const void* w_u, const void* s_u, int N_u, int N_u_blk, const void* w_d, const void* s_d,
                     int N_d, int N_d_blk, void* output, void* ws, void* gate_buf, void* up_buf, void* silu_buf,
                     int h_dim, int attn_dim, int K_blk_o, int K_blk_gu, int K_blk_d, cudaStream_t stream);
/* output = hidden + o_out; MLP with residual.  Replaces layer_post_o_fp8_mlp (1156-1195). */
void layer_post_o_fp8_mlp(const void* hidden, const void* o_out, const float* norm_weight, const void* w_g,
                          const void* s_g, int N_g, const void* w_u, const void* s_u, int N_u, const void* w_d,
                          const void* s_d, int N_d, void* output, void* ws, void* gate_buf, void* up_buf,
                          void* silu_buf, int h_dim, int K_blk_gu, int K_blk_d, cudaStream_t stream);
/* Gated delta-rule decode, FP32 state in place, head_dim 64 or 128.  Replaces launch_delta_rule_decode (967-979). */
void launch_delta_rule_decode(const void* q, const void* k, const void* v, const void* g, const void* beta,
                              void* state, void* output, int n_heads, int head_dim, cudaStream_t stream);
/* g = -exp(A_log)*softplus(a+dt_bias), beta = sigmoid(b).  Replaces launch_prepare_linear_gates (942-954). */
void launch_prepare_linear_gates(const void* a, const void* beta_in, const float* A_log, const float* dt_bias,
                                 void* g_out, void* beta_out, int heads, cudaStream_t stream);
/* RMSNorm(core)*w*silu(z) per head, FP32.  Replaces launch_rmsnorm_gated_decode (956-965). */
void launch_rmsnorm_gated_decode(const void* core, const void* z, const void* weight, void* out, int heads,
                                 int head_dim, float eps, cudaStream_t stream);
/* Single-query GQA attention over seq_len cached positions.  Replaces launch_fused_attn_v2 (1300-1326). */
void launch_fused_attn_v2(const void* q, const void* k_cache, const void* v_cache, void* output, int seq_len,
                          int max_seq_len, int head_dim, int n_heads, int n_kv_heads, cudaStream_t stream);
/* Same math.  Replaces launch_fused_attn (1027-1043). */
void launch_fused_attn(const void* q, const void* k_cache, const void* v_cache, void* output, int seq_len,
                       int max_seq_len, int head_dim, int n_heads, int n_kv_heads, cudaStream_t stream);
/* Q/K norm + RoPE in place, KV write at past_len, attention.  Replaces layer_mid_attn (1224-1297). */
void layer_mid_attn(void* q_buf, void* k_buf, const void* v_buf, void* attn_out, const float* q_norm_weight,
                    const float* k_norm_weight, const float* cos_table, const float* sin_table, void* k_cache,
                    void* v_cache, int pos, int past_len, int total_seq, int max_seq_len, int head_dim,
                    int rotary_dim, int n_heads, int n_kv_heads, cudaStream_t stream);

/* ---- status (new) --------------------------------------------------------- */

/* Last error recorded by a call on this host thread, then cleared (0 = none). */
int qwen_last_error(void);
/* Read and clear the device error word (first error wins): 1-4 a bounded wait
 * on a copy or a stage timed out, 5 a device-side cache position outside
 * [0, max_seq), 6 a tensor-parallel peer exchange timed out, 7 a K-slice
 * count outside [1, max_slices]. */
int qwen_get_device_error(unsigned int* out);
/* Limit in ns of the waits on other CTAs or ranks (step-kernel stage
 * counters, tensor-parallel peer flags): 1e6 .. 2e9, or 0 for the default
 * 2e9.  A wait that runs out records its error code above and gives up; the
 * launch returns and the context stays usable. */
int qwen_set_wait_timeout_ns(unsigned long long ns);
/* Enable (default) or disable programmatic dependent launch in the engine entry points. */
void qwen_set_pdl(int enable);
/* Up to four device regions (null / 0 ignored; 16-byte aligned) that the next
 * engine launch issued on this host thread pulls into L2 while it runs --
 * normally the weights of the launch after it.  New; no reference counterpart. */
void qwen_set_prefetch(const void* p0, unsigned long long n0, const void* p1, unsigned long long n1,
                       const void* p2, unsigned long long n2, const void* p3, unsigned long long n3);
int qwen_abi_version(void);

/* ---- new compute entry points --------------------------------------------- */

/* launch_gemv_v4_extern with FP32 scales.  New; the FP32 weight_scale_inv the
 * reference rounds to BF16 at load (main.py:597). */
int launch_gemv_f32s(const void* x, const void* w, const float* s, void* y, int N, int K, int K_blk,
                     cudaStream_t stream);
/* Same GEMV through the generic one-warp-per-row kernel (coverage of the fallback). */
int qwen_gemv_generic(const void* x, const void* w, const void* s, int scale_f32, void* y, int N, int K, int K_blk,
                      cudaStream_t stream);
/* Final RMSNorm(1+w) (norm_w nullable) + LM-head GEMV + greedy argmax over rows
 * [row_offset, row_offset+N).  Replaces the LM head of forward (main.py:1599-1603)
 * and the caller's logits.argmax() (_benchmark_native_fp8.py:33).  ws: 16 bytes,
 * zero before first use, left zeroed.  key_out = orderable(bf16 max) << 32 |
 * (0xFFFFFFFF - index); token_out = first maximal index; each output nullable. */
int launch_lm_head_argmax(const void* x, const float* norm_w, float eps, const void* w, const void* s, int N, int K,
                          int K_blk, int row_offset, void* ws, unsigned long long* key_out, long long* token_out,
                          void* logits_out, int* pos_inc, cudaStream_t stream);
/* hidden = embed[*token] (F.embedding of forward, main.py:1587). */
int qwen_embed(const void* embed, const long long* token, void* hidden, int H, cudaStream_t stream);
/* RMSNorm + q/k/v GEMVs of a full-attention layer (main.py:1521-1524, 994-999). */
int qwen_attn_in_proj(const void* hidden, const float* norm_w, float eps, const void* w_q, const void* s_q, int N_q,
                      const void* w_k, const void* s_k, int N_k, const void* w_v, const void* s_v, int N_v, int K,
                      int K_blk, void* q_out, void* k_out, void* v_out, cudaStream_t stream);
/* RMSNorm + GatedDeltaNet input projections with the conv1d update / SiLU and
 * gate math fused into the epilogues (main.py:1079-1122). */
int qwen_gdn_in_proj(const void* hidden, const float* norm_w, float eps, int K, int K_blk, const void* w_qkv,
                     const void* s_qkv, int N_qkv, const void* conv_w, void* conv_state, int conv_width,
                     void* qkv_out, const void* w_z, const void* s_z, int N_z, void* z_out, const void* w_a,
                     const void* s_a, const void* w_b, const void* s_b, int N_heads, const float* A_log,
                     const float* dt_bias, float* g_out, void* beta_out, cudaStream_t stream);
/* Delta rule + RMSNormGated from the post-conv [q|k|v] (main.py:1124-1159, 623-684). */
int qwen_gdn_decode(const void* qkv, const float* g, const void* beta, float* state, const void* z,
                    const void* norm_w, float eps, void* out, int n_k_heads, int n_v_heads, int head_dim,
                    cudaStream_t stream);
/* GatedDeltaNet recurrent step writing the un-normed core output (value
 * columns of a head over 4 CTAs); the gated norm then runs in the next
 * GEMV's prologue after qwen_set_gated_input.  No counterpart in the
 * reference (its gated norm is a separate kernel, 592-618). */
int qwen_gdn_decode_core(const void* qkv, const float* g, const void* beta, float* state, void* core_out,
                         int n_k_heads, int n_v_heads, int head_dim, cudaStream_t stream);
/* The next launch without a prologue on this host thread (qwen_linear_resid,
 * qwen_linear_partial, qwen_linear_partial_p2p) applies RMSNormGated per
 * 128-wide head to its x: z like x, norm_w [128] BF16 (main.py:1152-1159). */
int qwen_set_gated_input(const void* z, const void* norm_w, float eps);
/* y = bf16(res + bf16(W x)): o_proj / out_proj / down with the residual add (553-559). */
int qwen_linear_resid(const void* x, const void* w, const void* s, int N, int K, int K_blk, const void* res, void* y,
                      cudaStream_t stream);
/* Replaces the residual-add launch pair of the same projections (553-559) on
 * one GPU: W x as per-K-slice FP32 partial rows slices[c][r], c < *count
 * (count <= max_slices, written by the launch), with no reduction of its own.
 * The next RMSNorm-prologue launch on this host thread, after
 * qwen_set_slices_input(slices, count, n, max_slices, res), builds its input
 * as bf16(res + bf16(sum of the slices in order)), writes it to the buffer
 * passed as its x (the residual stream) and normalises it.  Tensor-core path
 * only (128x128 block scales, K a multiple of 128, K >= 256, at least
 * ceil(K / 4096) slices allowed): otherwise cudaErrorNotSupported, nothing
 * launched. */
int qwen_linear_slices(const void* x, const void* w, const void* s, int N, int K, int K_blk, float* slices,
                       int* count, int max_slices, cudaStream_t stream);
int qwen_set_slices_input(const float* slices, const int* count, int n, int max_slices, const void* res);
/* Tensor parallelism (row/column sharding of the decode step across GPUs;
 * the reference has no multi-GPU path, these replace nothing):
 * y_f32 = this rank's partial GEMV over its slice of K, to be all-reduced. */
int qwen_linear_partial(const void* x, const void* w, const void* s, int N, int K, int K_blk, float* y,
                        cudaStream_t stream);
/* y = bf16(res + bf16(v)) for n elements, v the all-reduced partial sums. */
int qwen_resid_add_f32(const void* res, const float* v, void* y, int n, cudaStream_t stream);
/* Writes {*token, ++*seq} to host_out (pinned host memory the device can
 * write, e.g. cudaHostAlloc under unified addressing): the token first, the
 * sequence number after a system-scope fence, so a host thread polling the
 * sequence number reads the matching token.  No counterpart in the reference. */
int qwen_publish_token(const long long* token, long long* host_out, unsigned long long* seq, cudaStream_t stream);
/* token = the greedy token id encoded in an all-reduced packed argmax key. */
int qwen_token_from_key(const long long* key, long long* token, cudaStream_t stream);
/* Tensor parallelism without a library collective: the partial sums and the
 * argmax keys are exchanged through a per-rank region mapped into every rank
 * with CUDA IPC (flags, key slots, counters, 2 x world x n FP32 buffers).
 * qwen_p2p_create allocates and zeroes this rank's region and writes its
 * 64-byte IPC handle; qwen_p2p_open maps a peer's; qwen_p2p_table builds the
 * device table from all regions (bases[rank] = own) for n-element sums. */
int qwen_p2p_create(int world, int n, void** base_out, void* ipc_handle_out);
int qwen_p2p_open(const void* ipc_handle, void** peer_base_out);
int qwen_p2p_close(void* peer_base);
int qwen_p2p_destroy(void* base);
int qwen_p2p_table(void* const* bases, int world, int rank, int n, void** table_out);
int qwen_p2p_table_free(void* table);
/* The next RMSNorm-prologue launch on this host thread (qwen_attn_in_proj,
 * qwen_gdn_in_proj, qwen_mlp_gate_up, launch_lm_head_argmax) builds its input
 * as bf16(res + bf16(sum of the ranks' n-element partials)) after waiting for
 * every rank's partial (bounded), writes it to the buffer passed as its x,
 * and normalises it; the launch then advances the exchange round. */
int qwen_set_p2p_input(const void* table, const void* res, int n);
/* This rank's partial GEMV, stored into slot [rank] of every rank's buffer. */
int qwen_linear_partial_p2p(const void* x, const void* w, const void* s, int N, int K, int K_blk, const void* table,
                            cudaStream_t stream);
/* y = bf16(res + bf16(sum of the ranks' partials)) once all have arrived (bounded wait). */
int qwen_resid_add_p2p(const void* table, const void* res, void* y, int n, cudaStream_t stream);
/* token = greedy token over every rank's packed argmax key (bounded wait). */
int qwen_token_p2p(const void* table, const long long* key, long long* token, cudaStream_t stream);
/* silu_out = bf16(silu(g)*u), g/u = GEMVs of RMSNorm(h2) (398-479, 1173-1190). */
int qwen_mlp_gate_up(const void* h2, const float* norm_w, float eps, const void* w_g, const void* s_g,
                     const void* w_u, const void* s_u, int N, int K, int K_blk, void* silu_out, cudaStream_t stream);
/* Full-attention decode with the position on the device: norm, RoPE, KV write,
 * split-KV attention and sigmoid gate (1224-1297, main.py:1001-1059).
 * The pos + 1 cached positions are spread over nsplit splits (CTAs per KV
 * head), at least chunk positions each.
 * ws_part: n_heads*nsplit*(head_dim+2) floats; ws_count: n_kv_heads zeroed uints. */
int qwen_attn_decode(const void* q_all, const void* k_new, const void* v_new, const float* q_norm,
                     const float* k_norm, const float* cos, const float* sin, void* k_cache, void* v_cache,
                     const int* pos, int max_seq, int n_heads, int n_kv_heads, int head_dim, int rotary_dim,
                     float eps, int chunk, int nsplit, float* ws_part, unsigned* ws_count, void* out,
                     cudaStream_t stream);

/* qwen_attn_decode without caller-provided scratch: no counterpart in the
 * reference.  For callers that cannot allocate device memory where they decode
 * (a runtime whose pool owns the GPU, a binding without a device allocator,
 * code that must avoid an allocation's implicit synchronisation).  The split
 * partials and counters live in a 4 MiB array compiled into the library:
 * 256-byte-rounded n_heads*nsplit*(head_dim+2)*4 bytes + 4*n_kv_heads bytes
 * must fit, else cudaErrorInvalidValue and nothing is launched.  The first
 * call on a device looks the array's address up for that device (make it
 * before any stream capture); calls share the array, so calls that may run
 * concurrently on the GPU race; the counters are cleared on `stream` before
 * each launch.  No cudaMalloc/cudaFree. */
int qwen_attn_decode_noalloc(const void* q_all, const void* k_new, const void* v_new, const float* q_norm,
                             const float* k_norm, const float* cos, const float* sin, void* k_cache, void* v_cache,
                             const int* pos, int max_seq, int n_heads, int n_kv_heads, int head_dim, int rotary_dim,
                             float eps, int chunk, int nsplit, void* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_FUSED_H */
