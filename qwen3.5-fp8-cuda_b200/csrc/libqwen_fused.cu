// libqwen_fused.so: drop-in replacement for the reference's fused_kernels
// library (the `QWEN_FUSED_DLL` the reference loader opens, main.py:113-118)
// plus the new decode-engine entry points.  Declarations: include/qwen_fused.h.
//
// Reference-named exports keep the exact C signatures, argument order and
// `void` return of qwen3_infer/csrc/fused_kernels.cu so main.py's argtypes
// bind unchanged; unlike the reference they validate their arguments and
// launch nothing on invalid input (the error is readable through
// qwen_last_error()).  New exports return an int status (0 = success,
// otherwise a cudaError_t value).
#include "common.cuh"
#include "gemv_host.cuh"
#include "norm.cuh"
#include "gdn.cuh"
#include "attn.cuh"

#include <cstdint>

using namespace qwen;

namespace {

thread_local int g_last_error = 0;
int g_pdl_enabled = 1;
// Regions the next engine launch on this host thread prefetches into L2
// (set by qwen_set_prefetch, consumed and cleared by that launch).
thread_local L2Prefetch g_next_pf = {};

inline L2Prefetch take_prefetch() {
  L2Prefetch pf = g_next_pf;
  g_next_pf = L2Prefetch{};
  return pf;
}

// Tensor-parallel input of the next RMSNorm-prologue launch on this host
// thread (set by qwen_set_p2p_input, consumed and cleared by that launch):
// the launch builds its x as bf16(res + bf16(sum of the ranks' partials)),
// writes it to the buffer it was given as x, and normalises it.
thread_local const void* g_p2p_table = nullptr;
thread_local const void* g_p2p_res = nullptr;
thread_local int g_p2p_n = 0;

// GatedDeltaNet gated norm of the next PRO_NONE launch on this host thread
// (set by qwen_set_gated_input, consumed and cleared by that launch).
thread_local const void* g_gz = nullptr;
thread_local const void* g_gw = nullptr;
thread_local float g_geps = 0.f;

inline cudaError_t take_gated_input(GemvArgs& a) {
  if (!g_gz) return cudaSuccess;
  const void* z = g_gz;
  const void* w = g_gw;
  const float eps = g_geps;
  g_gz = g_gw = nullptr;
  if (a.pro != PRO_NONE || a.K % 128 != 0 || a.xn_out || a.h2_out || a.x_row) return cudaErrorInvalidValue;
  a.pro = PRO_GATED_NORM;
  a.gz = static_cast<const bf16*>(z);
  a.gw = static_cast<const bf16*>(w);
  a.eps = eps;
  return cudaSuccess;
}

// Single-GPU sliced input of the next RMSNorm-prologue launch on this host
// thread (set by qwen_set_slices_input, consumed and cleared by that launch):
// the launch builds its x as bf16(res + bf16(sum of the previous launch's
// K-slice rows)), writes it to the buffer it was given as x, and normalises it.
thread_local const float* g_sl_buf = nullptr;
thread_local const int* g_sl_count = nullptr;
thread_local const void* g_sl_res = nullptr;
thread_local int g_sl_n = 0;
thread_local int g_sl_max = 0;

inline cudaError_t take_slices_input(GemvArgs& a) {
  if (!g_sl_buf) return cudaSuccess;
  const float* b = g_sl_buf;
  const int* c = g_sl_count;
  const void* r = g_sl_res;
  const int n = g_sl_n, mx = g_sl_max;
  g_sl_buf = nullptr;
  g_sl_count = nullptr;
  g_sl_res = nullptr;
  g_sl_n = g_sl_max = 0;
  if (a.pro != PRO_RMSNORM || n != a.K || a.xn_out || a.h2_out || a.x_row) return cudaErrorInvalidValue;
  a.pro = PRO_SLICES_RMSNORM;
  a.sl_buf = b;
  a.sl_count = c;
  a.sl_n = n;
  a.sl_max = mx;
  a.h2_out = const_cast<bf16*>(a.x);
  a.x = static_cast<const bf16*>(r);
  return cudaSuccess;
}

inline cudaError_t take_p2p_input(GemvArgs& a) {
  if (g_sl_buf && g_p2p_table) {  // one pending input at a time: drop both
    g_sl_buf = nullptr;
    g_p2p_table = nullptr;
    return cudaErrorInvalidValue;
  }
  if (!g_p2p_table) return take_slices_input(a);
  const void* t = g_p2p_table;
  const void* r = g_p2p_res;
  const int n = g_p2p_n;
  g_p2p_table = g_p2p_res = nullptr;
  g_p2p_n = 0;
  if (a.pro != PRO_RMSNORM || n != a.K || a.xn_out || a.h2_out || a.x_row) return cudaErrorInvalidValue;
  a.pro = PRO_P2P_RMSNORM;
  a.p2p = static_cast<const P2PTable*>(t);
  a.h2_out = const_cast<bf16*>(a.x);
  a.x = static_cast<const bf16*>(r);
  return cudaSuccess;
}

inline int record(cudaError_t e) {
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) g_last_error = (int)e;
  return (int)e;
}

inline bool engine_pdl() { return g_pdl_enabled != 0; }

inline GemvSeg seg(const void* w, const void* s, void* y, int n, int kblk, int epi = EPI_STORE) {
  return make_seg(w, s, y, n, kblk, epi);
}

// layer_post_* MLP tail shared by the two composite entry points:
// gate/up/SiLU from `h2` (already holding hidden + attention output) and the
// down projection with the residual add, in place on `h2`.
int mlp_tail(const void* h2_src_a, const void* h2_src_b, const float* norm_w, const void* w_g, const void* s_g,
             const void* w_u, const void* s_u, int N_g, const void* w_d, const void* s_d, int N_d, void* output,
             void* ws, void* gate_buf, void* up_buf, void* silu_buf, int h_dim, int kblk_gu, int kblk_d,
             cudaStream_t st) {
  GemvArgs a = make_args(h2_src_a, h_dim);
  if (h2_src_b) {
    a.pro = PRO_ADD_RMSNORM;
    a.x2 = static_cast<const bf16*>(h2_src_b);
    a.h2_out = static_cast<bf16*>(output);
  } else {
    a.pro = PRO_RMSNORM;
  }
  a.norm_w = norm_w;
  a.eps = 1e-6f;
  a.nseg = 1;
  a.seg[0] = seg(w_g, s_g, silu_buf, N_g, kblk_gu, EPI_SILU_PAIR);
  a.seg[0].w2 = static_cast<const uint8_t*>(w_u);
  a.seg[0].s2 = s_u;
  a.seg[0].y2 = gate_buf;
  a.seg[0].y3 = up_buf;
  int e = record(gemv_run(a, false, st, false));
  if (e) return e;
  GemvArgs d = make_args(silu_buf, N_g);
  d.nseg = 1;
  d.seg[0] = seg(w_d, s_d, output, N_d, kblk_d, EPI_RESID);
  d.seg[0].aux0 = output;
  d.seg[0].y2 = ws;
  return record(gemv_run(d, false, st, false));
}

}  // namespace

// Tensor-parallel exchange helpers (used by the qwen_p2p_* / *_p2p exports).
static size_t p2p_region_bytes(int world, int n) { return P2P_DATA_OFF + 2ull * world * n * sizeof(float); }
static cudaError_t launch_small(const void* kern, int grid, int block, void** args, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = engine_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

extern "C" {

// ---------------------------------------------------------------------------
// Status and configuration
// ---------------------------------------------------------------------------
int qwen_last_error(void) {
  const int e = g_last_error;
  g_last_error = 0;
  return e;
}

int qwen_set_wait_timeout_ns(unsigned long long ns) {
  if (ns == 0) ns = QWEN_WAIT_TIMEOUT_NS;
  if (ns < 1000000ull || ns > QWEN_WAIT_TIMEOUT_NS) return record(cudaErrorInvalidValue);
  return record(cudaMemcpyToSymbol(g_qwen_wait_ns, &ns, sizeof(ns)));
}

int qwen_get_device_error(unsigned int* out) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_qwen_err, sizeof(v));
  if (e == cudaSuccess) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_qwen_err, &zero, sizeof(zero));
  }
  if (out) *out = v;
  return (int)e;
}

void qwen_set_pdl(int enable) { g_pdl_enabled = enable; }

// Weight regions (up to four; null / 0 entries ignored) that the next engine
// launch issued on this host thread pulls into L2 while it runs -- normally
// the weights of the launch after it.  Sizes are rounded down to 16 bytes.
// The next RMSNorm-prologue launch on this host thread takes its input from
// the tensor-parallel exchange `table` (n-element partial sums) plus the
// residual `res` (see take_p2p_input).
// The next launch without a prologue on this host thread (an out_proj after
// qwen_gdn_decode_core) applies the GatedDeltaNet gated RMSNorm to its x per
// 128-wide head: z [like x], norm weight [128] BF16.
int qwen_set_gated_input(const void* z, const void* norm_w, float eps) {
  if (!z || !norm_w) return record(cudaErrorInvalidValue);
  g_gz = z;
  g_gw = norm_w;
  g_geps = eps;
  return 0;
}

int qwen_set_slices_input(const float* slices, const int* count, int n, int max_slices, const void* res) {
  if (!slices || !count || !res || n <= 0 || max_slices < 1) return record(cudaErrorInvalidValue);
  g_sl_buf = slices;
  g_sl_count = count;
  g_sl_res = res;
  g_sl_n = n;
  g_sl_max = max_slices;
  return 0;
}

int qwen_set_p2p_input(const void* table, const void* res, int n) {
  if (!table || !res || n <= 0) return record(cudaErrorInvalidValue);
  g_p2p_table = table;
  g_p2p_res = res;
  g_p2p_n = n;
  return 0;
}

void qwen_set_prefetch(const void* p0, unsigned long long n0, const void* p1, unsigned long long n1,
                       const void* p2, unsigned long long n2, const void* p3, unsigned long long n3) {
  const void* p[4] = {p0, p1, p2, p3};
  const unsigned long long n[4] = {n0, n1, n2, n3};
  for (int i = 0; i < 4; ++i) {
    const bool ok = p[i] && (reinterpret_cast<uintptr_t>(p[i]) & 15u) == 0;
    g_next_pf.p[i] = ok ? p[i] : nullptr;
    g_next_pf.n[i] = ok ? (n[i] & ~15ull) : 0ull;
  }
}

int qwen_abi_version(void) { return 1; }

// ---------------------------------------------------------------------------
// Reference-compatible exports (fused_kernels.cu:940-1356)
// ---------------------------------------------------------------------------
void launch_gemv_v4_extern(const void* x, const void* w, const void* s, void* y, int N, int K, int K_blk,
                           cudaStream_t stream) {
  GemvArgs a = make_args(x, K);
  a.nseg = 1;
  a.seg[0] = seg(w, s, y, N, K_blk);
  record(gemv_run(a, false, stream, false));
}

void launch_gemv_v3_extern(const void* x, const void* w, const void* s, void* y, int N, int K, int K_blk,
                           cudaStream_t stream) {
  launch_gemv_v4_extern(x, w, s, y, N, K, K_blk, stream);
}

void launch_linear_in_proj4(const void* x, const void* w0, const void* s0, void* y0, int n0, int kb0,
                            const void* w1, const void* s1, void* y1, int n1, int kb1, const void* w2,
                            const void* s2, void* y2, int n2, int kb2, const void* w3, const void* s3, void* y3,
                            int n3, int kb3, int K, cudaStream_t stream) {
  GemvArgs a = make_args(x, K);
  a.nseg = 4;
  a.seg[0] = seg(w0, s0, y0, n0, kb0);
  a.seg[1] = seg(w1, s1, y1, n1, kb1);
  a.seg[2] = seg(w2, s2, y2, n2, kb2);
  a.seg[3] = seg(w3, s3, y3, n3, kb3);
  record(gemv_run(a, false, stream, false));
}

void launch_fused_qkv(const void* x, const void* w_q, const void* w_k, const void* w_v, const void* s_q,
                      const void* s_k, const void* s_v, void* q_out, void* k_out, void* v_out, int K, int N_q,
                      int N_k, int N_v, int K_blk, int N_q_blk, int N_k_blk, int N_v_blk, cudaStream_t stream) {
  (void)N_q_blk;
  (void)N_k_blk;
  (void)N_v_blk;
  GemvArgs a = make_args(x, K);
  a.nseg = 3;
  a.seg[0] = seg(w_q, s_q, q_out, N_q, K_blk);
  a.seg[1] = seg(w_k, s_k, k_out, N_k, K_blk);
  a.seg[2] = seg(w_v, s_v, v_out, N_v, K_blk);
  record(gemv_run(a, false, stream, false));
}

void launch_fused_gate_up(const void* x, const void* w_gate, const void* w_up, const void* s_gate, const void* s_up,
                          void* gate_out, void* up_out, int K, int N_gate, int N_up, int K_blk, int N_gate_blk,
                          int N_up_blk, cudaStream_t stream) {
  (void)N_gate_blk;
  (void)N_up_blk;
  GemvArgs a = make_args(x, K);
  a.nseg = 2;
  a.seg[0] = seg(w_gate, s_gate, gate_out, N_gate, K_blk);
  a.seg[1] = seg(w_up, s_up, up_out, N_up, K_blk);
  record(gemv_run(a, false, stream, false));
}

void launch_rmsnorm_ip(void* x, const void* weight, int N, int D, float eps, cudaStream_t stream) {
  record(launch_rmsnorm_rows(x, static_cast<const float*>(weight), x, N, D, eps, stream));
}

void launch_rmsnorm_out(const void* x, const void* weight, void* out, int N, int D, float eps,
                        cudaStream_t stream) {
  record(launch_rmsnorm_rows(x, static_cast<const float*>(weight), out, N, D, eps, stream));
}

void layer_pre_attn(const void* hidden, const float* norm_weight, const void* w_q, const void* s_q, int N_q,
                    int N_q_blk, const void* w_k, const void* s_k, int N_k, int N_k_blk, const void* w_v,
                    const void* s_v, int N_v, int N_v_blk, void* q_out, void* k_out, void* v_out, void* norm_ws,
                    int h_dim, int K_blk, cudaStream_t stream) {
  (void)N_q_blk;
  (void)N_k_blk;
  (void)N_v_blk;
  GemvArgs a = make_args(hidden, h_dim);
  a.pro = PRO_RMSNORM;
  a.norm_w = norm_weight;
  a.eps = 1e-6f;
  a.xn_out = static_cast<bf16*>(norm_ws);
  a.nseg = 3;
  a.seg[0] = seg(w_q, s_q, q_out, N_q, K_blk);
  a.seg[1] = seg(w_k, s_k, k_out, N_k, K_blk);
  a.seg[2] = seg(w_v, s_v, v_out, N_v, K_blk);
  record(gemv_run(a, false, stream, false));
}

void layer_post_attn(const void* hidden, const void* attn_out, const void* w_o, const void* s_o, int N_o,
                     int N_o_blk, const float* norm_weight, const void* w_g, const void* s_g, int N_g, int N_g_blk,
                     const void* w_u, const void* s_u, int N_u, int N_u_blk, const void* w_d, const void* s_d,
                     int N_d, int N_d_blk, void* output, void* ws, void* gate_buf, void* up_buf, void* silu_buf,
                     int h_dim, int attn_dim, int K_blk_o, int K_blk_gu, int K_blk_d, cudaStream_t stream) {
  (void)N_o_blk;
  (void)N_g_blk;
  (void)N_u_blk;
  (void)N_d_blk;
  if (N_u != N_g || N_o != h_dim || N_d != h_dim) {
    g_last_error = (int)cudaErrorInvalidValue;
    return;
  }
  // output = bf16(hidden + bf16(O_proj(attn_out)))
  GemvArgs a = make_args(attn_out, attn_dim);
  a.nseg = 1;
  a.seg[0] = seg(w_o, s_o, output, N_o, K_blk_o, EPI_RESID);
  a.seg[0].aux0 = hidden;
  if (record(gemv_run(a, false, stream, false))) return;
  mlp_tail(output, nullptr, norm_weight, w_g, s_g, w_u, s_u, N_g, w_d, s_d, N_d, output, ws, gate_buf, up_buf,
           silu_buf, h_dim, K_blk_gu, K_blk_d, stream);
}

void layer_post_o_fp8_mlp(const void* hidden, const void* o_out, const float* norm_weight, const void* w_g,
                          const void* s_g, int N_g, const void* w_u, const void* s_u, int N_u, const void* w_d,
                          const void* s_d, int N_d, void* output, void* ws, void* gate_buf, void* up_buf,
                          void* silu_buf, int h_dim, int K_blk_gu, int K_blk_d, cudaStream_t stream) {
  if (N_u != N_g || N_d != h_dim) {
    g_last_error = (int)cudaErrorInvalidValue;
    return;
  }
  mlp_tail(hidden, o_out, norm_weight, w_g, s_g, w_u, s_u, N_g, w_d, s_d, N_d, output, ws, gate_buf, up_buf,
           silu_buf, h_dim, K_blk_gu, K_blk_d, stream);
}

void launch_delta_rule_decode(const void* q, const void* k, const void* v, const void* g, const void* beta,
                              void* state, void* output, int n_heads, int head_dim, cudaStream_t stream) {
  GdnArgs a = {};
  a.q = static_cast<const bf16*>(q);
  a.k = static_cast<const bf16*>(k);
  a.v = static_cast<const bf16*>(v);
  a.g = static_cast<const float*>(g);
  a.beta = static_cast<const bf16*>(beta);
  a.state = static_cast<float*>(state);
  a.out = static_cast<bf16*>(output);
  a.rep = 1;
  a.gated = 0;
  record(launch_gdn(a, n_heads, head_dim, stream, false));
}

void launch_prepare_linear_gates(const void* a, const void* beta_in, const float* A_log, const float* dt_bias,
                                 void* g_out, void* beta_out, int heads, cudaStream_t stream) {
  if (heads <= 0) return;
  linear_gates_kernel<<<(heads + 31) / 32, 32, 0, stream>>>(static_cast<const bf16*>(a),
                                                             static_cast<const bf16*>(beta_in), A_log, dt_bias,
                                                             static_cast<float*>(g_out), static_cast<bf16*>(beta_out),
                                                             heads);
  record(cudaSuccess);
}

void launch_rmsnorm_gated_decode(const void* core, const void* z, const void* weight, void* out, int heads,
                                 int head_dim, float eps, cudaStream_t stream) {
  if (heads <= 0) return;
  if (head_dim <= 0) {
    g_last_error = (int)cudaErrorInvalidValue;
    return;
  }
  rmsnorm_gated_f32_kernel<<<heads, 128, 0, stream>>>(static_cast<const bf16*>(core), static_cast<const bf16*>(z),
                                                      static_cast<const bf16*>(weight), static_cast<bf16*>(out),
                                                      head_dim, eps);
  record(cudaSuccess);
}

void launch_fused_attn_v2(const void* q, const void* k_cache, const void* v_cache, void* output, int seq_len,
                          int max_seq_len, int head_dim, int n_heads, int n_kv_heads, cudaStream_t stream) {
  if (seq_len <= 0 || seq_len > max_seq_len) {
    g_last_error = (int)cudaErrorInvalidValue;
    return;
  }
  AttnArgs a = {};
  a.q = static_cast<const bf16*>(q);
  a.k_cache = static_cast<bf16*>(const_cast<void*>(k_cache));
  a.v_cache = static_cast<bf16*>(const_cast<void*>(v_cache));
  a.out = static_cast<bf16*>(output);
  a.seq_len = seq_len;
  a.q_stride = head_dim;
  a.max_seq = max_seq_len;
  a.n_heads = n_heads;
  a.n_kv = n_kv_heads;
  a.chunk = seq_len;
  a.nsplit = 1;
  record(launch_attn(a, head_dim, stream, false));
}

void launch_fused_attn(const void* q, const void* k_cache, const void* v_cache, void* output, int seq_len,
                       int max_seq_len, int head_dim, int n_heads, int n_kv_heads, cudaStream_t stream) {
  launch_fused_attn_v2(q, k_cache, v_cache, output, seq_len, max_seq_len, head_dim, n_heads, n_kv_heads, stream);
}

void layer_mid_attn(void* q_buf, void* k_buf, const void* v_buf, void* attn_out, const float* q_norm_weight,
                    const float* k_norm_weight, const float* cos_table, const float* sin_table, void* k_cache,
                    void* v_cache, int pos, int past_len, int total_seq, int max_seq_len, int head_dim,
                    int rotary_dim, int n_heads, int n_kv_heads, cudaStream_t stream) {
  if (past_len < 0 || past_len >= max_seq_len || total_seq <= 0 || total_seq > max_seq_len ||
      rotary_dim % 2 || rotary_dim > head_dim || (head_dim != 128 && head_dim != 256)) {
    g_last_error = (int)cudaErrorInvalidValue;
    return;
  }
  const int heads = n_heads + 2 * n_kv_heads;
  const int blocks = (heads + 7) / 8;
  if (head_dim == 256)
    attn_prep_inplace_kernel<256><<<blocks, 256, 0, stream>>>(
        static_cast<bf16*>(q_buf), static_cast<bf16*>(k_buf), static_cast<const bf16*>(v_buf), q_norm_weight,
        k_norm_weight, cos_table, sin_table, pos, rotary_dim, 1e-6f, static_cast<bf16*>(k_cache),
        static_cast<bf16*>(v_cache), past_len, max_seq_len, n_heads, n_kv_heads);
  else
    attn_prep_inplace_kernel<128><<<blocks, 256, 0, stream>>>(
        static_cast<bf16*>(q_buf), static_cast<bf16*>(k_buf), static_cast<const bf16*>(v_buf), q_norm_weight,
        k_norm_weight, cos_table, sin_table, pos, rotary_dim, 1e-6f, static_cast<bf16*>(k_cache),
        static_cast<bf16*>(v_cache), past_len, max_seq_len, n_heads, n_kv_heads);
  if (record(cudaSuccess)) return;
  launch_fused_attn_v2(q_buf, k_cache, v_cache, attn_out, total_seq, max_seq_len, head_dim, n_heads, n_kv_heads,
                       stream);
}

// ---------------------------------------------------------------------------
// New exports: f32-scale GEMV, fused LM head + greedy argmax, decode engine
// ---------------------------------------------------------------------------

// launch_gemv_v4_extern with FP32 scales (BASELINE configs keep the
// checkpoint's FP32 weight_scale_inv instead of rounding it to BF16).
int launch_gemv_f32s(const void* x, const void* w, const float* s, void* y, int N, int K, int K_blk,
                     cudaStream_t stream) {
  GemvArgs a = make_args(x, K);
  a.nseg = 1;
  a.seg[0] = seg(w, s, y, N, K_blk);
  return record(gemv_run(a, true, stream, false));
}

// Same as launch_gemv_v4_extern but always through the generic one-warp-per-row
// kernel (used by tests to cover the fallback on production shapes).
int qwen_gemv_generic(const void* x, const void* w, const void* s, int scale_f32, void* y, int N, int K, int K_blk,
                      cudaStream_t stream) {
  GemvArgs a = make_args(x, K);
  a.nseg = 1;
  a.seg[0] = seg(w, s, y, N, K_blk);
  return record(gemv_run(a, scale_f32 != 0, stream, false, true));
}

// LM head GEMV with the final RMSNorm(1+w) folded in (norm_w may be null)
// and a fused greedy argmax over this shard's rows.  `ws` is 16 bytes of
// device memory, zero before the first call and left zeroed by every call.
// Outputs (each nullable): key_out = orderable(bf16 logit) << 32 |
// (0xFFFFFFFF - (row_offset + row)); token_out = argmax row index
// (row_offset + row, the first maximal BF16 logit); logits_out = BF16 logits;
// pos_inc is incremented once.
int launch_lm_head_argmax(const void* x, const float* norm_w, float eps, const void* w, const void* s, int N, int K,
                          int K_blk, int row_offset, void* ws, unsigned long long* key_out, long long* token_out,
                          void* logits_out, int* pos_inc, cudaStream_t stream) {
  if (!ws) return record(cudaErrorInvalidValue);
  GemvArgs a = make_args(x, K);
  if (norm_w) {
    a.pro = PRO_RMSNORM;
    a.norm_w = norm_w;
    a.eps = eps;
  }
  a.nseg = 1;
  a.seg[0] = seg(w, s, logits_out, N, K_blk, EPI_ARGMAX);
  a.seg[0].row_offset = row_offset;
  a.am_ws = static_cast<unsigned long long*>(ws);
  a.am_key_out = key_out;
  a.am_token_out = token_out;
  a.pos_inc = pos_inc;
  a.pf = take_prefetch();
  if (cudaError_t pe = take_p2p_input(a)) return record(pe);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// Token embedding row gather: hidden = embed[*token].
__global__ void embed_kernel(const bf16* __restrict__ embed, const long long* __restrict__ token,
                             bf16* __restrict__ hidden, int H) {
  if (threadIdx.x == 0 && blockIdx.x == 0) pdl_trigger();
  pdl_wait();
  const long long t = *token;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H / 8; i += gridDim.x * blockDim.x)
    reinterpret_cast<uint4*>(hidden)[i] = reinterpret_cast<const uint4*>(embed + (size_t)t * H)[i];
}

int qwen_embed(const void* embed, const long long* token, void* hidden, int H, cudaStream_t stream) {
  if (!embed || !token || !hidden || H % 8) return record(cudaErrorInvalidValue);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((H / 8 + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = engine_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return record(cudaLaunchKernelEx(&cfg, embed_kernel, static_cast<const bf16*>(embed), token,
                                   static_cast<bf16*>(hidden), H));
}

// Full-attention layer input projections: RMSNorm(1+w)(hidden) then the
// q (with output gate), k and v GEMVs as one grouped launch.
int qwen_attn_in_proj(const void* hidden, const float* norm_w, float eps, const void* w_q, const void* s_q, int N_q,
                      const void* w_k, const void* s_k, int N_k, const void* w_v, const void* s_v, int N_v, int K,
                      int K_blk, void* q_out, void* k_out, void* v_out, cudaStream_t stream) {
  GemvArgs a = make_args(hidden, K);
  a.pro = PRO_RMSNORM;
  a.norm_w = norm_w;
  a.eps = eps;
  a.nseg = 3;
  a.seg[0] = seg(w_q, s_q, q_out, N_q, K_blk);
  a.seg[1] = seg(w_k, s_k, k_out, N_k, K_blk);
  a.seg[2] = seg(w_v, s_v, v_out, N_v, K_blk);
  a.pf = take_prefetch();
  if (cudaError_t pe = take_p2p_input(a)) return record(pe);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// GatedDeltaNet layer input projections in one grouped launch:
// RMSNorm(1+w)(hidden); qkv rows -> causal conv update + SiLU (conv_state
// updated in place); z rows stored; a rows -> g = -exp(A_log)*softplus(a+dt_bias);
// b rows -> beta = sigmoid(b).
int qwen_gdn_in_proj(const void* hidden, const float* norm_w, float eps, int K, int K_blk, const void* w_qkv,
                     const void* s_qkv, int N_qkv, const void* conv_w, void* conv_state, int conv_width,
                     void* qkv_out, const void* w_z, const void* s_z, int N_z, void* z_out, const void* w_a,
                     const void* s_a, const void* w_b, const void* s_b, int N_heads, const float* A_log,
                     const float* dt_bias, float* g_out, void* beta_out, cudaStream_t stream) {
  GemvArgs a = make_args(hidden, K);
  a.pro = PRO_RMSNORM;
  a.norm_w = norm_w;
  a.eps = eps;
  a.nseg = 4;
  a.seg[0] = seg(w_qkv, s_qkv, qkv_out, N_qkv, K_blk, EPI_CONV);
  a.seg[0].aux0 = conv_w;
  a.seg[0].aux2 = conv_state;
  a.seg[0].cw = conv_width;
  a.seg[1] = seg(w_z, s_z, z_out, N_z, K_blk);
  a.seg[2] = seg(w_a, s_a, g_out, N_heads, K_blk, EPI_GATE_G);
  a.seg[2].aux0 = A_log;
  a.seg[2].aux1 = dt_bias;
  a.seg[3] = seg(w_b, s_b, beta_out, N_heads, K_blk, EPI_GATE_BETA);
  a.pf = take_prefetch();
  if (cudaError_t pe = take_p2p_input(a)) return record(pe);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// GatedDeltaNet recurrent decode + RMSNormGated, reading q/k/v from the
// post-conv projection output [q (Hk*D) | k (Hk*D) | v (Hv*D)].
int qwen_gdn_decode(const void* qkv, const float* g, const void* beta, float* state, const void* z,
                    const void* norm_w, float eps, void* out, int n_k_heads, int n_v_heads, int head_dim,
                    cudaStream_t stream) {
  if (n_k_heads <= 0 || n_v_heads % n_k_heads) return record(cudaErrorInvalidValue);
  const bf16* base = static_cast<const bf16*>(qkv);
  GdnArgs a = {};
  a.q = base;
  a.k = base + (size_t)n_k_heads * head_dim;
  a.v = base + (size_t)2 * n_k_heads * head_dim;
  a.g = g;
  a.beta = static_cast<const bf16*>(beta);
  a.state = state;
  a.out = static_cast<bf16*>(out);
  a.z = static_cast<const bf16*>(z);
  a.norm_w = static_cast<const bf16*>(norm_w);
  a.eps = eps;
  a.rep = n_v_heads / n_k_heads;
  a.gated = 1;
  a.pf = take_prefetch();
  return record(launch_gdn(a, n_v_heads, head_dim, stream, engine_pdl()));
}

// GatedDeltaNet recurrent step writing the un-normed core output (the gated
// norm then runs in the next GEMV's prologue, qwen_set_gated_input); the
// value columns of a head are split over 4 CTAs.
int qwen_gdn_decode_core(const void* qkv, const float* g, const void* beta, float* state, void* core_out,
                         int n_k_heads, int n_v_heads, int head_dim, cudaStream_t stream) {
  if (n_k_heads <= 0 || n_v_heads % n_k_heads) return record(cudaErrorInvalidValue);
  const bf16* base = static_cast<const bf16*>(qkv);
  GdnArgs a = {};
  a.q = base;
  a.k = base + (size_t)n_k_heads * head_dim;
  a.v = base + (size_t)2 * n_k_heads * head_dim;
  a.g = g;
  a.beta = static_cast<const bf16*>(beta);
  a.state = state;
  a.out = static_cast<bf16*>(core_out);
  a.rep = n_v_heads / n_k_heads;
  a.gated = 0;
  a.pf = take_prefetch();
  return record(launch_gdn(a, n_v_heads, head_dim, stream, engine_pdl()));
}

// y = bf16(res + bf16(W x)) (o_proj / out_proj / down with the residual add).
int qwen_linear_resid(const void* x, const void* w, const void* s, int N, int K, int K_blk, const void* res, void* y,
                      cudaStream_t stream) {
  GemvArgs a = make_args(x, K);
  a.nseg = 1;
  a.seg[0] = seg(w, s, y, N, K_blk, EPI_RESID);
  a.seg[0].aux0 = res;
  a.pf = take_prefetch();
  if (cudaError_t ge = take_gated_input(a)) return record(ge);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// y = W x as per-K-slice FP32 partial rows: slices[c][r] for c < *count
// (count <= max_slices, written by the launch).  The next RMSNorm-prologue
// launch, given qwen_set_slices_input, adds them (in slice order) to its
// residual; nothing reduces them here.
int qwen_linear_slices(const void* x, const void* w, const void* s, int N, int K, int K_blk, float* slices,
                       int* count, int max_slices, cudaStream_t stream) {
  if (!slices || !count || max_slices < 1) return record(cudaErrorInvalidValue);
  GemvArgs a = make_args(x, K);
  a.nseg = 1;
  a.seg[0] = seg(w, s, slices, N, K_blk, EPI_SLICES);
  a.seg[0].y2 = count;
  a.sl_max = max_slices;
  a.pf = take_prefetch();
  if (cudaError_t ge = take_gated_input(a)) return record(ge);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// Tensor parallelism, K-sliced projection: y_f32 = partial GEMV over this
// rank's slice of K (the caller all-reduces y_f32 and then applies
// qwen_resid_add_f32).
int qwen_linear_partial(const void* x, const void* w, const void* s, int N, int K, int K_blk, float* y,
                        cudaStream_t stream) {
  GemvArgs a = make_args(x, K);
  a.nseg = 1;
  a.seg[0] = seg(w, s, y, N, K_blk, EPI_F32);
  a.pf = take_prefetch();
  if (cudaError_t ge = take_gated_input(a)) return record(ge);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// y = bf16(res + bf16(v)) for n elements (v: all-reduced FP32 partial sums).
int qwen_resid_add_f32(const void* res, const float* v, void* y, int n, cudaStream_t stream) {
  if (n <= 0 || !res || !v || !y) return record(cudaErrorInvalidValue);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((n + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = engine_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return record(cudaLaunchKernelEx(&cfg, resid_add_f32_kernel, static_cast<const bf16*>(res), v,
                                   static_cast<bf16*>(y), n));
}

// Copies the step's token to host-mapped pinned memory host_out[0..1] =
// {token, sequence number} (see publish_token_kernel).
int qwen_publish_token(const long long* token, long long* host_out, unsigned long long* seq, cudaStream_t stream) {
  if (!token || !host_out || !seq) return record(cudaErrorInvalidValue);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = engine_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return record(cudaLaunchKernelEx(&cfg, publish_token_kernel, token, host_out, seq));
}

// token = greedy token encoded in an all-reduced packed argmax key.
int qwen_token_from_key(const long long* key, long long* token, cudaStream_t stream) {
  if (!key || !token) return record(cudaErrorInvalidValue);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = engine_pdl() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return record(cudaLaunchKernelEx(&cfg, token_from_key_kernel, reinterpret_cast<const unsigned long long*>(key),
                                   token));
}

// ---------------------------------------------------------------------------
// Tensor parallel over NVLink peer memory (p2p.cuh)
// ---------------------------------------------------------------------------
// Allocates this rank's exchange region for `world` ranks and n-element
// partial sums (zeroed) and writes its CUDA IPC handle (64 bytes).
int qwen_p2p_create(int world, int n, void** base_out, void* ipc_handle_out) {
  if (world < 1 || world > P2P_MAX_WORLD || n <= 0 || !base_out || !ipc_handle_out)
    return record(cudaErrorInvalidValue);
  void* base = nullptr;
  const size_t bytes = p2p_region_bytes(world, n);
  cudaError_t e = cudaMalloc(&base, bytes);
  if (e != cudaSuccess) return record(e);
  e = cudaMemset(base, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) {
    cudaFree(base);
    return record(e);
  }
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  *base_out = base;
  return 0;
}

// Maps another rank's exchange region (its IPC handle) into this process.
int qwen_p2p_open(const void* ipc_handle, void** peer_base_out) {
  if (!ipc_handle || !peer_base_out) return record(cudaErrorInvalidValue);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return record(cudaIpcOpenMemHandle(peer_base_out, h, cudaIpcMemLazyEnablePeerAccess));
}

int qwen_p2p_close(void* peer_base) { return record(cudaIpcCloseMemHandle(peer_base)); }
int qwen_p2p_destroy(void* base) { return record(cudaFree(base)); }

// Builds the device table of a rank: bases[p] = rank p's region as mapped in
// this process (bases[rank] = its own).  Returns a device pointer.
int qwen_p2p_table(void* const* bases, int world, int rank, int n, void** table_out) {
  if (!bases || world < 1 || world > P2P_MAX_WORLD || rank < 0 || rank >= world || n <= 0 || !table_out)
    return record(cudaErrorInvalidValue);
  P2PTable t;
  std::memset(&t, 0, sizeof(t));
  for (int p = 0; p < world; ++p) {
    char* b = static_cast<char*>(bases[p]);
    if (!b) return record(cudaErrorInvalidValue);
    t.flag[p] = reinterpret_cast<unsigned*>(b);
    t.key[p] = reinterpret_cast<unsigned long long*>(b + 64);
    for (int par = 0; par < 2; ++par)
      t.buf[p][par] = reinterpret_cast<float*>(b + P2P_DATA_OFF) + (size_t)par * world * n;
  }
  char* own = static_cast<char*>(bases[rank]);
  t.seq = reinterpret_cast<unsigned*>(own + 256);
  t.done = reinterpret_cast<unsigned*>(own + 260);
  t.world = world;
  t.rank = rank;
  t.n = n;
  void* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(t));
  if (e == cudaSuccess) e = cudaMemcpy(d, &t, sizeof(t), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    if (d) cudaFree(d);
    return record(e);
  }
  *table_out = d;
  return 0;
}
int qwen_p2p_table_free(void* table) { return record(cudaFree(table)); }

// Column-shard GEMV whose FP32 rows go to slot [rank] of every rank's buffer.
int qwen_linear_partial_p2p(const void* x, const void* w, const void* s, int N, int K, int K_blk, const void* table,
                            cudaStream_t stream) {
  if (!table) return record(cudaErrorInvalidValue);
  GemvArgs a = make_args(x, K);
  a.nseg = 1;
  a.seg[0] = seg(w, s, nullptr, N, K_blk, EPI_F32_P2P);
  a.seg[0].aux0 = table;
  a.pf = take_prefetch();
  if (cudaError_t ge = take_gated_input(a)) return record(ge);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// y = bf16(res + bf16(sum over ranks)) once every rank's partial has arrived.
int qwen_resid_add_p2p(const void* table, const void* res, void* y, int n, cudaStream_t stream) {
  if (!table || !res || !y || n <= 0) return record(cudaErrorInvalidValue);
  const P2PTable* t = static_cast<const P2PTable*>(table);
  const bf16* r = static_cast<const bf16*>(res);
  bf16* yy = static_cast<bf16*>(y);
  void* args[] = {&t, &r, &yy};
  return record(launch_small(reinterpret_cast<const void*>(p2p_resid_kernel), (n + 255) / 256, 256, args, stream));
}

// token = greedy token over every rank's packed argmax key.
int qwen_token_p2p(const void* table, const long long* key, long long* token, cudaStream_t stream) {
  if (!table || !key || !token) return record(cudaErrorInvalidValue);
  const P2PTable* t = static_cast<const P2PTable*>(table);
  const unsigned long long* k = reinterpret_cast<const unsigned long long*>(key);
  void* args[] = {&t, &k, &token};
  return record(launch_small(reinterpret_cast<const void*>(p2p_token_kernel), 1, 32, args, stream));
}

// silu_out = bf16(silu(g) * u) with g, u = GEMV(RMSNorm(1+w)(h2)).
int qwen_mlp_gate_up(const void* h2, const float* norm_w, float eps, const void* w_g, const void* s_g,
                     const void* w_u, const void* s_u, int N, int K, int K_blk, void* silu_out, cudaStream_t stream) {
  GemvArgs a = make_args(h2, K);
  a.pro = PRO_RMSNORM;
  a.norm_w = norm_w;
  a.eps = eps;
  a.nseg = 1;
  a.seg[0] = seg(w_g, s_g, silu_out, N, K_blk, EPI_SILU_PAIR);
  a.seg[0].w2 = static_cast<const uint8_t*>(w_u);
  a.seg[0].s2 = s_u;
  a.pf = take_prefetch();
  if (cudaError_t pe = take_p2p_input(a)) return record(pe);
  return record(gemv_run(a, false, stream, engine_pdl()));
}

// Decode attention of one full-attention layer: q/k RMSNorm, partial RoPE,
// KV-cache write at *pos, split-KV GQA attention and the sigmoid output gate.
// q_all holds [q | gate] per head (head stride 2*head_dim).
int qwen_attn_decode(const void* q_all, const void* k_new, const void* v_new, const float* q_norm,
                     const float* k_norm, const float* cos, const float* sin, void* k_cache, void* v_cache,
                     const int* pos, int max_seq, int n_heads, int n_kv_heads, int head_dim, int rotary_dim,
                     float eps, int chunk, int nsplit, float* ws_part, unsigned* ws_count, void* out,
                     cudaStream_t stream) {
  AttnArgs a = {};
  a.q = static_cast<const bf16*>(q_all);
  a.gate = static_cast<const bf16*>(q_all) + head_dim;
  a.k_new = static_cast<const bf16*>(k_new);
  a.v_new = static_cast<const bf16*>(v_new);
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.cos = cos;
  a.sin = sin;
  a.k_cache = static_cast<bf16*>(k_cache);
  a.v_cache = static_cast<bf16*>(v_cache);
  a.pos_ptr = pos;
  a.q_stride = 2 * head_dim;
  a.max_seq = max_seq;
  a.n_heads = n_heads;
  a.n_kv = n_kv_heads;
  a.rot = rotary_dim;
  a.eps = eps;
  a.prep = 1;
  a.chunk = chunk;
  a.nsplit = nsplit;
  a.ws_part = ws_part;
  a.ws_count = ws_count;
  a.out = static_cast<bf16*>(out);
  a.pf = take_prefetch();
  if (!pos || chunk < 1 || nsplit < 1) return record(cudaErrorInvalidValue);
  return record(launch_attn(a, head_dim, stream, engine_pdl()));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free attention decode.
//
// Some callers cannot allocate device memory where they run the decode step:
// a serving runtime that hands out all GPU memory from its own pool and bans
// cudaMalloc afterwards, a foreign-language binding (ctypes, cgo, JNI) that
// has no device allocator of its own, or code that must not trigger the
// implicit device synchronisation an allocation can cause.  For them,
// qwen_attn_decode_noalloc takes the split-KV scratch from a fixed array
// compiled into this library instead of from caller-provided buffers.
//
// Limit: partials of n_heads * nsplit * (head_dim + 2) floats, rounded up to
// 256 bytes, plus n_kv_heads counters must fit QWEN_ATTN_NOALLOC_SCRATCH_BYTES
// (4 MiB); larger requests return cudaErrorInvalidValue and launch nothing.
// Every GPU that loads the library holds the 4 MiB until the process exits.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t QWEN_ATTN_NOALLOC_SCRATCH_BYTES = size_t(4) << 20;
}  // namespace

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[QWEN_ATTN_NOALLOC_SCRATCH_BYTES];

// Device address of g_attn_noalloc_scratch per device.  In host code the
// array's name is only a host-side handle, so the address is looked up with
// cudaGetSymbolAddress, with the device current, by the first call on each
// device and cached together with the CUDA context it belongs to: a call under
// another context (after cudaDeviceReset, or a new primary context) looks the
// address up again instead of using a stale one.  The cache is guarded by a
// mutex, so concurrent first calls from several host threads are safe.
namespace {
struct NoallocAddr {
  void* ctx = nullptr;
  void* addr = nullptr;
};
NoallocAddr g_attn_noalloc_addr[64];
std::mutex g_attn_noalloc_mu;

typedef int (*PFN_ctx_get_current)(void**);
PFN_ctx_get_current ctx_get_current() {
  static PFN_ctx_get_current fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_ctx_get_current>(f);
  });
  return fn;
}

// Address of the scratch array on the current device (looked up on first use
// per device and context).
cudaError_t attn_noalloc_base(unsigned char** base) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  PFN_ctx_get_current get = ctx_get_current();
  if (!get) return cudaErrorInitializationError;
  void* ctx = nullptr;  // null until the runtime has made a context current
  if (get(&ctx) != 0) return cudaErrorInitializationError;
  std::lock_guard<std::mutex> lock(g_attn_noalloc_mu);
  NoallocAddr& slot = g_attn_noalloc_addr[dev];
  if (!ctx || slot.ctx != ctx || !slot.addr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_attn_noalloc_scratch);  // initialises the context if needed
    if (e != cudaSuccess) return e;
    if (get(&ctx) != 0 || !ctx) return cudaErrorInitializationError;
    slot.addr = addr;
    slot.ctx = ctx;
  }
  *base = static_cast<unsigned char*>(slot.addr);
  return cudaSuccess;
}
}  // namespace

extern "C" int qwen_attn_decode_noalloc(const void* q_all, const void* k_new, const void* v_new,
                                        const float* q_norm, const float* k_norm, const float* cos,
                                        const float* sin, void* k_cache, void* v_cache, const int* pos, int max_seq,
                                        int n_heads, int n_kv_heads, int head_dim, int rotary_dim, float eps,
                                        int chunk, int nsplit, void* out, cudaStream_t stream) {
  unsigned char* base = nullptr;
  cudaError_t e = attn_noalloc_base(&base);
  if (e != cudaSuccess) return record(e);
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || nsplit < 1) return record(cudaErrorInvalidValue);
  const size_t part_bytes = (size_t)n_heads * (size_t)nsplit * (size_t)(head_dim + 2) * sizeof(float);
  const size_t count_off = (part_bytes + 255) / 256 * 256;
  const size_t need = count_off + (size_t)n_kv_heads * sizeof(unsigned);
  if (need > QWEN_ATTN_NOALLOC_SCRATCH_BYTES) return record(cudaErrorInvalidValue);
  unsigned* counts = reinterpret_cast<unsigned*>(base + count_off);
  // The array keeps whatever the previous call left; the split counters must
  // start at zero, so clear them on the stream ahead of the kernel.
  e = cudaMemsetAsync(counts, 0, (size_t)n_kv_heads * sizeof(unsigned), stream);
  if (e != cudaSuccess) return record(e);
  return qwen_attn_decode(q_all, k_new, v_new, q_norm, k_norm, cos, sin, k_cache, v_cache, pos, max_seq, n_heads,
                          n_kv_heads, head_dim, rotary_dim, eps, chunk, nsplit, reinterpret_cast<float*>(base),
                          counts, out, stream);
}

// Persistent decode-step kernel (include/qwen_step.h).
#include "step_host.cuh"
