/* Persistent decode-step API of libqwen_fused.so (sm_100a).
 *
 * No counterpart in the reference, which runs its decode step as ~1,000
 * separate launches per token from Python (QwenEngineFP8Opt._decode_step,
 * main.py:1509-1547, and forward, main.py:1569-1604).  Here the whole step
 * is one cooperative kernel launch (one CTA per SM) that walks a list of
 * stages; each CTA streams its share of every stage's weights into a
 * shared-memory ring ahead of the dependency chain, so the HBM stream does
 * not stop at stage boundaries.
 *
 * The stage kinds restate the reference's hot path:
 *   GEMV stages  - the block-scaled E4M3 GEMV family (gemv_v4_kernel and its
 *                  grouped / fused variants, fused_kernels.cu:91-479) with
 *                  RMSNorm(1+w) (489-547) and residual adds (553-559) fused;
 *   GDN stages   - the GatedDeltaNet decode step with the default path's
 *                  gated RMSNorm (623-684, main.py:1064-1163);
 *   ATTN stages  - decode attention (layer_mid_attn, 1224-1297, and the
 *                  output gate of main.py:1059).
 *
 * Weights of GEMV stages are packed once for this kernel (qwen_step_pack).
 * All pointers are device pointers owned by the caller.  Functions return 0
 * or a cudaError_t code (also kept for qwen_last_error()).  A wait that runs
 * out (2 s) abandons the step: qwen_get_device_error() then reports 8, and
 * qwen_step_reset() must run before the next launch.
 */
#ifndef QWEN_STEP_H
#define QWEN_STEP_H

#include <stddef.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Stage kinds */
#define QWEN_STEP_GEMV 0
#define QWEN_STEP_GDN 1
#define QWEN_STEP_ATTN 2

/* GEMV x prologues */
#define QWEN_STEP_PRO_PLAIN 0       /* x as given (BF16) */
#define QWEN_STEP_PRO_NORM 1        /* x <- RMSNorm(1+w)(x) */
#define QWEN_STEP_PRO_EMBED_NORM 2  /* h <- table[*token] (stored to h_out), x <- RMSNorm(1+w)(h) */
#define QWEN_STEP_PRO_SLICES_NORM 3 /* h <- bf16(res + bf16(sum of sl_in rows)) (stored to h_out), x <- RMSNorm(1+w)(h) */

/* GEMV segment epilogues (output row r, FP32 sum v; v2 = up-projection sum of a pair) */
#define QWEN_STEP_EPI_STORE 0      /* y[r] = bf16(v) */
#define QWEN_STEP_EPI_SILU_PAIR 2  /* y[r] = bf16(silu(v) * v2) */
#define QWEN_STEP_EPI_ARGMAX 3     /* greedy argmax of bf16(v) (y: optional BF16 logits) */
#define QWEN_STEP_EPI_CONV 4       /* y[r] = bf16(silu(bf16(conv1d(state[r], bf16(v))))), state updated */
#define QWEN_STEP_EPI_GATE_G 5     /* y(f32)[r] = -exp(A_log[r]) * softplus(bf16(v) + dt_bias[r]) */
#define QWEN_STEP_EPI_GATE_BETA 6  /* y[r] = bf16(sigmoid(bf16(v))) */
#define QWEN_STEP_EPI_SLICES 9     /* FP32 partial rows into the stage's sl_out [nslice][sl_rows] */
#define QWEN_STEP_EPI_SILU 10      /* y[r] = bf16(silu(bf16(v))) */

typedef struct qwen_step_seg {
  const void* w;         /* packed weights (qwen_step_pack) */
  const void* w2;        /* SILU_PAIR: packed up-projection weights */
  int n;                 /* output rows */
  int epi;               /* QWEN_STEP_EPI_* */
  void* y;
  void* y2;              /* CONV: optional bf16(v) */
  const void* aux0;      /* CONV: conv weight BF16 [n][cw]; GATE_G: A_log FP32 [n] */
  const void* aux1;      /* GATE_G: dt_bias FP32 [n] */
  void* aux2;            /* CONV: conv state BF16 [n][cw], updated in place */
  int cw;                /* CONV: kernel width (<= 8) */
  int row_offset;        /* ARGMAX: global index of row 0 */
} qwen_step_seg;

typedef struct qwen_step_stage {
  int kind;              /* QWEN_STEP_GEMV / _GDN / _ATTN */
  /* GEMV */
  int K;                 /* input length, a multiple of 512, at most 9216 (3072 unless PRO_PLAIN) */
  int pro;               /* QWEN_STEP_PRO_* */
  int nseg;              /* 1..6 segments over one shared input */
  int pair;              /* 1: every segment is a gate/up pair (SILU_PAIR) */
  int nslice;            /* EPI_SLICES: K slices (0: chosen by the library) */
  const void* x;         /* PLAIN / NORM: input BF16 [K]; EMBED_NORM: table BF16 [x_rows][K] */
  int x_rows;
  const void* res;       /* SLICES_NORM: residual BF16 [K] */
  const float* norm_w;   /* RMSNorm(1+w) weight FP32 [K] */
  float eps;
  void* h_out;           /* EMBED_NORM / SLICES_NORM: residual stream out BF16 [K] */
  const long long* token;        /* EMBED_NORM: row index (device) */
  const float* sl_in;    /* SLICES_NORM: partial rows FP32 [count][sl_stride] */
  int sl_in_count;       /* <= 0: the nslice of the stage that writes sl_in */
  int sl_stride;
  float* sl_out;         /* EPI_SLICES output FP32 [nslice][sl_rows] */
  int sl_rows;
  unsigned long long* am_ws;     /* ARGMAX workspace (2 x u64, zero before the first step, left zeroed) */
  unsigned long long* am_key_out;
  long long* am_token_out;
  int* pos_inc;          /* ARGMAX: ++*pos_inc by the finaliser */
  qwen_step_seg seg[6];
  /* GatedDeltaNet (head dim 128; value head h reads key head h / g_rep) */
  const void* g_q;       /* BF16 key-head queries [key heads][128] */
  const void* g_k;
  const void* g_v;       /* BF16 [value heads][128] */
  const float* g_g;      /* FP32 [value heads] log-decay */
  const void* g_beta;    /* BF16 [value heads] */
  float* g_state;        /* FP32 [value heads][4][128 keys][32 values] (value block b holds
                            columns 32 b .. 32 b + 31 of the [keys][values] state), in place */
  void* g_out;           /* BF16 [value heads][128]: the core output */
  const void* g_z;       /* gated RMSNorm: BF16 silu(z) [value heads][128] (an EPI_SILU
                            output; null: none).  The norm is
                            applied by the next stage, which must be a PLAIN GEMV whose x is
                            whole heads of g_out (K <= 4096): its prologue normalises them */
  const void* g_norm_w;  /* BF16 [128] */
  float g_eps;
  int g_heads;
  int g_dim;
  int g_rep;
  /* attention (the Qwen3.5 layout: head dim 256, 4 query heads per KV head;
     other layouts are refused with cudaErrorNotSupported) */
  const void* a_q;       /* BF16 [heads][2 * dim]: per head [q | gate] */
  const void* a_k_new;
  const void* a_v_new;
  const float* a_q_norm;
  const float* a_k_norm;
  const float* a_cos;    /* FP32 [max_seq][rot] */
  const float* a_sin;
  void* a_k_cache;       /* BF16 [kv][max_seq][dim] */
  void* a_v_cache;
  const int* a_pos;      /* device position */
  int a_max_seq;
  int a_heads;
  int a_kv;
  int a_dim;
  int a_rot;
  float a_eps;
  int a_chunk;
  int a_nsplit;
  float* a_ws;           /* FP32 [heads][nsplit][dim + 2] */
  unsigned* a_cnt;       /* [kv] zeroed counters (left zeroed) */
  void* a_out;           /* BF16 [heads][dim] */
  /* GEMV with BF16 weights (packed by qwen_step_pack_bf16; one STORE / ARGMAX /
     SLICES segment, K a multiple of 256): x is used as BF16, no block scales */
  int wbf16;
  /* A share of the stage (tensor parallel): GEMV 32-row tiles
     [shard0, shard0 + shard_n) of the segments' tiles in order, GatedDeltaNet
     value heads, or attention KV heads (with all their splits); shard_n = 0:
     the whole stage.  A column-parallel GEMV share is usually described by
     segments over row ranges instead (seg.w at tile r0 / 32 of the packed
     matrix, y and the per-row epilogue operands at row r0, ARGMAX row_offset
     += r0).  Outputs stay on the rank, except EPI_ARGMAX logits. */
  int shard0;
  int shard_n;
  /* Tensor parallel, GEMV: xrank = 1 for a row-parallel EPI_SLICES stage (this
     rank's K range of every row): its K-slice rows go to slots [rank x nslice,
     +nslice) of every rank's sl_out as tagged 8-byte words (FP32 bits | tag
     << 32; sl_out then holds 16 x sl_rows words, in the IPC arena), and the
     SLICES_NORM stage reading them polls every word for this step's tag of
     the producing stage before summing the world x nslice slices in order;
     nslice x world <= 16.  cstride: chunks per tile row of the packed matrices
     (K/512 of the whole matrix when seg[].w points at a K range inside it;
     0: K/512). */
  int xrank;
  int cstride;
} qwen_step_stage;

/* Bytes of a packed [N, K] matrix: ceil(N/32) * (K/512) * 16400 (0 if K % 512). */
size_t qwen_step_packed_bytes(int N, int K);

/* Packs E4M3 weights w [N, K] with 128x128 block scales s ([ceil(N/128)][K/128],
 * BF16, or FP32 with scale_f32 = 1) for GEMV stages.  K_blk must be K/128. */
int qwen_step_pack(const void* w, const void* s, int scale_f32, int N, int K, int K_blk, void* out,
                   cudaStream_t stream);

/* BF16 weights w [N, K] for a GEMV stage with wbf16 = 1: chunks of 32 rows x
 * 256 K (16 KB, each lane's m16n8k16 A fragments contiguous) + 16 zero bytes;
 * ceil(N/32) * (K/256) * 16400 bytes (0 if K % 256). */
size_t qwen_step_packed_bytes_bf16(int N, int K);
int qwen_step_pack_bf16(const void* w, int N, int K, void* out, cudaStream_t stream);

/* Builds a program from `nstages` stage descriptions (copied; the pointers
 * they hold must stay valid while the program is used) on the current device. */
int qwen_step_create(const qwen_step_stage* stages, int nstages, void** program_out);

/* Tensor-parallel program over `world` GPUs (one process and one program per
 * GPU, every rank launching once per token; Megatron-style split): stages
 * carry this rank's share - column-parallel GEMVs a row range, GatedDeltaNet
 * / attention the heads those rows feed, row-parallel (xrank) GEMVs the
 * matching K range of every row.  The K-slice buffers of xrank stages, the
 * EPI_ARGMAX logits and workspace and the counters
 * (qwen_step_counter_bytes(nstages), zeroed) must lie in an arena that every
 * rank allocates with the same layout (qwen_ipc_alloc) and maps from its
 * peers (qwen_p2p_open): peer_bases[r] = rank r's arena as mapped here
 * (peer_bases[rank] = local_base).  An xrank stage stores its tagged slice
 * words on every rank; the next stage polls them in local memory instead of
 * waiting on a counter (one NVLink crossing, no fence).  Other stages
 * synchronise within their GPU (counters[nstages, 2 nstages]; counters[0,
 * nstages) are unused).  The argmax keys are folded into every rank's
 * workspace; each rank finalises its own token.  Every rank must run the same
 * steps: the tags derive from the count of completed steps (a reset on one
 * rank needs a reset on all). */
int qwen_step_create_tp(const qwen_step_stage* stages, int nstages, int world, int rank, void* const* peer_bases,
                        const void* local_base, void* counters, void** program_out);
size_t qwen_step_counter_bytes(int nstages);
/* A zeroed device allocation of `bytes` and its 64-byte CUDA IPC handle. */
int qwen_ipc_alloc(size_t bytes, void** base_out, void* ipc_handle_out);

/* One launch of the whole program on `stream`. */
int qwen_step_launch(void* program, cudaStream_t stream);

/* Clears the program's stage counters, abort flag, argmax and attention
 * workspaces on `stream` (after an abandoned step). */
int qwen_step_reset(void* program, cudaStream_t stream);

/* Failure-detection hook: on the following launches CTA 0 does not report
 * stage `stage` done (-1: off), so the next stage's grid-wide wait runs out
 * (qwen_set_wait_timeout_ns) and the step is abandoned with device error 8. */
int qwen_step_set_drop(void* program, int stage);

int qwen_step_destroy(void* program);

/* Profiling: launches record, per stage and CTA, ten words into timeline
 * [nstages][grid][10]: five %globaltimer stamps (low 32 bits, ns) - the
 * consumers' wait for the previous stage begins, ends, their work on the stage
 * ends, the producer issues the stage's first item, has issued its last - then
 * the producer's ns blocked on a full ring while issuing the stage, consumer
 * warp 0's ns blocked on copies not yet landed, and for GEMV stages the stamps
 * at which the x prologue and the last batch's chunk math were done and warp
 * 0's SM clock cycles inside the chunk math.  Null stops it. */
int qwen_step_set_timeline(void* program, unsigned* timeline);

/* CTAs a launch uses (one per SM) and its dynamic shared memory in bytes. */
int qwen_step_grid(void* program);
int qwen_step_smem_bytes(void);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_STEP_H */
