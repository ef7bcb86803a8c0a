// Persistent decode-step kernel: one launch per token.
//
// The batch-1 decode step of the Qwen3.5 hybrid (main.py:1509-1604 with the
// kernels of fused_kernels.cu) is a chain of ~160 dependent stages: grouped
// GEMVs with fused prologues / epilogues, the GatedDeltaNet recurrent step,
// decode attention and the LM head with greedy argmax.  Launched one kernel
// per stage, every stage pays a kernel boundary and its weight stream stops
// while the chain waits.  Here one cooperative grid (one CTA per SM) walks
// the whole stage list:
//
//  * a producer warp per CTA streams the CTA's share of every stage's
//    weights, in stage order, into a ring of shared-memory slots with 1-D bulk
//    copies (cp.async.bulk, TMA engine, no multicast).  Weights are static, so
//    the producer runs ahead across stage boundaries, limited only by the
//    ring: while the chain waits for a stage's input, the HBM stream keeps
//    filling the next stages' slots.  The GatedDeltaNet state of a head is
//    streamed the same way by the CTA that owns the head;
//  * eight consumer warps run the stages.  A stage starts once every CTA has
//    finished the previous one (a per-stage arrival counter in global memory,
//    release / acquire at GPU scope, every wait bounded by %globaltimer);
//  * GEMV stages compute on the FP8 tensor cores (mma.sync m16n8k32 E4M3,
//    FP32 accumulation): the weights are the A operand (16 rows x 32 K per
//    MMA), x is the B operand with its E4M3 hi part in column 0 and lo part
//    in column 1 (x * 2^e = hi + lo / 32 per 128-wide K block, exact for the
//    BF16 values within 2^-14 of the block maximum), so one MMA gives both
//    partial sums of 16 rows.  Scale x 2^-e is applied per 128-K block in
//    FP32, as the reference's explicit dequantisation does (main.py:497-501).
//
// Weights are stored pre-packed for this kernel (qwen_step_pack): per 32-row
// tile and 512-wide K chunk, 16 KB laid out so that one 16-byte shared load
// per lane is exactly the lane's A fragments of two MMAs, followed by the
// chunk's four FP32 block scales.  A chunk is one bulk copy.
//
// Summation order differs from the reference kernels (per-chunk tensor-core
// sums, then chunk partials in order); products are exact and sums FP32, as
// in the reference.  The result does not depend on timing: every sum is taken
// in a fixed order.
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "gdn.cuh"
#include "attn.cuh"

namespace qwen {

#ifndef QWEN_STEP_SLOTS
#define QWEN_STEP_SLOTS 12
#endif
#ifndef QWEN_STEP_ATTN_SLOTS
#define QWEN_STEP_ATTN_SLOTS 3
#endif

enum : int { ST_GEMV = 0, ST_GDN = 1, ST_ATTN = 2 };
// x prologue of a GEMV stage
enum : int {
  STP_PLAIN = 0,        // x as given (BF16 vector)
  STP_NORM = 1,         // x <- RMSNorm(1+w)(x)
  STP_EMBED_NORM = 2,   // h <- table[*token] (CTA 0 stores h), x <- RMSNorm(1+w)(h)
  STP_SLICES_NORM = 3,  // h <- bf16(res + bf16(sum of the slices, in order)) (CTA 0 stores h), x <- RMSNorm(1+w)(h)
};
enum : unsigned {
  ERR_STEP_TIMEOUT = 8,  // a bounded wait of the step kernel gave up (the step was abandoned)
  ERR_TOKEN_RANGE = 9,   // an embedding row index outside the table (row 0 used)
};

constexpr int ST_ROWS = 32;                    // weight rows per tile (two MMA row groups of 16)
constexpr int ST_KC = 512;                     // K per chunk
constexpr int ST_WBYTES = ST_ROWS * ST_KC;     // 16384 weight bytes per chunk
constexpr int ST_CHUNK = ST_WBYTES + 16;       // + four FP32 block scales
// Ring of chunk slots.  The bulk-copy engine's rate grows with the size of a
// copy (measured on B200 through a 128-192 KB ring: 8 KB copies 5.2 TB/s,
// 16 KB 6.4-6.8, 32 KB 6.9), hence 16 KB chunks.  A chunk is computed by a
// pair of consumer warps (one 16-row group each), so a slot is held half as
// long and more of the ring stays in flight.  The slot count is a multiple of
// the warp pairs: items m and m + ST_SLOTS share a slot and go to the same
// pair, so no thread ever waits on a phase beyond the next one of a slot's
// barrier (a parity wait cannot tell those apart).
constexpr int ST_SLOTS = QWEN_STEP_SLOTS;
constexpr int ST_CW = 8;                       // consumer warps
constexpr int ST_PAIRS = ST_CW / 2;            // consumer warp pairs (one chunk each)
constexpr int ST_NT = ST_CW * 32;
constexpr int ST_THREADS = ST_NT + 32;         // + the producer warp
constexpr int ST_MAXK = 9216;                  // longest GEMV input
constexpr int ST_MAXB = (ST_MAXK / 128 + ST_CW - 1) / ST_CW;  // 128-blocks per warp in the prologue
constexpr int ST_NORM_MAXK = 3072;             // longest input of a normalising (or embedding) prologue
constexpr int ST_NORM_MAXB = ST_NORM_MAXK / 128 / ST_CW;
constexpr int ST_SL_REG = 4;                   // K-slice rows a prologue loads in one round trip
constexpr int ST_BATCH = 48;                   // chunk partials held before a reduction
constexpr int ST_MAX_SEG = 6;
constexpr int ST_ATTN_SLOTS = QWEN_STEP_ATTN_SLOTS;  // contiguous ring slots of scratch for an attention unit
constexpr int ST_GDN_D = 128;                  // GatedDeltaNet head dim of the step kernel
// A GatedDeltaNet unit is one block of ST_GDN_DC value columns of one head:
// its FP32 state [D keys][DC values] is one contiguous ring slot (the step
// kernel's state layout is [head][value block][key][DC]).
constexpr int ST_GDN_VS = 4;
constexpr int ST_GDN_DC = ST_GDN_D / ST_GDN_VS;  // 32
constexpr int ST_GDN_KG = ST_NT / ST_GDN_DC;     // 8 key groups (a thread: one column, KR keys)
constexpr int ST_GDN_KR = ST_GDN_D / ST_GDN_KG;  // 16
constexpr int ST_GATED_MAXB = 4096 / 128 / ST_CW;  // 128-blocks per warp of a gated prologue (K <= 4096)
static_assert(ST_GDN_D * ST_GDN_DC * 4 == ST_WBYTES, "a GatedDeltaNet unit's state is one ring slot");
static_assert(ST_GDN_KG * ST_GDN_KR == ST_GDN_D && ST_GDN_KG == 8, "key groups");
static_assert(ST_SLOTS % ST_PAIRS == 0, "items m and m + ST_SLOTS must go to the same consumer warp pair");
static_assert(ST_SLOTS % ST_ATTN_SLOTS == 0, "attention scratch groups must not wrap the ring");
// an attention unit waits for its alignment padding plus its scratch slots at
// once (up to 2 * ST_ATTN_SLOTS - 1 items): they must fit the ring together
static_assert(2 * ST_ATTN_SLOTS - 1 <= ST_SLOTS, "attention padding + scratch must fit the ring");
static_assert(ST_NT == ATTN_WARPS * 32, "attention units run on the consumer warps");


struct alignas(16) StStage {
  int kind;
  // GEMV
  int K, C;            // input length; 512-wide chunks per tile row
  int pro;
  int nseg, pair, nslice, tiles, nunits, ipu;  // units = tiles x nslice; ipu = chunks (items) per unit
  int x_rows;          // EMBED: rows of the table
  const bf16* x;       // PLAIN / NORM input, EMBED table
  const bf16* res;     // SLICES_NORM residual
  const float* norm_w;
  float eps;
  bf16* h_out;         // EMBED / SLICES_NORM: the residual stream h (written by CTA 0)
  const long long* token;
  const float* sl_in;  // SLICES_NORM: [sl_in_count][sl_stride] FP32 partial rows
  int sl_in_count, sl_stride;
  float* sl_out;       // K-sliced output: [nslice][sl_rows]
  int sl_rows;
  unsigned long long* am_ws;        // ARGMAX: {key, count}, zero before the first step, left zeroed
  unsigned long long* am_key_out;
  long long* am_token_out;
  int* pos_inc;
  int seg_tile0[ST_MAX_SEG + 1];
  GemvSeg seg[ST_MAX_SEG];          // w / w2: packed weights
  // GatedDeltaNet: one unit per value head
  GdnArgs gdn;
  int gdn_heads;
  // attention: one unit per (KV head, split)
  AttnArgs attn;
  int attn_dim, attn_g;
  int wbf16;           // GEMV: BF16 weights (chunks of 32 rows x 256 K), x kept as BF16
  // this rank's share (tensor parallel): GEMV units cover tiles shard0 ..,
  // GatedDeltaNet heads shard0 .. shard0 + gdn_heads, attention KV heads
  // shard0 .. shard0 + attn_kv (0 and the whole stage on one GPU)
  int shard0, attn_kv;
  // tensor parallel: the stage's K-slice partial rows go to every rank as
  // tagged words (row-parallel projections); other stages stay on their rank
  int xrank;
  int cstride;         // GEMV: chunks per tile row of the packed matrices (> C when a rank takes a K range)
  // SLICES_NORM prologue: index of the xrank stage whose tagged slices it
  // sums (polled until they carry that stage's tag of this step), or -1
  int sl_src;
  // PLAIN prologue over a GatedDeltaNet stage's core output (x): the gated
  // RMSNorm of every 128-wide block (one head) is applied first,
  // bf16(bf16(bf16(c / rms(c)) w) zs), with zs = bf16(silu(z)) at gz (same
  // layout as x) and the head's norm weights gnw [128]
  int gated_pro;
  const bf16* gz;
  const bf16* gnw;
  float geps;
  int pad_[3];
};

// Shared memory plan (bytes from the dynamic shared memory base).
struct StSmem {
  static constexpr int ring = 0;
  static constexpr int xh = ST_SLOTS * ST_CHUNK;
  static constexpr int xl = xh + ST_MAXK;
  static constexpr int xinv = xl + ST_MAXK;
  static constexpr int part = xinv + ST_MAXK / 128 * 4;
  static constexpr int red = part + ST_BATCH * ST_ROWS * 4;
  static constexpr int misc = red + 64 * 4;
  static constexpr int bars = misc + 32 * 8;
  // the descriptors of the running stage and the next one (16-byte copies)
  static constexpr int desc = (bars + 2 * ST_SLOTS * 8 + 15) / 16 * 16;
  static constexpr int total = desc + 2 * (int)sizeof(StStage);
};
static_assert(StSmem::xh % 16 == 0 && StSmem::part % 16 == 0 && StSmem::bars % 8 == 0, "alignment");
static_assert(sizeof(StStage) % 16 == 0, "stage descriptors are copied in 16-byte pieces");
static_assert(StSmem::total <= 227 * 1024, "shared memory");

constexpr int ST_MAX_WORLD = 8;  // ranks of a tensor-parallel program (one GPU each)

struct StProgram {
  const StStage* stages;
  int nstages;
  // [2 nstages + 1], monotonic over the program's steps (nothing is cleared):
  // [0, nstages) unused, [nstages, 2 nstages) this GPU's CTAs done with each
  // stage, [2 nstages] this GPU's completed steps x grid, from which a launch
  // takes its epoch e.  Stage s is complete on this GPU when
  // counters[nstages + s] reaches (e + 1) x grid.  Tensor parallel: the
  // stage after a row-parallel (xrank) stage polls that stage's tagged
  // K-slice words of every rank instead (tag e x nstages + 1 + s).
  unsigned long long* counters;
  unsigned* abort_flag;  // set by a timed-out wait; every wait then gives up at once
  unsigned* timeline;    // optional [nstages][grid][ST_TL]: %globaltimer (low 32 bits, ns) per stage and CTA
  const int* pos;        // decode position read by the attention stages (constant within a step), or null
  int drop_stage;        // test hook: CTA 0 does not report stage drop_stage done (-1: off)
  // Tensor parallel (world > 1): rank r's copy of any shared-arena object is
  // at the local address + peer_off[r] (peer_off[rank] = 0).  The tagged
  // K-slice words of row-parallel stages, the LM-head logits and the argmax
  // workspace are written to every rank; everything else stays local.
  int world, rank;
  long long peer_off[ST_MAX_WORLD];
};

// rank r's copy of a shared-arena object
template <typename T>
__device__ __forceinline__ T* st_peer(const StProgram& P, T* p, int r) {
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p) + P.peer_off[r]);
}
template <typename T>
__device__ __forceinline__ void st_put_local(T* p, T v) {
  *p = v;
}
// a stage output element, stored on every rank
template <typename T>
__device__ __forceinline__ void st_put(const StProgram& P, T* p, T v) {
  if (P.world == 1) {
    *p = v;
    return;
  }
  for (int r = 0; r < P.world; ++r) *st_peer(P, p, r) = v;
}

// Tagged K-slice words of a row-parallel stage (tensor parallel): the FP32
// value's bits | tag << 32, stored on every rank with one 8-byte store each.
// 64-bit accesses are single-copy atomic, so a reader that sees the tag of
// this step's stage sees the value; no fence or counter orders them.
__device__ __forceinline__ void st_put_tagged(const StProgram& P, unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  for (int r = 0; r < P.world; ++r)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(st_peer(P, p, r)), "l"(w) : "memory");
}
__device__ __forceinline__ void st_ll_load(const unsigned long long* p, ulonglong2& a, ulonglong2& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a.x), "=l"(a.y) : "l"(p) : "memory");
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(b.x), "=l"(b.y) : "l"(p + 2) : "memory");
}
__device__ __forceinline__ bool st_ll_ok(const ulonglong2& a, const ulonglong2& b, uint32_t tag) {
  return ((uint32_t)(a.x >> 32) == tag) & ((uint32_t)(a.y >> 32) == tag) & ((uint32_t)(b.x >> 32) == tag) &
         ((uint32_t)(b.y >> 32) == tag);
}

// Timeline fields of one (stage, CTA): the consumers' wait for the previous
// stage begins / ends, their work ends; the producer issues the stage's first
// item / has issued its last one.
// Also, in ns: the producer's time blocked on a full ring while issuing the
// stage, and consumer warp 0's time blocked on copies not yet landed.
// Then, for GEMV stages: the stamps at which the x prologue was done and the
// last batch's chunks were, and consumer warp 0's SM cycles inside the chunk
// math; for GatedDeltaNet stages the stamps at which the last head's inputs
// had arrived and its state update was done; for attention stages the
// stamps after the unit's q / k / v preparation, after its partials were
// published and (the combining unit) after the combine.
enum : int {
  ST_TL_WAIT = 0, ST_TL_START = 1, ST_TL_END = 2, ST_TL_P0 = 3, ST_TL_P1 = 4, ST_TL_PBLOCK = 5, ST_TL_CBLOCK = 6,
  ST_TL_PRO = 7, ST_TL_CHUNKS = 8, ST_TL_WCOMP = 9, ST_TL = 10
};
__device__ __forceinline__ void st_stamp(const StProgram& P, int s, int field) {
  if (P.timeline) P.timeline[((size_t)s * gridDim.x + blockIdx.x) * ST_TL + field] = (unsigned)globaltimer_ns();
}
__device__ __forceinline__ void st_tl_put(unsigned* tl, int s, int field, unsigned v) {
  if (tl) tl[((size_t)s * gridDim.x + blockIdx.x) * ST_TL + field] = v;
}

// ---------------------------------------------------------------------------
// Waits and arrivals
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool st_aborted(const unsigned* abort_flag) {
  return *reinterpret_cast<const volatile unsigned*>(abort_flag) != 0u;
}
__device__ __forceinline__ void st_abort(unsigned* abort_flag) {
  qwen_err_set(ERR_STEP_TIMEOUT);
  atomicExch(abort_flag, 1u);
}

// mbarrier phase wait, bounded by QWEN_WAIT_TIMEOUT_NS and by the abort flag.
__device__ __forceinline__ bool st_mbar_wait(uint32_t bar, uint32_t parity, unsigned* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns(), lim = qwen_wait_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (st_aborted(abort_flag)) return false;
    if (globaltimer_ns() - t0 > lim) {
      st_abort(abort_flag);
      return false;
    }
  }
}

// Wait until `count` CTAs have arrived at `counter` (acquire, GPU scope).
__device__ __forceinline__ unsigned long long st_ld_acq_u64(const unsigned long long* p, bool sys) {
  unsigned long long v;
  if (sys)
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Wait until `counter` reaches `count` (acquire; system scope when other GPUs arrive on it).
__device__ __forceinline__ bool st_wait_count(const unsigned long long* counter, unsigned long long count,
                                              unsigned* abort_flag, bool sys) {
  if (st_ld_acq_u64(counter, sys) >= count) return true;
  const uint64_t t0 = globaltimer_ns(), lim = qwen_wait_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (st_ld_acq_u64(counter, sys) >= count) return true;
    if (st_aborted(abort_flag)) return false;
    if (globaltimer_ns() - t0 > lim) {
      st_abort(abort_flag);
      return false;
    }
  }
}

// Named barrier over `n` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool named_bar_and(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred pi, po;\n setp.ne.u32 pi, %1, 0;\n bar.red.and.pred po, %2, %3, pi;\n selp.u32 %0, 1, 0, po;\n}\n"
      : "=r"(r) : "r"((uint32_t)v), "r"(id), "r"(n) : "memory");
  return r != 0;
}

// This CTA's contiguous share [u0, u1) of n units.
__device__ __forceinline__ int st_attn_pad(uint32_t n) {
  return (int)((ST_ATTN_SLOTS - n % ST_ATTN_SLOTS) % ST_ATTN_SLOTS);
}
__device__ __forceinline__ void st_range(int n, int& u0, int& u1) {
  u0 = (int)(((long long)n * blockIdx.x) / gridDim.x);
  u1 = (int)(((long long)n * (blockIdx.x + 1)) / gridDim.x);
}
__device__ __forceinline__ int st_find_seg(const StStage& S, int t) {
  int sg = 0;
#pragma unroll
  for (int i = 1; i < ST_MAX_SEG; ++i)
    if (i < S.nseg && t >= S.seg_tile0[i]) sg = i;
  return sg;
}

// ---------------------------------------------------------------------------
// Producer: one thread streams every item of this CTA, stage by stage.
// Item m goes to slot m % ST_SLOTS; the slot's `full` barrier completes with
// the copy, its `empty` barrier when the consumer has finished with it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_producer(const StProgram& P, uint32_t ring, uint32_t full0, uint32_t empty0) {
  const uint64_t pol = l2_policy_evict_first();
  uint32_t n = 0;
  bool ok = true;
  uint64_t blocked = 0;  // timeline only
  auto acquire = [&](uint32_t& slot) -> bool {
    slot = n % ST_SLOTS;
    if (n < (uint32_t)ST_SLOTS) return true;
    const uint32_t bar = empty0 + 8 * slot, par = ((n / ST_SLOTS) - 1) & 1u;
    if (P.timeline ? mbar_test_wait(bar, par) : mbar_try_wait(bar, par)) return true;
    const uint64_t t0 = P.timeline ? globaltimer_ns() : 0;
    const bool r = st_mbar_wait(bar, par, P.abort_flag);
    if (P.timeline) blocked += globaltimer_ns() - t0;
    return r;
  };
  for (int s = 0; s < P.nstages && ok; ++s) {
    const StStage& S = P.stages[s];
    int u0, u1;
    st_stamp(P, s, ST_TL_P0);
    blocked = 0;
    if (S.kind == ST_GEMV) {
      // the stage's fields in registers: the copies below are asm with memory
      // clobbers, after which the compiler would reload them from global memory
      const int ns = S.nslice, ipu = S.ipu, pair = S.pair, nseg = S.nseg, tiles_my = S.nunits / ns;
      const size_t tile_bytes = (size_t)S.cstride * ST_CHUNK, slice_bytes = (size_t)(S.C / ns) * ST_CHUNK;
      int t0[ST_MAX_SEG];
      const uint8_t* wa[ST_MAX_SEG];
      const uint8_t* wb[ST_MAX_SEG];
#pragma unroll
      for (int i = 0; i < ST_MAX_SEG; ++i) {
        t0[i] = S.seg_tile0[i];
        wa[i] = S.seg[i].w;
        wb[i] = S.seg[i].w2;
      }
      st_range(S.nunits, u0, u1);
      const int shard0 = S.shard0;
      for (int u = u0; u < u1 && ok; ++u) {
        const int sl = u / tiles_my, tl = u - sl * tiles_my, t = shard0 + tl;  // slice-major units
        const uint8_t* a = wa[0];
        const uint8_t* b = wb[0];
        int tb = t0[0];
#pragma unroll
        for (int i = 1; i < ST_MAX_SEG; ++i)
          if (i < nseg && t >= t0[i]) {
            a = wa[i];
            b = wb[i];
            tb = t0[i];
          }
        const size_t off = (size_t)(t - tb) * tile_bytes + (size_t)sl * slice_bytes;
        a += off;
        b = pair ? b + off : nullptr;
        for (int i = 0; i < ipu; ++i) {
          const uint8_t* src = pair ? ((i & 1) ? b : a) + (size_t)(i >> 1) * ST_CHUNK : a + (size_t)i * ST_CHUNK;
          uint32_t slot;
          if (!(ok = acquire(slot))) break;
          mbar_arrive_expect_tx(full0 + 8 * slot, ST_CHUNK);
          bulk_g2s(ring + slot * ST_CHUNK, src, ST_CHUNK, full0 + 8 * slot, pol);
          ++n;
        }
      }
    } else if (S.kind == ST_GDN) {
      // one slot per (head, value block): that block's state
      st_range(S.gdn_heads * ST_GDN_VS, u0, u1);
      const uint8_t* state = reinterpret_cast<const uint8_t*>(S.gdn.state);
      for (int u = u0; u < u1 && ok; ++u) {
        const uint8_t* src = state + ((size_t)S.shard0 * ST_GDN_VS + u) * ST_WBYTES;
        uint32_t slot;
        if (!(ok = acquire(slot))) break;
        mbar_arrive_expect_tx(full0 + 8 * slot, ST_WBYTES);
        bulk_g2s(ring + slot * ST_CHUNK, src, ST_WBYTES, full0 + 8 * slot, pol);
        ++n;
      }
    } else {  // ST_ATTN: scratch slots, no copy (a plain arrival completes the phase)
      st_range(S.attn_kv * S.attn.nsplit, u0, u1);
      for (int u = u0; u < u1 && ok; ++u) {
        const int cnt = st_attn_pad(n) + ST_ATTN_SLOTS;
        for (int i = 0; i < cnt; ++i) {
          uint32_t slot;
          if (!(ok = acquire(slot))) break;
          mbar_arrive(full0 + 8 * slot);
          ++n;
        }
      }
    }
    st_stamp(P, s, ST_TL_P1);
    st_tl_put(P.timeline, s, ST_TL_PBLOCK, (unsigned)blocked);
  }
  // Drain: never leave the CTA with bulk copies in flight into its shared memory.
  const uint32_t first = n > (uint32_t)ST_SLOTS ? n - ST_SLOTS : 0u;
  for (uint32_t m = first; m < n; ++m) {
    const uint32_t bar = full0 + 8 * (m % ST_SLOTS), par = (m / ST_SLOTS) & 1u;
    if (mbar_try_wait(bar, par)) continue;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, par)) {
      if (globaltimer_ns() - t0 > QWEN_WAIT_TIMEOUT_NS) {
        st_abort(P.abort_flag);
        break;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// GEMV stage pieces
// ---------------------------------------------------------------------------
// x prologue (consumer threads, named barrier 1): the stage input in shared
// memory as E4M3 hi (xh) and lo (xl) bytes per element and 2^-e per 128-K
// block (xinv).  Warp w takes 128-blocks w, w + 8, ...; lane l elements
// 4l .. 4l + 3 of each.  Inputs written earlier in the step are read at L2.
// Every load of a phase is issued before any is used: while the weight
// stream saturates HBM an L2 round trip takes ~0.5 us, so dependent loads
// would cost a round trip each.  MB: 128-blocks per warp this instantiation
// holds (norm stages: K <= 3072); SLR: K-slice rows loaded with the first
// round trip (0 for the plain prologue).
// Four K-slice values at element `idx` of a slice buffer: FP32, or the low
// halves of tagged words (tensor parallel, already seen with their tag).
__device__ __forceinline__ float4 st_slice4(const float* sl, size_t idx, bool tagged) {
  if (!tagged) return __ldcg(reinterpret_cast<const float4*>(sl + idx));
  ulonglong2 a, b;
  st_ll_load(reinterpret_cast<const unsigned long long*>(sl) + idx, a, b);
  return make_float4(__uint_as_float((uint32_t)a.x), __uint_as_float((uint32_t)a.y), __uint_as_float((uint32_t)b.x),
                     __uint_as_float((uint32_t)b.y));
}

// Wait until every tagged word this thread's prologue reads (nsl slices of
// the 128-blocks warp, warp + 8, ... of K) carries `tag`: all tags loaded at
// once, the whole set again while any is missing (bounded by the wait limit
// and the abort flag; on time-out the step is abandoned with error 8).
__device__ __forceinline__ void st_ll_wait_all(const unsigned long long* sl, int nsl, int stride, int nb, uint32_t tag,
                                            unsigned* abort_flag) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t t0 = 0;
  for (int tries = 0;; ++tries) {
    bool ok = true;
    for (int c = 0; c < nsl; ++c)
#pragma unroll 4
      for (int b = warp; b < nb; b += ST_CW) {
        ulonglong2 x, y;
        st_ll_load(sl + (size_t)c * stride + b * 128 + lane * 4, x, y);
        ok &= st_ll_ok(x, y, tag);
      }
    if (ok || st_aborted(abort_flag)) return;
    if (tries == 0) t0 = globaltimer_ns();
    if (globaltimer_ns() - t0 > qwen_wait_ns()) {
      st_abort(abort_flag);
      return;
    }
  }
}

template <int MB, int SLR, bool GATED = false>
__device__ __forceinline__ void st_prologue(const StStage& S, uint8_t* xh, uint8_t* xl, float* xinv, float* red,
                                            uint32_t ll_tag, unsigned* abort_flag, int blo, int bhi) {
  // 128-wide blocks [blo, bhi) of x (a PLAIN prologue prepares only the K
  // range of this CTA's units; a normalising one needs all of K)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = S.K, nb = bhi, pro = S.pro, nsl = S.sl_in_count, sl_stride = S.sl_stride;
  // tagged slices of a row-parallel stage (tensor parallel): waited for
  // first, then read like FP32 slices (the low halves of the words)
  const bool ll = pro == STP_SLICES_NORM && S.sl_src >= 0;
  const float* sl_in = S.sl_in;
  const float* norm_w = S.norm_w;
  const bool norm = pro != STP_PLAIN;
  const bf16* xin = S.x;
  if (pro == STP_EMBED_NORM) {
    long long tok = __ldcg(S.token);
    if (tok < 0 || tok >= S.x_rows) {
      if (tid == 0 && blockIdx.x == 0) qwen_err_set(ERR_TOKEN_RANGE);
      tok = 0;
    }
    xin += (size_t)tok * K;
  }
  const bf16* src = pro == STP_SLICES_NORM ? S.res : xin;
  bf16* h_out = (blockIdx.x == 0 && (pro == STP_SLICES_NORM || pro == STP_EMBED_NORM)) ? S.h_out : nullptr;
  // every load at once (the input or residual, the norm weights and up to
  // ST_SL_REG K-slice rows), added in slice order once they have arrived
  uint2 raw[MB];
  float4 wv[MB];
  float4 sp[MB][SLR > 0 ? SLR : 1];
  uint2 zr[GATED ? MB : 1];
  uint2 gw = make_uint2(0u, 0u);
  if (GATED) gw = __ldg(reinterpret_cast<const uint2*>(S.gnw + lane * 4));  // a block is one head
  const int nreg = pro == STP_SLICES_NORM ? (nsl < SLR ? nsl : SLR) : 0;
#pragma unroll
  for (int i = 0; i < MB; ++i) {
    const int b = blo + warp + i * ST_CW;
    const int k0 = b * 128 + lane * 4;
    if (b < nb) {
      raw[i] = pro == STP_EMBED_NORM ? __ldg(reinterpret_cast<const uint2*>(src + k0))
                                     : __ldcg(reinterpret_cast<const uint2*>(src + k0));
      if (norm) wv[i] = __ldg(reinterpret_cast<const float4*>(norm_w + k0));
      if (GATED) zr[GATED ? i : 0] = __ldcg(reinterpret_cast<const uint2*>(S.gz + k0));
    }
  }
  // (the residual and norm loads above are in flight while the tags are polled)
  if (ll) st_ll_wait_all(reinterpret_cast<const unsigned long long*>(sl_in), nsl, sl_stride, nb, ll_tag, abort_flag);
#pragma unroll
  for (int i = 0; i < MB; ++i) {
    const int b = blo + warp + i * ST_CW;
    const int k0 = b * 128 + lane * 4;
    if (b < nb) {
#pragma unroll
      for (int c = 0; c < SLR; ++c)
        if (c < nreg) sp[i][c] = st_slice4(sl_in, (size_t)c * sl_stride + k0, ll);
    }
  }
  float v[MB][4];
#pragma unroll
  for (int i = 0; i < MB; ++i) {
    const float2 a01 = bf2x_to_f2(raw[i].x), a23 = bf2x_to_f2(raw[i].y);
    v[i][0] = a01.x; v[i][1] = a01.y; v[i][2] = a23.x; v[i][3] = a23.y;
  }
  if (GATED) {
    // the GatedDeltaNet's gated RMSNorm per head (main.py:1152-1159):
    // bf16(c / rms(c)), times the norm weight, times bf16(silu(z))
    const float2 w01 = bf2x_to_f2(gw.x), w23 = bf2x_to_f2(gw.y);
    const float nw[4] = {w01.x, w01.y, w23.x, w23.y};
#pragma unroll
    for (int i = 0; i < MB; ++i) {
      const int b = blo + warp + i * ST_CW;
      const float cs = warp_sum(v[i][0] * v[i][0] + v[i][1] * v[i][1] + v[i][2] * v[i][2] + v[i][3] * v[i][3]);
      if (b >= nb) continue;  // warp-uniform
      const float inv = rsqrtf(cs / (float)ST_GDN_D + S.geps);
      const float2 z01 = bf2x_to_f2(zr[GATED ? i : 0].x), z23 = bf2x_to_f2(zr[GATED ? i : 0].y);
      const float zs[4] = {z01.x, z01.y, z23.x, z23.y};  // bf16(silu(z)), from in_proj's EPI_SILU
#pragma unroll
      for (int q = 0; q < 4; ++q) v[i][q] = bfround(bfround(bfround(v[i][q] * inv) * nw[q]) * zs[q]);
    }
  }
  if (pro == STP_SLICES_NORM) {
    float sum[MB][4];
#pragma unroll
    for (int i = 0; i < MB; ++i) {
      sum[i][0] = sum[i][1] = sum[i][2] = sum[i][3] = 0.f;
#pragma unroll
      for (int c = 0; c < SLR; ++c)
        if (c < nreg) {
          sum[i][0] += sp[i][c].x; sum[i][1] += sp[i][c].y; sum[i][2] += sp[i][c].z; sum[i][3] += sp[i][c].w;
        }
    }
    // slices beyond SLR: SLR more rows per round trip, added in slice order
    for (int c0 = nreg; c0 < nsl; c0 += SLR) {
#pragma unroll
      for (int i = 0; i < MB; ++i) {
        const int b = blo + warp + i * ST_CW;
#pragma unroll
        for (int c = 0; c < SLR; ++c)
          if (b < nb && c0 + c < nsl)
            sp[i][c] = st_slice4(sl_in, (size_t)(c0 + c) * sl_stride + b * 128 + lane * 4, ll);
      }
#pragma unroll
      for (int i = 0; i < MB; ++i)
#pragma unroll
        for (int c = 0; c < SLR; ++c)
          if (c0 + c < nsl) {
            sum[i][0] += sp[i][c].x; sum[i][1] += sp[i][c].y; sum[i][2] += sp[i][c].z; sum[i][3] += sp[i][c].w;
          }
    }
#pragma unroll
    for (int i = 0; i < MB; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q) v[i][q] = bfround(v[i][q] + bfround(sum[i][q]));
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MB; ++i) {
    const int b = blo + warp + i * ST_CW;
    if (b >= nb) continue;
    const int k0 = b * 128 + lane * 4;
    if (h_out) {
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(v[i][0], v[i][1]);
      const __nv_bfloat162 h23 = __floats2bfloat162_rn(v[i][2], v[i][3]);
      uint2 hv;
      hv.x = *reinterpret_cast<const uint32_t*>(&h01);
      hv.y = *reinterpret_cast<const uint32_t*>(&h23);
      *reinterpret_cast<uint2*>(h_out + k0) = hv;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) ss = fmaf(v[i][q], v[i][q], ss);
  }
  float rms = 1.f;
  if (norm) {
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    named_bar(1, ST_NT);
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < ST_CW; ++i) tot += red[i];
    rms = rsqrtf(tot / (float)K + S.eps);
  }
  // normalised values and every block's maximum, the blocks' shuffle
  // reductions interleaved
  float mx[MB];
#pragma unroll
  for (int i = 0; i < MB; ++i) {
    if (norm) {
      const float4 w = wv[i];
      v[i][0] = bfround(v[i][0] * rms * (1.0f + w.x));
      v[i][1] = bfround(v[i][1] * rms * (1.0f + w.y));
      v[i][2] = bfround(v[i][2] * rms * (1.0f + w.z));
      v[i][3] = bfround(v[i][3] * rms * (1.0f + w.w));
    }
    mx[i] = fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int i = 0; i < MB; ++i) mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], o));
#pragma unroll
  for (int i = 0; i < MB; ++i) {
    const int b = blo + warp + i * ST_CW;
    if (b >= nb) continue;  // warp-uniform
    const int k0 = b * 128 + lane * 4;
    if (S.wbf16) {  // BF16 weights: x stays BF16 (xh holds K BF16 values)
      const __nv_bfloat162 p01 = __floats2bfloat162_rn(v[i][0], v[i][1]);
      const __nv_bfloat162 p23 = __floats2bfloat162_rn(v[i][2], v[i][3]);
      uint2 pv;
      pv.x = *reinterpret_cast<const uint32_t*>(&p01);
      pv.y = *reinterpret_cast<const uint32_t*>(&p23);
      *reinterpret_cast<uint2*>(xh + 2 * k0) = pv;
      continue;
    }
    const float x[4] = {v[i][0], v[i][1], v[i][2], v[i][3]};
    const float m = mx[i];
    // m = 1.f * 2^(ebits - 127): e = 134 - ebits puts m * 2^e in [2^7, 2^8)
    const int ebits = (int)((__float_as_uint(m) >> 23) & 0xffu);
    int e = m > 0.f ? (ebits == 0 ? 100 : 134 - ebits) : 0;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
    const float sc = exp2i(e);
    float xs[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) xs[q] = x[q] * sc;
    const uint32_t h01 = f32x2_to_e4m3x2(xs[0], xs[1]), h23 = f32x2_to_e4m3x2(xs[2], xs[3]);
    const float2 g01 = h2u_to_f2(e4m3x2_to_f16x2(h01)), g23 = h2u_to_f2(e4m3x2_to_f16x2(h23));
    // lo carries 32 * (x * 2^e - hi): |x * 2^e - hi| <= 8, so 32x stays below 448
    const uint32_t l01 = f32x2_to_e4m3x2((xs[0] - g01.x) * 32.f, (xs[1] - g01.y) * 32.f);
    const uint32_t l23 = f32x2_to_e4m3x2((xs[2] - g23.x) * 32.f, (xs[3] - g23.y) * 32.f);
    *reinterpret_cast<uint32_t*>(xh + k0) = h01 | (h23 << 16);
    *reinterpret_cast<uint32_t*>(xl + k0) = l01 | (l23 << 16);
    if (lane == 0) xinv[b] = exp2i(-e);
  }
  named_bar(1, ST_NT);
}

// FP8 tensor-core MMA D (16x8 f32) = A (16x32 E4M3) x B (32x8 E4M3) (+ C),
// as plain (non-volatile) asm so the compiler may interleave independent
// MMAs and hoist the shared-memory loads that feed them.
__device__ __forceinline__ void st_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 16-row group (rg) of a chunk (32 rows x 512 K) on one warp: FP32
// partial sums of rows 16 rg + g and 16 rg + g + 8, valid in lanes with
// lane % 4 == 0 (g = lane / 4).  All 24 shared loads are issued first; the
// four 128-K blocks are four independent accumulator chains.
__device__ __forceinline__ void st_chunk(const uint8_t* base, const uint8_t* xh, const uint8_t* xl, const float* xinv,
                                         int c, int rg, int lane, float& a0, float& a1) {
  const float4 sc = *reinterpret_cast<const float4*>(base + ST_WBYTES);
  const float* xi = xinv + c * 4;
  // B fragments: lanes 0-3 (column 0) the hi bytes, lanes 4-7 (column 1) the
  // lo bytes of K [512c + 64j + 16(lane % 4), +16) for group j; other columns zero
  uint4 xr[8];
  const uint8_t* xs = (lane < 4 ? xh : xl) + c * ST_KC + (lane & 3) * 16;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    xr[j] = lane < 8 ? *reinterpret_cast<const uint4*>(xs + 64 * j) : make_uint4(0u, 0u, 0u, 0u);
  const uint8_t* wl = base + rg * (ST_WBYTES / 2) + lane * 16;
  uint4 w0[8], w1[8];  // group j: row g (w0) and row g + 8 (w1)
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    w0[j] = *reinterpret_cast<const uint4*>(wl + (2 * j) * 512);
    w1[j] = *reinterpret_cast<const uint4*>(wl + (2 * j + 1) * 512);
  }
  float d[4][4];
#pragma unroll
  for (int kb = 0; kb < 4; ++kb) d[kb][0] = d[kb][1] = d[kb][2] = d[kb][3] = 0.f;
#pragma unroll
  for (int step = 0; step < 4; ++step)  // MMA `step` of every block's chain
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
      const int j = 2 * kb + (step >> 1);
      if ((step & 1) == 0)
        st_mma(d[kb], w0[j].x, w1[j].x, w0[j].y, w1[j].y, xr[j].x, xr[j].y);
      else
        st_mma(d[kb], w0[j].z, w1[j].z, w0[j].w, w1[j].w, xr[j].z, xr[j].w);
    }
  const float f[4] = {sc.x * xi[0], sc.y * xi[1], sc.z * xi[2], sc.w * xi[3]};
  a0 = 0.f;
  a1 = 0.f;
#pragma unroll
  for (int kb = 0; kb < 4; ++kb) {
    a0 = fmaf(f[kb], d[kb][0] + d[kb][1] * 0.03125f, a0);
    a1 = fmaf(f[kb], d[kb][2] + d[kb][3] * 0.03125f, a1);
  }
}

// BF16 MMA D (16x8 f32) = A (16x16 BF16) x B (16x8 BF16) + D.
__device__ __forceinline__ void st_mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 16-row group (rg) of a BF16 chunk (32 rows x 256 K) on one warp: the
// chunk holds, per group and 16-K step j, each lane's A fragment as 16
// contiguous bytes; x (BF16) is the B operand's column 0 (lanes 0-3), so
// lanes with lane % 4 == 0 end with the FP32 sums of rows 16 rg + lane / 4
// (a0) and + 8 (a1).  Four independent accumulator chains.
__device__ __forceinline__ void st_chunk_bf16(const uint8_t* base, const bf16* xs, int c, int rg, int lane, float& a0,
                                              float& a1) {
  const uint8_t* wl = base + rg * (ST_WBYTES / 2) + lane * 16;
  const bf16* xc = xs + c * 256 + 2 * (lane & 3);
  float d[4][4];
#pragma unroll
  for (int q = 0; q < 4; ++q) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint4 w = *reinterpret_cast<const uint4*>(wl + j * 512);
    uint32_t b0 = 0u, b1 = 0u;
    if (lane < 4) {
      b0 = *reinterpret_cast<const uint32_t*>(xc + 16 * j);
      b1 = *reinterpret_cast<const uint32_t*>(xc + 16 * j + 8);
    }
    st_mma_bf16(d[j & 3], w.x, w.y, w.z, w.w, b0, b1);
  }
  a0 = (d[0][0] + d[1][0]) + (d[2][0] + d[3][0]);
  a1 = (d[0][2] + d[1][2]) + (d[2][2] + d[3][2]);
}

// Row epilogue of a GEMV stage: gemv_epilogue's arithmetic (gemv.cuh).
__device__ __forceinline__ unsigned long long st_epilogue(const StProgram& P, const GemvSeg& sg, int r, float v,
                                                          float v2, unsigned long long am_best) {
  // (tensor parallel: these stages keep their outputs on their rank)
  switch (sg.epi) {
    case EPI_STORE:
      st_put_local(reinterpret_cast<bf16*>(sg.y) + r, f2bf(v));
      break;
    case EPI_SILU_PAIR:
      if (sg.y2) reinterpret_cast<bf16*>(sg.y2)[r] = f2bf(v);
      st_put_local(reinterpret_cast<bf16*>(sg.y) + r, f2bf(silu_f(v) * v2));
      break;
    case EPI_ARGMAX: {
      const bf16 l = f2bf(v);
      if (sg.y) st_put(P, reinterpret_cast<bf16*>(sg.y) + r, l);  // logits (optional) on every rank
      const unsigned long long k = argmax_key(l, (uint32_t)(sg.row_offset + r));
      am_best = k > am_best ? k : am_best;
    } break;
    case EPI_CONV: {
      const bf16 xb = f2bf(v);
      if (sg.y2) reinterpret_cast<bf16*>(sg.y2)[r] = xb;
      const int cw = sg.cw;
      const bf16* wr = reinterpret_cast<const bf16*>(sg.aux0) + (size_t)r * cw;
      bf16* st = reinterpret_cast<bf16*>(sg.aux2) + (size_t)r * cw;
      bf16 win[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) win[t] = t < cw - 1 ? st[t + 1] : xb;
      float acc = 0.f;
#pragma unroll
      for (int t = 0; t < 8; ++t)
        if (t < cw) acc = fmaf(bf2f(wr[t]), bf2f(win[t]), acc);
#pragma unroll
      for (int t = 0; t < 8; ++t)
        if (t < cw) st[t] = win[t];
      st_put_local(reinterpret_cast<bf16*>(sg.y) + r, f2bf(silu_f(bfround(acc))));
    } break;
    case EPI_GATE_G: {
      const float a = bfround(v) + reinterpret_cast<const float*>(sg.aux1)[r];
      const float sp = a > 20.0f ? a : log1pf(expf(a));
      st_put_local(reinterpret_cast<float*>(sg.y) + r, -expf(reinterpret_cast<const float*>(sg.aux0)[r]) * sp);
    } break;
    case EPI_GATE_BETA:
      st_put_local(reinterpret_cast<bf16*>(sg.y) + r, f2bf(1.0f / (1.0f + expf(-bfround(v)))));
      break;
    case EPI_SILU: {  // the gated RMSNorm's bf16(silu(z)) of the BF16 z row
      const float z = bfround(v);
      st_put_local(reinterpret_cast<bf16*>(sg.y) + r, f2bf(z / (1.0f + expf(-z))));
    } break;
    default:
      break;
  }
  return am_best;
}

// CTA-wide max of the running argmax keys, the cross-CTA maximum and its
// finalisation by the last CTA (token, packed key, position increment).
__device__ __forceinline__ void st_argmax_finish(const StProgram& P, const StStage& S, unsigned long long best,
                                                 unsigned long long* misc) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = shfl_xor_u64(best, o);
    best = other > best ? other : best;
  }
  if (lane == 0) misc[warp] = best;
  named_bar(1, ST_NT);
  if (tid == 0) {
    best = 0;
    for (int i = 0; i < ST_CW; ++i) best = misc[i] > best ? misc[i] : best;
    // every CTA of every rank folds its key into every rank's workspace and
    // counts itself there; CTA 0 of each rank then waits for all of them
    // (bounded) and finalises its own rank (token, key, position) and clears
    // the workspace
    const unsigned total = (unsigned)P.world * gridDim.x;
    const bool sys = P.world > 1;
    for (int r = 0; r < P.world; ++r)
      if (best) sys ? (void)atomicMax_system(st_peer(P, S.am_ws, r), best) : (void)atomicMax(S.am_ws, best);
    sys ? __threadfence_system() : __threadfence();
    for (int r = 0; r < P.world; ++r) {
      unsigned* cnt = reinterpret_cast<unsigned*>(st_peer(P, S.am_ws, r) + 1);
      sys ? (void)atomicAdd_system(cnt, 1u) : (void)atomicAdd(cnt, 1u);
    }
    if (blockIdx.x == 0) {
      unsigned long long* ws = S.am_ws;
      unsigned* cnt = reinterpret_cast<unsigned*>(ws + 1);
      const uint64_t t0 = globaltimer_ns(), lim = qwen_wait_ns();
      bool ok = true;
      while (true) {
        unsigned c;
        if (sys)
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(c) : "l"(cnt) : "memory");
        else
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(c) : "l"(cnt) : "memory");
        if (c >= total) break;
        if (st_aborted(P.abort_flag) || globaltimer_ns() - t0 > lim) {
          st_abort(P.abort_flag);
          ok = false;
          break;
        }
      }
      if (ok) {
        const unsigned long long key = *reinterpret_cast<volatile unsigned long long*>(ws);
        if (S.am_key_out) *S.am_key_out = key;
        if (S.am_token_out) *S.am_token_out = (long long)(0xffffffffu - (uint32_t)(key & 0xffffffffu));
        if (S.pos_inc) *S.pos_inc += 1;
        *ws = 0ull;
        *cnt = 0u;
        __threadfence();
      }
    }
  }
}

struct StCtx {
  uint8_t* ring;
  uint8_t* xh;
  uint8_t* xl;
  float* xinv;
  float* part;
  float* red;
  unsigned long long* misc;
  int* flag;
  uint32_t full0, empty0;
  unsigned* abort_flag;
  unsigned* timeline;  // optional (see StProgram)
  int stage;           // index of the stage being run (timeline)
  const StProgram* prog;  // the kernel's parameter block (peers, world)
  uint32_t tag0;       // tag of stage 0 of this step (tensor parallel): epoch x nstages + 1
};

__device__ __forceinline__ void st_gemv(const StStage& S, const StCtx& X, uint32_t& n) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int u0, u1;
  st_range(S.nunits, u0, u1);
  const int nslice = S.nslice, tiles_my = S.nunits / nslice;  // units are slice-major: u = sl x tiles_my + tile
  if (S.pro == STP_PLAIN) {
    // the K blocks of the slices this CTA's units cover
    const int bps = (S.C / nslice) * (ST_KC / 128);
    const int blo = u1 > u0 ? (u0 / tiles_my) * bps : 0, bhi = u1 > u0 ? ((u1 - 1) / tiles_my + 1) * bps : 0;
    if (S.gated_pro)
      st_prologue<ST_GATED_MAXB, 0, true>(S, X.xh, X.xl, X.xinv, X.red, 0u, X.abort_flag, blo, bhi);
    else
      st_prologue<ST_MAXB, 0>(S, X.xh, X.xl, X.xinv, X.red, 0u, X.abort_flag, blo, bhi);
  } else {
    st_prologue<ST_NORM_MAXB, ST_SL_REG>(S, X.xh, X.xl, X.xinv, X.red, X.tag0 + (uint32_t)S.sl_src, X.abort_flag,
                                         0, S.K >> 7);
  }
  if (tid == 0 && X.timeline) st_tl_put(X.timeline, X.stage, ST_TL_PRO, (unsigned)globaltimer_ns());
  const int ipu = S.ipu, pair = S.pair;
  const int upb = ST_BATCH / ipu > 0 ? ST_BATCH / ipu : 1;
  const int per = S.C / nslice;
  unsigned long long am_best = 0;
  bool good = true;
  uint64_t blocked = 0, comp = 0;  // timeline only: warp 0's wait for copies to land, its chunk math
  for (int ub = u0; ub < u1; ub += upb) {
    const int ue = min(u1, ub + upb);
    const int nit = (ue - ub) * ipu;
    const uint32_t m0 = n + (uint32_t)(ub - u0) * ipu;
    const int pair_id = warp >> 1, rg = warp & 1;
    for (int q = pair_id; q < nit && good; q += ST_PAIRS) {
      const uint32_t m = m0 + q, slot = m % ST_SLOTS;
      if (!(X.timeline ? mbar_test_wait(X.full0 + 8 * slot, (m / ST_SLOTS) & 1u)
                       : mbar_try_wait(X.full0 + 8 * slot, (m / ST_SLOTS) & 1u))) {
        const uint64_t t0 = X.timeline ? globaltimer_ns() : 0;
        if (!st_mbar_wait(X.full0 + 8 * slot, (m / ST_SLOTS) & 1u, X.abort_flag)) {
          good = false;
          break;
        }
        if (X.timeline) blocked += globaltimer_ns() - t0;
      }
      const int u = ub + q / ipu, i = q % ipu;
      const int sl = u / tiles_my;
      const int c = sl * per + (pair ? (i >> 1) : i);
      float a0, a1;
      const long long tc = X.timeline ? clock64() : 0;
      if (S.wbf16)
        st_chunk_bf16(X.ring + slot * ST_CHUNK, reinterpret_cast<const bf16*>(X.xh), c, rg, lane, a0, a1);
      else
        st_chunk(X.ring + slot * ST_CHUNK, X.xh, X.xl, X.xinv, c, rg, lane, a0, a1);
      if (X.timeline) comp += (uint64_t)(clock64() - tc);
      __syncwarp();
      if (lane == 0) mbar_arrive(X.empty0 + 8 * slot);  // one of the pair's two arrivals
      if ((lane & 3) == 0) {
        float* pq = X.part + q * ST_ROWS + 16 * rg + (lane >> 2);
        pq[0] = a0;
        pq[8] = a1;
      }
    }
    named_bar(1, ST_NT);
    if (tid == 0 && X.timeline) st_tl_put(X.timeline, X.stage, ST_TL_CHUNKS, (unsigned)globaltimer_ns());
    for (int idx = tid; idx < (ue - ub) * ST_ROWS && good; idx += ST_NT) {
      const int ul = idx / ST_ROWS, r = idx % ST_ROWS;
      const int u = ub + ul;
      const float* pp = X.part + ul * ipu * ST_ROWS + r;
      float v = 0.f, v2 = 0.f;
      if (pair) {
        for (int i = 0; i < ipu; i += 2) {
          v += pp[i * ST_ROWS];
          v2 += pp[(i + 1) * ST_ROWS];
        }
      } else {
        for (int i = 0; i < ipu; ++i) v += pp[i * ST_ROWS];
      }
      const int sl = u / tiles_my, tl = u - sl * tiles_my, t = S.shard0 + tl;
      const int sg = st_find_seg(S, t);
      const GemvSeg& G = S.seg[sg];
      const int row = (t - S.seg_tile0[sg]) * ST_ROWS + r;
      if (row >= G.n) continue;
      if (S.sl_out) {
        if (S.xrank)  // rank r's slices are slots [r nslice, (r + 1) nslice) on every rank
          st_put_tagged(*X.prog,
                        reinterpret_cast<unsigned long long*>(S.sl_out) +
                            (size_t)(X.prog->rank * nslice + sl) * S.sl_rows + row,
                        v, X.tag0 + (uint32_t)X.stage);
        else
          S.sl_out[(size_t)sl * S.sl_rows + row] = v;
      } else {
        am_best = st_epilogue(*X.prog, G, row, v, v2, am_best);
      }
    }
    named_bar(1, ST_NT);
  }
  n += (uint32_t)(u1 - u0) * ipu;
  if (tid == 0) {
    st_tl_put(X.timeline, X.stage, ST_TL_CBLOCK, (unsigned)blocked);
    st_tl_put(X.timeline, X.stage, ST_TL_WCOMP, (unsigned)comp);
  }
  if (S.am_ws) st_argmax_finish(*X.prog, S, am_best, X.misc);
}

// GatedDeltaNet step of one (value head, block of 32 value columns) unit on
// the consumer warps: thread (d = tid % 32, kg = tid / 32) keeps key rows
// [16 kg, 16 kg + 16) of value column 32 c + d in registers, read once from
// the ring (the unit's state slot), and writes the updated column to global
// memory once.  The arithmetic is the reference's delta_rule_decode_kernel
// (fused_kernels.cu:623-684): L2-normalised q (times D^-1/2) and k, decay
// exp(g), delta = (v - decay S^T k) beta, S' = decay S + k delta^T,
// o = S'^T q.  The unit writes the core output bf16(o) of its 32 columns; the
// default path's gated RMSNorm (main.py:1152-1159) needs the whole head and
// is applied by the next GEMV's prologue (StStage::gated_pro).
__device__ __forceinline__ void st_gdn(const StStage& S, const StCtx& X, uint32_t& n) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int D = ST_GDN_D, DC = ST_GDN_DC, KG = ST_GDN_KG, KR = ST_GDN_KR;
  const GdnArgs& a = S.gdn;
  int u0, u1;
  st_range(S.gdn_heads * ST_GDN_VS, u0, u1);
  float* qs = X.part;
  float* ks = X.part + D;
  float* red2 = X.part + 2 * D;  // [KG][DC]
  for (int u = u0; u < u1; ++u) {
    const int h = S.shard0 + u / ST_GDN_VS, c = u % ST_GDN_VS;  // this rank's heads
    const uint32_t slot = n % ST_SLOTS, par = (n / ST_SLOTS) & 1u;
    if (tid == 0) *X.flag = st_mbar_wait(X.full0 + 8 * slot, par, X.abort_flag) ? 1 : 0;
    named_bar(1, ST_NT);
    if (*X.flag) {
      // every thread observes the completed phase itself (acquire of the
      // bulk-copied state); it has completed, so the wait returns at once
      for (int it = 0; it < (1 << 16) && !mbar_try_wait(X.full0 + 8 * slot, par); ++it) {
      }
      const int d = tid % DC, kg = tid / DC, t = tid & (D - 1);
      const int kh = h / a.rep, col = c * DC + d;
      // every global load of the unit at once (one L2 round trip): q on
      // warps 0-3, k on warps 4-7
      const float qk = bf2f(__ldcg((tid < D ? a.q : a.k) + (size_t)kh * D + t));
      const float gval = __ldcg(a.g + h);
      const float bval = bf2f(__ldcg(a.beta + h));
      const float vval = bf2f(__ldcg(a.v + (size_t)h * D + col));
      const float sq = warp_sum(qk * qk);
      if (lane == 0) X.red[warp] = sq;
      float s[KR];
      const float* st = reinterpret_cast<const float*>(X.ring + slot * ST_CHUNK);
#pragma unroll
      for (int i = 0; i < KR; ++i) s[i] = st[(kg * KR + i) * DC + d];
      named_bar(1, ST_NT);
      if (tid == 0 && X.timeline) st_tl_put(X.timeline, X.stage, ST_TL_PRO, (unsigned)globaltimer_ns());
      const float tq = X.red[0] + X.red[1] + X.red[2] + X.red[3];
      const float tk = X.red[4] + X.red[5] + X.red[6] + X.red[7];
      if (tid < D)
        qs[t] = qk * (rsqrtf(tq + 1e-6f) * rsqrtf((float)D));
      else
        ks[t] = qk * rsqrtf(tk + 1e-6f);
      named_bar(1, ST_NT);
      const float decay = expf(gval);
      float pred = 0.f;
#pragma unroll
      for (int i = 0; i < KR; ++i) pred += s[i] * decay * ks[kg * KR + i];
      red2[kg * DC + d] = pred;
      named_bar(1, ST_NT);
      float ptot = 0.f;
#pragma unroll
      for (int g = 0; g < KG; ++g) ptot += red2[g * DC + d];
      const float delta = (vval - ptot) * bval;
      named_bar(1, ST_NT);  // red2 is read before it is reused
      float o = 0.f;
      float* Sg = a.state + ((size_t)h * ST_GDN_VS + c) * (D * DC);
#pragma unroll
      for (int i = 0; i < KR; ++i) {
        const int k = kg * KR + i;
        const float v = s[i] * decay + ks[k] * delta;
        Sg[k * DC + d] = v;
        o += v * qs[k];
      }
      red2[kg * DC + d] = o;
      named_bar(1, ST_NT);
      if (tid == 0 && X.timeline) st_tl_put(X.timeline, X.stage, ST_TL_CHUNKS, (unsigned)globaltimer_ns());
      if (tid < DC) {
        float core = 0.f;
#pragma unroll
        for (int g = 0; g < KG; ++g) core += red2[g * DC + tid];
        st_put_local(a.out + (size_t)h * D + c * DC + tid, f2bf(core));
      }
    }
    named_bar(1, ST_NT);
    if (tid == 0) {  // a slot's empty barrier takes two arrivals
      mbar_arrive(X.empty0 + 8 * slot);
      mbar_arrive(X.empty0 + 8 * slot);
    }
    ++n;
  }
}

// Attention units on the consumer warps, each over ST_ATTN_SLOTS contiguous
// ring slots of scratch (the producer hands them over in sequence, aligned so
// they never wrap the ring; the KV rows are read directly).  The step
// kernel carries the Qwen3.5 layout only (head dim 256, four query heads per
// KV head): two positions per warp in flight and the queries read from
// shared memory keep the unit inside this kernel's register budget (9 warps:
// 168 registers a thread); other layouts use the per-launch attention kernel.
__device__ __forceinline__ void st_attn(const StStage& S, const StCtx& X, uint32_t& n) {
  const int tid = threadIdx.x;
  int u0, u1;
  st_range(S.attn_kv * S.attn.nsplit, u0, u1);
  for (int u = u0; u < u1; ++u) {
    const int cnt = st_attn_pad(n) + ST_ATTN_SLOTS;
    bool ok = true;
    if (tid == 0)
      for (int i = 0; i < cnt && ok; ++i) {
        const uint32_t m = n + i;
        ok = st_mbar_wait(X.full0 + 8 * (m % ST_SLOTS), (m / ST_SLOTS) & 1u, X.abort_flag);
      }
    if (named_bar_and(1, ST_NT, ok)) {
      float* scratch = reinterpret_cast<float*>(X.ring + ((n + cnt - ST_ATTN_SLOTS) % ST_SLOTS) * ST_CHUNK);
      const int ku = u / S.attn.nsplit, split = u - ku * S.attn.nsplit, kh = S.shard0 + ku;
      unsigned* tl = X.timeline ? X.timeline + ((size_t)X.stage * gridDim.x + blockIdx.x) * ST_TL + ST_TL_PRO : nullptr;
      attn_unit<256, 4, 2, false>(S.attn, kh, split, scratch, X.flag + 1, tl, X.flag[2]);
    }
    named_bar(1, ST_NT);
    if (tid == 0)
      for (int i = 0; i < cnt; ++i) {  // a slot's empty barrier takes two arrivals
        mbar_arrive(X.empty0 + 8 * ((n + i) % ST_SLOTS));
        mbar_arrive(X.empty0 + 8 * ((n + i) % ST_SLOTS));
      }
    n += cnt;
  }
}

// Copies one stage descriptor into shared memory in 16-byte cp.async pieces
// spread over the consumer threads (each thread waits for its own pieces with
// cp.async.wait_group 0; a barrier then publishes them).
__device__ __forceinline__ void st_desc_fetch(uint32_t dst, const StStage* src, int tid) {
  constexpr int n16 = (int)(sizeof(StStage) / 16);
  for (int i = tid; i < n16; i += ST_NT)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst + 16u * i),
                 "l"(reinterpret_cast<const uint4*>(src) + i) : "memory");
  cp_async_commit();
}

__global__ void __launch_bounds__(ST_THREADS, 1) step_kernel(const __grid_constant__ StProgram P) {
  extern __shared__ __align__(128) uint8_t st_smem[];
  const uint32_t sbase = smem_u32(st_smem);
  StCtx X;
  X.ring = st_smem + StSmem::ring;
  X.xh = st_smem + StSmem::xh;
  X.xl = st_smem + StSmem::xl;
  X.xinv = reinterpret_cast<float*>(st_smem + StSmem::xinv);
  X.part = reinterpret_cast<float*>(st_smem + StSmem::part);
  X.red = reinterpret_cast<float*>(st_smem + StSmem::red);
  X.misc = reinterpret_cast<unsigned long long*>(st_smem + StSmem::misc);
  X.flag = reinterpret_cast<int*>(X.misc + 16);
  X.full0 = sbase + StSmem::bars;
  X.empty0 = X.full0 + 8 * ST_SLOTS;
  X.abort_flag = P.abort_flag;
  X.timeline = P.timeline;
  X.stage = 0;
  if (threadIdx.x == 0) {
    // the decode position is constant within a step (the LM head stage
    // increments it last), so attention stages read it once per launch
    X.flag[2] = P.pos ? __ldcg(P.pos) : -1;
    for (int i = 0; i < ST_SLOTS; ++i) {
      mbar_init(X.full0 + 8 * i, 1);
      mbar_init(X.empty0 + 8 * i, 2);  // released by both warps of a pair
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x >= ST_NT) {
    if (threadIdx.x == ST_NT) st_producer(P, sbase + StSmem::ring, X.full0, X.empty0);
    return;
  }
  const int tid = threadIdx.x;
  uint32_t n = 0;
  bool alive = true;
  X.prog = &P;
  // this launch's epoch: the steps this rank has completed (counters[2 nstages],
  // advanced once per CTA at the end of each step); stage s of this step is
  // complete when counters[nstages + s] reaches (epoch + 1) x grid.  The tag of
  // stage s's K-slice words (tensor parallel) is epoch x nstages + 1 + s.
  unsigned long long local_target = 0;
  int prev_xrank = 0;  // thread 0: the previous stage's slices are tagged words
  if (tid == 0) {
    const unsigned long long epoch = st_ld_acq_u64(P.counters + 2 * P.nstages, false) / gridDim.x;
    local_target = (epoch + 1) * gridDim.x;
    X.flag[3] = (int)(uint32_t)(epoch * (unsigned long long)P.nstages + 1ull);
  }
  // Stage descriptors are read from shared memory: the next stage's one is
  // copied in while the current stage runs, so a stage's first loads do not
  // wait for its descriptor to come from L2.
  const StStage* desc = reinterpret_cast<const StStage*>(st_smem + StSmem::desc);
  st_desc_fetch(sbase + StSmem::desc, P.stages, tid);
  for (int s = 0; s < P.nstages; ++s) {
    if (tid == 0) st_stamp(P, s, ST_TL_WAIT);
    cp_async_wait<0>();  // this thread's pieces of stage s's descriptor
    if (s > 0) {
      bool ok = true;
      // after a row-parallel stage nothing is counted: the prologue polls the
      // tagged slices of every rank (which also orders this stage after the
      // previous one: a CTA that wrote slices had passed the wait before it)
      if (tid == 0 && !prev_xrank)
        ok = st_wait_count(P.counters + P.nstages + s - 1, local_target, P.abort_flag, false);
      if (tid == 0 && prev_xrank) ok = !st_aborted(P.abort_flag);
      alive = named_bar_and(1, ST_NT, ok);
      if (!alive) break;
    } else {
      named_bar(1, ST_NT);
      X.tag0 = (uint32_t)X.flag[3];
    }
    const StStage& S = desc[s & 1];
    // the other buffer held stage s - 1, which every consumer has finished
    if (s + 1 < P.nstages)
      st_desc_fetch(sbase + StSmem::desc + ((s + 1) & 1) * (uint32_t)sizeof(StStage), P.stages + s + 1, tid);
    if (tid == 0) st_stamp(P, s, ST_TL_START);
    X.stage = s;
    const int kind = S.kind;
    if (kind == ST_GEMV) {
      st_gemv(S, X, n);
    } else if (kind == ST_GDN) {
      st_gdn(S, X, n);
    } else {
      st_attn(S, X, n);
    }
    named_bar(1, ST_NT);
    if (tid == 0) {
      st_stamp(P, s, ST_TL_END);
      if (s != P.drop_stage || blockIdx.x != 0)  // the release publishes what the CTA wrote (barrier-ordered)
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" :: "l"(P.counters + P.nstages + s) : "memory");
      prev_xrank = S.xrank;
    }
  }
  // End of the step: the rank's completed-step count advances once per CTA
  // (counters keep counting: nothing is cleared).  An abandoned step leaves
  // it behind; the host clears every counter (qwen_step_reset).
  if (tid == 0 && alive && !st_aborted(P.abort_flag)) atomicAdd(P.counters + 2 * P.nstages, 1ull);
}

// ---------------------------------------------------------------------------
// Weight packing: [N, K] E4M3 row-major + block scales -> chunks of 32 rows x
// 512 K.  Chunk (t, c) holds, for row group rg = 0, 1, group j = 0..7 (64 K
// each) and half h = 0, 1, the 512 bytes lane*16 + i = W[32t + 16rg + 8h +
// lane/4][512c + 64j + 16(lane%4) + i], then the FP32 scales of its four
// 128-K blocks (row block 32t / 128).  Rows past N are zero.  One thread per
// 16 bytes.
// ---------------------------------------------------------------------------
template <typename ST>
__global__ void step_pack_kernel(const uint8_t* __restrict__ w, const void* __restrict__ s, int N, int K, int kblk,
                                 uint8_t* __restrict__ out) {
  const int C = K / ST_KC;
  const long long tiles = (N + ST_ROWS - 1) / ST_ROWS;
  const long long total = tiles * C * (ST_WBYTES / 16 + 1);
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long chunk = idx / (ST_WBYTES / 16 + 1);
    const int p = (int)(idx - chunk * (ST_WBYTES / 16 + 1));
    const int t = (int)(chunk / C), c = (int)(chunk - (long long)t * C);
    uint8_t* dst = out + chunk * ST_CHUNK;
    if (p < ST_WBYTES / 16) {
      const int rg = p >> 9, j = (p >> 6) & 7, h = (p >> 5) & 1, lane = p & 31;
      const int row = t * ST_ROWS + 16 * rg + 8 * h + (lane >> 2);
      const int k = c * ST_KC + 64 * j + 16 * (lane & 3);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < N) v = *reinterpret_cast<const uint4*>(w + (size_t)row * K + k);
      *reinterpret_cast<uint4*>(dst + p * 16) = v;
    } else {
      const int rb = (t * ST_ROWS) >> 7;
      float f[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) f[i] = load_scale<ST>(s, rb * kblk + c * 4 + i);
      *reinterpret_cast<float4*>(dst + ST_WBYTES) = make_float4(f[0], f[1], f[2], f[3]);
    }
  }
}

// BF16 weights [N, K] -> chunks of 32 rows x 256 K: chunk (t, c) holds, for
// row group rg = 0, 1, K step j = 0..15 and lane, the 16 bytes of the lane's
// m16n8k16 A fragment: W[r][k .. k+1], W[r+8][k .. k+1], W[r][k+8 .. k+9],
// W[r+8][k+8 .. k+9] with r = 32t + 16rg + lane/4, k = 256c + 16j + 2(lane%4),
// then 16 zero bytes.  Rows past N are zero.  One thread per 4 bytes.
__global__ void step_pack_bf16_kernel(const bf16* __restrict__ w, int N, int K, uint8_t* __restrict__ out) {
  const int C = K / 256;
  const long long tiles = (N + ST_ROWS - 1) / ST_ROWS;
  constexpr int WORDS = ST_CHUNK / 4;
  const long long total = tiles * C * WORDS;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long chunk = idx / WORDS;
    const int p = (int)(idx - chunk * WORDS);
    const int t = (int)(chunk / C), c = (int)(chunk - (long long)t * C);
    uint32_t v = 0u;
    if (p < ST_WBYTES / 4) {
      const int rg = p >> 11, j = (p >> 7) & 15, lane = (p >> 2) & 31, reg = p & 3;
      const int row = t * ST_ROWS + 16 * rg + (lane >> 2) + ((reg & 1) ? 8 : 0);
      const int k = c * 256 + 16 * j + 2 * (lane & 3) + ((reg & 2) ? 8 : 0);
      if (row < N) v = *reinterpret_cast<const uint32_t*>(w + (size_t)row * K + k);
    }
    reinterpret_cast<uint32_t*>(out + chunk * ST_CHUNK)[p] = v;
  }
}

}  // namespace qwen
