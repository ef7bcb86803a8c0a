// All-reduce of tensor-parallel partial sums and of the argmax key over
// NVLink peer memory (no library collective).
//
// Each rank owns one exchange region, mapped into every other rank's address
// space with CUDA IPC:
//   [0, 64)      flags  u32 [2 parity][8 source rank]
//   [64, 192)    keys   u64 [2 parity][8 source rank]
//   [256, 264)   seq, done: this rank's round counter and CTA counter
//   [1024, ...)  bufs   f32 [2 parity][world][n]
// Collectives run in rounds numbered by seq (a device counter advanced by
// the consuming kernel, identical on every rank because every rank runs the
// same sequence of collectives); round s uses parity s & 1 and flag value
// s + 1.  A round:
//   * the producing GEMV (EPI_F32_P2P epilogue) stores its FP32 partial row
//     r into slot [rank] of parity buffer p of every rank (NVLink stores);
//   * the consuming kernel (p2p_resid_kernel, or the next GEMV's x
//     preparation with PRO_P2P_RMSNORM), after griddepcontrol.wait (the
//     producing GEMV has completed and its stores are performed), fences and
//     release-stores flag[p][rank] = s + 1 into every rank's region, then
//     waits with acquire loads for flag[p][src] >= s + 1 of every source in
//     its own region (bounded: after QWEN_WAIT_TIMEOUT_NS it records
//     ERR_P2P_TIMEOUT and goes on), sums the slots in rank order (so every
//     rank computes identical bits) and adds the residual; the last CTA of
//     the consuming grid advances seq.
// A rank can run at most one round ahead of another (it needs the other's
// flag of the current round to finish it), so two parity buffers suffice: a
// buffer is rewritten two rounds later, after every rank has consumed it.
#pragma once

#include "common.cuh"

namespace qwen {

constexpr int P2P_MAX_WORLD = 8;
constexpr int P2P_DATA_OFF = 1024;
enum : unsigned { ERR_P2P_TIMEOUT = 6 };

struct P2PTable {
  float* buf[P2P_MAX_WORLD][2];            // rank p's buffer of parity b: [world][n]
  unsigned* flag[P2P_MAX_WORLD];           // rank p's flags [2][8]
  unsigned long long* key[P2P_MAX_WORLD];  // rank p's key slots [2][8]
  unsigned* seq;                           // this rank's round counter
  unsigned* done;                          // this rank's CTA counter
  int world, rank, n;
};

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Producer side, one output row (called from the GEMV epilogue).
__device__ __forceinline__ void p2p_store_row(const P2PTable* t, int r, float v) {
  const unsigned par = *reinterpret_cast<const volatile unsigned*>(t->seq) & 1u;
  const int w = t->world;
  const size_t off = (size_t)t->rank * t->n + r;
  for (int p = 0; p < w; ++p) t->buf[p][par][off] = v;
  __threadfence_system();
}

// Publish this rank's flag of round s to every rank, then wait for every
// source's flag of round s in this rank's region.  One thread.
__device__ __forceinline__ void p2p_publish(const P2PTable& t, unsigned par, unsigned want) {
  __threadfence_system();
  for (int p = 0; p < t.world; ++p) st_release_sys_u32(t.flag[p] + par * 8 + t.rank, want);
}
__device__ __forceinline__ bool p2p_wait_all(const P2PTable& t, unsigned par, unsigned want) {
  const unsigned* f = t.flag[t.rank] + par * 8;
  for (int src = 0; src < t.world; ++src) {
    if (ld_acquire_sys_u32(f + src) >= want) continue;
    const uint64_t t0 = globaltimer_ns(), lim = qwen_wait_ns();
    while (ld_acquire_sys_u32(f + src) < want)
      if (globaltimer_ns() - t0 > lim) return false;
  }
  return true;
}

// The consumer of a round, one thread per CTA after the CTA has read seq:
// the last CTA of the grid advances seq.
__device__ __forceinline__ void p2p_round_done(const P2PTable& t) {
  __threadfence();
  if (atomicAdd(t.done, 1u) == gridDim.x - 1) {
    *t.done = 0u;
    __threadfence();
    atomicAdd(t.seq, 1u);
  }
}

// y[i] = bf16(res[i] + bf16(sum over ranks of the partials)), i < n.
__global__ void __launch_bounds__(256) p2p_resid_kernel(const P2PTable* __restrict__ tab, const bf16* __restrict__ res,
                                                        bf16* __restrict__ y) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const P2PTable& t = *tab;
  const unsigned s = *reinterpret_cast<const volatile unsigned*>(t.seq);
  const unsigned par = s & 1u, want = s + 1u;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) p2p_publish(t, par, want);
    if (!p2p_wait_all(t, par, want)) qwen_err_set(ERR_P2P_TIMEOUT);
  }
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < t.n) {
    const float* b = t.buf[t.rank][par];
    float sum = 0.f;
    for (int src = 0; src < t.world; ++src) sum += __ldcv(b + (size_t)src * t.n + i);
    y[i] = f2bf(bf2f(res[i]) + bfround(sum));
  }
  __syncthreads();
  if (threadIdx.x == 0) p2p_round_done(t);
}

// Greedy token from the per-rank packed argmax keys (orderable logit << 32 |
// ~global index): every rank stores its key into every rank's slot, then
// takes the maximum in its own region.  One thread.
__global__ void p2p_token_kernel(const P2PTable* __restrict__ tab, const unsigned long long* __restrict__ key,
                                 long long* __restrict__ token) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  if (threadIdx.x != 0) return;
  const P2PTable& t = *tab;
  const unsigned s = *reinterpret_cast<const volatile unsigned*>(t.seq);
  const unsigned par = s & 1u, want = s + 1u;
  const unsigned long long k = *key;
  for (int p = 0; p < t.world; ++p) t.key[p][par * 8 + t.rank] = k;
  p2p_publish(t, par, want);
  if (!p2p_wait_all(t, par, want)) qwen_err_set(ERR_P2P_TIMEOUT);
  unsigned long long best = 0ull;
  const volatile unsigned long long* mine = t.key[t.rank] + par * 8;
  for (int src = 0; src < t.world; ++src) best = mine[src] > best ? mine[src] : best;
  *token = (long long)(0xffffffffu - (uint32_t)(best & 0xffffffffull));
  __threadfence();
  atomicAdd(t.seq, 1u);
}

}  // namespace qwen
