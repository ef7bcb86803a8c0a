// Shared device helpers for the sm_100a decode-path kernels.
//
// Everything here is inline PTX or plain CUDA; nothing is taken from a
// vendor library.  The kernels that wait on an mbarrier bound every wait by
// wall time (globaltimer) and report a timeout through a device error word
// instead of hanging: see qwen_err_set() / qwen_get_device_error().
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#ifndef QWEN_WAIT_TIMEOUT_NS
#define QWEN_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: far above any legitimate wait
#endif

namespace qwen {

typedef __nv_bfloat16 bf16;

// Error codes recorded in the device error word (first error wins).
enum : unsigned {
  ERR_NONE = 0,
  ERR_TIMEOUT_FULL = 1,     // consumer gave up waiting for a bulk copy
  ERR_TIMEOUT_EMPTY = 2,    // producer gave up waiting for a free stage
  ERR_TIMEOUT_DRAIN = 3,    // producer gave up waiting for its own copies
  ERR_POS_RANGE = 5,        // a device-side cache position outside [0, max_seq)
  ERR_SLICES_COUNT = 7,     // a K-slice count outside [1, sl_max] (PRO_SLICES_RMSNORM)
};

// One error word per shared library (each library is a single translation
// unit).  Kernels set it with atomicCAS; the host reads and clears it.
__device__ unsigned int g_qwen_err;

__device__ __forceinline__ void qwen_err_set(unsigned code) {
  atomicCAS(&g_qwen_err, 0u, code);
}

// Limit of the waits on other CTAs or ranks (step-kernel stage counters, p2p
// flags), in ns; the host may lower it (qwen_set_wait_timeout_ns), e.g. for a
// test that lets such a wait run out.  Waits on a CTA's own bulk copies keep
// the fixed QWEN_WAIT_TIMEOUT_NS.
__device__ unsigned long long g_qwen_wait_ns = QWEN_WAIT_TIMEOUT_NS;

__device__ __forceinline__ unsigned long long qwen_wait_ns() {
  return *reinterpret_cast<volatile unsigned long long*>(&g_qwen_wait_ns);
}

// 16-byte global load through the read-only path without L1 allocation
// (streamed weights: each byte is read once).
__device__ __forceinline__ uint4 ld_nc_na_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// Conversions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16(v); }
__device__ __forceinline__ float bfround(float v) { return __bfloat162float(__float2bfloat16(v)); }

// Two BF16 packed in a 32-bit word -> two floats (exact).
__device__ __forceinline__ float2 bf2x_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

// Two E4M3 bytes (low byte = element 0) -> f16x2 (exact: every E4M3 value is an f16).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two_bytes) {
  uint32_t out;
  unsigned short in16 = (unsigned short)(two_bytes & 0xffffu);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(in16));
  return out;
}

// Two floats -> two E4M3 bytes (round to nearest even, saturating); `lo`
// goes to the low byte.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  unsigned short out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(hi), "f"(lo));
  return (uint32_t)out;
}

__device__ __forceinline__ float2 h2u_to_f2(uint32_t h) {
  __half2 v = *reinterpret_cast<__half2*>(&h);
  return __half22float2(v);
}

// ---------------------------------------------------------------------------
// Warp / block reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Named barrier over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory addressing, mbarriers and bulk async copies
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Non-blocking form (try_wait may suspend the thread for a while first).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait until the phase with `parity` of mbarrier `bar` has completed.
// Returns false after QWEN_WAIT_TIMEOUT_NS of wall time.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > QWEN_WAIT_TIMEOUT_NS) return false;
  }
}

// L2 policy for data read exactly once per step (weights): evict first.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> shared, completion counted on mbarrier `bar` (bytes).
// Both addresses 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      :: "r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy) : "memory");
}

// ---------------------------------------------------------------------------
// Look-ahead L2 prefetch.  A decode-step kernel is handed the weight regions of
// the launch that follows it and pulls its share of them into L2 (bulk
// prefetch, no shared-memory destination, no completion to wait for) while it
// runs, so consecutive kernels keep HBM busy across their boundaries.  The
// regions are static weights, so this is safe before griddepcontrol.wait.
// ---------------------------------------------------------------------------
struct L2Prefetch {
  const void* p[4];
  unsigned long long n[4];  // bytes, multiples of 16; p 16-byte aligned
};

// Called by one warp of every CTA: the CTA prefetches a 1/gridDim.x share of
// each region in pieces of up to 32 KB, one piece per lane at a time.
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf, int lane) {
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const unsigned long long total = pf.n[r];
    if (total == 0 || pf.p[r] == nullptr) continue;
    unsigned long long per = (total + gridDim.x - 1) / gridDim.x;
    per = (per + 15) & ~15ull;
    const unsigned long long beg = (unsigned long long)blockIdx.x * per;
    const unsigned long long end = beg + per < total ? beg + per : total;
    const char* base = static_cast<const char*>(pf.p[r]);
    for (unsigned long long off = beg + (unsigned long long)lane * 32768ull; off < end; off += 32ull * 32768ull) {
      const unsigned long long rem = end - off;
      const uint32_t len = (uint32_t)(rem < 32768ull ? rem : 32768ull);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(base + off), "r"(len) : "memory");
    }
  }
}

// 2^e as a float for |e| <= 126 (exact).
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL)
// ---------------------------------------------------------------------------
// Block until the grids this grid depends on have completed and flushed.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next grid on the stream to start launching.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Loads that bypass L1 allocation (streamed data read once).
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// Same, with an L2 eviction-priority policy (evict_first for data read once).
__device__ __forceinline__ uint4 ld_nc_v4_policy(const void* p, uint64_t policy) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(policy));
  return r;
}
// 16-byte async copy global -> shared (L1 bypass, L2 cache policy).  With
// ok == false nothing is read and the destination is zero-filled.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool ok, uint64_t policy) {
  const uint32_t n = ok ? 16u : 0u;
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;"
               :: "r"(dst), "l"(src), "r"(n), "l"(policy) : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" :: "r"(dst), "l"(src), "l"(policy) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }
__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}

// BF16 orderable key: unsigned order equals value order; -0 maps to +0.
__device__ __forceinline__ uint32_t bf16_orderable(uint32_t bits16) {
  bits16 &= 0xffffu;
  if ((bits16 & 0x7fffu) == 0) bits16 = 0;
  return (bits16 & 0x8000u) ? (~bits16 & 0xffffu) : (bits16 | 0x8000u);
}
__device__ __forceinline__ unsigned long long argmax_key(bf16 v, uint32_t index) {
  uint32_t bits = __bfloat16_as_ushort(v);
  return ((unsigned long long)bf16_orderable(bits) << 32) | (unsigned long long)(0xffffffffu - index);
}

}  // namespace qwen
