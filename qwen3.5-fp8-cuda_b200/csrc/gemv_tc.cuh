// Block-scaled E4M3 x BF16 GEMV on the 5th-generation tensor cores (tcgen05).
//
// Same contract as the rest of the GEMV family (gemv.cuh): for every output
// row r of one or more weight segments
//     v[r] = sum_kb scale[r / 128, kb] * sum_{k in kb} x[k] * e4m3(W[r, k])
// with FP32 accumulation, followed by the fused epilogue of the segment.
// Restates gemv_v4_kernel and its fused variants (fused_kernels.cu:91-479).
//
// Work is cut into items: 128 weight rows (the M of one tcgen05.mma; 128
// gate + 128 up rows for the paired MLP) times a slice of the 128-wide K
// blocks.  Each CTA walks its items with three roles:
//   * warp 0, one thread: TMA producer.  Streams 16 KB tiles (128 rows x 128
//     bytes, 128-byte swizzle) of each item's K-blocks into a ring of shared
//     memory stages; weights are static, so it fills the ring before
//     griddepcontrol.wait and keeps it full.
//   * warp 1, one thread: MMA issuer.  Four tcgen05.mma kind::f8f6f4
//     (M=128, N=16, K=32) per K-block and matrix, A = the weight tile, B = x,
//     each K-block into its own TMEM slot (16 columns per matrix, 16 slots);
//     tcgen05.commit releases the ring stage and hands the slot over.
//   * warps 4-7 (one TMEM lane = one weight row per thread): read the slot
//     with tcgen05.ld, apply scale[row block, kb] * 2^-e per K-block in FP32,
//     and run the segment epilogue at the end of the item.
// x is prepared once per CTA by warps 2-7 (RMSNorm prologue included) as the
// B operand of the CTA's K slice: per K-block 16 rows x 128 bytes in the
// canonical K-major 128-byte-swizzled layout, row 0 = hi, row 1 = lo of
// x * 2^e = hi + lo / 32 (E4M3, exact for every element within 2^-14 of the
// block maximum), rows 2-15 zero.  Columns 0 and 1 of the MMA result are the
// hi and lo partial sums.
//
// Launches that stream for less than two waves keep to half of an SM's
// shared memory so that the next kernel of the stream (programmatic
// dependent launch) becomes resident beside this one and starts its own
// weight copies while this one finishes.
//
// When there are fewer units than SMs, K is split into C slices; each item
// writes its FP32 partial rows to a per-device scratch area and the last CTA
// of a unit (atomic counter, reset after use) adds the C partials in slice
// order and runs the epilogue, so results do not depend on timing.  The
// scratch is shared by all launches on a device: K-split launches on one
// device must not run concurrently (one stream, as the decode engine uses).
//
// Every mbarrier wait is bounded (QWEN_WAIT_TIMEOUT_NS); on a timeout the
// thread records an error in the device error word, the producer drains its
// copies in flight (again bounded) and the CTA frees its TMEM and exits.
#pragma once

#include "gemv.cuh"

#include <cuda.h>

namespace qwen {

constexpr int TC_ROWS = 128;        // weight rows per item (M of one MMA)
constexpr int TC_TILE = 128 * 128;  // bytes of one K-block of one matrix
constexpr int TC_XBLK = 2048;       // B operand bytes per K-block (16 rows x 128 B)
constexpr int TC_MAX_STAGES = 24;
constexpr int TC_TMEM_COLS = 256;   // accumulator slots of 16 columns per matrix
constexpr int TC_MAX_TSLOTS = TC_TMEM_COLS / 16;
constexpr int TC_THREADS = 256;
constexpr int TC_PART_FLOATS = 1 << 17;  // K-split scratch (512 KB)
constexpr int TC_MAX_CNT = 4096;         // K-split unit counters
constexpr int TC_SMEM_MAX = 227 * 1024;
constexpr int TC_SMEM_SHARED = 113 * 1024;  // half an SM: two CTAs side by side

enum : unsigned { ERR_TC_TIMEOUT = 4 };

// Tensor maps of each segment's weight matrices ([segment][gate, up]).
struct GemvMaps {
  CUtensorMap map[GEMV_MAX_SEG][2];
};

__device__ float g_tc_part[TC_PART_FLOATS];
__device__ unsigned int g_tc_cnt[TC_MAX_CNT];

// Shared memory plan (offsets from a 1024-byte aligned base): the ring of
// weight stages, the B operand of this CTA's K slice (at most ceil(nkb / C)
// blocks), BF16 staging of the slice of x, the RMSNorm weights of the slice,
// 2^-e per slice block, the mbarriers and a small misc area.
struct TcSmem {
  int ring_off, xb_off, stg_off, nw_off, xinv_off, bar_off, misc_off, total, stage_bytes;
};
__host__ __device__ inline TcSmem tc_smem_layout(int K, int P, int C, int stages) {
  TcSmem L;
  const int nkb = K >> 7;
  const int nxb = (nkb + C - 1) / C;
  L.stage_bytes = P * TC_TILE;
  L.ring_off = 0;
  L.xb_off = stages * L.stage_bytes;
  L.stg_off = L.xb_off + nxb * TC_XBLK;
  L.nw_off = L.stg_off + nxb * 256;
  L.xinv_off = L.nw_off + nxb * 512;
  L.bar_off = L.xinv_off + align_up(4 * nxb, 16);
  L.misc_off = L.bar_off + 1024;
  L.total = 1024 /* alignment slack */ + L.misc_off + 256;
  return L;
}
// Largest ring (<= TC_MAX_STAGES stages) that fits `budget` bytes, or 0 when
// fewer than two fit.
__host__ __device__ inline int tc_stages_for(int K, int P, int C, int budget) {
  const int fixed = tc_smem_layout(K, P, C, 0).total;
  const int s = (budget - fixed) / (P * TC_TILE);
  return s < 2 ? 0 : (s > TC_MAX_STAGES ? TC_MAX_STAGES : s);
}

// Item i -> unit i / C, K slice i % C.
struct TcItem {
  int seg, row0, kb0, kb1, unit;
};
__device__ __forceinline__ TcItem tc_item(const GemvArgs& a, int i, int nkb) {
  TcItem t;
  const int C = a.nslice;
  t.unit = i / C;
  const int sl = i - t.unit * C;
  t.seg = gemv_find_seg(a, t.unit);
  t.row0 = (t.unit - a.seg[t.seg].unit0) * TC_ROWS;
  t.kb0 = (sl * nkb) / C;
  t.kb1 = ((sl + 1) * nkb) / C;
  return t;
}

// ---------------------------------------------------------------------------
// tcgen05 / TMA primitives (inline PTX)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2-D tiled TMA load global -> shared, completion on mbarrier `bar` (no multicast).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;"
      :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), sm_100 descriptor version 1.  The start address is
// in 16-byte units in the low 14 bits, so +2 advances one 32-byte K step.
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: D = F32, A = B = E4M3, both K-major, N = 16, M = 128.
constexpr uint32_t TC_IDESC = (1u << 4) | ((16u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n"
      :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(accumulate), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_ld2(uint32_t taddr, uint32_t& v0, uint32_t& v1) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(v0), "=r"(v1) : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Rows 2.. of every slice block of the x operand (XBLK bytes per K-block)
// are zero; rows 0 and 1 are written by tc_x_prepare.  Static: runs before
// griddepcontrol.wait.
template <int XBLK = TC_XBLK>
__device__ __forceinline__ void tc_x_zero(int nxb, uint8_t* xbg) {
  for (int o = (threadIdx.x - 64) * 16; o < nxb * XBLK; o += 192 * 16)
    if ((o & (XBLK - 1)) >= 256) *reinterpret_cast<uint4*>(xbg + o) = make_uint4(0, 0, 0, 0);
}

// x -> B operand of K-blocks [kb0, kb0 + nxb) (warps 2..7, 192 threads;
// named barrier 1).  Pass 1 reads x once (h = x + x2 for ADD_RMSNORM), sums
// squares over the whole of K (only the slice's blocks are read when no
// whole-vector norm follows) and stages the slice's blocks in shared
// memory; pass 2 normalises, splits into E4M3 hi / lo and writes the
// swizzled B operand.  CTA 0 also writes h2_out and, over every block, xn_out
// (re-reading the blocks outside its slice).  XBLK: bytes per K-block of the
// operand (rows 0 and 1 of a 128-byte-swizzled row group).
// ---------------------------------------------------------------------------
template <int XBLK = TC_XBLK>
__device__ __forceinline__ void tc_x_prepare(const GemvArgs& a, int kb0, int nxb, uint8_t* xbg, uint8_t* stg,
                                             const float* nws, float* xinv, float* red) {
  const int K = a.K, nkb = K >> 7;
  const int t = threadIdx.x - 64, lane = threadIdx.x & 31, w = (threadIdx.x >> 5) - 2;
  constexpr int NT = 192, NW = 6, MAXC = 8;
  const bf16* xin = a.x;
  if (a.x_row) xin += (size_t)(*a.x_row) * K;
  const bool all = blockIdx.x == 0 && a.xn_out != nullptr && a.pro != PRO_NONE;
  const int sb0 = all ? 0 : kb0, sb1 = all ? nkb : kb0 + nxb;  // blocks of pass 2
  // Tensor-parallel input: publish this rank's partial of the round (CTA 0),
  // wait for every rank's (bounded), then read the slots below.
  const float* pbuf = nullptr;
  int pworld = 0, pn = 0;
  if (a.pro == PRO_P2P_RMSNORM) {
    const P2PTable& pt = *a.p2p;
    const unsigned s = *reinterpret_cast<const volatile unsigned*>(pt.seq);
    if (t == 0) {
      if (blockIdx.x == 0) p2p_publish(pt, s & 1u, s + 1u);
      if (!p2p_wait_all(pt, s & 1u, s + 1u)) qwen_err_set(ERR_P2P_TIMEOUT);
    }
    pbuf = pt.buf[pt.rank][s & 1u];
    pworld = pt.world;
    pn = pt.n;
    named_bar(1, NT);
  }
  // Single-GPU input: the previous launch's K-slice partial rows (EPI_SLICES,
  // complete once griddepcontrol.wait has returned).  A count outside
  // [1, sl_max] is recorded as an error and read as no slices.
  if (a.pro == PRO_SLICES_RMSNORM) {
    pbuf = a.sl_buf;
    pworld = *reinterpret_cast<const volatile int*>(a.sl_count);
    pn = a.sl_n;
    if (pworld < 1 || pworld > a.sl_max) {
      if (t == 0 && blockIdx.x == 0) qwen_err_set(ERR_SLICES_COUNT);
      pworld = 0;
    }
  }
  const bool psum = a.pro == PRO_P2P_RMSNORM || a.pro == PRO_SLICES_RMSNORM;
  // pass 1: up to MAXC chunks of 8 elements per thread are loaded before any
  // is used, so the loads overlap
  float ss = 0.f;
  const int nch = K >> 3;
  // Tensor-parallel or sliced input: h = bf16(res + bf16(sum of the ranks' (or
  // slices') partials in order)), two chunks per thread in flight, the loads
  // of one rank (slice) for both chunks issued before they are added.
  for (int base = t; psum && base < nch; base += NT * 2) {
    uint4 v[2];
    float sum[2][8];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = base + j * NT;
      if (i < nch) v[j] = __ldg(reinterpret_cast<const uint4*>(xin) + i);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum[j][e] = 0.f;
    }
    for (int src = 0; src < pworld; ++src) {
      float4 pv[2][2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int i = base + j * NT;
        const float4* pp = reinterpret_cast<const float4*>(pbuf + (size_t)src * pn + (size_t)(i < nch ? i : 0) * 8);
        pv[j][0] = __ldcv(pp);
        pv[j][1] = __ldcv(pp + 1);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sum[j][0] += pv[j][0].x; sum[j][1] += pv[j][0].y; sum[j][2] += pv[j][0].z; sum[j][3] += pv[j][0].w;
        sum[j][4] += pv[j][1].x; sum[j][5] += pv[j][1].y; sum[j][6] += pv[j][1].z; sum[j][7] += pv[j][1].w;
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = base + j * NT;
      if (i >= nch) continue;
      uint32_t* vw = reinterpret_cast<uint32_t*>(&v[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = bf2x_to_f2(vw[q]);
        const __nv_bfloat162 h = __floats2bfloat162_rn(f.x + bfround(sum[j][2 * q]), f.y + bfround(sum[j][2 * q + 1]));
        vw[q] = *reinterpret_cast<const uint32_t*>(&h);
        const float2 g = bf2x_to_f2(vw[q]);
        ss = fmaf(g.x, g.x, ss);
        ss = fmaf(g.y, g.y, ss);
      }
      if (blockIdx.x == 0 && a.h2_out) reinterpret_cast<uint4*>(a.h2_out)[i] = v[j];
      const int b = i >> 4;
      if (b >= kb0 && b < kb0 + nxb) reinterpret_cast<uint4*>(stg)[i - kb0 * 16] = v[j];
    }
  }
  // Without a whole-vector norm (PRO_NONE, PRO_GATED_NORM) only the slice's
  // own blocks are read.
  const bool local = a.pro == PRO_NONE || a.pro == PRO_GATED_NORM;
  const int c0 = local ? kb0 * 16 : 0, c1 = local ? (kb0 + nxb) * 16 : nch;
  for (int base = c0 + t; !psum && base < c1; base += NT * MAXC) {
    uint4 v[MAXC], r[MAXC];
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
      const int i = base + j * NT;
      if (i < c1) {
        v[j] = __ldg(reinterpret_cast<const uint4*>(xin) + i);
        if (a.pro == PRO_ADD_RMSNORM) r[j] = __ldg(reinterpret_cast<const uint4*>(a.x2) + i);
        // gated norm: z of the slice's blocks in the same round trip as x
        if (a.pro == PRO_GATED_NORM && (i >> 4) >= kb0 && (i >> 4) < kb0 + nxb)
          r[j] = __ldg(reinterpret_cast<const uint4*>(a.gz) + i);
      }
    }
#pragma unroll
    for (int j = 0; j < MAXC; ++j) {
      const int i = base + j * NT;
      if (i >= c1) continue;
      uint32_t* vw = reinterpret_cast<uint32_t*>(&v[j]);
      if (a.pro == PRO_ADD_RMSNORM) {
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(&r[j]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = bf2x_to_f2(vw[q]), g = bf2x_to_f2(rw[q]);
          const __nv_bfloat162 h = __floats2bfloat162_rn(f.x + g.x, f.y + g.y);
          vw[q] = *reinterpret_cast<const uint32_t*>(&h);
        }
        if (blockIdx.x == 0 && a.h2_out) reinterpret_cast<uint4*>(a.h2_out)[i] = v[j];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = bf2x_to_f2(vw[q]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
      const int b = i >> 4;  // 16 chunks of 8 elements per 128-block
      if (b >= kb0 && b < kb0 + nxb) {
        reinterpret_cast<uint4*>(stg)[i - kb0 * 16] = v[j];
        // gated norm: z staged where the RMSNorm weights would be
        if (a.pro == PRO_GATED_NORM) reinterpret_cast<uint4*>(const_cast<float*>(nws))[i - kb0 * 16] = r[j];
      }
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[w] = ss;
  named_bar(1, NT);
  float rms = 1.f;
  if (a.pro != PRO_NONE && a.pro != PRO_GATED_NORM) {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) tot += red[i];
    rms = rsqrtf(tot / (float)K + a.eps);
  }
  // pass 2: one warp per 128-wide block, 4 elements per lane
  for (int b = sb0 + w; b < sb1; b += NW) {
    const int k0 = b * 128 + lane * 4;
    const bool in_slice = b >= kb0 && b < kb0 + nxb;
    float v[4];
    if (in_slice) {
      const uint2 raw = reinterpret_cast<const uint2*>(stg)[(b - kb0) * 32 + lane];
      const float2 v01 = bf2x_to_f2(raw.x), v23 = bf2x_to_f2(raw.y);
      v[0] = v01.x; v[1] = v01.y; v[2] = v23.x; v[3] = v23.y;
    } else {  // CTA 0 writing xn_out: the same h as pass 1, from global memory
      const uint2 raw = *reinterpret_cast<const uint2*>(xin + k0);
      const float2 v01 = bf2x_to_f2(raw.x), v23 = bf2x_to_f2(raw.y);
      v[0] = v01.x; v[1] = v01.y; v[2] = v23.x; v[3] = v23.y;
      if (a.pro == PRO_ADD_RMSNORM) {
        const uint2 r2 = *reinterpret_cast<const uint2*>(a.x2 + k0);
        const float2 g01 = bf2x_to_f2(r2.x), g23 = bf2x_to_f2(r2.y);
        v[0] = bfround(v[0] + g01.x); v[1] = bfround(v[1] + g01.y);
        v[2] = bfround(v[2] + g23.x); v[3] = bfround(v[3] + g23.y);
      }
    }
    if (a.pro == PRO_GATED_NORM) {
      // RMSNormGated over this 128-wide block (one GatedDeltaNet value head),
      // the default decode path's rounding points (main.py:1152-1159):
      // bf16(bf16(bf16(c * rsqrt(mean(c^2) + eps)) * w) * bf16(silu(z)))
      float cs = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
      cs = warp_sum(cs);
      const float r = rsqrtf(cs / 128.0f + a.eps);
      // z staged in pass 1, the norm weight before griddepcontrol.wait
      const uint2 zr = reinterpret_cast<const uint2*>(nws)[(b - kb0) * 32 + lane];
      const uint2 wr = reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(nws) + nxb * 256)[lane];
      const float2 z01 = bf2x_to_f2(zr.x), z23 = bf2x_to_f2(zr.y);
      const float2 w01 = bf2x_to_f2(wr.x), w23 = bf2x_to_f2(wr.y);
      const float zv[4] = {z01.x, z01.y, z23.x, z23.y}, wv[4] = {w01.x, w01.y, w23.x, w23.y};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float t = bfround(bfround(v[q] * r) * wv[q]);
        const float zs = bfround(zv[q] / (1.0f + expf(-zv[q])));
        v[q] = bfround(t * zs);
      }
    } else if (a.pro != PRO_NONE) {
      const float4 wn = in_slice ? reinterpret_cast<const float4*>(nws)[(b - kb0) * 32 + lane]
                                 : __ldg(reinterpret_cast<const float4*>(a.norm_w + k0));
      const float wv[4] = {wn.x, wn.y, wn.z, wn.w};
      bf16 o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        o[q] = f2bf(v[q] * rms * (1.0f + wv[q]));
        v[q] = bf2f(o[q]);
      }
      if (all) {
        uint2 ov;
        ov.x = (uint32_t)__bfloat16_as_ushort(o[0]) | ((uint32_t)__bfloat16_as_ushort(o[1]) << 16);
        ov.y = (uint32_t)__bfloat16_as_ushort(o[2]) | ((uint32_t)__bfloat16_as_ushort(o[3]) << 16);
        *reinterpret_cast<uint2*>(a.xn_out + k0) = ov;
      }
    }
    if (!in_slice) continue;  // warp-uniform
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    m = warp_max(m);
    // m = 1.f * 2^(ebits - 127): e = 134 - ebits puts m * 2^e in [2^7, 2^8)
    const int ebits = (int)((__float_as_uint(m) >> 23) & 0xffu);
    int e = m > 0.f ? (ebits == 0 ? 100 : 134 - ebits) : 0;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
    const float sc = exp2i(e);
    float xs[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) xs[q] = v[q] * sc;
    const uint32_t h01 = f32x2_to_e4m3x2(xs[0], xs[1]), h23 = f32x2_to_e4m3x2(xs[2], xs[3]);
    const float2 g01 = h2u_to_f2(e4m3x2_to_f16x2(h01)), g23 = h2u_to_f2(e4m3x2_to_f16x2(h23));
    // lo carries 32 * (x * 2^e - hi): |x * 2^e - hi| <= 8, so 32x stays below 448
    const uint32_t l01 = f32x2_to_e4m3x2((xs[0] - g01.x) * 32.f, (xs[1] - g01.y) * 32.f);
    const uint32_t l23 = f32x2_to_e4m3x2((xs[2] - g23.x) * 32.f, (xs[3] - g23.y) * 32.f);
    // 128-byte swizzle: 16-byte chunk c of row n sits at chunk c ^ n
    const int c = lane >> 2, within = (lane & 3) * 4;
    uint8_t* blk = xbg + (b - kb0) * XBLK;
    *reinterpret_cast<uint32_t*>(blk + (c << 4) + within) = h01 | (h23 << 16);
    *reinterpret_cast<uint32_t*>(blk + 128 + ((c ^ 1) << 4) + within) = l01 | (l23 << 16);
    if (lane == 0) xinv[b - kb0] = exp2i(-e);
  }
  fence_proxy_async_smem();  // the tensor core reads these bytes through the async proxy
  named_bar(1, NT);
}

// ---------------------------------------------------------------------------
// The kernel.  PAIR: gate/up segments (two matrices per item).
// ---------------------------------------------------------------------------
template <typename ST, bool PAIR>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemv_tc_kernel(const __grid_constant__ GemvArgs a, const __grid_constant__ GemvMaps m) {
  constexpr int P = PAIR ? 2 : 1;
  constexpr int TS = TC_MAX_TSLOTS / P;  // TMEM accumulator slots
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t sbase = (raw_s + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw_s);
  const int K = a.K, nkb = K >> 7;
  const int C = a.nslice;
  const int S = a.stages;
  const TcSmem L = tc_smem_layout(K, P, C, S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nitems = a.nunits * C;
  // gridDim.x is a multiple of C, so every item of this CTA has the same K slice
  const int csl = blockIdx.x % C;
  const int ckb0 = (csl * nkb) / C, cnxb = ((csl + 1) * nkb) / C - ckb0;
  const uint32_t ring = sbase + L.ring_off;
  const uint32_t xb = sbase + L.xb_off;
  float* xinv = reinterpret_cast<float*>(gbase + L.xinv_off);
  const uint32_t bar = sbase + L.bar_off;
  auto full_bar = [&](int s) { return bar + 8u * s; };
  auto empty_bar = [&](int s) { return bar + 8u * (S + s); };
  auto tfull_bar = [&](int t) { return bar + 8u * (2 * S + t); };
  auto tempty_bar = [&](int t) { return bar + 8u * (2 * S + TS + t); };
  const uint32_t xready_bar = bar + 8u * (2 * S + 2 * TS);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gbase + L.misc_off);
  float* red = reinterpret_cast<float*>(gbase + L.misc_off + 16);
  int* last_flag = reinterpret_cast<int*>(gbase + L.misc_off + 48);
  unsigned long long* am_misc = reinterpret_cast<unsigned long long*>(gbase + L.misc_off + 64);

  // Producer state (thread 0 = warp 0 lane 0): walks (item, K-block) pairs;
  // K-block number p_blk goes to ring stage p_blk % S.
  const uint64_t pol = l2_policy_evict_first();  // weights are read once per step
  int p_i = blockIdx.x, p_kb = -1, p_kb1 = 0, p_blk = 0, p_seg = 0, p_row0 = 0;
  auto p_next = [&]() -> bool {
    if (p_kb >= 0 && ++p_kb < p_kb1) return true;
    if (p_kb >= 0) p_i += gridDim.x;
    if (p_i >= nitems) return false;
    const TcItem t = tc_item(a, p_i, nkb);
    p_seg = t.seg;
    p_row0 = t.row0;
    p_kb = t.kb0;
    p_kb1 = t.kb1;
    return true;
  };
  auto p_issue = [&]() {
    const int s = p_blk % S;
    mbar_arrive_expect_tx(full_bar(s), (uint32_t)(P * TC_TILE));
    const uint32_t dst = ring + (uint32_t)s * L.stage_bytes;
    tma_load_2d(dst, &m.map[p_seg][0], p_kb * 128, p_row0, full_bar(s), pol);
    if (PAIR) tma_load_2d(dst + TC_TILE, &m.map[p_seg][1], p_kb * 128, p_row0, full_bar(s), pol);
    ++p_blk;
  };
  bool p_has = false;

  if (threadIdx.x == 0) {
    pdl_trigger();
    for (int i = 0; i < S; ++i) {
      mbar_init(full_bar(i), 1);
      mbar_init(empty_bar(i), 1);
    }
    for (int i = 0; i < TS; ++i) {
      mbar_init(tfull_bar(i), 1);
      mbar_init(tempty_bar(i), 4);
    }
    mbar_init(xready_bar, 1);
    mbar_fence_init();
    // weights are static: fill the ring right away
    p_has = p_next();
    while (p_has && p_blk < S) {
      p_issue();
      p_has = p_next();
    }
  }
  if (warp >= 2 && a.pro != PRO_NONE && a.pro != PRO_GATED_NORM) {
    // RMSNorm weights of this CTA's slice (static data: before griddepcontrol.wait)
    float4* nws = reinterpret_cast<float4*>(gbase + L.nw_off);
    const float4* src = reinterpret_cast<const float4*>(a.norm_w + ckb0 * 128);
    for (int o = threadIdx.x - 64; o < cnxb * 32; o += 192) nws[o] = __ldg(src + o);
  }
  if (warp >= 2 && a.pro == PRO_GATED_NORM && threadIdx.x - 64 < 16) {
    // gated-norm weight (one head, static) after the staged z
    reinterpret_cast<uint4*>(gbase + L.nw_off + cnxb * 256)[threadIdx.x - 64] =
        __ldg(reinterpret_cast<const uint4*>(a.gw) + (threadIdx.x - 64));
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_holder)), "r"(TC_TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  unsigned long long am_best = 0ull;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      bool ok = true;
      while (p_has) {
        if (!mbar_wait_bounded(empty_bar(p_blk % S), ((p_blk / S) & 1) ^ 1)) {
          ok = false;
          break;
        }
        p_issue();
        p_has = p_next();
      }
      if (!ok) qwen_err_set(ERR_TC_TIMEOUT);
      // every copy issued has landed before the CTA may exit
      for (int j = p_blk - S < 0 ? 0 : p_blk - S; j < p_blk; ++j)
        if (!mbar_wait_bounded(full_bar(j % S), (j / S) & 1)) qwen_err_set(ERR_TC_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool ok = mbar_wait_bounded(xready_bar, 0);
      tc_fence_after();
      const uint64_t bdesc0 = tc_smem_desc(xb);
      int it = 0;
      for (int i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
        const TcItem t = tc_item(a, i, nkb);
        for (int kb = t.kb0; kb < t.kb1; ++kb, ++it) {
          const int s = it % S, ts = it % TS;
          if (!mbar_wait_bounded(full_bar(s), (it / S) & 1) ||
              (it >= TS && !mbar_wait_bounded(tempty_bar(ts), ((it / TS) & 1) ^ 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = tc_smem_desc(ring + (uint32_t)s * L.stage_bytes);
          const uint64_t bd = bdesc0 + (uint64_t)((kb - ckb0) * (TC_XBLK >> 4));
#pragma unroll
          for (int p = 0; p < P; ++p)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma(tmem + ts * (16 * P) + p * 16, ad + (uint64_t)(p * (TC_TILE >> 4) + 2 * k), bd + 2 * k,
                     k > 0 ? 1u : 0u);
          tc_commit(empty_bar(s));  // the stage is free once these MMAs complete
          tc_commit(tfull_bar(ts));
        }
      }
      if (!ok) qwen_err_set(ERR_TC_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ---------------- x preparation (warps 2..7), then epilogue (warps 4..7) ----------------
    if (warp == 2) l2_prefetch_share(a.pf, lane);  // next launch's weights (static data)
    tc_x_zero(cnxb, gbase + L.xb_off);
    pdl_wait();
    tc_x_prepare(a, ckb0, cnxb, gbase + L.xb_off, gbase + L.stg_off,
                 reinterpret_cast<const float*>(gbase + L.nw_off), xinv, red);
    if (threadIdx.x == 64) mbar_arrive(xready_bar);
    if (warp >= 4) {
      const int q = warp & 3;  // TMEM lane quadrant
      const int r = q * 32 + lane;
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
      // A failed wait (timeout) stops all further waits of this warp but not
      // the walk over the items, so the named barriers below stay matched.
      int it = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < nitems; i += gridDim.x) {
        const TcItem t = tc_item(a, i, nkb);
        const GemvSeg& sg = a.seg[t.seg];
        const int nkbs = t.kb1 - t.kb0;
        // block scales of this item: lane l holds K-block kb0 + l (nkbs <= 32)
        float scl[P];
#pragma unroll
        for (int p = 0; p < P; ++p) scl[p] = 0.f;
        if (lane < nkbs) {
          const int idx = (t.row0 >> 7) * sg.kblk + t.kb0 + lane;
          scl[0] = load_scale<ST>(sg.s, idx);
          if (PAIR) scl[P - 1] = load_scale<ST>(sg.s2, idx);
        }
        float acc[P];
#pragma unroll
        for (int p = 0; p < P; ++p) acc[p] = 0.f;
        // K-blocks in groups of G = TS / 2: one wait on the group's last
        // block (a commit covers every earlier MMA of the issuing thread), G
        // TMEM loads in flight, one wait::ld.  The MMA issuer meanwhile fills
        // the other half of the slots.
        constexpr int G = TS / 2;
        for (int g0 = t.kb0; g0 < t.kb1; g0 += G, it += G) {
          const int n = t.kb1 - g0 < G ? t.kb1 - g0 : G;
          const int itl = it + n - 1;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(tfull_bar(itl % TS), (itl / TS) & 1));
          if (!ok) continue;
          tc_fence_after();
          uint32_t v[G][2 * P];
#pragma unroll
          for (int j = 0; j < G; ++j)
            if (j < n) {
              const int ts = (it + j) % TS;
#pragma unroll
              for (int p = 0; p < P; ++p) tc_ld2(tl + ts * (16 * P) + p * 16, v[j][2 * p], v[j][2 * p + 1]);
            }
          tc_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane < n) mbar_arrive(tempty_bar((it + lane) % TS));
#pragma unroll
          for (int j = 0; j < G; ++j)
            if (j < n) {
              const int kb = g0 + j;
              const float f = xinv[kb - ckb0];
#pragma unroll
              for (int p = 0; p < P; ++p) {
                const float sf = __shfl_sync(0xffffffffu, scl[p], kb - t.kb0) * f;
                acc[p] = fmaf(__uint_as_float(v[j][2 * p]) + __uint_as_float(v[j][2 * p + 1]) * 0.03125f, sf, acc[p]);
              }
            }
        }
        it += t.kb1 - t.kb0 - ((t.kb1 - t.kb0 + G - 1) / G) * G;  // undo the last group's overshoot
        const int row = t.row0 + r;
        if (C == 1) {
          if (row < sg.n) am_best = gemv_epilogue(sg, row, acc[0], PAIR ? acc[P - 1] : 0.f, am_best);
        } else if (sg.epi == EPI_SLICES) {
          // K split without the reduction: the next launch adds the slices
          if (row < sg.n) reinterpret_cast<float*>(sg.y)[(size_t)csl * sg.n + row] = acc[0];
        } else {
          // K split: publish this slice, the last CTA of the unit reduces in slice order
          float* part = g_tc_part + (size_t)i * P * TC_ROWS;
#pragma unroll
          for (int p = 0; p < P; ++p) part[p * TC_ROWS + r] = acc[p];
          __threadfence();
          named_bar(2, 128);
          if (threadIdx.x == 128) *last_flag = atomicAdd(&g_tc_cnt[t.unit], 1u) == (unsigned)(C - 1);
          named_bar(2, 128);
          if (*last_flag) {
            __threadfence();
            // up to 8 slices' loads in flight at once, added in slice order
            float tot[P];
#pragma unroll
            for (int p = 0; p < P; ++p) tot[p] = 0.f;
            for (int c0 = 0; c0 < C; c0 += 8) {
              float v[8][P];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float* pp = g_tc_part + (size_t)(t.unit * C + c0 + j) * P * TC_ROWS;
#pragma unroll
                for (int p = 0; p < P; ++p) v[j][p] = c0 + j < C ? __ldcg(pp + p * TC_ROWS + r) : 0.f;
              }
#pragma unroll
              for (int j = 0; j < 8; ++j)
#pragma unroll
                for (int p = 0; p < P; ++p)
                  if (c0 + j < C) tot[p] += v[j][p];
            }
            if (row < sg.n) am_best = gemv_epilogue(sg, row, tot[0], PAIR ? tot[P - 1] : 0.f, am_best);
            if (threadIdx.x == 128) g_tc_cnt[t.unit] = 0u;
          }
          named_bar(2, 128);  // last_flag is reused by the next item
        }
      }
      if (!ok) qwen_err_set(ERR_TC_TIMEOUT);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (a.am_ws) argmax_finish(a, am_best, am_misc);
  if (a.pro == PRO_P2P_RMSNORM && threadIdx.x == 0) p2p_round_done(*a.p2p);
  if (a.seg[0].epi == EPI_SLICES && blockIdx.x == 0 && threadIdx.x == 0) *static_cast<int*>(a.seg[0].y2) = C;
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TC_TMEM_COLS) : "memory");
  }
}

}  // namespace qwen
