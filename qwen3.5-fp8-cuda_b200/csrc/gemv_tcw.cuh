// Block-scaled E4M3 x BF16 GEMV on tcgen05 with the weights as the wide
// operand: one MMA covers 256 weight rows x 32 K.
//
// Same contract as gemv_tc.cuh (and the reference's gemv_v4_kernel family,
// fused_kernels.cu:91-479):
//     v[r] = sum_kb scale[r / 128, kb] * sum_{k in kb} x[k] * e4m3(W[r, k])
// with FP32 accumulation, then the segment epilogue.
//
// Why: a tcgen05.mma instruction of kind::f8f6f4 costs about the same time
// whatever its N (up to 256) on B200, so the number of instructions per
// weight byte bounds a GEMV.  With the weights as A (M = 128 rows) each MMA
// consumes 4 KB of weights; here they are B (N = 256 rows), 8 KB per MMA.
//
//   D[m][n] = sum_k A[m][k] * B[n][k],  M = 128, N = 256, K = 32 per MMA
//   A = x: one 128-byte-swizzled row group (1 KB) per 128-wide K-block, row
//       0 = hi, row 1 = lo of x * 2^e = hi + lo / 32 (E4M3, exact within
//       2^-14 of the block maximum), rows 2-7 zero.  The descriptor's
//       8-row-group stride is 0, so all 16 row groups of the M = 128 operand
//       read that same 1 KB: TMEM lanes 32q + 0 / 32q + 1 hold the hi / lo
//       sums in every lane quarter q.
//   B = weights: two 128-row TMA tiles (16 KB each) side by side: rows
//       r0..r0+255 of one matrix, or 128 gate rows then the same 128 up rows.
//   D = 256 FP32 columns per K-block; two accumulators (512 TMEM columns)
//       alternate between K-blocks.
//
// Roles (256 threads, up to 128 registers each): warp 0 lane 0 streams the weight
// tiles (32 KB stages, filled before griddepcontrol.wait); warp 1 lane 0
// issues four MMAs per K-block and commits the stage and the accumulator;
// warps 2-7 prepare x; warps 4-7 (lane quarter q) read columns 64q..64q+63
// of lanes 32q and 32q+1 and accumulate them times scale[row block, kb] *
// 2^-e (1/32 more for lo) in 64 FP32 registers, the hi lane and the lo lane
// separately.  At the end of an item the four warps gather hi + lo of the
// 256 columns in shared memory and 128 threads run the epilogue, two rows
// each (one gate/up row for the paired MLP).
//
// K split, determinism, error handling and the per-device scratch are as in
// gemv_tc.cuh: the last CTA of a unit adds the slices' partial rows in slice
// order; every mbarrier wait is bounded and reports through the device error
// word; on a timeout the producer drains its copies and the CTA frees TMEM.
#pragma once

#include "gemv_tc.cuh"

namespace qwen {

constexpr int TW_N = 256;               // weight rows per MMA (N) and per item
constexpr int TW_STAGE = 2 * TC_TILE;   // 32 KB: two 128-row tiles
constexpr int TW_XBLK = 1024;           // x operand bytes per K-block
constexpr int TW_TMEM_COLS = 512;       // two accumulators of 256 columns
constexpr int TW_THREADS = 256;
constexpr int TW_MAX_STAGES = 8;

struct TwSmem {
  int ring_off, xa_off, stg_off, nw_off, xinv_off, red_off, bar_off, misc_off, total;
};
__host__ __device__ inline TwSmem tw_smem_layout(int K, int C, int stages) {
  TwSmem L;
  const int nkb = K >> 7;
  const int nxb = (nkb + C - 1) / C;
  L.ring_off = 0;
  L.xa_off = stages * TW_STAGE;
  L.stg_off = L.xa_off + nxb * TW_XBLK;
  L.nw_off = L.stg_off + nxb * 256;
  L.xinv_off = L.nw_off + nxb * 512;
  L.red_off = L.xinv_off + align_up(4 * nxb, 16);  // 2 x 256 floats: hi and lo sums of an item
  L.bar_off = L.red_off + 2048;
  L.misc_off = L.bar_off + 256;
  L.total = 1024 /* alignment slack */ + L.misc_off + 256;
  return L;
}
__host__ __device__ inline int tw_stages_for(int K, int C, int budget) {
  const int fixed = tw_smem_layout(K, C, 0).total;
  const int s = (budget - fixed) / TW_STAGE;
  return s < 2 ? 0 : (s > TW_MAX_STAGES ? TW_MAX_STAGES : s);
}

// x operand descriptor: K-major, 128-byte swizzle, 8-row-group stride 0 (every
// row group of the 128-row operand is the same 1 KB).
__device__ __forceinline__ uint64_t tw_x_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | (0ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: D = F32, A = B = E4M3, both K-major, N = 256, M = 128.
constexpr uint32_t TW_IDESC = (1u << 4) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void tw_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n"
      :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(TW_IDESC), "r"(accumulate), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tw_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

// Item i -> unit i / C, K slice i % C.  A unit is 256 rows of one matrix, or
// 128 rows of a gate/up pair.
__device__ __forceinline__ TcItem tw_item(const GemvArgs& a, int i, int nkb, int unit_rows) {
  TcItem t;
  const int C = a.nslice;
  t.unit = i / C;
  const int sl = i - t.unit * C;
  t.seg = gemv_find_seg(a, t.unit);
  t.row0 = (t.unit - a.seg[t.seg].unit0) * unit_rows;
  t.kb0 = (sl * nkb) / C;
  t.kb1 = ((sl + 1) * nkb) / C;
  return t;
}

// At most 128 registers per thread.  The host sizes the ring so that one CTA
// fills an SM's shared memory: a CTA holds all 512 TMEM columns.
template <typename ST, bool PAIR>
__global__ void __launch_bounds__(TW_THREADS, 2)
    gemv_tcw_kernel(const __grid_constant__ GemvArgs a, const __grid_constant__ GemvMaps m) {
  constexpr int UROWS = PAIR ? 128 : 256;  // output rows per unit
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t sbase = (raw_s + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw_s);
  const int K = a.K, nkb = K >> 7;
  const int C = a.nslice;
  const int S = a.stages;
  const TwSmem L = tw_smem_layout(K, C, S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nitems = a.nunits * C;
  const int csl = blockIdx.x % C;  // gridDim.x is a multiple of C
  const int ckb0 = (csl * nkb) / C, cnxb = ((csl + 1) * nkb) / C - ckb0;
  const uint32_t ring = sbase + L.ring_off;
  const uint32_t xa = sbase + L.xa_off;
  float* xinv = reinterpret_cast<float*>(gbase + L.xinv_off);
  float* red = reinterpret_cast<float*>(gbase + L.red_off);
  const uint32_t bar = sbase + L.bar_off;
  auto full_bar = [&](int s) { return bar + 8u * s; };
  auto empty_bar = [&](int s) { return bar + 8u * (TW_MAX_STAGES + s); };
  auto tfull_bar = [&](int b) { return bar + 8u * (2 * TW_MAX_STAGES + b); };
  auto tempty_bar = [&](int b) { return bar + 8u * (2 * TW_MAX_STAGES + 2 + b); };
  const uint32_t xready_bar = bar + 8u * (2 * TW_MAX_STAGES + 4);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gbase + L.misc_off);
  float* wred = reinterpret_cast<float*>(gbase + L.misc_off + 16);
  int* last_flag = reinterpret_cast<int*>(gbase + L.misc_off + 48);
  unsigned long long* am_misc = reinterpret_cast<unsigned long long*>(gbase + L.misc_off + 64);

  const uint64_t pol = l2_policy_evict_first();
  int p_i = blockIdx.x, p_kb = -1, p_kb1 = 0, p_blk = 0, p_seg = 0, p_row0 = 0;
  auto p_next = [&]() -> bool {
    if (p_kb >= 0 && ++p_kb < p_kb1) return true;
    if (p_kb >= 0) p_i += gridDim.x;
    if (p_i >= nitems) return false;
    const TcItem t = tw_item(a, p_i, nkb, UROWS);
    p_seg = t.seg;
    p_row0 = t.row0;
    p_kb = t.kb0;
    p_kb1 = t.kb1;
    return true;
  };
  auto p_issue = [&]() {
    const int s = p_blk % S;
    mbar_arrive_expect_tx(full_bar(s), (uint32_t)TW_STAGE);
    const uint32_t dst = ring + (uint32_t)s * TW_STAGE;
    tma_load_2d(dst, &m.map[p_seg][0], p_kb * 128, p_row0, full_bar(s), pol);
    if (PAIR)
      tma_load_2d(dst + TC_TILE, &m.map[p_seg][1], p_kb * 128, p_row0, full_bar(s), pol);
    else  // rows past the matrix end read as zero
      tma_load_2d(dst + TC_TILE, &m.map[p_seg][0], p_kb * 128, p_row0 + 128, full_bar(s), pol);
    ++p_blk;
  };
  bool p_has = false;

  if (threadIdx.x == 0) {
    pdl_trigger();
    for (int i = 0; i < S; ++i) {
      mbar_init(full_bar(i), 1);
      mbar_init(empty_bar(i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(tfull_bar(i), 1);
      mbar_init(tempty_bar(i), 4);
    }
    mbar_init(xready_bar, 1);
    mbar_fence_init();
    p_has = p_next();
    while (p_has && p_blk < S) {
      p_issue();
      p_has = p_next();
    }
  }
  if (warp >= 2) {
    if (a.pro != PRO_NONE && a.pro != PRO_GATED_NORM) {
      float4* nws = reinterpret_cast<float4*>(gbase + L.nw_off);
      const float4* src = reinterpret_cast<const float4*>(a.norm_w + ckb0 * 128);
      for (int o = threadIdx.x - 64; o < cnxb * 32; o += 192) nws[o] = __ldg(src + o);
    }
    if (a.pro == PRO_GATED_NORM && threadIdx.x - 64 < 16)  // gated-norm weight after the staged z
      reinterpret_cast<uint4*>(gbase + L.nw_off + cnxb * 256)[threadIdx.x - 64] =
          __ldg(reinterpret_cast<const uint4*>(a.gw) + (threadIdx.x - 64));
    tc_x_zero<TW_XBLK>(cnxb, gbase + L.xa_off);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_holder)), "r"(TW_TMEM_COLS) : "memory");
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
      for (int j = p_blk - S < 0 ? 0 : p_blk - S; j < p_blk; ++j)
        if (!mbar_wait_bounded(full_bar(j % S), (j / S) & 1)) qwen_err_set(ERR_TC_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      bool ok = mbar_wait_bounded(xready_bar, 0);
      tc_fence_after();
      const uint64_t adesc0 = tw_x_desc(xa);
      int it = 0;
      for (int i = blockIdx.x; i < nitems && ok; i += gridDim.x) {
        const TcItem t = tw_item(a, i, nkb, UROWS);
        for (int kb = t.kb0; kb < t.kb1; ++kb, ++it) {
          const int s = it % S, b = it & 1;
          if (!mbar_wait_bounded(full_bar(s), (it / S) & 1) ||
              (it >= 2 && !mbar_wait_bounded(tempty_bar(b), ((it >> 1) & 1) ^ 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bd = tc_smem_desc(ring + (uint32_t)s * TW_STAGE);
          const uint64_t ad = adesc0 + (uint64_t)((kb - ckb0) * (TW_XBLK >> 4));
#pragma unroll
          for (int k = 0; k < 4; ++k) tw_mma(tmem + (uint32_t)(b * 256), ad + 2 * k, bd + 2 * k, k > 0 ? 1u : 0u);
          tc_commit(empty_bar(s));
          tc_commit(tfull_bar(b));
        }
      }
      if (!ok) qwen_err_set(ERR_TC_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ---------------- x preparation (warps 2..7), then epilogue (warps 4..7) ----------------
    if (warp == 2) l2_prefetch_share(a.pf, lane);
    pdl_wait();
    tc_x_prepare<TW_XBLK>(a, ckb0, cnxb, gbase + L.xa_off, gbase + L.stg_off,
                          reinterpret_cast<const float*>(gbase + L.nw_off), xinv, wred);
    if (threadIdx.x == 64) mbar_arrive(xready_bar);
    if (warp >= 4) {
      const int q = warp & 3;     // TMEM lane quarter; columns 64q..64q+63
      const int e = threadIdx.x - 128;  // 0..127: epilogue thread
      const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(64 * q);
      int it = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < nitems; i += gridDim.x) {
        const TcItem t = tw_item(a, i, nkb, UROWS);
        const GemvSeg& sg = a.seg[t.seg];
        const int nkbs = t.kb1 - t.kb0;
        // this warp's 64 columns lie in one 128-row scale block of one matrix
        const void* smat = (PAIR && q >= 2) ? sg.s2 : sg.s;
        const int srow = PAIR ? t.row0 : t.row0 + 64 * q;
        float scl = 0.f;
        if (lane < nkbs && srow < sg.n) scl = load_scale<ST>(smat, (srow >> 7) * sg.kblk + t.kb0 + lane);
        float acc[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = 0.f;
        for (int kb = t.kb0; kb < t.kb1; ++kb, ++it) {
          const int b = it & 1;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(tfull_bar(b), (it >> 1) & 1));
          const float sf = __shfl_sync(0xffffffffu, scl, kb - t.kb0);
          if (!ok) continue;
          tc_fence_after();
          // lane 0 holds the hi sums, lane 1 the lo sums (weight 1/32); the
          // two 32-column halves one after the other keep registers low
          const float f = xinv[kb - ckb0] * sf * (lane == 1 ? 0.03125f : 1.0f);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t v[32];
            tw_ld32(tl + (uint32_t)(b * 256 + 32 * h), v);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[32 * h + j] = fmaf(__uint_as_float(v[j]), f, acc[32 * h + j]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar(b));
        }
        // gather: red[c] = hi sum, red[256 + c] = lo sum of column c
        if (lane < 2) {
#pragma unroll
          for (int j = 0; j < 64; ++j) red[lane * 256 + 64 * q + j] = acc[j];
        }
        named_bar(2, 128);
        // thread e: single matrix -> local rows e and e + 128; pair -> row e (gate e, up 128 + e)
        float val[2];
        val[0] = red[e] + red[256 + e];
        val[1] = red[128 + e] + red[384 + e];
        named_bar(2, 128);  // red is rewritten by the next item
        const int rowa = t.row0 + e, rowb = t.row0 + 128 + e;
        if (C == 1) {
          if (PAIR) {
            if (rowa < sg.n) am_best = gemv_epilogue(sg, rowa, val[0], val[1], am_best);
          } else {
            if (rowa < sg.n) am_best = gemv_epilogue(sg, rowa, val[0], 0.f, am_best);
            if (rowb < sg.n) am_best = gemv_epilogue(sg, rowb, val[1], 0.f, am_best);
          }
        } else {
          float* part = g_tc_part + (size_t)i * TW_N;
          part[e] = val[0];
          part[128 + e] = val[1];
          __threadfence();
          named_bar(2, 128);
          if (threadIdx.x == 128) *last_flag = atomicAdd(&g_tc_cnt[t.unit], 1u) == (unsigned)(C - 1);
          named_bar(2, 128);
          if (*last_flag) {
            __threadfence();
            float tot[2] = {0.f, 0.f};
            for (int c0 = 0; c0 < C; c0 += 8) {
              float pv[8][2];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float* pp = g_tc_part + (size_t)(t.unit * C + c0 + j) * TW_N;
                pv[j][0] = c0 + j < C ? __ldcg(pp + e) : 0.f;
                pv[j][1] = c0 + j < C ? __ldcg(pp + 128 + e) : 0.f;
              }
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (c0 + j < C) {
                  tot[0] += pv[j][0];
                  tot[1] += pv[j][1];
                }
            }
            if (PAIR) {
              if (rowa < sg.n) am_best = gemv_epilogue(sg, rowa, tot[0], tot[1], am_best);
            } else {
              if (rowa < sg.n) am_best = gemv_epilogue(sg, rowa, tot[0], 0.f, am_best);
              if (rowb < sg.n) am_best = gemv_epilogue(sg, rowb, tot[1], 0.f, am_best);
            }
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
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(TW_TMEM_COLS) : "memory");
  }
}

}  // namespace qwen
