// Block-scaled E4M3 x BF16 prefill GEMM on the tcgen05 tensor cores.
//
//     y[m, n] = bf16( sum_kb scale[n / 128, kb] * sum_{k in kb} x[m, k] * e4m3(W[n, k]) )
//
// for M >= 2 token rows (the reference's fp8_gemm_batch, fp8_kernels.cu:23-89,
// called by fp8_linear main.py:262-269 during prefill).  FP8 MMAs with the
// weights exactly as stored and a per-128-K-block scale promotion in FP32:
//
//   * gemm_x_split_kernel turns x into the A operand once per call: for every
//     token tile of 64 rows a [128, K] E4M3 block; token 16 g + j (g < 4,
//     j < 16) has hi = RN(x * 2^e) in row 32 g + j and lo = RN(32 (x * 2^e -
//     hi)) in row 32 g + 16 + j, with e per (token, 128-K block) chosen so
//     that the block's largest magnitude lands in [2^7, 2^8) (hi + lo / 32
//     equals the BF16 value for every element within 2^-14 of that maximum),
//     plus 2^-e per (token, block).
//   * gemm_tc_kernel walks (128 weight rows) x (64 tokens) output tiles,
//     weight-row-major so that consecutive tiles reuse the weight tile from
//     L2.  Warp 0 streams the split x (A) and weight (B) K-blocks with 2-D
//     TMA (128-byte swizzle) into a ring of 32 KB stages; warp 1 issues four
//     tcgen05.mma kind::f8f6f4 (M=128, N=128, K=32) per K-block into one of
//     two TMEM accumulators, whose lanes are then split-x rows and whose
//     columns are weight rows.  A K-block's scale scale[n/128, kb] *
//     2^-e[token, kb] is one number per TMEM lane (the weight block covers all
//     128 columns), so each of the eight epilogue warps (one TMEM lane quarter
//     = 16 tokens' hi and lo rows, one 64-column half) adds its 64 columns
//     times that number into FP32 registers: one FMA per accumulator element
//     and K-block.  At the end of the tile the hi and lo lanes of a token
//     exchange their sums (one shuffle per column), form hi + lo / 32 and
//     store BF16 y.
// Every mbarrier wait is bounded (QWEN_WAIT_TIMEOUT_NS) and reports a timeout
// through the device error word.
#pragma once

#include "gemv_tc.cuh"

namespace qwen {

constexpr int GM_TOK = 64;           // tokens per output tile
constexpr int GM_STAGE = 2 * TC_TILE;  // A tile + B tile of one K-block
constexpr int GM_THREADS = 384;      // 12 warps: producer, MMA, 2 idle, 8 epilogue
constexpr int GM_TMEM_COLS = 256;    // two accumulators of 128 columns

// x [M, K] BF16 -> split operand xs [ceil(M/64)][128][K] E4M3 and
// xinv [ceil(M/64) * 64][K/128] FP32.  One warp per (token, 128-K block).
__global__ void __launch_bounds__(256) gemm_x_split_kernel(const bf16* __restrict__ x, int M, int K,
                                                           uint8_t* __restrict__ xs, float* __restrict__ xinv) {
  const int nkb = K >> 7;
  const int lane = threadIdx.x & 31;
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int mpad = (M + GM_TOK - 1) / GM_TOK * GM_TOK;
  if (wid >= mpad * nkb) return;
  const int m = wid / nkb, kb = wid - m * nkb;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (m < M) {
    const uint2 raw = *reinterpret_cast<const uint2*>(x + (size_t)m * K + kb * 128 + lane * 4);
    const float2 a = bf2x_to_f2(raw.x), b = bf2x_to_f2(raw.y);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  }
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  mx = warp_max(mx);
  const int ebits = (int)((__float_as_uint(mx) >> 23) & 0xffu);
  int e = mx > 0.f ? (ebits == 0 ? 100 : 134 - ebits) : 0;
  e = e < -100 ? -100 : (e > 100 ? 100 : e);
  const float sc = exp2i(e);
  float s[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) s[q] = v[q] * sc;
  const uint32_t h01 = f32x2_to_e4m3x2(s[0], s[1]), h23 = f32x2_to_e4m3x2(s[2], s[3]);
  const float2 g01 = h2u_to_f2(e4m3x2_to_f16x2(h01)), g23 = h2u_to_f2(e4m3x2_to_f16x2(h23));
  const uint32_t l01 = f32x2_to_e4m3x2((s[0] - g01.x) * 32.f, (s[1] - g01.y) * 32.f);
  const uint32_t l23 = f32x2_to_e4m3x2((s[2] - g23.x) * 32.f, (s[3] - g23.y) * 32.f);
  const int t = m / GM_TOK, r = m - t * GM_TOK;
  const int row_hi = (r >> 4) * 32 + (r & 15);  // lo: row_hi + 16 (same TMEM lane quarter)
  uint8_t* tile = xs + (size_t)t * 128 * K;
  *reinterpret_cast<uint32_t*>(tile + (size_t)row_hi * K + kb * 128 + lane * 4) = h01 | (h23 << 16);
  *reinterpret_cast<uint32_t*>(tile + (size_t)(row_hi + 16) * K + kb * 128 + lane * 4) = l01 | (l23 << 16);
  if (lane == 0) xinv[(size_t)m * nkb + kb] = exp2i(-e);
}

// 32 consecutive TMEM columns of this warp's lane quarter (one 32-bit value
// per column and lane).
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&p);
}

struct GemmArgs {
  const void* s;   // weight scales, block layout [ceil(N/128), K/128]
  const float* xinv;
  bf16* y;         // [M, N]
  int M, N, K, stages;
};

template <typename ST>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ GemmArgs a, const __grid_constant__ CUtensorMap wmap,
                   const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t sbase = (raw_s + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw_s);
  const int K = a.K, nkb = K >> 7, S = a.stages;
  const int ntn = (a.N + TC_ROWS - 1) / TC_ROWS, ntm = (a.M + GM_TOK - 1) / GM_TOK;
  const int ntiles = ntn * ntm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ring = sbase;
  const uint32_t bar = sbase + (uint32_t)S * GM_STAGE;
  auto full_bar = [&](int s) { return bar + 8u * s; };
  auto empty_bar = [&](int s) { return bar + 8u * (S + s); };
  auto tfull_bar = [&](int b) { return bar + 8u * (2 * S + b); };
  auto tempty_bar = [&](int b) { return bar + 8u * (2 * S + 2 + b); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(gbase + S * GM_STAGE + 512);

  if (threadIdx.x == 0) {
    pdl_trigger();
    for (int i = 0; i < S; ++i) {
      mbar_init(full_bar(i), 1);
      mbar_init(empty_bar(i), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 8);
    }
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_holder)), "r"(GM_TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // tile t -> weight rows n0 = (t / ntm) * 128, tokens m0 = (t % ntm) * 64

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      const uint64_t pol = l2_policy_evict_first();
      pdl_wait();  // the split x comes from the previous kernel
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int n0 = (t / ntm) * TC_ROWS, mt = t % ntm;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          if (it >= S && !mbar_wait_bounded(empty_bar(s), ((it / S) & 1) ^ 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(s), (uint32_t)GM_STAGE);
          const uint32_t dst = ring + (uint32_t)s * GM_STAGE;
          tma_load_2d(dst, &wmap, kb * 128, n0, full_bar(s), pol);
          tma_load_2d(dst + TC_TILE, &xmap, kb * 128, mt * 128, full_bar(s), pol);
        }
      }
      if (!ok) qwen_err_set(ERR_TC_TIMEOUT);
      for (int j = it - S < 0 ? 0 : it - S; j < it; ++j)
        if (!mbar_wait_bounded(full_bar(j % S), (j / S) & 1)) qwen_err_set(ERR_TC_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = (1u << 4) | ((128u >> 3) << 17) | ((128u >> 4) << 24);  // F32 <- E4M3 x E4M3
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S, b = it & 1;
          if (!mbar_wait_bounded(full_bar(s), (it / S) & 1) ||
              (it >= 2 && !mbar_wait_bounded(tempty_bar(b), ((it >> 1) & 1) ^ 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          // A = the split x tile (lanes: x rows), B = the weight tile (columns: weight rows)
          const uint64_t ad = tc_smem_desc(ring + (uint32_t)s * GM_STAGE + TC_TILE);
          const uint64_t bd = tc_smem_desc(ring + (uint32_t)s * GM_STAGE);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n"
                :: "r"(tmem + b * 128), "l"(ad + 2 * k), "l"(bd + 2 * k), "r"(idesc), "r"(k > 0 ? 1u : 0u),
                   "r"(0u)
                : "memory");
          tc_commit(empty_bar(s));
          tc_commit(tfull_bar(b));
        }
      }
      if (!ok) qwen_err_set(ERR_TC_TIMEOUT);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---------------- epilogue: 8 warps, lane quarter q, column half h ----------------
    pdl_wait();  // xinv comes from the previous kernel; y may still be read by it
    const int q = warp & 3, h = (warp - 4) >> 2;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * 64);
    const bool lo_lane = lane >= 16;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const int n0 = (t / ntm) * TC_ROWS + h * 64, m = (t % ntm) * GM_TOK + q * 16 + (lane & 15);
      const int srow = (n0 >> 7) * nkb;
      const float* xi_row = a.xinv + (size_t)m * nkb;
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int b = it & 1;
        // this lane's scale for the block: the token's 2^-e times the weight block's scale
        const float f = xi_row[kb] * load_scale<ST>(a.s, srow + kb);
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(tfull_bar(b), (it >> 1) & 1));
        if (!ok) continue;
        tc_fence_after();
        uint32_t v0[32], v1[32];
        tc_ld32(tl + b * 128, v0);
        tc_ld32(tl + b * 128 + 32, v1);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty_bar(b));
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          acc[j] = fmaf(__uint_as_float(v0[j]), f, acc[j]);
          acc[32 + j] = fmaf(__uint_as_float(v1[j]), f, acc[32 + j]);
        }
      }
      // hi + lo / 32: lanes j and j + 16 hold the same token's hi and lo sums;
      // lane j stores columns [0, 32), lane j + 16 columns [32, 64)
      float y[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float mine_a = acc[j], mine_b = acc[32 + j];
        const float other_a = __shfl_xor_sync(0xffffffffu, mine_a, 16);
        const float other_b = __shfl_xor_sync(0xffffffffu, mine_b, 16);
        y[j] = lo_lane ? other_b + mine_b * 0.03125f : mine_a + other_a * 0.03125f;
      }
      const int c0 = n0 + (lo_lane ? 32 : 0);
      if (m < a.M) {
        bf16* dst = a.y + (size_t)m * a.N + c0;
        if (c0 + 32 <= a.N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            pk.x = pack_bf16x2(y[j], y[j + 1]);
            pk.y = pack_bf16x2(y[j + 2], y[j + 3]);
            pk.z = pack_bf16x2(y[j + 4], y[j + 5]);
            pk.w = pack_bf16x2(y[j + 6], y[j + 7]);
            *reinterpret_cast<uint4*>(dst + j) = pk;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < a.N) dst[j] = f2bf(y[j]);
        }
      }
    }
    if (!ok) qwen_err_set(ERR_TC_TIMEOUT);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(GM_TMEM_COLS) : "memory");
  }
}

inline int gemm_smem_bytes(int stages) { return 1024 + stages * GM_STAGE + 512 + 64; }

}  // namespace qwen
