// Block-scaled E4M3 x BF16 GEMV family for batch-1 decode on sm_100a.
//
// Computes, for every output row r of one or more weight segments,
//     v[r] = sum_kb scale[r, kb] * sum_{k in kb} x[k] * e4m3(W[r, k])
// with FP32 accumulation, then applies a fused epilogue (store, residual add,
// gate/up SiLU pairing, greedy argmax, GatedDeltaNet conv / gate math).
// Restates gemv_v4_kernel and its fused variants (fused_kernels.cu:91-479) as
// an HBM stream:
//
//  * a warp owns a tile of 8 weight rows (8 gate + 8 up rows for the paired
//    MLP) and a range of 128-wide K blocks; each lane streams 16 contiguous
//    bytes of one row per 64-K step with ld.global.nc (L1 bypass, L2
//    evict-first), a batch of JB steps in flight before any is consumed;
//  * the inner products run on the tensor cores as FP8 MMAs
//    (mma.sync m16n8k32 e4m3 x e4m3 -> f32): the weights are the B operand
//    exactly as stored; x is the A operand, split in two E4M3 terms, hi in
//    A rows 0-7 and lo in rows 8-15, so one MMA yields both partial sums; a
//    fixed permutation of K inside each 32-K step makes one 16-byte load per
//    lane exactly the lane's B fragments of two MMAs, and one 16-byte shared
//    load exactly its A fragment of one;
//  * x is staged once per CTA in shared memory as E4M3 pairs per 128-K
//    block, x * 2^e = hi + lo / 32, with e chosen so that the block's largest
//    magnitude lands in [2^7, 2^8): hi + lo / 32 equals the BF16 value
//    exactly for every element within 2^-14 of that maximum and to within
//    2^-15 absolute (2^-22 of the maximum) below it.  The hi and lo rows of
//    the MMA result are combined in FP32 and the block scale times 2^-e is
//    applied once per 128-K block;
//  * when a launch has fewer tiles than resident warps, the warps of a CTA
//    split K and add their partial sums through shared memory;
//  * the first batch of weight loads and a look-ahead L2 prefetch of the next
//    launch's weights are issued before griddepcontrol.wait.
//
// Products are exact (E4M3 x E4M3) and sums are FP32, as in the reference;
// the summation order and the split of x are the only differences.
#pragma once

#include "common.cuh"
#include "p2p.cuh"

namespace qwen {

constexpr int GEMV_MAX_SEG = 6;
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
#ifndef GEMV_CTAS_PER_SM
#define GEMV_CTAS_PER_SM 3     // resident CTAs per SM
#endif
#ifndef GEMV_RING_BYTES
#define GEMV_RING_BYTES 8192   // per-warp cp.async ring (2 stages of 4 KB)
#endif
constexpr int GEMV_NORM_REG_BLOCKS = 3;  // RMSNorm weights held in registers for K <= 3072
constexpr int GEMV_TILE = 8;  // weight rows per warp work unit (the N of one MMA)

enum GemvEpi : int {
  EPI_STORE = 0,      // y[r] = bf16(v)
  EPI_RESID = 1,      // y[r] = bf16(res[r] + bf16(v)); y2 (optional) = bf16(v)
  EPI_SILU_PAIR = 2,  // y[r] = bf16(silu(g) * u) from FP32 g, u; y2/y3 (optional) = bf16(g), bf16(u)
  EPI_ARGMAX = 3,     // running argmax of bf16(v); y (optional) = bf16 logits
  EPI_CONV = 4,       // y[r] = bf16(silu(bf16(conv(state[r,1:], bf16(v))))); state updated
  EPI_GATE_G = 5,     // y(f32)[r] = -exp(A_log[r]) * softplus(bf16(v) + dt_bias[r])
  EPI_GATE_BETA = 6,  // y[r] = bf16(sigmoid(bf16(v)))
  EPI_F32 = 7,        // y(f32)[r] = v (partial sums of a K-sliced tensor-parallel GEMV)
  EPI_F32_P2P = 8,    // v into slot [rank] of every rank's exchange buffer (aux0 = P2PTable*)
  EPI_SLICES = 9,     // y(f32)[slice * n + r] = this K slice's partial v; y2 (int*) = slice count
                      // (tensor-core kernel, one segment: the next launch adds the slices)
  EPI_SILU = 10,      // y[r] = bf16(silu(bf16(v))) (step kernel: the GatedDeltaNet output gate)
};

enum GemvPro : int {
  PRO_NONE = 0,         // x as given
  PRO_RMSNORM = 1,      // x <- bf16(x * rsqrt(mean(x^2) + eps) * (1 + w))
  PRO_ADD_RMSNORM = 2,  // h2 <- bf16(x + x2) (stored by CTA 0); x <- rmsnorm(h2)
  PRO_P2P_RMSNORM = 3,  // h2 <- bf16(x + bf16(sum of the ranks' partials, p2p)) (stored by CTA 0); x <- rmsnorm(h2)
  PRO_GATED_NORM = 4,   // per 128-block (one GatedDeltaNet head): x <- RMSNormGated(x, z) (gz, gw, eps)
  PRO_SLICES_RMSNORM = 5,  // h2 <- bf16(x + bf16(sum of the previous launch's EPI_SLICES rows in slice
                           // order)) (stored by CTA 0); x <- rmsnorm(h2)
};

struct GemvSeg {
  const uint8_t* w;   // [n, K] E4M3, row-major
  const void* s;      // scales (reference K_blk encoding)
  const uint8_t* w2;  // EPI_SILU_PAIR: up matrix
  const void* s2;
  void* y;
  void* y2;
  void* y3;
  const void* aux0;   // RESID: residual bf16 [n]; CONV: conv weight bf16 [n, cw]; GATE_G: A_log f32 [n]
  const void* aux1;   // GATE_G: dt_bias f32 [n]
  void* aux2;         // CONV: conv state bf16 [n, cw], updated in place
  int n;
  int kblk;
  int epi;
  int unit0;          // first work unit of this segment (filled by the planner)
  int row_offset;     // ARGMAX: global index of row 0 (vocabulary shard offset)
  int cw;             // CONV: kernel width (<= 8)
};

struct GemvArgs {
  const bf16* x;
  const bf16* x2;
  const float* norm_w;
  bf16* xn_out;        // optional: normalised x (CTA 0)
  bf16* h2_out;        // PRO_ADD_RMSNORM: x + x2 (CTA 0)
  const long long* x_row;  // optional: x <- x + (*x_row) * K (embedding row gather)
  float eps;
  int K;
  int pro;
  int nseg;
  int nunits;          // total work units (filled by the planner)
  int nslice;          // K split: warps sharing one unit (streaming kernel) or CTAs (tensor-core kernel)
  int stages;          // tensor-core kernel: weight stages in the shared-memory ring
  unsigned long long* am_ws;       // ARGMAX workspace {key, count}: zero before first use, left zeroed
  unsigned long long* am_key_out;  // optional: final packed key
  long long* am_token_out;         // optional: final token id
  int* pos_inc;                    // optional: ++*pos_inc by the argmax finaliser
  L2Prefetch pf;                   // weights of the next launch, pulled into L2 while this one runs
  const P2PTable* p2p;             // PRO_P2P_RMSNORM: the tensor-parallel exchange of this round
  const bf16* gz;                  // PRO_GATED_NORM: gate z, same layout as x
  const bf16* gw;                  // PRO_GATED_NORM: norm weight of one 128-wide head
  const float* sl_buf;             // PRO_SLICES_RMSNORM: the slices [count][sl_n]
  const int* sl_count;             // PRO_SLICES_RMSNORM: their count (written by the producing launch)
  int sl_n;                        // PRO_SLICES_RMSNORM: row stride of sl_buf (== K)
  int sl_max;                      // EPI_SLICES / PRO_SLICES_RMSNORM: slices the buffer holds
  GemvSeg seg[GEMV_MAX_SEG];
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

// Shared memory of the MMA kernel: x (BF16 staging, then in place the E4M3
// hi / lo words, 256 bytes per 128-K block: elements 4l..4l+3 of the block
// as {hi word, lo word} at byte 8l, which is where they were staged), the
// per-128-block 2^-e factors, slice partials, a small reduction area and one
// cp.async ring per warp.
struct GemvSmem {
  int x8_off, xinv_off, red_off, misc_off, ring_off, total;
};
__host__ __device__ inline GemvSmem gemv_smem_layout(int K) {
  GemvSmem L;
  const int nb = (K + 127) / 128;
  L.x8_off = 0;
  L.xinv_off = align_up(2 * K, 16);
  L.red_off = align_up(L.xinv_off + 4 * nb, 16);
  L.misc_off = L.red_off + 4 * 2 * GEMV_WARPS * GEMV_TILE * 2;
  L.ring_off = L.misc_off + 8 * 64;
  L.total = L.ring_off + GEMV_WARPS * GEMV_RING_BYTES;
  return L;
}

// ---------------------------------------------------------------------------
// Scales
// ---------------------------------------------------------------------------
__device__ __forceinline__ int scale_index(int kblk, int row, int kb) {
  if (kblk < 0) return row * (-kblk) + kb;
  if (kblk == 1) return row;
  return (row >> 7) * kblk + kb;
}
template <typename ST>
__device__ __forceinline__ float load_scale(const void* s, int idx) {
  if constexpr (sizeof(ST) == 4) {
    return __ldg(reinterpret_cast<const float*>(s) + idx);
  } else {
    unsigned short b = __ldg(reinterpret_cast<const unsigned short*>(s) + idx);
    return __uint_as_float(((uint32_t)b) << 16);
  }
}

// ---------------------------------------------------------------------------
// Epilogues
// ---------------------------------------------------------------------------
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Returns the updated running argmax key (EPI_ARGMAX).
__device__ __noinline__ unsigned long long gemv_epilogue(const GemvSeg& sg, int r, float v, float v2,
                                                         unsigned long long am_best) {
  switch (sg.epi) {
    case EPI_STORE:
      reinterpret_cast<bf16*>(sg.y)[r] = f2bf(v);
      break;
    case EPI_RESID: {
      bf16 d = f2bf(v);
      if (sg.y2) reinterpret_cast<bf16*>(sg.y2)[r] = d;
      const float res = bf2f(reinterpret_cast<const bf16*>(sg.aux0)[r]);
      reinterpret_cast<bf16*>(sg.y)[r] = f2bf(res + bf2f(d));
    } break;
    case EPI_SILU_PAIR:
      if (sg.y2) reinterpret_cast<bf16*>(sg.y2)[r] = f2bf(v);
      if (sg.y3) reinterpret_cast<bf16*>(sg.y3)[r] = f2bf(v2);
      reinterpret_cast<bf16*>(sg.y)[r] = f2bf(silu_f(v) * v2);
      break;
    case EPI_ARGMAX: {
      bf16 l = f2bf(v);
      if (sg.y) reinterpret_cast<bf16*>(sg.y)[r] = l;
      unsigned long long k = argmax_key(l, (uint32_t)(sg.row_offset + r));
      am_best = k > am_best ? k : am_best;
    } break;
    case EPI_CONV: {
      bf16 xb = f2bf(v);
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
      float c = bfround(acc);
      reinterpret_cast<bf16*>(sg.y)[r] = f2bf(silu_f(c));
    } break;
    case EPI_GATE_G: {
      float a = bfround(v) + reinterpret_cast<const float*>(sg.aux1)[r];
      float sp = a > 20.0f ? a : log1pf(expf(a));
      reinterpret_cast<float*>(sg.y)[r] = -expf(reinterpret_cast<const float*>(sg.aux0)[r]) * sp;
    } break;
    case EPI_GATE_BETA: {
      float b = bfround(v);
      reinterpret_cast<bf16*>(sg.y)[r] = f2bf(1.0f / (1.0f + expf(-b)));
    } break;
    case EPI_F32:
    case EPI_SLICES:  // slice 0 of an unsplit launch
      reinterpret_cast<float*>(sg.y)[r] = v;
      break;
    case EPI_F32_P2P:
      p2p_store_row(static_cast<const P2PTable*>(sg.aux0), r, v);
      break;
    default:
      break;
  }
  return am_best;
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int o) {
  uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
  lo = __shfl_xor_sync(0xffffffffu, lo, o);
  hi = __shfl_xor_sync(0xffffffffu, hi, o);
  return ((unsigned long long)hi << 32) | lo;
}

// CTA-wide max of am_best followed by the cross-CTA argmax and its
// finalisation by the last CTA to arrive.  `misc` holds >= 32 u64 of smem.
// All threads of the CTA must call it (uses __syncthreads).
__device__ __forceinline__ void argmax_finish(const GemvArgs& a, unsigned long long am_best,
                                              unsigned long long* misc) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = shfl_xor_u64(am_best, o);
    am_best = other > am_best ? other : am_best;
  }
  if (lane == 0) misc[warp] = am_best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long best = 0;
    const int nw = blockDim.x >> 5;
    for (int i = 0; i < nw; ++i) best = misc[i] > best ? misc[i] : best;
    unsigned long long* ws = a.am_ws;
    if (best) atomicMax(ws, best);
    __threadfence();
    unsigned int* cnt = reinterpret_cast<unsigned int*>(ws + 1);
    unsigned int prev = atomicAdd(cnt, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence();
      unsigned long long key = atomicAdd(ws, 0ull);
      if (a.am_key_out) *a.am_key_out = key;
      if (a.am_token_out) *a.am_token_out = (long long)(0xffffffffu - (uint32_t)(key & 0xffffffffu));
      if (a.pos_inc) *a.pos_inc += 1;
      *ws = 0ull;
      *cnt = 0u;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// Prologue: build x (bf16) in shared memory; all `nthr` threads of the
// calling group take part (they are synchronised with named barrier `bar`).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void gemv_prologue(const GemvArgs& a, bf16* xs, float* red32, int tid, int nthr,
                                              int bar) {
  const int K = a.K;
  const bf16* xin = a.x;
  if (a.x_row) xin += (size_t)(*a.x_row) * K;
  float ss = 0.f;
  for (int i = tid; i < K; i += nthr) {
    float v = bf2f(xin[i]);
    if (a.pro == PRO_ADD_RMSNORM) {
      bf16 h = f2bf(v + bf2f(a.x2[i]));
      if (blockIdx.x == 0 && a.h2_out) a.h2_out[i] = h;
      v = bf2f(h);
    }
    xs[i] = f2bf(v);
    ss = fmaf(v, v, ss);
  }
  if (a.pro == PRO_NONE) {
    named_bar(bar, nthr);
    return;
  }
  ss = warp_sum(ss);
  const int w = tid >> 5, nw = nthr >> 5;
  if ((tid & 31) == 0) red32[w] = ss;
  named_bar(bar, nthr);
  float tot = 0.f;
  for (int i = 0; i < nw; ++i) tot += red32[i];
  const float rms = rsqrtf(tot / (float)K + a.eps);
  for (int i = tid; i < K; i += nthr) {
    float v = bf2f(xs[i]);
    bf16 o = f2bf(v * rms * (1.0f + a.norm_w[i]));
    xs[i] = o;
    if (blockIdx.x == 0 && a.xn_out) a.xn_out[i] = o;
  }
  named_bar(bar, nthr);
}

// RMSNorm weights of the first GEMV_NORM_REG_BLOCKS 128-blocks a warp
// normalises (static data: loaded before griddepcontrol.wait).
struct NormRegs {
  float4 w[GEMV_NORM_REG_BLOCKS];
};
__device__ __forceinline__ void gemv_norm_preload(const GemvArgs& a, NormRegs& nr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nb = a.K >> 7;
#pragma unroll
  for (int i = 0; i < GEMV_NORM_REG_BLOCKS; ++i) {
    const int b = warp + i * GEMV_WARPS;
    nr.w[i] = (a.pro != PRO_NONE && b < nb) ? __ldg(reinterpret_cast<const float4*>(a.norm_w + b * 128) + lane)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Kernel prologue (K % 128 == 0), two passes and two barriers:
//  1. all threads, 8 elements each: x (+ x2) -> BF16 into the x8 area, sum
//     of squares for RMSNorm;
//  2. one warp per 128-wide block, 4 elements per lane, in place: RMSNorm(1+w)
//     (BF16 rounded), exponent e with max|x| * 2^e in [2^7, 2^8), x * 2^e
//     split into E4M3 hi + lo / 32 (hi = RN(x * 2^e), lo = RN(32 (x * 2^e -
//     hi))) and 2^-e per block (xinv).  Each lane overwrites exactly the 8 bytes it
//     staged: {hi word, lo word} of its 4 elements.
__device__ __forceinline__ void gemv_x_prepare(const GemvArgs& a, const NormRegs& nr, uint8_t* x8raw, float* xinv,
                                               float* red32) {
  const int K = a.K;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bf16* xin = a.x;
  if (a.x_row) xin += (size_t)(*a.x_row) * K;
  uint4* xs8 = reinterpret_cast<uint4*>(x8raw);
  float ss = 0.f;
  for (int i = tid; i < (K >> 3); i += GEMV_THREADS) {
    uint4 v = __ldg(reinterpret_cast<const uint4*>(xin) + i);
    if (a.pro == PRO_ADD_RMSNORM) {
      const uint4 r = __ldg(reinterpret_cast<const uint4*>(a.x2) + i);
      uint32_t* vw = reinterpret_cast<uint32_t*>(&v);
      const uint32_t* rw = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = bf2x_to_f2(vw[t]), g = bf2x_to_f2(rw[t]);
        const __nv_bfloat162 h = __floats2bfloat162_rn(f.x + g.x, f.y + g.y);
        vw[t] = *reinterpret_cast<const uint32_t*>(&h);
      }
      if (blockIdx.x == 0 && a.h2_out) reinterpret_cast<uint4*>(a.h2_out)[i] = v;
    }
    const uint32_t* vw = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 f = bf2x_to_f2(vw[t]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
    xs8[i] = v;
  }
  ss = warp_sum(ss);
  if (lane == 0) red32[warp] = ss;
  __syncthreads();
  float rms = 1.f;
  if (a.pro != PRO_NONE) {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < GEMV_WARPS; ++i) tot += red32[i];
    rms = rsqrtf(tot / (float)K + a.eps);
  }
  const int nb = K >> 7;
  for (int b = warp, i = 0; b < nb; b += GEMV_WARPS, ++i) {
    const uint2 raw = reinterpret_cast<const uint2*>(x8raw)[b * 32 + lane];
    const float2 v01 = bf2x_to_f2(raw.x), v23 = bf2x_to_f2(raw.y);
    float v[4] = {v01.x, v01.y, v23.x, v23.y};
    if (a.pro != PRO_NONE) {
      float4 w;
      if (i < GEMV_NORM_REG_BLOCKS) {
        w = nr.w[0];
#pragma unroll
        for (int j = 1; j < GEMV_NORM_REG_BLOCKS; ++j)
          if (i == j) w = nr.w[j];
      } else {
        w = __ldg(reinterpret_cast<const float4*>(a.norm_w + b * 128) + lane);
      }
      const float wv[4] = {w.x, w.y, w.z, w.w};
      bf16 o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        o[t] = f2bf(v[t] * rms * (1.0f + wv[t]));
        v[t] = bf2f(o[t]);
      }
      if (blockIdx.x == 0 && a.xn_out) {
        uint2 ov;
        ov.x = (uint32_t)__bfloat16_as_ushort(o[0]) | ((uint32_t)__bfloat16_as_ushort(o[1]) << 16);
        ov.y = (uint32_t)__bfloat16_as_ushort(o[2]) | ((uint32_t)__bfloat16_as_ushort(o[3]) << 16);
        reinterpret_cast<uint2*>(a.xn_out)[b * 32 + lane] = ov;
      }
    }
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    m = warp_max(m);
    // m = 1.f * 2^(ebits - 127): e = 134 - ebits puts m * 2^e in [2^7, 2^8)
    // (denormal m: e = 100, far below anything that matters)
    const int ebits = (int)((__float_as_uint(m) >> 23) & 0xffu);
    int e = m > 0.f ? (ebits == 0 ? 100 : 134 - ebits) : 0;
    e = e < -100 ? -100 : (e > 100 ? 100 : e);
    const float sc = exp2i(e);
    float xs[4], hi[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) xs[t] = v[t] * sc;
    const uint32_t h01 = f32x2_to_e4m3x2(xs[0], xs[1]), h23 = f32x2_to_e4m3x2(xs[2], xs[3]);
    const float2 g01 = h2u_to_f2(e4m3x2_to_f16x2(h01)), g23 = h2u_to_f2(e4m3x2_to_f16x2(h23));
    hi[0] = g01.x; hi[1] = g01.y; hi[2] = g23.x; hi[3] = g23.y;
    // lo carries 32 * (x * 2^e - hi): |x * 2^e - hi| <= 8, so 32x stays below 448
    const uint32_t l01 = f32x2_to_e4m3x2((xs[0] - hi[0]) * 32.f, (xs[1] - hi[1]) * 32.f);
    const uint32_t l23 = f32x2_to_e4m3x2((xs[2] - hi[2]) * 32.f, (xs[3] - hi[3]) * 32.f);
    reinterpret_cast<uint2*>(x8raw)[b * 32 + lane] = make_uint2(h01 | (h23 << 16), l01 | (l23 << 16));
    if (lane == 0) xinv[b] = exp2i(-e);
  }
  __syncthreads();
}

// D (16x8, f32) (+)= A (16x32 E4M3, row) * B (32x8 E4M3, col): one FP8
// tensor-core MMA; a = {a0, a1, a2, a3} is the lane's A fragment as loaded.
// The _zc form starts from a zero accumulator.
__device__ __forceinline__ void mma_e4m3(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_e4m3_zc(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%10,%10,%10,%10};"
               : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
               : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ int gemv_find_seg(const GemvArgs& a, int u) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < GEMV_MAX_SEG; ++i)
    if (i < a.nseg && u >= a.seg[i].unit0) s = i;
  return s;
}

// One work unit: two 8-row tiles, p = 0, 1.  For a gate/up pair they are
// the same 8 rows of the gate and the up matrix; otherwise 16 consecutive
// rows of one matrix.  w[p] points at tile p's first row.
struct GemvTile {
  const uint8_t* w[2];
  int r0[2];     // output row of tile p's first row
  int nrows[2];  // valid rows in tile p (0..8)
  int seg;
};

template <bool PAIR>
__device__ __forceinline__ GemvTile gemv_tile(const GemvArgs& a, int u) {
  GemvTile T;
  T.seg = gemv_find_seg(a, u);
  const GemvSeg& sg = a.seg[T.seg];
  const int K = a.K;
  if (PAIR) {
    const int row0 = (u - sg.unit0) * GEMV_TILE;
    T.r0[0] = T.r0[1] = row0;
    T.nrows[0] = T.nrows[1] = min(GEMV_TILE, sg.n - row0);
    T.w[0] = sg.w + (size_t)row0 * K;
    T.w[1] = sg.w2 + (size_t)row0 * K;
  } else {
    const int row0 = (u - sg.unit0) * 2 * GEMV_TILE;
    T.r0[0] = row0;
    T.r0[1] = row0 + GEMV_TILE;
    T.nrows[0] = min(GEMV_TILE, sg.n - row0);
    T.nrows[1] = max(0, min(GEMV_TILE, sg.n - row0 - GEMV_TILE));
    T.w[0] = sg.w + (size_t)row0 * K;
    T.w[1] = T.nrows[1] > 0 ? T.w[0] + (size_t)GEMV_TILE * K : T.w[0];
  }
  return T;
}

// Block-mode scales of one unit for the 128-K blocks of a slice: lane l
// holds scale[row0 / 128, kb0 + l] of tile p (l < nkbs <= 32).  Both tiles of
// an unpaired unit lie in one 128-row block.
template <typename ST, bool PAIR>
__device__ __forceinline__ void gemv_unit_scales(const GemvArgs& a, int u, int kb0, int nkbs, float (&sc)[2]) {
  const int lane = threadIdx.x & 31;
  sc[0] = sc[1] = 0.f;
  if (u >= a.nunits || lane >= nkbs) return;
  const GemvSeg& sg = a.seg[gemv_find_seg(a, u)];
  const int row0 = (u - sg.unit0) * (PAIR ? GEMV_TILE : 2 * GEMV_TILE);
  const int idx = (row0 >> 7) * sg.kblk + kb0 + lane;
  sc[0] = load_scale<ST>(sg.s, idx);
  sc[1] = PAIR ? load_scale<ST>(sg.s2, idx) : sc[0];
}

// ---------------------------------------------------------------------------
// Tensor-core streaming GEMV over units of two 8-row tiles (block-mode
// scales only; the planner sends the other scale layouts to the generic
// kernel).  The CTA's warps form groups of S = a.nslice warps; a group works
// on one unit at a time and its warps split the unit's 128-K blocks (at most
// 32 per warp), reducing through shared memory.  Each warp is its own
// producer and consumer: a stage is two 128-K blocks of the unit's 16 rows
// (4 KB), copied with cp.async so that every instruction reads 256
// contiguous bytes of each of two rows, and placed in shared memory where
// each lane finds its MMA fragments with one 16-byte load; the warp keeps
// R - 1 stages of loads in flight ahead of the stage it multiplies.
// ---------------------------------------------------------------------------
template <typename ST, bool PAIR>
__global__ void __launch_bounds__(GEMV_THREADS, GEMV_CTAS_PER_SM) gemv_mma_kernel(const __grid_constant__ GemvArgs a) {
  constexpr int STAGE = 4096;  // 2 K-blocks x 2 tiles x 8 rows x 128 B
  constexpr int R = GEMV_RING_BYTES / STAGE;
  static_assert(R >= 2, "ring too small");
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K;
  const int nkb = K >> 7;  // K % 128 == 0 on this path
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;  // MMA groupID / thread-in-group
  const GemvSmem L = gemv_smem_layout(K);
  const uint32_t x8 = smem_u32(smem + L.x8_off) + tq * 32;
  const float* xinv = reinterpret_cast<const float*>(smem + L.xinv_off);
  float* red = reinterpret_cast<float*>(smem + L.red_off);  // [2][GEMV_WARPS][GEMV_TILE][2]
  unsigned long long* misc = reinterpret_cast<unsigned long long*>(smem + L.misc_off);
  const uint32_t ring = smem_u32(smem + L.ring_off) + warp * GEMV_RING_BYTES;

  const int S = a.nslice;
  const int G = GEMV_WARPS / S;
  const int g = warp / S, sl = warp % S;
  const int kb0 = (sl * nkb) / S, kb1 = ((sl + 1) * nkb) / S;
  const int nkbs = kb1 - kb0;          // 128-K blocks of this slice (1..32)
  const int nst = (nkbs + 1) >> 1;     // stages of this slice
  const int ngroups = gridDim.x * G;
  const uint64_t pol = l2_policy_evict_first();  // weights are read once per step

  // Producer.  Copy instruction i (0..7) of a stage covers unit rows 2i and
  // 2i+1, i.e. tile p = i / 4, rows 2 (i % 4) + lane / 16; lane moves bytes
  // 16 (lane % 16) .. +15 of the stage's 256-byte row piece, which are
  // K-block bi, half h, MMA column group tq' of that row.  Its shared-memory
  // slot is the one lane (row, tq') reads for (bi, tile, h).
  const int prow = lane >> 4, pbi = (lane >> 3) & 1;
  const uint32_t pdst = ring + pbi * 2048 + ((lane >> 2) & 1) * 512 + (prow * 4 + (lane & 3)) * 16;
  const size_t K2 = (size_t)2 * K;
  int up = blockIdx.x * G + g, qp = 0, ps = 0;
  const uint8_t* pw[2];
  int pn[2];
  auto producer_unit = [&]() {
    const GemvTile T = gemv_tile<PAIR>(a, up);
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      pn[p] = T.nrows[p];
      pw[p] = T.w[p] + (size_t)prow * K + (size_t)kb0 * 128 + (lane & 15) * 16;
    }
  };
  if (up < a.nunits) producer_unit();
  auto produce = [&]() {
    if (up < a.nunits) {
      const uint32_t dst = pdst + ps * STAGE;
      if (pn[0] == GEMV_TILE && pn[1] == GEMV_TILE && 2 * qp + 1 < nkbs) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const uint8_t* src = pw[p];
#pragma unroll
          for (int i = 0; i < 4; ++i) cp_async16(dst + p * 1024 + i * 128, src + i * K2, pol);
        }
      } else {
        // ragged unit (rows past the segment end) or a single-block stage
        const bool kok = 2 * qp + pbi < nkbs;
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const bool ok = kok && 2 * i + prow < pn[p];
            cp_async16(dst + p * 1024 + i * 128, ok ? pw[p] + i * K2 : pw[0], ok, pol);
          }
      }
      pw[0] += 256;
      pw[1] += 256;
      if (++qp == nst) {
        qp = 0;
        up += ngroups;
        if (up < a.nunits) producer_unit();
      }
    }
    cp_async_commit();
    ps = ps + 1 == R ? 0 : ps + 1;
  };

  // Weights and scales are static: start streaming before waiting on the
  // previous kernel.
  if (threadIdx.x == 0) pdl_trigger();
#pragma unroll 1
  for (int i = 0; i < R - 1; ++i) produce();
  int uc = blockIdx.x * G + g, qc = 0, cs = 0;
  float sc[2], sc_next[2];
  gemv_unit_scales<ST, PAIR>(a, uc, kb0, nkbs, sc);
  gemv_unit_scales<ST, PAIR>(a, uc + ngroups, kb0, nkbs, sc_next);
  NormRegs nr;
  gemv_norm_preload(a, nr);
  if (warp == 0) l2_prefetch_share(a.pf, lane);
  pdl_wait();
  gemv_x_prepare(a, nr, smem + L.x8_off, const_cast<float*>(xinv), reinterpret_cast<float*>(misc));

  unsigned long long am_best = 0ull;
  float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
  int parity = 0;

  // One 128-K block of both tiles: 8 MMAs, then promotion with the block
  // scale and 2^-e of x.  Rows 0-7 of D carry the hi products, rows 8-15 the
  // lo products (x 32).
  auto consume_block = [&](uint32_t src, int kbl) {
    const int kb = kb0 + kbl;
    float d[2][2][4];  // [tile][MMA j of a 32-K pair][fragment]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // A fragments of this lane for K offset kb*128 + 64h + 16tq + 8j:
      // {hi, lo, hi, lo} words, one 16-byte load per j
      const uint4 xa0 = lds_v4(x8 + kb * 256 + h * 128);
      const uint4 xa1 = lds_v4(x8 + kb * 256 + h * 128 + 16);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const uint4 wv = lds_v4(src + p * 1024 + h * 512);
        if (h == 0) {
          mma_e4m3_zc(d[p][0], xa0, wv.x, wv.y);
          mma_e4m3_zc(d[p][1], xa1, wv.z, wv.w);
        } else {
          mma_e4m3(d[p][0], xa0, wv.x, wv.y);
          mma_e4m3(d[p][1], xa1, wv.z, wv.w);
        }
      }
    }
    const float f = xinv[kb];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float sf = __shfl_sync(0xffffffffu, sc[p], kbl) * f;
      const float v0 = (d[p][0][0] + d[p][1][0]) + (d[p][0][2] + d[p][1][2]) * 0.03125f;
      const float v1 = (d[p][0][1] + d[p][1][1]) + (d[p][0][3] + d[p][1][3]) * 0.03125f;
      acc[p][0] = fmaf(v0, sf, acc[p][0]);
      acc[p][1] = fmaf(v1, sf, acc[p][1]);
    }
  };

#pragma unroll 1
  while (uc < a.nunits) {
    __syncwarp();  // every lane is done reading the slot that produce() refills
    produce();
    cp_async_wait<R - 1>();
    __syncwarp();  // the stage was copied by other lanes of this warp
    const uint32_t src = ring + cs * STAGE + lane * 16;
    cs = cs + 1 == R ? 0 : cs + 1;
    consume_block(src, 2 * qc);
    if (2 * qc + 1 < nkbs) consume_block(src + 2048, 2 * qc + 1);
    if (++qc == nst) {
      // unit finished: lanes 0..3 hold rows 2*tq, 2*tq+1 of both tiles
      const GemvTile T = gemv_tile<PAIR>(a, uc);
      const GemvSeg& sg = a.seg[T.seg];
      bool lead = true;
      if (S > 1) {
        float* rb = red + (parity * GEMV_WARPS + warp) * GEMV_TILE * 2;
        if (gq == 0) {
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            rb[(2 * tq) * 2 + p] = acc[p][0];
            rb[(2 * tq + 1) * 2 + p] = acc[p][1];
          }
        }
        named_bar(2 + g, S * 32);
        lead = sl == 0;
        if (lead && gq == 0) {
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            float t0 = 0.f, t1 = 0.f;
            for (int q2 = 0; q2 < S; ++q2) {
              const float* ob = red + (parity * GEMV_WARPS + g * S + q2) * GEMV_TILE * 2;
              t0 += ob[(2 * tq) * 2 + p];
              t1 += ob[(2 * tq + 1) * 2 + p];
            }
            acc[p][0] = t0;
            acc[p][1] = t1;
          }
        }
        parity ^= 1;
      }
      if (lead && gq == 0) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int r = 2 * tq + i;
          if (PAIR) {
            if (r < T.nrows[0]) am_best = gemv_epilogue(sg, T.r0[0] + r, acc[0][i], acc[1][i], am_best);
          } else {
#pragma unroll
            for (int p = 0; p < 2; ++p)
              if (r < T.nrows[p]) am_best = gemv_epilogue(sg, T.r0[p] + r, acc[p][i], 0.f, am_best);
          }
        }
      }
      acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.f;
      qc = 0;
      uc += ngroups;
      sc[0] = sc_next[0];
      sc[1] = sc_next[1];
      gemv_unit_scales<ST, PAIR>(a, uc + ngroups, kb0, nkbs, sc_next);
    }
  }
  cp_async_wait<0>();

  if (a.am_ws) argmax_finish(a, am_best, misc + 32);
}

// ---------------------------------------------------------------------------
// Generic fallback: one warp per output row, weights read straight from global
// memory in 4-byte words (any K % 8 == 0, rows 4-byte aligned), FP32 x in
// shared memory.  Used for shapes the row-streaming kernel does not cover.
// ---------------------------------------------------------------------------
// Direct-load GEMV for plain-x launches (the reference ABI's
// launch_gemv_v4_extern and its grouped forms): one warp per output row, the
// whole row's weights loaded at once (lane l holds K bytes [16 l + 512 j,
// +16) for j < J, K = 512 J) before x is even read, so a launch puts every
// weight byte it needs in flight in one wave and pays one memory latency.
// The weights are static, so the loads are issued before
// griddepcontrol.wait; x (BF16) is then staged in shared memory as FP32.
// Per lane and j the 16 products are summed in FP32 and scaled once by the
// row's scale of that 128-wide K block; the warp sum is the row's value.
// Restates gemv_v4_kernel (fused_kernels.cu:91-151) with the same FP32
// accumulation (a different summation order).
template <typename ST, int J>
__global__ void __launch_bounds__(256) gemv_direct_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int K = 512 * J;
  float* xf = reinterpret_cast<float*>(smem);
  unsigned long long* misc = reinterpret_cast<unsigned long long*>(smem + 4 * K);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  int total = 0;
  for (int s = 0; s < a.nseg; ++s) total += a.seg[s].n;
  int gr = blockIdx.x * nw + warp;
  // the first row's weights and scales before anything else
  uint4 wv[J];
  float sc[J];
  auto issue = [&](int row_g, int& si, int& r) {
    si = 0;
    r = row_g;
    while (r >= a.seg[si].n) {
      r -= a.seg[si].n;
      ++si;
    }
    const GemvSeg& sg = a.seg[si];
    const uint8_t* wr = sg.w + (size_t)r * K + lane * 16;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      wv[j] = ld_nc_na_v4(wr + 512 * j);
      sc[j] = load_scale<ST>(sg.s, scale_index(sg.kblk, r, (lane * 16 + 512 * j) >> 7));
    }
  };
  int si = 0, r = 0;
  if (gr < total) issue(gr, si, r);
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  {  // x: every load issued before any is used (one round trip)
    constexpr int XI = (K / 8 + 255) / 256;
    uint4 xv[XI];
#pragma unroll
    for (int t = 0; t < XI; ++t) {
      const int i = threadIdx.x + 256 * t;
      if (i < K / 8) xv[t] = __ldg(reinterpret_cast<const uint4*>(a.x) + i);
    }
    // lane-interleaved: the 4 elements x[512 j + 16 l + 4 q, +4) live in
    // float4 slot (4 j + q) * 32 + l, so lane l's reads below are
    // consecutive 16-byte words across the warp (no bank conflicts)
    float4* xf4 = reinterpret_cast<float4*>(xf);
#pragma unroll
    for (int t = 0; t < XI; ++t) {
      const int i = threadIdx.x + 256 * t;
      if (i >= K / 8) continue;
      const uint32_t* vw = reinterpret_cast<const uint32_t*>(&xv[t]);
      const int k0 = 8 * i, j = k0 >> 9, l = (k0 & 511) >> 4, q = (k0 & 15) >> 2;  // q even
      const float2 f0 = bf2x_to_f2(vw[0]), f1 = bf2x_to_f2(vw[1]), f2 = bf2x_to_f2(vw[2]), f3 = bf2x_to_f2(vw[3]);
      xf4[(4 * j + q) * 32 + l] = make_float4(f0.x, f0.y, f1.x, f1.y);
      xf4[(4 * j + q + 1) * 32 + l] = make_float4(f2.x, f2.y, f3.x, f3.y);
    }
  }
  __syncthreads();
  unsigned long long am_best = 0ull;
  while (gr < total) {
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float4* x4 = reinterpret_cast<const float4*>(xf) + (4 * j) * 32 + lane;
      const uint32_t* wq = reinterpret_cast<const uint32_t*>(&wv[j]);
      float p = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f0 = h2u_to_f2(e4m3x2_to_f16x2(wq[q])), f1 = h2u_to_f2(e4m3x2_to_f16x2(wq[q] >> 16));
        const float4 xv = x4[q * 32];
        p = fmaf(xv.x, f0.x, p);
        p = fmaf(xv.y, f0.y, p);
        p = fmaf(xv.z, f1.x, p);
        p = fmaf(xv.w, f1.y, p);
      }
      sum = fmaf(p, sc[j], sum);
    }
    sum = warp_sum(sum);
    const GemvSeg& sg = a.seg[si];
    const int rr = r;
    gr += gridDim.x * nw;
    if (gr < total) issue(gr, si, r);  // the next row's loads go out before this row's store
    if (lane == 0) am_best = gemv_epilogue(sg, rr, sum, 0.f, am_best);
  }
  if (a.am_ws) argmax_finish(a, am_best, misc + 32);
}

template <typename ST>
__global__ void __launch_bounds__(256) gemv_simple_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K;
  bf16* xs = reinterpret_cast<bf16*>(smem);
  float* xf = reinterpret_cast<float*>(smem + align_up(2 * K, 16));
  unsigned long long* misc = reinterpret_cast<unsigned long long*>(smem + align_up(2 * K, 16) + 4 * K);
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  gemv_prologue(a, xs, reinterpret_cast<float*>(misc), threadIdx.x, blockDim.x, 1);
  for (int i = threadIdx.x; i < K; i += blockDim.x) xf[i] = bf2f(xs[i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  unsigned long long am_best = 0ull;
  int total = 0;
  for (int s = 0; s < a.nseg; ++s) total += a.seg[s].n;
  for (int gr = blockIdx.x * nw + warp; gr < total; gr += gridDim.x * nw) {
    int si = 0, r = gr;
    while (r >= a.seg[si].n) { r -= a.seg[si].n; ++si; }
    const GemvSeg& sg = a.seg[si];
    const bool paired = sg.epi == EPI_SILU_PAIR;
    float acc[2] = {0.f, 0.f};
    for (int m = 0; m < (paired ? 2 : 1); ++m) {
      const uint8_t* wr = (m ? sg.w2 : sg.w) + (size_t)r * K;
      const void* sp = m ? sg.s2 : sg.s;
      float sum = 0.f;
      for (int k = lane * 8; k < K; k += 256) {
        const uint32_t p0 = __ldg(reinterpret_cast<const unsigned int*>(wr + k));
        const uint32_t p1 = __ldg(reinterpret_cast<const unsigned int*>(wr + k + 4));
        const float2 f0 = h2u_to_f2(e4m3x2_to_f16x2(p0)), f1 = h2u_to_f2(e4m3x2_to_f16x2(p0 >> 16));
        const float2 f2 = h2u_to_f2(e4m3x2_to_f16x2(p1)), f3 = h2u_to_f2(e4m3x2_to_f16x2(p1 >> 16));
        const float* x8 = xf + k;
        float p = x8[0] * f0.x + x8[1] * f0.y + x8[2] * f1.x + x8[3] * f1.y +
                  x8[4] * f2.x + x8[5] * f2.y + x8[6] * f3.x + x8[7] * f3.y;
        sum = fmaf(p, load_scale<ST>(sp, scale_index(sg.kblk, r, k >> 7)), sum);
      }
      acc[m] = warp_sum(sum);
    }
    if (lane == 0) am_best = gemv_epilogue(sg, r, acc[0], acc[1], am_best);
  }
  if (a.am_ws) argmax_finish(a, am_best, misc + 32);
}

}  // namespace qwen
