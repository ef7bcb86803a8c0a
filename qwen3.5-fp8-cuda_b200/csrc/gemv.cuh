// Block-scaled E4M3 x BF16 GEMV family for batch-1 decode on sm_100a.
//
// Computes, for every output row r of one or more weight segments,
//     v[r] = sum_kb scale[r, kb] * sum_{k in kb} x[k] * e4m3(W[r, k])
// with FP32 accumulation, then applies a fused epilogue (store, residual add,
// gate/up SiLU pairing, greedy argmax, GatedDeltaNet conv / gate math).
// Restates gemv_v4_kernel and its fused variants (fused_kernels.cu:91-479) as
// an HBM stream:
//
//  * rows are contiguous, so a tile of `rs` rows x K bytes is one contiguous
//    range; a producer warp moves tiles into a shared-memory ring with 1-D
//    bulk async copies (cp.async.bulk, no multicast) completing on mbarriers;
//  * consumer warps keep their slice of x in registers for the whole kernel
//    (loaded once) and read the weights from shared memory, 16 bytes a lane;
//  * the scale is applied once per 16-element chunk into FP32 accumulators;
//  * one CTA per SM, persistent over tiles; with programmatic dependent
//    launch the producer prefetches the first tiles before waiting on the
//    previous kernel, so weight streaming continues across kernel boundaries.
//
// Dot-product arithmetic: E4M3 pairs are widened exactly to f16x2 with
// cvt.rn.f16x2.e4m3x2.  x is held as f16 scaled by a power of two per
// 128-wide K block (exact for every element within 2^-32 of the block's
// largest magnitude), products are formed by the mixed-precision
// fma.rn.f32.f16, and the power of two is folded into the block scale.
#pragma once

#include "common.cuh"

namespace qwen {

constexpr int GEMV_MAX_SEG = 6;

enum GemvEpi : int {
  EPI_STORE = 0,      // y[r] = bf16(v)
  EPI_RESID = 1,      // y[r] = bf16(res[r] + bf16(v)); y2 (optional) = bf16(v)
  EPI_SILU_PAIR = 2,  // y[r] = bf16(silu(g) * u) from FP32 g, u; y2/y3 (optional) = bf16(g), bf16(u)
  EPI_ARGMAX = 3,     // running argmax of bf16(v); y (optional) = bf16 logits
  EPI_CONV = 4,       // y[r] = bf16(silu(bf16(conv(state[r,1:], bf16(v))))); state updated
  EPI_GATE_G = 5,     // y(f32)[r] = -exp(A_log[r]) * softplus(bf16(v) + dt_bias[r])
  EPI_GATE_BETA = 6,  // y[r] = bf16(sigmoid(bf16(v)))
};

enum GemvPro : int {
  PRO_NONE = 0,         // x as given
  PRO_RMSNORM = 1,      // x <- bf16(x * rsqrt(mean(x^2) + eps) * (1 + w))
  PRO_ADD_RMSNORM = 2,  // h2 <- bf16(x + x2) (stored by CTA 0); x <- rmsnorm(h2)
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
  int tile0;          // first tile index of this segment (filled by the planner)
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
  int ntiles;
  int rs, npart, nslice, nstages, stage_bytes;
  unsigned long long* am_ws;       // ARGMAX workspace {key, count}: zero before first use, left zeroed
  unsigned long long* am_key_out;  // optional: final packed key
  long long* am_token_out;         // optional: final token id
  int* pos_inc;                    // optional: ++*pos_inc by the argmax finaliser
  GemvSeg seg[GEMV_MAX_SEG];
};

// ---------------------------------------------------------------------------
// Shared-memory layout of the streaming kernel (host and device agree).
// ---------------------------------------------------------------------------
struct GemvSmem {
  int x_off, ex_off, red_off, misc_off, bar_off, total;
};
__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }
__host__ __device__ inline GemvSmem gemv_smem_layout(int K, int nstages, int stage_bytes, int rs, int npart) {
  GemvSmem L;
  L.x_off = nstages * stage_bytes;                       // stages first: 128-byte aligned base
  L.ex_off = align_up(L.x_off + 2 * K, 16);              // per-128-block x exponents (int32)
  L.red_off = align_up(L.ex_off + 4 * ((K + 127) / 128), 16);
  L.misc_off = align_up(L.red_off + 4 * nstages * rs * npart, 16);
  L.bar_off = align_up(L.misc_off + 8 * 64, 16);
  L.total = L.bar_off + 16 * nstages;
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

__device__ __noinline__ void gemv_epilogue(const GemvSeg& sg, int r, float v, float v2,
                                           unsigned long long& am_best) {
  switch (sg.epi) {
    case EPI_STORE:
      reinterpret_cast<bf16*>(sg.y)[r] = f2bf(v);
      break;
    case EPI_RESID: {
      bf16 d = f2bf(v);
      if (sg.y2) reinterpret_cast<bf16*>(sg.y2)[r] = d;
      float res = bf2f(reinterpret_cast<const bf16*>(sg.aux0)[r]);
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
    default:
      break;
  }
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

// Power-of-two exponent per 128-wide block of x so that max|x| * 2^e lies in
// [2^14, 2^15): x * 2^e is then exact in f16 for every element >= max * 2^-32.
__device__ __forceinline__ void gemv_x_exponents(const bf16* xs, int* ex, int K, int tid, int nthr, int bar) {
  const int nb = (K + 127) / 128;
  const int lane = tid & 31, w = tid >> 5, nw = nthr >> 5;
  for (int b = w; b < nb; b += nw) {
    float m = 0.f;
    for (int i = b * 128 + lane; i < min(K, b * 128 + 128); i += 32) m = fmaxf(m, fabsf(bf2f(xs[i])));
    m = warp_max(m);
    if (lane == 0) {
      int e = 0;
      if (m > 0.f) {
        int E;
        frexpf(m, &E);  // m = f * 2^E, f in [0.5, 1)
        e = 15 - E;
        e = e < -100 ? -100 : (e > 100 ? 100 : e);
      }
      ex[b] = e;
    }
  }
  named_bar(bar, nthr);
}

// Mixed-precision multiply-add of 16 E4M3 weights with 16 f16 x values.
__device__ __forceinline__ void dot16_f16(const uint4 w, const uint32_t (&xh)[8], float& a0, float& a1) {
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t h01 = e4m3x2_to_f16x2(ww[i]);
    const uint32_t h23 = e4m3x2_to_f16x2(ww[i] >> 16);
    asm("{\n .reg .b16 w0, w1, x0, x1;\n"
        " mov.b32 {w0, w1}, %2;\n mov.b32 {x0, x1}, %3;\n"
        " fma.rn.f32.f16 %0, w0, x0, %0;\n fma.rn.f32.f16 %1, w1, x1, %1;\n}\n"
        : "+f"(a0), "+f"(a1) : "r"(h01), "r"(xh[2 * i]));
    asm("{\n .reg .b16 w0, w1, x0, x1;\n"
        " mov.b32 {w0, w1}, %2;\n mov.b32 {x0, x1}, %3;\n"
        " fma.rn.f32.f16 %0, w0, x0, %0;\n fma.rn.f32.f16 %1, w1, x1, %1;\n}\n"
        : "+f"(a0), "+f"(a1) : "r"(h23), "r"(xh[2 * i + 1]));
  }
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ int gemv_find_seg(const GemvArgs& a, int t) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < GEMV_MAX_SEG; ++i)
    if (i < a.nseg && t >= a.seg[i].tile0) s = i;
  return s;
}

// ---------------------------------------------------------------------------
// Streaming kernel: NC consumer warps + 1 producer warp, J 16-byte chunks of
// each row per lane (K = 512 * J * nslice).
// ---------------------------------------------------------------------------
template <typename ST, int NC, int J>
__global__ void __launch_bounds__((NC + 1) * 32, 2) gemv_stream_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = a.K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = a.nstages, sb = a.stage_bytes, rs = a.rs, npart = a.npart, nslice = a.nslice;
  const GemvSmem L = gemv_smem_layout(K, ns, sb, rs, npart);
  bf16* xs = reinterpret_cast<bf16*>(smem + L.x_off);
  int* ex = reinterpret_cast<int*>(smem + L.ex_off);
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  unsigned long long* misc = reinterpret_cast<unsigned long long*>(smem + L.misc_off);
  const uint32_t bar0 = smem_u32(smem + L.bar_off);  // full[s] at bar0+8s, empty[s] at bar0+8(ns+s)
  const uint32_t stage0 = smem_u32(smem);

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(bar0 + 8 * s, 1);
      mbar_init(bar0 + 8 * (ns + s), NC);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_trigger();

  unsigned long long am_best = 0ull;

  if (warp == NC) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, ++it) {
        const int slot = it % ns;
        if (it >= ns) {
          if (!mbar_wait_bounded(bar0 + 8 * (ns + slot), ((it / ns) & 1) ^ 1)) {
            qwen_err_set(ERR_TIMEOUT_EMPTY);
            ok = false;
            break;
          }
        }
        const int si = gemv_find_seg(a, t);
        const GemvSeg& sg = a.seg[si];
        const int row0 = (t - sg.tile0) * rs;
        const int nrows = min(rs, sg.n - row0);
        const uint32_t bytes = (uint32_t)nrows * (uint32_t)K;
        const bool paired = sg.epi == EPI_SILU_PAIR;
        mbar_arrive_expect_tx(bar0 + 8 * slot, paired ? 2 * bytes : bytes);
        const uint32_t dst = stage0 + slot * sb;
        bulk_g2s(dst, sg.w + (size_t)row0 * K, bytes, bar0 + 8 * slot, pol);
        if (paired) bulk_g2s(dst + rs * K, sg.w2 + (size_t)row0 * K, bytes, bar0 + 8 * slot, pol);
      }
      // Drain: every issued copy must have landed before this thread leaves.
      const int issued = it;
      for (int j = issued - ns; j < issued; ++j) {
        if (j < 0) continue;
        if (!mbar_wait_bounded(bar0 + 8 * (j % ns), (j / ns) & 1)) {
          qwen_err_set(ERR_TIMEOUT_DRAIN);
          break;
        }
      }
      (void)ok;
    }
  } else {
    // ---------------- consumers ----------------
    const int ctid = threadIdx.x;  // 0 .. NC*32-1
    const int nthr = NC * 32;
    pdl_wait();
    gemv_prologue(a, xs, reinterpret_cast<float*>(misc), ctid, nthr, 1);
    gemv_x_exponents(xs, ex, K, ctid, nthr, 1);

    const int part = warp % npart;
    const int mat = part / nslice;
    const int slice = part % nslice;
    const int row_step = NC / npart;

    // x slice in registers as f16 (scaled per 128-block), chunk c_j = (slice*J + j)*32 + lane.
    uint32_t xh[J][8];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = (slice * J + j) * 32 + lane;
      const int e = ex[c >> 3];
      const uint4 raw = *reinterpret_cast<const uint4*>(xs + c * 16);
      const uint4 raw2 = *reinterpret_cast<const uint4*>(xs + c * 16 + 8);
      const uint32_t u[8] = {raw.x, raw.y, raw.z, raw.w, raw2.x, raw2.y, raw2.z, raw2.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 f = bf2x_to_f2(u[i]);
        xh[j][i] = pack_f16x2(ldexpf(f.x, e), ldexpf(f.y, e));
      }
    }

    // After a timed-out wait the warp stops computing but keeps taking part in
    // every barrier, so a fault degrades to an error code, never a hang.
    bool failed = false;
    int it = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, ++it) {
      const int slot = it % ns;
      if (!failed && !mbar_wait_bounded(bar0 + 8 * slot, (it / ns) & 1)) {
        qwen_err_set(ERR_TIMEOUT_FULL);
        failed = true;
      }
      const int si = gemv_find_seg(a, t);
      const GemvSeg& sg = a.seg[si];
      const int row0 = (t - sg.tile0) * rs;
      const int nrows = min(rs, sg.n - row0);
      const void* sp = mat ? sg.s2 : sg.s;
      const int kblk = sg.kblk;
      float sc[J];
      if (kblk > 1) {
#pragma unroll
        for (int j = 0; j < J; ++j) {
          const int c = (slice * J + j) * 32 + lane;
          sc[j] = ldexpf(load_scale<ST>(sp, scale_index(kblk, row0, c >> 3)), -ex[c >> 3]);
        }
      }
      const uint32_t sbase = stage0 + slot * sb + (uint32_t)(mat * rs) * K;
      for (int ri = warp / npart; ri < rs; ri += row_step) {
        if (ri < nrows && !failed) {
          if (kblk <= 1) {
#pragma unroll
            for (int j = 0; j < J; ++j) {
              const int c = (slice * J + j) * 32 + lane;
              sc[j] = ldexpf(load_scale<ST>(sp, scale_index(kblk, row0 + ri, c >> 3)), -ex[c >> 3]);
            }
          }
          const uint32_t rbase = sbase + (uint32_t)ri * K;
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < J; ++j) {
            const int c = (slice * J + j) * 32 + lane;
            const uint4 w = lds_v4(rbase + c * 16);
            float p0 = 0.f, p1 = 0.f;
            dot16_f16(w, xh[j], p0, p1);
            acc = fmaf(p0 + p1, sc[j], acc);
          }
          acc = warp_sum(acc);
          if (npart == 1) {
            if (lane == 0) gemv_epilogue(sg, row0 + ri, acc, 0.f, am_best);
          } else if (lane == 0) {
            red[(slot * rs + ri) * npart + part] = acc;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar0 + 8 * (ns + slot));
      if (npart > 1) {
        named_bar(1, nthr);
        if (ctid < nrows && !failed) {
          const float* rr = red + (slot * rs + ctid) * npart;
          float v = 0.f, v2 = 0.f;
          for (int s = 0; s < nslice; ++s) v += rr[s];
          if (npart > nslice)
            for (int s = 0; s < nslice; ++s) v2 += rr[nslice + s];
          gemv_epilogue(sg, row0 + ctid, v, v2, am_best);
        }
      }
    }
  }

  if (a.am_ws) argmax_finish(a, am_best, misc + 32);
}

// ---------------------------------------------------------------------------
// Generic fallback: one warp per output row, weights read straight from global
// memory in 4-byte words (any K % 8 == 0, rows 4-byte aligned), FP32 x in
// shared memory.  Used for shapes the streaming plan does not cover.
// ---------------------------------------------------------------------------
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
    if (lane == 0) gemv_epilogue(sg, r, acc[0], acc[1], am_best);
  }
  if (a.am_ws) argmax_finish(a, am_best, misc + 32);
}

}  // namespace qwen
