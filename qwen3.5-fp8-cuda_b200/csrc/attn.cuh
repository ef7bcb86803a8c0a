// Single-query GQA attention for the full-attention layers (decode).
//
// Semantics follow the reference's layer_mid_attn / fused_attn_v2_kernel
// (fused_kernels.cu:787-903, 1199-1297) and the output gate of main.py:1059:
//   q, k <- bf16(RMSNorm(1+w)) per head; partial rotate-half RoPE on the first
//   `rot` channels (bf16 out); k, v written to the BF16 cache at `pos`;
//   out = softmax(q k^T / sqrt(D)) v in FP32, bf16(out * (1/sum));
//   gated: out = bf16(out * bf16(sigmoid(gate))).
//
// Inputs produced earlier in the same step (q, gate, the new k / v, split
// partials) are read at L2 (ld.global.cg), so the same code serves the
// persistent step kernel, where an SM's L1 may hold an older layer's lines.
//
// Mapping: one CTA per (KV head, position split).  The CTA handles all G query
// heads of its KV head, so each K/V row is read once for G heads.  The current
// context (pos + 1 positions, known only on the device) is spread over the
// nsplit splits, at least `chunk` positions each, so a graph captured once
// keeps every split busy as the context grows.  Warps take
// positions round-robin with a per-warp online softmax; warps are merged in
// shared memory and splits through an FP32 workspace, the last CTA of each
// KV head (atomic counter, self-resetting) doing the final merge.
#pragma once

#include "common.cuh"

namespace qwen {

struct AttnArgs {
  const bf16* q;       // query heads; head h at q + h * q_stride
  const bf16* gate;    // gated: gate head h at gate + h * q_stride (nullable)
  const bf16* k_new;   // prep: new key / value heads [n_kv][D]
  const bf16* v_new;
  const float* q_norm;  // prep: FP32 [D] or null
  const float* k_norm;
  const float* cos;    // prep: [max_pos][rot]
  const float* sin;
  bf16* k_cache;       // [n_kv][max_seq][D]
  bf16* v_cache;
  const int* pos_ptr;  // position of the new token (device) or null -> pos_const
  int pos_const;
  int seq_len;         // > 0: attend over exactly seq_len cached positions (no prep)
  int q_stride;
  int max_seq;
  int n_heads, n_kv, rot;
  float eps;
  int prep;
  int chunk;           // at least this many positions per split (see below)
  int nsplit;
  float* ws_part;      // nsplit > 1: [n_heads][nsplit][D + 2]
  unsigned* ws_count;  // nsplit > 1: [n_kv], zero before first use, left zeroed
  bf16* out;           // [n_heads][D]
  L2Prefetch pf;       // weights of the next launch (see common.cuh)
};

constexpr int ATTN_WARPS = 8;

template <int D>
__device__ __forceinline__ void attn_prep_head(const bf16* src, const float* norm_w, const float* cs,
                                               const float* sn, int rot, float eps, float* vals_sm, float (&v)[D / 32],
                                               int lane) {
  constexpr int EPL = D / 32;
  // every load first (the head, the norm weights, this lane's RoPE factors):
  // one round trip instead of one per phase
  float nw[EPL], cf[EPL], sf[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int i = lane * EPL + e;
    v[e] = bf2f(__ldcg(src + i));
    nw[e] = norm_w ? norm_w[i] : 0.f;
    cf[e] = cs && i < rot ? cs[i] : 0.f;
    sf[e] = sn && i < rot ? sn[i] : 0.f;
  }
  if (norm_w) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) ss = fmaf(v[e], v[e], ss);
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = bfround(v[e] * r * (1.0f + nw[e]));
  }
  if (cs) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) vals_sm[lane * EPL + e] = v[e];
    __syncwarp();
    const int half = rot / 2;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int i = lane * EPL + e;
      if (i < half) {
        v[e] = bfround(vals_sm[i] * cf[e] - vals_sm[i + half] * sf[e]);
      } else if (i < rot) {
        v[e] = bfround(vals_sm[i] * cf[e] + vals_sm[i - half] * sf[e]);
      }
    }
    __syncwarp();
  }
}

// One (KV head, split) unit of the attention step on ATTN_WARPS warps (threads
// 0 .. ATTN_WARPS*32-1 of the caller, named barrier 1).  `asmem` holds
// attn_smem_bytes<D, G>() bytes; `s_last` is one shared int.  Every exit is
// uniform over the calling threads.  `tl` (optional, profiling): thread 0
// stores %globaltimer stamps after the query / key / value preparation, after
// the split's partials are published, and (last unit only) after the combine
// into tl[0], tl[1], tl[2].  `pos_known` >= 0: the position, already read by
// the caller (else *a.pos_ptr).  U: positions per warp in flight; QREG:
// the scaled queries held in registers (else re-read from shared memory per
// position, for callers with a tighter register budget).
template <int D, int G, int U = 4, bool QREG = true>
__device__ __forceinline__ void attn_unit(const AttnArgs& a, int kh, int split, float* asmem, int* s_last_p,
                                          unsigned* tl = nullptr, int pos_known = -1) {
  auto put_out = [&](size_t idx, bf16 ob) { a.out[idx] = ob; };
  constexpr int EPL = D / 32;
  constexpr int NT = ATTN_WARPS * 32;
  float* qsm = asmem;                       // [G][D] scaled query
  float* wo = qsm + G * D;                  // [ATTN_WARPS][G][D]
  float* wm = wo + ATTN_WARPS * G * D;      // [ATTN_WARPS][G]
  float* wl = wm + ATTN_WARPS * G;          // [ATTN_WARPS][G]
  float* kv_sm = wl + ATTN_WARPS * G;       // [2][D] new k, v (fp32 of bf16 values)
  float* tmp = kv_sm + 2 * D;               // [ATTN_WARPS][D] rope scratch
  int& s_last = *s_last_p;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int pos = pos_known >= 0 ? pos_known : (a.pos_ptr ? __ldcg(a.pos_ptr) : a.pos_const);
  if (pos < 0 || pos >= a.max_seq) {  // uniform over the grid: every unit leaves
    if (threadIdx.x == 0 && kh == 0 && split == 0) qwen_err_set(ERR_POS_RANGE);
    return;
  }
  const int total = a.seq_len > 0 ? a.seq_len : pos + 1;
  const float qscale = rsqrtf((float)D);
  const float* cs = a.prep && a.cos ? a.cos + (size_t)pos * a.rot : nullptr;
  const float* sn = a.prep && a.sin ? a.sin + (size_t)pos * a.rot : nullptr;

  // ---- Phase A: query heads (and the new key / value) ----
  for (int task = warp; task < G + (a.prep ? 2 : 0); task += ATTN_WARPS) {
    float v[EPL];
    if (task < G) {
      const int h = kh * G + task;
      const bf16* src = a.q + (size_t)h * a.q_stride;
      if (a.prep) {
        attn_prep_head<D>(src, a.q_norm, cs, sn, a.rot, a.eps, tmp + warp * D, v, lane);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) v[e] = bf2f(__ldcg(src + lane * EPL + e));
      }
#pragma unroll
      for (int e = 0; e < EPL; ++e) qsm[task * D + lane * EPL + e] = v[e] * qscale;
    } else if (task == G) {
      attn_prep_head<D>(a.k_new + (size_t)kh * D, a.k_norm, cs, sn, a.rot, a.eps, tmp + warp * D, v, lane);
#pragma unroll
      for (int e = 0; e < EPL; ++e) kv_sm[lane * EPL + e] = v[e];
      if (split == 0) {
#pragma unroll
        for (int e = 0; e < EPL; ++e)
          a.k_cache[((size_t)kh * a.max_seq + pos) * D + lane * EPL + e] = f2bf(v[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const bf16 x = __ldcg(a.v_new + (size_t)kh * D + lane * EPL + e);
        kv_sm[D + lane * EPL + e] = bf2f(x);
        if (split == 0) a.v_cache[((size_t)kh * a.max_seq + pos) * D + lane * EPL + e] = x;
      }
    }
  }
  named_bar(1, NT);
  if (tl && threadIdx.x == 0) tl[0] = (unsigned)globaltimer_ns();

  // ---- Phase B: positions of this split ----
  float qr[QREG ? G : 1][EPL];
  if constexpr (QREG) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int e = 0; e < EPL; ++e) qr[g][e] = qsm[g * D + lane * EPL + e];
  }
  float m[G], l[G], o[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[g][e] = 0.f;
  }
  const int chunk = max(a.chunk, (total + a.nsplit - 1) / a.nsplit);
  const int p0 = split * chunk;
  const int p1 = min(total, p0 + chunk);
  const bf16* kbase = a.k_cache + (size_t)kh * a.max_seq * D;
  const bf16* vbase = a.v_cache + (size_t)kh * a.max_seq * D;
  // Each warp takes U consecutive positions at a time and issues all their
  // K / V row loads (one vector load per lane and row) before using them.
  auto load_row = [&](int p, uint32_t (&kr)[EPL / 2], uint32_t (&vr)[EPL / 2]) {
    const bf16* kp = kbase + (size_t)p * D + lane * EPL;
    const bf16* vp = vbase + (size_t)p * D + lane * EPL;
    if constexpr (EPL == 8) {
      const uint4 k4 = *reinterpret_cast<const uint4*>(kp), v4 = *reinterpret_cast<const uint4*>(vp);
      kr[0] = k4.x; kr[1] = k4.y; kr[2] = k4.z; kr[3] = k4.w;
      vr[0] = v4.x; vr[1] = v4.y; vr[2] = v4.z; vr[3] = v4.w;
    } else {
#pragma unroll
      for (int e = 0; e < EPL / 2; ++e) {
        kr[e] = reinterpret_cast<const uint32_t*>(kp)[e];
        vr[e] = reinterpret_cast<const uint32_t*>(vp)[e];
      }
    }
  };
  for (int pb = p0 + warp * U; pb < p1; pb += ATTN_WARPS * U) {
  uint32_t kb[U][EPL / 2], vb[U][EPL / 2];
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (pb + u < p1 && !(a.prep && pb + u == pos)) load_row(pb + u, kb[u], vb[u]);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int p = pb + u;
    if (p >= p1) continue;  // warp-uniform
    float kx[EPL], vx[EPL];
    if (a.prep && p == pos) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        kx[e] = kv_sm[lane * EPL + e];
        vx[e] = kv_sm[D + lane * EPL + e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < EPL; e += 2) {
        const float2 kf = bf2x_to_f2(kb[u][e / 2]);
        const float2 vf = bf2x_to_f2(vb[u][e / 2]);
        kx[e] = kf.x;
        kx[e + 1] = kf.y;
        vx[e] = vf.x;
        vx[e + 1] = vf.y;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) dot = fmaf(QREG ? qr[QREG ? g : 0][e] : qsm[g * D + lane * EPL + e], kx[e], dot);
      dot = warp_sum(dot);
      const float nm = fmaxf(m[g], dot);
      const float eo = expf(m[g] - nm);
      const float en = expf(dot - nm);
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[g][e] = o[g][e] * eo + en * vx[e];
      l[g] = l[g] * eo + en;
      m[g] = nm;
    }
  }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      wm[warp * G + g] = m[g];
      wl[warp * G + g] = l[g];
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) wo[(warp * G + g) * D + lane * EPL + e] = o[g][e];
  }
  named_bar(1, NT);

  // Merge warps: thread handles (g, d) pairs.
  const int nsplit = a.nsplit;
  for (int idx = threadIdx.x; idx < G * D; idx += NT) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int w = 0; w < ATTN_WARPS; ++w) M = fmaxf(M, wm[w * G + g]);
    float Ls = 0.f, Os = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < ATTN_WARPS; ++w) {
        const float f = expf(wm[w * G + g] - M);
        Ls += wl[w * G + g] * f;
        Os += wo[(w * G + g) * D + d] * f;
      }
    }
    const int h = kh * G + g;
    if (nsplit == 1) {
      const float r = Os * (1.0f / Ls);
      bf16 ob = f2bf(r);
      if (a.gate) {
        const float gv = bf2f(__ldcg(a.gate + (size_t)h * a.q_stride + d));
        ob = f2bf(bf2f(ob) * bfround(1.0f / (1.0f + expf(-gv))));
      }
      put_out((size_t)h * D + d, ob);
    } else {
      float* part = a.ws_part + ((size_t)h * nsplit + split) * (D + 2);
      if (d == 0) {
        part[0] = M;
        part[1] = Ls;
      }
      part[2 + d] = Os;
    }
  }
  if (nsplit == 1) return;

  // one acquire-release count per CTA: its release publishes the CTA's
  // partials (ordered before it by the barrier), its acquire lets the last
  // CTA's threads (ordered after it by the barrier) read every split's
  named_bar(1, NT);
  if (threadIdx.x == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.ws_count + kh) : "memory");
    s_last = prev == (unsigned)(nsplit - 1);
  }
  named_bar(1, NT);
  if (tl && threadIdx.x == 0) tl[1] = (unsigned)globaltimer_ns();
  if (!s_last) return;
  const int n_active = (total + chunk - 1) / chunk;
  // Split weights f_s = exp(m_s - M) (held in the per-warp output area),
  // then every thread adds its (head, channel) pairs over the splits.
  float* fac = wo;
  constexpr int FCAP = ATTN_WARPS * D;  // splits per head that fit
  const bool fits = n_active <= FCAP;
  if (fits) {
    // every thread's (head, channel) pairs, added over the splits in split
    // order below; the first SPI splits' partials and the output gates are
    // loaded here, in the same round trip as the split weights
    constexpr int PER = (G * D + NT - 1) / NT;
    constexpr int SPI = PER <= 4 ? 8 : 4;  // splits per iteration: up to 32 loads in flight
    float o[SPI][PER], gv[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int idx = threadIdx.x + k * NT;
      gv[k] = (idx < G * D && a.gate) ? bf2f(__ldcg(a.gate + (size_t)(kh * G + idx / D) * a.q_stride + idx % D))
                                      : 0.f;
#pragma unroll
      for (int j = 0; j < SPI; ++j)
        o[j][k] = (idx < G * D && j < n_active)
                      ? __ldcg(a.ws_part + ((size_t)(kh * G + idx / D) * nsplit + j) * (D + 2) + 2 + idx % D)
                      : 0.f;
    }
    // split weights: warp g, lanes over the splits; (M, L) of a split is one
    // 8-byte load, every lane's loads issued before the reductions
    constexpr int MAXL = 4;  // splits per lane held in registers (n_active <= 128)
    for (int g = warp; g < G; g += ATTN_WARPS) {
      const float* base = a.ws_part + (size_t)(kh * G + g) * nsplit * (D + 2);
      float M = -INFINITY, L = 0.f;
      if (n_active <= 32 * MAXL) {
        float2 ml[MAXL];
#pragma unroll
        for (int k = 0; k < MAXL; ++k) {
          const int sp = lane + 32 * k;
          ml[k] = sp < n_active ? __ldcg(reinterpret_cast<const float2*>(base + sp * (D + 2)))
                                : make_float2(-INFINITY, 0.f);
        }
#pragma unroll
        for (int k = 0; k < MAXL; ++k) M = fmaxf(M, ml[k].x);
        M = warp_max(M);
#pragma unroll
        for (int k = 0; k < MAXL; ++k) {
          const int sp = lane + 32 * k;
          const float f = ml[k].x == -INFINITY ? 0.f : expf(ml[k].x - M);
          L += ml[k].y * f;
          if (sp < n_active) fac[g * FCAP + sp] = f;
        }
      } else {
        for (int sp = lane; sp < n_active; sp += 32) M = fmaxf(M, __ldcg(base + sp * (D + 2)));
        M = warp_max(M);
        for (int sp = lane; sp < n_active; sp += 32) {
          const float ms = __ldcg(base + sp * (D + 2));
          const float f = ms == -INFINITY ? 0.f : expf(ms - M);
          L += __ldcg(base + sp * (D + 2) + 1) * f;
          fac[g * FCAP + sp] = f;
        }
      }
      L = warp_sum(L);
      if (lane == 0) wl[g] = L;
    }
    named_bar(1, NT);
    float Os[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) Os[k] = 0.f;
    for (int s = 0; s < n_active; s += SPI) {
      if (s > 0) {  // the next SPI splits (the first are loaded above)
#pragma unroll
        for (int j = 0; j < SPI; ++j)
#pragma unroll
          for (int k = 0; k < PER; ++k) {
            const int idx = threadIdx.x + k * NT;
            o[j][k] = (idx < G * D && s + j < n_active)
                          ? __ldcg(a.ws_part + ((size_t)(kh * G + idx / D) * nsplit + s + j) * (D + 2) + 2 + idx % D)
                          : 0.f;
          }
      }
#pragma unroll
      for (int j = 0; j < SPI; ++j)
#pragma unroll
        for (int k = 0; k < PER; ++k) {
          const int idx = threadIdx.x + k * NT;
          if (idx < G * D && s + j < n_active) Os[k] = fmaf(o[j][k], fac[(idx / D) * FCAP + s + j], Os[k]);
        }
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int idx = threadIdx.x + k * NT;
      if (idx >= G * D) continue;
      const int g = idx / D, d = idx % D;
      bf16 ob = f2bf(Os[k] * (1.0f / wl[g]));
      if (a.gate) ob = f2bf(bf2f(ob) * bfround(1.0f / (1.0f + expf(-gv[k]))));
      put_out((size_t)(kh * G + g) * D + d, ob);
    }
  } else {
    named_bar(1, NT);
    for (int idx = threadIdx.x; idx < G * D; idx += NT) {
      const int g = idx / D, d = idx % D;
      const int h = kh * G + g;
      const float* base = a.ws_part + (size_t)h * nsplit * (D + 2);
      float Os = 0.f, Ls = 0.f;
      float M = -INFINITY;
      for (int sp = 0; sp < n_active; ++sp) M = fmaxf(M, __ldcg(base + sp * (D + 2)));
      for (int sp = 0; sp < n_active; ++sp) {
        const float ms = __ldcg(base + sp * (D + 2));
        if (ms == -INFINITY) continue;
        const float f = expf(ms - M);
        Ls += __ldcg(base + sp * (D + 2) + 1) * f;
        Os += __ldcg(base + sp * (D + 2) + 2 + d) * f;
      }
      bf16 ob = f2bf(Os * (1.0f / Ls));
      if (a.gate) {
        const float gv = bf2f(__ldcg(a.gate + (size_t)h * a.q_stride + d));
        ob = f2bf(bf2f(ob) * bfround(1.0f / (1.0f + expf(-gv))));
      }
      put_out((size_t)h * D + d, ob);
    }
  }
  if (threadIdx.x == 0) {
    a.ws_count[kh] = 0u;
    if (tl) tl[2] = (unsigned)globaltimer_ns();
  }
}

template <int D, int G>
__global__ void __launch_bounds__(ATTN_WARPS * 32) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(16) float asmem[];
  __shared__ int s_last;
  if (threadIdx.x == 0) pdl_trigger();
  if ((threadIdx.x >> 5) == 0) l2_prefetch_share(a.pf, threadIdx.x & 31);
  pdl_wait();
  attn_unit<D, G>(a, blockIdx.x, blockIdx.y, asmem, &s_last);
}

template <int D, int G>
static inline int attn_smem_bytes() {
  return 4 * (G * D + ATTN_WARPS * G * D + 2 * ATTN_WARPS * G + 2 * D + ATTN_WARPS * D);
}

template <int D, int G>
static cudaError_t launch_attn_inst(const AttnArgs& a, cudaStream_t st, bool pdl) {
  auto kern = attn_decode_kernel<D, G>;
  const int smem = attn_smem_bytes<D, G>();
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_kv, a.nsplit);
  cfg.blockDim = dim3(ATTN_WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

static inline cudaError_t launch_attn(const AttnArgs& a, int head_dim, cudaStream_t st, bool pdl) {
  if (a.n_kv <= 0 || a.n_heads <= 0 || a.n_heads % a.n_kv) return cudaErrorInvalidValue;
  if (!a.q || !a.k_cache || !a.v_cache || !a.out || a.nsplit < 1 || a.chunk < 1) return cudaErrorInvalidValue;
  if (a.nsplit > 1 && (!a.ws_part || !a.ws_count)) return cudaErrorInvalidValue;
  if (a.prep && (!a.k_new || !a.v_new)) return cudaErrorInvalidValue;
  if (a.prep && a.cos && (a.rot <= 0 || a.rot > head_dim || a.rot % 2)) return cudaErrorInvalidValue;
  const int G = a.n_heads / a.n_kv;
#define QWEN_ATTN_CASE(DD, GG) \
  if (head_dim == DD && G == GG) return launch_attn_inst<DD, GG>(a, st, pdl);
  QWEN_ATTN_CASE(256, 1) QWEN_ATTN_CASE(256, 2) QWEN_ATTN_CASE(256, 4) QWEN_ATTN_CASE(256, 8)
  QWEN_ATTN_CASE(128, 1) QWEN_ATTN_CASE(128, 2) QWEN_ATTN_CASE(128, 4) QWEN_ATTN_CASE(128, 8)
#undef QWEN_ATTN_CASE
  return cudaErrorInvalidValue;
}

// In-place Q/K RMSNorm + RoPE of layer_mid_attn (fused_kernels.cu:1238-1262)
// and the KV-cache write (1264-1272): one warp per head.
template <int D>
__global__ void attn_prep_inplace_kernel(bf16* q, bf16* k, const bf16* v, const float* q_norm, const float* k_norm,
                                         const float* cos, const float* sin, int pos, int rot, float eps,
                                         bf16* k_cache, bf16* v_cache, int cache_pos, int max_seq, int n_heads,
                                         int n_kv) {
  constexpr int EPL = D / 32;
  __shared__ float tmp[8][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.x * 8 + warp;
  if (head >= n_heads + 2 * n_kv) return;
  const float* cs = cos ? cos + (size_t)pos * rot : nullptr;
  const float* sn = sin ? sin + (size_t)pos * rot : nullptr;
  float v8[EPL];
  if (head < n_heads) {
    bf16* src = q + (size_t)head * D;
    attn_prep_head<D>(src, q_norm, cs, sn, rot, eps, tmp[warp], v8, lane);
#pragma unroll
    for (int e = 0; e < EPL; ++e) src[lane * EPL + e] = f2bf(v8[e]);
  } else if (head < n_heads + n_kv) {
    const int h = head - n_heads;
    bf16* src = k + (size_t)h * D;
    attn_prep_head<D>(src, k_norm, cs, sn, rot, eps, tmp[warp], v8, lane);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      src[lane * EPL + e] = f2bf(v8[e]);
      k_cache[((size_t)h * max_seq + cache_pos) * D + lane * EPL + e] = f2bf(v8[e]);
    }
  } else {
    const int h = head - n_heads - n_kv;
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      v_cache[((size_t)h * max_seq + cache_pos) * D + lane * EPL + e] = v[(size_t)h * D + lane * EPL + e];
  }
}

}  // namespace qwen
