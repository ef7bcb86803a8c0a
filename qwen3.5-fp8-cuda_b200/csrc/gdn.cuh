// GatedDeltaNet recurrent-state decode step (one token), in place on the
// FP32 state.
//
// Restates delta_rule_decode_kernel (fused_kernels.cu:623-684) per value head h:
//   q_hat = q * rsqrt(sum q^2 + 1e-6) / sqrt(D);  k_hat = k * rsqrt(sum k^2 + 1e-6)
//   pred_d = sum_kd S[kd,d] * e^g * k_hat[kd];    delta_d = (v_d - pred_d) * beta
//   S[kd,d] <- S[kd,d] * e^g + k_hat[kd] * delta_d;  out_d = sum_kd S[kd,d] * q_hat[kd]
// State layout [H][Dk][Dv] FP32 (thread d indexes v), as the reference.
//
// Differences from the reference kernel, all in how the work is mapped:
//  * the state is read once and written once (the reference reads it twice):
//    each thread keeps its Dk/KG slice of column d in registers between the
//    prediction and the update;
//  * KG thread groups split the key dimension, so a head runs D*KG threads;
//  * value head h reads key head h / rep directly (no repeat_interleave copy);
//  * without the fused epilogue the D value columns of a head are split over
//    VS CTAs (the columns are independent), which spreads the state traffic
//    over VS times more SMs;
//  * optional fused epilogue: the default decode path's RMSNormGated
//    (main.py:1152-1159): out = bf16(bf16(bf16(o*rsqrt(mean(o^2)+eps)) * w) * bf16(silu(z)))
//    with o = bf16(core).
#pragma once

#include "common.cuh"

namespace qwen {

struct GdnArgs {
  const bf16* q;       // query heads, head stride D
  const bf16* k;       // key heads, head stride D
  const bf16* v;       // value heads, head stride D
  const float* g;      // [H] log-decay
  const bf16* beta;    // [H]
  float* state;        // [H][D][D]
  bf16* out;           // [H][D]: core output, or the gated output when `gated`
  const bf16* z;       // gated: [H][D]
  const bf16* norm_w;  // gated: [D] BF16
  float eps;
  int rep;             // value heads per key head
  int gated;
  L2Prefetch pf;       // weights of the next launch (see common.cuh)
};

template <int D, int KG, int VS>
__global__ void __launch_bounds__(D * KG / VS) gdn_decode_kernel(const __grid_constant__ GdnArgs a) {
  static_assert(VS <= KG, "q / k loads need at least D threads");
  constexpr int DC = D / VS;  // value columns of this CTA
  constexpr int NT = DC * KG;
  constexpr int KS = D / KG;  // key rows per thread
  __shared__ float qs[D], ks[D];
  __shared__ float red[KG][DC];
  __shared__ float wsum[NT / 32 + 1];
  const int h = blockIdx.x;
  const int tid = threadIdx.x;
  const int dl = tid % DC, grp = tid / DC;
  const int d = blockIdx.y * DC + dl;
  const int lane = tid & 31, warp = tid >> 5;

  if (tid == 0) pdl_trigger();
  if (tid < 32) l2_prefetch_share(a.pf, tid);
  // q/k/v/g/beta come from the projection kernel and the state from the
  // previous step, so every load below waits for the previous grid.
  pdl_wait();

  float* S = a.state + (size_t)h * D * D;
  // Issue the state loads first: they are the bulk of the traffic.
  float s[KS];
#pragma unroll
  for (int i = 0; i < KS; ++i) s[i] = S[(size_t)(grp * KS + i) * D + d];

  const int kh = h / a.rep;
  float qv = 0.f, kv = 0.f;
  if (tid < D) {
    qv = bf2f(a.q[(size_t)kh * D + tid]);
    kv = bf2f(a.k[(size_t)kh * D + tid]);
  }
  // Block sums of q^2 and k^2 over the D threads of group 0.
  __shared__ float rq[D / 32], rk[D / 32];
  float sq = warp_sum(qv * qv), sk = warp_sum(kv * kv);
  if (lane == 0 && tid < D) {
    rq[warp] = sq;
    rk[warp] = sk;
  }
  __syncthreads();
  float tq = 0.f, tk = 0.f;
#pragma unroll
  for (int i = 0; i < D / 32; ++i) {
    tq += rq[i];
    tk += rk[i];
  }
  const float q_scale = rsqrtf(tq + 1e-6f) * rsqrtf((float)D);
  const float k_scale = rsqrtf(tk + 1e-6f);
  if (tid < D) {
    qs[tid] = qv * q_scale;
    ks[tid] = kv * k_scale;
  }
  __syncthreads();

  const float decay = expf(a.g[h]);
  const float beta = bf2f(a.beta[h]);
  float pred = 0.f;
#pragma unroll
  for (int i = 0; i < KS; ++i) pred += s[i] * decay * ks[grp * KS + i];
  red[grp][dl] = pred;
  __syncthreads();
  float ptot = 0.f;
#pragma unroll
  for (int gI = 0; gI < KG; ++gI) ptot += red[gI][dl];
  const float delta = (bf2f(a.v[(size_t)h * D + d]) - ptot) * beta;
  __syncthreads();  // everyone has read red before it is reused

  float o = 0.f;
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    const float u = s[i] * decay + ks[grp * KS + i] * delta;
    S[(size_t)(grp * KS + i) * D + d] = u;
    o += u * qs[grp * KS + i];
  }
  red[grp][dl] = o;
  __syncthreads();
  if (grp != 0) return;
  float ot = 0.f;
#pragma unroll
  for (int gI = 0; gI < KG; ++gI) ot += red[gI][dl];
  const bf16 core = f2bf(ot);
  bf16* out = a.out + (size_t)h * D + d;
  if (VS > 1 || !a.gated) {
    *out = core;
    return;
  }
  // Gated RMSNorm over the D outputs of this head (threads of group 0 only).
  const float c = bf2f(core);
  float cs = warp_sum(c * c);
  if (lane == 0) wsum[warp] = cs;
  named_bar(1, D);
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < D / 32; ++i) tot += wsum[i];
  const float var = tot / (float)D;
  const bf16 normed = f2bf(c * rsqrtf(var + a.eps));
  const bf16 t = f2bf(bf2f(normed) * bf2f(a.norm_w[d]));
  const float zv = bf2f(a.z[(size_t)h * D + d]);
  const bf16 zs = f2bf(zv / (1.0f + expf(-zv)));
  *out = f2bf(bf2f(t) * bf2f(zs));
}

static inline cudaError_t launch_gdn(const GdnArgs& a, int n_heads, int head_dim, cudaStream_t st, bool pdl) {
  if (n_heads <= 0) return cudaSuccess;
  if (!a.q || !a.k || !a.v || !a.g || !a.beta || !a.state || !a.out || a.rep <= 0) return cudaErrorInvalidValue;
  if (a.gated && (!a.z || !a.norm_w)) return cudaErrorInvalidValue;
  // The fused gated norm needs a whole head per CTA; the core output alone is
  // split over 4 CTAs per head.
  const int vs = a.gated ? 1 : 4;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_heads, vs);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  switch (head_dim) {
    case 64:
      cfg.blockDim = dim3(64 * 4 / vs);
      return vs == 1 ? cudaLaunchKernelEx(&cfg, gdn_decode_kernel<64, 4, 1>, a)
                     : cudaLaunchKernelEx(&cfg, gdn_decode_kernel<64, 4, 4>, a);
    case 128:
      cfg.blockDim = dim3(128 * 4 / vs);
      return vs == 1 ? cudaLaunchKernelEx(&cfg, gdn_decode_kernel<128, 4, 1>, a)
                     : cudaLaunchKernelEx(&cfg, gdn_decode_kernel<128, 4, 4>, a);
    default:  // head dims of the Qwen3.5 family are 128 (64 kept for small tests)
      return cudaErrorInvalidValue;
  }
}

// Reference-compatible gate preparation (prepare_linear_gates_kernel,
// fused_kernels.cu:575-590): g = -exp(A_log) * softplus(a + dt_bias) and
// beta = bf16(sigmoid(b)).  softplus switches to the identity above 20, as
// torch's F.softplus does, instead of overflowing.
__global__ void linear_gates_kernel(const bf16* a, const bf16* b, const float* A_log, const float* dt_bias,
                                    float* g_out, bf16* beta_out, int heads) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= heads) return;
  const float x = bf2f(a[h]) + dt_bias[h];
  const float sp = x > 20.0f ? x : log1pf(expf(x));
  g_out[h] = -expf(A_log[h]) * sp;
  const float bv = bf2f(b[h]);
  beta_out[h] = f2bf(1.0f / (1.0f + expf(-bv)));
}

// Reference-compatible gated RMSNorm (rmsnorm_gated_decode_kernel,
// fused_kernels.cu:592-618): FP32 throughout, one BF16 rounding at the end.
__global__ void rmsnorm_gated_f32_kernel(const bf16* core, const bf16* z, const bf16* w, bf16* out, int D,
                                         float eps) {
  __shared__ float wsum[32];
  const int h = blockIdx.x;
  float ss = 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const float x = bf2f(core[(size_t)h * D + d]);
    ss = fmaf(x, x, ss);
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += wsum[i];
  const float r = rsqrtf(tot / (float)D + eps);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    const size_t o = (size_t)h * D + d;
    const float x = bf2f(core[o]);
    const float zv = bf2f(z[o]);
    out[o] = f2bf(x * r * bf2f(w[d]) * (zv / (1.0f + expf(-zv))));
  }
}

}  // namespace qwen
