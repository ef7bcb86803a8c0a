// RMSNorm(1+w) and small elementwise kernels.
//
// rmsnorm_rows_kernel restates rmsnorm_ip_kernel / rmsnorm_out_kernel
// (fused_kernels.cu:489-547): per row, rms = rsqrt(sum(x^2)/D + eps),
// out = bf16(x * rms * (1 + w)) with FP32 weights.  One CTA per row keeps the
// row in registers (D <= 8 * blockDim) so in-place operation reads x once.
#pragma once

#include "common.cuh"

namespace qwen {

constexpr int NORM_THREADS = 256;
constexpr int NORM_MAX_PER_THREAD = 16;  // D <= 4096 on the register path

__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_rows_kernel(const bf16* x,
                                                                    const float* __restrict__ w,
                                                                    bf16* out, int D, float eps,
                                                                    int use_pdl) {
  __shared__ float red[NORM_THREADS / 32];
  if (use_pdl) {
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
  }
  const bf16* xr = x + (size_t)blockIdx.x * D;
  bf16* orow = out + (size_t)blockIdx.x * D;
  float v[NORM_MAX_PER_THREAD];
  float ss = 0.f;
  const bool reg_path = D <= NORM_MAX_PER_THREAD * NORM_THREADS;
  if (reg_path) {
#pragma unroll
    for (int i = 0; i < NORM_MAX_PER_THREAD; ++i) {
      const int idx = threadIdx.x + i * NORM_THREADS;
      v[i] = idx < D ? bf2f(xr[idx]) : 0.f;
      ss = fmaf(v[i], v[i], ss);
    }
  } else {
    for (int idx = threadIdx.x; idx < D; idx += NORM_THREADS) {
      const float t = bf2f(xr[idx]);
      ss = fmaf(t, t, ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NORM_THREADS / 32; ++i) tot += red[i];
  const float rms = rsqrtf(tot / (float)D + eps);
  if (reg_path) {
#pragma unroll
    for (int i = 0; i < NORM_MAX_PER_THREAD; ++i) {
      const int idx = threadIdx.x + i * NORM_THREADS;
      if (idx < D) orow[idx] = f2bf(v[i] * rms * (1.0f + w[idx]));
    }
  } else {
    for (int idx = threadIdx.x; idx < D; idx += NORM_THREADS)
      orow[idx] = f2bf(bf2f(xr[idx]) * rms * (1.0f + w[idx]));
  }
}

// out = bf16(a + b) (elem_add_kernel, fused_kernels.cu:553-559).
__global__ void add_bf16_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b, bf16* __restrict__ out,
                                int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f2bf(bf2f(a[i]) + bf2f(b[i]));
}

static inline cudaError_t launch_rmsnorm_rows(const void* x, const float* w, void* out, int rows, int D,
                                              float eps, cudaStream_t st, bool pdl = false) {
  if (rows <= 0) return cudaSuccess;
  if (D <= 0 || !x || !w || !out) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(NORM_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rmsnorm_rows_kernel, static_cast<const bf16*>(x), w, static_cast<bf16*>(out),
                            D, eps, pdl ? 1 : 0);
}

static inline cudaError_t launch_add(const void* a, const void* b, void* out, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  add_bf16_kernel<<<(n + 255) / 256, 256, 0, st>>>(static_cast<const bf16*>(a), static_cast<const bf16*>(b),
                                                     static_cast<bf16*>(out), n);
  return cudaGetLastError();
}

// Tensor-parallel helpers.
// y = bf16(res + bf16(v)) from the all-reduced FP32 partial sums v of a
// K-sliced projection: the residual epilogue of qwen_linear_resid applied
// after the reduction.
__global__ void resid_add_f32_kernel(const bf16* __restrict__ res, const float* __restrict__ v, bf16* __restrict__ y,
                                     int n) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = f2bf(bf2f(res[i]) + bfround(v[i]));
}
// Publishes the step's token to mapped pinned host memory: host_out[0] =
// token, then (after a system-scope fence) host_out[1] = ++*seq, so a host
// thread that sees the new sequence number reads the matching token.
__global__ void publish_token_kernel(const long long* __restrict__ token, volatile long long* host_out,
                                     unsigned long long* seq) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  if (threadIdx.x != 0) return;
  const unsigned long long s = *seq + 1ull;
  *seq = s;
  host_out[0] = *token;
  __threadfence_system();
  host_out[1] = (long long)s;
}
// token = index part of the all-reduced packed argmax key.
__global__ void token_from_key_kernel(const unsigned long long* key, long long* token) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  *token = (long long)(0xffffffffu - (uint32_t)(*key & 0xffffffffull));
}

}  // namespace qwen
