// libqwen_fp8.so: drop-in replacement for the reference's fp8_kernels library
// (the `QWEN_FP8_DLL` the reference loader opens, main.py:102-111).
// Declarations: include/qwen_fp8.h.
//
// fp8_gemm_batch keeps the reference signature (fp8_kernels.cu:72-79):
// y[M, N] = bf16(x[M, K] . Wdq^T) with the reference scale-mode encoding.
#include "common.cuh"
#include "gemv_host.cuh"

using namespace qwen;

namespace {
thread_local int g_last_error = 0;
inline int record(cudaError_t e) {
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) g_last_error = (int)e;
  return (int)e;
}
}  // namespace

extern "C" {

int qwen_fp8_last_error(void) {
  const int e = g_last_error;
  g_last_error = 0;
  return e;
}

// Row-by-row block-scaled GEMV over the M input rows.
void fp8_gemm_batch(const void* x_bf16, const void* w_fp8, const void* w_scale_bf16, void* y_bf16, int M, int N,
                    int K, int K_blocks, cudaStream_t stream) {
  if (M < 0 || N < 0 || K <= 0) {
    g_last_error = (int)cudaErrorInvalidValue;
    return;
  }
  const bf16* x = static_cast<const bf16*>(x_bf16);
  bf16* y = static_cast<bf16*>(y_bf16);
  for (int m = 0; m < M; ++m) {
    GemvArgs a = make_args(x + (size_t)m * K, K);
    a.nseg = 1;
    a.seg[0] = make_seg(w_fp8, w_scale_bf16, y + (size_t)m * N, N, K_blocks);
    if (record(gemv_run(a, false, stream, false))) return;
  }
}

}  // extern "C"
