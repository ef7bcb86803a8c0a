/*
 * qwen_fp8.h -- C ABI of libqwen_fp8.so, the sm_100a (B200) drop-in for the
 * reference's fp8_kernels library (opened through QWEN_FP8_DLL,
 * main.py:102-111; argtypes main.py:108-111).
 */
#ifndef QWEN_FP8_H
#define QWEN_FP8_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y[M, N] = bf16(x[M, K] . dequant(W)^T), reference K_blk scale encoding.
 * Replaces fp8_gemm_batch (qwen3_infer/csrc/fp8_kernels.cu:72-89). */
void fp8_gemm_batch(const void* x_bf16, const void* w_fp8, const void* w_scale_bf16, void* y_bf16, int M, int N,
                    int K, int K_blocks, cudaStream_t stream);

/* Last error recorded by a call on this host thread, then cleared. */
int qwen_fp8_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_FP8_H */
