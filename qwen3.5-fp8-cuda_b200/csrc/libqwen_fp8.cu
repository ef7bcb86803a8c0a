// libqwen_fp8.so: drop-in replacement for the reference's fp8_kernels library
// (the `QWEN_FP8_DLL` the reference loader opens, main.py:102-111).
// Declarations: include/qwen_fp8.h.
//
// fp8_gemm_batch keeps the reference signature (fp8_kernels.cu:72-79):
// y[M, N] = bf16(x[M, K] . Wdq^T) with the reference scale-mode encoding.
// Block-scaled weights (K_blk = K/128 > 1) go to the tcgen05 GEMM
// (gemm_tc.cuh); the other scale layouts run the block-scaled GEMV once per
// token row.
#include "common.cuh"
#include "gemv_host.cuh"
#include "gemm_tc.cuh"

using namespace qwen;

namespace {
thread_local int g_last_error = 0;
inline int record(cudaError_t e) {
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) g_last_error = (int)e;
  return (int)e;
}

// Per-device workspace for the split x operand of the GEMM: allocated on
// the first call that needs it and grown when a larger call comes (this is
// the one place the library allocates; prefill runs outside graph capture).
struct GemmWorkspace {
  uint8_t* xs = nullptr;
  size_t xs_bytes = 0;
  float* xinv = nullptr;
  size_t xinv_bytes = 0;
};
GemmWorkspace g_ws[64];
std::mutex g_ws_mu;

cudaError_t ensure(void** p, size_t* have, size_t need) {
  if (*have >= need) return cudaSuccess;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  cudaError_t e = cudaMalloc(p, need);
  if (e == cudaSuccess) *have = need;
  return e;
}

// tcgen05 path; cudaErrorNotSupported when the call is not eligible.
cudaError_t gemm_tc_run(const bf16* x, const void* w, const void* s, bf16* y, int M, int N, int K, int K_blk,
                        cudaStream_t st) {
  if (M < 2 || N <= 0 || K % 128 != 0 || K < 256 || K_blk != K / 128) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(x) & 7u) || (reinterpret_cast<uintptr_t>(w) & 15u)) return cudaErrorNotSupported;
  const int nkb = K / 128;
  const int ntm = (M + GM_TOK - 1) / GM_TOK;
  const int mpad = ntm * GM_TOK;
  const int d = current_device();
  std::lock_guard<std::mutex> lock(g_ws_mu);
  GemmWorkspace& ws = g_ws[d];
  cudaError_t e = ensure(reinterpret_cast<void**>(&ws.xs), &ws.xs_bytes, (size_t)ntm * 128 * K);
  if (e != cudaSuccess) return e;
  e = ensure(reinterpret_cast<void**>(&ws.xinv), &ws.xinv_bytes, (size_t)mpad * nkb * sizeof(float));
  if (e != cudaSuccess) return e;
  CUtensorMap wmap, xmap;
  if (!weight_tmap(&wmap, w, N, K) || !weight_tmap(&xmap, ws.xs, ntm * 128, K)) return cudaErrorNotSupported;
  const long long warps = (long long)mpad * nkb;
  gemm_x_split_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(x, M, K, ws.xs, ws.xinv);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  GemmArgs a;
  a.s = s;
  a.xinv = ws.xinv;
  a.y = y;
  a.M = M;
  a.N = N;
  a.K = K;
  a.stages = (TC_SMEM_MAX - gemm_smem_bytes(0)) / GM_STAGE;
  if (a.stages > 6) a.stages = 6;
  const int smem = gemm_smem_bytes(a.stages);
  static bool attr_done[64] = {};
  if (!attr_done[d]) {
    e = cudaFuncSetAttribute(gemm_tc_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX);
    if (e != cudaSuccess) return e;
    attr_done[d] = true;
  }
  const int ntiles = ((N + TC_ROWS - 1) / TC_ROWS) * ntm;
  const int sms = sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ntiles < sms ? ntiles : sms);
  cfg.blockDim = dim3(GM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<bf16>, a, wmap, xmap);
}
}  // namespace

extern "C" {

int qwen_fp8_last_error(void) {
  const int e = g_last_error;
  g_last_error = 0;
  return e;
}

// Block-scaled weights: tcgen05 GEMM; other scale layouts: the GEMV per row.
void fp8_gemm_batch(const void* x_bf16, const void* w_fp8, const void* w_scale_bf16, void* y_bf16, int M, int N,
                    int K, int K_blocks, cudaStream_t stream) {
  if (M < 0 || N < 0 || K <= 0 || (M > 0 && (!x_bf16 || !w_fp8 || !w_scale_bf16 || !y_bf16))) {
    g_last_error = (int)cudaErrorInvalidValue;
    return;
  }
  const bf16* x = static_cast<const bf16*>(x_bf16);
  bf16* y = static_cast<bf16*>(y_bf16);
  if (M == 0 || N == 0) return;
  const cudaError_t e = gemm_tc_run(x, w_fp8, w_scale_bf16, y, M, N, K, K_blocks, stream);
  if (e != cudaErrorNotSupported) {
    record(e);
    return;
  }
  for (int m = 0; m < M; ++m) {
    GemvArgs a = make_args(x + (size_t)m * K, K);
    a.nseg = 1;
    a.seg[0] = make_seg(w_fp8, w_scale_bf16, y + (size_t)m * N, N, K_blocks);
    if (record(gemv_run(a, false, stream, false))) return;
  }
}

}  // extern "C"
