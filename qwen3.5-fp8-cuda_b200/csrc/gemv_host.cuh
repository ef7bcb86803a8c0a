// Host-side planning and launch of the GEMV family (gemv.cuh).
#pragma once

#include "gemv.cuh"

#include <cstring>

namespace qwen {

// Per-device facts cached on first use.
struct DevInfo {
  int sms = 0;
  bool attrs_set = false;
};
static DevInfo g_dev[64];

static inline int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}
static inline int sm_count() {
  const int d = current_device();
  if (g_dev[d].sms == 0) cudaDeviceGetAttribute(&g_dev[d].sms, cudaDevAttrMultiProcessorCount, d);
  return g_dev[d].sms;
}

template <typename ST, bool PAIR>
static cudaError_t launch_mma_inst(const GemvArgs& a, int grid, int smem, cudaStream_t st, bool pdl) {
  auto kern = gemv_mma_kernel<ST, PAIR>;
  static bool attr_done[64] = {};
  const int d = current_device();
  if (!attr_done[d]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[d] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename ST>
static cudaError_t launch_simple(const GemvArgs& a, cudaStream_t st, bool pdl) {
  auto kern = gemv_simple_kernel<ST>;
  const int K = a.K;
  const int smem = align_up(2 * K, 16) + 4 * K + 8 * 64;
  static bool attr_done[64] = {};
  const int d = current_device();
  if (!attr_done[d]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[d] = true;
  }
  int rows = 0;
  for (int s = 0; s < a.nseg; ++s) rows += a.seg[s].n;
  const int warps_total = rows;
  int grid = (warps_total + 7) / 8;
  const int cap = sm_count() * 4;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Validate, plan and launch.  `f32_scales` selects FP32 scale storage.
// Returns cudaErrorInvalidValue on bad arguments (nothing launched).
static cudaError_t gemv_run(GemvArgs a, bool f32_scales, cudaStream_t st, bool pdl, bool force_simple = false) {
  if (a.K <= 0 || a.K % 8 != 0 || a.nseg <= 0 || a.nseg > GEMV_MAX_SEG || !a.x) return cudaErrorInvalidValue;
  // Tensor-core path: K a multiple of 128, 16-byte aligned weights, and
  // either every segment a gate/up pair or none.
  bool mma_ok = a.K % 128 == 0 && !force_simple && aligned16(a.x) && (!a.x2 || aligned16(a.x2)) &&
                (!a.h2_out || aligned16(a.h2_out)) && (!a.norm_w || aligned16(a.norm_w)) &&
                (reinterpret_cast<uintptr_t>(a.xn_out) & 7u) == 0;
  int npair = 0, nunits = 0, rows = 0;
  for (int s = 0; s < a.nseg; ++s) {
    GemvSeg& sg = a.seg[s];
    if (sg.n < 0 || !sg.w || !sg.s) return cudaErrorInvalidValue;
    if (sg.epi != EPI_ARGMAX && sg.n > 0 && !sg.y) return cudaErrorInvalidValue;
    if (sg.epi == EPI_SILU_PAIR && (!sg.w2 || !sg.s2)) return cudaErrorInvalidValue;
    if (sg.epi == EPI_CONV && (sg.cw < 1 || sg.cw > 8 || !sg.aux0 || !sg.aux2)) return cudaErrorInvalidValue;
    if (sg.epi == EPI_ARGMAX && !a.am_ws) return cudaErrorInvalidValue;
    if (!aligned16(sg.w) || (sg.epi == EPI_SILU_PAIR && !aligned16(sg.w2))) mma_ok = false;
    if (sg.kblk <= 1 || sg.kblk != (a.K + 127) / 128) mma_ok = false;  // block scales only
    npair += sg.epi == EPI_SILU_PAIR;
    rows += sg.n;
  }
  if (rows == 0) return cudaSuccess;
  if (npair != 0 && npair != a.nseg) mma_ok = false;
  if (mma_ok && (a.K / 128 + GEMV_WARPS - 1) / GEMV_WARPS > 32) mma_ok = false;  // K > 32768
  if (mma_ok) {
    // Work units: 8 rows of a gate/up pair, else 16 rows of one matrix.
    const bool pair = npair != 0;
    const int unit_rows = pair ? GEMV_TILE : 2 * GEMV_TILE;
    for (int s = 0; s < a.nseg; ++s) {
      a.seg[s].unit0 = nunits;
      nunits += (a.seg[s].n + unit_rows - 1) / unit_rows;
    }
    a.nunits = nunits;
    // Split K over S warps of a CTA when there are too few units to give
    // every resident warp one; a warp holds the scales of at most 32 K-blocks
    // (one per lane).
    const int nkb = a.K / 128;
    const int warps = sm_count() * GEMV_CTAS_PER_SM * GEMV_WARPS;
    int S = 1;
    while (S < GEMV_WARPS && (long long)nunits * S < warps && 2 * S <= nkb) S *= 2;
    while (S < GEMV_WARPS && (nkb + S - 1) / S > 32) S *= 2;
    a.nslice = S;
    const int smem = gemv_smem_layout(a.K).total;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    const int cap = sm_count() * GEMV_CTAS_PER_SM;
    const int groups = GEMV_WARPS / S;
    int grid = (nunits + groups - 1) / groups;
    grid = grid < cap ? grid : cap;
    if (pair)
      return f32_scales ? launch_mma_inst<float, true>(a, grid, smem, st, pdl)
                        : launch_mma_inst<bf16, true>(a, grid, smem, st, pdl);
    return f32_scales ? launch_mma_inst<float, false>(a, grid, smem, st, pdl)
                      : launch_mma_inst<bf16, false>(a, grid, smem, st, pdl);
  }
  return f32_scales ? launch_simple<float>(a, st, pdl) : launch_simple<bf16>(a, st, pdl);
}

static inline GemvSeg make_seg(const void* w, const void* s, void* y, int n, int kblk, int epi = EPI_STORE) {
  GemvSeg g;
  std::memset(&g, 0, sizeof(g));
  g.w = static_cast<const uint8_t*>(w);
  g.s = s;
  g.y = y;
  g.n = n;
  g.kblk = kblk;
  g.epi = epi;
  return g;
}

static inline GemvArgs make_args(const void* x, int K) {
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  a.x = static_cast<const bf16*>(x);
  a.K = K;
  a.eps = 1e-6f;
  a.pro = PRO_NONE;
  return a;
}

}  // namespace qwen
