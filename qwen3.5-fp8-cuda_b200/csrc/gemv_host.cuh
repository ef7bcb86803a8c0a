// Host-side planning and launch of the GEMV family (gemv.cuh).
#pragma once

#include "gemv.cuh"
#include "gemv_tc.cuh"
#include "gemv_tcw.cuh"

#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

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

// Direct-load kernel (gemv.cuh) for K = 512 J, J in {4, 5, 6, 8, 18}.
template <typename ST, int J>
static cudaError_t launch_direct_j(const GemvArgs& a, int rows, cudaStream_t st, bool pdl) {
  auto kern = gemv_direct_kernel<ST, J>;
  const int smem = 4 * 512 * J + 8 * 64;
  static bool attr_done[64] = {};
  const int d = current_device();
  if (!attr_done[d]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[d] = true;
  }
  int grid = (rows + 7) / 8;
  const int cap = sm_count() * 8;
  grid = grid < cap ? grid : cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid < 1 ? 1 : grid);
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
template <typename ST>
static cudaError_t launch_direct(const GemvArgs& a, int rows, cudaStream_t st, bool pdl) {
  switch (a.K) {
    case 2048: return launch_direct_j<ST, 4>(a, rows, st, pdl);
    case 2560: return launch_direct_j<ST, 5>(a, rows, st, pdl);
    case 3072: return launch_direct_j<ST, 6>(a, rows, st, pdl);
    case 4096: return launch_direct_j<ST, 8>(a, rows, st, pdl);
    case 9216: return launch_direct_j<ST, 18>(a, rows, st, pdl);
    default: return cudaErrorNotSupported;
  }
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

// GEMV path selection: 0 = tcgen05 with the weights as the N = 256 operand
// (default, gemv_tcw.cuh), 1 = mma.sync streaming kernel, 2 = tcgen05 with
// the weights as the M = 128 operand (gemv_tc.cuh), 3 = the one-warp-per-row
// SIMT kernel.  QWEN_GEMV_PATH=mma, =tc128 or =simple in the environment
// selects the others (for comparison).
static inline int gemv_path() {
  static int path = -1;
  if (path < 0) {
    const char* e = getenv("QWEN_GEMV_PATH");
    path = (e && std::strcmp(e, "mma") == 0)     ? 1
           : (e && std::strcmp(e, "tc128") == 0)  ? 2
           : (e && std::strcmp(e, "simple") == 0) ? 3
                                                  : 0;
  }
  return path;
}

// Weight bytes from which an unpaired launch takes the N = 256 kernel
// (QWEN_TCW_MIN_MB overrides; default 48 MB).
static inline long long tcw_min_bytes() {
  static long long v = -1;
  if (v < 0) {
    const char* e = getenv("QWEN_TCW_MIN_MB");
    v = (e ? atoll(e) : 48ll) << 20;
  }
  return v;
}

// Weight bytes up to which a plain launch takes the direct-load kernel
// (QWEN_DIRECT_MAX_MB overrides; default 12 MB).
static inline long long direct_max_bytes() {
  static long long v = -1;
  if (v < 0) {
    const char* e = getenv("QWEN_DIRECT_MAX_MB");
    v = (e ? atoll(e) : 12ll) << 20;
  }
  return v;
}

// ---------------------------------------------------------------------------
// Tensor-core (tcgen05 + TMA) path
// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor map of an [rows, K] E4M3 matrix: boxes of 128 rows x 128 bytes,
// 128-byte swizzle, rows past the end read as zero.  Cached per (matrix,
// rows, K).
static bool weight_tmap(CUtensorMap* out, const void* w, int rows, int K) {
  struct Key {
    const void* w;
    int rows, K;
    bool operator==(const Key& o) const { return w == o.w && rows == o.rows && K == o.K; }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.w) ^ ((size_t)k.rows * 0x9E3779B97F4A7C15ull) ^ (size_t)k.K;
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  const Key key{w, rows, K};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return true;
    }
  }
  PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  *out = m;
  return true;
}

template <typename ST, bool PAIR>
static cudaError_t launch_tc_inst(const GemvArgs& a, const GemvMaps& m, int grid, int smem, cudaStream_t st,
                                  bool pdl) {
  auto kern = gemv_tc_kernel<ST, PAIR>;
  static bool attr_done[64] = {};
  const int d = current_device();
  if (!attr_done[d]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX);
    if (e != cudaSuccess) return e;
    attr_done[d] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a, m);
}

// Plans and launches the tensor-core path.  Returns cudaErrorNotSupported
// (nothing launched) when the launch is not eligible for it: K not a
// multiple of 128 (or below 256), scales not in 128x128 block layout,
// misaligned buffers, or mixed paired and unpaired segments.
static cudaError_t gemv_tc_run(GemvArgs a, bool f32_scales, cudaStream_t st, bool pdl) {
  const int K = a.K;
  if (K % 128 != 0 || K < 256) return cudaErrorNotSupported;
  const int nkb = K / 128;
  if (!aligned16(a.x) || (a.x2 && !aligned16(a.x2)) || (a.h2_out && !aligned16(a.h2_out)) ||
      (a.norm_w && !aligned16(a.norm_w)) || (reinterpret_cast<uintptr_t>(a.xn_out) & 7u) != 0)
    return cudaErrorNotSupported;
  int npair = 0;
  for (int s = 0; s < a.nseg; ++s) {
    const GemvSeg& sg = a.seg[s];
    if (sg.kblk != nkb || !aligned16(sg.w)) return cudaErrorNotSupported;  // block scales only
    if (sg.epi == EPI_SILU_PAIR) {
      if (!aligned16(sg.w2)) return cudaErrorNotSupported;
      ++npair;
    }
  }
  if (npair != 0 && npair != a.nseg) return cudaErrorNotSupported;
  const bool pair = npair != 0;
  const int P = pair ? 2 : 1;
  GemvMaps m;
  std::memset(&m, 0, sizeof(m));
  int nunits = 0;
  for (int s = 0; s < a.nseg; ++s) {
    GemvSeg& sg = a.seg[s];
    sg.unit0 = nunits;
    nunits += (sg.n + TC_ROWS - 1) / TC_ROWS;
    if (sg.n > 0) {
      if (!weight_tmap(&m.map[s][0], sg.w, sg.n, K)) return cudaErrorNotSupported;
      if (pair && !weight_tmap(&m.map[s][1], sg.w2, sg.n, K)) return cudaErrorNotSupported;
    }
  }
  a.nunits = nunits;
  // K split C: at most 32 K-blocks per item (the epilogue keeps one scale per
  // lane); otherwise the C that minimises the work of the busiest CTA,
  // counting about two K-blocks of fixed cost per item and the partial-sum
  // reduction that a split adds.  The grid is a multiple of C so that each
  // CTA keeps one K slice.
  const int sms = sm_count();
  int best_c = 0;
  double best_cost = 0;
  const int cmin = (nkb + 31) / 32;
  // EPI_SLICES: at most sl_max slices (the rows the caller's buffer holds)
  const int cmax = a.seg[0].epi == EPI_SLICES ? a.sl_max : 64;
  for (int c = cmin; c <= nkb && c <= cmax && c <= sms; ++c) {
    const long long items = (long long)nunits * c;
    if (c > 1 && a.seg[0].epi != EPI_SLICES && (items * P * TC_ROWS > TC_PART_FLOATS || nunits > TC_MAX_CNT))
      break;
    const long long slots = (long long)(sms / c) * c;
    const long long waves = (items + slots - 1) / slots;
    const double cost = (double)waves * ((nkb + c - 1) / c + 2) + (c > 1 ? 1.0 + c / 8.0 : 0.0);
    if (best_c == 0 || cost < best_cost) {
      best_c = c;
      best_cost = cost;
    }
  }
  if (best_c == 0) return cudaErrorNotSupported;
  a.nslice = best_c;
  const long long items = (long long)nunits * best_c;
  const long long slots = (long long)(sms / best_c) * best_c;
  const int grid = (int)(items < slots ? items : slots);
  // Launches that stream for several waves get the whole shared memory; the
  // others stay within half of it (see gemv_tc.cuh).  The deepest ring that
  // fits streams best: under full load the HBM round trip is several us.
  const int budget = items >= 2 * slots ? TC_SMEM_MAX : TC_SMEM_SHARED;
  int S = tc_stages_for(K, P, best_c, budget);
  if (S == 0) S = tc_stages_for(K, P, best_c, TC_SMEM_MAX);
  if (S == 0) return cudaErrorNotSupported;
  a.stages = S;
  const TcSmem L = tc_smem_layout(K, P, best_c, S);
  if (pair)
    return f32_scales ? launch_tc_inst<float, true>(a, m, grid, L.total, st, pdl)
                      : launch_tc_inst<bf16, true>(a, m, grid, L.total, st, pdl);
  return f32_scales ? launch_tc_inst<float, false>(a, m, grid, L.total, st, pdl)
                    : launch_tc_inst<bf16, false>(a, m, grid, L.total, st, pdl);
}

template <typename ST, bool PAIR>
static cudaError_t launch_tcw_inst(const GemvArgs& a, const GemvMaps& m, int grid, int smem, cudaStream_t st,
                                   bool pdl) {
  auto kern = gemv_tcw_kernel<ST, PAIR>;
  static bool attr_done[64] = {};
  const int d = current_device();
  if (!attr_done[d]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_MAX);
    if (e != cudaSuccess) return e;
    attr_done[d] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(TW_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a, m);
}

// Plans and launches the N = 256 tensor-core path (gemv_tcw.cuh); same
// eligibility as gemv_tc_run.  Units are 256 rows of one matrix or 128 rows
// of a gate/up pair.
static cudaError_t gemv_tcw_run(GemvArgs a, bool f32_scales, cudaStream_t st, bool pdl) {
  const int K = a.K;
  if (K % 128 != 0 || K < 256) return cudaErrorNotSupported;
  const int nkb = K / 128;
  if (!aligned16(a.x) || (a.x2 && !aligned16(a.x2)) || (a.h2_out && !aligned16(a.h2_out)) ||
      (a.norm_w && !aligned16(a.norm_w)) || (reinterpret_cast<uintptr_t>(a.xn_out) & 7u) != 0)
    return cudaErrorNotSupported;
  int npair = 0;
  for (int s = 0; s < a.nseg; ++s) {
    const GemvSeg& sg = a.seg[s];
    if (sg.kblk != nkb || !aligned16(sg.w)) return cudaErrorNotSupported;
    if (sg.epi == EPI_SILU_PAIR) {
      if (!aligned16(sg.w2)) return cudaErrorNotSupported;
      ++npair;
    }
  }
  if (npair != 0 && npair != a.nseg) return cudaErrorNotSupported;
  const bool pair = npair != 0;
  const int urows = pair ? 128 : TW_N;
  GemvMaps m;
  std::memset(&m, 0, sizeof(m));
  int nunits = 0;
  for (int s = 0; s < a.nseg; ++s) {
    GemvSeg& sg = a.seg[s];
    sg.unit0 = nunits;
    nunits += (sg.n + urows - 1) / urows;
    if (sg.n > 0) {
      if (!weight_tmap(&m.map[s][0], sg.w, sg.n, K)) return cudaErrorNotSupported;
      if (pair && !weight_tmap(&m.map[s][1], sg.w2, sg.n, K)) return cudaErrorNotSupported;
    }
  }
  a.nunits = nunits;
  // K split C: at most 32 K-blocks per item (one scale per lane), else the C
  // that minimises the busiest CTA's work in 32 KB stages, counting about
  // one stage of fixed cost per item and the cost of the partial-sum
  // reduction.  The grid is a multiple of C.
  const int sms = sm_count();
  int best_c = 0;
  double best_cost = 0;
  const int cmin = (nkb + 31) / 32;
  for (int c = cmin; c <= nkb && c <= 64 && c <= sms; ++c) {
    const long long items = (long long)nunits * c;
    if (c > 1 && (items * TW_N > TC_PART_FLOATS || nunits > TC_MAX_CNT)) break;
    const long long slots = (long long)(sms / c) * c;
    const long long waves = (items + slots - 1) / slots;
    const double cost = (double)waves * ((nkb + c - 1) / c + 1) + (c > 1 ? 1.0 + c / 8.0 : 0.0);
    if (best_c == 0 || cost < best_cost) {
      best_c = c;
      best_cost = cost;
    }
  }
  if (best_c == 0) return cudaErrorNotSupported;
  a.nslice = best_c;
  const long long items = (long long)nunits * best_c;
  const long long slots = (long long)(sms / best_c) * best_c;
  const int grid = (int)(items < slots ? items : slots);
  // One CTA per SM: each CTA holds all 512 TMEM columns, so two CTAs of one
  // grid on an SM would run one after the other (the second waits in
  // tcgen05.alloc).  The ring takes the whole shared memory instead.
  const int S = tw_stages_for(K, best_c, TC_SMEM_MAX);
  if (S == 0) return cudaErrorNotSupported;
  a.stages = S;
  const TwSmem L = tw_smem_layout(K, best_c, S);
  if (pair)
    return f32_scales ? launch_tcw_inst<float, true>(a, m, grid, L.total, st, pdl)
                      : launch_tcw_inst<bf16, true>(a, m, grid, L.total, st, pdl);
  return f32_scales ? launch_tcw_inst<float, false>(a, m, grid, L.total, st, pdl)
                    : launch_tcw_inst<bf16, false>(a, m, grid, L.total, st, pdl);
}

// Validate, plan and launch.  `f32_scales` selects FP32 scale storage.
// Returns cudaErrorInvalidValue on bad arguments (nothing launched).
static cudaError_t gemv_run(GemvArgs a, bool f32_scales, cudaStream_t st, bool pdl, bool force_simple = false) {
  if (gemv_path() == 3) force_simple = true;
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
    if (sg.epi != EPI_ARGMAX && sg.epi != EPI_F32_P2P && sg.n > 0 && !sg.y) return cudaErrorInvalidValue;
    if (sg.epi == EPI_F32_P2P && !sg.aux0) return cudaErrorInvalidValue;
    if (sg.epi == EPI_SLICES && (!sg.y2 || a.nseg != 1 || a.sl_max < 1)) return cudaErrorInvalidValue;
    if (sg.epi == EPI_SILU_PAIR && (!sg.w2 || !sg.s2)) return cudaErrorInvalidValue;
    if (sg.epi == EPI_CONV && (sg.cw < 1 || sg.cw > 8 || !sg.aux0 || !sg.aux2)) return cudaErrorInvalidValue;
    if (sg.epi == EPI_ARGMAX && !a.am_ws) return cudaErrorInvalidValue;
    if (!aligned16(sg.w) || (sg.epi == EPI_SILU_PAIR && !aligned16(sg.w2))) mma_ok = false;
    if (sg.kblk <= 1 || sg.kblk != (a.K + 127) / 128) mma_ok = false;  // block scales only
    npair += sg.epi == EPI_SILU_PAIR;
    rows += sg.n;
  }
  if (rows == 0) return cudaSuccess;
  // Plain x, BF16 stores (the reference ABI's launch_gemv_v4_extern and its
  // grouped forms): the direct-load kernel has the lowest fixed cost (every
  // weight load of a row issued at once, no ring, no K-split round trips).
  // The engines' fused launches keep their kernels (and their summation
  // order); QWEN_GEMV_PATH selects the others.
  // Up to QWEN_DIRECT_MAX_MB (default 12 MB of weights): above that the
  // tcgen05 kernels' deeper pipelines win (measured per config-1 shape).
  if (!force_simple && gemv_path() == 0 && a.pro == PRO_NONE && npair == 0 && aligned16(a.x) &&
      (long long)rows * a.K <= direct_max_bytes()) {
    bool direct = true;
    for (int s = 0; s < a.nseg; ++s) direct &= aligned16(a.seg[s].w) && a.seg[s].epi == EPI_STORE;
    if (direct) {
      const cudaError_t e = f32_scales ? launch_direct<float>(a, rows, st, pdl) : launch_direct<bf16>(a, rows, st, pdl);
      if (e != cudaErrorNotSupported) return e;
    }
  }
  if (!force_simple && (gemv_path() == 0 || gemv_path() == 2)) {
    // The N = 256 kernel needs a whole SM per CTA, so it cannot start beside
    // the previous launch; it pays off for gate/up pairs and for launches
    // that stream at least tcw_min_bytes() of weights.
    bool wide = gemv_path() == 0;
    if (wide) {
      long long bytes = 0;
      bool pair = false;
      for (int s = 0; s < a.nseg; ++s) {
        bytes += (long long)a.seg[s].n * a.K * (a.seg[s].epi == EPI_SILU_PAIR ? 2 : 1);
        pair |= a.seg[s].epi == EPI_SILU_PAIR;
      }
      wide = pair || bytes >= tcw_min_bytes();
    }
    if (a.seg[0].epi == EPI_SLICES) wide = false;  // the M = 128 kernel writes slices
    const cudaError_t e = wide ? gemv_tcw_run(a, f32_scales, st, pdl) : gemv_tc_run(a, f32_scales, st, pdl);
    if (e != cudaErrorNotSupported) return e;
  }
  if (a.pro == PRO_P2P_RMSNORM || a.pro == PRO_GATED_NORM || a.pro == PRO_SLICES_RMSNORM ||
      a.seg[0].epi == EPI_SLICES)
    return cudaErrorNotSupported;  // tcgen05 kernels only
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
