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

// Shared memory budget of one streaming CTA: two CTAs (this kernel's and the
// next kernel's, overlapped through programmatic dependent launch) fit in
// one SM's 228 KB.
constexpr int GEMV_SMEM_BUDGET = 104 * 1024;
constexpr int GEMV_STAGE_TARGET = 32 * 1024;
// Chunks per lane held in registers: above 6 the x slice no longer fits the
// 113-register budget of two co-resident CTAs, so larger K splits into slices.
constexpr int GEMV_MAX_J = 6;

struct GemvPlan {
  bool stream = false;
  int nc = 8, j = 0, nslice = 1, npart = 1, rs = 1, nstages = 0, stage_bytes = 0, smem = 0, grid = 0;
};

// Streaming plan for a given K: K = 512 * J * nslice with J <= 8, nslice
// dividing the consumer warp count, tiles of rs rows that never cross a
// 128-row scale block.
static inline bool plan_stream(int K, bool paired, GemvPlan& p) {
  if (K <= 0 || K % 512 != 0) return false;
  const int L = K / 512;
  const int pair = paired ? 2 : 1;
  struct Opt { int nc, nslice; };
  const Opt opts[] = {{8, 1}, {8, 2}, {8, 4}, {6, 3}, {6, 6}};
  for (const Opt& o : opts) {
    if (L % o.nslice) continue;
    const int J = L / o.nslice;
    if (J > GEMV_MAX_J) continue;
    if (o.nc == 6 && J != 6 && J != 3) continue;  // instantiated (6, J) kernels
    const int npart = o.nslice * pair;
    if (o.nc % npart) continue;
    int rs = o.nc / npart;  // one item per warp per stage
    if (rs & (rs - 1)) continue;
    while (rs * 2 <= 128 && rs * 2 * K * pair <= GEMV_STAGE_TARGET / 2) rs *= 2;
    const int sb = rs * K * pair;
    if (sb > GEMV_SMEM_BUDGET / 2) continue;
    int ns = 2;
    while (ns < 8 && gemv_smem_layout(K, ns + 1, sb, rs, npart).total <= GEMV_SMEM_BUDGET) ++ns;
    const GemvSmem L2 = gemv_smem_layout(K, ns, sb, rs, npart);
    if (L2.total > 227 * 1024) continue;
    p.stream = true;
    p.nc = o.nc;
    p.j = J;
    p.nslice = o.nslice;
    p.npart = npart;
    p.rs = rs;
    p.nstages = ns;
    p.stage_bytes = sb;
    p.smem = L2.total;
    return true;
  }
  return false;
}

template <typename ST, int NC, int J>
static cudaError_t launch_stream_inst(const GemvArgs& a, const GemvPlan& p, cudaStream_t st, bool pdl) {
  auto kern = gemv_stream_kernel<ST, NC, J>;
  static bool attr_done[64] = {};
  const int d = current_device();
  if (!attr_done[d]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[d] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3((NC + 1) * 32);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <typename ST>
static cudaError_t launch_stream(const GemvArgs& a, const GemvPlan& p, cudaStream_t st, bool pdl) {
  if (p.nc == 8) {
    switch (p.j) {
      case 1: return launch_stream_inst<ST, 8, 1>(a, p, st, pdl);
      case 2: return launch_stream_inst<ST, 8, 2>(a, p, st, pdl);
      case 3: return launch_stream_inst<ST, 8, 3>(a, p, st, pdl);
      case 4: return launch_stream_inst<ST, 8, 4>(a, p, st, pdl);
      case 5: return launch_stream_inst<ST, 8, 5>(a, p, st, pdl);
      case 6: return launch_stream_inst<ST, 8, 6>(a, p, st, pdl);
    }
  } else if (p.nc == 6) {
    switch (p.j) {
      case 3: return launch_stream_inst<ST, 6, 3>(a, p, st, pdl);
      case 6: return launch_stream_inst<ST, 6, 6>(a, p, st, pdl);
    }
  }
  return cudaErrorInvalidConfiguration;
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
  bool paired = false, can_stream = aligned16(a.x) && !force_simple;
  int ntiles = 0;
  for (int s = 0; s < a.nseg; ++s) {
    const GemvSeg& sg = a.seg[s];
    if (sg.n < 0 || !sg.w || !sg.s) return cudaErrorInvalidValue;
    if (sg.epi != EPI_ARGMAX && sg.n > 0 && !sg.y) return cudaErrorInvalidValue;
    if (sg.epi == EPI_SILU_PAIR) {
      if (!sg.w2 || !sg.s2) return cudaErrorInvalidValue;
      paired = true;
      if (!aligned16(sg.w2)) can_stream = false;
    }
    if (sg.epi == EPI_CONV && (sg.cw < 1 || sg.cw > 8 || !sg.aux0 || !sg.aux2)) return cudaErrorInvalidValue;
    if (sg.epi == EPI_ARGMAX && !a.am_ws) return cudaErrorInvalidValue;
    if (!aligned16(sg.w)) can_stream = false;
  }
  if (paired) {
    for (int s = 0; s < a.nseg; ++s)
      if (a.seg[s].epi != EPI_SILU_PAIR) can_stream = false;  // one tile shape per launch
  }
  GemvPlan p;
  if (can_stream && plan_stream(a.K, paired, p)) {
    for (int s = 0; s < a.nseg; ++s) {
      a.seg[s].tile0 = ntiles;
      ntiles += (a.seg[s].n + p.rs - 1) / p.rs;
    }
    if (ntiles == 0) return cudaSuccess;
    a.ntiles = ntiles;
    a.rs = p.rs;
    a.npart = p.npart;
    a.nslice = p.nslice;
    a.nstages = p.nstages;
    a.stage_bytes = p.stage_bytes;
    const int sms = sm_count();
    p.grid = ntiles < sms ? ntiles : sms;
    return f32_scales ? launch_stream<float>(a, p, st, pdl) : launch_stream<bf16>(a, p, st, pdl);
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
