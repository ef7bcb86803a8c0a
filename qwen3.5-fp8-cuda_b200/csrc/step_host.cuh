// Host side of the persistent decode-step kernel (include/qwen_step.h):
// weight packing, program construction (unit partition of every stage,
// K-slice choice, the stage array in device memory) and the cooperative
// launch.  Included by libqwen_fused.cu after its status helpers.
#pragma once

#include "step.cuh"
#include "../../include/qwen_step.h"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <vector>

namespace {

struct StepProgramHost {
  int dev = 0;
  int grid = 0;
  int nstages = 0;
  qwen::StStage* d_stages = nullptr;
  unsigned long long* d_counters = nullptr;  // nstages stage counters + the completed-step count
  bool own_counters = true;                  // allocated here (one GPU) or in the caller's shared arena
  unsigned* d_abort = nullptr;
  int world = 1, rank = 0;
  long long peer_off[qwen::ST_MAX_WORLD] = {};
  unsigned* timeline = nullptr;    // optional per-stage timestamps (qwen_step_set_timeline)
  const int* pos = nullptr;        // the attention stages' position (all of them share one)
  int drop_stage = -1;             // test hook (qwen_step_set_drop)
  // workspaces a completed step leaves zeroed and an abandoned one may not:
  // ARGMAX {key, count} words and attention split counters (cleared by reset)
  std::vector<std::pair<void*, size_t>> scratch;
};

bool g_step_attr_done[64] = {};

cudaError_t step_kernel_attr(int dev) {
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (g_step_attr_done[dev]) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(qwen::step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       qwen::StSmem::total);
  if (e == cudaSuccess) g_step_attr_done[dev] = true;
  return e;
}

// Weight of one extra K slice in the slice-count choice, in chunks (each
// slice costs every CTA of the next stage one more FP32 row read at L2).
double step_slice_cost() {
  static double v = -1.0;
  if (v < 0.0) {
    const char* e = getenv("QWEN_STEP_SLICE_COST");
    v = e ? atof(e) : 2.0;
  }
  return v;
}

// K slices of a single-segment EPI_SLICES stage: a divisor of C that
// minimises the busiest CTA's chunks plus the slices' read cost.
int step_choose_slices(int tiles, int C, int grid, int max_slices = 16) {
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= C && s <= max_slices; ++s) {
    if (C % s) continue;
    const long long units = (long long)tiles * s;
    const long long per_cta = (units + grid - 1) / grid;
    const double cost = (double)(per_cta * (C / s)) + step_slice_cost() * s;
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

cudaError_t step_convert(const qwen_step_stage& in, qwen::StStage& o, int grid, int world,
                         const std::vector<qwen::StStage>& prev, const std::vector<qwen_step_stage>& prev_in) {
  using namespace qwen;
  o = StStage{};
  o.kind = in.kind;
  if (in.kind == QWEN_STEP_GEMV) {
    if (in.K <= 0 || in.K % ST_KC || in.K > ST_MAXK || in.nseg < 1 || in.nseg > ST_MAX_SEG)
      return cudaErrorInvalidValue;
    // BF16 weights: one segment, K a multiple of 256 that the BF16 x buffer holds
    if (in.wbf16 && (in.nseg != 1 || in.pair || in.K % 256 || in.K > ST_MAXK / 2)) return cudaErrorInvalidValue;
    if (in.pro < QWEN_STEP_PRO_PLAIN || in.pro > QWEN_STEP_PRO_SLICES_NORM) return cudaErrorInvalidValue;
    if (in.pro != QWEN_STEP_PRO_SLICES_NORM && !in.x) return cudaErrorInvalidValue;
    if (in.pro != QWEN_STEP_PRO_PLAIN && (!in.norm_w || in.K > ST_NORM_MAXK)) return cudaErrorInvalidValue;
    if (in.pro == QWEN_STEP_PRO_EMBED_NORM && (!in.token || in.x_rows <= 0)) return cudaErrorInvalidValue;
    if (in.pro == QWEN_STEP_PRO_SLICES_NORM && (!in.res || !in.sl_in || in.sl_stride < in.K))
      return cudaErrorInvalidValue;
    o.K = in.K;
    o.wbf16 = in.wbf16 ? 1 : 0;
    o.C = in.K / (o.wbf16 ? 256 : ST_KC);
    o.pro = in.pro;
    o.nseg = in.nseg;
    o.pair = in.pair ? 1 : 0;
    o.x = static_cast<const bf16*>(in.x);
    o.x_rows = in.x_rows;
    o.res = static_cast<const bf16*>(in.res);
    o.norm_w = in.norm_w;
    o.eps = in.eps;
    o.h_out = static_cast<bf16*>(in.h_out);
    o.token = in.token;
    o.sl_in = in.sl_in;
    o.sl_stride = in.sl_stride;
    o.sl_in_count = in.sl_in_count;
    o.sl_src = -1;
    if (in.pro == QWEN_STEP_PRO_SLICES_NORM) {
      // the latest earlier stage writing these rows: its slice count, and
      // whether they are tagged words from every rank (row-parallel stage)
      int src = -1;
      for (int i = (int)prev.size() - 1; i >= 0 && src < 0; --i)
        if (prev_in[i].sl_out == in.sl_in) src = i;
      if (src >= 0 && prev[src].xrank) {
        o.sl_src = src;
        o.sl_in_count = prev[src].nslice * world;
      } else if (o.sl_in_count <= 0) {
        if (src < 0) return cudaErrorInvalidValue;
        o.sl_in_count = prev[src].nslice;
      }
    }
    if (o.sl_in_count > 16) return cudaErrorInvalidValue;
    // a PLAIN GEMV over the previous GatedDeltaNet stage's output applies
    // that stage's gated RMSNorm in its prologue (whole heads of x)
    o.gated_pro = 0;
    if (in.pro == QWEN_STEP_PRO_PLAIN && !prev_in.empty() && prev_in.back().kind == QWEN_STEP_GDN &&
        prev_in.back().g_z) {
      const qwen_step_stage& g = prev_in.back();
      const long long off = static_cast<const char*>(in.x) - static_cast<const char*>(g.g_out);
      const long long head_bytes = (long long)g.g_dim * 2, span = (long long)g.g_heads * head_bytes;
      if (off >= 0 && off < span) {
        if (off % head_bytes || in.K % g.g_dim || off + 2LL * in.K > span || in.K > 4096 || in.wbf16)
          return cudaErrorInvalidValue;
        o.gated_pro = 1;
        o.gz = static_cast<const bf16*>(g.g_z) + off / 2;
        o.gnw = static_cast<const bf16*>(g.g_norm_w);
        o.geps = g.g_eps;
      }
    }
    o.am_ws = in.am_ws;
    o.am_key_out = in.am_key_out;
    o.am_token_out = in.am_token_out;
    o.pos_inc = in.pos_inc;
    int tiles = 0;
    bool slices = false, argmax = false;
    for (int i = 0; i < in.nseg; ++i) {
      const qwen_step_seg& s = in.seg[i];
      if (!s.w || s.n <= 0 || (o.pair && !s.w2)) return cudaErrorInvalidValue;
      switch (s.epi) {
        case QWEN_STEP_EPI_STORE:
        case QWEN_STEP_EPI_GATE_BETA:
        case QWEN_STEP_EPI_SILU:
          if (!s.y) return cudaErrorInvalidValue;
          break;
        case QWEN_STEP_EPI_SILU_PAIR:
          if (!s.y || !o.pair) return cudaErrorInvalidValue;
          break;
        case QWEN_STEP_EPI_ARGMAX:
          argmax = true;
          break;
        case QWEN_STEP_EPI_CONV:
          if (!s.y || !s.aux0 || !s.aux2 || s.cw < 1 || s.cw > 8) return cudaErrorInvalidValue;
          break;
        case QWEN_STEP_EPI_GATE_G:
          if (!s.y || !s.aux0 || !s.aux1) return cudaErrorInvalidValue;
          break;
        case QWEN_STEP_EPI_SLICES:
          slices = true;
          break;
        default:
          return cudaErrorInvalidValue;
      }
      if (o.pair && s.epi != QWEN_STEP_EPI_SILU_PAIR) return cudaErrorInvalidValue;
      GemvSeg& g = o.seg[i];
      g = GemvSeg{};
      g.w = static_cast<const uint8_t*>(s.w);
      g.w2 = static_cast<const uint8_t*>(s.w2);
      g.y = s.y;
      g.y2 = s.y2;
      g.aux0 = s.aux0;
      g.aux1 = s.aux1;
      g.aux2 = s.aux2;
      g.n = s.n;
      g.epi = s.epi == QWEN_STEP_EPI_SLICES ? EPI_SLICES : s.epi;
      g.cw = s.cw;
      g.row_offset = s.row_offset;
      o.seg_tile0[i] = tiles;
      tiles += (s.n + ST_ROWS - 1) / ST_ROWS;
    }
    for (int i = in.nseg; i <= ST_MAX_SEG; ++i) o.seg_tile0[i] = tiles;
    if (slices && (in.nseg != 1 || !in.sl_out || in.sl_rows < in.seg[0].n)) return cudaErrorInvalidValue;
    if (argmax && (!in.am_ws || in.nseg != 1)) return cudaErrorInvalidValue;
    o.tiles = tiles;
    // this rank's tiles (tensor parallel): [shard0, shard0 + shard_n)
    const int my_tiles = in.shard_n > 0 ? in.shard_n : tiles;
    if (in.shard0 < 0 || in.shard_n < 0 || in.shard0 + my_tiles > tiles) return cudaErrorInvalidValue;
    o.shard0 = in.shard_n > 0 ? in.shard0 : 0;
    int ns = 1;
    if (slices) {
      // (a cross-rank stage's W x nslice slices fill the 16 slice rows)
      const int cap = (world > 1 && in.xrank) ? 16 / world : 16;
      ns = in.nslice > 0 ? in.nslice : step_choose_slices(my_tiles, o.C, grid, cap);
      if (o.C % ns || ns > 16) return cudaErrorInvalidValue;
      o.sl_out = in.sl_out;
      o.sl_rows = in.sl_rows;
    } else if (in.nslice > 1) {
      return cudaErrorInvalidValue;
    }
    o.nslice = ns;
    o.nunits = my_tiles * ns;
    // tensor parallel: a row-parallel stage (this rank's K range, every row)
    // writes its K-slice rows to every rank as tagged words
    o.xrank = (world > 1 && in.xrank) ? 1 : 0;
    if (o.xrank && (!slices || ns * world > 16)) return cudaErrorInvalidValue;
    o.cstride = in.cstride > 0 ? in.cstride : o.C;
    if (o.cstride < o.C) return cudaErrorInvalidValue;
    o.ipu = (o.C / ns) * (o.pair ? 2 : 1);
    if (o.ipu > ST_BATCH) return cudaErrorInvalidValue;
    return cudaSuccess;
  }
  if (in.kind == QWEN_STEP_GDN) {
    if (in.g_dim != ST_GDN_D || in.g_heads <= 0 || in.g_rep <= 0 || !in.g_q || !in.g_k || !in.g_v || !in.g_g ||
        !in.g_beta || !in.g_state || !in.g_out)
      return cudaErrorInvalidValue;
    if ((in.g_z == nullptr) != (in.g_norm_w == nullptr)) return cudaErrorInvalidValue;
    GdnArgs& a = o.gdn;
    a = GdnArgs{};
    a.q = static_cast<const bf16*>(in.g_q);
    a.k = static_cast<const bf16*>(in.g_k);
    a.v = static_cast<const bf16*>(in.g_v);
    a.g = in.g_g;
    a.beta = static_cast<const bf16*>(in.g_beta);
    a.state = in.g_state;
    a.out = static_cast<bf16*>(in.g_out);
    a.z = static_cast<const bf16*>(in.g_z);
    a.norm_w = static_cast<const bf16*>(in.g_norm_w);
    a.eps = in.g_eps;
    a.rep = in.g_rep;
    a.gated = in.g_z != nullptr;
    if (in.shard0 < 0 || in.shard_n < 0 || in.shard0 + (in.shard_n > 0 ? in.shard_n : in.g_heads) > in.g_heads)
      return cudaErrorInvalidValue;
    o.gdn_heads = in.shard_n > 0 ? in.shard_n : in.g_heads;
    o.shard0 = in.shard_n > 0 ? in.shard0 : 0;
    return cudaSuccess;
  }
  if (in.kind == QWEN_STEP_ATTN) {
    if (in.a_kv <= 0 || in.a_heads <= 0 || in.a_heads % in.a_kv || in.a_nsplit < 1 || in.a_chunk < 1)
      return cudaErrorInvalidValue;
    if (!in.a_q || !in.a_k_new || !in.a_v_new || !in.a_k_cache || !in.a_v_cache || !in.a_pos || !in.a_out)
      return cudaErrorInvalidValue;
    if (in.a_nsplit > 1 && (!in.a_ws || !in.a_cnt)) return cudaErrorInvalidValue;
    if (in.a_cos && (in.a_rot <= 0 || in.a_rot > in.a_dim || in.a_rot % 2)) return cudaErrorInvalidValue;
    const int G = in.a_heads / in.a_kv;
    const int smem = 4 * (G * in.a_dim + ATTN_WARPS * G * in.a_dim + 2 * ATTN_WARPS * G + 2 * in.a_dim +
                          ATTN_WARPS * in.a_dim);
    if (in.a_dim != 256 || G != 4 || smem > ST_ATTN_SLOTS * ST_CHUNK) return cudaErrorNotSupported;
    AttnArgs& a = o.attn;
    a = AttnArgs{};
    a.q = static_cast<const bf16*>(in.a_q);
    a.gate = a.q + in.a_dim;
    a.k_new = static_cast<const bf16*>(in.a_k_new);
    a.v_new = static_cast<const bf16*>(in.a_v_new);
    a.q_norm = in.a_q_norm;
    a.k_norm = in.a_k_norm;
    a.cos = in.a_cos;
    a.sin = in.a_sin;
    a.k_cache = static_cast<bf16*>(in.a_k_cache);
    a.v_cache = static_cast<bf16*>(in.a_v_cache);
    a.pos_ptr = in.a_pos;
    a.q_stride = 2 * in.a_dim;
    a.max_seq = in.a_max_seq;
    a.n_heads = in.a_heads;
    a.n_kv = in.a_kv;
    a.rot = in.a_rot;
    a.eps = in.a_eps;
    a.prep = 1;
    a.chunk = in.a_chunk;
    a.nsplit = in.a_nsplit;
    a.ws_part = in.a_ws;
    a.ws_count = in.a_cnt;
    a.out = static_cast<bf16*>(in.a_out);
    o.attn_dim = in.a_dim;
    o.attn_g = G;
    if (in.shard0 < 0 || in.shard_n < 0 || in.shard0 + (in.shard_n > 0 ? in.shard_n : in.a_kv) > in.a_kv)
      return cudaErrorInvalidValue;
    o.attn_kv = in.shard_n > 0 ? in.shard_n : in.a_kv;
    o.shard0 = in.shard_n > 0 ? in.shard0 : 0;
    return cudaSuccess;
  }
  return cudaErrorInvalidValue;
}

}  // namespace

extern "C" {

size_t qwen_step_packed_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || K % qwen::ST_KC) return 0;
  return (size_t)((N + qwen::ST_ROWS - 1) / qwen::ST_ROWS) * (size_t)(K / qwen::ST_KC) * qwen::ST_CHUNK;
}

size_t qwen_step_packed_bytes_bf16(int N, int K) {
  if (N <= 0 || K <= 0 || K % 256) return 0;
  return (size_t)((N + qwen::ST_ROWS - 1) / qwen::ST_ROWS) * (size_t)(K / 256) * qwen::ST_CHUNK;
}

int qwen_step_pack_bf16(const void* w, int N, int K, void* out, cudaStream_t stream) {
  if (!w || !out || N <= 0 || K <= 0 || K % 256) return record(cudaErrorInvalidValue);
  const long long words = (long long)((N + qwen::ST_ROWS - 1) / qwen::ST_ROWS) * (K / 256) * (qwen::ST_CHUNK / 4);
  const int block = 256;
  const long long want = (words + block - 1) / block;
  const int grid = (int)(want < 65535 ? want : 65535);
  qwen::step_pack_bf16_kernel<<<grid, block, 0, stream>>>(static_cast<const qwen::bf16*>(w), N, K,
                                                          static_cast<uint8_t*>(out));
  return record(cudaGetLastError());
}

int qwen_step_pack(const void* w, const void* s, int scale_f32, int N, int K, int K_blk, void* out,
                   cudaStream_t stream) {
  if (!w || !s || !out || N <= 0 || K <= 0 || K % qwen::ST_KC || K_blk != K / 128)
    return record(cudaErrorInvalidValue);
  const long long items = (long long)((N + 15) / 16) * (K / qwen::ST_KC) * (qwen::ST_WBYTES / 16 + 1);
  const int block = 256;
  const long long want = (items + block - 1) / block;
  const int grid = (int)(want < 65535 ? want : 65535);
  if (scale_f32)
    qwen::step_pack_kernel<float><<<grid, block, 0, stream>>>(static_cast<const uint8_t*>(w), s, N, K, K_blk,
                                                              static_cast<uint8_t*>(out));
  else
    qwen::step_pack_kernel<qwen::bf16><<<grid, block, 0, stream>>>(static_cast<const uint8_t*>(w), s, N, K, K_blk,
                                                                   static_cast<uint8_t*>(out));
  return record(cudaSuccess);
}

// Shared by qwen_step_create (one GPU) and qwen_step_create_tp.  `counters`:
// null to allocate the 2 nstages + 1 u64 counters here, else the caller's
// (inside the shared arena, zeroed).
static int step_create_impl(const qwen_step_stage* stages, int nstages, int world, int rank,
                            void* const* peer_bases, const void* local_base, unsigned long long* counters,
                            void** program_out) {
  if (!stages || nstages <= 0 || !program_out) return record(cudaErrorInvalidValue);
  if (world < 1 || world > qwen::ST_MAX_WORLD || rank < 0 || rank >= world) return record(cudaErrorInvalidValue);
  if (world > 1 && (!peer_bases || !local_base || !counters)) return record(cudaErrorInvalidValue);
  *program_out = nullptr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record(e);
  int sms = 0, coop = 0;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return record(e);
  if ((e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess) return record(e);
  if (!coop) return record(cudaErrorNotSupported);
  if ((e = step_kernel_attr(dev)) != cudaSuccess) return record(e);
  int per_sm = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qwen::step_kernel, qwen::ST_THREADS,
                                                         qwen::StSmem::total)) != cudaSuccess)
    return record(e);
  if (per_sm < 1) return record(cudaErrorInvalidConfiguration);
  const int grid = sms;  // one CTA per SM: the ring takes the SM's shared memory
  std::vector<qwen::StStage> conv;
  std::vector<qwen_step_stage> ins;
  conv.reserve(nstages);
  for (int i = 0; i < nstages; ++i) {
    qwen::StStage o;
    e = step_convert(stages[i], o, grid, world, conv, ins);
    if (e != cudaSuccess) return record(e);
    conv.push_back(o);
    ins.push_back(stages[i]);
  }
  // a gated GatedDeltaNet stage leaves the gated RMSNorm to the GEMV after it
  for (int i = 0; i < nstages; ++i)
    if (stages[i].kind == QWEN_STEP_GDN && stages[i].g_z && (i + 1 >= nstages || !conv[i + 1].gated_pro))
      return record(cudaErrorInvalidValue);
  const int* pos = nullptr;
  for (int i = 0; i < nstages; ++i)
    if (stages[i].kind == QWEN_STEP_ATTN) {
      if (pos && stages[i].a_pos != pos) return record(cudaErrorInvalidValue);  // one position per program
      pos = stages[i].a_pos;
    }
  StepProgramHost* p = new StepProgramHost();
  p->dev = dev;
  p->pos = pos;
  p->grid = grid;
  p->nstages = nstages;
  p->world = world;
  p->rank = rank;
  for (int r = 0; r < world; ++r)
    p->peer_off[r] = world > 1 ? (long long)(static_cast<const char*>(peer_bases[r]) -
                                             static_cast<const char*>(local_base))
                               : 0ll;
  for (int i = 0; i < nstages; ++i) {
    const qwen_step_stage& st = stages[i];
    auto add = [&](void* ptr, size_t bytes) {
      for (auto& e2 : p->scratch)
        if (e2.first == ptr) return;
      p->scratch.emplace_back(ptr, bytes);
    };
    if (st.kind == QWEN_STEP_GEMV && st.am_ws) add(st.am_ws, 2 * sizeof(unsigned long long));
    // tagged slice words: a reset program restarts its tags, so old words must not match
    if (st.kind == QWEN_STEP_GEMV && conv[i].xrank) add(st.sl_out, sizeof(unsigned long long) * 16 * (size_t)st.sl_rows);
    if (st.kind == QWEN_STEP_ATTN && st.a_cnt) add(st.a_cnt, sizeof(unsigned) * st.a_kv);
  }
  const size_t cbytes = sizeof(unsigned long long) * (2 * nstages + 1);
  e = cudaMalloc(&p->d_stages, sizeof(qwen::StStage) * nstages);
  if (e == cudaSuccess) e = cudaMalloc(&p->d_abort, sizeof(unsigned));
  if (e == cudaSuccess && counters) {
    p->d_counters = counters;
    p->own_counters = false;
  } else if (e == cudaSuccess) {
    e = cudaMalloc(&p->d_counters, cbytes);
  }
  if (e == cudaSuccess)
    e = cudaMemcpy(p->d_stages, conv.data(), sizeof(qwen::StStage) * nstages, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(p->d_counters, 0, cbytes);
  if (e == cudaSuccess) e = cudaMemset(p->d_abort, 0, sizeof(unsigned));
  if (e != cudaSuccess) {
    cudaFree(p->d_stages);
    cudaFree(p->d_abort);
    if (p->own_counters) cudaFree(p->d_counters);
    delete p;
    return record(e);
  }
  *program_out = p;
  return 0;
}

int qwen_step_create(const qwen_step_stage* stages, int nstages, void** program_out) {
  return step_create_impl(stages, nstages, 1, 0, nullptr, nullptr, nullptr, program_out);
}

int qwen_step_create_tp(const qwen_step_stage* stages, int nstages, int world, int rank, void* const* peer_bases,
                        const void* local_base, void* counters, void** program_out) {
  return step_create_impl(stages, nstages, world, rank, peer_bases, local_base,
                          static_cast<unsigned long long*>(counters), program_out);
}

size_t qwen_step_counter_bytes(int nstages) {
  return nstages > 0 ? sizeof(unsigned long long) * (size_t)(2 * nstages + 1) : 0;
}

int qwen_ipc_alloc(size_t bytes, void** base_out, void* ipc_handle_out) {
  if (bytes == 0 || !base_out || !ipc_handle_out) return record(cudaErrorInvalidValue);
  void* base = nullptr;
  cudaError_t e = cudaMalloc(&base, bytes);
  if (e != cudaSuccess) return record(e);
  e = cudaMemset(base, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) {
    cudaFree(base);
    return record(e);
  }
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  *base_out = base;
  return 0;
}

int qwen_step_launch(void* program, cudaStream_t stream) {
  StepProgramHost* p = static_cast<StepProgramHost*>(program);
  if (!p) return record(cudaErrorInvalidValue);
  qwen::StProgram P;
  P.stages = p->d_stages;
  P.nstages = p->nstages;
  P.counters = p->d_counters;
  P.abort_flag = p->d_abort;
  P.world = p->world;
  P.rank = p->rank;
  for (int r = 0; r < qwen::ST_MAX_WORLD; ++r) P.peer_off[r] = p->peer_off[r];
  P.timeline = p->timeline;
  P.pos = p->pos;
  P.drop_stage = p->drop_stage;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p->grid);
  cfg.blockDim = dim3(qwen::ST_THREADS);
  cfg.dynamicSmemBytes = qwen::StSmem::total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return record(cudaLaunchKernelEx(&cfg, qwen::step_kernel, P));
}

int qwen_step_reset(void* program, cudaStream_t stream) {
  StepProgramHost* p = static_cast<StepProgramHost*>(program);
  if (!p) return record(cudaErrorInvalidValue);
  cudaError_t e = cudaMemsetAsync(p->d_counters, 0, sizeof(unsigned long long) * (2 * p->nstages + 1), stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(p->d_abort, 0, sizeof(unsigned), stream);
  for (size_t i = 0; i < p->scratch.size() && e == cudaSuccess; ++i)
    e = cudaMemsetAsync(p->scratch[i].first, 0, p->scratch[i].second, stream);
  return record(e);
}

int qwen_step_set_drop(void* program, int stage) {
  StepProgramHost* p = static_cast<StepProgramHost*>(program);
  if (!p || stage < -1 || stage >= p->nstages) return record(cudaErrorInvalidValue);
  p->drop_stage = stage;
  return 0;
}

int qwen_step_destroy(void* program) {
  StepProgramHost* p = static_cast<StepProgramHost*>(program);
  if (!p) return 0;
  cudaFree(p->d_stages);
  cudaFree(p->d_abort);
  if (p->own_counters) cudaFree(p->d_counters);
  delete p;
  return 0;
}

int qwen_step_set_timeline(void* program, unsigned* timeline) {
  StepProgramHost* p = static_cast<StepProgramHost*>(program);
  if (!p) return record(cudaErrorInvalidValue);
  p->timeline = timeline;
  return 0;
}

int qwen_step_grid(void* program) {
  StepProgramHost* p = static_cast<StepProgramHost*>(program);
  return p ? p->grid : 0;
}

int qwen_step_smem_bytes(void) { return qwen::StSmem::total; }

}  // extern "C"
