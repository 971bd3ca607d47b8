// tsg_api.cu -- the C ABI of libtsugumi_cuda.so (include/tsugumi_cuda.h).
//
// Host-side mirror of the reference's encoder classes: a context plays the
// part of MetalContext plus the kernel objects' owned scratch
// (MoE.swift:184-198 router logits and argument buffer), a layer holds the
// resident weights the Swift runners keep per layer.  Every entry point
// validates its arguments the way the reference's preconditions and throws
// do, then enqueues kernels on the context's stream.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/tsugumi_cuda.h"
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

using namespace tsg;

namespace {

// Workspace capacity in elements of each dimension.
struct Caps {
  uint32_t T = 0, D = 0, F = 0, E = 0, K = 0;
  uint32_t dense = 0;  // 1: a layer with a dense branch (its routed result is staged in f32)
  uint32_t fusion = 0;  // 1: the Gemma fused entry's block inputs and branch outputs
  bool covers(const Caps& o) const {
    return T >= o.T && D >= o.D && F >= o.F && E >= o.E && K >= o.K && dense >= o.dense &&
           fusion >= o.fusion;
  }
  Caps max_with(const Caps& o) const {
    Caps c;
    c.T = std::max(T, o.T);
    c.D = std::max(D, o.D);
    c.F = std::max(F, o.F);
    c.E = std::max(E, o.E);
    c.K = std::max(K, o.K);
    c.dense = std::max(dense, o.dense);
    c.fusion = std::max(fusion, o.fusion);
    return c;
  }
};

constexpr int kMaxSplit = 8;

}  // namespace

struct tsg_ctx_s {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  // the streaming decode kernel up to T = 3; at T = 4 the batched GEMVs
  // measured faster (Gemma-like 58.5 against 68.5 us a layer)
  uint32_t decode_max_tokens = 3;
  uint32_t gemv_max_tokens = 16;  // router-driven batches up to this size use the batched GEMVs
  std::string last_error;
  // workspace
  void* ws = nullptr;
  size_t ws_bytes = 0;
  Caps caps;
  RouteBuffers rb{};
  __half* act_buf = nullptr;
  __half* xp = nullptr;
  __half* partials = nullptr;
  float* dense_y = nullptr;  // [T][D] f32: a dense-branch layer's routed result
  // the Gemma fused entry: [T][D] bf16 router, routed and dense inputs; [T][D]
  // f32 routed and dense outputs
  uint16_t* fx_in = nullptr;
  float* fx_out = nullptr;
  // fused decode scratch
  void* f_logits = nullptr;  // fused decode: tagged logits
  size_t f_logits_bytes = 0;
  void* f_actfrag = nullptr;
  uint32_t* f_counters = nullptr;
  void* f_stream = nullptr;        // streaming decode: act fragments, sums, partials
  uint32_t* f_flags = nullptr;     // streaming decode: act flags (launch tags)
  size_t f_flags_bytes = 0;
  bool use_fused = true;
  int fused_kind = 1;              // 1: streaming decode kernel, 2: the earlier fused kernel
  bool allow_pdl = true;  // programmatic dependent launch of the decode kernels
  bool cooperative = true;  // decode kernels launched with the cooperative attribute
  unsigned long long* stamps = nullptr;  // debug phase timestamps (device)
  // device status words: [0] error bits, [1] code, [2] value, [3] pad;
  // [4] last-CTA counter
  uint32_t* status = nullptr;
  // last call's routing
  uint32_t last_T = 0, last_K = 0;
  // stage profiling: 5 events per recorded call
  std::vector<cudaEvent_t> prof_events;
  uint32_t prof_max = 0, prof_calls = 0;
  bool profiling = false;
  // expert parallelism
  void* nccl_comm = nullptr;  // ncclComm_t
  int ep_rank = 0, ep_world = 1;
  size_t ep_rows_cap = 0;            // rows of ep_rows / ep_act / ep_out
  __half* ep_rows = nullptr;         // received rows (+ own shared rows) [cap][D]
  __half* ep_act = nullptr;          // [cap][F]
  __half* ep_out = nullptr;          // local expert outputs [cap][D]
  __half* ep_ret = nullptr;          // returned outputs in this rank's sorted order [cap][D]
  size_t ep_ret_cap = 0;
  uint32_t* ep_counts_recv = nullptr;  // device: [512] received counts, [512] sent counts,
                                       // [2][world] received status words, [2] own status words
  uint32_t* ep_h_counts = nullptr;     // pinned: [E] sent counts, [E] received, [world] statuses
  RowTile* ep_tiles = nullptr;         // device row-tile schedule
  RowTile* ep_h_tiles = nullptr;       // pinned staging
  uint32_t* ep_ntiles = nullptr;       // device [1] (follows ep_tiles' capacity)
  size_t ep_tiles_cap = 0;
  // peer-memory transport (ep_transport 1).  Buffers, by kind (EpBuf):
  // the pair rows expanded for the contraction (then this rank's
  // shared-expert rows) and their activations, local; and the three that
  // peers write -- the returned outputs in this rank's sorted order (then its
  // shared rows), the token rows received (one per token and owner) and the
  // map from each received pair to its token row.  ep_caps holds every
  // rank's capacities, the same on every rank (each is a function of the
  // exchanged counts); ep_peer the views of the peers' buffers.
  int ep_transport = 1;                // 0: NCCL all-to-all; 1: peer memory
  int ep_dispatch = 0;                 // 0: rows stored by the dispatch kernel; 1: staged and copied
  void* ep_buf[6] = {};
  size_t ep_buf_elems[6] = {};         // this rank's allocations
  std::vector<size_t> ep_caps[7];      // [kind][world] elements; [6]: row tiles
  std::vector<void*> ep_peer[6];       // [kind][world]; own entry = own buffer
  uint32_t* ep_slots = nullptr;        // [world][T] token slots per owner
  size_t ep_slots_cap = 0;
  uint32_t* ep_ag = nullptr;           // device: send [kAgWords], receive [world][kAgWords], barriers
  uint32_t* ep_h_ag = nullptr;         // pinned copy of the received words
  RowTile* ep_ptiles = nullptr;        // device row tiles, then their count
  RowTile* ep_h_ptiles = nullptr;      // pinned staging
  uint32_t* ep_pntiles = nullptr;      // device [1] (follows ep_ptiles' capacity)
  size_t ep_ptiles_cap = 0;
  unsigned long long* ep_tile_out = nullptr;    // device [ep_ptiles_cap]: per tile, rows' destination
  unsigned long long* ep_h_tile_out = nullptr;  // pinned staging
  cudaEvent_t ep_ev[9] = {};           // phase boundaries of the last call (peer transport)
  // the return through the copy engines (ep_return 1): GEMM2 runs in chunks,
  // one per source rank, into local rows, and a second stream copies each
  // finished chunk into its rank's buffer while the next chunk computes
  int ep_return = 1;                   // 0: GEMM2's epilogue stores into the peers' buffers
  cudaStream_t ep_copy = nullptr;
  cudaEvent_t ep_chunk_ev[kEpMaxRanks + 1] = {};
  bool ep_chunk_ok = false;
  bool ep_ev_ok = false;
};

struct tsg_moe_layer_s {
  tsg_ctx ctx = nullptr;
  tsg_moe_layer_desc desc{};
  float* router_rows = nullptr;  // [E + has_gate][D], owned
  void* router_w3 = nullptr;     // [3][router_tc_pad(E)][D] bf16 planes of the first E rows, owned
  int has_gate = 0;
  int has_shared = 0;
  DecodeMaps dmaps{};       // down-slice tensor maps of the streaming decode kernel
  bool dmaps_ok = false;
  // the dense branch (a shared int4 MLP whose F differs from the experts',
  // Gemma's dense MLP): a one-expert view of it, run beside the routed
  // experts and added to their result; owned
  tsg_moe_layer_s* dense = nullptr;
};

EncodeTiledFn tsg::encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

namespace {

tsg_status fail(tsg_ctx ctx, tsg_status st, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return st;
}

tsg_status cuda_fail(tsg_ctx ctx, cudaError_t e, const char* where) {
  return fail(ctx, e == cudaErrorMemoryAllocation ? TSG_ERR_OOM : TSG_ERR_CUDA,
              std::string(where) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) +
                  ")");
}

#define TSG_CUDA_TRY(ctx, expr, where)                 \
  do {                                                 \
    cudaError_t e__ = (expr);                          \
    if (e__ != cudaSuccess) return cuda_fail(ctx, e__, where); \
  } while (0)

// Rows a prefill schedule can need: one tile per tile_rows routed rows plus
// one partial tile per expert, plus the shared expert's tiles.
uint32_t max_row_tiles(uint32_t T, uint32_t K, uint32_t E, uint32_t tile_rows) {
  return (T * K + tile_rows - 1) / tile_rows + E + (T + tile_rows - 1) / tile_rows + 1;
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Per-CTA launch epochs and gate/up flags of the fused decode kernel.
constexpr size_t kFusedSignalBytes = 2 * 256 * sizeof(uint32_t);

// Zeroes the fused decode kernel's signals (epochs, flags, tagged logits):
// at allocation, and after a launch that reported an error, since such a
// launch may leave CTAs at different epochs.
cudaError_t reset_fused_signals(tsg_ctx ctx) {
  cudaError_t e = cudaMemset(ctx->f_counters, 0, kFusedSignalBytes);
  if (e == cudaSuccess && ctx->f_logits) e = cudaMemset(ctx->f_logits, 0, ctx->f_logits_bytes);
  if (e == cudaSuccess && ctx->f_flags) e = cudaMemset(ctx->f_flags, 0, ctx->f_flags_bytes);
  return e;
}

// Carves the workspace; with base == nullptr only returns the size.
size_t carve(tsg_ctx ctx, const Caps& c, uint8_t* base) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    off = align_up(off, 256);
    void* p = base ? base + off : nullptr;
    off += bytes;
    return p;
  };
  const size_t T = c.T, D = c.D, F = c.F, E = c.E, K = c.K;
  const size_t P = T * K;
  const size_t rows = P + T;
  RouteBuffers rb{};
  rb.logits_raw = static_cast<float*>(take(kMaxSplit * T * E * 4));
  rb.gate_raw = static_cast<float*>(take(T * 4));
  rb.sumsq = static_cast<float*>(take(kMaxSplit * T * 4));
  rb.inv_rms = static_cast<float*>(take(T * 4));
  rb.ids = static_cast<uint32_t*>(take(P * 4));
  rb.weights = static_cast<float*>(take(P * 4));
  rb.weights_f16 = static_cast<uint16_t*>(take(P * 2));
  rb.counts = static_cast<uint32_t*>(take(E * 4));
  rb.offsets = static_cast<uint32_t*>(take(E * 4));
  rb.sorted_pairs = static_cast<Pair*>(take(P * sizeof(Pair)));
  rb.pair_pos = static_cast<uint32_t*>(take(P * 4));
  rb.groups = static_cast<Group*>(take(E * sizeof(Group)));
  rb.n_groups = static_cast<uint32_t*>(take(4));
  rb.tiles = static_cast<Tile*>(take(E * sizeof(Tile)));
  rb.n_tiles = static_cast<uint32_t*>(take(4));
  const uint32_t tr = static_cast<uint32_t>(qmm_tile_rows());
  rb.row_tiles = static_cast<RowTile*>(
      take(max_row_tiles(static_cast<uint32_t>(T), static_cast<uint32_t>(K),
                         static_cast<uint32_t>(E), tr) * sizeof(RowTile)));
  rb.n_row_tiles = static_cast<uint32_t*>(take(4));
  rb.hist = static_cast<uint32_t*>(
      take(static_cast<size_t>(permute_chunks(static_cast<int>(P))) * E * 4));
  const size_t Td = std::min<size_t>(T, 64);
  rb.xn = static_cast<float*>(take(Td * D * 4));
  rb.xs8 = static_cast<float*>(take(Td * (D / 8) * 4));
  __half* act = static_cast<__half*>(take(rows * F * 2));
  __half* xp = static_cast<__half*>(take(rows * D * 2));
  __half* part = static_cast<__half*>(take(rows * D * 2));
  float* dense_y = static_cast<float*>(take(c.dense ? T * D * 4 : 0));
  uint16_t* fx_in = static_cast<uint16_t*>(take(c.fusion ? 3 * T * D * 2 : 0));
  float* fx_out = static_cast<float*>(take(c.fusion ? 2 * T * D * 4 : 0));
  // fused decode (T <= 4)
  const size_t Tf = std::min<size_t>(T, 4);
  const size_t rows_f = Tf * K + Tf;
  // fused decode: (tag, logit) words in 4 copies, and the per-CTA signals
  void* f_logits = take(4 * Tf * (E + 1) * 8);
  void* f_actfrag = take(rows_f * F * 2);
  uint32_t* f_counters = static_cast<uint32_t*>(take(kFusedSignalBytes));
  // streaming decode: data scratch and act flags
  const size_t fs_bytes = decode_stream_scratch_bytes(static_cast<int>(Tf), static_cast<int>(D),
                                                      static_cast<int>(F), static_cast<int>(K));
  const size_t ff_bytes =
      decode_stream_flag_bytes(static_cast<int>(Tf), static_cast<int>(F), static_cast<int>(K));
  void* f_stream = take(fs_bytes);
  uint32_t* f_flags = static_cast<uint32_t*>(take(ff_bytes));
  if (base) {
    ctx->f_stream = f_stream;
    ctx->f_flags = f_flags;
    ctx->f_flags_bytes = ff_bytes;
    ctx->f_logits = f_logits;
    ctx->f_logits_bytes = 4 * Tf * (E + 1) * 8;
    ctx->f_actfrag = f_actfrag;
    ctx->f_counters = f_counters;
    rb.sync_counter = ctx->status + 4;
    rb.err = ctx->status;
    ctx->rb = rb;
    ctx->act_buf = act;
    ctx->xp = xp;
    ctx->partials = part;
    ctx->dense_y = c.dense ? dense_y : nullptr;
    ctx->fx_in = c.fusion ? fx_in : nullptr;
    ctx->fx_out = c.fusion ? fx_out : nullptr;
  }
  return align_up(off, 256);
}

tsg_status ensure_workspace(tsg_ctx ctx, const Caps& want) {
  if (ctx->ws && ctx->caps.covers(want)) return TSG_OK;
  const Caps c = ctx->caps.max_with(want);
  const size_t bytes = carve(ctx, c, nullptr);
  TSG_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  if (ctx->ws) {
    TSG_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    cudaFree(ctx->ws);
    ctx->ws = nullptr;
  }
  void* p = nullptr;
  TSG_CUDA_TRY(ctx, cudaMalloc(&p, bytes), "cudaMalloc(workspace)");
  ctx->ws = p;
  ctx->ws_bytes = bytes;
  ctx->caps = c;
  carve(ctx, c, static_cast<uint8_t*>(p));
  // the fused decode kernel's launch epochs, flags and tags start at zero
  TSG_CUDA_TRY(ctx, reset_fused_signals(ctx), "cudaMemset");
  return TSG_OK;
}

Caps layer_caps(const tsg_moe_layer_s* L, uint32_t T) {
  Caps c;
  c.T = T;
  c.D = L->desc.d;
  c.F = L->desc.f;
  c.E = L->desc.num_experts;
  c.K = std::max<uint32_t>(L->desc.top_k, 1);
  if (L->dense) {
    c.F = std::max(c.F, L->dense->desc.f);
    c.dense = 1;
  }
  return c;
}

RouterParams router_params(const tsg_moe_layer_s* L, const void* x, uint32_t x_stride,
                           uint32_t T) {
  RouterParams p{};
  p.x = static_cast<const uint16_t*>(x);
  p.x_stride = x_stride;
  p.T = static_cast<int>(T);
  p.D = static_cast<int>(L->desc.d);
  p.E = static_cast<int>(L->desc.num_experts);
  p.K = static_cast<int>(L->desc.top_k);
  p.w = L->router_rows;
  p.w_bf16x3 = L->router_w3;
  p.has_gate = L->has_gate;
  p.has_shared = L->has_shared;
  p.per_expert_scale = L->desc.per_expert_scale;
  p.logit_bias = L->desc.logit_bias;
  p.norm = L->desc.router_norm ? 1 : 0;
  p.eps = L->desc.norm_eps;
  p.tile_rows = qmm_tile_rows();
  p.tile_expert_count = 16;
  p.tile_break = -1;
  p.sort_keys = nullptr;
  return p;
}

ExpertSet expert_set(const tsg_moe_layer_s* L) {
  ExpertSet s{};
  s.base = static_cast<const uint8_t*>(L->desc.experts);
  s.stride = L->desc.expert_stride;
  std::memcpy(&s.off, &L->desc.offsets, sizeof(ExpertOffsets));
  s.shared = static_cast<const uint8_t*>(L->desc.shared_expert);
  std::memcpy(&s.shared_off, &L->desc.shared_offsets, sizeof(ExpertOffsets));
  return s;
}


// Records stage boundary `k` (0..4) of the current profiled call.  Inside
// stream capture the record must be "external" to become a graph node that
// every replay re-records (a plain record there only orders streams);
// outside capture a plain record is used.  Profiling never leaves an error
// behind: on failure it switches itself off.
void prof_mark(tsg_ctx ctx, int k) {
  if (!ctx->profiling || ctx->prof_calls >= ctx->prof_max) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(ctx->stream, &cs);
  cudaEvent_t ev = ctx->prof_events[ctx->prof_calls * 5 + k];
  if (e == cudaSuccess) {
    e = cs == cudaStreamCaptureStatusActive
            ? cudaEventRecordWithFlags(ev, ctx->stream, cudaEventRecordExternal)
            : cudaEventRecord(ev, ctx->stream);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    ctx->profiling = false;
  }
}

// A CUDA error left pending by earlier work (ours or the caller's) would be
// misattributed to the next launch; report it at the entry instead.
tsg_status take_pending_error(tsg_ctx ctx) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return TSG_OK;
  return fail(ctx, TSG_ERR_CUDA, std::string("error pending from earlier CUDA work: ") +
                                     cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

bool valid_dtype(tsg_dtype t) { return t == TSG_DTYPE_BF16 || t == TSG_DTYPE_F32; }

// ---- the two regimes ----

tsg_status run_decode_experts(tsg_ctx ctx, tsg_moe_layer_s* L, const void* x, uint32_t x_stride,
                              uint32_t T, const float* residual, void* y, uint32_t y_stride,
                              tsg_dtype y_dtype) {
  DecodeParams dp{};
  dp.T = static_cast<int>(T);
  dp.D = static_cast<int>(L->desc.d);
  dp.F = static_cast<int>(L->desc.f);
  dp.E = static_cast<int>(L->desc.num_experts);
  dp.K = static_cast<int>(L->desc.top_k);
  dp.act = static_cast<int>(L->desc.activation);
  dp.has_shared = L->has_shared;
  dp.x = static_cast<const uint16_t*>(x);
  dp.x_stride = x_stride;
  dp.experts = expert_set(L);
  dp.rb = ctx->rb;
  if (!L->has_gate) dp.rb.gate_raw = nullptr;
  dp.act_buf = ctx->act_buf;
  dp.xn = ctx->rb.xn;
  dp.xs8 = ctx->rb.xs8;
  dp.y = y;
  dp.y_stride = y_stride;
  dp.y_f32 = y_dtype == TSG_DTYPE_F32 ? 1 : 0;
  dp.residual = residual;
  dp.num_sms = ctx->num_sms;
  TSG_CUDA_TRY(ctx, launch_decode_gate_up(dp, ctx->stream), "decode gate/up");
  prof_mark(ctx, 2);
  TSG_CUDA_TRY(ctx, launch_decode_down(dp, ctx->stream), "decode down");
  prof_mark(ctx, 3);
  prof_mark(ctx, 4);
  return TSG_OK;
}

bool stream_ok(tsg_ctx ctx, const tsg_moe_layer_s* L, uint32_t T);

tsg_status run_decode_fused(tsg_ctx ctx, tsg_moe_layer_s* L, const void* x, uint32_t x_stride,
                            uint32_t T, const uint32_t* ids_in, const float* w_in,
                            const float* residual, void* y, uint32_t y_stride, tsg_dtype y_dtype,
                            uint32_t* ids_out, float* w_out, uint16_t* w16_out) {
  DecodeFusedArgs a{};
  a.x = static_cast<const uint16_t*>(x);
  a.x_stride = x_stride;
  a.T = static_cast<int>(T);
  a.D = static_cast<int>(L->desc.d);
  a.F = static_cast<int>(L->desc.f);
  a.E = static_cast<int>(L->desc.num_experts);
  a.K = static_cast<int>(L->desc.top_k);
  a.act = static_cast<int>(L->desc.activation);
  a.norm = L->desc.router_norm ? 1 : 0;
  a.eps = L->desc.norm_eps;
  a.router_rows = L->router_rows;
  a.has_gate = L->has_gate;
  a.has_shared = L->has_shared;
  a.per_expert_scale = L->desc.per_expert_scale;
  a.logit_bias = L->desc.logit_bias;
  a.ids_in = ids_in;
  a.w_in = w_in;
  a.experts = expert_set(L);
  a.y = y;
  a.y_stride = y_stride;
  a.y_f32 = y_dtype == TSG_DTYPE_F32 ? 1 : 0;
  a.residual = residual;
  a.logits = ctx->f_logits;
  a.inv_rms = ctx->rb.inv_rms;
  a.actfrag = ctx->f_actfrag;
  a.counters = ctx->f_counters;
  a.ids_out = ids_out;
  a.w_out = w_out;
  a.w16_out = w16_out;
  a.pairs_out = ctx->rb.sorted_pairs;
  a.err = ctx->rb.err;
  a.num_sms = ctx->num_sms;
  a.allow_pdl = ctx->allow_pdl ? 1 : 0;
  a.cooperative = ctx->cooperative ? 1 : 0;
  a.stamps = ctx->stamps;
  if (stream_ok(ctx, L, T)) {
    TSG_CUDA_TRY(ctx, launch_decode_stream(a, L->dmaps, ctx->f_stream, ctx->f_flags, ctx->stream),
                 "streaming decode");
  } else {
    TSG_CUDA_TRY(ctx, launch_decode_fused(a, ctx->stream), "fused decode");
  }
  prof_mark(ctx, 1);
  prof_mark(ctx, 2);
  prof_mark(ctx, 3);
  prof_mark(ctx, 4);
  return TSG_OK;
}

// The streaming decode kernel takes the batch when it is selected (the
// default) and the shape is one it supports.
bool stream_ok(tsg_ctx ctx, const tsg_moe_layer_s* L, uint32_t T) {
  return ctx->use_fused && ctx->fused_kind == 1 && L->dmaps_ok &&
         decode_stream_supported(static_cast<int>(T), static_cast<int>(L->desc.d),
                                 static_cast<int>(L->desc.f), static_cast<int>(L->desc.top_k),
                                 static_cast<int>(L->desc.num_experts), L->has_gate,
                                 L->has_shared, ctx->num_sms);
}

bool fused_ok(tsg_ctx ctx, const tsg_moe_layer_s* L, uint32_t T) {
  if (stream_ok(ctx, L, T)) return true;
  return ctx->use_fused &&
         decode_fused_supported(static_cast<int>(T), static_cast<int>(L->desc.top_k),
                                static_cast<int>(L->desc.num_experts), L->has_gate, ctx->num_sms) &&
         decode_fused_fits(static_cast<int>(T), static_cast<int>(L->desc.d),
                           static_cast<int>(L->desc.f), static_cast<int>(L->desc.top_k),
                           L->has_shared, ctx->num_sms);
}

// `routed`: the pairs come from this layer's router, so an expert holds at
// most T rows (distinct experts per token) and every row tile has <= T rows.
tsg_status run_prefill_experts(tsg_ctx ctx, tsg_moe_layer_s* L, const void* x, uint32_t x_stride,
                               uint32_t T, const float* residual, void* y, uint32_t y_stride,
                               tsg_dtype y_dtype, bool routed = false) {
  // assumes rb.ids / rb.weights / rb.inv_rms are filled for T tokens
  const RouterParams rp = router_params(L, x, x_stride, T);
  const uint32_t K = L->desc.top_k;
  const uint32_t P = T * K;
  TSG_CUDA_TRY(ctx, launch_permute(rp, ctx->rb, nullptr, ctx->stream), "permute");
  const float* gate_w = L->has_gate ? L->router_rows + static_cast<size_t>(L->desc.num_experts) * L->desc.d
                                    : nullptr;
  const uint32_t rows = P + (L->has_shared ? T : 0u);
  QmmParams qp{};
  qp.D = static_cast<int>(L->desc.d);
  qp.F = static_cast<int>(L->desc.f);
  qp.E = static_cast<int>(L->desc.num_experts);
  qp.act = static_cast<int>(L->desc.activation);
  qp.n_rows_total = static_cast<int>(rows);
  qp.experts = expert_set(L);
  qp.row_tiles = ctx->rb.row_tiles;
  qp.n_row_tiles = ctx->rb.n_row_tiles;
  qp.xp = ctx->xp;
  qp.act_buf = ctx->act_buf;
  qp.partials = ctx->partials;
  qp.err = ctx->rb.err;
  qp.num_sms = ctx->num_sms;
  // few tokens per expert: batched GEMVs (the cost is the weight bytes);
  // else the tcgen05 grouped contraction
  const bool gemv = routed && T <= ctx->gemv_max_tokens &&
                    T <= static_cast<uint32_t>(gemv_max_tile_rows()) && gemv_usable(qp);
  TSG_CUDA_TRY(ctx,
               launch_gather_rows_gate(static_cast<const uint16_t*>(x), x_stride, ctx->rb.inv_rms,
                                       ctx->rb.sorted_pairs, static_cast<int>(P),
                                       static_cast<int>(T), static_cast<int>(L->desc.d),
                                       L->has_shared, ctx->xp, gate_w, ctx->rb.gate_raw,
                                       ctx->stream, gemv ? 1 : 0),
               "gather rows");
  prof_mark(ctx, 1);
  if (gemv) {
    TSG_CUDA_TRY(ctx, launch_gemv_gate_up(qp, static_cast<int>(T), ctx->stream), "gemv gate/up");
  } else {
    TSG_CUDA_TRY(ctx, launch_qmm_gate_up(qp, ctx->stream), "qmm gate/up");
  }
  prof_mark(ctx, 2);
  if (gemv) {
    TSG_CUDA_TRY(ctx, launch_gemv_down(qp, static_cast<int>(T), ctx->stream), "gemv down");
  } else {
    TSG_CUDA_TRY(ctx, launch_qmm_down(qp, ctx->stream), "qmm down");
  }
  prof_mark(ctx, 3);
  CombineParams cp{};
  cp.T = static_cast<int>(T);
  cp.D = static_cast<int>(L->desc.d);
  cp.K = static_cast<int>(K);
  cp.has_shared = L->has_shared;
  cp.E = static_cast<int>(L->desc.num_experts);
  cp.partials = ctx->partials;
  cp.pair_pos = ctx->rb.pair_pos;
  cp.weights = ctx->rb.weights;
  cp.gate_raw = L->has_gate ? ctx->rb.gate_raw : nullptr;
  cp.inv_rms = ctx->rb.inv_rms;
  cp.residual = residual;
  cp.y = y;
  cp.y_stride = y_stride;
  cp.y_f32 = y_dtype == TSG_DTYPE_F32 ? 1 : 0;
  TSG_CUDA_TRY(ctx, launch_combine(cp, ctx->stream), "combine");
  prof_mark(ctx, 4);
  return TSG_OK;
}

__global__ void dense_route_kernel(uint32_t* ids, float* w, uint16_t* w16, int T) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x) {
    ids[i] = 0u;
    w[i] = 1.0f;
    w16[i] = 0x3C00u;  // fp16 1.0
  }
}

// A layer's dense branch (SharedExpertInt4.encode, SharedExpertInt4.swift:
// 30-94: gate and up GEMVs, act(g)·u, the down GEMV, on every token):
// y = residual + dense(x), through the one-expert view of the layer that
// every token takes with weight 1 -- the batched int4 GEMVs for up to
// gemv_max_tokens tokens (its wide F does not fit the decode kernels'
// shared-memory plan), else the tcgen05 contraction.  The input is the
// routed experts' (the no-scale RMSNorm when the layer normalises).
tsg_status run_dense_branch(tsg_ctx ctx, tsg_moe_layer_s* L, const void* x, uint32_t x_stride,
                            uint32_t T, const float* residual, void* y, uint32_t y_stride,
                            tsg_dtype y_dtype) {
  tsg_moe_layer_s* Dn = L->dense;
  const int blocks = static_cast<int>(std::min<uint32_t>((T + 255) / 256, 148u));
  dense_route_kernel<<<blocks, 256, 0, ctx->stream>>>(ctx->rb.ids, ctx->rb.weights,
                                                      ctx->rb.weights_f16, static_cast<int>(T));
  TSG_CUDA_TRY(ctx, cudaGetLastError(), "dense branch routing");
  const RouterParams p = router_params(Dn, x, x_stride, T);
  TSG_CUDA_TRY(ctx, launch_rowprep(p, ctx->rb, 0, ctx->stream), "row prep (dense branch)");
  return run_prefill_experts(ctx, Dn, x, x_stride, T, residual, y, y_stride, y_dtype, true);
}

tsg_status check_common(tsg_ctx ctx, tsg_moe_layer L, const void* x, uint32_t x_stride,
                        uint32_t T, const void* y, uint32_t y_stride, tsg_dtype y_dtype) {
  if (!ctx || !L) return fail(ctx, TSG_ERR_INVALID_ARG, "null context or layer");
  if (L->ctx != ctx) return fail(ctx, TSG_ERR_INVALID_ARG, "layer belongs to another context");
  if (T == 0) return TSG_OK;
  if (!x || !y) return fail(ctx, TSG_ERR_INVALID_ARG, "null input or output");
  if (x_stride < L->desc.d || x_stride % 8)
    return fail(ctx, TSG_ERR_INVALID_ARG, "hidden stride is too small or not a multiple of 8");
  if (y_stride < L->desc.d || y_stride % 8)
    return fail(ctx, TSG_ERR_INVALID_ARG, "output stride is too small or not a multiple of 8");
  if (!valid_dtype(y_dtype)) return fail(ctx, TSG_ERR_INVALID_ARG, "output dtype must be bf16 or f32");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u)
    return fail(ctx, TSG_ERR_INVALID_ARG, "input and output must be 16-byte aligned");
  return TSG_OK;
}

const char* grouping_error_text(uint32_t code) {
  switch (code) {
    case 6: return "route token %u is out of range";
    case 7: return "route rank %u is out of range";
    case 8: return "route expert %u is out of range";
    case 9: return "duplicate route pair for token %u";
    case 10: return "imported scale of group %u is not an fp16 value (import is exact or fails)";
    case 11: return "imported bias of group %u is not -8 x scale (not the symmetric int4 scheme)";
    default: return "routing metadata failed validation (value %u)";
  }
}

__global__ void fold_router_kernel(const float* w, const float* eff, const float* gate, int E,
                                   int D, float* out) {
  const size_t n = static_cast<size_t>(E) * D;
  for (size_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n + (gate ? D : 0);
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    if (i < n) {
      const float s = eff ? eff[i % D] : 1.0f;
      out[i] = w[i] * s;
    } else {
      out[i] = gate[i - n];
    }
  }
}

// ---- NCCL, loaded on first use --------------------------------------------
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;  // optional
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    auto sym = [&](const char* n) { return dlsym(h, n); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    api.send = reinterpret_cast<decltype(api.send)>(sym("ncclSend"));
    api.recv = reinterpret_cast<decltype(api.recv)>(sym("ncclRecv"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.send && api.recv &&
             api.group_start && api.group_end && api.error_string && api.all_gather;
  });
  return api;
}

tsg_status nccl_fail(tsg_ctx ctx, ncclResult_t r, const char* where) {
  const NcclApi& n = nccl();
  return fail(ctx, TSG_ERR_NCCL,
              std::string(where) + ": " + (n.error_string ? n.error_string(r) : "NCCL error"));
}

#define TSG_NCCL_TRY(ctx, expr, where)                              \
  do {                                                              \
    ncclResult_t r__ = (expr);                                      \
    if (r__ != ncclSuccess) return nccl_fail(ctx, r__, where);      \
  } while (0)

// kEpStage: this rank's token rows for its remote owners, one contiguous
// run per owner, before the copy engines send them
enum EpBuf { kEpXp = 0, kEpAct, kEpRet, kEpRows, kEpMap, kEpStage, kEpBufs };
constexpr int kEpTiles = kEpBufs, kEpKinds = kEpBufs + 1;  // capacities: buffers, then row tiles
constexpr size_t kEpElemBytes[kEpBufs] = {2, 2, 2, 2, 4, 2};
constexpr bool kEpShared[kEpBufs] = {false, false, true, true, true, false};  // written by peers

// Unmaps the peers' buffers (the peers keep their own) and forgets every
// rank's capacities, so the next call grows them all again.
void close_peer_views(tsg_ctx ctx) {
  for (int b = 0; b < kEpBufs; ++b) {
    std::vector<void*>& v = ctx->ep_peer[b];
    for (size_t q = 0; q < v.size(); ++q)
      if (static_cast<int>(q) != ctx->ep_rank && v[q] && kEpShared[b]) cudaIpcCloseMemHandle(v[q]);
    v.assign(v.size(), nullptr);
  }
  for (std::vector<size_t>& c : ctx->ep_caps) c.assign(c.size(), 0);
}

// Word layout of ep_ag (device) and ep_h_ag (pinned), both kAgTotal words.
constexpr uint32_t kAgWordsMax = 512 + 16 + 4;         // counts[E], tokens[R], T, status, pad
constexpr uint32_t kAgRecv = kAgWordsMax;              // [world][W]
constexpr uint32_t kAgBar = kAgRecv + 16 * kAgWordsMax;  // barrier: send [1], receive [16]
constexpr uint32_t kHxWords = 4 + 3 * 16;              // status, pad, three 64-byte IPC handles
constexpr uint32_t kAgHx = kAgBar + 32;                // handles: send [kHxWords], receive [16][..]
constexpr uint32_t kAgHost = kAgHx + 17 * kHxWords;    // pinned only: T, status, barrier words
constexpr uint32_t kAgTotal = kAgHost + 8;
static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
inline uint32_t ep_ag_words(uint32_t E, int R) { return (E + static_cast<uint32_t>(R) + 2 + 3) & ~3u; }

void release_ep(tsg_ctx ctx) {
  if (ctx->nccl_comm && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(ctx->nccl_comm));
  ctx->nccl_comm = nullptr;
  close_peer_views(ctx);
  for (int b = 0; b < kEpBufs; ++b) {
    if (ctx->ep_buf[b]) cudaFree(ctx->ep_buf[b]);
    ctx->ep_buf[b] = nullptr;
    ctx->ep_buf_elems[b] = 0;
  }
  for (void* p : {static_cast<void*>(ctx->ep_ag), static_cast<void*>(ctx->ep_tile_out),
                  static_cast<void*>(ctx->ep_ptiles), static_cast<void*>(ctx->ep_slots)})
    if (p) cudaFree(p);
  if (ctx->ep_h_ag) cudaFreeHost(ctx->ep_h_ag);
  if (ctx->ep_h_tile_out) cudaFreeHost(ctx->ep_h_tile_out);
  if (ctx->ep_h_ptiles) cudaFreeHost(ctx->ep_h_ptiles);
  ctx->ep_ptiles = ctx->ep_h_ptiles = nullptr;
  ctx->ep_pntiles = nullptr;
  ctx->ep_ptiles_cap = 0;
  ctx->ep_ag = ctx->ep_h_ag = nullptr;
  ctx->ep_tile_out = ctx->ep_h_tile_out = nullptr;
  ctx->ep_slots = nullptr;
  ctx->ep_slots_cap = 0;
  if (ctx->ep_ev_ok)
    for (cudaEvent_t& e : ctx->ep_ev) cudaEventDestroy(e);
  ctx->ep_ev_ok = false;
  if (ctx->ep_chunk_ok) {
    for (cudaEvent_t& e : ctx->ep_chunk_ev) cudaEventDestroy(e);
    cudaStreamDestroy(ctx->ep_copy);
  }
  ctx->ep_copy = nullptr;
  ctx->ep_chunk_ok = false;
  for (void* p : {static_cast<void*>(ctx->ep_rows), static_cast<void*>(ctx->ep_act),
                  static_cast<void*>(ctx->ep_out), static_cast<void*>(ctx->ep_ret),
                  static_cast<void*>(ctx->ep_counts_recv), static_cast<void*>(ctx->ep_tiles)})
    if (p) cudaFree(p);
  if (ctx->ep_h_counts) cudaFreeHost(ctx->ep_h_counts);
  if (ctx->ep_h_tiles) cudaFreeHost(ctx->ep_h_tiles);
  ctx->ep_rows = ctx->ep_act = ctx->ep_out = ctx->ep_ret = nullptr;
  ctx->ep_counts_recv = nullptr;
  ctx->ep_tiles = nullptr;
  ctx->ep_h_counts = nullptr;
  ctx->ep_h_tiles = nullptr;
  ctx->ep_rows_cap = ctx->ep_ret_cap = ctx->ep_tiles_cap = 0;
}

// Grows a device buffer of `n` elements of T (contents not kept).
template <typename T>
cudaError_t grow(T** p, size_t* cap, size_t need) {
  if (*p && *cap >= need) return cudaSuccess;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(need, 1) * sizeof(T));
  if (e == cudaSuccess) *cap = need;
  return e;
}

}  // namespace

// ---- scratch of tsg_moe_group_pairs_noalloc --------------------------------
// Some hosts cannot let a library allocate device memory once they are
// running: a serving runtime that carved all of HBM into its own pools at
// start-up sees a cudaMalloc fail or eat into memory it promised elsewhere,
// and cudaFree waits for the whole device, stalling every other stream the
// host keeps busy.  tsg_moe_group_pairs may grow the context workspace with
// both, so the no-alloc variant takes its scratch from this one array,
// sized for TSG_GROUP_NOALLOC_MAX_PAIRS pairs and 512 experts.  Every word
// the permutation kernels read from it is written earlier in the same call,
// so nothing in it has to start at zero.
static __device__ __align__(256) uint8_t g_group_scratch[TSG_GROUP_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr size_t kGsPairs = TSG_GROUP_NOALLOC_MAX_PAIRS;
constexpr uint32_t kGsExperts = 512;
// Row tiles for any tile height >= 16 (max_row_tiles with T <= P).
constexpr size_t kGsRowTiles = 2 * (kGsPairs / 16 + 1) + kGsExperts + 1;
constexpr size_t gs_align(size_t x) { return (x + 255) / 256 * 256; }
constexpr size_t kGsOffIds = 0;                                         // u32 [P]
constexpr size_t kGsOffW16 = kGsOffIds + gs_align(kGsPairs * 4);        // u16 [P]
constexpr size_t kGsOffPos = kGsOffW16 + gs_align(kGsPairs * 2);        // u32 [P]
constexpr size_t kGsOffTiles = kGsOffPos + gs_align(kGsPairs * 4);      // RowTile [..]
constexpr size_t kGsOffNTiles = kGsOffTiles + gs_align(kGsRowTiles * sizeof(RowTile));
constexpr size_t kGsOffHist = kGsOffNTiles + 256;                       // u32 [chunks][512]
constexpr size_t kGsEnd = kGsOffHist + gs_align((kGsPairs + 2047) / 2048 * 512 * 4);
static_assert(kGsEnd <= TSG_GROUP_NOALLOC_SCRATCH_BYTES, "group scratch layout overflows");

constexpr int kGsMaxDevices = 64;
std::mutex g_gs_mu;
uint8_t* g_gs_addr[kGsMaxDevices] = {};
unsigned long long g_gs_ctx_id[kGsMaxDevices] = {};

// The id of the device's current (primary) context, or 0 when the driver
// cannot say: a cudaDeviceReset makes a new context with a new id, and the
// module (and the array) is loaded again at another address.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&c) == CUDA_SUCCESS && c &&
      get_id(c, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

// The array's address on ctx's device.  It is resolved on the first call for
// that device, with the device current, and kept; it is resolved again when
// the device's context has changed since (after a cudaDeviceReset).
tsg_status group_scratch_on(tsg_ctx ctx, uint8_t** out) {
  if (ctx->device < 0 || ctx->device >= kGsMaxDevices)
    return fail(ctx, TSG_ERR_INVALID_ARG, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_gs_mu);
  TSG_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  const unsigned long long cid = current_context_id();
  if (!g_gs_addr[ctx->device] || cid != g_gs_ctx_id[ctx->device]) {
    void* p = nullptr;
    TSG_CUDA_TRY(ctx, cudaGetSymbolAddress(&p, g_group_scratch),
                 "cudaGetSymbolAddress(group scratch)");
    if (!p || reinterpret_cast<uintptr_t>(p) % 256 != 0)
      return fail(ctx, TSG_ERR_CUDA, "group scratch: unexpected symbol address");
    g_gs_addr[ctx->device] = static_cast<uint8_t*>(p);
    g_gs_ctx_id[ctx->device] = cid;
  }
  *out = g_gs_addr[ctx->device];
  return TSG_OK;
}

}  // namespace

extern "C" {

int tsg_abi_version(void) { return TSG_ABI_VERSION; }

tsg_status tsg_ctx_create(int device, void* stream, tsg_ctx* out) {
  if (!out) return TSG_ERR_INVALID_ARG;
  *out = nullptr;
  tsg_ctx ctx = new (std::nothrow) tsg_ctx_s();
  if (!ctx) return TSG_ERR_OOM;
  ctx->device = device;
  ctx->stream = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  int major = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess && major != 10) {
    delete ctx;
    return TSG_ERR_UNSUPPORTED_SHAPE;  // sm_100a only
  }
  if (e == cudaSuccess) e = cudaMalloc(&ctx->status, 8 * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(ctx->status, 0, 8 * sizeof(uint32_t));
  if (e != cudaSuccess) {
    delete ctx;
    return e == cudaErrorMemoryAllocation ? TSG_ERR_OOM : TSG_ERR_CUDA;
  }
  *out = ctx;
  return TSG_OK;
}

tsg_status tsg_ctx_destroy(tsg_ctx ctx) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->status) cudaFree(ctx->status);
  for (cudaEvent_t e : ctx->prof_events) cudaEventDestroy(e);
  release_ep(ctx);
  delete ctx;
  return TSG_OK;
}

tsg_status tsg_ctx_set_stream(tsg_ctx ctx, void* stream) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  ctx->stream = static_cast<cudaStream_t>(stream);
  return TSG_OK;
}

tsg_status tsg_ctx_set_decode_max_tokens(tsg_ctx ctx, uint32_t t) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  if (t > 64) return fail(ctx, TSG_ERR_INVALID_ARG, "decode regime handles at most 64 tokens");
  ctx->decode_max_tokens = t;
  return TSG_OK;
}

tsg_status tsg_ctx_set_option(tsg_ctx ctx, const char* name, int64_t value) {
  if (!ctx || !name) return fail(ctx, TSG_ERR_INVALID_ARG, "null argument");
  const std::string n(name);
  if (n == "fused_decode") {
    // 0: router / gate-up / down kernels; 1: the streaming single kernel
    // (default); 2: the earlier single kernel with a grid-wide act exchange
    ctx->use_fused = value != 0;
    ctx->fused_kind = value == 2 ? 2 : 1;
  }
  else if (n == "programmatic_launch") ctx->allow_pdl = value != 0;
  else if (n == "cooperative_launch") ctx->cooperative = value != 0;
  else if (n == "gemv_max_tokens") ctx->gemv_max_tokens = static_cast<uint32_t>(value < 0 ? 0 : value);
  else if (n == "ep_return") {
    // every rank of a group sets the same value (it changes no collective)
    if (value != 0 && value != 1) return fail(ctx, TSG_ERR_INVALID_ARG, "ep_return is 0 or 1");
    ctx->ep_return = static_cast<int>(value);
  }
  else if (n == "ep_dispatch") {
    // every rank of a group sets the same value (it enters the plan)
    if (value != 0 && value != 1) return fail(ctx, TSG_ERR_INVALID_ARG, "ep_dispatch is 0 or 1");
    ctx->ep_dispatch = static_cast<int>(value);
  }
  else if (n == "ep_transport") {
    // every rank of a group must pass the same value before its next call
    if (value != 0 && value != 1) return fail(ctx, TSG_ERR_INVALID_ARG, "ep_transport is 0 or 1");
    ctx->ep_transport = static_cast<int>(value);
  }
  else if (n == "debug_phase_stamps")
    ctx->stamps = reinterpret_cast<unsigned long long*>(static_cast<uintptr_t>(value));
  else return fail(ctx, TSG_ERR_INVALID_ARG, "unknown option " + n);
  return TSG_OK;
}

tsg_status tsg_ctx_reserve(tsg_ctx ctx, tsg_moe_layer layer, uint32_t max_tokens) {
  if (!ctx || !layer) return fail(ctx, TSG_ERR_INVALID_ARG, "null context or layer");
  return ensure_workspace(ctx, layer_caps(layer, max_tokens));
}

tsg_status tsg_sync(tsg_ctx ctx) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  cudaError_t e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "stream");
  uint32_t st[3] = {0, 0, 0};
  e = cudaMemcpy(st, ctx->status, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "status readback");
  if (st[0] == 0u) return TSG_OK;
  cudaMemset(ctx->status, 0, 4 * sizeof(uint32_t));
  if (ctx->ws) reset_fused_signals(ctx);
  if (st[0] & TSG_DEVERR_TIMEOUT) {
    return fail(ctx, TSG_ERR_TIMEOUT, "a device-side wait ran out of time (pipeline fault)");
  }
  char buf[160];
  std::snprintf(buf, sizeof(buf), grouping_error_text(st[1]), st[2]);
  return fail(ctx, TSG_ERR_METADATA, buf);
}

const char* tsg_last_error_string(tsg_ctx ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

tsg_status tsg_moe_layer_create(tsg_ctx ctx, const tsg_moe_layer_desc* d, tsg_moe_layer* out) {
  if (!ctx || !d || !out) return fail(ctx, TSG_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (d->group_size != 32) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "group size must be 32");
  if (d->d == 0 || d->d % 256) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "D must be a multiple of 256");
  if (d->f == 0 || d->f % 64) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "F must be a multiple of 64");
  if (d->num_experts == 0 || d->num_experts > 512)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "numExperts must be in 1...512");
  if (d->top_k == 0 || d->top_k > 32 || d->top_k > d->num_experts)
    return fail(ctx, TSG_ERR_INVALID_ARG, "topK must be in 1...min(32, numExperts)");
  if (d->activation != TSG_ACT_GELU_PYTORCH_TANH && d->activation != TSG_ACT_SILU)
    return fail(ctx, TSG_ERR_INVALID_ARG, "unknown gate activation");
  if (!d->experts || !d->router_weight) return fail(ctx, TSG_ERR_INVALID_ARG, "null experts or router");
  const tsg_expert_offsets& o = d->offsets;
  const uint64_t align_bits = reinterpret_cast<uintptr_t>(d->experts) | d->expert_stride |
                              o.gate_w_off | o.gate_s_off | o.up_w_off | o.up_s_off |
                              o.down_w_off | o.down_s_off;
  if (align_bits & 15u)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "expert blobs and sub-tensors must be 16-byte aligned");
  const bool dense = d->shared_expert && d->shared_f != d->f;
  if (d->shared_expert) {
    if (d->shared_f == 0 || d->shared_f % 64)
      return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "shared F must be a multiple of 64");
    if (dense && d->shared_gate)
      return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE,
                  "a gated shared expert must have the experts' F (a dense branch has no gate)");
    const tsg_expert_offsets& so = d->shared_offsets;
    const uint64_t sb = reinterpret_cast<uintptr_t>(d->shared_expert) | so.gate_w_off |
                        so.gate_s_off | so.up_w_off | so.up_s_off | so.down_w_off | so.down_s_off;
    if (sb & 15u) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "shared expert must be 16-byte aligned");
  }
  tsg_moe_layer L = new (std::nothrow) tsg_moe_layer_s();
  if (!L) return fail(ctx, TSG_ERR_OOM, "layer");
  L->ctx = ctx;
  L->desc = *d;
  if (dense) {
    // the dense MLP as a one-expert layer that every token takes with weight
    // 1 (no router of its own); the routed view of the layer has no shared slot
    tsg_moe_layer_s* Dn = new (std::nothrow) tsg_moe_layer_s();
    if (!Dn) {
      delete L;
      return fail(ctx, TSG_ERR_OOM, "layer");
    }
    Dn->ctx = ctx;
    Dn->desc = *d;
    Dn->desc.f = d->shared_f;
    Dn->desc.num_experts = 1;
    Dn->desc.top_k = 1;
    Dn->desc.experts = d->shared_expert;
    Dn->desc.expert_stride = 0;
    Dn->desc.offsets = d->shared_offsets;
    Dn->desc.shared_expert = nullptr;
    Dn->desc.shared_gate = nullptr;
    Dn->desc.per_expert_scale = nullptr;
    Dn->desc.logit_bias = nullptr;
    L->dense = Dn;
    L->desc.shared_expert = nullptr;
    L->desc.shared_f = 0;
  }
  L->has_shared = L->desc.shared_expert ? 1 : 0;
  L->has_gate = (L->desc.shared_expert && d->shared_gate) ? 1 : 0;
  const size_t rows = d->num_experts + (L->has_gate ? 1 : 0);
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e == cudaSuccess) e = cudaMalloc(&L->router_rows, rows * d->d * sizeof(float));
  if (e == cudaSuccess) {
    fold_router_kernel<<<256, 256, 0, ctx->stream>>>(d->router_weight, d->effective_scale,
                                                     L->has_gate ? d->shared_gate : nullptr,
                                                     static_cast<int>(d->num_experts),
                                                     static_cast<int>(d->d), L->router_rows);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && d->d % 64 == 0) {
    // exact bf16 planes for the tensor-core prefill router
    const size_t bytes = 3ull * router_tc_pad(static_cast<int>(d->num_experts)) * d->d * 2;
    e = cudaMalloc(&L->router_w3, bytes);
    if (e == cudaSuccess)
      e = launch_split_router(L->router_rows, static_cast<int>(d->num_experts),
                              static_cast<int>(d->d), L->router_w3, ctx->stream);
  }
  if (e == cudaSuccess)
    L->dmaps_ok = encode_decode_maps(expert_set(L), static_cast<int>(d->d),
                                     static_cast<int>(d->f), static_cast<int>(d->num_experts),
                                     &L->dmaps);
  if (e != cudaSuccess) {
    if (L->router_rows) cudaFree(L->router_rows);
    if (L->router_w3) cudaFree(L->router_w3);
    delete L->dense;
    delete L;
    return cuda_fail(ctx, e, "layer create");
  }
  *out = L;
  return TSG_OK;
}

tsg_status tsg_moe_layer_destroy(tsg_moe_layer L) {
  if (!L) return TSG_ERR_INVALID_ARG;
  // the layer does not touch its context here: contexts and layers may be
  // destroyed in either order (cudaFree waits for outstanding work itself)
  if (L->router_rows) cudaFree(L->router_rows);
  if (L->router_w3) cudaFree(L->router_w3);
  delete L->dense;
  delete L;
  return TSG_OK;
}

tsg_status tsg_router_topk(tsg_ctx ctx, tsg_moe_layer L, const void* hidden, uint32_t hidden_stride,
                           uint32_t T, uint32_t* out_indices, float* out_weights,
                           uint16_t* out_weights_f16) {
  if (!ctx || !L) return fail(ctx, TSG_ERR_INVALID_ARG, "null context or layer");
  if (T == 0) return TSG_OK;
  if (!hidden || !out_indices || !out_weights) return fail(ctx, TSG_ERR_INVALID_ARG, "null buffer");
  if (hidden_stride < L->desc.d || hidden_stride % 8)
    return fail(ctx, TSG_ERR_INVALID_ARG, "hidden stride is too small");
  tsg_status st = ensure_workspace(ctx, layer_caps(L, T));
  if (st != TSG_OK) return st;
  RouterParams p = router_params(L, hidden, hidden_stride, T);
  RouteBuffers rb = ctx->rb;
  rb.ids = out_indices;
  rb.weights = out_weights;
  rb.weights_f16 = out_weights_f16;
  if (T <= ctx->decode_max_tokens) {
    TSG_CUDA_TRY(ctx, launch_router_decode(p, rb, ctx->stream), "router (decode)");
  } else {
    TSG_CUDA_TRY(ctx, launch_router_prefill(p, rb, ctx->stream), "router (prefill)");
  }
  return TSG_OK;
}

tsg_status tsg_router_logits(tsg_ctx ctx, tsg_moe_layer L, const void* hidden,
                             uint32_t hidden_stride, uint32_t T, float* out_logits) {
  if (!ctx || !L) return fail(ctx, TSG_ERR_INVALID_ARG, "null context or layer");
  if (L->ctx != ctx) return fail(ctx, TSG_ERR_INVALID_ARG, "layer belongs to another context");
  if (T == 0) return TSG_OK;
  if (!hidden || !out_logits) return fail(ctx, TSG_ERR_INVALID_ARG, "null buffer");
  if (hidden_stride < L->desc.d || hidden_stride % 8)
    return fail(ctx, TSG_ERR_INVALID_ARG, "hidden stride is too small");
  tsg_status st = take_pending_error(ctx);
  if (st != TSG_OK) return st;
  st = ensure_workspace(ctx, layer_caps(L, T));
  if (st != TSG_OK) return st;
  const RouterParams p = router_params(L, hidden, hidden_stride, T);
  TSG_CUDA_TRY(ctx, launch_router_prefill(p, ctx->rb, ctx->stream, out_logits), "router logits");
  return TSG_OK;
}

tsg_status tsg_make_token_expert_pairs(tsg_ctx ctx, const uint32_t* indices,
                                       const uint16_t* weights_f16, uint32_t T, uint32_t K,
                                       tsg_token_expert_pair* out) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  if (T * K == 0) return TSG_OK;
  if (!indices || !out) return fail(ctx, TSG_ERR_INVALID_ARG, "null buffer");
  TSG_CUDA_TRY(ctx,
               launch_make_pairs(indices, weights_f16, static_cast<int>(T), static_cast<int>(K),
                                 reinterpret_cast<Pair*>(out), ctx->stream),
               "make pairs");
  return TSG_OK;
}

tsg_status tsg_moe_group_pairs(tsg_ctx ctx, const tsg_token_expert_pair* pairs, uint32_t n_pairs,
                               int32_t query_count, int32_t top_k, int32_t num_experts,
                               int32_t tile_expert_count, const uint64_t* sort_keys,
                               int32_t n_sort_keys, int32_t tile_break,
                               tsg_token_expert_pair* sorted_pairs, uint32_t* offsets,
                               uint32_t* counts, tsg_moe_group* groups, uint32_t* n_groups,
                               tsg_moe_tile* tiles, uint32_t* n_tiles) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  char buf[128];
  // argument checks in the order of PrefillMoEGrouping.swift:100-120
  if (query_count < 0) {
    std::snprintf(buf, sizeof(buf), "queryCount must be non-negative, got %d", query_count);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (top_k <= 0) {
    std::snprintf(buf, sizeof(buf), "topK must be positive, got %d", top_k);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (num_experts <= 0) {
    std::snprintf(buf, sizeof(buf), "numExperts must be positive, got %d", num_experts);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (tile_expert_count < 1 || tile_expert_count > 16) {
    std::snprintf(buf, sizeof(buf), "tileExpertCount must be in 1...16, got %d", tile_expert_count);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (sort_keys && n_sort_keys != num_experts) {
    std::snprintf(buf, sizeof(buf), "expected %d expert sort keys, got %d", num_experts, n_sort_keys);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  const uint64_t expected = static_cast<uint64_t>(query_count) * static_cast<uint64_t>(top_k);
  if (n_pairs != expected) {
    std::snprintf(buf, sizeof(buf), "expected %llu route pairs, got %u",
                  static_cast<unsigned long long>(expected), n_pairs);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (num_experts > 512) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "numExperts > 512");
  if (n_pairs > 0 && (!pairs || !sorted_pairs)) return fail(ctx, TSG_ERR_INVALID_ARG, "null pairs");
  if (!offsets || !counts || !groups || !n_groups || !tiles || !n_tiles)
    return fail(ctx, TSG_ERR_INVALID_ARG, "null output");
  Caps c;
  c.T = static_cast<uint32_t>(query_count);
  c.K = static_cast<uint32_t>(top_k);
  c.E = static_cast<uint32_t>(num_experts);
  c.D = 256;
  c.F = 64;
  tsg_status st = ensure_workspace(ctx, c);
  if (st != TSG_OK) return st;
  RouterParams p{};
  p.T = query_count;
  p.K = top_k;
  p.E = num_experts;
  p.tile_rows = qmm_tile_rows();
  p.tile_expert_count = tile_expert_count;
  p.tile_break = tile_break;
  p.sort_keys = sort_keys;
  RouteBuffers rb = ctx->rb;
  rb.sorted_pairs = reinterpret_cast<Pair*>(sorted_pairs);
  rb.offsets = offsets;
  rb.counts = counts;
  rb.groups = reinterpret_cast<Group*>(groups);
  rb.n_groups = n_groups;
  rb.tiles = reinterpret_cast<Tile*>(tiles);
  rb.n_tiles = n_tiles;
  if (n_pairs == 0) {
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(offsets, 0xFF, num_experts * 4u, ctx->stream), "memset");
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(counts, 0, num_experts * 4u, ctx->stream), "memset");
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(n_groups, 0, 4, ctx->stream), "memset");
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(n_tiles, 0, 4, ctx->stream), "memset");
    return TSG_OK;
  }
  TSG_CUDA_TRY(ctx, launch_permute(p, rb, reinterpret_cast<const Pair*>(pairs), ctx->stream),
               "group pairs");
  return TSG_OK;
}

tsg_status tsg_moe_group_pairs_noalloc(tsg_ctx ctx, const tsg_token_expert_pair* pairs,
                                       uint32_t n_pairs, int32_t query_count, int32_t top_k,
                                       int32_t num_experts, int32_t tile_expert_count,
                                       const uint64_t* sort_keys, int32_t n_sort_keys,
                                       int32_t tile_break, tsg_token_expert_pair* sorted_pairs,
                                       uint32_t* offsets, uint32_t* counts, tsg_moe_group* groups,
                                       uint32_t* n_groups, tsg_moe_tile* tiles,
                                       uint32_t* n_tiles) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  char buf[160];
  // the argument checks and messages of tsg_moe_group_pairs
  if (query_count < 0) {
    std::snprintf(buf, sizeof(buf), "queryCount must be non-negative, got %d", query_count);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (top_k <= 0) {
    std::snprintf(buf, sizeof(buf), "topK must be positive, got %d", top_k);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (num_experts <= 0) {
    std::snprintf(buf, sizeof(buf), "numExperts must be positive, got %d", num_experts);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (tile_expert_count < 1 || tile_expert_count > 16) {
    std::snprintf(buf, sizeof(buf), "tileExpertCount must be in 1...16, got %d", tile_expert_count);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  if (sort_keys && n_sort_keys != num_experts) {
    std::snprintf(buf, sizeof(buf), "expected %d expert sort keys, got %d", num_experts, n_sort_keys);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  const uint64_t expected = static_cast<uint64_t>(query_count) * static_cast<uint64_t>(top_k);
  if (n_pairs != expected) {
    std::snprintf(buf, sizeof(buf), "expected %llu route pairs, got %u",
                  static_cast<unsigned long long>(expected), n_pairs);
    return fail(ctx, TSG_ERR_INVALID_ARG, buf);
  }
  // the static scratch's limits
  if (n_pairs > kGsPairs) {
    std::snprintf(buf, sizeof(buf),
                  "tsg_moe_group_pairs_noalloc: %u route pairs exceed its static scratch limit of "
                  "%u pairs; use tsg_moe_group_pairs",
                  n_pairs, static_cast<unsigned>(kGsPairs));
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, buf);
  }
  if (num_experts > static_cast<int32_t>(kGsExperts)) {
    std::snprintf(buf, sizeof(buf),
                  "tsg_moe_group_pairs_noalloc: %d experts exceed its static scratch limit of %u",
                  num_experts, kGsExperts);
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, buf);
  }
  const uint32_t tr = static_cast<uint32_t>(qmm_tile_rows());
  if (tr < 16 || max_row_tiles(static_cast<uint32_t>(query_count), static_cast<uint32_t>(top_k),
                               static_cast<uint32_t>(num_experts), tr) > kGsRowTiles)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE,
                "tsg_moe_group_pairs_noalloc: row-tile schedule exceeds its static scratch");
  if (n_pairs > 0 && (!pairs || !sorted_pairs)) return fail(ctx, TSG_ERR_INVALID_ARG, "null pairs");
  if (!offsets || !counts || !groups || !n_groups || !tiles || !n_tiles)
    return fail(ctx, TSG_ERR_INVALID_ARG, "null output");

  uint8_t* base = nullptr;
  tsg_status st = group_scratch_on(ctx, &base);
  if (st != TSG_OK) return st;
  TSG_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  if (n_pairs == 0) {
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(offsets, 0xFF, num_experts * 4u, ctx->stream), "memset");
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(counts, 0, num_experts * 4u, ctx->stream), "memset");
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(n_groups, 0, 4, ctx->stream), "memset");
    TSG_CUDA_TRY(ctx, cudaMemsetAsync(n_tiles, 0, 4, ctx->stream), "memset");
    return TSG_OK;
  }
  RouterParams p{};
  p.T = query_count;
  p.K = top_k;
  p.E = num_experts;
  p.tile_rows = static_cast<int>(tr);
  p.tile_expert_count = tile_expert_count;
  p.tile_break = tile_break;
  p.sort_keys = sort_keys;
  // Only the fields the permutation kernels touch; per-pair errors go to the
  // context's status words, read back by tsg_sync as for tsg_moe_group_pairs.
  RouteBuffers rb{};
  rb.ids = reinterpret_cast<uint32_t*>(base + kGsOffIds);
  rb.weights_f16 = reinterpret_cast<uint16_t*>(base + kGsOffW16);
  rb.pair_pos = reinterpret_cast<uint32_t*>(base + kGsOffPos);
  rb.row_tiles = reinterpret_cast<RowTile*>(base + kGsOffTiles);
  rb.n_row_tiles = reinterpret_cast<uint32_t*>(base + kGsOffNTiles);
  rb.sync_counter = nullptr;  // the permutation kernels keep no cross-CTA counter
  rb.hist = reinterpret_cast<uint32_t*>(base + kGsOffHist);
  rb.err = ctx->status;
  rb.sorted_pairs = reinterpret_cast<Pair*>(sorted_pairs);
  rb.offsets = offsets;
  rb.counts = counts;
  rb.groups = reinterpret_cast<Group*>(groups);
  rb.n_groups = n_groups;
  rb.tiles = reinterpret_cast<Tile*>(tiles);
  rb.n_tiles = n_tiles;
  TSG_CUDA_TRY(ctx, launch_permute(p, rb, reinterpret_cast<const Pair*>(pairs), ctx->stream),
               "group pairs (no-alloc)");
  return TSG_OK;
}

tsg_status tsg_plan_routed_gemm(const tsg_moe_group* groups, uint32_t n_groups,
                                uint32_t max_rows_per_batch, uint32_t tile_rows,
                                tsg_routed_gemm_block* blocks, uint32_t max_blocks,
                                uint32_t* n_blocks, uint32_t* batch_rows,
                                uint32_t* batch_first_block, uint32_t* batch_block_count,
                                uint32_t max_batches, uint32_t* n_batches) {
  if ((n_groups && !groups) || !n_blocks || !n_batches || tile_rows == 0) return TSG_ERR_INVALID_ARG;
  uint32_t budget = (max_rows_per_batch / tile_rows) * tile_rows;
  if (budget < tile_rows) budget = tile_rows;
  uint32_t nb = 0, nbatch = 0, rows = 0, first = 0;
  bool overflow = false;
  auto flush = [&]() {
    if (rows == 0) return;
    if (nbatch < max_batches) {
      batch_rows[nbatch] = rows;
      batch_first_block[nbatch] = first;
      batch_block_count[nbatch] = nb - first;
    } else {
      overflow = true;
    }
    ++nbatch;
    first = nb;
    rows = 0;
  };
  for (uint32_t slot = 0; slot < n_groups; ++slot) {
    uint32_t taken = 0;
    const uint32_t count = groups[slot].pair_count;
    while (taken < count) {
      if (rows == budget) flush();
      if (rows > 0 && rows + (count - taken) > budget) flush();  // never split a group that fits
      const uint32_t take = std::min(count - taken, budget - rows);
      uint32_t done = 0;
      while (done < take) {
        const uint32_t rc = std::min(tile_rows, take - done);
        if (nb < max_blocks) {
          blocks[nb].local_slot = slot;
          blocks[nb].pair_start = groups[slot].pair_start + taken + done;
          blocks[nb].row_count = rc;
          blocks[nb].local_row = rows + done;
        } else {
          overflow = true;
        }
        ++nb;
        done += rc;
      }
      rows += take;
      taken += take;
    }
  }
  flush();
  *n_blocks = nb;
  *n_batches = nbatch;
  return overflow ? TSG_ERR_INVALID_ARG : TSG_OK;
}

tsg_status tsg_moe_block_forward(tsg_ctx ctx, tsg_moe_layer L, const void* hidden,
                                 uint32_t hidden_stride, uint32_t T, const float* residual,
                                 void* y, uint32_t y_stride, tsg_dtype y_dtype) {
  tsg_status st = check_common(ctx, L, hidden, hidden_stride, T, y, y_stride, y_dtype);
  if (st != TSG_OK || T == 0) return st;
  st = take_pending_error(ctx);
  if (st != TSG_OK) return st;
  st = ensure_workspace(ctx, layer_caps(L, T));
  if (st != TSG_OK) return st;
  // the dense branch first (its result becomes the routed pass's residual),
  // so that the routing left behind for tsg_last_routing is the router's
  if (L->dense) {
    st = run_dense_branch(ctx, L, hidden, hidden_stride, T, residual, ctx->dense_y, L->desc.d,
                          TSG_DTYPE_F32);
    if (st != TSG_OK) return st;
    residual = ctx->dense_y;
  }
  RouterParams p = router_params(L, hidden, hidden_stride, T);
  ctx->last_T = T;
  ctx->last_K = L->desc.top_k;
  prof_mark(ctx, 0);
  tsg_status r;
  if (T <= ctx->decode_max_tokens && fused_ok(ctx, L, T)) {
    r = run_decode_fused(ctx, L, hidden, hidden_stride, T, nullptr, nullptr, residual, y, y_stride,
                         y_dtype, ctx->rb.ids, ctx->rb.weights, ctx->rb.weights_f16);
  } else if (T <= ctx->decode_max_tokens) {
    TSG_CUDA_TRY(ctx, launch_router_decode(p, ctx->rb, ctx->stream), "router (decode)");
    prof_mark(ctx, 1);
    r = run_decode_experts(ctx, L, hidden, hidden_stride, T, residual, y, y_stride, y_dtype);
  } else {
    TSG_CUDA_TRY(ctx, launch_router_prefill(p, ctx->rb, ctx->stream), "router (prefill)");
    r = run_prefill_experts(ctx, L, hidden, hidden_stride, T, residual, y, y_stride, y_dtype,
                            true);
  }
  if (ctx->profiling && ctx->prof_calls < ctx->prof_max) ++ctx->prof_calls;
  return r;
}

// A speculative-verify block, row by row as decode computes it: the rows go
// through the streaming decode kernel two at a time (one for an odd last
// row).  That kernel's down split, reduction orders and accumulator starts
// are the same for one and two tokens, and an MMA column does not see its
// neighbours, so each row's y has the bits tsg_moe_block_forward gives that
// row alone.
tsg_status tsg_moe_verify_rows_forward(tsg_ctx ctx, tsg_moe_layer L, const void* hidden,
                                       uint32_t hidden_stride, uint32_t T, const float* residual,
                                       void* y, uint32_t y_stride, tsg_dtype y_dtype) {
  tsg_status st = check_common(ctx, L, hidden, hidden_stride, T, y, y_stride, y_dtype);
  if (st != TSG_OK || T == 0) return st;
  st = take_pending_error(ctx);
  if (st != TSG_OK) return st;
  if (!stream_ok(ctx, L, 1) || (T > 1 && !stream_ok(ctx, L, 2)))
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE,
                "verify rows need the streaming decode kernel (option fused_decode = 1) for this shape");
  st = ensure_workspace(ctx, layer_caps(L, T < 2 ? 2 : T));
  if (st != TSG_OK) return st;
  ctx->last_T = T;
  ctx->last_K = L->desc.top_k;
  const size_t K = L->desc.top_k, D = L->desc.d;
  const size_t ysz = y_dtype == TSG_DTYPE_F32 ? 4 : 2;
  prof_mark(ctx, 0);
  if (L->dense) {
    // the dense branch row by row, as a one-token block runs it
    for (uint32_t i = 0; i < T; ++i) {
      st = run_dense_branch(ctx, L, static_cast<const uint8_t*>(hidden) + static_cast<size_t>(i) * hidden_stride * 2,
                            hidden_stride, 1, residual ? residual + i * D : nullptr,
                            ctx->dense_y + i * D, static_cast<uint32_t>(D), TSG_DTYPE_F32);
      if (st != TSG_OK) return st;
    }
    residual = ctx->dense_y;
  }
  for (uint32_t i = 0; i < T; i += 2) {
    const uint32_t n = T - i < 2 ? T - i : 2;
    st = run_decode_fused(ctx, L, static_cast<const uint8_t*>(hidden) + static_cast<size_t>(i) * hidden_stride * 2,
                          hidden_stride, n, nullptr, nullptr, residual ? residual + i * D : nullptr,
                          static_cast<uint8_t*>(y) + static_cast<size_t>(i) * y_stride * ysz, y_stride,
                          y_dtype, ctx->rb.ids + i * K, ctx->rb.weights + i * K,
                          ctx->rb.weights_f16 + i * K);
    if (st != TSG_OK) return st;
  }
  if (ctx->profiling && ctx->prof_calls < ctx->prof_max) ++ctx->prof_calls;
  return TSG_OK;
}

// Gemma's layer FFN between attention and the next layer: the fused setup
// (post-attention norm, residual, the three normalised inputs), the dense
// branch, the routed experts (routed on router_x, run on routed_x), and the
// fused tail (the three post-norms, the residual, the layer scalar).
tsg_status tsg_gemma_ffn_forward(tsg_ctx ctx, tsg_moe_layer L, const tsg_gemma_norms* norms,
                                 void* hidden, uint32_t hidden_stride, const void* attn,
                                 uint32_t attn_stride, uint32_t T) {
  tsg_status st = check_common(ctx, L, hidden, hidden_stride, T, hidden, hidden_stride,
                               TSG_DTYPE_BF16);
  if (st != TSG_OK || T == 0) return st;
  if (!norms || !norms->post_attn || !norms->pre_ffn || !norms->pre_ffn2 || !norms->post_dense ||
      !norms->post_routed || !norms->post_ffn || !attn)
    return fail(ctx, TSG_ERR_INVALID_ARG, "null norm weight or attention input");
  if (attn_stride < L->desc.d || attn_stride % 8 || (reinterpret_cast<uintptr_t>(attn) & 15u))
    return fail(ctx, TSG_ERR_INVALID_ARG, "attention stride is too small or not aligned");
  if (L->desc.router_norm)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE,
                "the fused Gemma path normalises its inputs itself: create the layer with router_norm = 0");
  if (L->has_shared)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE,
                "the fused Gemma path takes a dense branch (shared_f != f), not a shared expert slot");
  if (L->desc.d > 4096) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "D above 4096");
  Caps want = layer_caps(L, T);
  want.fusion = 1;
  st = ensure_workspace(ctx, want);
  if (st != TSG_OK) return st;
  st = take_pending_error(ctx);
  if (st != TSG_OK) return st;
  const uint32_t D = L->desc.d;
  const size_t TD = static_cast<size_t>(T) * D;
  uint16_t* router_x = ctx->fx_in;
  uint16_t* routed_x = ctx->fx_in + TD;
  uint16_t* dense_x = ctx->fx_in + 2 * TD;
  float* h2 = ctx->fx_out;
  float* h1 = ctx->fx_out + TD;
  GemmaNorms n{};
  n.post_attn = norms->post_attn;
  n.pre_ffn = norms->pre_ffn;
  n.pre_ffn2 = norms->pre_ffn2;
  n.post_dense = norms->post_dense;
  n.post_routed = norms->post_routed;
  n.post_ffn = norms->post_ffn;
  n.eps = norms->eps;
  n.layer_scalar = norms->layer_scalar;
  TSG_CUDA_TRY(ctx,
               launch_gemma_setup(static_cast<uint16_t*>(hidden), hidden_stride,
                                  static_cast<const uint16_t*>(attn), attn_stride,
                                  static_cast<int>(T), static_cast<int>(D), n, router_x, routed_x,
                                  dense_x, ctx->stream),
               "gemma setup");
  if (L->dense) {
    st = run_dense_branch(ctx, L, dense_x, D, T, nullptr, h1, D, TSG_DTYPE_F32);
    if (st != TSG_OK) return st;
  }
  // the routed experts: the router on router_x, the experts on routed_x
  const RouterParams p = router_params(L, router_x, D, T);
  ctx->last_T = T;
  ctx->last_K = L->desc.top_k;
  if (T <= ctx->decode_max_tokens) {
    TSG_CUDA_TRY(ctx, launch_router_decode(p, ctx->rb, ctx->stream), "router (decode)");
    if (fused_ok(ctx, L, T)) {
      st = run_decode_fused(ctx, L, routed_x, D, T, ctx->rb.ids, ctx->rb.weights, nullptr, h2, D,
                            TSG_DTYPE_F32, nullptr, nullptr, nullptr);
    } else {
      const RouterParams pr = router_params(L, routed_x, D, T);
      TSG_CUDA_TRY(ctx, launch_rowprep(pr, ctx->rb, 1, ctx->stream), "row prep");
      st = run_decode_experts(ctx, L, routed_x, D, T, nullptr, h2, D, TSG_DTYPE_F32);
    }
  } else {
    TSG_CUDA_TRY(ctx, launch_router_prefill(p, ctx->rb, ctx->stream), "router (prefill)");
    st = run_prefill_experts(ctx, L, routed_x, D, T, nullptr, h2, D, TSG_DTYPE_F32, true);
  }
  if (st != TSG_OK) return st;
  TSG_CUDA_TRY(ctx,
               launch_gemma_tail(h2, L->dense ? h1 : nullptr, static_cast<uint16_t*>(hidden),
                                 hidden_stride, static_cast<int>(T), static_cast<int>(D), n,
                                 ctx->stream),
               "gemma tail");
  return TSG_OK;
}

tsg_status tsg_import_int4_affine(tsg_ctx ctx, const void* codes_u32, const uint16_t* scales_bf16,
                                  const uint16_t* biases_bf16, uint32_t rows, uint32_t cols,
                                  uint32_t group_size, void* out_codes, uint16_t* out_scales_f16) {
  if (!ctx || !codes_u32 || !scales_bf16 || !out_codes || !out_scales_f16)
    return fail(ctx, TSG_ERR_INVALID_ARG, "null argument");
  if (rows == 0 || cols == 0 || cols % 32)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "columns must be a positive multiple of 32");
  if (group_size == 0 || group_size % 32 || cols % group_size)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE,
                "group size must be a multiple of 32 that divides the columns");
  if (static_cast<uint64_t>(rows) * cols / 2 % 16 ||
      ((reinterpret_cast<uintptr_t>(codes_u32) | reinterpret_cast<uintptr_t>(out_codes)) & 15u))
    return fail(ctx, TSG_ERR_INVALID_ARG, "codes must be 16-byte aligned whole vectors");
  tsg_status st = take_pending_error(ctx);
  if (st != TSG_OK) return st;
  TSG_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  TSG_CUDA_TRY(ctx,
               launch_import_int4(codes_u32, scales_bf16, biases_bf16, static_cast<int>(rows),
                                  static_cast<int>(cols), static_cast<int>(group_size), out_codes,
                                  reinterpret_cast<__half*>(out_scales_f16), ctx->status,
                                  ctx->stream),
               "import int4");
  return TSG_OK;
}

tsg_status tsg_ctx_profile_begin(tsg_ctx ctx, uint32_t max_calls) {
  if (!ctx || max_calls == 0) return fail(ctx, TSG_ERR_INVALID_ARG, "max_calls must be positive");
  cudaSetDevice(ctx->device);
  for (cudaEvent_t e : ctx->prof_events) cudaEventDestroy(e);
  ctx->prof_events.assign(static_cast<size_t>(max_calls) * 5, nullptr);
  for (auto& e : ctx->prof_events) TSG_CUDA_TRY(ctx, cudaEventCreate(&e), "cudaEventCreate");
  ctx->prof_max = max_calls;
  ctx->prof_calls = 0;
  ctx->profiling = true;
  return TSG_OK;
}

tsg_status tsg_ctx_profile_end(tsg_ctx ctx, float* stage_ms, uint32_t* n_calls) {
  if (!ctx || !stage_ms) return fail(ctx, TSG_ERR_INVALID_ARG, "null argument");
  ctx->profiling = false;
  TSG_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "stream");
  for (int k = 0; k < 4; ++k) stage_ms[k] = 0.0f;
  for (uint32_t c = 0; c < ctx->prof_calls; ++c) {
    for (int k = 0; k < 4; ++k) {
      float ms = 0.0f;
      TSG_CUDA_TRY(ctx, cudaEventElapsedTime(&ms, ctx->prof_events[c * 5 + k],
                                             ctx->prof_events[c * 5 + k + 1]),
                   "cudaEventElapsedTime");
      stage_ms[k] += ms;
    }
  }
  if (n_calls) *n_calls = ctx->prof_calls;
  return TSG_OK;
}

static tsg_status experts_with_routing(tsg_ctx ctx, tsg_moe_layer L, const void* x,
                                       uint32_t x_stride, uint32_t T, const uint32_t* indices,
                                       const float* weights, const float* residual, void* y,
                                       uint32_t y_stride, tsg_dtype y_dtype, bool decode) {
  tsg_status st = check_common(ctx, L, x, x_stride, T, y, y_stride, y_dtype);
  if (st != TSG_OK || T == 0) return st;
  if (!indices || !weights) return fail(ctx, TSG_ERR_INVALID_ARG, "null routing");
  if (decode && T > 64) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "decode regime takes at most 64 tokens");
  st = ensure_workspace(ctx, layer_caps(L, T));
  if (st != TSG_OK) return st;
  if (L->dense) {
    st = run_dense_branch(ctx, L, x, x_stride, T, residual, ctx->dense_y, L->desc.d, TSG_DTYPE_F32);
    if (st != TSG_OK) return st;
    residual = ctx->dense_y;
  }
  const size_t P = static_cast<size_t>(T) * L->desc.top_k;
  TSG_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->rb.ids, indices, P * 4, cudaMemcpyDeviceToDevice, ctx->stream),
               "copy ids");
  TSG_CUDA_TRY(ctx,
               cudaMemcpyAsync(ctx->rb.weights, weights, P * 4, cudaMemcpyDeviceToDevice, ctx->stream),
               "copy weights");
  RouterParams p = router_params(L, x, x_stride, T);
  ctx->last_T = T;
  ctx->last_K = L->desc.top_k;
  if (decode && fused_ok(ctx, L, T)) {
    return run_decode_fused(ctx, L, x, x_stride, T, ctx->rb.ids, ctx->rb.weights, residual, y,
                            y_stride, y_dtype, nullptr, nullptr, nullptr);
  }
  TSG_CUDA_TRY(ctx, launch_rowprep(p, ctx->rb, decode ? 1 : 0, ctx->stream), "row prep");
  if (decode) {
    TSG_CUDA_TRY(ctx, launch_group_small(p, ctx->rb, ctx->stream), "group");
    return run_decode_experts(ctx, L, x, x_stride, T, residual, y, y_stride, y_dtype);
  }
  return run_prefill_experts(ctx, L, x, x_stride, T, residual, y, y_stride, y_dtype);
}

tsg_status tsg_moe_experts_decode(tsg_ctx ctx, tsg_moe_layer L, const void* x, uint32_t x_stride,
                                  uint32_t T, const uint32_t* indices, const float* weights,
                                  const float* residual, void* y, uint32_t y_stride,
                                  tsg_dtype y_dtype) {
  return experts_with_routing(ctx, L, x, x_stride, T, indices, weights, residual, y, y_stride,
                              y_dtype, true);
}

tsg_status tsg_moe_experts_prefill(tsg_ctx ctx, tsg_moe_layer L, const void* x, uint32_t x_stride,
                                   uint32_t T, const uint32_t* indices, const float* weights,
                                   const float* residual, void* y, uint32_t y_stride,
                                   tsg_dtype y_dtype) {
  return experts_with_routing(ctx, L, x, x_stride, T, indices, weights, residual, y, y_stride,
                              y_dtype, false);
}

tsg_status tsg_moe_reduce_token_major(tsg_ctx ctx, const uint16_t* partials, const float* weights,
                                      uint32_t T, uint32_t K, uint32_t D, void* h2,
                                      tsg_dtype h2_dtype) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  if (T == 0) return TSG_OK;
  if (!partials || !weights || !h2) return fail(ctx, TSG_ERR_INVALID_ARG, "null buffer");
  if (h2_dtype != TSG_DTYPE_F32 && h2_dtype != TSG_DTYPE_F16)
    return fail(ctx, TSG_ERR_INVALID_ARG, "h2 dtype must be f16 or f32");
  TSG_CUDA_TRY(ctx,
               launch_reduce_token_major(reinterpret_cast<const __half*>(partials), weights,
                                         static_cast<int>(T), static_cast<int>(K),
                                         static_cast<int>(D), h2, h2_dtype == TSG_DTYPE_F32,
                                         ctx->stream),
               "reduce token major");
  return TSG_OK;
}

tsg_status tsg_shared_expert(tsg_ctx ctx, tsg_moe_layer L, const void* x, uint32_t x_stride,
                             uint32_t T, void* y, uint32_t y_stride, tsg_dtype y_dtype) {
  tsg_status st = check_common(ctx, L, x, x_stride, T, y, y_stride, y_dtype);
  if (st != TSG_OK || T == 0) return st;
  if (!L->has_shared && !L->dense) return fail(ctx, TSG_ERR_INVALID_ARG, "layer has no shared expert");
  st = ensure_workspace(ctx, layer_caps(L, T));
  if (st != TSG_OK) return st;
  if (L->dense) return run_dense_branch(ctx, L, x, x_stride, T, nullptr, y, y_stride, y_dtype);
  // a view of the layer with no routed slots: the schedule holds only the
  // shared expert's row tiles
  tsg_moe_layer_s V = *L;
  V.desc.top_k = 0;
  RouterParams p = router_params(&V, x, x_stride, T);
  TSG_CUDA_TRY(ctx, launch_rowprep(p, ctx->rb, 0, ctx->stream), "row prep");
  RouteBuffers rb = ctx->rb;
  TSG_CUDA_TRY(ctx, cudaMemsetAsync(rb.n_groups, 0, 4, ctx->stream), "memset");
  // shared-only schedule: T rows appended after zero routed rows
  const uint32_t tr = static_cast<uint32_t>(qmm_tile_rows());
  const uint32_t ntile = (T + tr - 1) / tr;
  RowTile host_tiles[64];
  if (ntile > 64)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE,
                "shared expert call limited to " + std::to_string(64u * tr) + " tokens");
  for (uint32_t j = 0; j < ntile; ++j) {
    host_tiles[j].expert = L->desc.num_experts;
    host_tiles[j].row_start = j * tr;
    host_tiles[j].rows = std::min(tr, T - j * tr);
    host_tiles[j].pad = 0;
  }
  TSG_CUDA_TRY(ctx, cudaMemcpyAsync(rb.row_tiles, host_tiles, ntile * sizeof(RowTile),
                                    cudaMemcpyHostToDevice, ctx->stream), "tiles");
  TSG_CUDA_TRY(ctx, cudaMemcpyAsync(rb.n_row_tiles, &ntile, 4, cudaMemcpyHostToDevice, ctx->stream),
               "tiles");
  TSG_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "tiles");  // host arrays are stack-local
  const float* gate_w = L->has_gate ? L->router_rows + static_cast<size_t>(L->desc.num_experts) * L->desc.d
                                    : nullptr;
  TSG_CUDA_TRY(ctx,
               launch_gather_rows_gate(static_cast<const uint16_t*>(x), x_stride, rb.inv_rms,
                                       rb.sorted_pairs, 0, static_cast<int>(T),
                                       static_cast<int>(L->desc.d), 1, ctx->xp, gate_w,
                                       rb.gate_raw, ctx->stream),
               "gather");
  QmmParams qp{};
  qp.D = static_cast<int>(L->desc.d);
  qp.F = static_cast<int>(L->desc.f);
  qp.E = static_cast<int>(L->desc.num_experts);
  qp.act = static_cast<int>(L->desc.activation);
  qp.n_rows_total = static_cast<int>(T);
  qp.experts = expert_set(L);
  qp.row_tiles = rb.row_tiles;
  qp.n_row_tiles = rb.n_row_tiles;
  qp.xp = ctx->xp;
  qp.act_buf = ctx->act_buf;
  qp.partials = ctx->partials;
  qp.err = rb.err;
  qp.num_sms = ctx->num_sms;
  TSG_CUDA_TRY(ctx, launch_qmm_gate_up(qp, ctx->stream), "qmm gate/up");
  TSG_CUDA_TRY(ctx, launch_qmm_down(qp, ctx->stream), "qmm down");
  CombineParams cp{};
  cp.T = static_cast<int>(T);
  cp.D = static_cast<int>(L->desc.d);
  cp.K = 0;
  cp.has_shared = 1;
  cp.partials = ctx->partials;
  cp.pair_pos = rb.pair_pos;
  cp.weights = rb.weights;
  cp.gate_raw = L->has_gate ? rb.gate_raw : nullptr;
  cp.inv_rms = rb.inv_rms;
  cp.y = y;
  cp.y_stride = y_stride;
  cp.y_f32 = y_dtype == TSG_DTYPE_F32 ? 1 : 0;
  TSG_CUDA_TRY(ctx, launch_combine(cp, ctx->stream), "combine");
  return TSG_OK;
}

tsg_status tsg_last_routing(tsg_ctx ctx, const uint32_t** ids, const float** weights,
                            const tsg_token_expert_pair** sorted_pairs, uint32_t* T, uint32_t* K) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  if (ids) *ids = ctx->rb.ids;
  if (weights) *weights = ctx->rb.weights;
  if (sorted_pairs) *sorted_pairs = reinterpret_cast<const tsg_token_expert_pair*>(ctx->rb.sorted_pairs);
  if (T) *T = ctx->last_T;
  if (K) *K = ctx->last_K;
  return TSG_OK;
}

// ---- expert parallelism ------------------------------------------------------

tsg_status tsg_ep_unique_id(void* out_id) {
  if (!out_id) return TSG_ERR_INVALID_ARG;
  static_assert(sizeof(ncclUniqueId) == TSG_EP_UNIQUE_ID_BYTES, "NCCL unique id size");
  const NcclApi& n = nccl();
  if (!n.ok) return TSG_ERR_NCCL;
  ncclUniqueId id;
  if (n.get_unique_id(&id) != ncclSuccess) return TSG_ERR_NCCL;
  std::memcpy(out_id, &id, sizeof(id));
  return TSG_OK;
}

tsg_status tsg_ep_init(tsg_ctx ctx, const void* unique_id, int rank, int world) {
  if (!ctx) return TSG_ERR_INVALID_ARG;
  if (!unique_id || world < 1 || rank < 0 || rank >= world)
    return fail(ctx, TSG_ERR_INVALID_ARG, "expert-parallel group: bad unique id, rank or world");
  if (ctx->nccl_comm) return fail(ctx, TSG_ERR_INVALID_ARG, "context already joined a group");
  const NcclApi& n = nccl();
  if (!n.ok) return fail(ctx, TSG_ERR_NCCL, "libnccl.so.2 could not be loaded");
  TSG_CUDA_TRY(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  // the count and status exchange buffers, allocated here so that a call
  // never allocates between its collectives
  if (!ctx->ep_counts_recv) {
    TSG_CUDA_TRY(ctx, cudaMalloc(&ctx->ep_counts_recv, (1024 + 4 * 1024) * sizeof(uint32_t)),
                 "cudaMalloc");
    TSG_CUDA_TRY(ctx, cudaHostAlloc(&ctx->ep_h_counts, (2 * 512 + 1024) * sizeof(uint32_t),
                                    cudaHostAllocDefault), "cudaHostAlloc");
  }
  if (world > 1024) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "at most 1024 ranks");
  if (!ctx->ep_ag) {
    TSG_CUDA_TRY(ctx, cudaMalloc(&ctx->ep_ag, kAgTotal * sizeof(uint32_t)), "cudaMalloc");
    TSG_CUDA_TRY(ctx, cudaMemset(ctx->ep_ag, 0, kAgTotal * sizeof(uint32_t)), "cudaMemset");
    TSG_CUDA_TRY(ctx, cudaHostAlloc(&ctx->ep_h_ag, kAgTotal * sizeof(uint32_t), cudaHostAllocDefault),
                 "cudaHostAlloc");
  }
  if (!ctx->ep_ev_ok) {
    bool ok = true;
    for (cudaEvent_t& e : ctx->ep_ev) ok = ok && cudaEventCreate(&e) == cudaSuccess;
    TSG_CUDA_TRY(ctx, ok ? cudaSuccess : cudaErrorMemoryAllocation, "cudaEventCreate");
    ctx->ep_ev_ok = true;
  }
  if (!ctx->ep_chunk_ok) {
    bool ok = cudaStreamCreateWithFlags(&ctx->ep_copy, cudaStreamNonBlocking) == cudaSuccess;
    for (cudaEvent_t& e : ctx->ep_chunk_ev)
      ok = ok && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
    TSG_CUDA_TRY(ctx, ok ? cudaSuccess : cudaErrorMemoryAllocation, "copy stream");
    ctx->ep_chunk_ok = true;
  }
  ncclComm_t comm = nullptr;
  TSG_NCCL_TRY(ctx, n.comm_init_rank(&comm, world, id, rank), "ncclCommInitRank");
  ctx->nccl_comm = comm;
  ctx->ep_rank = rank;
  ctx->ep_world = world;
  for (std::vector<void*>& v : ctx->ep_peer) v.assign(world, nullptr);
  for (std::vector<size_t>& c : ctx->ep_caps) c.assign(world, 0);
  return TSG_OK;
}

}  // extern "C"

namespace {

// The peer-memory transport of tsg_ep_moe_block_forward, after its local
// phase (routing and sorting; the per-expert counts are in ep_ag's send
// words).  One all-gather carries every rank's counts, token count and
// status; from them every rank computes the same plan for all ranks -- the
// pair runs, where each run lands in its owner's receive buffer, and every
// buffer's needed capacity -- so a growth of any buffer is decided alike
// everywhere.  Then: this rank's kernel writes its pair rows straight into
// the owners' receive buffers (peer stores over NVLink), one barrier, the
// owner's grouped contraction writes each output row straight into the
// token's rank's return buffer from the GEMM2 epilogue, one barrier, and the
// combine reads them in this rank's sorted order.  No host round trip after
// the counts; no allocation unless a capacity grows.
tsg_status ep_peer_forward(tsg_ctx ctx, tsg_moe_layer L, const void* hidden,
                           uint32_t hidden_stride, uint32_t T, const float* residual, void* y,
                           uint32_t y_stride, tsg_dtype y_dtype, tsg_status local,
                           std::string local_msg) {
  const int R = ctx->ep_world, me = ctx->ep_rank;
  const uint32_t E = L->desc.num_experts, K = L->desc.top_k, D = L->desc.d, F = L->desc.f;
  const uint32_t El = E / static_cast<uint32_t>(R);
  const uint32_t P = T * K;
  const bool sh = L->has_shared != 0;
  const NcclApi& n = nccl();
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  cudaStream_t s = ctx->stream;
  RouteBuffers& rb = ctx->rb;
  const uint32_t W = ep_ag_words(E, R);  // words per rank: counts[E], tokens[R], T, status
  uint32_t* ag_send = ctx->ep_ag;
  uint32_t* ag_recv = ctx->ep_ag + kAgRecv;
  uint32_t* bar_send = ctx->ep_ag + kAgBar;
  uint32_t* bar_recv = bar_send + 1;
  uint32_t* hx_send = ctx->ep_ag + kAgHx;
  uint32_t* hx_recv = hx_send + kHxWords;
  uint32_t* h = ctx->ep_h_ag;
  auto ev = [&](int i) {
    if (ctx->ep_ev_ok) cudaEventRecord(ctx->ep_ev[i], s);
  };
  auto note = [&](tsg_status st) {
    if (local == TSG_OK && st != TSG_OK) {
      local = st;
      local_msg = ctx->last_error;
    }
  };
  auto nccl_abort = [&](ncclResult_t r, const char* where) {
    if (n.comm_abort) n.comm_abort(comm);
    else n.comm_destroy(comm);
    ctx->nccl_comm = nullptr;
    close_peer_views(ctx);
    return nccl_fail(ctx, r, where);
  };
#define EPP_NCCL(expr, where)                               \
  do {                                                      \
    const ncclResult_t r__ = (expr);                        \
    if (r__ != ncclSuccess) return nccl_abort(r__, where);  \
  } while (0)
  // a barrier whose word carries this rank's status; with `read`, the host
  // waits for it and learns whether every rank was fine (each barrier
  // stages its word in its own pinned slot, kAgHost + 2 .., since the host
  // does not wait between them)
  auto barrier = [&](int slot, bool ok_local, bool read, bool* all_ok,
                     int* first_bad) -> tsg_status {
    h[kAgHost + slot] = ok_local ? 1u : 0u;
    if (cudaMemcpyAsync(bar_send, &h[kAgHost + slot], 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
      note(fail(ctx, TSG_ERR_CUDA, "expert-parallel: barrier word"));
    EPP_NCCL(n.all_gather(bar_send, bar_recv, 1, ncclUint32, comm, s), "ncclAllGather(barrier)");
    if (!read) return TSG_OK;
    uint32_t* hb = h + kAgBar;
    if (cudaMemcpyAsync(hb, bar_recv, R * 4u, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return nccl_abort(ncclSystemError, "expert-parallel barrier readback");
    *all_ok = true;
    for (int q = 0; q < R; ++q)
      if (hb[q] != 1u) {
        *all_ok = false;
        if (*first_bad < 0) *first_bad = q;
      }
    return TSG_OK;
  };

  // ---- agreement 1: every rank's counts, token count and status ----
  h[kAgHost] = T;
  h[kAgHost + 1] = local == TSG_OK ? 1u : 0u;
  if (cudaMemcpyAsync(ag_send + E + R, &h[kAgHost], 8, cudaMemcpyHostToDevice, s) != cudaSuccess)
    note(fail(ctx, TSG_ERR_CUDA, "expert-parallel: count words"));
  ev(1);
  EPP_NCCL(n.all_gather(ag_send, ag_recv, W, ncclUint32, comm, s), "ncclAllGather(counts)");
  if (cudaMemcpyAsync(h, ag_recv, static_cast<size_t>(R) * W * 4u, cudaMemcpyDeviceToHost, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return nccl_abort(ncclSystemError, "expert-parallel count readback");
  int first_bad = -1;
  for (int q = 0; q < R && first_bad < 0; ++q)
    if (h[q * W + E + R + 1] != 1u) first_bad = q;
  if (local != TSG_OK) return fail(ctx, local, local_msg);
  if (first_bad >= 0)
    return fail(ctx, TSG_ERR_NCCL, "expert-parallel: rank " + std::to_string(first_bad) +
                                       " failed before the row exchange (its own call reports why)");

  // ---- the plan, the same on every rank ----
  // snd[q][o]: pairs q sends to o, at soff[q][o] of q's sorted order, landing
  // at rpo[o][q] of o's received pairs; tok[q][o]: token rows q sends to o,
  // at rro[o][q] of o's received rows
  std::vector<uint32_t> M(h, h + static_cast<size_t>(R) * W);
  const uint32_t tr = static_cast<uint32_t>(qmm_tile_rows());
  std::vector<uint32_t> Tq(R), snd(R * R), soff(R * R), rpo(R * R), tok(R * R), rro(R * R);
  std::vector<uint32_t> recv_pairs(R), recv_rows(R);
  std::vector<size_t> need[kEpKinds];
  for (std::vector<size_t>& v : need) v.assign(R, 0);
  bool sums_ok = true;
  for (int q = 0; q < R; ++q) {
    Tq[q] = M[q * W + E + R];
    uint32_t off = 0;
    for (int o = 0; o < R; ++o) {
      uint64_t c = 0;
      for (uint32_t j = 0; j < El; ++j) c += M[q * W + o * El + j];
      snd[q * R + o] = static_cast<uint32_t>(c);
      soff[q * R + o] = off;
      off += static_cast<uint32_t>(c);
      tok[q * R + o] = M[q * W + E + o];
      if (tok[q * R + o] > Tq[q] || tok[q * R + o] > c) sums_ok = false;
    }
    if (static_cast<uint64_t>(off) != static_cast<uint64_t>(Tq[q]) * K) sums_ok = false;
  }
  if (!sums_ok)  // (every rank sees the same counts and returns here)
    return fail(ctx, TSG_ERR_CUDA, "expert-parallel: pair counts do not add up");
  for (int o = 0; o < R; ++o) {
    uint64_t acc = 0, rows = 0, tiles = 0;
    for (int q = 0; q < R; ++q) {
      rpo[o * R + q] = static_cast<uint32_t>(acc);
      rro[o * R + q] = static_cast<uint32_t>(rows);
      acc += snd[q * R + o];
      rows += tok[q * R + o];
      for (uint32_t j = 0; j < El; ++j) tiles += (M[q * W + o * El + j] + tr - 1) / tr;
    }
    if (acc > UINT32_MAX / 2) sums_ok = false;
    recv_pairs[o] = static_cast<uint32_t>(acc);
    recv_rows[o] = static_cast<uint32_t>(rows);
    const size_t xrows = acc + (sh ? Tq[o] : 0u);
    need[kEpXp][o] = xrows * D;
    need[kEpAct][o] = xrows * F;
    need[kEpRet][o] = (static_cast<size_t>(Tq[o]) * K + (sh ? Tq[o] : 0u)) * D;
    need[kEpRows][o] = rows * D;
    need[kEpMap][o] = acc;
    need[kEpTiles][o] = tiles + (sh ? (Tq[o] + tr - 1) / tr : 0u);
    uint64_t staged = 0;  // rows rank o stages for its remote owners
    for (int q = 0; q < R; ++q)
      if (q != o) staged += tok[o * R + q];
    need[kEpStage][o] = ctx->ep_dispatch == 1 ? staged * D : 0u;
  }
  if (!sums_ok) return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "expert-parallel: too many pairs");

  // ---- growth (decided alike on every rank): unmap, barrier, replace what
  // is short, publish the handles of the buffers peers write, map the
  // peers', agree ----
  bool grow_all = false;
  for (int b = 0; b < kEpKinds; ++b)
    for (int r = 0; r < R; ++r)
      if (need[b][r] > ctx->ep_caps[b][r]) grow_all = true;
  if (grow_all) {
    std::vector<size_t> cap[kEpKinds];
    for (int b = 0; b < kEpKinds; ++b) {
      cap[b].resize(R);
      for (int r = 0; r < R; ++r) {
        const size_t nd = need[b][r], c = ctx->ep_caps[b][r];
        cap[b][r] = nd > c ? std::max<size_t>(nd + nd / 4, b == kEpTiles ? 256u : 1u << 16) : c;
      }
    }
    close_peer_views(ctx);
    bool all_ok = false;
    first_bad = -1;
    {
      const tsg_status st = barrier(4, true, true, &all_ok, &first_bad);
      if (st != TSG_OK) return st;
    }
    // no rank maps another's buffers now
    bool ok = true;
    for (int b = 0; b < kEpBufs && ok; ++b) {
      if (cap[b][me] <= ctx->ep_buf_elems[b] && (ctx->ep_buf[b] || cap[b][me] == 0)) continue;
      if (ctx->ep_buf[b]) cudaFree(ctx->ep_buf[b]);
      ctx->ep_buf[b] = nullptr;
      ctx->ep_buf_elems[b] = 0;
      ok = cudaMalloc(&ctx->ep_buf[b], cap[b][me] * kEpElemBytes[b]) == cudaSuccess;
      if (ok) ctx->ep_buf_elems[b] = cap[b][me];
    }
    if (ok && (!ctx->ep_ptiles || ctx->ep_ptiles_cap < cap[kEpTiles][me] + 1)) {
      for (void* p : {static_cast<void*>(ctx->ep_ptiles), static_cast<void*>(ctx->ep_tile_out)})
        if (p) cudaFree(p);
      for (void* p : {static_cast<void*>(ctx->ep_h_ptiles), static_cast<void*>(ctx->ep_h_tile_out)})
        if (p) cudaFreeHost(p);
      ctx->ep_ptiles = ctx->ep_h_ptiles = nullptr;
      ctx->ep_tile_out = ctx->ep_h_tile_out = nullptr;
      ctx->ep_ptiles_cap = 0;
      const size_t c = cap[kEpTiles][me] + 1;  // tiles, then the count and a count per chunk
      ok = cudaMalloc(&ctx->ep_ptiles, (c + 1 + kEpMaxRanks) * sizeof(RowTile)) == cudaSuccess &&
           cudaHostAlloc(&ctx->ep_h_ptiles, (c + 1 + kEpMaxRanks) * sizeof(RowTile),
                         cudaHostAllocDefault) == cudaSuccess &&
           cudaMalloc(&ctx->ep_tile_out, c * sizeof(unsigned long long)) == cudaSuccess &&
           cudaHostAlloc(&ctx->ep_h_tile_out, c * sizeof(unsigned long long),
                         cudaHostAllocDefault) == cudaSuccess;
      if (ok) ctx->ep_ptiles_cap = c;
    }
    if (!ok) cudaGetLastError();  // (reported through the handle exchange)
    // publish: status, pad, then a handle per buffer that peers write
    uint32_t* hs = h + kAgHx;
    std::memset(hs, 0, kHxWords * 4);
    for (int b = 0, k = 0; b < kEpBufs && ok; ++b) {
      if (!kEpShared[b]) continue;
      cudaIpcMemHandle_t hd;
      ok = cudaIpcGetMemHandle(&hd, ctx->ep_buf[b]) == cudaSuccess;
      std::memcpy(hs + 4 + 16 * k++, &hd, 64);
    }
    hs[0] = ok ? 1u : 0u;
    if (cudaMemcpyAsync(hx_send, hs, kHxWords * 4, cudaMemcpyHostToDevice, s) != cudaSuccess)
      return nccl_abort(ncclSystemError, "expert-parallel handle staging");
    EPP_NCCL(n.all_gather(hx_send, hx_recv, kHxWords, ncclUint32, comm, s),
             "ncclAllGather(handles)");
    uint32_t* hrv = h + kAgHx + kHxWords;
    if (cudaMemcpyAsync(hrv, hx_recv, static_cast<size_t>(R) * kHxWords * 4,
                        cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return nccl_abort(ncclSystemError, "expert-parallel handle readback");
    first_bad = -1;
    for (int q = 0; q < R && first_bad < 0; ++q)
      if (hrv[q * kHxWords] != 1u) first_bad = q;
    if (first_bad >= 0)
      return fail(ctx, TSG_ERR_CUDA, "expert-parallel: rank " + std::to_string(first_bad) +
                                         " could not allocate its exchange buffers");
    // map the peers' buffers (this rank's own are used directly)
    for (int q = 0; q < R; ++q)
      for (int b = 0, k = 0; b < kEpBufs; ++b) {
        if (q == me || !kEpShared[b]) {
          ctx->ep_peer[b][q] = q == me ? ctx->ep_buf[b] : nullptr;
          continue;
        }
        cudaIpcMemHandle_t hd;
        std::memcpy(&hd, hrv + q * kHxWords + 4 + 16 * k++, 64);
        void* ptr = nullptr;
        if (ok) ok = cudaIpcOpenMemHandle(&ptr, hd, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        ctx->ep_peer[b][q] = ok ? ptr : nullptr;
      }
    if (!ok) cudaGetLastError();  // (reported through the agreement)
    first_bad = -1;
    {
      const tsg_status st = barrier(5, ok, true, &all_ok, &first_bad);
      if (st != TSG_OK) return st;
    }
    if (!all_ok) {
      close_peer_views(ctx);
      return fail(ctx, TSG_ERR_CUDA, "expert-parallel: rank " + std::to_string(first_bad) +
                                         " could not map its peers' buffers");
    }
    for (int b = 0; b < kEpKinds; ++b) ctx->ep_caps[b] = cap[b];
  }
  __half* xp = static_cast<__half*>(ctx->ep_buf[kEpXp]);
  __half* act = static_cast<__half*>(ctx->ep_buf[kEpAct]);
  __half* ret = static_cast<__half*>(ctx->ep_buf[kEpRet]);
  const __half* rows_in = static_cast<const __half*>(ctx->ep_buf[kEpRows]);
  const uint32_t* map_in = static_cast<const uint32_t*>(ctx->ep_buf[kEpMap]);

  // ---- this rank's row tiles, each with its rows' destination, in chunks:
  // chunk c holds the pairs of source rank (me + 1 + c) % R, the last one
  // this rank's own pairs and its shared-expert rows.  With the copy-engine
  // return, a remote chunk's GEMM2 rows go to this rank's expanded-row
  // buffer (dead after GEMM1, same row order) and are copied on; else
  // straight into the source's return buffer ----
  const bool by_copy = ctx->ep_return == 1 && ctx->ep_chunk_ok && R > 1;
  const uint32_t rows_here = recv_pairs[me] + (sh ? T : 0u);
  RowTile* ht = ctx->ep_h_ptiles;
  unsigned long long* hto = ctx->ep_h_tile_out;
  const size_t tcap = ctx->ep_ptiles_cap;  // tiles; counts follow at tcap, tcap + 1 + c
  std::vector<uint32_t> chunk_first(R, 0), chunk_n(R, 0);
  uint32_t n_tiles = 0;
  for (int c = 0; c < R && local == TSG_OK; ++c) {
    const int q = (me + 1 + c) % R;
    chunk_first[c] = n_tiles;
    uint32_t row = rpo[me * R + q];    // in this rank's received pairs
    uint32_t back = soff[q * R + me];  // in q's sorted order
    __half* qret = static_cast<__half*>(ctx->ep_peer[kEpRet][q]);
    for (uint32_t j = 0; j < El; ++j) {
      const uint32_t cnt = M[q * W + me * El + j];
      for (uint32_t b = 0; b < cnt && local == TSG_OK; b += tr) {
        const uint32_t rows = std::min(tr, cnt - b);
        if (n_tiles >= tcap || static_cast<size_t>(back + b + rows) * D > ctx->ep_caps[kEpRet][q]) {
          note(fail(ctx, TSG_ERR_CUDA, "expert-parallel: tile plan exceeds a buffer"));
          break;
        }
        ht[n_tiles] = {j, row + b, rows, 0};
        __half* dst = by_copy && q != me ? xp + static_cast<size_t>(row + b) * D
                                         : qret + static_cast<size_t>(back + b) * D;
        hto[n_tiles] = reinterpret_cast<unsigned long long>(dst);
        ++n_tiles;
      }
      row += cnt;
      back += cnt;
    }
    if (q == me)
      for (uint32_t b = 0; sh && b < T && local == TSG_OK; b += tr) {
        const uint32_t rows = std::min(tr, T - b);
        if (n_tiles >= tcap) {
          note(fail(ctx, TSG_ERR_CUDA, "expert-parallel: tile plan exceeds a buffer"));
          break;
        }
        ht[n_tiles] = {El, recv_pairs[me] + b, rows, 0};
        hto[n_tiles] = reinterpret_cast<unsigned long long>(ret + static_cast<size_t>(P + b) * D);
        ++n_tiles;
      }
    chunk_n[c] = n_tiles - chunk_first[c];
  }
  if (local != TSG_OK) {
    n_tiles = 0;
    std::fill(chunk_n.begin(), chunk_n.end(), 0u);
  }
  ht[tcap].expert = n_tiles;
  for (int c = 0; c < R; ++c) ht[tcap + 1 + c].expert = chunk_n[c];
  ctx->ep_pntiles = &ctx->ep_ptiles[tcap].expert;
  auto cuda_note = [&](cudaError_t e, const char* where) {
    if (e != cudaSuccess) note(cuda_fail(ctx, e, where));
  };
  if (n_tiles) {
    cuda_note(cudaMemcpyAsync(ctx->ep_ptiles, ht, n_tiles * sizeof(RowTile), cudaMemcpyHostToDevice,
                              s),
              "tiles");
    cuda_note(cudaMemcpyAsync(ctx->ep_tile_out, hto, n_tiles * sizeof(unsigned long long),
                              cudaMemcpyHostToDevice, s),
              "tiles");
  }
  cuda_note(cudaMemcpyAsync(&ctx->ep_ptiles[tcap], &ht[tcap], (1 + R) * sizeof(RowTile),
                            cudaMemcpyHostToDevice, s),
            "tiles");
  // this rank's shared-expert rows (and the shared gate's dots) after the
  // pair rows it expands
  if (sh && T > 0 && local == TSG_OK) {
    const float* gate_w = L->has_gate ? L->router_rows + static_cast<size_t>(E) * D : nullptr;
    cuda_note(launch_gather_rows_gate(static_cast<const uint16_t*>(hidden), hidden_stride,
                                      rb.inv_rms, rb.sorted_pairs, 0, static_cast<int>(T),
                                      static_cast<int>(D), 1,
                                      xp + static_cast<size_t>(recv_pairs[me]) * D, gate_w,
                                      rb.gate_raw, s),
              "shared rows");
  }
  ev(2);
  // ---- dispatch: each token row once to every owner of one of its
  // experts, and each pair's row index, into the owners' buffers ----
  const bool staged_dispatch = ctx->ep_dispatch == 1 && ctx->ep_chunk_ok && R > 1;
  if (P > 0 && local == TSG_OK) {
    EpDispatch d{};
    d.x = static_cast<const uint16_t*>(hidden);
    d.x_stride = hidden_stride;
    d.inv_rms = rb.inv_rms;
    d.sorted_pairs = rb.sorted_pairs;
    d.slots = ctx->ep_slots;
    d.P = static_cast<int>(P);
    d.T = static_cast<int>(T);
    d.D = static_cast<int>(D);
    d.experts_per_rank = static_cast<int>(El);
    d.world = R;
    // with staging, the rows for a remote owner o go to this rank's stage
    // buffer (run st_off[o]) and the copy engines move each run; the map
    // entries (4 bytes a pair) are stored into the owners' maps directly
    std::vector<uint32_t> st_off(R, 0);
    uint32_t st_rows = 0;
    for (int o = 0; o < R; ++o)
      if (staged_dispatch && o != me) {
        st_off[o] = st_rows;
        st_rows += tok[me * R + o];
      }
    __half* stage = static_cast<__half*>(ctx->ep_buf[kEpStage]);
    for (int o = 0; o < R; ++o) {
      const bool st = staged_dispatch && o != me;
      d.rows[o] = st ? stage + static_cast<size_t>(st_off[o]) * D
                     : static_cast<__half*>(ctx->ep_peer[kEpRows][o]);
      d.map[o] = static_cast<uint32_t*>(ctx->ep_peer[kEpMap][o]);
      d.row0[o] = st ? 0u : rro[o * R + me];
      d.row_cap[o] = st ? tok[me * R + o]
                        : static_cast<uint32_t>(std::min<size_t>(ctx->ep_caps[kEpRows][o] / D,
                                                                 UINT32_MAX));
      d.map_base[o] = rro[o * R + me];
      d.n_rows[o] = tok[me * R + o];
      d.map0[o] = rpo[o * R + me];
      d.map_cap[o] = static_cast<uint32_t>(std::min<size_t>(ctx->ep_caps[kEpMap][o], UINT32_MAX));
      d.send_off[o] = soff[me * R + o];
      d.send_cnt[o] = snd[me * R + o];
    }
    d.err = rb.err;
    if (staged_dispatch && static_cast<size_t>(st_rows) * D > ctx->ep_buf_elems[kEpStage])
      note(fail(ctx, TSG_ERR_CUDA, "expert-parallel: stage buffer too small"));
    if (local == TSG_OK) cuda_note(launch_ep_dispatch(d, s), "dispatch");
    if (staged_dispatch && local == TSG_OK) {
      cuda_note(cudaEventRecord(ctx->ep_chunk_ev[0], s), "stage event");
      cuda_note(cudaStreamWaitEvent(ctx->ep_copy, ctx->ep_chunk_ev[0], 0), "stage event");
      for (int c = 1; c < R; ++c) {  // (rotated: at any moment the ranks send to different owners)
        const int o = (me + c) % R;
        const uint32_t cnt = tok[me * R + o];
        if (cnt)
          cuda_note(cudaMemcpyAsync(static_cast<__half*>(ctx->ep_peer[kEpRows][o]) +
                                        static_cast<size_t>(rro[o * R + me]) * D,
                                    stage + static_cast<size_t>(st_off[o]) * D,
                                    static_cast<size_t>(cnt) * D * sizeof(__half),
                                    cudaMemcpyDeviceToDevice, ctx->ep_copy),
                    "dispatch copy");
      }
      cuda_note(cudaEventRecord(ctx->ep_chunk_ev[R], ctx->ep_copy), "stage event");
      cuda_note(cudaStreamWaitEvent(s, ctx->ep_chunk_ev[R], 0), "stage event");
    }
  }
  {
    bool all_ok = false;
    const tsg_status st = barrier(2, local == TSG_OK, false, &all_ok, &first_bad);
    if (st != TSG_OK) return st;
  }
  ev(3);
  // ---- the received pairs' rows, in (source rank, expert) runs ----
  if (local == TSG_OK)
    cuda_note(launch_ep_expand(rows_in,
                               static_cast<uint32_t>(std::min<size_t>(ctx->ep_caps[kEpRows][me] / D,
                                                                      UINT32_MAX)),
                               map_in, static_cast<int>(recv_pairs[me]), static_cast<int>(D), xp,
                               rb.err, s),
              "expand");
  ev(4);
  // ---- the grouped contraction; GEMM2 writes each row to its token's rank ----
  if (n_tiles && local == TSG_OK) {
    QmmParams qp{};
    qp.D = static_cast<int>(D);
    qp.F = static_cast<int>(F);
    qp.E = static_cast<int>(El);
    qp.act = static_cast<int>(L->desc.activation);
    qp.n_rows_total = static_cast<int>(rows_here);
    qp.experts = expert_set(L);
    qp.row_tiles = ctx->ep_ptiles;
    qp.n_row_tiles = ctx->ep_pntiles;
    qp.xp = xp;
    qp.act_buf = act;
    qp.partials = ret;
    qp.tile_out = ctx->ep_tile_out;
    qp.err = rb.err;
    qp.num_sms = ctx->num_sms;
    cuda_note(launch_qmm_gate_up(qp, s), "qmm gate/up");
    ev(5);
    if (!by_copy) {
      if (local == TSG_OK) cuda_note(launch_qmm_down(qp, s), "qmm down");
    } else {
      // a chunk per source rank; each remote chunk's rows are copied to
      // their rank by the copy stream while the next chunk computes
      for (int c = 0; c < R && local == TSG_OK; ++c) {
        const int q = (me + 1 + c) % R;
        if (chunk_n[c]) {
          QmmParams qc = qp;
          qc.row_tiles = ctx->ep_ptiles + chunk_first[c];
          qc.n_row_tiles = &ctx->ep_ptiles[tcap + 1 + c].expert;
          qc.tile_out = ctx->ep_tile_out + chunk_first[c];
          cuda_note(launch_qmm_down(qc, s), "qmm down");
        }
        const uint32_t cnt = snd[q * R + me];
        if (q != me && cnt && local == TSG_OK) {
          cuda_note(cudaEventRecord(ctx->ep_chunk_ev[c], s), "chunk event");
          cuda_note(cudaStreamWaitEvent(ctx->ep_copy, ctx->ep_chunk_ev[c], 0), "chunk event");
          cuda_note(cudaMemcpyAsync(static_cast<__half*>(ctx->ep_peer[kEpRet][q]) +
                                        static_cast<size_t>(soff[q * R + me]) * D,
                                    xp + static_cast<size_t>(rpo[me * R + q]) * D,
                                    static_cast<size_t>(cnt) * D * sizeof(__half),
                                    cudaMemcpyDeviceToDevice, ctx->ep_copy),
                    "return copy");
        }
      }
      cuda_note(cudaEventRecord(ctx->ep_chunk_ev[R], ctx->ep_copy), "chunk event");
      cuda_note(cudaStreamWaitEvent(s, ctx->ep_chunk_ev[R], 0), "chunk event");
    }
  } else {
    ev(5);
  }
  ev(6);
  {
    bool all_ok = false;
    const tsg_status st = barrier(3, local == TSG_OK, false, &all_ok, &first_bad);
    if (st != TSG_OK) return st;
  }
#undef EPP_NCCL
  ev(7);
  if (local != TSG_OK) return fail(ctx, local, local_msg);
  // combine this rank's tokens, ranks in order (as on one GPU)
  if (T > 0) {
    CombineParams cp{};
    cp.T = static_cast<int>(T);
    cp.D = static_cast<int>(D);
    cp.K = static_cast<int>(K);
    cp.has_shared = L->has_shared;
    cp.E = static_cast<int>(E);
    cp.partials = ret;
    cp.pair_pos = rb.pair_pos;
    cp.weights = rb.weights;
    cp.gate_raw = L->has_gate ? rb.gate_raw : nullptr;
    cp.inv_rms = rb.inv_rms;
    cp.residual = residual;
    cp.y = y;
    cp.y_stride = y_stride;
    cp.y_f32 = y_dtype == TSG_DTYPE_F32 ? 1 : 0;
    TSG_CUDA_TRY(ctx, launch_combine(cp, s), "combine");
  }
  ev(8);
  return TSG_OK;
}

}  // namespace

extern "C" {

// Every rank of the group takes the same collective steps in the same order,
// whatever fails where: a local failure (bad arguments, a launch, an
// allocation, the pair counts) is carried to the peers in a status word at
// the next of two agreement points -- beside the count exchange, and after
// the plan and its allocations -- and then every rank returns together,
// before any further collective.  Past the second point nothing allocates;
// a CUDA failure there is reported after the return exchange, and an NCCL
// failure aborts the communicator (the group must be built again).
tsg_status tsg_ep_moe_block_forward(tsg_ctx ctx, tsg_moe_layer L, uint32_t expert_first,
                                    const void* hidden, uint32_t hidden_stride, uint32_t T,
                                    const float* residual, void* y, uint32_t y_stride,
                                    tsg_dtype y_dtype) {
  if (!ctx || !L) return fail(ctx, TSG_ERR_INVALID_ARG, "null context or layer");
  if (!ctx->nccl_comm) return fail(ctx, TSG_ERR_INVALID_ARG, "tsg_ep_init has not been called");
  const int R = ctx->ep_world, rank = ctx->ep_rank;
  const uint32_t E = L->desc.num_experts, K = L->desc.top_k, D = L->desc.d, F = L->desc.f;
  const NcclApi& n = nccl();
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  cudaStream_t s = ctx->stream;
  RouteBuffers& rb = ctx->rb;
  const uint32_t El = E % static_cast<uint32_t>(R) ? 0u : E / static_cast<uint32_t>(R);
  const uint32_t P = T * K;
  const uint32_t shared_rows = L->has_shared ? T : 0u;
  uint32_t* counts_recv = ctx->ep_counts_recv;      // [512]
  uint32_t* counts_send = ctx->ep_counts_recv + 512;  // [512]
  uint32_t* status_recv = ctx->ep_counts_recv + 1024;  // [2][1024]
  uint32_t* status_send = ctx->ep_counts_recv + 1024 + 2048;  // [2]
  uint32_t* hc = ctx->ep_h_counts;  // [E] sent, [E] received, [R] statuses

  // an NCCL failure leaves the group in no known state: abort it
  auto nccl_abort = [&](ncclResult_t r, const char* where) {
    if (n.comm_abort) n.comm_abort(comm);
    else n.comm_destroy(comm);
    ctx->nccl_comm = nullptr;
    return nccl_fail(ctx, r, where);
  };
#define EP_NCCL(expr, where)                                  \
  do {                                                        \
    const ncclResult_t r__ = (expr);                          \
    if (r__ != ncclSuccess) return nccl_abort(r__, where);    \
  } while (0)
  // agreement: every rank sends its status word to every peer; true when
  // every rank (this one included) is fine
  auto agree = [&](int round, bool ok_local) -> tsg_status {
    if (cudaMemsetAsync(status_send + round, ok_local ? 1 : 0, 4, s) != cudaSuccess) ok_local = false;
    EP_NCCL(n.group_start(), "ncclGroupStart");
    for (int q = 0; q < R; ++q) {
      EP_NCCL(n.send(status_send + round, 1, ncclUint32, q, comm, s), "ncclSend(status)");
      EP_NCCL(n.recv(status_recv + round * 1024 + q, 1, ncclUint32, q, comm, s),
              "ncclRecv(status)");
    }
    EP_NCCL(n.group_end(), "ncclGroupEnd");
    return TSG_OK;
  };
  auto read_statuses = [&](int round, bool* all_ok, int* first_bad) -> tsg_status {
    if (cudaMemcpyAsync(hc + 2 * 512, status_recv + round * 1024, R * 4u,
                        cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return fail(ctx, TSG_ERR_CUDA, "expert-parallel: status readback");
    *all_ok = true;
    for (int q = 0; q < R; ++q)
      if (hc[2 * 512 + q] == 0u) {
        *all_ok = false;
        if (*first_bad < 0) *first_bad = q;
      }
    return TSG_OK;
  };

  const bool peer = ctx->ep_transport == 1;
  if (peer && R > kEpMaxRanks)  // (the same on every rank: all return here)
    return fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "peer transport: at most 16 ranks");
  if (peer && ctx->ep_ev_ok) cudaEventRecord(ctx->ep_ev[0], s);
  uint32_t* csend = peer ? ctx->ep_ag : counts_send;

  // ---- phase 1 (local): checks, routing, sorting, the rows to send ----
  tsg_status local = TSG_OK;
  std::string local_msg;
  auto note = [&](tsg_status st) {
    if (local == TSG_OK && st != TSG_OK) {
      local = st;
      local_msg = ctx->last_error;
    }
  };
  note(check_common(ctx, L, hidden, hidden_stride, T, y, y_stride, y_dtype));
  if (local == TSG_OK && El == 0)
    note(fail(ctx, TSG_ERR_UNSUPPORTED_SHAPE, "numExperts must be a multiple of the group size"));
  if (local == TSG_OK && expert_first != static_cast<uint32_t>(rank) * El)
    note(fail(ctx, TSG_ERR_INVALID_ARG, "expert_first must be rank * numExperts / world"));
  if (local == TSG_OK) note(take_pending_error(ctx));
  if (local == TSG_OK) note(ensure_workspace(ctx, layer_caps(L, std::max<uint32_t>(T, 1))));
  if (local == TSG_OK) {
    ctx->last_T = T;
    ctx->last_K = K;
  }
  // the dense branch, local (every rank holds it in full); its result is the
  // residual of the routed combine
  if (local == TSG_OK && L->dense && T > 0) {
    note(run_dense_branch(ctx, L, hidden, hidden_stride, T, residual, ctx->dense_y, D,
                          TSG_DTYPE_F32));
    residual = ctx->dense_y;
  }
  // route and group this rank's tokens over all E experts: the sorted order
  // puts the pairs of each owner rank in one contiguous run
  auto route = [&]() -> tsg_status {
    if (T > 0) {
      const RouterParams p = router_params(L, hidden, hidden_stride, T);
      TSG_CUDA_TRY(ctx, launch_router_prefill(p, rb, s), "router");
      TSG_CUDA_TRY(ctx, launch_permute(p, rb, nullptr, s), "permute");
      const float* gate_w = L->has_gate ? L->router_rows + static_cast<size_t>(E) * D : nullptr;
      if (!peer)  // (the peer transport converts the rows as it sends them)
        TSG_CUDA_TRY(ctx,
                     launch_gather_rows_gate(static_cast<const uint16_t*>(hidden), hidden_stride,
                                             rb.inv_rms, rb.sorted_pairs, static_cast<int>(P),
                                             static_cast<int>(T), static_cast<int>(D),
                                             L->has_shared, ctx->xp, gate_w, rb.gate_raw, s),
                     "gather rows");
      TSG_CUDA_TRY(ctx, cudaMemcpyAsync(csend, rb.counts, E * 4u, cudaMemcpyDeviceToDevice, s),
                   "counts");
      if (peer) {
        // each token's slot among the rows sent to each owner, and the
        // number of rows per owner beside the counts
        TSG_CUDA_TRY(ctx, grow(&ctx->ep_slots, &ctx->ep_slots_cap, static_cast<size_t>(R) * T),
                     "cudaMalloc");
        TSG_CUDA_TRY(ctx,
                     launch_ep_owner_slots(rb.ids, static_cast<int>(T), static_cast<int>(K),
                                           static_cast<int>(El), R, ctx->ep_slots, csend + E, s),
                     "owner slots");
      }
    } else {
      TSG_CUDA_TRY(ctx, cudaMemsetAsync(csend, 0, (E + (peer ? R : 0)) * 4u, s), "memset");
    }
    return TSG_OK;
  };
  if (local == TSG_OK) note(route());
  if (local != TSG_OK) cudaMemsetAsync(csend, 0, 512 * 4u, s);  // (what is sent is not read)
  if (peer) {
    const tsg_status st = ep_peer_forward(ctx, L, hidden, hidden_stride, T, residual, y, y_stride,
                                          y_dtype, local, local_msg);
    return st;
  }

  // ---- agreement 1, with the per-expert pair counts to their owners ----
  const uint32_t Elx = El ? El : E / static_cast<uint32_t>(R);  // counts each peer expects
  {
    bool ok_local = local == TSG_OK;
    if (cudaMemsetAsync(status_send, ok_local ? 1 : 0, 4, s) != cudaSuccess) ok_local = false;
    EP_NCCL(n.group_start(), "ncclGroupStart");
    for (int q = 0; q < R; ++q) {
      if (Elx) {
        EP_NCCL(n.send(counts_send + q * Elx, Elx, ncclUint32, q, comm, s), "ncclSend(counts)");
        EP_NCCL(n.recv(counts_recv + q * Elx, Elx, ncclUint32, q, comm, s), "ncclRecv(counts)");
      }
      EP_NCCL(n.send(status_send, 1, ncclUint32, q, comm, s), "ncclSend(status)");
      EP_NCCL(n.recv(status_recv + q, 1, ncclUint32, q, comm, s), "ncclRecv(status)");
    }
    EP_NCCL(n.group_end(), "ncclGroupEnd");
  }
  bool all_ok = false;
  int first_bad = -1;
  if (cudaMemcpyAsync(hc, counts_send, E * 4u, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyAsync(hc + E, counts_recv, E * 4u, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    note(fail(ctx, TSG_ERR_CUDA, "expert-parallel: counts readback"));
  {
    const tsg_status st = read_statuses(0, &all_ok, &first_bad);
    if (st != TSG_OK) return nccl_abort(ncclSystemError, "expert-parallel status readback");
  }
  if (local != TSG_OK) return fail(ctx, local, local_msg);
  if (!all_ok)
    return fail(ctx, TSG_ERR_NCCL, "expert-parallel: rank " + std::to_string(first_bad) +
                                       " failed before the row exchange (its own call reports why)");

  // ---- phase 2 (local): the plan and its buffers ----
  // send/receive runs per peer, and the local row tiles -- one run per
  // (source rank, local expert), then the shared expert's rows
  std::vector<uint32_t> send_cnt(R), send_off(R), recv_cnt(R), recv_off(R);
  uint32_t so = 0, ro = 0;
  for (int q = 0; q < R; ++q) {
    uint32_t sc = 0, rc = 0;
    for (uint32_t j = 0; j < El; ++j) {
      sc += hc[q * El + j];
      rc += hc[E + q * El + j];
    }
    send_cnt[q] = sc;
    send_off[q] = so;
    recv_cnt[q] = rc;
    recv_off[q] = ro;
    so += sc;
    ro += rc;
  }
  if (so != P) note(fail(ctx, TSG_ERR_CUDA, "expert-parallel: pair counts do not add up"));
  const uint32_t recv_rows = ro;
  const uint32_t rows_local = recv_rows + shared_rows;
  const uint32_t tr = static_cast<uint32_t>(qmm_tile_rows());
  std::vector<RowTile> tiles;
  for (int q = 0; q < R; ++q) {
    uint32_t off = recv_off[q];
    for (uint32_t j = 0; j < El; ++j) {
      const uint32_t c = hc[E + q * El + j];
      for (uint32_t b = 0; b < c; b += tr) tiles.push_back({j, off + b, std::min(tr, c - b), 0});
      off += c;
    }
  }
  for (uint32_t b = 0; b < shared_rows; b += tr)
    tiles.push_back({El, recv_rows + b, std::min(tr, shared_rows - b), 0});
  const uint32_t n_tiles = static_cast<uint32_t>(tiles.size());
  auto buffers = [&]() -> tsg_status {
    // (the stream is idle here, so buffers can be replaced)
    if (rows_local > ctx->ep_rows_cap || static_cast<size_t>(D) * ctx->ep_rows_cap == 0) {
      const size_t rows = std::max<size_t>(rows_local + rows_local / 4, 1024);
      size_t c1 = 0, c2 = 0, c3 = 0;
      ctx->ep_rows_cap = 0;
      TSG_CUDA_TRY(ctx, grow(&ctx->ep_rows, &c1, rows * D), "cudaMalloc");
      TSG_CUDA_TRY(ctx, grow(&ctx->ep_act, &c2, rows * F), "cudaMalloc");
      TSG_CUDA_TRY(ctx, grow(&ctx->ep_out, &c3, rows * D), "cudaMalloc");
      ctx->ep_rows_cap = rows;
    }
    TSG_CUDA_TRY(ctx, grow(&ctx->ep_ret, &ctx->ep_ret_cap, static_cast<size_t>(P + shared_rows) * D),
                 "cudaMalloc");
    if (!ctx->ep_tiles || ctx->ep_tiles_cap < n_tiles + 1) {
      if (ctx->ep_tiles) cudaFree(ctx->ep_tiles);
      if (ctx->ep_h_tiles) cudaFreeHost(ctx->ep_h_tiles);
      ctx->ep_tiles = nullptr;
      ctx->ep_h_tiles = nullptr;
      ctx->ep_tiles_cap = 0;
      const size_t cap = std::max<size_t>(2 * (n_tiles + 1), 256);
      TSG_CUDA_TRY(ctx, cudaMalloc(&ctx->ep_tiles, (cap + 1) * sizeof(RowTile)), "cudaMalloc");
      TSG_CUDA_TRY(ctx, cudaHostAlloc(&ctx->ep_h_tiles, (cap + 1) * sizeof(RowTile),
                                      cudaHostAllocDefault), "cudaHostAlloc");
      ctx->ep_tiles_cap = cap;
    }
    // the tile count rides in the slot after the tiles
    RowTile* ht = ctx->ep_h_tiles;
    std::copy(tiles.begin(), tiles.end(), ht);
    ht[ctx->ep_tiles_cap].expert = n_tiles;
    ctx->ep_ntiles = &ctx->ep_tiles[ctx->ep_tiles_cap].expert;
    if (n_tiles)
      TSG_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->ep_tiles, ht, n_tiles * sizeof(RowTile),
                                        cudaMemcpyHostToDevice, s), "tiles");
    TSG_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->ep_ntiles, &ht[ctx->ep_tiles_cap].expert,
                                      sizeof(uint32_t), cudaMemcpyHostToDevice, s), "tiles");
    return TSG_OK;
  };
  if (local == TSG_OK) note(buffers());

  // ---- agreement 2: every rank's plan and buffers are in place ----
  {
    const tsg_status st = agree(1, local == TSG_OK);
    if (st != TSG_OK) return st;
  }
  first_bad = -1;
  {
    const tsg_status st = read_statuses(1, &all_ok, &first_bad);
    if (st != TSG_OK) return nccl_abort(ncclSystemError, "expert-parallel status readback");
  }
  if (local != TSG_OK) return fail(ctx, local, local_msg);
  if (!all_ok)
    return fail(ctx, TSG_ERR_NCCL, "expert-parallel: rank " + std::to_string(first_bad) +
                                       " failed before the row exchange (its own call reports why)");

  // ---- phase 3: dispatch, contraction, return, combine (no allocation; a
  // CUDA failure is reported after the return exchange) ----
  auto cuda_note = [&](cudaError_t e, const char* where) {
    if (e != cudaSuccess) note(cuda_fail(ctx, e, where));
  };
  const size_t rowb = D;  // elements per row
  EP_NCCL(n.group_start(), "ncclGroupStart");
  for (int q = 0; q < R; ++q) {
    if (send_cnt[q])
      EP_NCCL(n.send(ctx->xp + send_off[q] * rowb, send_cnt[q] * rowb, ncclFloat16, q, comm, s),
              "ncclSend(rows)");
    if (recv_cnt[q])
      EP_NCCL(n.recv(ctx->ep_rows + recv_off[q] * rowb, recv_cnt[q] * rowb, ncclFloat16, q, comm,
                     s),
              "ncclRecv(rows)");
  }
  EP_NCCL(n.group_end(), "ncclGroupEnd");
  if (shared_rows)
    cuda_note(cudaMemcpyAsync(ctx->ep_rows + recv_rows * rowb, ctx->xp + P * rowb,
                              shared_rows * rowb * 2, cudaMemcpyDeviceToDevice, s),
              "shared rows");
  // the grouped contraction over the rows this rank holds
  if (n_tiles && local == TSG_OK) {
    QmmParams qp{};
    qp.D = static_cast<int>(D);
    qp.F = static_cast<int>(F);
    qp.E = static_cast<int>(El);
    qp.act = static_cast<int>(L->desc.activation);
    qp.n_rows_total = static_cast<int>(rows_local);
    qp.experts = expert_set(L);
    qp.row_tiles = ctx->ep_tiles;
    qp.n_row_tiles = ctx->ep_ntiles;
    qp.xp = ctx->ep_rows;
    qp.act_buf = ctx->ep_act;
    qp.partials = ctx->ep_out;
    qp.err = rb.err;
    qp.num_sms = ctx->num_sms;
    cuda_note(launch_qmm_gate_up(qp, s), "qmm gate/up");
    if (local == TSG_OK) cuda_note(launch_qmm_down(qp, s), "qmm down");
  }
  // return the outputs to the tokens' ranks, into their sorted positions
  EP_NCCL(n.group_start(), "ncclGroupStart");
  for (int q = 0; q < R; ++q) {
    if (recv_cnt[q])
      EP_NCCL(n.send(ctx->ep_out + recv_off[q] * rowb, recv_cnt[q] * rowb, ncclFloat16, q, comm,
                     s),
              "ncclSend(outputs)");
    if (send_cnt[q])
      EP_NCCL(n.recv(ctx->ep_ret + send_off[q] * rowb, send_cnt[q] * rowb, ncclFloat16, q, comm,
                     s),
              "ncclRecv(outputs)");
  }
  EP_NCCL(n.group_end(), "ncclGroupEnd");
#undef EP_NCCL
  if (local != TSG_OK) return fail(ctx, local, local_msg);
  if (shared_rows)
    TSG_CUDA_TRY(ctx, cudaMemcpyAsync(ctx->ep_ret + P * rowb, ctx->ep_out + recv_rows * rowb,
                                      shared_rows * rowb * 2, cudaMemcpyDeviceToDevice, s),
                 "shared outputs");

  // combine this rank's tokens, ranks in order (as on one GPU)
  if (T > 0) {
    CombineParams cp{};
    cp.T = static_cast<int>(T);
    cp.D = static_cast<int>(D);
    cp.K = static_cast<int>(K);
    cp.has_shared = L->has_shared;
    cp.E = static_cast<int>(E);
    cp.partials = ctx->ep_ret;
    cp.pair_pos = rb.pair_pos;
    cp.weights = rb.weights;
    cp.gate_raw = L->has_gate ? rb.gate_raw : nullptr;
    cp.inv_rms = rb.inv_rms;
    cp.residual = residual;
    cp.y = y;
    cp.y_stride = y_stride;
    cp.y_f32 = y_dtype == TSG_DTYPE_F32 ? 1 : 0;
    TSG_CUDA_TRY(ctx, launch_combine(cp, s), "combine");
  }
  return TSG_OK;
}

tsg_status tsg_ep_phase_ms(tsg_ctx ctx, float* ms, int n) {
  if (!ctx || (!ms && n > 0)) return fail(ctx, TSG_ERR_INVALID_ARG, "null argument");
  if (!ctx->ep_ev_ok) return fail(ctx, TSG_ERR_INVALID_ARG, "tsg_ep_init has not been called");
  TSG_CUDA_TRY(ctx, cudaEventSynchronize(ctx->ep_ev[8]), "phase events");
  for (int i = 0; i < n && i < 8; ++i) {
    float t = 0.0f;
    TSG_CUDA_TRY(ctx, cudaEventElapsedTime(&t, ctx->ep_ev[i], ctx->ep_ev[i + 1]), "phase events");
    ms[i] = t;
  }
  return TSG_OK;
}

}  // extern "C"
