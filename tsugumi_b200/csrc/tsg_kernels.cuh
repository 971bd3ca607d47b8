// tsg_kernels.cuh -- launch-side declarations shared by the .cu files and the
// C-ABI implementation.  Plain structs of device pointers and sizes.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tsg {

// cuTensorMapEncodeTiled, found once through the runtime's driver entry
// point query (nullptr when the driver does not offer it).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();

// Byte offsets of an expert's sub-tensors inside its blob (MoEExpertOffsets,
// Sources/Tsugumi/Kernels/MoE/MoE.swift:4-29).  Bias offsets are carried
// for layout compatibility and never read: the scheme is symmetric.
struct ExpertOffsets {
  uint32_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b;
};

// 16-byte token/expert pair (PrefillTokenExpertPair,
// Sources/Tsugumi/Kernels/Prefill/MoE/PrefillRouter.swift:4-28).
struct Pair {
  uint32_t token, expert, rank, weight_bits;
};

struct Group {
  uint32_t expert, pair_start, pair_count;
};

struct Tile {
  uint32_t group_start, group_count, pair_start, pair_count;
};

// One unit of the grouped contraction's schedule: `rows` consecutive sorted
// rows starting at `row_start`, all routed to `expert` (expert == E marks
// the shared expert).
struct RowTile {
  uint32_t expert, row_start, rows, pad;
};

// Everything a kernel needs to find an expert's weights.
struct ExpertSet {
  const uint8_t* base;     // expert 0's blob
  uint64_t stride;         // bytes between blobs
  ExpertOffsets off;
  const uint8_t* shared;   // shared expert's blob, or nullptr
  ExpertOffsets shared_off;
};

// Per-layer routing workspace written by the router / permutation kernels.
struct RouteBuffers {
  float* logits_raw;      // [ksplit, T, E] raw router dots (no norm factor)
  float* gate_raw;        // [T] raw shared-gate dot w_s . x (no norm factor)
  float* sumsq;           // [ksplit, T] row sums of squares
  float* inv_rms;         // [T]
  uint32_t* ids;          // [T, K]
  float* weights;         // [T, K]
  uint16_t* weights_f16;  // [T, K] (optional)
  uint32_t* counts;       // [E]
  uint32_t* offsets;      // [E] (0xFFFFFFFF when empty)
  Pair* sorted_pairs;     // [T*K]
  uint32_t* pair_pos;     // [T*K]: sorted position of token-major pair t*K+r
  Group* groups;          // [E]
  uint32_t* n_groups;     // [1]
  Tile* tiles;            // [E]
  uint32_t* n_tiles;      // [1]
  RowTile* row_tiles;     // [ceil(T*K/tile_rows) + E + ceil(T/tile_rows)]
  uint32_t* n_row_tiles;  // [1]
  float* xn;              // [T, D] decode only: x * inv_rms in fp32
  float* xs8;             // [T, D/8] decode only: 1.5 x sum of each 8-element run of xn
  uint32_t* hist;         // [permute_chunks(T*K), E] per-chunk expert counts, then prefixes
  uint32_t* sync_counter; // [1] last-CTA counter, self-resetting
  uint32_t* err;          // [1] device error word
};

struct RouterParams {
  const uint16_t* x;       // [T, x_stride] bf16
  uint32_t x_stride;
  int T, D, E, K;
  const float* w;          // [E + has_gate, D] router rows (effective scale folded in)
  const void* w_bf16x3;    // [3][router_tc_pad(E)][D] bf16 hi/mid/lo planes of w, or nullptr
  int has_gate;            // 1: row E is the shared-expert gate vector
  int has_shared;          // 1: the layer has a shared expert
  const float* per_expert_scale;  // [E] or nullptr
  const float* logit_bias;        // [E] or nullptr
  int norm;                // 1: no-scale RMSNorm of x
  float eps;
  int tile_rows;           // rows per RowTile in the schedule
  int tile_expert_count;   // PrefillMoEGrouping tiles
  int tile_break;          // forced tile cut after this group, -1 none
  const uint64_t* sort_keys;  // [E] or nullptr
};

// router.cu
cudaError_t launch_router_decode(const RouterParams& p, const RouteBuffers& rb,
                                 cudaStream_t s);
// With logits_out, writes the fp32 logits [T][E] (norm factor and bias
// applied) instead of selecting.
cudaError_t launch_router_prefill(const RouterParams& p, const RouteBuffers& rb,
                                  cudaStream_t s, float* logits_out = nullptr);
cudaError_t launch_rowprep(const RouterParams& p, const RouteBuffers& rb, int write_rows,
                           cudaStream_t s);
cudaError_t launch_group_small(const RouterParams& p, const RouteBuffers& rb, cudaStream_t s);

// router_tc.cu: the prefill router GEMM on tcgen05 (exact fp32 through three
// bf16 planes of the router rows, made once per layer)
int router_tc_pad(int E);
cudaError_t launch_split_router(const float* w, int E, int D, void* planes, cudaStream_t s);
bool router_tc_usable(const RouterParams& p);
int router_tc_ksplit(int T, int E, int D);
cudaError_t launch_router_tc(const RouterParams& p, const RouteBuffers& rb, int ksplit,
                             cudaStream_t s);
// permute.cu
// Chunks of the permutation's counting sort (RouteBuffers::hist rows).
int permute_chunks(int P);
cudaError_t launch_permute(const RouterParams& p, const RouteBuffers& rb, const Pair* pairs_in,
                           cudaStream_t s);
cudaError_t launch_make_pairs(const uint32_t* ids, const uint16_t* w_f16, int T, int K,
                              Pair* out, cudaStream_t s);
cudaError_t launch_gather_rows_gate(const uint16_t* x, uint32_t x_stride, const float* inv_rms,
                                    const Pair* sorted_pairs, int n_rows, int T, int D,
                                    int append_tokens, __half* xp, const float* gate_w,
                                    float* gate_raw, cudaStream_t s, int frag_order = 0);

// Expert parallelism over peer memory.  A token is sent once to each rank
// that owns at least one of its experts: slots[o][t] is the token's index
// among the tokens this rank sends to owner o (token order), kEpNoSlot when
// none of its experts is on o; counts[o] the number of such tokens.
constexpr int kEpMaxRanks = 16;
constexpr uint32_t kEpNoSlot = 0xFFFFFFFFu;
cudaError_t launch_ep_owner_slots(const uint32_t* ids, int T, int K, int experts_per_rank,
                                  int world, uint32_t* slots, uint32_t* counts, cudaStream_t s);
// The dispatch writes the token's fp16 row (gather_rows_kernel's conversion)
// to row row0[o] + slot of rows[o] (the owner's buffer, or a local run that
// is copied there), and for pair i of this rank's sorted order, owned by o,
// the row's index in the owner's buffer, map_base[o] + slot, to entry
// map0[o] + (i - send_off[o]) of map[o].
struct EpDispatch {
  const uint16_t* x;
  uint32_t x_stride;
  const float* inv_rms;
  const Pair* sorted_pairs;
  const uint32_t* slots;  // [world][T]
  int P, T, D, experts_per_rank, world;
  __half* rows[kEpMaxRanks];
  uint32_t* map[kEpMaxRanks];
  uint32_t row0[kEpMaxRanks], row_cap[kEpMaxRanks], n_rows[kEpMaxRanks];  // rows: first, capacity, sent
  uint32_t map_base[kEpMaxRanks];  // a pair's map entry: map_base[o] + the token's slot
  uint32_t map0[kEpMaxRanks], map_cap[kEpMaxRanks];
  uint32_t send_off[kEpMaxRanks], send_cnt[kEpMaxRanks];  // this rank's pairs to o
  uint32_t* err;
};
cudaError_t launch_ep_dispatch(const EpDispatch& d, cudaStream_t s);
// The owner's expansion: xp[i] = rows[map[i]] for the n pairs it received.
cudaError_t launch_ep_expand(const __half* rows, uint32_t rows_cap, const uint32_t* map, int n,
                             int D, __half* xp, uint32_t* err, cudaStream_t s);

// decode.cu
struct DecodeParams {
  int T, D, F, E, K, act, has_shared;
  const uint16_t* x;  // [T, x_stride] bf16
  uint32_t x_stride;
  ExpertSet experts;
  RouteBuffers rb;
  __half* act_buf;    // [T*K + T, F]
  const float* xn;    // [T, D] normalised input, fp32 (written by the router)
  const float* xs8;   // [T, D/8] 1.5 x sums of 8-element runs of xn
  void* y;            // [T, y_stride]
  uint32_t y_stride;
  int y_f32;
  const float* residual;  // [T, D] fp32 or nullptr
  int num_sms;
};
cudaError_t launch_decode_experts(const DecodeParams& p, cudaStream_t s);
cudaError_t launch_decode_gate_up(const DecodeParams& p, cudaStream_t s);
cudaError_t launch_decode_down(const DecodeParams& p, cudaStream_t s);

// decode_fused.cu: the whole block for T <= 4 in one cooperative kernel
struct DecodeFusedArgs {
  const uint16_t* x;
  uint32_t x_stride;
  int T, D, F, E, K, act, norm;
  float eps;
  const float* router_rows;
  int has_gate, has_shared;
  const float* per_expert_scale;
  const float* logit_bias;
  const uint32_t* ids_in;  // caller routing, or nullptr
  const float* w_in;
  ExpertSet experts;
  void* y;
  uint32_t y_stride;
  int y_f32;
  const float* residual;
  void* logits;     // [4][T][E + 1] (tag, logit) words
  float* inv_rms;   // [T]
  void* actfrag;    // [T*K + T][F] fp16, fragment order
  uint32_t* counters;  // [4 + D / 16], zero between launches
  uint32_t* ids_out;
  float* w_out;
  uint16_t* w16_out;
  Pair* pairs_out;
  uint32_t* err;
  int num_sms;
  int allow_pdl;
  int cooperative;  // launch with the cooperative attribute (co-residency checked by the driver)
  unsigned long long* stamps;  // debug phase timestamps [grid][8], or nullptr
};
// decode_stream.cu: the same block, streaming every selected weight byte in
// one phase.  Its down slices arrive by TMA; the maps are encoded once per
// layer (routed experts, and the shared expert when there is one).
struct DecodeMaps {
  CUtensorMap down128, down16;    // routed down codes: [E][D][F/2], 32-byte x 128 / 16 rows
  CUtensorMap sdown128, sdown16;  // the shared expert's [D][F/2]
  CUtensorMap gate8, up8;         // routed gate / up codes: 8 rows x D/2 bytes, 128-byte swizzle
  CUtensorMap sgate8, sup8;       // the shared expert's
};
bool encode_decode_maps(const ExpertSet& ex, int D, int F, int E, DecodeMaps* out);
bool decode_stream_supported(int T, int D, int F, int K, int E, int has_gate, int has_shared,
                             int num_sms);
// workspace of decode_stream (bytes) for at most T tokens: partial sums,
// and the tagged act words (zero at allocation and after an error)
size_t decode_stream_scratch_bytes(int T, int D, int F, int K);
size_t decode_stream_flag_bytes(int T, int F, int K);
cudaError_t launch_decode_stream(const DecodeFusedArgs& a, const DecodeMaps& maps,
                                 void* scratch, void* acts, cudaStream_t s);

bool decode_fused_supported(int T, int K, int E, int has_gate, int num_sms);
bool decode_fused_fits(int T, int D, int F, int K, int has_shared, int num_sms);
cudaError_t launch_decode_fused(const DecodeFusedArgs& a, cudaStream_t s);

// umma.cu
struct QmmParams {
  int D, F, E, act, n_rows_total;  // n_rows_total: rows of xp / act / partials
  ExpertSet experts;
  const RowTile* row_tiles;
  const uint32_t* n_row_tiles;
  int max_row_tiles;
  const __half* xp;      // [rows, D] fp16 (GEMM1 input)
  __half* act_buf;       // [rows, F] fp16 (GEMM1 output, GEMM2 input)
  __half* partials;      // [rows, D] fp16 (GEMM2 output)
  // optional: per row tile, where GEMM2 writes the tile's rows instead of
  // partials (row r of the tile at tile_out[tile] + r * D; expert
  // parallelism points these into the token's rank's memory)
  const unsigned long long* tile_out;
  uint32_t* err;
  int num_sms;
};
// The launchers encode their own tensor maps (token rows of xp / act_buf,
// int4 code planes of the routed and shared experts); a failed encode is
// reported as cudaErrorInvalidValue.
cudaError_t launch_qmm_gate_up(const QmmParams& p, cudaStream_t s);
cudaError_t launch_qmm_down(const QmmParams& p, cudaStream_t s);
int qmm_tile_rows();

// gemv.cu: the same products as batched GEMVs for row tiles of at most
// max_rows <= 64 rows
cudaError_t launch_gemv_gate_up(const QmmParams& p, int max_rows, cudaStream_t s);
cudaError_t launch_gemv_down(const QmmParams& p, int max_rows, cudaStream_t s);
int gemv_max_tile_rows();
bool gemv_usable(const QmmParams& p);  // D % 128 == 0, F % 64 == 0, aligned scales

// combine.cu
struct CombineParams {
  int T, D, K, has_shared, E;
  const __half* partials;   // [T*K (+T), D] in sorted order (+ shared rows in token order)
  const uint32_t* pair_pos; // [T*K]
  const float* weights;     // [T, K]
  const float* gate_raw;    // [T] raw shared-gate dot, or nullptr (ungated)
  const float* inv_rms;     // [T]
  const float* residual;    // [T, D] fp32 or nullptr
  void* y;
  uint32_t y_stride;
  int y_f32;
};
cudaError_t launch_combine(const CombineParams& p, cudaStream_t s);
cudaError_t launch_reduce_token_major(const __half* partials, const float* w, int T, int K, int D,
                                      void* h2, int h2_f32, cudaStream_t s);

// fusions.cu: the norms and residuals around Gemma's MoE block
struct GemmaNorms {
  const uint16_t* post_attn;    // [D] bf16: post-attention norm weight
  const uint16_t* pre_ffn;      // [D] bf16: the dense branch's input norm weight
  const uint16_t* pre_ffn2;     // [D] bf16: the routed experts' input norm weight
  const uint16_t* post_dense;   // [D] bf16: the dense branch's output norm weight
  const uint16_t* post_routed;  // [D] bf16: the routed output's norm weight
  const uint16_t* post_ffn;     // [D] bf16: the summed branches' norm weight
  float eps;
  float layer_scalar;
};
cudaError_t launch_gemma_setup(uint16_t* hidden, uint32_t h_stride, const uint16_t* attn,
                               uint32_t a_stride, int T, int D, const GemmaNorms& n,
                               uint16_t* router_x, uint16_t* routed_x, uint16_t* dense_x,
                               cudaStream_t s);
cudaError_t launch_gemma_tail(const float* h2, const float* h1, uint16_t* hidden, uint32_t h_stride,
                              int T, int D, const GemmaNorms& n, cudaStream_t s);

// import.cu: one int4 matrix of a .moepack blob (U32 codes, BF16 scales of
// `group` elements, optional BF16 biases) into codes bytes + fp16 32-group
// scales, exactly (failures recorded in err: code 10 scale, 11 bias)
cudaError_t launch_import_int4(const void* codes, const uint16_t* scales, const uint16_t* biases,
                               int rows, int cols, int group, void* out_codes, __half* out_scales,
                               uint32_t* err, cudaStream_t s);

}  // namespace tsg
