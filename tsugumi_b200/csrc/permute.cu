// permute.cu -- the token->expert permutation on the GPU.
//
// Restates PrefillMoEGrouping.groupTokenExpertPairs
// (Sources/Tsugumi/Kernels/Prefill/MoE/PrefillMoEGrouping.swift:91-201), which
// the reference runs on the CPU, as a stable counting sort over the
// token-major pairs, in chunks of kChunk pairs:
//   0. (caller-supplied pairs only) validate each pair and place it at its
//      token-major slot token*K + rank; a second pair for the same slot is a
//      duplicate (PrefillMoEGroupingError.duplicateTokenRank);
//   1. one CTA per chunk histograms its expert ids in shared memory;
//   2. one CTA turns the histograms into per-(chunk, expert) prefixes and the
//      per-expert counts, orders the experts (by optional sort key, then
//      index), scans the counts into offsets (UINT32_MAX for empty experts),
//      and writes the groups, the tiles of <= tileExpertCount groups (with
//      the optional forced cut) and the row-tile schedule of the grouped
//      contraction;
//   3. one CTA per chunk writes its pairs to their sorted positions, ranking
//      equal ids inside a warp with match/popc and across warps with
//      per-warp counts, so the order inside an expert is (token, rank).
// Output is bit-identical to the reference's sort by (key, expert, token,
// rank).
#include "int4_mma.cuh"
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 2048;       // pairs per histogram / scatter CTA
constexpr int kScanThreads = 512;

// Error record: [0] bits, [1] first error code, [2] offending value.
TSG_DEV void record_error(uint32_t* err, uint32_t code, uint32_t value) {
  if (!err) return;
  atomicOr(err, TSG_DEVERR_METADATA);
  if (atomicCAS(err + 1, 0u, code) == 0u) err[2] = value;
}

// ---- 1. caller pairs -> token-major slots ----------------------------------
__global__ void place_pairs_kernel(const Pair* pairs, int n, int T, int K, int E,
                                   uint32_t* tm_ids, uint16_t* tm_w16, uint32_t* occupied,
                                   uint32_t* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const Pair pr = pairs[i];
  // codes follow PrefillMoEGroupingError: 6 token, 7 rank, 8 expert, 9 duplicate
  if (pr.token >= static_cast<uint32_t>(T)) { record_error(err, 6u, pr.token); return; }
  if (pr.rank >= static_cast<uint32_t>(K)) { record_error(err, 7u, pr.rank); return; }
  if (pr.expert >= static_cast<uint32_t>(E)) { record_error(err, 8u, pr.expert); return; }
  const uint32_t slot = pr.token * static_cast<uint32_t>(K) + pr.rank;
  if (atomicExch(&occupied[slot], 1u) != 0u) { record_error(err, 9u, pr.token); return; }
  tm_ids[slot] = pr.expert;
  tm_w16[slot] = static_cast<uint16_t>(pr.weight_bits & 0xFFFFu);
}

// ---- 2. counts + last-CTA scan ---------------------------------------------
// Exclusive scan of v over the block (thread order); returns the prefix and
// writes the block total to *total.
__device__ uint32_t block_excl_scan(uint32_t v, uint32_t* s_tmp, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) s_tmp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < nw ? s_tmp[lane] : 0u;
    uint32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xFFFFFFFFu, wi, o);
      if (lane >= o) wi += x;
    }
    if (lane < nw) s_tmp[lane] = wi - w;
    if (lane == nw - 1) s_tmp[32] = wi;
  }
  __syncthreads();
  const uint32_t r = s_tmp[warp] + incl - v;
  *total = s_tmp[32];
  __syncthreads();
  return r;
}

struct PermuteArgs {
  const uint32_t* tm_ids;  // [T*K] token-major expert ids
  int T, K, E, P;
  int tile_rows, tile_expert_count, tile_break, has_shared;
  const uint64_t* sort_keys;
};

// ---- 1. per-chunk histograms -------------------------------------------------
__global__ void __launch_bounds__(kThreads) permute_hist_kernel(PermuteArgs a, RouteBuffers rb) {
  extern __shared__ uint32_t s_h[];  // [E]
  const int c = blockIdx.x;
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) s_h[e] = 0u;
  __syncthreads();
  const int end = min(a.P, (c + 1) * kChunk);
  for (int i = c * kChunk + threadIdx.x; i < end; i += blockDim.x) {
    const uint32_t id = a.tm_ids[i];
    if (id < static_cast<uint32_t>(a.E)) atomicAdd(&s_h[id], 1u);
    else record_error(rb.err, 8u, id);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x)
    rb.hist[static_cast<size_t>(c) * a.E + e] = s_h[e];
}

// ---- 2. prefixes, counts, expert order, groups and schedules ----------------
// From the per-expert counts in s_dyn[0, E): the expert order, offsets,
// groups, tiles and row tiles.  s_dyn holds 3 E words.
TSG_DEV void order_and_schedule(const PermuteArgs& a, const RouteBuffers& rb, uint32_t* s_dyn,
                                   uint32_t* s_tmp) {
  uint32_t* s_cnt = s_dyn;
  const int E = a.E;
  uint32_t* s_order = s_dyn + E;    // [E] order position -> expert
  uint32_t* s_rank = s_dyn + 2 * E; // [E] expert -> order position
  // order experts by (sort key, index): rank = number of experts before it
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    uint32_t r = static_cast<uint32_t>(x);
    if (a.sort_keys) {
      const uint64_t kx = a.sort_keys[x];
      r = 0;
      for (int y = 0; y < E; ++y) {
        const uint64_t ky = a.sort_keys[y];
        r += (ky < kx || (ky == kx && y < x)) ? 1u : 0u;
      }
    }
    s_rank[x] = r;
    s_order[r] = static_cast<uint32_t>(x);
  }
  __syncthreads();
  // scan counts in order; groups are the non-empty experts in order
  uint32_t run = 0, grun = 0, trun = 0;
  const int ntl = a.tile_rows;
  for (int base = 0; base < E; base += blockDim.x) {
    const int r = base + threadIdx.x;
    const uint32_t ex = r < E ? s_order[r] : 0u;
    const uint32_t c = r < E ? s_cnt[ex] : 0u;
    uint32_t tot_c, tot_g, tot_t;
    const uint32_t off = run + block_excl_scan(c, s_tmp, &tot_c);
    const uint32_t gi = grun + block_excl_scan(c > 0u ? 1u : 0u, s_tmp, &tot_g);
    const uint32_t nrt = (c + ntl - 1) / ntl;
    const uint32_t ti = trun + block_excl_scan(nrt, s_tmp, &tot_t);
    if (r < E) {
      rb.offsets[ex] = c ? off : 0xFFFFFFFFu;
      if (c) {
        rb.groups[gi].expert = ex;
        rb.groups[gi].pair_start = off;
        rb.groups[gi].pair_count = c;
        for (uint32_t j = 0; j < nrt; ++j) {
          RowTile t;
          t.expert = ex;
          t.row_start = off + j * ntl;
          t.rows = min(static_cast<uint32_t>(ntl), c - j * ntl);
          t.pad = 0;
          rb.row_tiles[ti + j] = t;
        }
      }
    }
    run += tot_c;
    grun += tot_g;
    trun += tot_t;
  }
  __syncthreads();  // groups written by all threads are read below
  if (threadIdx.x == 0) {
    uint32_t nrt = trun;
    if (a.has_shared) {
      const uint32_t P = static_cast<uint32_t>(a.P);
      for (uint32_t j = 0; j * ntl < static_cast<uint32_t>(a.T); ++j) {
        RowTile t;
        t.expert = static_cast<uint32_t>(E);
        t.row_start = P + j * ntl;
        t.rows = min(static_cast<uint32_t>(ntl), static_cast<uint32_t>(a.T) - j * ntl);
        t.pad = 0;
        rb.row_tiles[nrt++] = t;
      }
    }
    *rb.n_row_tiles = nrt;
    *rb.n_groups = grun;
    // tiles of <= tile_expert_count groups, with the optional forced cut
    const int ng = static_cast<int>(grun);
    int nt = 0, gs = 0;
    while (gs < ng) {
      int ge = min(ng, gs + a.tile_expert_count);
      if (a.tile_break >= 0 && gs < a.tile_break && ge > a.tile_break) ge = a.tile_break;
      Tile t;
      t.group_start = static_cast<uint32_t>(gs);
      t.group_count = static_cast<uint32_t>(ge - gs);
      const Group g0 = rb.groups[gs];
      const Group g1 = rb.groups[ge - 1];
      t.pair_start = g0.pair_start;
      t.pair_count = g1.pair_start + g1.pair_count - g0.pair_start;
      rb.tiles[nt++] = t;
      gs = ge;
    }
    *rb.n_tiles = static_cast<uint32_t>(nt);
  }
}

__global__ void __launch_bounds__(kScanThreads) permute_scan_kernel(PermuteArgs a, RouteBuffers rb,
                                                                    int n_chunks) {
  __shared__ uint32_t s_tmp[33];
  extern __shared__ uint32_t s_dyn[];  // [3 * E]
  // each thread turns one expert's column of chunk counts into prefixes
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
    uint32_t run = 0;
    for (int c = 0; c < n_chunks; ++c) {
      uint32_t* h = rb.hist + static_cast<size_t>(c) * a.E + e;
      const uint32_t v = *h;
      *h = run;
      run += v;
    }
    s_dyn[e] = run;
    rb.counts[e] = run;
  }
  __syncthreads();
  order_and_schedule(a, rb, s_dyn, s_tmp);
}

// ---- 3. stable scatter -----------------------------------------------------
// Chunk c of NTHREADS-thread rounds; s_dyn holds (2 + NTHREADS / 32) E words.
// `chunk_prefix`: the chunk's per-expert prefixes in rb.hist (else zero).
template <int NTHREADS>
TSG_DEV void scatter_chunk(const PermuteArgs& a, const RouteBuffers& rb, const uint16_t* tm_w16,
                              const float* w_f32, int c, bool chunk_prefix, uint32_t* s_dyn) {
  const int E = a.E;
  uint32_t* s_base = s_dyn;          // [E] sorted position of this chunk's first pair of e
  uint32_t* s_run = s_dyn + E;       // [E] pairs of e already placed by this chunk
  uint32_t* s_wc = s_dyn + 2 * E;    // [NTHREADS / 32][E] per-warp counts of the sub-block
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = NTHREADS / 32;
  constexpr int kThreads = NTHREADS;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const uint32_t off = __ldcg(rb.offsets + e);
    // unused when e is empty
    s_base[e] = off + (chunk_prefix ? rb.hist[static_cast<size_t>(c) * E + e] : 0u);
    s_run[e] = 0u;
  }
  for (int x = threadIdx.x; x < kWarps * E; x += blockDim.x) s_wc[x] = 0u;
  __syncthreads();
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int end = min(a.P, (c + 1) * kChunk);
  for (int sb = c * kChunk; sb < end; sb += kThreads) {
    const int i = sb + static_cast<int>(threadIdx.x);
    const uint32_t raw = i < end ? a.tm_ids[i] : 0xFFFFFFFFu;
    const bool valid = raw < static_cast<uint32_t>(E);
    const uint32_t id = valid ? raw : 0xFFFFFFFFu;
    const uint32_t peers = __match_any_sync(0xFFFFFFFFu, id);
    const uint32_t lt = __popc(peers & lt_mask);
    const uint32_t cnt_w = __popc(peers);
    if (valid && lt == 0u) s_wc[warp * E + id] = cnt_w;
    __syncthreads();
    uint32_t rank = 0;
    bool last = false;
    if (valid) {
      uint32_t pre = 0, later = 0;
      for (int w = 0; w < kWarps; ++w) {
        const uint32_t v = s_wc[w * E + id];
        pre += w < warp ? v : 0u;
        later += w > warp ? v : 0u;
      }
      rank = s_run[id] + pre + lt;
      last = (lt == cnt_w - 1u) && later == 0u;
      const uint32_t pos = s_base[id] + rank;
      Pair pr;
      pr.token = static_cast<uint32_t>(i / a.K);
      pr.expert = id;
      pr.rank = static_cast<uint32_t>(i % a.K);
      pr.weight_bits = tm_w16 ? tm_w16[i] : __half_as_ushort(__float2half_rn(w_f32[i]));
      rb.sorted_pairs[pos] = pr;
      rb.pair_pos[i] = pos;
    }
    __syncthreads();
    if (last) s_run[id] = rank + 1u;
    if (valid && lt == 0u) s_wc[warp * E + id] = 0u;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kThreads) permute_scatter_kernel(PermuteArgs a, RouteBuffers rb,
                                                                  const uint16_t* tm_w16,
                                                                  const float* w_f32) {
  extern __shared__ uint32_t s_dyn[];
  scatter_chunk<kThreads>(a, rb, tm_w16, w_f32, static_cast<int>(blockIdx.x), true, s_dyn);
}

// All three steps in one CTA when the pairs fit one chunk (small batches):
// counts in shared memory, then the same ordering, schedules and scatter.
__global__ void __launch_bounds__(kScanThreads) permute_small_kernel(PermuteArgs a, RouteBuffers rb,
                                                                     const uint16_t* tm_w16,
                                                                     const float* w_f32) {
  __shared__ uint32_t s_tmp[33];
  extern __shared__ uint32_t s_dyn[];
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) s_dyn[e] = 0u;
  __syncthreads();
  for (int i = threadIdx.x; i < a.P; i += blockDim.x) {
    const uint32_t id = a.tm_ids[i];
    if (id < static_cast<uint32_t>(a.E)) atomicAdd(&s_dyn[id], 1u);
    else record_error(rb.err, 8u, id);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) rb.counts[e] = s_dyn[e];
  order_and_schedule(a, rb, s_dyn, s_tmp);
  __syncthreads();  // offsets (global, this CTA's writes) are read below
  scatter_chunk<kScanThreads>(a, rb, tm_w16, w_f32, 0, false, s_dyn);
}

__global__ void make_pairs_kernel(const uint32_t* ids, const uint16_t* w16, int T, int K,
                                  Pair* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * K) return;
  Pair p;
  p.token = static_cast<uint32_t>(i / K);
  p.expert = ids[i];
  p.rank = static_cast<uint32_t>(i % K);
  p.weight_bits = w16 ? w16[i] : 0u;
  out[i] = p;
}

// ---- gather: sorted rows of the normalised input, as fp16 ------------------
// Row i < n_rows takes token sorted_pairs[i].token; rows n_rows + t (when
// append_tokens) take token t in order (the shared expert's input).  One warp
// per row; also computes the raw shared-gate dot for the appended rows.
// With `frag_order` each 8 elements are stored as x0 x4 x2 x6 x1 x5 x3 x7,
// the mma.sync operand order of the batched GEMVs (int4_mma.cuh).
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* x, uint32_t x_stride,
                                                          const float* inv_rms,
                                                          const Pair* sorted_pairs, int n_rows,
                                                          int T, int D, int append_tokens,
                                                          __half* xp, const float* gate_w,
                                                          float* gate_raw, int frag_order) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int total = n_rows + (append_tokens ? T : 0);
  if (warp >= total) return;
  const int t = warp < n_rows ? static_cast<int>(sorted_pairs[warp].token) : warp - n_rows;
  if (t >= T) return;
  const float inv = inv_rms[t];
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * x_stride);
  uint4* dst = reinterpret_cast<uint4*>(xp + static_cast<size_t>(warp) * D);
  const bool do_gate = warp >= n_rows && gate_w != nullptr;
  float g = 0.0f;
  for (int c = lane; c < D / 8; c += 32) {
    const uint4 v = __ldg(src + c);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = __uint_as_float(wv[j] << 16);
      const float b = __uint_as_float(wv[j] & 0xFFFF0000u);
      if (do_gate) {
        g = fmaf(gate_w[c * 8 + 2 * j], a, g);
        g = fmaf(gate_w[c * 8 + 2 * j + 1], b, g);
      }
      __half2 h = __floats2half2_rn(a * inv, b * inv);
      o[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    const uint4 v8 = make_uint4(o[0], o[1], o[2], o[3]);
    dst[c] = frag_order ? frag_from_row(v8) : v8;
  }
  if (do_gate) {
    g = warp_sum(g);
    if (lane == 0) gate_raw[t] = g;
  }
}

// One CTA per owner rank, 1024 tokens per pass: a token is on owner o when
// one of its experts is; its slot is the count of such tokens before it.
__global__ void __launch_bounds__(1024) ep_owner_slots_kernel(const uint32_t* ids, int T, int K,
                                                              int El, uint32_t* slots,
                                                              uint32_t* counts) {
  __shared__ uint32_t warp_sum[32];
  __shared__ uint32_t carry;
  const uint32_t o = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < T; base += 1024) {
    const int t = base + static_cast<int>(threadIdx.x);
    bool on = false;
    if (t < T)
      for (int k = 0; k < K; ++k) on |= ids[static_cast<size_t>(t) * K + k] / static_cast<uint32_t>(El) == o;
    const uint32_t bal = __ballot_sync(0xffffffffu, on);
    if (lane == 0) warp_sum[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
      uint32_t v = warp_sum[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const uint32_t u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      warp_sum[lane] = v;  // inclusive
    }
    __syncthreads();
    const uint32_t before = carry + (warp ? warp_sum[warp - 1] : 0u) + __popc(bal & ((1u << lane) - 1u));
    if (t < T) slots[static_cast<size_t>(o) * T + t] = on ? before : kEpNoSlot;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sum[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[o] = carry;
}

// Threads write the pairs' map entries (grid-stride); warps write the rows,
// one per (owner, token).  Every index is checked against its buffer before
// the store.
__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __grid_constant__ EpDispatch d) {
  const uint32_t gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t nthr = gridDim.x * blockDim.x;
  const uint32_t El = static_cast<uint32_t>(d.experts_per_rank);
  const uint32_t R = static_cast<uint32_t>(d.world), T = static_cast<uint32_t>(d.T);
  for (uint32_t i = gtid; i < static_cast<uint32_t>(d.P); i += nthr) {
    const Pair pr = d.sorted_pairs[i];
    const uint32_t o = pr.expert / El;
    if (o >= R || pr.token >= T) {
      flag_error(d.err, TSG_DEVERR_BOUNDS);
      continue;
    }
    const uint32_t k = i - d.send_off[o];
    const uint32_t slot = d.slots[static_cast<size_t>(o) * T + pr.token];
    const uint32_t e = d.map0[o] + k;
    if (i < d.send_off[o] || k >= d.send_cnt[o] || slot >= d.n_rows[o] || e >= d.map_cap[o]) {
      flag_error(d.err, TSG_DEVERR_BOUNDS);
      continue;
    }
    d.map[o][e] = d.map_base[o] + slot;
  }
  const uint32_t w = gtid >> 5;
  const int lane = threadIdx.x & 31;
  if (w < R * T) {
    const uint32_t o = w / T, t = w % T;
    const uint32_t slot = d.slots[static_cast<size_t>(o) * T + t];
    if (slot != kEpNoSlot) {
      const uint32_t row = d.row0[o] + slot;
      if (slot >= d.n_rows[o] || row >= d.row_cap[o]) {
        if (lane == 0) flag_error(d.err, TSG_DEVERR_BOUNDS);
      } else {
        const float inv = d.inv_rms[t];
        const uint4* src = reinterpret_cast<const uint4*>(d.x + static_cast<size_t>(t) * d.x_stride);
        uint4* dst = reinterpret_cast<uint4*>(d.rows[o] + static_cast<size_t>(row) * d.D);
        for (int c = lane; c < d.D / 8; c += 32) {
          const uint4 v = __ldg(src + c);
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
          uint32_t h4[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float a = __uint_as_float(wv[j] << 16);
            const float b = __uint_as_float(wv[j] & 0xFFFF0000u);
            __half2 h = __floats2half2_rn(a * inv, b * inv);
            h4[j] = *reinterpret_cast<uint32_t*>(&h);
          }
          dst[c] = make_uint4(h4[0], h4[1], h4[2], h4[3]);
        }
      }
    }
  }
  // the stores reach the owners before this thread's later writes (the
  // owners read them after a collective that follows this kernel)
  __threadfence_system();
}

__global__ void __launch_bounds__(256) ep_expand_kernel(const __half* rows, uint32_t rows_cap,
                                                        const uint32_t* map, int n, int D,
                                                        __half* xp, uint32_t* err) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const uint32_t r = map[i];
  if (r >= rows_cap) {
    if (lane == 0) flag_error(err, TSG_DEVERR_BOUNDS);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(rows + static_cast<size_t>(r) * D);
  uint4* dst = reinterpret_cast<uint4*>(xp + static_cast<size_t>(i) * D);
  // eight 16-byte loads in flight per lane before their stores
  const int n16 = D / 8;
  for (int c0 = 0; c0 < n16; c0 += 256) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = c0 + 32 * k + lane;
      if (c < n16) v[k] = src[c];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = c0 + 32 * k + lane;
      if (c < n16) dst[c] = v[k];
    }
  }
}

}  // namespace

cudaError_t launch_ep_owner_slots(const uint32_t* ids, int T, int K, int experts_per_rank,
                                  int world, uint32_t* slots, uint32_t* counts, cudaStream_t s) {
  if (world < 1 || world > kEpMaxRanks || experts_per_rank < 1 || T < 0) return cudaErrorInvalidValue;
  ep_owner_slots_kernel<<<world, 1024, 0, s>>>(ids, T, K, experts_per_rank, slots, counts);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const EpDispatch& d, cudaStream_t s) {
  if (d.P <= 0 || d.T <= 0) return cudaSuccess;
  if (d.world < 1 || d.world > kEpMaxRanks || d.experts_per_rank < 1 || d.D % 8)
    return cudaErrorInvalidValue;
  const int warps_per_cta = 8;
  const int warps = d.world * d.T;
  ep_dispatch_kernel<<<(warps + warps_per_cta - 1) / warps_per_cta, 256, 0, s>>>(d);
  return cudaGetLastError();
}

cudaError_t launch_ep_expand(const __half* rows, uint32_t rows_cap, const uint32_t* map, int n,
                             int D, __half* xp, uint32_t* err, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (D % 8) return cudaErrorInvalidValue;
  const int warps_per_cta = 8;
  ep_expand_kernel<<<(n + warps_per_cta - 1) / warps_per_cta, 256, 0, s>>>(rows, rows_cap, map, n,
                                                                           D, xp, err);
  return cudaGetLastError();
}

int permute_chunks(int P) { return (P + kChunk - 1) / kChunk; }

// Places caller-supplied pairs into token-major order (validating them) when
// pairs_in is given; otherwise the router's ids/weights are already token
// major.  Then counts, scans and scatters.
cudaError_t launch_permute(const RouterParams& p, const RouteBuffers& rb, const Pair* pairs_in,
                           cudaStream_t s) {
  const int P = p.T * p.K;
  if (P <= 0) return cudaSuccess;
  const uint16_t* w16 = nullptr;
  const uint32_t* tm_ids = rb.ids;
  if (pairs_in) {
    // ids / weights_f16 / pair_pos double as token-major scratch
    uint32_t* occ = rb.pair_pos;
    cudaError_t e = cudaMemsetAsync(occ, 0, sizeof(uint32_t) * P, s);
    if (e != cudaSuccess) return e;
    place_pairs_kernel<<<(P + 255) / 256, 256, 0, s>>>(pairs_in, P, p.T, p.K, p.E, rb.ids,
                                                       rb.weights_f16, occ, rb.err);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    w16 = rb.weights_f16;
  }
  PermuteArgs a;
  a.tm_ids = tm_ids;
  a.T = p.T;
  a.K = p.K;
  a.E = p.E;
  a.P = P;
  a.tile_rows = p.tile_rows;
  a.tile_expert_count = p.tile_expert_count;
  a.tile_break = p.tile_break;
  a.has_shared = p.has_shared;
  a.sort_keys = p.sort_keys;
  const int n_chunks = permute_chunks(P);
  if (n_chunks == 1) {
    const size_t smem = (2u + kScanThreads / 32) * p.E * sizeof(uint32_t);
    if (smem > 48u * 1024u) {
      const cudaError_t e = allow_max_smem(permute_small_kernel);
      if (e != cudaSuccess) return e;
    }
    permute_small_kernel<<<1, kScanThreads, smem, s>>>(a, rb, w16, rb.weights);
    return cudaGetLastError();
  }
  permute_hist_kernel<<<n_chunks, kThreads, p.E * sizeof(uint32_t), s>>>(a, rb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  permute_scan_kernel<<<1, kScanThreads, 3u * p.E * sizeof(uint32_t), s>>>(a, rb, n_chunks);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem = (2u + kThreads / 32) * p.E * sizeof(uint32_t);
  permute_scatter_kernel<<<n_chunks, kThreads, smem, s>>>(a, rb, w16, rb.weights);
  return cudaGetLastError();
}

cudaError_t launch_make_pairs(const uint32_t* ids, const uint16_t* w_f16, int T, int K, Pair* out,
                              cudaStream_t s) {
  const int n = T * K;
  if (n <= 0) return cudaSuccess;
  make_pairs_kernel<<<(n + 255) / 256, 256, 0, s>>>(ids, w_f16, T, K, out);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows_gate(const uint16_t* x, uint32_t x_stride, const float* inv_rms,
                                    const Pair* sorted_pairs, int n_rows, int T, int D,
                                    int append_tokens, __half* xp, const float* gate_w,
                                    float* gate_raw, cudaStream_t s, int frag_order) {
  const int total = n_rows + (append_tokens ? T : 0);
  if (total <= 0) return cudaSuccess;
  const int warps_per_cta = 8;
  gather_rows_kernel<<<(total + warps_per_cta - 1) / warps_per_cta, 256, 0, s>>>(
      x, x_stride, inv_rms, sorted_pairs, n_rows, T, D, append_tokens, xp, gate_w, gate_raw,
      frag_order);
  return cudaGetLastError();
}


}  // namespace tsg
