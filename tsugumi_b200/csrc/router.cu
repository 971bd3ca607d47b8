// router.cu -- router logits, top-K gating and (for decode-sized T) the
// token->expert grouping, all on the GPU.
//
// Semantics follow the reference's router:
//   * input norm: rmsnorm_no_scale (Metal/Primitives/rmsnorm.metal:154-175),
//     applied as a per-row factor inv_rms[t] on the raw dot products;
//   * logits: router_gemv_gemma4_bf16_body (Metal/MoE/moe.metal:187-213) with
//     the effective scale folded into the fp32 router rows once per layer;
//   * top-K: router_topk_select_k8_body (moe.metal:281-329) and
//     prefill_router_emit_topk (Metal/Prefill/prefill.metal:555-606): a score
//     beats another when strictly greater, or equal with a lower expert index;
//     weights are the softmax over the K selected scores times the
//     per-expert scale.
// The skewed benchmark configurations add a per-expert logit bias.
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kDecodeRowsPerCta = 8;  // one warp per router row
constexpr int kDecodeTokChunk = 8;    // tokens staged per pass
constexpr int kMaxK = 32;
constexpr int kMaxSplitParts = 8;  // split-K partials of the prefill router GEMMs

// Select the top K of `v` (lane holds v[lane + 32 j], j < per_lane) with the
// reference's tie rule.  Lane 0 ends with ids[0..K) and scores[0..K).
template <int PER_LANE>
__device__ void warp_topk(float (&v)[PER_LANE], int E, int K, uint32_t* ids_out,
                          float* score_out) {
  const int lane = threadIdx.x & 31;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bidx = 0x7FFFFFFF;
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j) {
      const int e = lane + 32 * j;
      if (e < E && (v[j] > best || (v[j] == best && e < bidx))) {
        best = v[j];
        bidx = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bidx, o);
      if (ob > best || (ob == best && oi < bidx)) {
        best = ob;
        bidx = oi;
      }
    }
    if (lane == 0) {
      ids_out[k] = static_cast<uint32_t>(bidx);
      score_out[k] = best;
    }
    // remove the winner: a NaN never compares greater or equal, so it can
    // not be selected again even when every remaining score is -inf
#pragma unroll
    for (int j = 0; j < PER_LANE; ++j)
      if (lane + 32 * j == bidx) v[j] = __int_as_float(0x7FC00000u);
  }
}

// Softmax over the K selected scores times the per-expert scale, by lane 0.
__device__ void emit_weights(const uint32_t* ids, const float* scores, int K,
                             const float* per_expert_scale, float* w_out, uint16_t* w16_out) {
  float ex[kMaxK];
  float sum = 0.0f;
  const float mx = scores[0];
  for (int k = 0; k < K; ++k) {
    ex[k] = expf(scores[k] - mx);
    sum += ex[k];
  }
  for (int k = 0; k < K; ++k) {
    const float gain = per_expert_scale ? per_expert_scale[ids[k]] : 1.0f;
    const float w = ex[k] / sum * gain;
    w_out[k] = w;
    if (w16_out) w16_out[k] = __half_as_ushort(__float2half_rn(w));
  }
}

// Top-K for one token by one warp, from raw logits and the row's norm factor.
template <int PER_LANE>
__device__ void token_topk(const float* raw, int nsplit, size_t split_stride, float inv,
                           const RouterParams& p, uint32_t* ids_out, float* w_out,
                           uint16_t* w16_out) {
  const int lane = threadIdx.x & 31;
  float v[PER_LANE];
#pragma unroll
  for (int j = 0; j < PER_LANE; ++j) {
    const int e = lane + 32 * j;
    float s = 0.0f;
    if (e < p.E) {
      float part[kMaxSplitParts];
#pragma unroll
      for (int sp = 0; sp < kMaxSplitParts; ++sp)  // loads issued together
        part[sp] = sp < nsplit ? __ldcg(raw + sp * split_stride + e) : 0.0f;
#pragma unroll
      for (int sp = 0; sp < kMaxSplitParts; ++sp) s += part[sp];
      s *= inv;
      if (p.logit_bias) s += p.logit_bias[e];
    } else {
      s = -INFINITY;
    }
    v[j] = s;
  }
  __shared__ uint32_t s_ids[kDecodeRowsPerCta][kMaxK];
  __shared__ float s_sc[kDecodeRowsPerCta][kMaxK];
  const int w = (threadIdx.x >> 5) & (kDecodeRowsPerCta - 1);
  warp_topk<PER_LANE>(v, p.E, p.K, s_ids[w], s_sc[w]);
  __syncwarp();
  if (lane == 0) {
    emit_weights(s_ids[w], s_sc[w], p.K, p.per_expert_scale, w_out, w16_out);
    for (int k = 0; k < p.K; ++k) ids_out[k] = s_ids[w][k];
  }
  __syncwarp();
}

__device__ void dispatch_token_topk(const float* raw, int nsplit, size_t split_stride, float inv,
                                    const RouterParams& p, uint32_t* ids_out, float* w_out,
                                    uint16_t* w16_out) {
  if (p.E <= 32) token_topk<1>(raw, nsplit, split_stride, inv, p, ids_out, w_out, w16_out);
  else if (p.E <= 64) token_topk<2>(raw, nsplit, split_stride, inv, p, ids_out, w_out, w16_out);
  else if (p.E <= 128) token_topk<4>(raw, nsplit, split_stride, inv, p, ids_out, w_out, w16_out);
  else if (p.E <= 256) token_topk<8>(raw, nsplit, split_stride, inv, p, ids_out, w_out, w16_out);
  else token_topk<16>(raw, nsplit, split_stride, inv, p, ids_out, w_out, w16_out);
}

// ---------------------------------------------------------------------------
// Block-level stable grouping for up to a few thousand pairs: counts,
// ascending-expert offsets, and the stable scatter that orders pairs by
// (expert, token, rank) -- PrefillMoEGrouping.groupTokenExpertPairs
// (Kernels/Prefill/MoE/PrefillMoEGrouping.swift:141-193).  Runs in one CTA of
// 256 threads; scratch arrays live in shared memory.
// ---------------------------------------------------------------------------
__device__ void block_group_pairs(const uint32_t* ids, const float* weights, int T, int K, int E,
                                  const RouteBuffers& rb, uint32_t* s_cnt, uint32_t* s_run) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int P = T * K;
  for (int e = tid; e < E; e += nthr) s_cnt[e] = 0u;
  __syncthreads();
  for (int i = tid; i < P; i += nthr) {
    const uint32_t e = ids[i];
    if (e < static_cast<uint32_t>(E)) atomicAdd(&s_cnt[e], 1u);
    else flag_error(rb.err, TSG_DEVERR_METADATA);
  }
  __syncthreads();
  // exclusive scan over experts by warp 0 (lane owns a contiguous span)
  if (tid < 32) {
    const int per = (E + 31) / 32;
    const int lo = tid * per, hi = min(E, lo + per);
    uint32_t local = 0;
    for (int e = lo; e < hi; ++e) local += s_cnt[e];
    uint32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (tid >= o) incl += n;
    }
    uint32_t run = incl - local;
    for (int e = lo; e < hi; ++e) {
      s_run[e] = run;
      run += s_cnt[e];
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += nthr) {
    rb.counts[e] = s_cnt[e];
    rb.offsets[e] = s_cnt[e] ? s_run[e] : 0xFFFFFFFFu;
  }
  // groups: compact non-empty experts in ascending order (warp 0)
  if (tid < 32) {
    uint32_t base = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + tid;
      const bool ne = e < E && s_cnt[e] > 0u;
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, ne);
      if (ne) {
        const uint32_t g = base + __popc(m & ((1u << tid) - 1u));
        rb.groups[g].expert = static_cast<uint32_t>(e);
        rb.groups[g].pair_start = s_run[e];
        rb.groups[g].pair_count = s_cnt[e];
      }
      base += __popc(m);
    }
    if (tid == 0) *rb.n_groups = base;
  }
  __syncthreads();
  // stable scatter: rounds of blockDim pairs, warps take turns
  const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
  for (int base = 0; base < P; base += nthr) {
    const int i = base + tid;
    const uint32_t e = i < P ? ids[i] : 0xFFFFFFFFu;
    const bool valid = i < P && e < static_cast<uint32_t>(E);
    const uint32_t key = valid ? e : 0xFFFFFFFEu;
    const uint32_t peers = __match_any_sync(0xFFFFFFFFu, key);
    const uint32_t rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    const bool leader = rank_in_warp == 0;
    for (int w = 0; w < nwarps; ++w) {
      if (warp == w && valid) {
        const uint32_t pos = s_run[e] + rank_in_warp;
        __syncwarp(peers);
        if (leader) s_run[e] += __popc(peers);
        Pair pr;
        pr.token = static_cast<uint32_t>(i / K);
        pr.expert = e;
        pr.rank = static_cast<uint32_t>(i % K);
        pr.weight_bits = __half_as_ushort(__float2half_rn(weights[i]));
        rb.sorted_pairs[pos] = pr;
        rb.pair_pos[i] = pos;
      }
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Decode router: one warp per router row, the last CTA to finish selects the
// top K for every token and groups the pairs.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) router_decode_kernel(RouterParams p, RouteBuffers rb) {
  extern __shared__ float4 smem_f4[];
  float* xs = reinterpret_cast<float*>(smem_f4);  // [kDecodeTokChunk][D]
  __shared__ float s_red[kDecodeTokChunk][8];
  __shared__ uint32_t s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rows = p.E + p.has_gate;
  const int row = blockIdx.x * kDecodeRowsPerCta + warp;
  const int D = p.D;

  for (int t0 = 0; t0 < p.T; t0 += kDecodeTokChunk) {
    const int nt = min(kDecodeTokChunk, p.T - t0);
    __syncthreads();
    float ss[kDecodeTokChunk];
#pragma unroll
    for (int t = 0; t < kDecodeTokChunk; ++t) ss[t] = 0.0f;
    for (int t = 0; t < nt; ++t) {
      const uint16_t* xr = p.x + static_cast<size_t>(t0 + t) * p.x_stride;
      for (int i = tid; i < D; i += blockDim.x) {
        const float v = bf16_bits_to_f32(xr[i]);
        xs[t * D + i] = v;
        ss[t] += v * v;
      }
    }
    if (blockIdx.x == 0) {
#pragma unroll
      for (int t = 0; t < kDecodeTokChunk; ++t) {
        const float v = warp_sum(ss[t]);
        if (lane == 0) s_red[t][warp] = v;
      }
    }
    __syncthreads();
    if (blockIdx.x == 0) {
      // CTA 0 publishes the norm factor, the normalised rows and the
      // per-8-element sums (x 1.5) the expert kernels stage with the codes
      for (int t = 0; t < nt; ++t) {
        float v = 0.0f;
        for (int w = 0; w < 8; ++w) v += s_red[t][w];
        const float inv = p.norm ? rsqrtf(v / static_cast<float>(D) + p.eps) : 1.0f;
        if (tid == 0) {
          rb.sumsq[t0 + t] = v;
          rb.inv_rms[t0 + t] = inv;
        }
        float* xn = rb.xn + static_cast<size_t>(t0 + t) * D;
        for (int i = tid; i < D; i += blockDim.x) xn[i] = xs[t * D + i] * inv;
        for (int w8 = tid; w8 < D / 8; w8 += blockDim.x) {
          float sum = 0.0f;
#pragma unroll
          for (int q = 0; q < 8; ++q) sum += xs[t * D + w8 * 8 + q] * inv;
          rb.xs8[static_cast<size_t>(t0 + t) * (D / 8) + w8] = 1.5f * sum;
        }
      }
    }
    if (row < rows) {
      const float* wr = p.w + static_cast<size_t>(row) * D;
      float acc[kDecodeTokChunk];
#pragma unroll
      for (int t = 0; t < kDecodeTokChunk; ++t) acc[t] = 0.0f;
      for (int i = lane * 4; i < D; i += 128) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(wr + i));
#pragma unroll
        for (int t = 0; t < kDecodeTokChunk; ++t) {
          if (t < nt) {
            const float4 xv = *reinterpret_cast<const float4*>(xs + t * D + i);
            acc[t] = fmaf(wv.x, xv.x, acc[t]);
            acc[t] = fmaf(wv.y, xv.y, acc[t]);
            acc[t] = fmaf(wv.z, xv.z, acc[t]);
            acc[t] = fmaf(wv.w, xv.w, acc[t]);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kDecodeTokChunk; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0 && t < nt) {
          if (row < p.E) rb.logits_raw[static_cast<size_t>(t0 + t) * p.E + row] = v;
          else rb.gate_raw[t0 + t] = v;
        }
      }
    }
  }

  // last CTA to arrive performs the selection and grouping
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t ticket = atomicAdd(rb.sync_counter, 1u);
    s_last = (ticket == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid == 0) *rb.sync_counter = 0u;  // ready for the next launch / graph replay

  for (int t = warp; t < p.T; t += blockDim.x / 32) {
    const float inv = __ldcg(rb.inv_rms + t);
    dispatch_token_topk(rb.logits_raw + static_cast<size_t>(t) * p.E, 1, 0, inv, p,
                        rb.ids + static_cast<size_t>(t) * p.K,
                        rb.weights + static_cast<size_t>(t) * p.K,
                        rb.weights_f16 ? rb.weights_f16 + static_cast<size_t>(t) * p.K : nullptr);
  }
  __threadfence_block();
  __syncthreads();
  uint32_t* s_cnt = reinterpret_cast<uint32_t*>(smem_f4);
  uint32_t* s_run = s_cnt + p.E;
  block_group_pairs(rb.ids, rb.weights, p.T, p.K, p.E, rb, s_cnt, s_run);
}

// ---------------------------------------------------------------------------
// Prefill router: split-K fp32 SIMT GEMM, 128 tokens x 128 router rows per
// CTA, 8x8 outputs per thread; partial dots go to logits_raw[split][T][E].
// ---------------------------------------------------------------------------
constexpr int kGBM = 128, kGBN = 128, kGBK = 16;

__global__ void __launch_bounds__(256) router_gemm_kernel(RouterParams p, RouteBuffers rb,
                                                          int ksplit) {
  __shared__ __align__(16) float As[2][kGBK][kGBM];
  __shared__ __align__(16) float Bs[2][kGBK][kGBN];
  __shared__ float s_ss[kGBM];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.x * kGBM;
  const int n0 = blockIdx.y * kGBN;
  const int split = blockIdx.z;
  const int D = p.D;
  const int kper = (D / ksplit + kGBK - 1) / kGBK * kGBK;
  const int kbeg = split * kper;
  const int kend = min(D, kbeg + kper);
  const int TT = p.T, NN = p.E;

  // loaders: each thread moves 8 A elements and 8 B elements per k-tile
  const int lrow = tid >> 1;        // 0..127
  const int lk = (tid & 1) * 8;     // 0 or 8
  float ra[8], rbv[8];
  float ssq = 0.0f;
  auto load_tile = [&](int k0) {
    const int gm = m0 + lrow, gn = n0 + lrow;
    const int kb = k0 + lk;
    if (gm < TT && kb + 8 <= kend) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(gm) * p.x_stride + kb));
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ra[2 * j] = __uint_as_float(wv[j] << 16);
        ra[2 * j + 1] = __uint_as_float(wv[j] & 0xFFFF0000u);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = kb + j;
        ra[j] = (gm < TT && k < kend)
                    ? bf16_bits_to_f32(p.x[static_cast<size_t>(gm) * p.x_stride + k])
                    : 0.0f;
      }
    }
    if (gn < NN && kb + 8 <= kend) {
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(p.w + static_cast<size_t>(gn) * D + kb));
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(p.w + static_cast<size_t>(gn) * D + kb + 4));
      rbv[0] = w0.x; rbv[1] = w0.y; rbv[2] = w0.z; rbv[3] = w0.w;
      rbv[4] = w1.x; rbv[5] = w1.y; rbv[6] = w1.z; rbv[7] = w1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = kb + j;
        rbv[j] = (gn < NN && k < kend) ? __ldg(p.w + static_cast<size_t>(gn) * D + k) : 0.0f;
      }
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      As[buf][lk + j][lrow] = ra[j];
      Bs[buf][lk + j][lrow] = rbv[j];
      ssq += ra[j] * ra[j];
    }
  };

  const int tx = tid & 15, ty = tid >> 4;  // 16 x 16 threads, 8 x 8 each
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  int buf = 0;
  if (kbeg < kend) {
    load_tile(kbeg);
    store_tile(0);
  }
  __syncthreads();
  for (int k0 = kbeg; k0 < kend; k0 += kGBK) {
    const bool more = k0 + kGBK < kend;
    if (more) load_tile(k0 + kGBK);
#pragma unroll
    for (int kk = 0; kk < kGBK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) store_tile(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }
  // row sums of squares: only the first column tile contributes
  if (blockIdx.y == 0) {
    // the two loaders of a row are adjacent lanes: combine in fixed order
    const float other = __shfl_xor_sync(0xFFFFFFFFu, ssq, 1);
    if ((tid & 1) == 0) s_ss[lrow] = ssq + other;
    __syncthreads();
    if (tid < kGBM && m0 + tid < TT)
      rb.sumsq[static_cast<size_t>(split) * TT + m0 + tid] = s_ss[tid];
  }
  float* out = rb.logits_raw + static_cast<size_t>(split) * TT * NN;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= TT) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn < NN) out[static_cast<size_t>(gm) * NN + gn] = acc[i][j];
    }
  }
}

// ---------------------------------------------------------------------------
// Prefill router for small batches (T <= 64): one warp per router row and
// split of D (chunks of 256 columns, 8 per lane); tokens in passes of 16
// accumulated in registers, then reduced across lanes by halving exchanges
// (16 values to one per lane pair in 16 shuffles).  The weight rows stream
// once from HBM; the token rows come from L1.  CTA column 0, warp 0 also
// writes the split's row sums of squares.  Same outputs as router_gemm.
// ---------------------------------------------------------------------------
constexpr int kSmallRows = 4;     // router rows (warps) per CTA
constexpr int kSmallChunk = 256;  // columns per lane pass (8 per lane)
constexpr int kSmallPass = 16;    // tokens per pass

// v[16] per lane -> lanes 2j and 2j + 1 hold the warp-wide sum of v[j].
TSG_DEV float reduce16(float (&v)[kSmallPass]) {
  const int lane = threadIdx.x & 31;
  float u[8];
  const bool b4 = lane & 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = b4 ? v[i] : v[i + 8];
    const float keep = b4 ? v[i + 8] : v[i];
    u[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 16);
  }
  const bool b3 = lane & 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b3 ? u[i] : u[i + 4];
    const float keep = b3 ? u[i + 4] : u[i];
    u[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 8);
  }
  const bool b2 = lane & 4;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b2 ? u[i] : u[i + 2];
    const float keep = b2 ? u[i + 2] : u[i];
    u[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 4);
  }
  const bool b1 = lane & 2;
  {
    const float send = b1 ? u[0] : u[1];
    const float keep = b1 ? u[1] : u[0];
    u[0] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, 2);
  }
  return u[0] + __shfl_xor_sync(0xFFFFFFFFu, u[0], 1);
}

__global__ void __launch_bounds__(kSmallRows * 32) router_small_kernel(RouterParams p,
                                                                        RouteBuffers rb,
                                                                        int chunks_per_split) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = blockIdx.x * kSmallRows + warp;
  const int split = blockIdx.y;
  const int k0 = split * chunks_per_split * kSmallChunk;
  const int k1 = min(p.D, k0 + chunks_per_split * kSmallChunk);
  const bool row_ok = e < p.E;
  const bool ss_warp = blockIdx.x == 0 && warp == 0;
  const float* wr = p.w + static_cast<size_t>(row_ok ? e : 0) * p.D;
  const int j = lane >> 1;  // the token slot this lane pair ends with
  for (int t0 = 0; t0 < p.T; t0 += kSmallPass) {
    float acc[kSmallPass], ss[kSmallPass];
#pragma unroll
    for (int t = 0; t < kSmallPass; ++t) acc[t] = ss[t] = 0.0f;
    for (int k = k0 + lane * 8; k < k1; k += kSmallChunk) {
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(wr + k));
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(wr + k + 4));
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      // every token load of the pass in flight before the first FMA
      uint4 xv[kSmallPass];
#pragma unroll
      for (int t = 0; t < kSmallPass; ++t)
        xv[t] = t0 + t < p.T ? __ldg(reinterpret_cast<const uint4*>(
                                   p.x + static_cast<size_t>(t0 + t) * p.x_stride + k))
                             : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int t = 0; t < kSmallPass; ++t) {
        {
          const uint32_t xw[4] = {xv[t].x, xv[t].y, xv[t].z, xv[t].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float lo = __uint_as_float(xw[q] << 16);
            const float hi = __uint_as_float(xw[q] & 0xFFFF0000u);
            acc[t] = fmaf(wv[2 * q], lo, acc[t]);
            acc[t] = fmaf(wv[2 * q + 1], hi, acc[t]);
            if (ss_warp) {
              ss[t] = fmaf(lo, lo, ss[t]);
              ss[t] = fmaf(hi, hi, ss[t]);
            }
          }
        }
      }
    }
    const float dot = reduce16(acc);
    if ((lane & 1) == 0 && t0 + j < p.T && row_ok)
      rb.logits_raw[(static_cast<size_t>(split) * p.T + t0 + j) * p.E + e] = dot;
    if (ss_warp) {
      const float sq = reduce16(ss);
      if ((lane & 1) == 0 && t0 + j < p.T)
        rb.sumsq[static_cast<size_t>(split) * p.T + t0 + j] = sq;
    }
  }
}

// Warp per token: combine the splits, apply the norm factor and bias, select.
// With ss_from_x the row's sum of squares is taken from its bf16 input (the
// tensor-core GEMM produces only the dots), else from the split partials.
__global__ void __launch_bounds__(256) router_topk_kernel(RouterParams p, RouteBuffers rb,
                                                          int ksplit, int ss_from_x) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.T) return;
  const int t = warp;
  float ssq = 0.0f;
  if (ss_from_x) {
    const uint16_t* xr = p.x + static_cast<size_t>(t) * p.x_stride;
    for (int i = lane; i < p.D; i += 32) {
      const float v = bf16_bits_to_f32(xr[i]);
      ssq = fmaf(v, v, ssq);
    }
    ssq = warp_sum(ssq);
  } else {
    float part[kMaxSplitParts];
#pragma unroll
    for (int s = 0; s < kMaxSplitParts; ++s)  // loads issued together
      part[s] = s < ksplit ? __ldcg(rb.sumsq + static_cast<size_t>(s) * p.T + t) : 0.0f;
#pragma unroll
    for (int s = 0; s < kMaxSplitParts; ++s) ssq += part[s];
  }
  const float inv = p.norm ? rsqrtf(ssq / static_cast<float>(p.D) + p.eps) : 1.0f;
  if (lane == 0) rb.inv_rms[t] = inv;
  dispatch_token_topk(rb.logits_raw + static_cast<size_t>(t) * p.E, ksplit,
                      static_cast<size_t>(p.T) * p.E, inv, p, rb.ids + static_cast<size_t>(t) * p.K,
                      rb.weights + static_cast<size_t>(t) * p.K,
                      rb.weights_f16 ? rb.weights_f16 + static_cast<size_t>(t) * p.K : nullptr);
}

// Logits only (no selection): warp per token, the same split sum, norm factor
// and bias as router_topk_kernel, written as fp32 [T][E].
__global__ void __launch_bounds__(256) router_logits_kernel(RouterParams p, RouteBuffers rb,
                                                            int ksplit, int ss_from_x,
                                                            float* out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.T) return;
  const int t = warp;
  float ssq = 0.0f;
  if (ss_from_x) {
    const uint16_t* xr = p.x + static_cast<size_t>(t) * p.x_stride;
    for (int i = lane; i < p.D; i += 32) {
      const float v = bf16_bits_to_f32(xr[i]);
      ssq = fmaf(v, v, ssq);
    }
    ssq = warp_sum(ssq);
  } else {
    for (int s = 0; s < ksplit; ++s) ssq += __ldcg(rb.sumsq + static_cast<size_t>(s) * p.T + t);
  }
  const float inv = p.norm ? rsqrtf(ssq / static_cast<float>(p.D) + p.eps) : 1.0f;
  const float* raw = rb.logits_raw + static_cast<size_t>(t) * p.E;
  const size_t split_stride = static_cast<size_t>(p.T) * p.E;
  for (int e = lane; e < p.E; e += 32) {
    float part[kMaxSplitParts];
#pragma unroll
    for (int sp = 0; sp < kMaxSplitParts; ++sp)  // the order of router_topk_kernel's sum
      part[sp] = sp < ksplit ? __ldcg(raw + sp * split_stride + e) : 0.0f;
    float sum = 0.0f;
#pragma unroll
    for (int sp = 0; sp < kMaxSplitParts; ++sp) sum += part[sp];
    sum *= inv;
    if (p.logit_bias) sum += p.logit_bias[e];
    out[static_cast<size_t>(t) * p.E + e] = sum;
  }
}

// Per-row statistics for caller-supplied routing: inv_rms, and for the
// decode regime the normalised rows xn and 1.5 x their 8-element sums; the
// raw shared-gate dot when the layer has a gate.  One CTA per token.
__global__ void __launch_bounds__(256) rowprep_kernel(RouterParams p, RouteBuffers rb,
                                                      int write_rows) {
  __shared__ float s_red[8];
  __shared__ float s_inv;
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = p.D;
  const uint16_t* xr = p.x + static_cast<size_t>(t) * p.x_stride;
  float ss = 0.0f, g = 0.0f;
  const float* gw = p.has_gate ? p.w + static_cast<size_t>(p.E) * D : nullptr;
  for (int i = tid; i < D; i += blockDim.x) {
    const float v = bf16_bits_to_f32(xr[i]);
    ss += v * v;
    if (gw) g = fmaf(gw[i], v, g);
  }
  ss = warp_sum(ss);
  if (lane == 0) s_red[warp] = ss;
  __syncthreads();
  if (tid == 0) {
    float v = 0.0f;
    for (int w = 0; w < 8; ++w) v += s_red[w];
    const float inv = p.norm ? rsqrtf(v / static_cast<float>(D) + p.eps) : 1.0f;
    rb.inv_rms[t] = inv;
    s_inv = inv;
  }
  __syncthreads();
  if (gw) {
    g = warp_sum(g);
    if (lane == 0) s_red[warp] = g;
    __syncthreads();
    if (tid == 0) {
      float v = 0.0f;
      for (int w = 0; w < 8; ++w) v += s_red[w];
      rb.gate_raw[t] = v;
    }
  }
  if (!write_rows) return;
  const float inv = s_inv;
  float* xn = rb.xn + static_cast<size_t>(t) * D;
  for (int i = tid; i < D; i += blockDim.x) xn[i] = bf16_bits_to_f32(xr[i]) * inv;
  for (int w8 = tid; w8 < D / 8; w8 += blockDim.x) {
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < 8; ++q) sum += bf16_bits_to_f32(xr[w8 * 8 + q]) * inv;
    rb.xs8[static_cast<size_t>(t) * (D / 8) + w8] = 1.5f * sum;
  }
}

// Stable grouping of caller-supplied routing in one CTA (decode sizes).
__global__ void __launch_bounds__(256) group_small_kernel(RouterParams p, RouteBuffers rb) {
  extern __shared__ uint32_t s_grp[];
  block_group_pairs(rb.ids, rb.weights, p.T, p.K, p.E, rb, s_grp, s_grp + p.E);
}

}  // namespace

cudaError_t launch_router_decode(const RouterParams& p, const RouteBuffers& rb, cudaStream_t s) {
  if (p.K > kMaxK || p.E > 512) return cudaErrorInvalidValue;
  const int rows = p.E + p.has_gate;
  const int grid = (rows + kDecodeRowsPerCta - 1) / kDecodeRowsPerCta;
  size_t smem = static_cast<size_t>(kDecodeTokChunk) * p.D * sizeof(float);
  const size_t need_group = 2u * p.E * sizeof(uint32_t);
  if (smem < need_group) smem = need_group;
  cudaError_t e = allow_max_smem(router_decode_kernel);
  if (e != cudaSuccess) return e;
  router_decode_kernel<<<grid, 256, smem, s>>>(p, rb);
  return cudaGetLastError();
}

namespace {
bool router_small_usable(const RouterParams& p) {
  return p.T <= 64 && p.D % kSmallChunk == 0 && p.x_stride % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(p.w) & 15u) == 0;
}
// Splits of whole 256-column chunks, at most kMaxSplitParts, enough for
// about two CTAs per SM.
int router_small_ksplit(int E, int D, int* chunks_per_split) {
  const int nchunk = D / kSmallChunk;
  const int row_ctas = (E + kSmallRows - 1) / kSmallRows;
  int want = (296 + row_ctas - 1) / row_ctas;
  want = want < 1 ? 1 : (want > kMaxSplitParts ? kMaxSplitParts : want);
  if (want > nchunk) want = nchunk;
  const int cps = (nchunk + want - 1) / want;
  *chunks_per_split = cps;
  return (nchunk + cps - 1) / cps;
}
}  // namespace

cudaError_t launch_router_prefill(const RouterParams& p, const RouteBuffers& rb, cudaStream_t s,
                                  float* logits_out) {
  if (p.K > kMaxK || p.E > 512) return cudaErrorInvalidValue;
  const int mt = (p.T + kGBM - 1) / kGBM;
  const int nt = (p.E + kGBN - 1) / kGBN;
  int ksplit = 1;
  int from_x = 0;
  cudaError_t e;
  if (router_tc_usable(p)) {
    ksplit = router_tc_ksplit(p.T, p.E, p.D);
    from_x = 1;
    e = launch_router_tc(p, rb, ksplit, s);
  } else if (router_small_usable(p)) {
    int cps = 1;
    ksplit = router_small_ksplit(p.E, p.D, &cps);
    dim3 grid((p.E + kSmallRows - 1) / kSmallRows, ksplit);
    router_small_kernel<<<grid, kSmallRows * 32, 0, s>>>(p, rb, cps);
    e = cudaGetLastError();
  } else {
    while (mt * nt * ksplit < 148 && ksplit < 8 && p.D / (ksplit * 2) >= 256) ksplit *= 2;
    dim3 grid(mt, nt, ksplit);
    router_gemm_kernel<<<grid, 256, 0, s>>>(p, rb, ksplit);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  const int warps_per_cta = 8;
  const int grid = (p.T + warps_per_cta - 1) / warps_per_cta;
  if (logits_out)
    router_logits_kernel<<<grid, 256, 0, s>>>(p, rb, ksplit, from_x, logits_out);
  else
    router_topk_kernel<<<grid, 256, 0, s>>>(p, rb, ksplit, from_x);
  return cudaGetLastError();
}


}  // namespace tsg

namespace tsg {
cudaError_t launch_rowprep(const RouterParams& p, const RouteBuffers& rb, int write_rows,
                           cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  rowprep_kernel<<<p.T, 256, 0, s>>>(p, rb, write_rows);
  return cudaGetLastError();
}
cudaError_t launch_group_small(const RouterParams& p, const RouteBuffers& rb, cudaStream_t s) {
  if (p.T <= 0) return cudaSuccess;
  group_small_kernel<<<1, 256, 2u * p.E * sizeof(uint32_t), s>>>(p, rb);
  return cudaGetLastError();
}
}  // namespace tsg
