// decode.cu -- the decode-regime (T <= 64) expert products as batched GEMVs.
//
// Reference behaviour: moe_phase1_gate_up_act_u16load and
// moe_phase2_down_reduce_k8 (Sources/Tsugumi/Metal/MoE/moe.metal:455-574,
// :651-687) with MoE.encodeRoutedPersistentPhase1U16Load / Phase2Reduce
// (Sources/Tsugumi/Kernels/MoE/MoE.swift:529-644): per routed slot and row,
// gate and up int4 dot products over shared activation loads,
// act = act_fn(g) * u; then per output row d, y = residual + sum over slots
// of w * (down . act).  The reference folds one slot per simdgroup; here:
//
//   gate/up kernel  persistent CTAs walk (expert, 8-row chunk) items; each
//                   item's int4 codes, fp16 scales and the expert's token rows
//                   arrive in shared memory through bulk copies (mbarrier
//                   pipeline, 4 stages); one warp per row, lanes over 8-element
//                   code words, codes decoded in registers; warp-shuffle
//                   reduction; act written as fp16 in sorted-pair order.
//   down kernel     one CTA per block of output rows; walks every active
//                   expert (bulk-copied rows + act), keeps each pair's value in
//                   shared memory, then writes y[t, d] = shared-branch +
//                   sum over ranks r (ascending) of w[t, r] * v[t, r, d].
//
// The int4 dot uses floats f = 1 + q/16 assembled by byte permutes (see
// nibbles_to_f32_plus1): sum((q - 8) x) = 16 (sum(f x) - 1.5 sum(x)).
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kRows = 8;      // gate/up rows per item (one warp each)
constexpr int kStages = 4;

struct ExpertRef {
  const uint8_t* blob;
  const ExpertOffsets* off;
  uint32_t pair_start;  // first act row
  uint32_t count;       // token rows
  bool shared;
};

TSG_DEV ExpertRef active_expert(const DecodeParams& p, const Group* groups, uint32_t n_groups,
                                uint32_t j) {
  ExpertRef r;
  if (j < n_groups) {
    const Group g = groups[j];
    r.blob = p.experts.base + static_cast<uint64_t>(g.expert) * p.experts.stride;
    r.off = &p.experts.off;
    r.pair_start = g.pair_start;
    r.count = g.pair_count;
    r.shared = false;
  } else {
    r.blob = p.experts.shared;
    r.off = &p.experts.shared_off;
    r.pair_start = static_cast<uint32_t>(p.T * p.K);
    r.count = static_cast<uint32_t>(p.T);
    r.shared = true;
  }
  return r;
}

TSG_DEV uint32_t token_of_row(const DecodeParams& p, const ExpertRef& ex, uint32_t i) {
  return ex.shared ? i : p.rb.sorted_pairs[ex.pair_start + i].token;
}

// ---------------------------------------------------------------------------
// gate/up
// ---------------------------------------------------------------------------
template <int TC>
struct GateUpLayout {
  uint32_t codes_bytes;   // per projection per item
  uint32_t scales_bytes;  // per projection per item
  uint32_t x_bytes;       // per token
  uint32_t xs_bytes;      // per token
  uint32_t stage_bytes;
  __host__ __device__ GateUpLayout(int D) {
    codes_bytes = kRows * (D / 2);
    scales_bytes = kRows * (D / 16);
    x_bytes = D * 4;
    xs_bytes = (D / 8) * 4;
    stage_bytes = 2 * codes_bytes + 2 * scales_bytes + TC * (x_bytes + xs_bytes);
  }
};

template <int TC>
__global__ void __launch_bounds__(256) decode_gate_up_kernel(DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages];
  const GateUpLayout<TC> L(p.D);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t n_groups = __ldcg(p.rb.n_groups);
  const uint32_t n_active = n_groups + (p.has_shared ? 1u : 0u);
  const uint32_t chunks = static_cast<uint32_t>(p.F / kRows);
  const uint32_t n_items = n_active * chunks;
  const int D = p.D, nwords = D / 8;
  uint32_t* err = p.rb.err;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // item k of this CTA -> global item index; experts interleave so that
  // neighbouring CTAs stream different experts
  auto item_of = [&](uint32_t k) { return blockIdx.x + k * gridDim.x; };
  auto issue = [&](uint32_t k, int s) {
    const uint32_t it = item_of(k);
    if (it >= n_items) return;
    const uint32_t j = it % n_active, c = it / n_active;
    const ExpertRef ex = active_expert(p, p.rb.groups, n_groups, j);
    uint8_t* st = smem + static_cast<size_t>(s) * L.stage_bytes;
    const uint32_t f0 = c * kRows;
    const int ntok = imin(TC, static_cast<int>(ex.count));
    const uint32_t bytes = 2 * L.codes_bytes + 2 * L.scales_bytes + ntok * (L.x_bytes + L.xs_bytes);
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_load(st, ex.blob + ex.off->gate_w + static_cast<size_t>(f0) * (D / 2), L.codes_bytes, &full[s]);
    bulk_load(st + L.codes_bytes, ex.blob + ex.off->up_w + static_cast<size_t>(f0) * (D / 2),
              L.codes_bytes, &full[s]);
    bulk_load(st + 2 * L.codes_bytes, ex.blob + ex.off->gate_s + static_cast<size_t>(f0) * (D / 16),
              L.scales_bytes, &full[s]);
    bulk_load(st + 2 * L.codes_bytes + L.scales_bytes,
              ex.blob + ex.off->up_s + static_cast<size_t>(f0) * (D / 16), L.scales_bytes, &full[s]);
    uint8_t* xs = st + 2 * L.codes_bytes + 2 * L.scales_bytes;
    for (int t = 0; t < ntok; ++t) {
      const uint32_t tok = token_of_row(p, ex, static_cast<uint32_t>(t));
      bulk_load(xs + t * L.x_bytes, p.xn + static_cast<size_t>(tok) * D, L.x_bytes, &full[s]);
      bulk_load(xs + TC * L.x_bytes + t * L.xs_bytes, p.xs8 + static_cast<size_t>(tok) * (D / 8),
                L.xs_bytes, &full[s]);
    }
  };

  if (tid == 0)
    for (int s = 0; s < kStages; ++s) issue(s, s);

  bool ok = true;
  for (uint32_t k = 0; item_of(k) < n_items; ++k) {
    const int s = static_cast<int>(k % kStages);
    const uint32_t it = item_of(k);
    const uint32_t j = it % n_active, c = it / n_active;
    const ExpertRef ex = active_expert(p, p.rb.groups, n_groups, j);
    if (!mbar_wait(&full[s], (k / kStages) & 1u, err)) { ok = false; break; }
    const uint8_t* st = smem + static_cast<size_t>(s) * L.stage_bytes;
    const uint32_t* gcodes = reinterpret_cast<const uint32_t*>(st);
    const uint32_t* ucodes = reinterpret_cast<const uint32_t*>(st + L.codes_bytes);
    const __half* gsc = reinterpret_cast<const __half*>(st + 2 * L.codes_bytes);
    const __half* usc = reinterpret_cast<const __half*>(st + 2 * L.codes_bytes + L.scales_bytes);
    const float* xs = reinterpret_cast<const float*>(st + 2 * L.codes_bytes + 2 * L.scales_bytes);
    const float* xs8 = reinterpret_cast<const float*>(st + 2 * L.codes_bytes + 2 * L.scales_bytes +
                                                      TC * L.x_bytes);
    const int row = warp;  // one warp per row of the chunk
    const uint32_t f = c * kRows + row;
    const uint32_t* gw = gcodes + row * nwords;
    const uint32_t* uw = ucodes + row * nwords;
    const __half* gs = gsc + row * (D / 32);
    const __half* us = usc + row * (D / 32);

    for (uint32_t t0 = 0; t0 < ex.count; t0 += TC) {
      const int nt = imin(TC, static_cast<int>(ex.count - t0));
      const float* xv = xs;
      const float* sv = xs8;
      if (t0 > 0) {
        // tokens beyond the staged chunk: read normalised rows from global
        // (rare: more than TC tokens routed to one expert)
        xv = nullptr;
      }
      float ag[TC], au[TC];
#pragma unroll
      for (int t = 0; t < TC; ++t) { ag[t] = 0.0f; au[t] = 0.0f; }
      for (int wi = lane; wi < nwords; wi += 32) {
        float fg[8], fu[8];
        nibbles_to_f32_plus1(gw[wi], fg);
        nibbles_to_f32_plus1(uw[wi], fu);
        const float sg = __half2float(gs[wi >> 2]);
        const float su = __half2float(us[wi >> 2]);
#pragma unroll
        for (int t = 0; t < TC; ++t) {
          if (t < nt) {
            float4 x0, x1;
            float sx;
            if (xv) {
              x0 = *reinterpret_cast<const float4*>(xv + t * D + wi * 8);
              x1 = *reinterpret_cast<const float4*>(xv + t * D + wi * 8 + 4);
              sx = sv[t * (D / 8) + wi];
            } else {
              const uint32_t tok = token_of_row(p, ex, t0 + t);
              x0 = __ldg(reinterpret_cast<const float4*>(p.xn + static_cast<size_t>(tok) * D + wi * 8));
              x1 = __ldg(reinterpret_cast<const float4*>(p.xn + static_cast<size_t>(tok) * D + wi * 8 + 4));
              sx = __ldg(p.xs8 + static_cast<size_t>(tok) * (D / 8) + wi);
            }
            float dg = fg[0] * x0.x;
            dg = fmaf(fg[1], x0.y, dg); dg = fmaf(fg[2], x0.z, dg); dg = fmaf(fg[3], x0.w, dg);
            dg = fmaf(fg[4], x1.x, dg); dg = fmaf(fg[5], x1.y, dg); dg = fmaf(fg[6], x1.z, dg);
            dg = fmaf(fg[7], x1.w, dg);
            float du = fu[0] * x0.x;
            du = fmaf(fu[1], x0.y, du); du = fmaf(fu[2], x0.z, du); du = fmaf(fu[3], x0.w, du);
            du = fmaf(fu[4], x1.x, du); du = fmaf(fu[5], x1.y, du); du = fmaf(fu[6], x1.z, du);
            du = fmaf(fu[7], x1.w, du);
            ag[t] = fmaf(sg, dg - sx, ag[t]);
            au[t] = fmaf(su, du - sx, au[t]);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < TC; ++t) {
        if (t < nt) {
          const float g = 16.0f * warp_sum(ag[t]);
          const float u = 16.0f * warp_sum(au[t]);
          if (lane == 0) {
            const float a = gate_act(p.act, g) * u;
            p.act_buf[static_cast<size_t>(ex.pair_start + t0 + t) * p.F + f] = __float2half_rn(a);
          }
        }
      }
    }
    __syncthreads();  // stage s fully consumed
    if (tid == 0) issue(k + kStages, s);
  }
  (void)ok;
  // drain: every copy this CTA issued has landed before shared memory is
  // released (bounded waits; stages past the last item were never issued)
  if (tid == 0) {
    uint32_t issued = 0;
    while (item_of(issued) < n_items) ++issued;
    for (uint32_t k = (issued > kStages ? issued - kStages : 0); k < issued; ++k)
      mbar_wait(&full[k % kStages], (k / kStages) & 1u, err);
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// down + combine
// ---------------------------------------------------------------------------
struct DownLayout {
  uint32_t rd;            // rows per CTA
  uint32_t codes_bytes;   // rd * F/2
  uint32_t scales_bytes;  // rd * F/16
  uint32_t act_bytes;     // per stage: up to max_tok act rows (fp16)
  uint32_t stage_bytes;
  uint32_t vbuf_off;      // [rows_total][rd] floats
  uint32_t xf_off;        // converted act [max_tok][F] floats + sums [max_tok][F/8]
  uint32_t total;
};

__global__ void __launch_bounds__(512) decode_down_kernel(DecodeParams p, DownLayout L,
                                                          int max_tok) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int D = p.D, F = p.F, fw = F / 8;
  const uint32_t d0 = blockIdx.x * L.rd;
  if (d0 >= static_cast<uint32_t>(D)) return;
  const uint32_t rd = umin32(L.rd, static_cast<uint32_t>(D) - d0);
  const uint32_t n_groups = __ldcg(p.rb.n_groups);
  const uint32_t n_active = n_groups + (p.has_shared ? 1u : 0u);
  uint32_t* err = p.rb.err;
  float* vbuf = reinterpret_cast<float*>(smem + L.vbuf_off);
  float* xf = reinterpret_cast<float*>(smem + L.xf_off);
  float* xf8 = xf + max_tok * F;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](uint32_t j, int s) {
    if (j >= n_active) return;
    const ExpertRef ex = active_expert(p, p.rb.groups, n_groups, j);
    uint8_t* st = smem + static_cast<size_t>(s) * L.stage_bytes;
    const uint32_t ntok = umin32(ex.count, static_cast<uint32_t>(max_tok));
    const uint32_t cb = rd * (F / 2), sb = rd * (F / 16);
    mbar_arrive_expect_tx(&full[s], cb + sb + ntok * F * 2);
    bulk_load(st, ex.blob + ex.off->down_w + static_cast<size_t>(d0) * (F / 2), cb, &full[s]);
    bulk_load(st + L.codes_bytes, ex.blob + ex.off->down_s + static_cast<size_t>(d0) * (F / 16), sb,
              &full[s]);
    if (ntok) {
      bulk_load(st + L.codes_bytes + L.scales_bytes,
                p.act_buf + static_cast<size_t>(ex.pair_start) * F, ntok * F * 2, &full[s]);
    }
  };
  if (tid == 0)
    for (int s = 0; s < kStages; ++s) issue(s, s);

  for (uint32_t j = 0; j < n_active; ++j) {
    const int s = static_cast<int>(j % kStages);
    const ExpertRef ex = active_expert(p, p.rb.groups, n_groups, j);
    if (!mbar_wait(&full[s], (j / kStages) & 1u, err)) break;
    const uint8_t* st = smem + static_cast<size_t>(s) * L.stage_bytes;
    const uint32_t* codes = reinterpret_cast<const uint32_t*>(st);
    const __half* scl = reinterpret_cast<const __half*>(st + L.codes_bytes);
    const __half* actv = reinterpret_cast<const __half*>(st + L.codes_bytes + L.scales_bytes);
    for (uint32_t t0 = 0; t0 < ex.count; t0 += max_tok) {
      const uint32_t nt = umin32(ex.count - t0, static_cast<uint32_t>(max_tok));
      // act rows -> fp32 plus 1.5 x the sum of each 8-element run
      for (uint32_t idx = tid; idx < nt * fw; idx += blockDim.x) {
        const uint32_t t = idx / fw, w = idx % fw;
        const __half* src = (t0 == 0) ? actv + t * F + w * 8
                                      : p.act_buf + static_cast<size_t>(ex.pair_start + t0 + t) * F + w * 8;
        const uint4 raw = *reinterpret_cast<const uint4*>(src);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
        float sum = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 v = __half22float2(h2[q]);
          xf[t * F + w * 8 + 2 * q] = v.x;
          xf[t * F + w * 8 + 2 * q + 1] = v.y;
          sum += v.x + v.y;
        }
        xf8[t * fw + w] = 1.5f * sum;
      }
      __syncthreads();
      for (uint32_t r = warp; r < rd; r += nwarps) {
        const uint32_t* cw = codes + r * fw;
        const __half* sr = scl + r * (F / 32);
        float acc[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[t] = 0.0f;
        for (int wi = lane; wi < fw; wi += 32) {
          float fv[8];
          nibbles_to_f32_plus1(cw[wi], fv);
          const float sc = __half2float(sr[wi >> 2]);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            if (t < static_cast<int>(nt)) {
              const float4 x0 = *reinterpret_cast<const float4*>(xf + t * F + wi * 8);
              const float4 x1 = *reinterpret_cast<const float4*>(xf + t * F + wi * 8 + 4);
              float dv = fv[0] * x0.x;
              dv = fmaf(fv[1], x0.y, dv); dv = fmaf(fv[2], x0.z, dv); dv = fmaf(fv[3], x0.w, dv);
              dv = fmaf(fv[4], x1.x, dv); dv = fmaf(fv[5], x1.y, dv); dv = fmaf(fv[6], x1.z, dv);
              dv = fmaf(fv[7], x1.w, dv);
              acc[t] = fmaf(sc, dv - xf8[t * fw + wi], acc[t]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          if (t < static_cast<int>(nt)) {
            const float v = 16.0f * warp_sum(acc[t]);
            if (lane == 0) vbuf[(ex.pair_start + t0 + t) * L.rd + r] = v;
          }
        }
      }
      __syncthreads();
    }
    if (tid == 0) issue(j + kStages, s);
  }
  // drain outstanding copies
  if (tid == 0) {
    const uint32_t last = n_active;
    for (uint32_t j = (last > kStages ? last - kStages : 0); j < last; ++j)
      mbar_wait(&full[j % kStages], (j / kStages) & 1u, err);
  }
  __syncthreads();
  if (error_raised(err)) return;

  // combine: y[t, d] = shared + sum_r w[t, r] * v[pair(t, r), d]
  const int T = p.T, K = p.K;
  for (uint32_t idx = tid; idx < static_cast<uint32_t>(T) * rd; idx += blockDim.x) {
    const uint32_t t = idx / rd, r = idx % rd;
    float acc = p.residual ? p.residual[static_cast<size_t>(t) * D + d0 + r] : 0.0f;
    if (p.has_shared) {
      float gate = 1.0f;
      if (p.rb.gate_raw) {
        const float z = __ldcg(p.rb.gate_raw + t) * __ldcg(p.rb.inv_rms + t);
        gate = 1.0f / (1.0f + __expf(-z));
      }
      acc = fmaf(gate, vbuf[(static_cast<uint32_t>(T * K) + t) * L.rd + r], acc);
    }
    for (int k = 0; k < K; ++k) {
      const uint32_t pos = __ldcg(p.rb.pair_pos + t * K + k);
      const float w = __ldcg(p.rb.weights + t * K + k);
      acc = fmaf(w, vbuf[pos * L.rd + r], acc);
    }
    if (p.y_f32)
      reinterpret_cast<float*>(p.y)[static_cast<size_t>(t) * p.y_stride + d0 + r] = acc;
    else
      reinterpret_cast<__nv_bfloat16*>(p.y)[static_cast<size_t>(t) * p.y_stride + d0 + r] =
          __float2bfloat16_rn(acc);
  }
}

}  // namespace

// Shared-memory plan for the down kernel.
static DownLayout down_layout(int T, int K, int D, int F, int num_sms, int max_tok) {
  DownLayout L;
  uint32_t rd = 4u * static_cast<uint32_t>((D + 4 * num_sms - 1) / (4 * num_sms));
  if (rd < 4) rd = 4;
  L.rd = rd;
  L.codes_bytes = rd * (F / 2);
  L.scales_bytes = (rd * (F / 16) + 15) / 16 * 16;
  L.act_bytes = static_cast<uint32_t>(max_tok) * F * 2;
  L.stage_bytes = (L.codes_bytes + L.scales_bytes + L.act_bytes + 127) / 128 * 128;
  L.vbuf_off = kStages * L.stage_bytes;
  const uint32_t rows_total = static_cast<uint32_t>(T * K + T);
  L.xf_off = L.vbuf_off + (rows_total * rd * 4 + 127) / 128 * 128;
  L.total = L.xf_off + static_cast<uint32_t>(max_tok) * (F + F / 8) * 4;
  return L;
}

cudaError_t launch_decode_gate_up(const DecodeParams& p, cudaStream_t s) {
  if (p.D % 256 || p.F % 64 || p.T <= 0) return cudaErrorInvalidValue;
  const int grid = p.num_sms;
  cudaError_t e;
  if (p.T == 1) {
    const GateUpLayout<1> L(p.D);
    const size_t smem = static_cast<size_t>(kStages) * L.stage_bytes;
    e = allow_max_smem(decode_gate_up_kernel<1>);
    if (e != cudaSuccess) return e;
    decode_gate_up_kernel<1><<<grid, 256, smem, s>>>(p);
  } else {
    const GateUpLayout<2> L(p.D);
    const size_t smem = static_cast<size_t>(kStages) * L.stage_bytes;
    e = allow_max_smem(decode_gate_up_kernel<2>);
    if (e != cudaSuccess) return e;
    decode_gate_up_kernel<2><<<grid, 256, smem, s>>>(p);
  }
  return cudaGetLastError();
}

cudaError_t launch_decode_down(const DecodeParams& p, cudaStream_t s) {
  const int max_tok = 8;
  const DownLayout L = down_layout(p.T, p.K, p.D, p.F, p.num_sms, max_tok);
  if (L.total > 220 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = allow_max_smem(decode_down_kernel);
  if (e != cudaSuccess) return e;
  const int nblk = (p.D + L.rd - 1) / L.rd;
  int threads = 32 * static_cast<int>((L.rd + 1) / 2);
  if (threads < 64) threads = 64;
  if (threads > 512) threads = 512;
  decode_down_kernel<<<nblk, threads, L.total, s>>>(p, L, max_tok);
  return cudaGetLastError();
}

cudaError_t launch_decode_experts(const DecodeParams& p, cudaStream_t s) {
  cudaError_t e = launch_decode_gate_up(p, s);
  if (e != cudaSuccess) return e;
  return launch_decode_down(p, s);
}

}  // namespace tsg
