// decode_fused.cu -- the whole MoE block for a decode batch (T <= 4 tokens)
// in one persistent cooperative kernel.
//
// Reference behaviour, per layer (RealForwardRunner.swift:3079-3330,
// QwenForwardRunner.swift:1460-1612): router GEMV + top-8 select
// (MoE.encodeRouterGemma4BF16, moe.metal:187-329), routed phase 1 gate/up +
// activation (moe.metal:455-574), phase 2 down + weighted reduce in slot
// order (moe.metal:651-687), and for Qwen the sigmoid-gated shared expert as
// the residual of that reduce.  The reference needs a host round trip after
// the router to page experts in; with every expert resident in HBM the block
// is one launch here, one CTA per SM:
//
//   prologue  the CTA's router rows arrive in shared memory by bulk copy
//             (input independent, so this overlaps the previous kernel);
//   router    every CTA reads the T token rows, computes their inverse RMS
//             and keeps them as fp16 MMA fragments plus per-32 sums; it then
//             writes the raw dots of its router rows; one grid barrier;
//   select    every CTA reads the T x E logits and selects the top K itself
//             (the reference's tie rule), then groups the pairs;
//   gate/up   units of (expert, 8 gate rows + the same 8 up rows) split
//             along K over the 16 warps; each warp loads its slice of int4
//             codes and fp16 scales straight from HBM into registers one unit
//             ahead, turns each 32-bit code word into four fp16 pairs
//             (1 + q/16) with a shift and a mask, and multiplies on the tensor
//             core (mma.sync m16n8k16, fp32 accumulate); per 32-wide group,
//             s * (16 sum(f x) - 24 sum(x)) = s * sum((q - 8) x); the last
//             warp of a unit adds the slices in order and writes
//             act = act_fn(g) * u as fp16;
//   barrier   (all act written);
//   down      units of (16 output rows, expert) split along K over 8 warps,
//             same arithmetic; the last warp of a unit writes its fp32 values
//             and the last unit of each 16-row block combines the block:
//             y = residual + shared + sum over ranks (ascending) w * v.
// Every wait is bounded; counters reset themselves for the next launch.
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = 16;
constexpr int kMaxTok = 4;
constexpr int kMaxPairs = 32;
constexpr int kMaxSlots = kMaxPairs + 1;
constexpr int kMaxK = 32;
constexpr int kGSlices = kWarps;  // gate/up unit K split
constexpr int kDSlices = 8;       // down unit K split
constexpr int kRed = 4;           // reduction slots in flight
constexpr int kMaxGPS = 8;        // groups per gate/up slice (D <= 4096)
constexpr int kMaxDPS = 4;        // groups per down slice (F <= 1024)

struct Counters {
  uint32_t router, gdone, done, pad;
  uint32_t dblock[1];  // [D / 16]
};

struct FusedParams {
  const uint16_t* x;
  uint32_t x_stride;
  int T, D, F, E, K, act, norm;
  float eps;
  const float* router_rows;  // [E + has_gate][D]
  int has_gate, has_shared;
  const float* per_expert_scale;
  const float* logit_bias;
  const uint32_t* ids_in;  // caller routing [T][K] or nullptr
  const float* w_in;
  ExpertSet experts;
  void* y;
  uint32_t y_stride;
  int y_f32;
  const float* residual;
  float* logits;   // [T][E + 1]
  float* inv_rms;  // [T]
  uint4* actfrag;  // [P + T][F / 8]
  float* actsum;   // [P + T][F / 8]
  float* vpart;    // [P + T][D]
  uint32_t* counters;
  uint32_t* ids_out;  // [T][K]
  float* w_out;       // [T][K]
  uint16_t* w16_out;  // [T][K] or nullptr
  Pair* pairs_out;    // [P] sorted pairs
  uint32_t* err;
  unsigned long long* stamps;  // debug: [grid][12] phase timestamps, or nullptr
};

struct Layout {
  uint32_t rows_per_cta;
  uint32_t rw_off, xf_off, xs_off, gred_off, dred_off, total;
};

__host__ __device__ inline uint32_t up128(uint32_t x) { return (x + 127u) & ~127u; }

__host__ __device__ inline Layout make_layout(int D, int rows_per_cta) {
  Layout L;
  L.rows_per_cta = rows_per_cta;
  uint32_t o = 0;
  L.rw_off = o;
  o = up128(o + rows_per_cta * D * 4);
  L.xf_off = o;
  o = up128(o + kMaxTok * D * 2);
  L.xs_off = o;
  o = up128(o + kMaxTok * (D / 32) * 4);
  L.gred_off = o;
  o = up128(o + kRed * kGSlices * 32 * 16);
  L.dred_off = o;
  o = up128(o + kRed * kDSlices * 32 * 16);
  L.total = o;
  return L;
}

TSG_DEV void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A 32-bit code word (elements e0..e7 of a row) as four fp16 pairs of
// 1 + q/16: (e0,e4), (e1,e5), (e2,e6), (e3,e7).
TSG_DEV void unpack_plus1(uint32_t w, uint32_t (&p)[4]) {
  p[0] = ((w << 6) & 0x03C003C0u) | 0x3C003C00u;
  p[1] = ((w << 2) & 0x03C003C0u) | 0x3C003C00u;
  p[2] = ((w >> 2) & 0x03C003C0u) | 0x3C003C00u;
  p[3] = ((w >> 6) & 0x03C003C0u) | 0x3C003C00u;
}

// Eight consecutive values as the matching B fragment chunk
// [(v0,v4), (v1,v5), (v2,v6), (v3,v7)] in fp16, and the sum of the values
// as rounded to fp16 (what the tensor core multiplies).
TSG_DEV uint4 frag_chunk(const float (&v)[8], float* sum) {
  __half2 h[4];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[i] = __floats2half2_rn(v[i], v[i + 4]);
    const float2 r = __half22float2(h[i]);
    s += r.x + r.y;
  }
  *sum = s;
  return make_uint4(*reinterpret_cast<uint32_t*>(&h[0]), *reinterpret_cast<uint32_t*>(&h[1]),
                    *reinterpret_cast<uint32_t*>(&h[2]), *reinterpret_cast<uint32_t*>(&h[3]));
}

TSG_DEV uint32_t ld_nc_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
TSG_DEV uint32_t ld_nc_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

TSG_DEV uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded spin until *ctr >= target.  Returns false on timeout/error.
TSG_DEV bool wait_counter(const uint32_t* ctr, uint32_t target, uint32_t* err) {
  if (ld_acquire(ctr) >= target) return true;
  const unsigned long long t0 = global_timer_ns();
  uint32_t spins = 0;
  while (ld_acquire(ctr) < target) {
    if ((++spins & 1023u) == 0u) {
      if (error_raised(err)) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        flag_error(err, TSG_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// Bounded spin on a shared-memory value.
TSG_DEV bool wait_shared(volatile const int* v, int target, uint32_t* err) {
  if (*v >= target) return true;
  const unsigned long long t0 = global_timer_ns();
  uint32_t spins = 0;
  while (*v < target) {
    if ((++spins & 1023u) == 0u) {
      if (error_raised(err)) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        flag_error(err, TSG_DEVERR_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// Grid-wide barrier on a self-resetting counter (the cooperative launch
// keeps every CTA resident).
TSG_DEV bool grid_barrier(uint32_t* ctr, uint32_t* err, volatile int* s_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, 1u);
    *s_ok = wait_counter(ctr, gridDim.x, err) ? 1 : 0;
  }
  __syncthreads();
  return *s_ok != 0;
}

__global__ void __launch_bounds__(kThreads, 1) decode_fused_kernel(FusedParams p, Layout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar_rw;
  __shared__ int s_ids[kMaxTok][kMaxK];
  __shared__ float s_w[kMaxTok][kMaxK];
  __shared__ float s_sc[kMaxTok][kMaxK];
  __shared__ int s_slot_expert[kMaxSlots], s_slot_start[kMaxSlots], s_slot_count[kMaxSlots];
  __shared__ int s_sorted_token[kMaxPairs + kMaxTok];
  __shared__ int s_pair_pos[kMaxPairs];
  __shared__ float s_inv[kMaxTok], s_gate[kMaxTok];
  __shared__ float s_red[kMaxTok][kWarps];
  __shared__ int s_nslots;
  __shared__ volatile int s_ok;
  __shared__ int s_gcnt[kRed], s_dcnt[kRed];
  __shared__ volatile int s_ggen[kRed], s_dgen[kRed];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = p.T, D = p.D, F = p.F, E = p.E, K = p.K;
  const int P = T * K;
  const int GD = D / 32, GF = F / 32;
  const int erows = E + p.has_gate;
  Counters* ctr = reinterpret_cast<Counters*>(p.counters);
  uint32_t* err = p.err;
  float* rw = reinterpret_cast<float*>(smem + L.rw_off);
  uint4* xf = reinterpret_cast<uint4*>(smem + L.xf_off);
  float* xs = reinterpret_cast<float*>(smem + L.xs_off);
  float4* gred = reinterpret_cast<float4*>(smem + L.gred_off);
  float4* dred = reinterpret_cast<float4*>(smem + L.dred_off);
  auto stamp = [&](int k) {
    if (p.stamps && tid == 0) p.stamps[blockIdx.x * 12 + k] = global_timer_ns();
  };
  stamp(0);

  // ---------------- prologue: router rows (input independent) ----------------
  int my_rows = 0;
  for (int r = blockIdx.x; r < erows && my_rows < static_cast<int>(L.rows_per_cta); r += gridDim.x)
    ++my_rows;
  if (tid == 0) {
    mbar_init(&bar_rw, 1);
    fence_mbar_init();
    if (my_rows > 0) {
      mbar_arrive_expect_tx(&bar_rw, my_rows * D * 4);
      for (int i = 0; i < my_rows; ++i)
        bulk_load(rw + i * D, p.router_rows + static_cast<size_t>(blockIdx.x + i * gridDim.x) * D,
                  D * 4, &bar_rw);
    }
  }
  if (tid < kRed) {
    s_gcnt[tid] = 0;
    s_dcnt[tid] = 0;
    s_ggen[tid] = 0;
    s_dgen[tid] = 0;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  stamp(1);

  // ---------------- tokens: norm, fp16 fragments, group sums ----------------
  const int nchunk = D / 8;
  float xv[kMaxTok][8];
  float ss[kMaxTok];
#pragma unroll
  for (int t = 0; t < kMaxTok; ++t) ss[t] = 0.0f;
  const bool has_chunk = tid < nchunk;  // D <= 4096
#pragma unroll
  for (int t = 0; t < kMaxTok; ++t) {
    if (t < T && has_chunk) {
      const uint4 raw =
          __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(t) * p.x_stride) + tid);
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xv[t][2 * j] = __uint_as_float(wv[j] << 16);
        xv[t][2 * j + 1] = __uint_as_float(wv[j] & 0xFFFF0000u);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss[t] = fmaf(xv[t][j], xv[t][j], ss[t]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) xv[t][j] = 0.0f;
    }
  }
#pragma unroll
  for (int t = 0; t < kMaxTok; ++t) {
    const float v = warp_sum(ss[t]);
    if (lane == 0) s_red[t][warp] = v;
  }
  __syncthreads();
  if (tid < T) {
    float s = 0.0f;
    for (int w = 0; w < kWarps; ++w) s += s_red[tid][w];
    const float inv = p.norm ? rsqrtf(s / static_cast<float>(D) + p.eps) : 1.0f;
    s_inv[tid] = inv;
    if (blockIdx.x == 0) p.inv_rms[tid] = inv;
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < kMaxTok; ++t) {
    if (t < T) {
      float v[8];
      const float inv = s_inv[t];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = xv[t][j] * inv;
      float s = 0.0f;
      const uint4 ch = frag_chunk(v, &s);
      if (has_chunk) xf[t * nchunk + tid] = ch;
      // a 32-wide group is four adjacent chunks = four adjacent lanes
      s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
      s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
      if (has_chunk && (tid & 3) == 0) xs[t * GD + tid / 4] = s;
    }
  }

  // ---------------- router dots ----------------
  if (my_rows > 0) {
    const int ok = mbar_wait(&bar_rw, 0, err) ? 1 : 0;
    if (!__syncthreads_and(ok)) return;
    for (int r = 0; r < my_rows; ++r) {
      float acc[kMaxTok];
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) acc[t] = 0.0f;
      if (has_chunk) {
        const float4 w0 = *reinterpret_cast<const float4*>(rw + r * D + tid * 8);
        const float4 w1 = *reinterpret_cast<const float4*>(rw + r * D + tid * 8 + 4);
        const float wr[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[t] = fmaf(wr[j], xv[t][j], acc[t]);
      }
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0) s_red[t][warp] = v;
      }
      __syncthreads();
      if (tid < T) {
        float s = 0.0f;
        for (int w = 0; w < kWarps; ++w) s += s_red[tid][w];
        p.logits[static_cast<size_t>(tid) * (E + 1) + (blockIdx.x + r * gridDim.x)] = s;
      }
      __syncthreads();
    }
  }
  stamp(2);
  if (!grid_barrier(&ctr->router, err, &s_ok)) return;
  stamp(3);

  // ---------------- selection and grouping (every CTA) ----------------
  if (warp < T) {
    const int t = warp;
    const float inv = s_inv[t];
    if (p.ids_in) {
      for (int k = lane; k < K; k += 32) {
        s_ids[t][k] = static_cast<int>(p.ids_in[t * K + k]);
        s_w[t][k] = p.w_in[t * K + k];
      }
    } else {
      // lane holds logits lane + 32 j; E <= 256
      float v[8];
      const float* lg = p.logits + static_cast<size_t>(t) * (E + 1);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = lane + 32 * j;
        float s = -INFINITY;
        if (e < E) {
          s = __ldcg(lg + e) * inv;
          if (p.logit_bias) s += __ldg(p.logit_bias + e);
        }
        v[j] = s;
      }
      for (int k = 0; k < K; ++k) {
        float best = -INFINITY;
        int bidx = 0x7FFFFFFF;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
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
          s_ids[t][k] = bidx;
          s_sc[t][k] = best;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (lane + 32 * j == bidx) v[j] = __int_as_float(0x7FC00000u);  // NaN: never again
      }
      __syncwarp();
      // softmax over the K selected scores (summed in slot order, as the
      // reference does) times the per-expert scale
      const float mx = s_sc[t][0];
      const float ex = lane < K ? expf(s_sc[t][lane] - mx) : 0.0f;
      __syncwarp();
      if (lane == 0) {
        float s = 0.0f;
        for (int k = 0; k < K; ++k) s += expf(s_sc[t][k] - mx);
        s_red[t][0] = s;
      }
      __syncwarp();
      if (lane < K) {
        const float gain = p.per_expert_scale ? __ldg(p.per_expert_scale + s_ids[t][lane]) : 1.0f;
        s_w[t][lane] = ex / s_red[t][0] * gain;
      }
    }
    if (t == 0) stamp(8);
    if (lane == 0 && p.has_gate)
      s_gate[t] =
          1.0f / (1.0f + __expf(-__ldcg(p.logits + static_cast<size_t>(t) * (E + 1) + E) * inv));
  }
  __syncthreads();
  stamp(9);
  if (warp == 0) {
    // stable grouping of the P <= 32 token-major pairs by expert
    const bool valid = lane < P;
    const int e = valid ? s_ids[lane / K][lane % K] : 0x7FFFFFFF;
    const uint32_t peers = __match_any_sync(0xFFFFFFFFu, e);
    const bool first = valid && (__ffs(peers) - 1) == lane;
    const uint32_t firsts = __ballot_sync(0xFFFFFFFFu, first);
    uint32_t below_first = 0, below = 0;
    for (int l = 0; l < P; ++l) {
      const int el = __shfl_sync(0xFFFFFFFFu, e, l);
      if (el < e) {
        below += 1u;
        if ((firsts >> l) & 1u) below_first += 1u;
      }
    }
    if (valid) {
      const int pos = static_cast<int>(below) + __popc(peers & ((1u << lane) - 1u));
      s_pair_pos[lane] = pos;
      s_sorted_token[pos] = lane / K;
      if (first) {
        s_slot_expert[below_first] = e;
        s_slot_start[below_first] = static_cast<int>(below);
        s_slot_count[below_first] = __popc(peers);
      }
      if (blockIdx.x == 0) {
        Pair pr;
        pr.token = static_cast<uint32_t>(lane / K);
        pr.expert = static_cast<uint32_t>(e);
        pr.rank = static_cast<uint32_t>(lane % K);
        pr.weight_bits = __half_as_ushort(__float2half_rn(s_w[lane / K][lane % K]));
        if (p.pairs_out) p.pairs_out[pos] = pr;
        if (p.ids_out) p.ids_out[lane] = static_cast<uint32_t>(e);
        if (p.w_out) p.w_out[lane] = s_w[lane / K][lane % K];
        if (p.w16_out) p.w16_out[lane] = pr.weight_bits;
      }
    }
    if (lane == 0) {
      int u = __popc(firsts);
      if (p.has_shared) {
        s_slot_expert[u] = -1;
        s_slot_start[u] = P;
        s_slot_count[u] = T;
        for (int t = 0; t < T; ++t) s_sorted_token[P + t] = t;
        ++u;
      }
      s_nslots = u;
    }
  }
  __syncthreads();
  stamp(4);
  const int nslots = s_nslots;

  auto slot_blob = [&](int j, const ExpertOffsets** off) -> const uint8_t* {
    const int e = s_slot_expert[j];
    if (e < 0) {
      *off = &p.experts.shared_off;
      return p.experts.shared;
    }
    *off = &p.experts.off;
    return p.experts.base + static_cast<uint64_t>(e) * p.experts.stride;
  };

  const int g = lane >> 2, c = lane & 3;
  const int fblocks = F / 8;

  // ---------------- gate/up ----------------
  {
    const int n_g = nslots * fblocks;
    const int my_g = n_g > static_cast<int>(blockIdx.x)
                         ? (n_g - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x
                         : 0;
    // this warp's K slice: groups [gi0, gi1)
    const int gi0 = (warp * GD) / kGSlices, gi1 = ((warp + 1) * GD) / kGSlices;
    const int ng = gi1 - gi0;
    // two register buffers of code words and scales, alternated at compile
    // time (a runtime index would put them in local memory)
    uint32_t cwa[kMaxGPS][2], swa[kMaxGPS][2], cwb[kMaxGPS][2], swb[kMaxGPS][2];
    auto load = [&](int i, uint32_t (&cw)[kMaxGPS][2], uint32_t (&sw)[kMaxGPS][2]) {
      const int k = static_cast<int>(blockIdx.x) + i * gridDim.x;
      const int j = k % nslots, fb = k / nslots;
      const ExpertOffsets* off;
      const uint8_t* blob = slot_blob(j, &off);
      const uint8_t* gr = blob + off->gate_w + static_cast<size_t>(fb * 8 + g) * (D / 2);
      const uint8_t* ur = blob + off->up_w + static_cast<size_t>(fb * 8 + g) * (D / 2);
      const __half* gs = reinterpret_cast<const __half*>(blob + off->gate_s) +
                         static_cast<size_t>(fb * 8 + g) * GD;
      const __half* us = reinterpret_cast<const __half*>(blob + off->up_s) +
                         static_cast<size_t>(fb * 8 + g) * GD;
#pragma unroll
      for (int q = 0; q < kMaxGPS; ++q) {
        if (q < ng) {
          const int gi = gi0 + q;
          cw[q][0] = ld_nc_u32(gr + gi * 16 + 4 * c);
          cw[q][1] = ld_nc_u32(ur + gi * 16 + 4 * c);
          sw[q][0] = ld_nc_u16(gs + gi);
          sw[q][1] = ld_nc_u16(us + gi);
        }
      }
    };
    // compute unit i from (cw, sw); returns false on a wait timeout
    auto step = [&](int i, const uint32_t (&cw)[kMaxGPS][2],
                    const uint32_t (&sw)[kMaxGPS][2]) -> bool {
      const int k = static_cast<int>(blockIdx.x) + i * gridDim.x;
      const int j = k % nslots, fb = k / nslots;
      const int cnt = s_slot_count[j], start = s_slot_start[j];
      const bool bvalid = g < cnt;
      const int btok = bvalid ? s_sorted_token[start + g] : 0;
      const int n0 = 2 * c, n1 = 2 * c + 1;
      const int tok0 = n0 < cnt ? s_sorted_token[start + n0] : -1;
      const int tok1 = n1 < cnt ? s_sorted_token[start + n1] : -1;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < kMaxGPS; ++q) {
        if (q < ng) {
          const int gi = gi0 + q;
          uint32_t pg[4], pu[4];
          unpack_plus1(cw[q][0], pg);
          unpack_plus1(cw[q][1], pu);
          uint4 bx = make_uint4(0u, 0u, 0u, 0u);
          if (bvalid) bx = xf[btok * nchunk + gi * 4 + c];
          float cf[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          mma_16816(cf, pg[0], pu[0], pg[1], pu[1], bx.x, bx.y);
          mma_16816(cf, pg[2], pu[2], pg[3], pu[3], bx.z, bx.w);
          const float sg = __half2float(__ushort_as_half(static_cast<unsigned short>(sw[q][0])));
          const float su = __half2float(__ushort_as_half(static_cast<unsigned short>(sw[q][1])));
          const float x0 = tok0 >= 0 ? xs[tok0 * GD + gi] : 0.0f;
          const float x1 = tok1 >= 0 ? xs[tok1 * GD + gi] : 0.0f;
          acc[0] = fmaf(sg, fmaf(16.0f, cf[0], -24.0f * x0), acc[0]);
          acc[1] = fmaf(sg, fmaf(16.0f, cf[1], -24.0f * x1), acc[1]);
          acc[2] = fmaf(su, fmaf(16.0f, cf[2], -24.0f * x0), acc[2]);
          acc[3] = fmaf(su, fmaf(16.0f, cf[3], -24.0f * x1), acc[3]);
        }
      }
      // hand the slice to the reduction slot of this unit
      const int r = i % kRed;
      if (!wait_shared(&s_ggen[r], i / kRed, err)) return false;
      gred[(r * kGSlices + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __threadfence_block();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&s_gcnt[r], 1) == kGSlices - 1;
      last = __shfl_sync(0xFFFFFFFFu, last, 0);
      if (last) {
        __threadfence_block();
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int w = 0; w < kGSlices; ++w) {
          const float4 q4 = gred[(r * kGSlices + w) * 32 + lane];
          v[0] += q4.x;
          v[1] += q4.y;
          v[2] += q4.z;
          v[3] += q4.w;
        }
        // rows g: gate f = 8 fb + g (v0, v1), up (v2, v3); columns n0, n1.
        // Gather the 8 act values of each column to one lane via shuffles.
        const float a0 = gate_act(p.act, v[0]) * v[2];
        const float a1 = gate_act(p.act, v[1]) * v[3];
        float col[8];
        const int src_c = (lane & 7) >> 1;  // lane n < 8 collects column n
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
          const float s0 = __shfl_sync(0xFFFFFFFFu, a0, gg * 4 + src_c);
          const float s1 = __shfl_sync(0xFFFFFFFFu, a1, gg * 4 + src_c);
          col[gg] = (lane & 1) ? s1 : s0;
        }
        if (lane < cnt) {
          float sum;
          const uint4 chunk = frag_chunk(col, &sum);
          const size_t row = static_cast<size_t>(start + lane);
          p.actfrag[row * fblocks + fb] = chunk;
          p.actsum[row * fblocks + fb] = sum;
        }
        __syncwarp();
        if (lane == 0) {
          s_gcnt[r] = 0;
          __threadfence_block();
          s_ggen[r] = i / kRed + 1;
        }
      }
      return true;
    };
    if (my_g > 0) load(0, cwa, swa);
    for (int i = 0; i < my_g; i += 2) {
      if (i + 1 < my_g) load(i + 1, cwb, swb);
      if (!step(i, cwa, swa)) return;
      if (i + 1 >= my_g) break;
      if (i + 2 < my_g) load(i + 2, cwa, swa);
      if (!step(i + 1, cwb, swb)) return;
    }
  }
  stamp(5);
  if (!grid_barrier(&ctr->gdone, err, &s_ok)) return;
  stamp(6);

  // ---------------- down + combine ----------------
  {
    const int dblocks = D / 16;
    const int n_d = nslots * dblocks;
    const int my_d = n_d > static_cast<int>(blockIdx.x)
                         ? (n_d - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x
                         : 0;
    const int n_sub = my_d * kDSlices;
    uint32_t cwa[kMaxDPS][2], swa[kMaxDPS][2], cwb[kMaxDPS][2], swb[kMaxDPS][2];
    uint4 bxa[kMaxDPS], bxb[kMaxDPS];
    auto load = [&](int q, uint32_t (&cw)[kMaxDPS][2], uint32_t (&sw)[kMaxDPS][2],
                    uint4 (&bx)[kMaxDPS]) {
      const int i = q / kDSlices, sl = q % kDSlices;
      const int k = static_cast<int>(blockIdx.x) + i * gridDim.x;
      const int j = k % nslots, db = k / nslots;
      const int gf0 = (sl * GF) / kDSlices, gf1 = ((sl + 1) * GF) / kDSlices;
      const ExpertOffsets* off;
      const uint8_t* blob = slot_blob(j, &off);
      const uint8_t* r0 = blob + off->down_w + static_cast<size_t>(db * 16 + g) * (F / 2);
      const uint8_t* r1 = r0 + static_cast<size_t>(8) * (F / 2);
      const __half* s0 = reinterpret_cast<const __half*>(blob + off->down_s) +
                         static_cast<size_t>(db * 16 + g) * GF;
      const __half* s1 = s0 + static_cast<size_t>(8) * GF;
      const int cnt = s_slot_count[j], start = s_slot_start[j];
#pragma unroll
      for (int u = 0; u < kMaxDPS; ++u) {
        const int gi = gf0 + u;
        if (gi < gf1) {
          cw[u][0] = ld_nc_u32(r0 + gi * 16 + 4 * c);
          cw[u][1] = ld_nc_u32(r1 + gi * 16 + 4 * c);
          sw[u][0] = ld_nc_u16(s0 + gi);
          sw[u][1] = ld_nc_u16(s1 + gi);
          bx[u] = g < cnt ? __ldcg(p.actfrag + static_cast<size_t>(start + g) * fblocks +
                                   gi * 4 + c)
                          : make_uint4(0u, 0u, 0u, 0u);
        }
      }
    };
    auto step = [&](int qi, const uint32_t (&cw)[kMaxDPS][2], const uint32_t (&sw)[kMaxDPS][2],
                    const uint4 (&bxv)[kMaxDPS]) -> bool {
      const int i = qi / kDSlices, sl = qi % kDSlices;
      const int k = static_cast<int>(blockIdx.x) + i * gridDim.x;
      const int j = k % nslots, db = k / nslots;
      const int cnt = s_slot_count[j], start = s_slot_start[j];
      const int gf0 = (sl * GF) / kDSlices, gf1 = ((sl + 1) * GF) / kDSlices;
      const int n0 = 2 * c, n1 = 2 * c + 1;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int u = 0; u < kMaxDPS; ++u) {
        const int gi = gf0 + u;
        if (gi < gf1) {
          uint32_t p0[4], p1[4];
          unpack_plus1(cw[u][0], p0);
          unpack_plus1(cw[u][1], p1);
          const uint4 bx = bxv[u];
          float cf[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          mma_16816(cf, p0[0], p1[0], p0[1], p1[1], bx.x, bx.y);
          mma_16816(cf, p0[2], p1[2], p0[3], p1[3], bx.z, bx.w);
          const float sa = __half2float(__ushort_as_half(static_cast<unsigned short>(sw[u][0])));
          const float sb = __half2float(__ushort_as_half(static_cast<unsigned short>(sw[u][1])));
          float a0 = 0.0f, a1 = 0.0f;
          if (n0 < cnt) {
            const float4 q = __ldcg(reinterpret_cast<const float4*>(
                p.actsum + static_cast<size_t>(start + n0) * fblocks + gi * 4));
            a0 = q.x + q.y + q.z + q.w;
          }
          if (n1 < cnt) {
            const float4 q = __ldcg(reinterpret_cast<const float4*>(
                p.actsum + static_cast<size_t>(start + n1) * fblocks + gi * 4));
            a1 = q.x + q.y + q.z + q.w;
          }
          acc[0] = fmaf(sa, fmaf(16.0f, cf[0], -24.0f * a0), acc[0]);
          acc[1] = fmaf(sa, fmaf(16.0f, cf[1], -24.0f * a1), acc[1]);
          acc[2] = fmaf(sb, fmaf(16.0f, cf[2], -24.0f * a0), acc[2]);
          acc[3] = fmaf(sb, fmaf(16.0f, cf[3], -24.0f * a1), acc[3]);
        }
      }
      const int r = i % kRed;
      if (!wait_shared(&s_dgen[r], i / kRed, err)) return false;
      dred[(r * kDSlices + sl) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __threadfence_block();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&s_dcnt[r], 1) == kDSlices - 1;
      last = __shfl_sync(0xFFFFFFFFu, last, 0);
      if (!last) return true;
      __threadfence_block();
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int w = 0; w < kDSlices; ++w) {
        const float4 q4 = dred[(r * kDSlices + w) * 32 + lane];
        v[0] += q4.x;
        v[1] += q4.y;
        v[2] += q4.z;
        v[3] += q4.w;
      }
      __syncwarp();
      if (lane == 0) {
        s_dcnt[r] = 0;
        __threadfence_block();
        s_dgen[r] = i / kRed + 1;
      }
      const int d0 = db * 16;
      if (n0 < cnt) {
        p.vpart[static_cast<size_t>(start + n0) * D + d0 + g] = v[0];
        p.vpart[static_cast<size_t>(start + n0) * D + d0 + 8 + g] = v[2];
      }
      if (n1 < cnt) {
        p.vpart[static_cast<size_t>(start + n1) * D + d0 + g] = v[1];
        p.vpart[static_cast<size_t>(start + n1) * D + d0 + 8 + g] = v[3];
      }
      __threadfence();
      __syncwarp();
      int lastblk = 0;
      if (lane == 0)
        lastblk = atomicAdd(&ctr->dblock[db], 1u) == static_cast<uint32_t>(nslots - 1);
      lastblk = __shfl_sync(0xFFFFFFFFu, lastblk, 0);
      if (lastblk) {
        // every expert of this 16-row block is written: combine it
        __threadfence();
        for (int q = lane; q < T * 16; q += 32) {
          const int t = q / 16, d = d0 + q % 16;
          float y = p.residual ? p.residual[static_cast<size_t>(t) * D + d] : 0.0f;
          if (p.has_shared) {
            const float sv = __ldcg(p.vpart + static_cast<size_t>(P + t) * D + d);
            y = p.has_gate ? fmaf(s_gate[t], sv, y) : y + sv;
          }
          for (int rr = 0; rr < K; ++rr)
            y = fmaf(s_w[t][rr],
                     __ldcg(p.vpart + static_cast<size_t>(s_pair_pos[t * K + rr]) * D + d), y);
          if (p.y_f32)
            reinterpret_cast<float*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] = y;
          else
            reinterpret_cast<__nv_bfloat16*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] =
                __float2bfloat16_rn(y);
        }
        if (lane == 0) ctr->dblock[db] = 0u;  // ready for the next launch
      }
      return true;
    };
    int qi = warp;
    if (qi < n_sub) load(qi, cwa, swa, bxa);
    for (; qi < n_sub; qi += 2 * kWarps) {
      if (qi + kWarps < n_sub) load(qi + kWarps, cwb, swb, bxb);
      if (!step(qi, cwa, swa, bxa)) return;
      if (qi + kWarps >= n_sub) break;
      if (qi + 2 * kWarps < n_sub) load(qi + 2 * kWarps, cwa, swa, bxa);
      if (!step(qi + kWarps, cwb, swb, bxb)) return;
    }
  }
  __syncthreads();
  stamp(7);
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&ctr->done, 1u) == gridDim.x - 1) {
      ctr->router = 0u;
      ctr->gdone = 0u;
      __threadfence();
      ctr->done = 0u;
    }
  }
}

}  // namespace

bool decode_fused_supported(int T, int K, int E, int has_gate, int num_sms) {
  return T >= 1 && T <= kMaxTok && T * K <= kMaxPairs && K <= kMaxK && E <= 256 &&
         E + has_gate <= 2 * num_sms;
}

size_t decode_fused_smem(int T, int D, int F, int K, int E, int has_gate, int num_sms) {
  (void)T;
  (void)F;
  (void)K;
  const int rows_per_cta = (E + has_gate + num_sms - 1) / num_sms;
  return make_layout(D, rows_per_cta).total;
}

cudaError_t launch_decode_fused(const DecodeFusedArgs& a, cudaStream_t s) {
  if (!decode_fused_supported(a.T, a.K, a.E, a.has_gate, a.num_sms) || a.D % 256 || a.F % 64 ||
      a.D > 4096 || a.F > 1024)
    return cudaErrorInvalidValue;
  FusedParams p{};
  p.x = a.x;
  p.x_stride = a.x_stride;
  p.T = a.T;
  p.D = a.D;
  p.F = a.F;
  p.E = a.E;
  p.K = a.K;
  p.act = a.act;
  p.norm = a.norm;
  p.eps = a.eps;
  p.router_rows = a.router_rows;
  p.has_gate = a.has_gate;
  p.has_shared = a.has_shared;
  p.per_expert_scale = a.per_expert_scale;
  p.logit_bias = a.logit_bias;
  p.ids_in = a.ids_in;
  p.w_in = a.w_in;
  p.experts = a.experts;
  p.y = a.y;
  p.y_stride = a.y_stride;
  p.y_f32 = a.y_f32;
  p.residual = a.residual;
  p.logits = a.logits;
  p.inv_rms = a.inv_rms;
  p.actfrag = reinterpret_cast<uint4*>(a.actfrag);
  p.actsum = a.actsum;
  p.vpart = a.vpart;
  p.counters = a.counters;
  p.ids_out = a.ids_out;
  p.w_out = a.w_out;
  p.w16_out = a.w16_out;
  p.pairs_out = a.pairs_out;
  p.err = a.err;
  p.stamps = a.stamps;
  const int rows_per_cta = (a.E + a.has_gate + a.num_sms - 1) / a.num_sms;
  const Layout L = make_layout(a.D, rows_per_cta);
  cudaError_t e = allow_max_smem(decode_fused_kernel);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = a.allow_pdl ? 1 : 0;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, decode_fused_kernel, p, L);
}

}  // namespace tsg
