// decode_fused.cu -- the whole MoE block for a decode batch (T <= 4 tokens)
// in one persistent cooperative kernel.
//
// Reference behaviour, per layer (RealForwardRunner.swift:3079-3330,
// QwenForwardRunner.swift:1460-1612): router GEMV + top-K select
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
//             and keeps them as fp16 MMA fragments; it then publishes the raw
//             dots of its router rows as (launch tag, value) words;
//   select    every CTA reads all logits of the launch (polling their tags)
//             and selects the top K of each token itself: four lanes per
//             logit count the logits ordered before it (larger value, or
//             equal value and smaller index: the reference's order and tie
//             rule), and ranks below K are the selection in slot order; the
//             pairs are grouped by expert with a 32-lane bitonic sort;
//   stream    the CTA requests, by 1-D bulk copies of contiguous rows, every
//             weight tile it will need -- its share of the gate/up rows and
//             the down rows of its blocks of y for all selected experts --
//             into shared-memory rings, as far ahead as the rings allow (for
//             one token all of it at once, about 200 KB per SM);
//   gate/up   units of (expert, 8 gate rows + the same 8 up rows); the 16
//             warps split a unit along K, dequantise int4 codes to scaled
//             fp16 and multiply on the tensor core (mma.sync m16n8k16, fp32
//             accumulate); a warp reduces the unit, writes
//             act = act_fn(g) * u to global memory as fp16 MMA fragments;
//             the CTA then adds itself to the launch's counter;
//   down      once the counter holds every CTA, the act rows are staged in
//             shared memory; each CTA owns whole 8-row blocks of y over all
//             experts, loaded per pair of experts and computed as tiles of two
//             experts' rows (rows 0-7 and 8-15 of the MMA, their tokens in
//             separate columns), and combines its blocks:
//             y = residual + gate * shared + sum over ranks (ascending) w * v.
//
// Fragments: a thread of the MMA (lane = 4 g + c) reads one whole 32-wide
// group of a weight row with one 16-byte load -- group 4 s + c of a
// super-group s of 4 groups -- so each MMA mixes the four groups of a
// super-group; both operands follow the same permutation of K, so the sum is
// unchanged.  A code word holds elements e0..e7 (e_{2i} in the low nibble of
// byte i); (w & 0x000F000F) | 0x64006400 is the fp16 pair (1024 + q0,
// 1024 + q4), the 0x00F000F0 mask gives (1024 + 16 q1, 1024 + 16 q5), the
// same on w >> 8 gives elements 2, 6 and 3, 7; subtracting 1032 (or 1152)
// is exact, and a multiply by the group's scale (or scale / 16) rounds once:
// fp16 weights s (q - 8).
//
// Warps reconverge (__syncwarp) after code that only one lane runs and
// before warp-collective code: a warp left split runs its shuffles and MMAs
// several times slower.  Every wait is bounded (one second); on an error the
// CTA waits, again bounded, for its own copies in flight before it exits and
// the host clears the cross-CTA signals.
#include <algorithm>

#include "tsg_common.cuh"
#include "tsg_kernels.cuh"
#include "int4_mma.cuh"

namespace tsg {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = 16;
constexpr int kMaxTok = 4;
constexpr int kMaxPairs = 32;
constexpr int kMaxSlots = kMaxPairs + 1;
constexpr int kMaxK = 32;
constexpr int kMaxGU = 16;   // gate/up ring slots
constexpr int kMaxDS = 32;   // down ring slots
constexpr int kStamps = 32;  // debug timestamps per CTA

// Cross-CTA signalling.  Every CTA counts its own launches in epoch[cta];
// all CTAs of a launch hold the same value, so "epoch + 1" tags this launch.
// The router logits are published as (tag, value) 64-bit words, in
// kLogitCopies copies to spread the readers over the L2, and a reader polls
// the words themselves.  The gate/up rows of the grid are counted in
// gcount[tag & 1]; the last launch's counter (the other one) is cleared by
// CTA 0 for the next launch.  (A shared counter measured cheaper than
// per-CTA flags that every CTA polls.)
constexpr int kMaxCtas = 256;
constexpr int kLogitCopies = 4;
struct Signals {
  uint32_t epoch[kMaxCtas];
  uint32_t gcount[2];
  uint32_t pad[kMaxCtas - 2];
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
  unsigned long long* tlogits;  // [kLogitCopies][T][E + 1] (tag << 32 | bits)
  float* inv_rms;               // [T]
  uint4* hfrag;                 // [P + T][F / 8] act fragments
  uint32_t* counters;           // Signals
  uint32_t* ids_out;            // [T][K]
  float* w_out;                 // [T][K]
  uint16_t* w16_out;            // [T][K] or nullptr
  Pair* pairs_out;              // [P] sorted pairs
  uint32_t* err;
  unsigned long long* stamps;   // debug: [grid][kStamps] timestamps, or nullptr
  uint32_t smem_bytes;          // dynamic shared memory of the launch
};

__host__ __device__ inline uint32_t align_up_u32(uint32_t x, uint32_t a) {
  return (x + a - 1u) / a * a;
}

// Shared-memory plan, the same on host and device.
struct Plan {
  uint32_t xf_off, gred_off, ring_off;
  uint32_t su;       // gate/up unit: gate codes, up codes (8 rows each), scales
  uint32_t hstride;  // bytes per staged act row (padded)
};

__host__ __device__ inline Plan make_plan(int T, int D, int F) {
  Plan L;
  uint32_t o = 0;
  L.xf_off = o;
  o = align_up_u32(o + static_cast<uint32_t>(T * D * 2), 128);
  L.gred_off = o;
  o += 2u * kWarps * 32u * 16u;
  L.ring_off = o;
  L.su = align_up_u32(static_cast<uint32_t>(9 * D), 128);
  L.hstride = static_cast<uint32_t>(2 * F + 16);
  return L;
}

// A down unit is a pair of slots over the CTA's nb blocks of y: codes of
// slot a, of slot b (8 nb rows each), scales of a, of b.
__host__ __device__ inline uint32_t down_unit_bytes(int nb, int F) {
  return align_up_u32(static_cast<uint32_t>(9 * F * nb), 128);
}

// Staged act rows and the down results [rows][vcols] of this CTA's blocks.
__host__ __device__ inline uint32_t h_v_off(const Plan& L, int rows) {
  return align_up_u32(static_cast<uint32_t>(rows) * L.hstride, 16);
}
__host__ __device__ inline uint32_t h_bytes(const Plan& L, int rows, int vcols) {
  return h_v_off(L, rows) + static_cast<uint32_t>(rows * vcols * 4);
}

// Ring sizes of one CTA: everything at once when it fits, else a streaming
// split.  Returns the gate/up region size (which also holds the staged act
// rows), 128-aligned.
__host__ __device__ inline uint32_t plan_rings(uint32_t su, uint32_t sd, uint32_t cap, int my_gu,
                                               int my_d, uint32_t hb, int* NU, int* NDS) {
  const uint32_t all_gu = static_cast<uint32_t>(my_gu) * su;
  const uint32_t all_region = align_up_u32(all_gu > hb ? all_gu : hb, 128);
  if (all_region + static_cast<uint32_t>(my_d) * sd <= cap && my_gu <= kMaxGU &&
      my_d <= kMaxDS) {
    *NU = my_gu;
    *NDS = my_d;
    return all_region;
  }
  int nu = static_cast<int>((cap * 5u / 8u) / su);
  nu = nu < 2 ? 2 : nu;
  nu = nu > kMaxGU ? kMaxGU : nu;
  nu = nu > my_gu ? my_gu : nu;
  const uint32_t gb = static_cast<uint32_t>(nu) * su;
  const uint32_t region = align_up_u32(gb > hb ? gb : hb, 128);
  int nd = region < cap ? static_cast<int>((cap - region) / sd) : 0;
  nd = nd > kMaxDS ? kMaxDS : nd;
  nd = nd > my_d ? my_d : nd;
  *NU = nu;
  *NDS = nd;
  return region;
}





// Eight consecutive activations as the matching B fragment chunk
// [(v0,v4), (v2,v6), (v1,v5), (v3,v7)] in fp16.
TSG_DEV uint4 frag_chunk(const float (&v)[8]) {
  return make_uint4(h2_bits(__floats2half2_rn(v[0], v[4])), h2_bits(__floats2half2_rn(v[2], v[6])),
                    h2_bits(__floats2half2_rn(v[1], v[5])), h2_bits(__floats2half2_rn(v[3], v[7])));
}

// One super-group: the thread's 16 bytes of two rows (row g of the first
// operand half, row g of the second) and the B chunks of its group; eight
// MMAs into acc.
TSG_DEV void mma_supergroup(float (&acc)[4], const uint4& ra, const uint4& rb, __half2 sa,
                            __half2 sa16, __half2 sb, __half2 sb16, const uint4 (&bx)[4]) {
  const uint32_t wa[4] = {ra.x, ra.y, ra.z, ra.w};
  const uint32_t wb[4] = {rb.x, rb.y, rb.z, rb.w};
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    uint32_t pa[4], pb[4];
    dequant_word(wa[wi], sa, sa16, pa);
    dequant_word(wb[wi], sb, sb16, pb);
    mma_16816(acc, pa[0], pb[0], pa[1], pb[1], bx[wi].x, bx[wi].y);
    mma_16816(acc, pa[2], pb[2], pa[3], pb[3], bx[wi].z, bx[wi].w);
  }
}


// a / b for small non-negative ints (a < 2^16, b <= 4096) through a float
// reciprocal of b: a few instructions instead of an integer division.
TSG_DEV int qdiv(int a, float inv_b) {
  return __float2int_rz((static_cast<float>(a) + 0.5f) * inv_b);
}

// Debug phase timestamp.
TSG_DEV void stamp_at(unsigned long long* stamps, int idx) { stamps[idx] = global_timer_ns(); }

TSG_DEV void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
TSG_DEV unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
TSG_DEV uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait on an mbarrier phase that ignores the error word: used only
// to let this CTA's own copies land before it exits after an error.
__device__ __noinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_timer_ns() - t0 > kWaitLimitNs) return;
}

// Bounded mbarrier wait with the spin loop inline (a call would spill the
// caller's registers to the stack).
TSG_DEV bool mbar_wait_inl(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      flag_error(err, TSG_DEVERR_TIMEOUT);
      return false;
    }
    if ((++spins & 15u) == 0u && error_raised(err)) return false;
  }
  return true;
}

// Whether a poll should give up (an error elsewhere, or the time limit).
__device__ __noinline__ bool poll_give_up(unsigned long long t0, uint32_t* err) {
  if (error_raised(err)) return true;
  if (global_timer_ns() - t0 > kWaitLimitNs) {
    flag_error(err, TSG_DEVERR_TIMEOUT);
    return true;
  }
  return false;
}

// Total order key of a logit: larger value first; NaN below everything.
TSG_DEV uint32_t order_key(float s) {
  if (s != s) return 0u;
  const uint32_t u = __float_as_uint(s + 0.0f);  // -0 -> +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
TSG_DEV float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Copies of one gate/up unit or one down unit into its ring slot (out of
// line: each is issued from two places).
struct Rings {
  uint8_t* ring;   // gate/up slots
  uint8_t* dring;  // down slots
  uint64_t* bar_g;
  uint64_t* bar_d;
  const int* slot_expert;
  int g0, fbk, NU, NDS, b0, nb, nslots;
  uint32_t su, sd;
};

__device__ __forceinline__ const uint8_t* slot_blob(const FusedParams& p, int e,
                                                     const ExpertOffsets** off) {
  if (e < 0) {
    *off = &p.experts.shared_off;
    return p.experts.shared;
  }
  *off = &p.experts.off;
  return p.experts.base + static_cast<uint64_t>(e) * p.experts.stride;
}

// gate rows 8 fb .. 8 fb + 7 and the same up rows, in four copies of four
// rows, then both scale rows
__device__ __forceinline__ void issue_gu(const FusedParams& p, const Rings& R, int i) {
  const int D = p.D;
  const int u = R.g0 + i, j = u / R.fbk, fb = u % R.fbk;
  uint8_t* dst = R.ring + static_cast<uint32_t>(i % R.NU) * R.su;
  uint64_t* bar = &R.bar_g[i % R.NU];
  const ExpertOffsets* off;
  const uint8_t* blob = slot_blob(p, R.slot_expert[j], &off);
  const uint8_t* gsrc = blob + off->gate_w + static_cast<size_t>(fb) * (4 * D);
  const uint8_t* usrc = blob + off->up_w + static_cast<size_t>(fb) * (4 * D);
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>(9 * D));
  bulk_load(dst, gsrc, 2 * D, bar);
  bulk_load(dst + 2 * D, gsrc + 2 * D, 2 * D, bar);
  bulk_load(dst + 4 * D, usrc, 2 * D, bar);
  bulk_load(dst + 6 * D, usrc + 2 * D, 2 * D, bar);
  bulk_load(dst + 8 * D, blob + off->gate_s + static_cast<size_t>(fb) * (D / 2), D / 2, bar);
  bulk_load(dst + 8 * D + D / 2, blob + off->up_s + static_cast<size_t>(fb) * (D / 2), D / 2, bar);
}

// a down unit: rows 8 b0 .. 8 (b0 + nb) - 1 of slot 2 k (and of slot 2 k + 1)
__device__ __forceinline__ void issue_d(const FusedParams& p, const Rings& R, int k) {
  const int F = p.F;
  const int ja = 2 * k;
  const bool two = ja + 1 < R.nslots;
  const uint32_t cb = static_cast<uint32_t>(4 * F * R.nb);   // code bytes of one slot
  const uint32_t sb = static_cast<uint32_t>(F / 2 * R.nb);   // scale bytes of one slot
  uint8_t* dst = R.dring + static_cast<uint32_t>(k % R.NDS) * R.sd;
  uint64_t* bar = &R.bar_d[k % R.NDS];
  mbar_arrive_expect_tx(bar, (cb + sb) * (two ? 2u : 1u));
  for (int h = 0; h < (two ? 2 : 1); ++h) {
    const ExpertOffsets* off;
    const uint8_t* blob = slot_blob(p, R.slot_expert[ja + h], &off);
    bulk_load(dst + h * cb, blob + off->down_w + static_cast<size_t>(R.b0) * (4 * F), cb, bar);
    bulk_load(dst + 2 * cb + h * sb, blob + off->down_s + static_cast<size_t>(R.b0) * (F / 2), sb,
              bar);
  }
}

// After an error: wait (bounded) for this CTA's copies still in flight.
__device__ __noinline__ void drain_rings(const Rings& R, int g_issued, int d_issued) {
  for (int i = (g_issued > R.NU ? g_issued - R.NU : 0); i < g_issued; ++i)
    drain_wait(&R.bar_g[i % R.NU], static_cast<uint32_t>(i / R.NU) & 1u);
  for (int k = (d_issued > R.NDS ? d_issued - R.NDS : 0); k < d_issued; ++k)
    drain_wait(&R.bar_d[k % R.NDS], static_cast<uint32_t>(k / R.NDS) & 1u);
}

template <int TT>
__global__ void __launch_bounds__(kThreads, 1)
    decode_fused_kernel(const __grid_constant__ FusedParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar_rw;
  __shared__ __align__(8) uint64_t bar_g[kMaxGU];
  __shared__ __align__(8) uint64_t bar_d[kMaxDS];
  __shared__ int s_ids[kMaxTok][kMaxK];
  __shared__ float s_w[kMaxTok][kMaxK];
  __shared__ float s_sc[kMaxTok][kMaxK];
  __shared__ int s_slot_expert[kMaxSlots], s_slot_start[kMaxSlots], s_slot_count[kMaxSlots];
  __shared__ int s_sorted_token[kMaxPairs + kMaxTok];
  __shared__ int s_pair_pos[kMaxPairs];
  __shared__ float s_inv[kMaxTok], s_gate[kMaxTok];
  __shared__ float s_red[2 * kMaxTok][kWarps];
  __shared__ int s_nslots;
  __shared__ volatile int s_ok;
  __shared__ int s_failed;
  __shared__ int s_g_issued;
  __shared__ int s_d_issued;
  __shared__ uint32_t s_epoch;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int T = TT;
  const int D = p.D, F = p.F, E = p.E, K = p.K;
  const int P = T * K;
  const int GD = D / 32, GF = F / 32;
  const int erows = E + p.has_gate;
  const int G = static_cast<int>(gridDim.x), bid = static_cast<int>(blockIdx.x);
  Signals* sig = reinterpret_cast<Signals*>(p.counters);
  uint32_t* err = p.err;
  const Plan L = make_plan(T, D, F);
  uint4* xf = reinterpret_cast<uint4*>(smem + L.xf_off);
  float4* gred = reinterpret_cast<float4*>(smem + L.gred_off);
  uint8_t* ring = smem + L.ring_off;
  const uint32_t ring_cap = p.smem_bytes - L.ring_off;
  // (callable from any branch: one thread stores, nothing waits)
  auto stamp = [&](int k) {
    if (p.stamps && tid == 0) stamp_at(p.stamps, bid * kStamps + k);
  };
  stamp(0);

  // ---------------- prologue: router rows (input independent) ----------------
  int my_rows = 0;
  for (int r = bid; r < erows && my_rows < 2; r += G) ++my_rows;
  float* rw = reinterpret_cast<float*>(ring);
  // barriers initialised by 48 threads at once; the epoch read by another
  if (tid > 0 && tid <= kMaxGU + kMaxDS) {
    mbar_init(tid <= kMaxGU ? &bar_g[tid - 1] : &bar_d[tid - 1 - kMaxGU], 1);
    fence_mbar_init();  // each initialising thread publishes its own barrier
  }
  if (tid == 64) s_epoch = __ldcg(&sig->epoch[bid]) + 1u;  // this launch's tag
  if (tid == 0) {
    mbar_init(&bar_rw, 1);
    fence_mbar_init();
    if (my_rows > 0) {
      mbar_arrive_expect_tx(&bar_rw, my_rows * D * 4);
      for (int i = 0; i < my_rows; ++i)
        bulk_load(rw + i * D, p.router_rows + static_cast<size_t>(bid + i * G) * D, D * 4,
                  &bar_rw);
    }
    s_failed = 0;
    s_g_issued = 0;
    s_d_issued = 0;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  stamp(1);

  // ---------------- tokens: norm, fp16 fragments ----------------
  const int nchunk = D / 8;
  float xv[TT][8];
  float ss[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) ss[t] = 0.0f;
  const bool has_chunk = tid < nchunk;  // D <= 4096
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    if (has_chunk) {
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
  for (int t = 0; t < TT; ++t) {
    const float v = warp_sum(ss[t]);
    if (lane == 0) s_red[t][warp] = v;
  }
  __syncthreads();
  if (tid < T) {
    float s = 0.0f;
    for (int w = 0; w < kWarps; ++w) s += s_red[tid][w];
    const float inv = p.norm ? rsqrtf(s / static_cast<float>(D) + p.eps) : 1.0f;
    s_inv[tid] = inv;
    if (bid == 0) p.inv_rms[tid] = inv;
  }
  __syncthreads();
  if (has_chunk) {
#pragma unroll
    for (int t = 0; t < TT; ++t) {
      float v[8];
      const float inv = s_inv[t];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = xv[t][j] * inv;
      xf[t * nchunk + tid] = frag_chunk(v);
    }
  }

  // ---------------- router dots, published with the launch tag ----------------
  if (my_rows > 0) {
    const int ok = mbar_wait_inl(&bar_rw, 0, err) ? 1 : 0;
    if (!__syncthreads_and(ok)) {
      if (tid == 0) drain_wait(&bar_rw, 0);
      return;
    }
    float acc[2][TT];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int t = 0; t < TT; ++t) acc[r][t] = 0.0f;
    if (has_chunk) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        if (r < my_rows) {
          const float4 w0 = *reinterpret_cast<const float4*>(rw + r * D + tid * 8);
          const float4 w1 = *reinterpret_cast<const float4*>(rw + r * D + tid * 8 + 4);
          const float wr[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int t = 0; t < TT; ++t)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[r][t] = fmaf(wr[j], xv[t][j], acc[r][t]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        const float v = warp_sum(acc[r][t]);
        if (lane == 0) s_red[r * kMaxTok + t][warp] = v;
      }
    __syncthreads();
    if (tid < 2 * kMaxTok) {
      const int r = tid / kMaxTok, t = tid % kMaxTok;
      if (r < my_rows && t < T) {
        float s = 0.0f;
        for (int w = 0; w < kWarps; ++w) s += s_red[tid][w];
        const unsigned long long word =
            (static_cast<unsigned long long>(s_epoch) << 32) | __float_as_uint(s);
        for (int cp = 0; cp < kLogitCopies; ++cp)
          st_relaxed_u64(p.tlogits + (static_cast<size_t>(cp) * T + t) * (E + 1) + (bid + r * G),
                         word);
      }
    }
  }
  stamp(2);

  // ---------------- selection (every CTA) ----------------
  // warp t < T waits for token t's logits (and its shared-expert gate) and
  // keeps their order keys in shared memory, after the router rows
  uint32_t* s_key = reinterpret_cast<uint32_t*>(ring + 2 * D * 4);  // [T][E]
  bool sel_failed = false;
  if (warp < T) {
    __syncwarp();
    const int t = warp;
    const float inv = s_inv[t];
    const uint32_t tag = s_epoch;
    const unsigned long long* lg =
        p.tlogits + (static_cast<size_t>(bid % kLogitCopies) * T + t) * (E + 1);
    const bool need = p.ids_in == nullptr;
    float lv[8], glv = 0.0f;
    const unsigned long long t0 = global_timer_ns();
    for (uint32_t spin = 0;; ++spin) {
      bool mine = true;
      if (need) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int e = lane + 32 * j;
          lv[j] = 0.0f;
          if (e < E) {
            const unsigned long long w = ld_relaxed_u64(lg + e);
            mine &= static_cast<uint32_t>(w >> 32) == tag;
            lv[j] = __uint_as_float(static_cast<uint32_t>(w));
          }
        }
      }
      if (p.has_gate && lane == 0) {
        const unsigned long long w = ld_relaxed_u64(lg + E);
        mine &= static_cast<uint32_t>(w >> 32) == tag;
        glv = __uint_as_float(static_cast<uint32_t>(w));
      }
      if (__all_sync(0xFFFFFFFFu, mine)) break;
      if ((spin & 7u) == 7u && __any_sync(0xFFFFFFFFu, lane == 0 && poll_give_up(t0, err))) {
        sel_failed = true;
        break;
      }
    }
    if (need) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = lane + 32 * j;
        if (e < E) {
          float sv = lv[j] * inv;
          if (p.logit_bias) sv += __ldg(p.logit_bias + e);
          s_key[t * E + e] = order_key(sv);
        }
      }
    } else {
      for (int k = lane; k < K; k += 32) {
        s_ids[t][k] = static_cast<int>(p.ids_in[t * K + k]);
        s_w[t][k] = p.w_in[t * K + k];
      }
    }
    if (lane == 0 && p.has_gate) s_gate[t] = 1.0f / (1.0f + __expf(-glv * inv));
  }
  if (__syncthreads_or(sel_failed ? 1 : 0)) return;  // nothing in flight
  stamp(3);
  if (p.ids_in == nullptr) {
    // the rank of a logit is the number of logits ordered before it (larger
    // key, or equal key and smaller index: the reference's order and tie
    // rule); ranks below K are the selection, in slot order
    // four lanes per logit, each counting every fourth run of 4 keys; the
    // quad's counts are summed with two shuffles
    const float inv_e = 1.0f / static_cast<float>(E);
    for (int base = warp * 8; base < T * E; base += kWarps * 8) {
      const int q = base + (lane >> 2), part = lane & 3;
      const bool valid = q < T * E;
      const int qq = valid ? q : 0;
      const int t = qdiv(qq, inv_e), e = qq - t * E;
      const uint32_t* row = s_key + t * E;
      const uint32_t ke = row[e];
      int rank = 0;
      for (int e2 = part * 4; e2 < E; e2 += 16) {
        const uint4 k4 = *reinterpret_cast<const uint4*>(row + e2);
        rank += (k4.x > ke || (k4.x == ke && e2 < e)) ? 1 : 0;
        rank += (k4.y > ke || (k4.y == ke && e2 + 1 < e)) ? 1 : 0;
        rank += (k4.z > ke || (k4.z == ke && e2 + 2 < e)) ? 1 : 0;
        rank += (k4.w > ke || (k4.w == ke && e2 + 3 < e)) ? 1 : 0;
      }
      __syncwarp();
      rank += __shfl_xor_sync(0xFFFFFFFFu, rank, 1);
      rank += __shfl_xor_sync(0xFFFFFFFFu, rank, 2);
      if (valid && part == 0 && rank < K) {
        s_ids[t][rank] = e;
        s_sc[t][rank] = key_value(ke);
      }
    }
    __syncthreads();
    if (warp < T) {
      __syncwarp();
      // softmax over the K selected scores (summed in slot order, as the
      // reference does) times the per-expert scale
      const int t = warp;
      const float mx = s_sc[t][0];
      const float ex = lane < K ? expf(s_sc[t][lane] - mx) : 0.0f;
      if (lane < K) s_w[t][lane] = ex;
      __syncwarp();
      if (lane == 0) {
        float sum = 0.0f;
        for (int k = 0; k < K; ++k) sum += s_w[t][k];
        s_red[t][0] = sum;
      }
      __syncwarp();
      if (lane < K) {
        const float gain = p.per_expert_scale ? __ldg(p.per_expert_scale + s_ids[t][lane]) : 1.0f;
        s_w[t][lane] = ex / s_red[t][0] * gain;
      }
    }
  }
  stamp(8);
  __syncthreads();
  stamp(9);
  if (warp == 0) {
    __syncwarp();  // reconverge after the lane-0 work above
    // stable grouping of the P <= 32 token-major pairs: sort (expert, index)
    const bool valid = lane < P;
    const float inv_k = 1.0f / static_cast<float>(K);
    const int lt = qdiv(lane, inv_k);
    const uint32_t e0 = valid ? static_cast<uint32_t>(s_ids[lt][lane - lt * K]) : 0u;
    uint32_t key = valid ? ((e0 << 5) | static_cast<uint32_t>(lane)) : 0xFFFFFFFFu;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1) {
        const uint32_t other = __shfl_xor_sync(0xFFFFFFFFu, key, j);
        const bool up = (lane & k) == 0;
        const bool lower = (lane & j) == 0;
        key = (lower == up) ? umin32(key, other) : (key > other ? key : other);
      }
    }
    const bool v = lane < P;  // sorted: the valid keys come first
    const uint32_t e = key >> 5;
    const int src = static_cast<int>(key & 31u);
    const uint32_t prev = __shfl_up_sync(0xFFFFFFFFu, e, 1);
    const bool first = v && (lane == 0 || prev != e);
    const uint32_t firsts = __ballot_sync(0xFFFFFFFFu, first);
    const uint32_t upto = (2u << lane) - 1u;
    if (v) {
      s_pair_pos[src] = lane;
      const int tt = qdiv(src, inv_k), rr = src - tt * K;
      s_sorted_token[lane] = tt;
      if (first) {
        const int slot = __popc(firsts & upto) - 1;
        const uint32_t later = firsts & ~upto;
        const int nf = later ? __ffs(later) - 1 : P;
        s_slot_expert[slot] = static_cast<int>(e);
        s_slot_start[slot] = lane;
        s_slot_count[slot] = nf - lane;
      }
      if (bid == 0) {
        Pair pr;
        pr.token = static_cast<uint32_t>(tt);
        pr.expert = e;
        pr.rank = static_cast<uint32_t>(rr);
        pr.weight_bits = __half_as_ushort(__float2half_rn(s_w[tt][rr]));
        if (p.pairs_out) p.pairs_out[lane] = pr;
        if (p.ids_out) p.ids_out[src] = e;
        if (p.w_out) p.w_out[src] = s_w[tt][rr];
        if (p.w16_out) p.w16_out[src] = pr.weight_bits;
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
  // (the router rows were read before this barrier; the copies below
  // overwrite them after it, as a pipeline stage is refilled after its
  // release)
  __syncthreads();
  stamp(4);
  const int nslots = s_nslots;

  // ---------------- work of this CTA ----------------
  // gate/up: units of (slot, 8 f rows), slot-major, split evenly over CTAs;
  // down: the CTA owns nb whole 8-row blocks of y over every slot, loaded as
  // units of a slot pair and computed as tiles of (pair, block)
  const int fbk = F / 8, nbk = D / 8;
  const int NG = nslots * fbk;
  const int g0 = (bid * NG) / G, my_gu = ((bid + 1) * NG) / G - g0;
  const int b0 = (bid * nbk) / G, my_nb = ((bid + 1) * nbk) / G - b0;
  // a CTA that owns no block of y (small D) has no down units
  const int npair = my_nb > 0 ? (nslots + 1) / 2 : 0;
  const int rows_h = P + (p.has_shared ? T : 0);
  const int vcols = my_nb * 8;
  const uint32_t sd = down_unit_bytes(my_nb, F);
  int NU = 0, NDS = 0;
  const uint32_t gu_region =
      plan_rings(L.su, sd, ring_cap, my_gu, npair, h_bytes(L, rows_h, vcols), &NU, &NDS);
  uint8_t* dring = ring + gu_region;
  if ((npair > 0 && NDS < 1) || (my_gu > 0 && NU < 1) ||
      gu_region + static_cast<uint32_t>(NDS) * sd > ring_cap) {
    // the host's shape checks rule this out
    if (tid == 0) flag_error(err, TSG_DEVERR_BOUNDS);
    return;  // nothing in flight yet
  }

  Rings R;
  R.ring = ring;
  R.dring = dring;
  R.bar_g = bar_g;
  R.bar_d = bar_d;
  R.slot_expert = s_slot_expert;
  R.g0 = g0;
  R.fbk = fbk;
  R.NU = NU;
  R.NDS = NDS;
  R.b0 = b0;
  R.nb = my_nb;
  R.nslots = nslots;
  R.su = L.su;
  R.sd = sd;

  // ---------------- stream: request every tile the rings can hold ----------------
  // one thread, in the order of use: gate/up units, then down units
  if (tid == 0) {
    for (int i = 0; i < NU; ++i) issue_gu(p, R, i);
    for (int k = 0; k < NDS; ++k) issue_d(p, R, k);
    s_g_issued = NU;
    s_d_issued = NDS;
  }
  __syncwarp();  // warp 0 reconverges before its MMAs
  stamp(10);

  const int g = lane >> 2, c = lane & 3;
  bool failed = false;

  // ---------------- gate/up ----------------
  {
    // this warp's super-groups of 4 groups: [sg0, sg1)
    const int NSG = GD / 4;
    const int sg0 = (warp * NSG) / kWarps, sg1 = ((warp + 1) * NSG) / kWarps;
    const float inv_fbk = 1.0f / static_cast<float>(fbk);
    for (int i = 0; i < my_gu; ++i) {
      const int u = g0 + i, j = qdiv(u, inv_fbk), fb = u - j * fbk;
      const int cnt = s_slot_count[j], start = s_slot_start[j];
      const uint8_t* base = ring + static_cast<uint32_t>(i % NU) * L.su;
      const uint8_t* grow = base + g * (D / 2);           // gate row g
      const uint8_t* urow = base + 4 * D + g * (D / 2);   // up row g
      const __half* gsc = reinterpret_cast<const __half*>(base + 8 * D) + g * GD;
      const __half* usc = reinterpret_cast<const __half*>(base + 8 * D + D / 2) + g * GD;
      const bool ok = mbar_wait_inl(&bar_g[i % NU], static_cast<uint32_t>(i / NU) & 1u, err);
      if (i < 5) stamp(20 + i);
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (ok) {
        const bool bvalid = g < cnt;
        const uint4* xrow = xf + (bvalid ? s_sorted_token[start + g] : 0) * nchunk;
        for (int sg = sg0; sg < sg1; ++sg) {
          const int grp = 4 * sg + c;
          const uint4 ra = *reinterpret_cast<const uint4*>(grow + grp * 16);
          const uint4 rb = *reinterpret_cast<const uint4*>(urow + grp * 16);
          __half2 sa, sa16, sb, sb16;
          scale_pair(gsc + grp, &sa, &sa16);
          scale_pair(usc + grp, &sb, &sb16);
          uint4 bx[4];
#pragma unroll
          for (int wi = 0; wi < 4; ++wi)
            bx[wi] = bvalid ? xrow[4 * grp + wi] : make_uint4(0u, 0u, 0u, 0u);
          mma_supergroup(acc, ra, rb, sa, sa16, sb, sb16, bx);
        }
      }
      gred[((i & 1) * kWarps + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      if (!__syncthreads_and(ok ? 1 : 0)) {
        failed = true;
        break;
      }
      if (i < 5) stamp(25 + i);
      // every warp is past slot i % NU: refill it
      if (tid == 0 && i + NU < my_gu) {
        issue_gu(p, R, i + NU);
        s_g_issued = i + NU + 1;
      }
      __syncwarp();
      if (warp == (i & (kWarps - 1))) {
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          const float4 q4 = gred[((i & 1) * kWarps + w) * 32 + lane];
          v[0] += q4.x;
          v[1] += q4.y;
          v[2] += q4.z;
          v[3] += q4.w;
        }
        // rows g: gate f = 8 fb + g (v0, v1), up (v2, v3); columns 2c, 2c+1.
        // Gather the 8 act values of each column to one lane via shuffles.
        const float a0 = gate_act_fast(p.act, v[0]) * v[2];
        const float a1 = gate_act_fast(p.act, v[1]) * v[3];
        float col[8];
        const int src_c = (lane & 7) >> 1;  // lane n < 8 collects column n
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
          const float s0 = __shfl_sync(0xFFFFFFFFu, a0, gg * 4 + src_c);
          const float s1 = __shfl_sync(0xFFFFFFFFu, a1, gg * 4 + src_c);
          col[gg] = (lane & 1) ? s1 : s0;
        }
        if (lane < cnt) p.hfrag[static_cast<size_t>(start + lane) * fbk + fb] = frag_chunk(col);
        __syncwarp();
      }
    }
  }
  stamp(5);

  // ---------------- all act rows of the grid ----------------
  // this CTA's act rows are written; the barrier orders them before the
  // release store of thread 0 (a release covers what its thread has
  // observed); then wait for every other CTA's flag
  if (!__syncthreads_or(failed ? 1 : 0)) {
    if (tid == 0) {
      // one counter per launch parity: (epoch & 1) selects it, and the
      // other one is reset for the next launch by this launch's last CTA
      uint32_t* ctr = &sig->gcount[s_epoch & 1u];
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
      stamp(18);
      const unsigned long long t0 = global_timer_ns();
      bool ok = true;
      for (uint32_t spin = 0; ld_relaxed_u32(ctr) < static_cast<uint32_t>(G); ++spin)
        if ((spin & 63u) == 63u && poll_give_up(t0, err)) {
          ok = false;
          break;
        }
      __threadfence();
      s_ok = ok ? 1 : 0;
      if (ok && bid == 0) sig->gcount[(s_epoch & 1u) ^ 1u] = 0u;
    }
    __syncthreads();
    failed = s_ok == 0;
  } else {
    failed = true;
  }
  stamp(6);

  // ---------------- down + combine ----------------
  if (!failed) {
    // stage the act rows (all slots) in the gate/up region
    uint4* hs = reinterpret_cast<uint4*>(ring);
    float* vs = reinterpret_cast<float*>(ring + h_v_off(L, rows_h));
    const int hs_row = static_cast<int>(L.hstride / 16);
    const float inv_fbk = 1.0f / static_cast<float>(fbk);
    for (int q = tid; q < rows_h * fbk; q += kThreads) {
      const int row = qdiv(q, inv_fbk), c8 = q - row * fbk;
      hs[row * hs_row + c8] = __ldcg(p.hfrag + static_cast<size_t>(row) * fbk + c8);
    }
    __syncthreads();
    stamp(12);
    const int NSGF = (GF + 3) / 4;
    const uint32_t cb = static_cast<uint32_t>(4 * F * my_nb);
    const uint32_t sbytes = static_cast<uint32_t>(F / 2 * my_nb);
    const float inv_nb = 1.0f / static_cast<float>(my_nb > 0 ? my_nb : 1);
    // rounds of NDS down units; all warps take the round's tiles
    for (int r0u = 0; r0u < npair; r0u += NDS) {
      const int nu_r = npair - r0u < NDS ? npair - r0u : NDS;
      const uint32_t par = static_cast<uint32_t>(r0u / NDS) & 1u;
      for (int tile = warp; tile < nu_r * my_nb; tile += kWarps) {
        const int ul = qdiv(tile, inv_nb), bi = tile - ul * my_nb;
        const int pp = r0u + ul;
        const int ja = 2 * pp, jb = ja + 1;
        const int ca = s_slot_count[ja], sa0 = s_slot_start[ja];
        const int cbn = jb < nslots ? s_slot_count[jb] : 0;
        const int sb0 = jb < nslots ? s_slot_start[jb] : 0;
        // column n of the tile: act row of slot a (n < ca), of slot b, or none
        auto col_row = [&](int n) { return n < ca ? sa0 + n : (n < ca + cbn ? sb0 + n - ca : -1); };
        const uint8_t* seg = dring + static_cast<uint32_t>(pp % NDS) * sd;
        const int rowi = bi * 8 + g;
        const uint8_t* arow = seg + rowi * (F / 2);        // slot a, row g of block bi
        const uint8_t* brow = seg + cb + rowi * (F / 2);   // slot b
        const __half* sca = reinterpret_cast<const __half*>(seg + 2 * cb) + rowi * GF;
        const __half* scb = reinterpret_cast<const __half*>(seg + 2 * cb + sbytes) + rowi * GF;
        const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_d[pp % NDS], par, err));
        if (!ok) {
          failed = true;
          break;
        }
        const int rg = col_row(g), r0 = col_row(2 * c), r1 = col_row(2 * c + 1);
        const uint4* hrow = hs + (rg >= 0 ? rg : 0) * hs_row;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int sg = 0; sg < NSGF; ++sg) {
          const int grp = 4 * sg + c;
          const bool gv = grp < GF;
          const int gq = gv ? grp : 0;
          const uint4 ra = *reinterpret_cast<const uint4*>(arow + gq * 16);
          const uint4 rb = *reinterpret_cast<const uint4*>(brow + gq * 16);
          __half2 sa, sa16, sb, sb16;
          scale_pair(sca + gq, &sa, &sa16);
          scale_pair(scb + gq, &sb, &sb16);
          if (!gv) sa = sa16 = sb = sb16 = __floats2half2_rn(0.0f, 0.0f);
          uint4 bx[4];
#pragma unroll
          for (int wi = 0; wi < 4; ++wi)
            bx[wi] = (rg >= 0 && gv) ? hrow[4 * grp + wi] : make_uint4(0u, 0u, 0u, 0u);
          mma_supergroup(acc, ra, rb, sa, sa16, sb, sb16, bx);
        }
        // rows g of slot a pair with columns n < ca, rows g of slot b
        // (tile rows 8 + g) with columns ca <= n < ca + cb
        if (r0 >= 0) vs[r0 * vcols + rowi] = 2 * c < ca ? acc[0] : acc[2];
        if (r1 >= 0) vs[r1 * vcols + rowi] = 2 * c + 1 < ca ? acc[1] : acc[3];
      }
      // the round's units are consumed: refill their slots with the next round
      if (__syncthreads_or(failed ? 1 : 0)) {
        failed = true;
        break;
      }
      if (tid == 0) {
        for (int k = r0u + NDS; k < r0u + 2 * NDS && k < npair; ++k) issue_d(p, R, k);
        s_d_issued = min(npair, r0u + 2 * NDS);
      }
      __syncwarp();
    }
    stamp(13);
    if (!failed && vcols > 0) {
      // y = residual + gate * shared + sum over ranks (ascending) w * v
      const float inv_v = 1.0f / static_cast<float>(vcols);
      for (int q = tid; q < T * vcols; q += kThreads) {
        const int t = qdiv(q, inv_v), dl = q - t * vcols;
        const int d = b0 * 8 + dl;
        float y = p.residual ? p.residual[static_cast<size_t>(t) * D + d] : 0.0f;
        if (p.has_shared) {
          const float sv = vs[(P + t) * vcols + dl];
          y = p.has_gate ? fmaf(s_gate[t], sv, y) : y + sv;
        }
        for (int rr = 0; rr < K; ++rr) y = fmaf(s_w[t][rr], vs[s_pair_pos[t * K + rr] * vcols + dl], y);
        if (p.y_f32)
          reinterpret_cast<float*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] = y;
        else
          reinterpret_cast<__nv_bfloat16*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] =
              __float2bfloat16_rn(y);
      }
    }
  }
  if (failed && lane == 0) atomicOr(&s_failed, 1);
  __syncthreads();
  stamp(7);
  if (tid == 0) {
    if (s_failed) {
      // let this CTA's own copies land before it exits
      drain_rings(R, s_g_issued, s_d_issued);
      return;  // the host clears the signals after reading the error word
    }
    sig->epoch[bid] = s_epoch;  // read by this CTA's next launch
  }
}

size_t fused_smem_limit() {
  static size_t limit = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    const void* kernels[4] = {reinterpret_cast<const void*>(decode_fused_kernel<1>),
                              reinterpret_cast<const void*>(decode_fused_kernel<2>),
                              reinterpret_cast<const void*>(decode_fused_kernel<3>),
                              reinterpret_cast<const void*>(decode_fused_kernel<4>)};
    size_t lim = ~static_cast<size_t>(0);
    for (const void* k : kernels) {
      if (allow_max_smem_ptr(k) != cudaSuccess) return;
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) return;
      lim = std::min(lim, static_cast<size_t>(fa.maxDynamicSharedSizeBytes));
    }
    limit = lim;
  });
  return limit;
}

}  // namespace

bool decode_fused_supported(int T, int K, int E, int has_gate, int num_sms) {
  return T >= 1 && T <= kMaxTok && T * K <= kMaxPairs && K <= kMaxK && E <= 256 &&
         E % 4 == 0 && E + has_gate <= 2 * num_sms && num_sms <= kMaxCtas;
}

// Whether every CTA's rings can be planned for this shape (checked for the
// largest number of distinct experts) within the kernel's shared memory.
bool decode_fused_fits(int T, int D, int F, int K, int has_shared, int num_sms) {
  if (D % 256 || F % 64 || D > 4096 || F > 1024 || D / 8 > kThreads) return false;
  const size_t smem = fused_smem_limit();
  const Plan L = make_plan(T, D, F);
  if (smem < L.ring_off + 1024u) return false;
  const uint32_t cap = static_cast<uint32_t>(smem) - L.ring_off;
  const int rows_h = T * K + (has_shared ? T : 0);
  const int my_nb = (D / 8 + num_sms - 1) / num_sms;
  // router rows and order keys live in the ring before it is planned
  if (2u * static_cast<uint32_t>(D) * 4u + static_cast<uint32_t>(T) * 256u * 4u > cap) return false;
  for (int P = K; P <= T * K; ++P) {
    const int nslots = P + (has_shared ? 1 : 0);
    const int my_gu = (nslots * (F / 8) + num_sms - 1) / num_sms;
    const uint32_t sd = down_unit_bytes(my_nb, F);
    int NU = 0, NDS = 0;
    const uint32_t region = plan_rings(L.su, sd, cap, my_gu, (nslots + 1) / 2,
                                       h_bytes(L, rows_h, my_nb * 8), &NU, &NDS);
    if (NU < 1 || NDS < 1 || region + static_cast<uint32_t>(NDS) * sd > cap) return false;
  }
  return true;
}

cudaError_t launch_decode_fused(const DecodeFusedArgs& a, cudaStream_t s) {
  if (!decode_fused_supported(a.T, a.K, a.E, a.has_gate, a.num_sms) ||
      !decode_fused_fits(a.T, a.D, a.F, a.K, a.has_shared, a.num_sms))
    return cudaErrorInvalidValue;
  const size_t smem = fused_smem_limit();
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
  p.tlogits = static_cast<unsigned long long*>(a.logits);
  p.inv_rms = a.inv_rms;
  p.hfrag = reinterpret_cast<uint4*>(a.actfrag);
  p.counters = a.counters;
  p.ids_out = a.ids_out;
  p.w_out = a.w_out;
  p.w16_out = a.w16_out;
  p.pairs_out = a.pairs_out;
  p.err = a.err;
  p.stamps = a.stamps;
  p.smem_bytes = static_cast<uint32_t>(smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = a.cooperative ? 1 : 0;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = a.allow_pdl ? 1 : 0;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  switch (a.T) {
    case 1: return cudaLaunchKernelEx(&cfg, decode_fused_kernel<1>, p);
    case 2: return cudaLaunchKernelEx(&cfg, decode_fused_kernel<2>, p);
    case 3: return cudaLaunchKernelEx(&cfg, decode_fused_kernel<3>, p);
    default: return cudaLaunchKernelEx(&cfg, decode_fused_kernel<4>, p);
  }
}

}  // namespace tsg
