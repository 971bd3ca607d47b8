// decode_stream.cu -- the whole MoE block for a decode batch (T <= 4 tokens)
// in one persistent cooperative kernel that streams every selected weight
// byte once, in one phase, with compute following the stream.
//
// Reference behaviour, per layer (RealForwardRunner.swift:3079-3330,
// QwenForwardRunner.swift:1460-1612): router GEMV + top-K select
// (MoE.encodeRouterGemma4BF16, moe.metal:187-329), routed phase 1 gate/up +
// activation (moe.metal:455-574), phase 2 down + weighted reduce in slot
// order (moe.metal:651-687), and for Qwen the sigmoid-gated shared expert
// added to that reduce.
//
// One CTA per SM (16 warps).  After the router and the selection (every CTA
// ranks all logits itself), the work of the layer is laid out as one byte
// sequence, slot by slot (a slot is a distinct selected expert with its
// tokens, plus the shared expert), and inside a slot chunk by chunk (64 f):
//
//   [8 gate/up blocks of the chunk: 8 gate + the same 8 up rows each]
//   [the chunk's down slice: D rows x 64 f, as D/16 blocks of 16 rows]
//
// and every CTA takes one contiguous, equal share of the bytes.  A CTA first
// runs its gate/up blocks, then its down blocks; the acts a down block needs
// come from the gate/up blocks just before it in the sequence (its own, or
// the previous CTA's, which that CTA also runs first), published through
// global memory with a per-block flag.  Every down block writes its partial
// sums over its 64 f to global memory; after one grid barrier each CTA adds
// the partials of its share of y in a fixed order and applies the combine:
// y = residual + gate * shared + sum over ranks (ascending) w * v.
//
// Weight tiles reach shared memory through a ring of equal stages, all
// requested as early as the ring allows: gate/up rows by 1-D bulk copies into
// rows padded by 16 bytes (conflict-free ldmatrix), down slices by TMA boxes
// with a 32-byte swizzle (conflict-free ldmatrix), down scales by 4-byte
// cp.async.  The stage a warp releases last is refilled by that warp.
//
// Arithmetic: each MMA (mma.sync m16n8k16, fp32 accumulate) covers one
// 32-wide scale group of 16 weight rows, so the group's scale is applied
// after the MMA, in fp32, and the int4 codes enter the tensor core
// unscaled.  A code word (elements e0..e7, e_2i in the low nibble of byte i)
// gives four fp16 pairs with one AND each: (w & 0x000F000F) holds q0, q4 as
// the fp16 subnormals q * 2^-24, (w & 0x00F000F0) holds q1, q5 as q * 2^-20,
// the same masks on w >> 8 give q2, q6 and q3, q7.  The token (or act)
// operand carries the matching order and a factor 16 on the 2^-24 elements,
// so every product is q * x * 2^-20 exactly; the accumulator starts at
// -8 * 2^-20 * sum(x) of the group, so it ends at 2^-20 * sum((q - 8) x).
// The scale multiplies that sum, and 2^20 is applied once per output.
//
// Warps reconverge (__syncwarp) after code that only some lanes run and
// before warp-collective code.  Every wait is bounded (one second); on an
// error a CTA waits, again bounded, for its own copies in flight before it
// exits, and the host clears the cross-CTA signals.
#include <algorithm>

#include "int4_mma.cuh"
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kWarps = 15;                  // compute warps
constexpr int kAllWarps = kWarps + 1;       // + the reduction and refill warp (16 x 32 threads
                                            // keep 128 registers per thread)
constexpr int kThreads = 32 * kAllWarps;
constexpr int kMaxTok = 4;
constexpr int kMaxPairs = 32;
constexpr int kMaxSlots = kMaxPairs + 1;
constexpr int kMaxK = 32;
constexpr int kMaxStages = 96;   // stages of one CTA's share
constexpr int kMaxRing = 12;     // ring slots
constexpr int kMaxCtas = 256;
constexpr int kLogitCopies = 4;
constexpr int kStamps = 96;
constexpr int kDownBox = 128;    // rows of the large down box (8 blocks of 16)
constexpr float kTwo20 = 1048576.0f;
// A down tile's K may be split over several work units, their partials
// added in unit order; the same split in every regime (T = 1 waves, rows
// owned), so that one token's down rows come out of the same arithmetic
// either way.  One unit per tile (the whole K) measured fastest: 47.7k
// layer-tokens/s against 46.8k with two parts, 46.2k with three and 45.5k
// with four (Gemma-like, T = 1, the same box).
constexpr int kParts = 1;

// Cross-CTA signalling (same scheme as the earlier fused decode kernel):
// per-CTA launch epochs, the grid counter of each launch parity.
struct Signals {
  uint32_t epoch[kMaxCtas];
  uint32_t gcount[2];
  uint32_t pad[kMaxCtas - 2];
};

struct StreamParams {
  DecodeMaps maps;  // down-slice tensor maps (first: 64-byte aligned)
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
  unsigned long long* hact;     // [slots][T][F / 8][4] act fragments, (tag << 32 | half2) words
  uint32_t* gdone;              // [grid] launch tag once a CTA's acts are all published
  float* partial;               // [slots][F / 64][T][D] down partial sums (x 2^-20)
  uint32_t* counters;           // Signals
  uint32_t* ids_out;            // [T][K]
  float* w_out;                 // [T][K]
  uint16_t* w16_out;            // [T][K] or nullptr
  Pair* pairs_out;              // [P] sorted pairs
  uint32_t* err;
  unsigned long long* stamps;   // debug: [grid][kStamps] timestamps, or nullptr
  uint32_t smem_bytes;          // dynamic shared memory of the launch
  int ring_slots;               // stages in the ring (host-planned)
};

__host__ __device__ inline uint32_t align_up_u32(uint32_t x, uint32_t a) {
  return (x + a - 1u) / a * a;
}

// Shared-memory plan, the same on host and device.
struct Plan {
  uint32_t xf_off;     // token fragments [T][D / 8] uint4
  uint32_t ci_off;     // accumulator starts [T][D / 32] float
  uint32_t red_off;    // gate/up partials [ring][16 warps][red_words] float
  uint32_t ring_off;   // stages, 1024-aligned
  uint32_t rs;         // bytes of one gate (or up) box: 8 rows x D/2, swizzled
  uint32_t sb;         // stage bytes
  uint32_t sd;         // down blocks (16 rows) per down stage
  uint32_t red_words;  // floats one warp leaves per gate/up block
  // T <= 2 ("rows of y owned"): the acts of every slot, their accumulator
  // starts, and the CTA's down results, all in shared memory
  uint32_t act_off;    // [slots][T][F / 8] uint4 act fragments
  uint32_t ast_off;    // [slots][F / 32][T] float accumulator starts
  uint32_t sv_off;     // [slots][T][16 nt] float down results of the CTA's rows
  // T = 1 router-routed ("waves"): the CTA's rows of every slot's down matrix
  // in one region (the down results in sv_off)
  uint32_t down_off;   // [slots][drb] down codes then scales of the CTA's rows
  uint32_t drb;        // bytes per slot
  uint32_t nrmax;      // rows of y a CTA owns at most (multiple of 4)
  uint32_t total;      // bytes of the whole plan for `ring` stages
};

// Whether the CTAs own rows of y (T <= 2: every slot's acts fit in shared
// memory, so a CTA computes whole down rows and combines them itself).
__host__ __device__ inline bool rows_owned(int T) { return T <= 2; }

__host__ __device__ inline uint32_t red_words_for(int T) {
  // lanes with c < ceil(T / 2) hold the valid columns; T = 1 keeps d0 and d2
  return T == 1 ? 16u : (T == 2 ? 32u : 64u);
}

__host__ __device__ inline Plan make_plan(int T, int D, int F, int K, int G, int ring,
                                          bool waves = false) {
  Plan L;
  uint32_t o = 0;
  L.xf_off = o;
  o += static_cast<uint32_t>(T * (D / 8) * 16);
  L.ci_off = o;
  o += static_cast<uint32_t>(T * (D / 32) * 4);
  o = align_up_u32(o, 16);
  L.red_off = o;
  L.red_words = red_words_for(T);
  o += static_cast<uint32_t>(ring) * kWarps * L.red_words * 4u;
  L.act_off = L.ast_off = L.sv_off = L.down_off = o;
  L.drb = L.nrmax = 0;
  if (waves) {
    const uint32_t slots = static_cast<uint32_t>(K + 1);
    L.nrmax = 4u * static_cast<uint32_t>((D / 4 + G - 1) / G);
    o = align_up_u32(o, 16);
    L.sv_off = o;
    o += kParts * slots * 32u * 4u;
    L.down_off = o;
    L.drb = align_up_u32(L.nrmax * static_cast<uint32_t>(F / 2 + F / 16), 16);
    // (rows past a slot's own, read by a partial last tile, stay inside)
    o += slots * L.drb + 16u * static_cast<uint32_t>(F / 2 + F / 16);
  } else if (rows_owned(T)) {
    const uint32_t slots = static_cast<uint32_t>(T * K + 1);
    const uint32_t ntmax = static_cast<uint32_t>((D / 16 + G - 1) / G);
    o = align_up_u32(o, 16);
    L.act_off = o;
    o += slots * static_cast<uint32_t>(T * (F / 8)) * 16u;
    L.ast_off = o;
    o += slots * static_cast<uint32_t>((F / 32) * T) * 4u;
    L.sv_off = o;
    o += kParts * slots * static_cast<uint32_t>(T) * 16u * ntmax * 4u;
  }
  L.ring_off = align_up_u32(o, 1024);
  L.rs = static_cast<uint32_t>(4 * D);  // bytes of one 8-row code box
  const uint32_t gu = 2u * L.rs + 2u * 8u * static_cast<uint32_t>(D / 16);
  L.sb = align_up_u32(gu, 1024);
  L.sd = L.sb / 512u;       // down blocks: 16 rows x 32 code bytes
  if (L.sd > 3u * kWarps) L.sd = 3u * kWarps;  // at most 3 per compute warp
  L.total = L.ring_off + static_cast<uint32_t>(ring) * L.sb;
  return L;
}

// Stage descriptor: kind (0 gate/up block, 1 down blocks), slot, chunk, and
// the gate/up block in the chunk or the first down block and their count.
// With rows owned, a down stage is `chunk` consecutive slots from `slot`,
// each with the down rows of 16-row tiles [a, a + n) of y.
struct Stage {
  uint16_t kind_slot;  // kind << 8 | slot
  uint16_t chunk;
  uint16_t a;          // gate/up: block 0..7; down: first block of 16 rows
  uint16_t n;          // down: blocks; gate/up: 1
};

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
TSG_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// mma.sync m16n8k16 fp16 x fp16 + C -> fp32, with a separate C operand.
// Not volatile: the MMAs have no side effects, so the compiler may interleave
// independent accumulation chains instead of issuing each dependent pair
// back to back.
TSG_DEV void mma_16816_c(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                         uint32_t b0, uint32_t b1, float c0, float c1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%10,%11};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1));
}
TSG_DEV void mma_16816_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                           uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The four unscaled fp16 pairs of a code word (see the file header):
// p[0] = (q0, q4) * 2^-24, p[1] = (q2, q6) * 2^-24,
// p[2] = (q1, q5) * 2^-20, p[3] = (q3, q7) * 2^-20.
TSG_DEV void split_word(uint32_t w, uint32_t (&p)[4]) {
  const uint32_t w8 = w >> 8;
  p[0] = w & 0x000F000Fu;
  p[1] = w8 & 0x000F000Fu;
  p[2] = w & 0x00F000F0u;
  p[3] = w8 & 0x00F000F0u;
}

// One scale group of 16 rows: the rows' code words ra (row g) and rb (row
// g + 8), the token fragment bx (x0 x4 | x2 x6 | x1 x5 | x3 x7, the first two
// pairs times 16) and the accumulator start (c0, c1) of columns 2c, 2c + 1.
TSG_DEV void mma_group(float (&d)[4], uint32_t ra, uint32_t rb, const uint4& bx, float c0,
                       float c1) {
  uint32_t pa[4], pb[4];
  split_word(ra, pa);
  split_word(rb, pb);
  mma_16816_c(d, pa[0], pb[0], pa[1], pb[1], bx.x, bx.y, c0, c1);
  mma_16816_acc(d, pa[2], pb[2], pa[3], pb[3], bx.z, bx.w);
}

// Eight consecutive values as the operand chunk of the unscaled scheme:
// [(16 v0, 16 v4), (16 v2, 16 v6), (v1, v5), (v3, v7)] in fp16; `sum`
// returns the sum of the eight fp16 values (unscaled), in a fixed order.
TSG_DEV uint4 op_chunk(const float (&v)[8], float* sum) {
  __half h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(v[i]);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += __half2float(h[i]);
  *sum = s;
  const __half k16 = __float2half_rn(16.0f);
  return make_uint4(h2_bits(__halves2half2(__hmul(h[0], k16), __hmul(h[4], k16))),
                    h2_bits(__halves2half2(__hmul(h[2], k16), __hmul(h[6], k16))),
                    h2_bits(__halves2half2(h[1], h[5])), h2_bits(__halves2half2(h[3], h[7])));
}

TSG_DEV float2 h2_to_f2(uint32_t u) { return __half22float2(bits_h2(u)); }


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
TSG_DEV void st_relaxed_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
TSG_DEV uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// a / b for small non-negative ints (a < 2^16, b <= 4096).
TSG_DEV int qdiv(int a, float inv_b) {
  return __float2int_rz((static_cast<float>(a) + 0.5f) * inv_b);
}

// Phase time stamps (the "debug_phase_stamps" option) exist only in a build
// with TSG_PHASE_STAMPS=1 (TSG_NVCC_DEFINES="-DTSG_PHASE_STAMPS=1" for the
// package build); otherwise their code is not in the kernel, which is
// measurably faster without it (the kernel's one-pass code runs from a cold
// instruction cache).
#ifndef TSG_PHASE_STAMPS
#define TSG_PHASE_STAMPS 0
#endif
constexpr bool kPhaseStamps = TSG_PHASE_STAMPS != 0;
TSG_DEV void stamp_at(unsigned long long* stamps, int idx) {
  if (kPhaseStamps) stamps[idx] = global_timer_ns();
}

// Bounded wait on an mbarrier phase that ignores the error word: used only
// to let this CTA's own copies land before it exits after an error.
__device__ __noinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_timer_ns() - t0 > kWaitLimitNs) return;
}

// Bounded mbarrier wait with the spin loop inline.
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

// ---------------------------------------------------------------------------
// the work plan: two phases, each cut into equal shares
// ---------------------------------------------------------------------------
// Phase 1: the gate/up blocks of every slot (slot-major, 8 f each), split
// evenly over the CTAs.  Phase 2: the down blocks (16 rows x 64 f), in
// (slot, chunk, row block) order, split evenly over the CTAs.  A CTA requests
// its phase-1 tiles, then its phase-2 tiles, so the grid's gate/up bytes
// arrive first; by the time the down tiles have landed, the acts they need
// (from any CTA) are published.
struct Work {
  uint32_t nslots, nc, nd;  // slots, 64-f chunks per slot, 16-row blocks per chunk
  uint32_t ng, ndt;         // gate/up blocks, down blocks of the layer
  bool rows_owned;          // T <= 2: phase 2 is whole rows of y per CTA
  uint32_t sb, tile_bytes;  // stage bytes; one slot's 16 down rows (codes + scales)
};

TSG_DEV Work make_work(int nslots, int D, int F, int T, uint32_t sb) {
  Work w;
  w.rows_owned = rows_owned(T);
  w.sb = sb;
  w.tile_bytes = 16u * static_cast<uint32_t>(F / 2 + F / 16);
  w.nslots = static_cast<uint32_t>(nslots);
  w.nc = static_cast<uint32_t>(F / 64);
  w.nd = static_cast<uint32_t>(D / 16);
  w.ng = w.nslots * static_cast<uint32_t>(F / 8);
  w.ndt = w.nslots * w.nc * w.nd;
  return w;
}

// This CTA's stages: its gate/up blocks, then its down blocks in stages of at
// most sd blocks of one chunk.  Returns the count (or -1 above kMaxStages).
TSG_DEV int build_stages(const Work& w, int bid, int G, uint32_t sd, Stage* st,
                        bool waves = false) {
  int n = 0;
  if (waves) {
    // gate/up blocks dealt round-robin: block i to CTA i mod G, so that the
    // k-th stages of all CTAs form one wave and each slot's acts complete
    // early, slot by slot; the down rows are not staged in the ring
    const uint32_t f8 = w.nc * 8;
    for (uint32_t b = static_cast<uint32_t>(bid); b < w.ng; b += static_cast<uint32_t>(G)) {
      if (n >= kMaxStages) return -1;
      const uint32_t slot = b / f8, rb = b - slot * f8;
      st[n].kind_slot = static_cast<uint16_t>(slot);
      st[n].chunk = static_cast<uint16_t>(rb >> 3);
      st[n].a = static_cast<uint16_t>(rb & 7u);
      st[n].n = 1;
      ++n;
    }
    return n;
  }
  const uint32_t ub = static_cast<uint32_t>(bid), ug = static_cast<uint32_t>(G);
  const uint32_t g0 = (w.ng * ub) / ug, g1 = (w.ng * (ub + 1)) / ug;
  const uint32_t f8 = w.nc * 8;
  for (uint32_t b = g0; b < g1; ++b) {
    if (n >= kMaxStages) return -1;
    const uint32_t slot = b / f8, rb = b - slot * f8;
    st[n].kind_slot = static_cast<uint16_t>(slot);
    st[n].chunk = static_cast<uint16_t>(rb >> 3);
    st[n].a = static_cast<uint16_t>(rb & 7u);
    st[n].n = 1;
    ++n;
  }
  if (w.rows_owned) {
    // the CTA's 16-row tiles of y [t0, t1), every slot's down rows of them,
    // as many slots per stage as fit
    const uint32_t t0 = (w.nd * ub) / ug, t1 = (w.nd * (ub + 1)) / ug, nt = t1 - t0;
    if (nt == 0) return n;
    uint32_t per = w.sb / (nt * w.tile_bytes);
    if (per > 32u) per = 32u;  // one issuing lane per slot
    for (uint32_t slot = 0; slot < w.nslots; slot += per) {
      if (n >= kMaxStages || per == 0) return -1;
      st[n].kind_slot = static_cast<uint16_t>((1u << 8) | slot);
      st[n].chunk = static_cast<uint16_t>(w.nslots - slot < per ? w.nslots - slot : per);
      st[n].a = static_cast<uint16_t>(t0);
      st[n].n = static_cast<uint16_t>(nt);
      ++n;
    }
    return n;
  }
  const uint32_t d0 = (w.ndt * ub) / ug, d1 = (w.ndt * (ub + 1)) / ug;
  for (uint32_t k = d0; k < d1;) {
    if (n >= kMaxStages) return -1;
    const uint32_t sc = k / w.nd, kb = k - sc * w.nd;  // (slot, chunk), first block
    uint32_t cnt = w.nd - kb;
    if (cnt > d1 - k) cnt = d1 - k;
    if (cnt > sd) cnt = sd;
    const uint32_t slot = sc / w.nc;
    st[n].kind_slot = static_cast<uint16_t>((1u << 8) | slot);
    st[n].chunk = static_cast<uint16_t>(sc - slot * w.nc);
    st[n].a = static_cast<uint16_t>(kb);
    st[n].n = static_cast<uint16_t>(cnt);
    ++n;
    k += cnt;
  }
  return n;
}

TSG_DEV const uint8_t* slot_blob(const StreamParams& p, int e, const ExpertOffsets** off) {
  if (e < 0) {
    *off = &p.experts.shared_off;
    return p.experts.shared;
  }
  *off = &p.experts.off;
  return p.experts.base + static_cast<uint64_t>(e) * p.experts.stride;
}

TSG_DEV void tma_load_3d_bar(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                             int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

TSG_DEV void tma_load_4d_bar(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int32_t c0,
                             int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Issues the copies of one stage into ring slot `dst` (warp-collective, all
// 32 lanes, converged).  The slot's barrier expects one arrival per phase,
// lane 0's expect-tx.  A down stage's scales are not copied: the warps that
// compute its blocks load them directly.
__device__ __noinline__ void issue_stage(const StreamParams& p, const Plan& L, const Stage& sg, const int* slot_expert,
                         uint8_t* dst, uint64_t* bar, int lane) {
  const int D = p.D, F = p.F;
  const int slot = sg.kind_slot & 0xFF;
  const bool down = (sg.kind_slot >> 8) != 0;
  const int e = slot_expert[slot];
  const ExpertOffsets* off;
  const uint8_t* blob = slot_blob(p, e, &off);
  if (!down) {
    const int f0 = 64 * sg.chunk + 8 * sg.a;
    const uint32_t sbytes = static_cast<uint32_t>(D / 16);
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, 2u * L.rs + 16u * sbytes);
      const uint32_t base = smem_u32(dst);
      const int z = e < 0 ? 0 : e;
      tma_load_4d_bar(base, e < 0 ? &p.maps.sgate8 : &p.maps.gate8, bar, 0, f0, 0, z);
      tma_load_4d_bar(base + L.rs, e < 0 ? &p.maps.sup8 : &p.maps.up8, bar, 0, f0, 0, z);
      bulk_load(dst + 2u * L.rs, blob + off->gate_s + static_cast<size_t>(f0) * sbytes,
                8u * sbytes, bar);
      bulk_load(dst + 2u * L.rs + 8u * sbytes, blob + off->up_s + static_cast<size_t>(f0) * sbytes,
                8u * sbytes, bar);
    }
  } else if (rows_owned(p.T)) {
    // `chunk` slots, each: down codes of rows [16 a, 16 (a + n)) (contiguous),
    // then their scales (contiguous)
    const int nsl = sg.chunk, nt = sg.n;
    const uint32_t cb = 16u * nt * static_cast<uint32_t>(F / 2);
    const uint32_t sbytes = 16u * nt * static_cast<uint32_t>(F / 16);
    if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nsl) * (cb + sbytes));
    __syncwarp();
    if (lane < nsl) {
      const ExpertOffsets* o2;
      const uint8_t* b2 = slot_blob(p, slot_expert[slot + lane], &o2);
      const size_t r0 = 16u * static_cast<size_t>(sg.a);
      bulk_load(dst + static_cast<uint32_t>(lane) * (cb + sbytes), b2 + o2->down_w + r0 * (F / 2), cb,
                bar);
      bulk_load(dst + static_cast<uint32_t>(lane) * (cb + sbytes) + cb,
                b2 + o2->down_s + r0 * (F / 16), sbytes, bar);
    }
  } else {
    const int n = sg.n, nbig = n / 8;
    const int r0 = 16 * sg.a;
    const CUtensorMap* mbig = e < 0 ? &p.maps.sdown128 : &p.maps.down128;
    const CUtensorMap* msmall = e < 0 ? &p.maps.sdown16 : &p.maps.down16;
    const int z = e < 0 ? 0 : e;
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, static_cast<uint32_t>(n) * 512u);
      const uint32_t base = smem_u32(dst);
      for (int b = 0; b < nbig; ++b)
        tma_load_3d_bar(base + static_cast<uint32_t>(b) * 4096u, mbig, bar, 32 * sg.chunk,
                        r0 + b * kDownBox, z);
      for (int b = nbig * 8; b < n; ++b)
        tma_load_3d_bar(base + static_cast<uint32_t>(b) * 512u, msmall, bar, 32 * sg.chunk,
                        r0 + 16 * b, z);
    }
  }
  __syncwarp();
}

// The sum of one group's 32 acts from its four operand chunks (words 0, 1 of
// a chunk hold 16x values), as a balanced tree over the 16 words: the order
// a 16-lane butterfly of shuffles gives, so that the waves regime (which sums
// across lanes) and the rows-owned regime (which sums in one thread) agree
// bit for bit.
TSG_DEV float group_act_sum(const uint4* fr) {
  float a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 u = fr[i];
    const float2 h0 = h2_to_f2(u.x), h1 = h2_to_f2(u.y);
    const float2 h2 = h2_to_f2(u.z), h3 = h2_to_f2(u.w);
    a[i] = ((h0.x + h0.y) * 0.0625f + (h1.x + h1.y) * 0.0625f) + ((h2.x + h2.y) + (h3.x + h3.y));
  }
  return (a[0] + a[1]) + (a[2] + a[3]);
}

// ---------------------------------------------------------------------------
// waves (one router-routed token): the down units of the CTA's rows of y,
// kept out of line (each runs a few times per launch; the gate/up loop keeps
// the instruction cache)
// ---------------------------------------------------------------------------
struct WaveRows {
  const uint8_t* down;  // [slots][drb]: the rows' down codes, then their scales
  uint32_t drb;
  float* sv;            // [kParts][K + 1][32] the rows' down partials
  int F, K, nr;         // nr rows (in at most two 16-row tiles)
};

// One down unit of slot j -- 16-row tile t, K part kp (of kParts) -- from the
// slot's acts in shared memory (act: [slots][F / 8] operand chunks, ast:
// [slots][F / 32] accumulator starts), the arithmetic of the rows-owned
// regime for one token.
__device__ __noinline__ void wave_unit(const WaveRows& w, int j, int t, int kp, const uint4* act,
                                       const float* ast, int lane) {
  const int F = w.F, GF = F / 32, NP2 = F / 64;
  const int g = lane >> 2, c = lane & 3, m = lane >> 3, r8 = lane & 7;
  const int p0 = (kp * NP2) / kParts, p1 = ((kp + 1) * NP2) / kParts;
  const uint8_t* dj = w.down + static_cast<uint32_t>(j) * w.drb;
  const __half* scs =
      reinterpret_cast<const __half*>(dj + static_cast<uint32_t>(w.nr) * (F / 2)) + 16 * t * GF;
  const uint32_t rowaddr = smem_u32(dj) + static_cast<uint32_t>(16 * t + r8 + 8 * (m & 1)) * (F / 2) +
                           static_cast<uint32_t>(m >> 1) * 16u;
  const uint4* af = act + static_cast<size_t>(j) * (F / 8) + c;
  const float* as = ast + static_cast<size_t>(j) * GF;
  float acc0 = 0.0f, acc2 = 0.0f;
  // (unrolled: the pairs' MMAs overlap; the sums stay in pair order)
#pragma unroll 4
  for (int pr = p0; pr < p1; ++pr) {
    uint32_t q0, q1, q2, q3;
    ldsm_x4(rowaddr + static_cast<uint32_t>(pr) * 32u, q0, q1, q2, q3);
    const uint4 b0 = g == 0 ? af[8 * pr] : make_uint4(0u, 0u, 0u, 0u);  // one token: column 0
    const uint4 b1 = g == 0 ? af[8 * pr + 4] : make_uint4(0u, 0u, 0u, 0u);
    const float c00 = c == 0 ? as[2 * pr] : 0.0f;
    const float c10 = c == 0 ? as[2 * pr + 1] : 0.0f;
    float d0[4], d1[4];
    mma_group(d0, q0, q1, b0, c00, 0.0f);
    mma_group(d1, q2, q3, b1, c10, 0.0f);
    const float2 sr = h2_to_f2(*reinterpret_cast<const uint32_t*>(scs + g * GF + 2 * pr));
    const float2 sh = h2_to_f2(*reinterpret_cast<const uint32_t*>(scs + (g + 8) * GF + 2 * pr));
    acc0 = fmaf(sr.y, d1[0], fmaf(sr.x, d0[0], acc0));
    acc2 = fmaf(sh.y, d1[2], fmaf(sh.x, d0[2], acc2));
  }
  if (c == 0) {
    float* o = w.sv + (static_cast<size_t>(kp) * (w.K + 1) + j) * 32 + 16 * t;
    o[g] = acc0;
    o[g + 8] = acc2;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int TT, bool WV>
__global__ void __launch_bounds__(kThreads, 1)
    decode_stream_kernel(const __grid_constant__ StreamParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar_rw;
  __shared__ __align__(8) uint64_t bar_st[kMaxRing];
  __shared__ __align__(8) uint64_t bar_rel[kMaxRing];
  __shared__ __align__(8) uint64_t bar_act, bar_act2;  // compute warps, once per launch
  __shared__ __align__(8) uint64_t bar_go;              // warp 0: every CTA's acts are out
  __shared__ __align__(8) uint64_t bar_down;             // waves: the CTA's down rows have landed
  __shared__ __align__(8) uint64_t bar_ld[kMaxSlots];    // waves: a slot's act words have landed
  __shared__ __align__(8) uint64_t bar_slot[kMaxSlots];  // waves: a slot's acts are unpacked
  __shared__ int s_issued[kMaxRing];
  __shared__ Stage s_stage[kMaxStages];
  __shared__ int s_ids[kMaxTok][kMaxK];
  __shared__ float s_w[kMaxTok][kMaxK];
  __shared__ float s_sc[kMaxTok][kMaxK];
  __shared__ int s_slot_expert[kMaxSlots], s_slot_start[kMaxSlots], s_slot_count[kMaxSlots];
  __shared__ int s_sorted_token[kMaxPairs + kMaxTok];
  __shared__ int s_pair_pos[kMaxPairs];
  __shared__ int s_pos_slot[kMaxPairs + kMaxTok], s_pos_col[kMaxPairs + kMaxTok];
  __shared__ float s_inv[kMaxTok], s_gate[kMaxTok];
  __shared__ float s_red[2 * kMaxTok][kAllWarps];
  __shared__ int s_nslots, s_nst, s_failed, s_down_issued;
  __shared__ uint32_t s_epoch;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int T = TT;
  const int D = p.D, F = p.F, E = p.E, K = p.K;
  const int P = T * K;
  const int GD = D / 32;
  const int erows = E + p.has_gate;
  const int G = static_cast<int>(gridDim.x), bid = static_cast<int>(blockIdx.x);
  const int NS = p.ring_slots;
  // one router-selected token: slots follow the ranks, so the weight copies
  // can start as soon as the ranks are known (before softmax and grouping)
  const bool fast1 = WV || (TT == 1 && p.ids_in == nullptr);
  Signals* sig = reinterpret_cast<Signals*>(p.counters);
  uint32_t* err = p.err;
  // one router-selected token: the gate/up blocks go out in waves and the
  // down rows of each slot are done as soon as the slot's acts are out
  constexpr bool waves = WV;
  const Plan L = make_plan(T, D, F, K, G, NS, waves);
  uint4* xf = reinterpret_cast<uint4*>(smem + L.xf_off);
  float* cinit = reinterpret_cast<float*>(smem + L.ci_off);
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  uint8_t* ring = smem + L.ring_off;
  auto stamp = [&](int k) {
    if (kPhaseStamps && p.stamps && tid == 0) stamp_at(p.stamps, bid * kStamps + k);
  };
  stamp(0);
  // with programmatic launch, the next layer's grid may be launched now: its
  // CTAs take each SM as this launch's CTA there exits, and wait
  // (griddepcontrol.wait) for this whole grid before reading what it wrote
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---------------- prologue: router rows (input independent) ----------------
  int my_rows = 0;
  for (int r = bid; r < erows && my_rows < 2; r += G) ++my_rows;
  float* rw = reinterpret_cast<float*>(ring);
  if (tid >= 32 && tid < 32 + kMaxRing) {
    mbar_init(&bar_st[tid - 32], 1);
    mbar_init(&bar_rel[tid - 32], kWarps);  // every compute warp releases each stage
    fence_mbar_init();
    s_issued[tid - 32] = 0;
  }
  if (tid >= 128 && tid < 128 + kMaxSlots) {
    mbar_init(&bar_ld[tid - 128], 1);
    mbar_init(&bar_slot[tid - 128], 1);
    fence_mbar_init();
  }
  if (tid == 96) {
    mbar_init(&bar_down, 1);
    mbar_init(&bar_act, kWarps);
    mbar_init(&bar_act2, kWarps);
    mbar_init(&bar_go, 1);
    fence_mbar_init();
  }
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
    s_down_issued = 0;
    s_nslots = 0;
    if (fast1) {
      // one token routed by this kernel: K distinct experts in rank order
      // (slot j = rank j), then the shared expert
      s_nslots = K + p.has_shared;
      if (p.has_shared) s_slot_expert[K] = -1;
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // this launch's tag, read after the previous launch has finished (with
  // programmatic launch this CTA may start before that launch's CTA of the
  // same index has written it)
  if (tid == 64) s_epoch = __ldcg(&sig->epoch[bid]) + 1u;
  stamp(1);

  // ---------------- tokens: norm, operand fragments, accumulator starts ----------------
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
    for (int w = 0; w < kAllWarps; ++w) s += s_red[tid][w];
    const float inv = p.norm ? rsqrtf(s / static_cast<float>(D) + p.eps) : 1.0f;
    s_inv[tid] = inv;
    if (bid == 0) p.inv_rms[tid] = inv;
  }
  __syncthreads();
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    float v[8];
    const float inv = s_inv[t];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = xv[t][j] * inv;
    float gs = 0.0f;
    const uint4 ch = op_chunk(v, &gs);
    if (has_chunk) xf[t * nchunk + tid] = ch;
    // the 4 chunks of a 32-wide group are 4 consecutive lanes
    gs += __shfl_xor_sync(0xFFFFFFFFu, gs, 1);
    gs += __shfl_xor_sync(0xFFFFFFFFu, gs, 2);
    if (has_chunk && (tid & 3) == 0) cinit[t * GD + (tid >> 2)] = -8.0f / kTwo20 * gs;
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
        for (int w = 0; w < kAllWarps; ++w) s += s_red[tid][w];
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
      __nanosleep(64);  // keep the L2 free for the other CTAs' words
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
  if (fast1 && warp == kWarps && lane == 0) {
    // the share of one token's layer does not depend on the input: plan it
    // while warp 0 waits for the logits
    const int n =
        build_stages(make_work(K + p.has_shared, D, F, T, L.sb), bid, G, L.sd, s_stage, waves);
    s_nst = n;
    if (n < 0) flag_error(err, TSG_DEVERR_BOUNDS);  // the host's shape checks rule this out
  }
  if (__syncthreads_or(sel_failed ? 1 : 0)) return;  // nothing in flight
  stamp(3);
  if (p.ids_in == nullptr) {
    // the rank of a logit is the number of logits ordered before it (larger
    // key, or equal key and smaller index: the reference's order and tie
    // rule); ranks below K are the selection, in slot order.  Four lanes per
    // logit, each counting every fourth run of 4 keys.
    const float inv_e = 1.0f / static_cast<float>(E);
    for (int base = warp * 8; base < T * E; base += kAllWarps * 8) {
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
        if (fast1) s_slot_expert[rank] = e;
      }
    }
    __syncthreads();
    if (fast1 && s_nst >= 0) {
      // (the order keys and router rows in the ring are read no more)
      for (int s = warp; s < s_nst && s < NS; s += kAllWarps) {
        issue_stage(p, L, s_stage[s], s_slot_expert, ring + static_cast<uint32_t>(s) * L.sb,
                    &bar_st[s], lane);
        if (lane == 0) s_issued[s] = 1;
      }
      if (waves && warp == kWarps) {
        // the CTA's rows of every slot's down matrix, codes then scales, one
        // region for the whole launch (requested after the first gate/up tiles)
        const int r0 = 4 * ((bid * (D / 4)) / G), nr = 4 * (((bid + 1) * (D / 4)) / G) - r0;
        const int ns1 = K + p.has_shared;
        const uint32_t cb = static_cast<uint32_t>(nr) * static_cast<uint32_t>(F / 2);
        const uint32_t sbytes = static_cast<uint32_t>(nr) * static_cast<uint32_t>(F / 16);
        if (lane == 0) {
          if (nr > 0)
            mbar_arrive_expect_tx(&bar_down, static_cast<uint32_t>(ns1) * (cb + sbytes));
          else
            mbar_arrive(&bar_down);
        }
        __syncwarp();
        if (nr > 0)
          for (int j = lane; j < ns1; j += 32) {
            const ExpertOffsets* o2;
            const uint8_t* b2 = slot_blob(p, s_slot_expert[j], &o2);
            uint8_t* dst = smem + L.down_off + static_cast<uint32_t>(j) * L.drb;
            bulk_load(dst, b2 + o2->down_w + static_cast<size_t>(r0) * (F / 2), cb, &bar_down);
            bulk_load(dst + cb, b2 + o2->down_s + static_cast<size_t>(r0) * (F / 16), sbytes,
                      &bar_down);
          }
        __syncwarp();
        if (lane == 0) s_down_issued = 1;
      }
      stamp(10);
    }
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
  __syncthreads();
  stamp(8);
  if (warp == 0) {
    __syncwarp();
    // stable grouping of the P <= 32 token-major pairs: sort (expert, index)
    const bool valid = lane < P;
    const float inv_k = 1.0f / static_cast<float>(K);
    const int lt = qdiv(lane, inv_k);
    const uint32_t e0 = valid ? static_cast<uint32_t>(s_ids[lt][lane - lt * K]) : 0u;
    // caller routing is validated before any weight address is formed
    const bool bad = valid && e0 >= static_cast<uint32_t>(E);
    if (__any_sync(0xFFFFFFFFu, bad)) {
      if (bad && atomicCAS(err + 1, 0u, 8u) == 0u) err[2] = e0;  // "expert out of range"
      if (lane == 0) {
        flag_error(err, TSG_DEVERR_METADATA);
        s_nslots = -1;
      }
    }
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
      const int slot = __popc(firsts & upto) - 1;
      const uint32_t at_or_before = firsts & upto;
      const int start = 31 - __clz(static_cast<int>(at_or_before));
      if (!fast1) {
        s_pos_slot[lane] = slot;
        s_pos_col[lane] = lane - start;
      }
      if (first && !fast1) {
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
    __syncwarp();
    if (lane == 0 && s_nslots >= 0 && !fast1) {
      int u = __popc(firsts);
      if (p.has_shared) {
        s_slot_expert[u] = -1;
        s_slot_start[u] = P;
        s_slot_count[u] = T;
        for (int t = 0; t < T; ++t) {
          s_sorted_token[P + t] = t;
          s_pos_slot[P + t] = u;
          s_pos_col[P + t] = t;
        }
        ++u;
      }
      s_nslots = u;
    }
  }
  __syncthreads();
  stamp(4);

  // ---------------- the CTA's share of the layer's bytes ----------------
  const int nslots = s_nslots;
  if (nslots < 0) return;  // invalid caller routing: nothing in flight
  if (!fast1) {
    if (tid == 0) {
      const int n = build_stages(make_work(nslots, D, F, T, L.sb), bid, G, L.sd, s_stage);
      s_nst = n;
      if (n < 0) flag_error(err, TSG_DEVERR_BOUNDS);  // the host's shape checks rule this out
    }
    __syncthreads();
    if (s_nst >= 0) {
      // (the router rows and order keys were read before the barrier above;
      // the copies below overwrite them) warp w requests stage w of the
      // first ring fill
      for (int s = warp; s < s_nst && s < NS; s += kAllWarps) {
        issue_stage(p, L, s_stage[s], s_slot_expert, ring + static_cast<uint32_t>(s) * L.sb,
                    &bar_st[s], lane);
        if (lane == 0) s_issued[s] = 1;
      }
    }
    stamp(10);
  }
  const int nst = s_nst;
  if (nst < 0) return;  // nothing in flight

  const int g = lane >> 2, c = lane & 3;
  const int NP = D / 64;   // pairs of scale groups along D
  const int F8 = F / 8, NC = F / 64;
  const uint32_t tag = s_epoch;
  // this warp's pairs of the gate/up K dimension: pr = warp + 15 k; the token
  // operand (column g = token g) and accumulator starts stay in registers
  uint4 bx[3][2];
  float cin[3][2][2];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int pr = warp + kWarps * k;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int grp = 2 * pr + h;
      const bool ok = pr < NP;
      bx[k][h] = (ok && g < T) ? xf[g * nchunk + 4 * grp + c] : make_uint4(0u, 0u, 0u, 0u);
      cin[k][h][0] = (ok && 2 * c < T) ? cinit[(2 * c) * GD + grp] : 0.0f;
      cin[k][h][1] = (ok && 2 * c + 1 < T) ? cinit[(2 * c + 1) * GD + grp] : 0.0f;
    }
  }
  const int m = lane >> 3, r8 = lane & 7;
  bool failed = false;
  // ---- waves (T = 1): the CTA's rows of y, slot by slot ----
  // Once its gate/up stages are done, the reduction warp bulk-loads every
  // slot's tagged act words into the (then free) ring, checks the tags
  // (loading again a slot with a word not out yet), unpacks the acts and
  // their accumulator starts next to them and releases the slot; every warp
  // (the reduction warp too, once its copies are requested) has at most one
  // down unit per slot (unit u of slot j goes to warp (j U + u) mod 16) and
  // runs it from shared memory once the slot is in.
  const int wr0 = 4 * ((bid * (D / 4)) / G);
  const int wnr = 4 * (((bid + 1) * (D / 4)) / G) - wr0;
  const int wU = ((wnr + 15) / 16) * kParts;
  // this thread's row of the residual, read long before the combine
  const float wres = waves && p.residual && tid < wnr ? p.residual[wr0 + tid] : 0.0f;
  float* sv_w = reinterpret_cast<float*>(smem + L.sv_off);
  WaveRows wrow;
  wrow.down = smem + L.down_off;
  wrow.drb = L.drb;
  wrow.sv = sv_w;
  wrow.F = F;
  wrow.K = K;
  wrow.nr = wnr;
  // the ring after the gate/up stages: [slots][F / 2] tagged words, then the
  // acts [slots][F / 8] uint4, then their accumulator starts [slots][F / 32]
  const uint32_t wstg_bytes = static_cast<uint32_t>(K + 1) * static_cast<uint32_t>(F) * 4u;
  unsigned long long* wstg = reinterpret_cast<unsigned long long*>(ring);
  uint4* wact = reinterpret_cast<uint4*>(ring + wstg_bytes);
  float* wast = reinterpret_cast<float*>(ring + wstg_bytes + static_cast<uint32_t>(K + 1) * F * 2u);
  const int GF = F / 32;
  uint4* afr = reinterpret_cast<uint4*>(smem + L.act_off);
  float* ast = reinterpret_cast<float*>(smem + L.ast_off);
  float* sv = reinterpret_cast<float*>(smem + L.sv_off);
  // acts of the last (slot, chunk) a down stage used, kept for the next one
  int act_key = -1;
  uint4 ba[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
  float cs0[2] = {0.0f, 0.0f}, cs1[2] = {0.0f, 0.0f};

  if (warp < kWarps) {
  for (int s = 0; s < nst && !failed; ++s) {
    const Stage sg = s_stage[s];
    const int rs = s % NS;
    uint8_t* base = ring + static_cast<uint32_t>(rs) * L.sb;
    const uint32_t sbase = smem_u32(base);
    const uint32_t par = static_cast<uint32_t>(s / NS) & 1u;
    const int slot = sg.kind_slot & 0xFF;
    const bool down = (sg.kind_slot >> 8) != 0;
    float* rd = red + static_cast<uint32_t>(rs) * kWarps * L.red_words;
    if (!down) {
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_st[rs], par, err))) {
        failed = true;
        break;
      }
      if (s < 8) stamp(24 + s);  // debug: warp 0 sees stage s's data
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      // box layout [D/256 chunks of 128 bytes][8 rows][128 bytes], the 16-byte
      // unit u of (row r, chunk) at ((u ^ r) << 4): matrix m reads the gate
      // (m even) or up (m odd) box, group 2 pr + (m >> 1)
      const uint32_t boxaddr = sbase + static_cast<uint32_t>(m & 1) * L.rs +
                               static_cast<uint32_t>(r8) * 128u;
      const __half* gsc = reinterpret_cast<const __half*>(base + 2u * L.rs);
      const __half* usc = gsc + 8 * GD;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int pr = warp + kWarps * k;
        if (pr < NP) {
          const uint32_t j = static_cast<uint32_t>(2 * pr + (m >> 1));
          uint32_t q0, q1, q2, q3;
          ldsm_x4(boxaddr + (j >> 3) * 1024u + (((j & 7u) ^ static_cast<uint32_t>(r8)) << 4), q0,
                  q1, q2, q3);
          float d0[4], d1[4];
          mma_group(d0, q0, q1, bx[k][0], cin[k][0][0], cin[k][0][1]);
          mma_group(d1, q2, q3, bx[k][1], cin[k][1][0], cin[k][1][1]);
          const float2 sgv = h2_to_f2(*reinterpret_cast<const uint32_t*>(gsc + g * GD + 2 * pr));
          const float2 suv = h2_to_f2(*reinterpret_cast<const uint32_t*>(usc + g * GD + 2 * pr));
          acc[0] = fmaf(sgv.x, d0[0], acc[0]);
          acc[1] = fmaf(sgv.x, d0[1], acc[1]);
          acc[2] = fmaf(suv.x, d0[2], acc[2]);
          acc[3] = fmaf(suv.x, d0[3], acc[3]);
          acc[0] = fmaf(sgv.y, d1[0], acc[0]);
          acc[1] = fmaf(sgv.y, d1[1], acc[1]);
          acc[2] = fmaf(suv.y, d1[2], acc[2]);
          acc[3] = fmaf(suv.y, d1[3], acc[3]);
        }
      }
      // this warp's partial sums of the block's valid columns
      float* mine = rd + warp * L.red_words;
      if (T == 1) {
        if (c == 0) { mine[2 * g] = acc[0]; mine[2 * g + 1] = acc[2]; }
      } else if (T == 2) {
        if (c == 0) *reinterpret_cast<float4*>(mine + 4 * g) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      } else {
        if (c < 2)
          *reinterpret_cast<float4*>(mine + 4 * (2 * g + c)) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      }
    } else if (!waves && rows_owned(T)) {
      // ---- (reached once, at the first down stage) ----
      // every slot's acts into shared memory: warp 0 first waits until every
      // CTA has flagged its gate/up blocks published, so that the tagged
      // words are read about once instead of polled by every thread (the tags
      // stay the proof: a word that is not there yet is read again)
      if (warp == 0) {
        const unsigned long long t0 = global_timer_ns();
        for (uint32_t spin = 0;; ++spin) {
          bool all = true;
          for (int i = lane; i < G; i += 32) all &= ld_relaxed_u32(p.gdone + i) == tag;
          if (__all_sync(0xFFFFFFFFu, all)) break;
          if ((spin & 15u) == 15u &&
              __any_sync(0xFFFFFFFFu, lane == 0 && poll_give_up(t0, err))) {
            failed = true;
            break;
          }
          __nanosleep(100);
        }
        if (lane == 0) mbar_arrive(&bar_go);
      }
      if (failed || !__all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_go, 0, err))) {
        failed = true;
        break;
      }
      stamp(9);  // debug: every CTA's acts seen out
      // the tagged words, coalesced (one word per lane, eight in flight per
      // thread), then the accumulator start of each (slot, token, group):
      // -8 * 2^-20 * sum of its 32 acts
      {
        const int nw = nslots * T * F8 * 4;
        uint32_t* a32 = reinterpret_cast<uint32_t*>(afr);
        const int ct = warp * 32 + lane;
        for (int w0 = ct; w0 < nw && !failed; w0 += 8 * kWarps * 32) {
          unsigned long long wv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int w = w0 + u * kWarps * 32;
            wv[u] = w < nw ? ld_relaxed_u64(p.hact + w) : (static_cast<unsigned long long>(tag) << 32);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int w = w0 + u * kWarps * 32;
            if (w >= nw) continue;
            const unsigned long long t0 = global_timer_ns();
            for (uint32_t spin = 0; static_cast<uint32_t>(wv[u] >> 32) != tag; ++spin) {
              if ((spin & 15u) == 15u && poll_give_up(t0, err)) {
                failed = true;
                break;
              }
              __nanosleep(128);
              wv[u] = ld_relaxed_u64(p.hact + w);
            }
            a32[w] = static_cast<uint32_t>(wv[u]);
          }
        }
      }
      failed = __any_sync(0xFFFFFFFFu, failed);
      if (failed) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_act);
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_act, 0, err))) {
        failed = true;
        break;
      }
      {
        const int na = nslots * T * GF;
        for (int q = warp * 32 + lane; q < na; q += kWarps * 32) {
          const int st_ = q / GF, grp = q - st_ * GF;  // st_ = slot * T + t
          const uint4* fr = afr + static_cast<size_t>(st_) * F8 + 4 * grp;
          const int sl = st_ / T, t = st_ - sl * T;
          ast[(static_cast<size_t>(sl) * GF + grp) * T + t] = -8.0f / kTwo20 * group_act_sum(fr);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_act2);
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_act2, 0, err))) {
        failed = true;
        break;
      }
      stamp(22);  // debug: acts loaded
      // ---- down work units: (slot k of a stage, 16-row tile j, part kp of
      // the K = F pairs); with every down stage resident in the ring at once
      // (the host checks it), the units of all of them are spread over the
      // warps together; else stage by stage ----
      const int NP2 = F / 64;
      const bool together = (nst - s) <= NS;
      int ubase = 0;
      int dbg_units = 0;
      for (int s2 = s; s2 < nst && !failed; ++s2) {
        const Stage sg2 = s_stage[s2];
        const int rs2 = s2 % NS;
        const uint8_t* base2 = ring + static_cast<uint32_t>(rs2) * L.sb;
        const uint32_t par2 = static_cast<uint32_t>(s2 / NS) & 1u;
        const int slot2 = sg2.kind_slot & 0xFF;
        const int nsl = sg2.chunk, nt = sg2.n, RWS = 16 * nt;
        const int nunits = nsl * nt * kParts;
        const uint32_t cb = 16u * nt * static_cast<uint32_t>(F / 2);
        const uint32_t sbb = cb + 16u * nt * static_cast<uint32_t>(F / 16);
        int first = together ? ((warp - ubase) % kWarps + kWarps) % kWarps : warp;
        if (first < nunits &&
            !__all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_st[rs2], par2, err))) {
          failed = true;
          break;
        }
        if (s2 == s) stamp(21);  // debug: warp 0 starts its down units
        for (int u = first; u < nunits; u += kWarps) {
          const int item = u / kParts, kp = u - item * kParts;
          const int k = item / nt, j = item - k * nt, sl = slot2 + k;
          const int p0 = (kp * NP2) / kParts, p1 = ((kp + 1) * NP2) / kParts;
          const uint32_t rowaddr = smem_u32(base2) + static_cast<uint32_t>(k) * sbb +
                                   static_cast<uint32_t>(16 * j + r8 + 8 * (m & 1)) * (F / 2) +
                                   static_cast<uint32_t>(m >> 1) * 16u;
          const __half* scs =
              reinterpret_cast<const __half*>(base2 + static_cast<uint32_t>(k) * sbb + cb) + 16 * j * GF;
          const uint4* af = afr + (static_cast<size_t>(sl) * T + (g < T ? g : 0)) * F8 + c;
          const float* as = ast + static_cast<size_t>(sl) * GF * T;
          float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
          for (int pr = p0; pr < p1; ++pr) {
            uint32_t q0, q1, q2, q3;
            ldsm_x4(rowaddr + static_cast<uint32_t>(pr) * 32u, q0, q1, q2, q3);
            const uint4 b0 = g < T ? af[8 * pr] : make_uint4(0u, 0u, 0u, 0u);
            const uint4 b1 = g < T ? af[8 * pr + 4] : make_uint4(0u, 0u, 0u, 0u);
            const float c00 = 2 * c < T ? as[(2 * pr) * T + 2 * c] : 0.0f;
            const float c01 = 2 * c + 1 < T ? as[(2 * pr) * T + 2 * c + 1] : 0.0f;
            const float c10 = 2 * c < T ? as[(2 * pr + 1) * T + 2 * c] : 0.0f;
            const float c11 = 2 * c + 1 < T ? as[(2 * pr + 1) * T + 2 * c + 1] : 0.0f;
            float d0[4], d1[4];
            mma_group(d0, q0, q1, b0, c00, c01);
            mma_group(d1, q2, q3, b1, c10, c11);
            const float2 sr = h2_to_f2(*reinterpret_cast<const uint32_t*>(scs + g * GF + 2 * pr));
            const float2 sh =
                h2_to_f2(*reinterpret_cast<const uint32_t*>(scs + (g + 8) * GF + 2 * pr));
            acc[0] = fmaf(sr.y, d1[0], fmaf(sr.x, d0[0], acc[0]));
            acc[1] = fmaf(sr.y, d1[1], fmaf(sr.x, d0[1], acc[1]));
            acc[2] = fmaf(sh.y, d1[2], fmaf(sh.x, d0[2], acc[2]));
            acc[3] = fmaf(sh.y, d1[3], fmaf(sh.x, d0[3], acc[3]));
          }
          float* svs = sv + (static_cast<size_t>(kp) * nslots + sl) * T * RWS + 16 * j;
          if (2 * c < T) {
            svs[(2 * c) * RWS + g] = acc[0];
            svs[(2 * c) * RWS + g + 8] = acc[2];
          }
          if (2 * c + 1 < T) {
            svs[(2 * c + 1) * RWS + g] = acc[1];
            svs[(2 * c + 1) * RWS + g + 8] = acc[3];
          }
          if (dbg_units < 2) stamp(19 + dbg_units);  // debug: warp 0's first units
          ++dbg_units;
        }
        ubase += nunits;
        if (!together) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar_rel[rs2]);
        }
      }
      if (failed) break;
      stamp(23);  // debug: warp 0's down units done
      if (together)
        for (int s2 = s; s2 < nst; ++s2) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar_rel[s2 % NS]);
        }
      break;  // every remaining stage is done and released
    } else {
      // this warp's blocks of the stage: k = warp + 15 j (at most 3); their
      // down scales (groups 2 ch, 2 ch + 1 of rows g and g + 8) are loaded
      // from global memory first, so their latency overlaps the act poll
      const int ch = sg.chunk;
      const int e = s_slot_expert[slot];
      const uint8_t* dsc = (e < 0 ? p.experts.shared + p.experts.shared_off.down_s
                                  : p.experts.base + static_cast<uint64_t>(e) * p.experts.stride +
                                        p.experts.off.down_s) + 4 * ch;
      uint32_t sreg[3][2];
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const int k = warp + kWarps * j;
        const int row = 16 * (sg.a + (k < sg.n ? k : 0)) + g;
        sreg[j][0] = __ldg(reinterpret_cast<const uint32_t*>(dsc + static_cast<size_t>(row) * (F / 16)));
        sreg[j][1] = __ldg(reinterpret_cast<const uint32_t*>(dsc + static_cast<size_t>(row + 8) * (F / 16)));
      }
      // the acts of the chunk for column g (token g): tagged words, polled
      // until every word carries this launch's tag
      const int key = slot * NC + ch;
      if (key != act_key) {
        act_key = key;
        const unsigned long long* src =
            p.hact + ((static_cast<size_t>(slot) * T + (g < T ? g : 0)) * F8 + 8 * ch + c) * 4;
        const unsigned long long t0 = global_timer_ns();
        for (uint32_t spin = 0;; ++spin) {
          bool ready = true;
          if (g < T) {
            unsigned long long wv[2][4];
#pragma unroll
            for (int gi = 0; gi < 2; ++gi)
#pragma unroll
              for (int j = 0; j < 4; ++j) wv[gi][j] = ld_relaxed_u64(src + 16 * gi + j);
#pragma unroll
            for (int gi = 0; gi < 2; ++gi)
#pragma unroll
              for (int j = 0; j < 4; ++j) ready &= static_cast<uint32_t>(wv[gi][j] >> 32) == tag;
            ba[0] = make_uint4(static_cast<uint32_t>(wv[0][0]), static_cast<uint32_t>(wv[0][1]),
                               static_cast<uint32_t>(wv[0][2]), static_cast<uint32_t>(wv[0][3]));
            ba[1] = make_uint4(static_cast<uint32_t>(wv[1][0]), static_cast<uint32_t>(wv[1][1]),
                               static_cast<uint32_t>(wv[1][2]), static_cast<uint32_t>(wv[1][3]));
          }
          if (__all_sync(0xFFFFFFFFu, ready)) break;
          if ((spin & 15u) == 15u &&
              __any_sync(0xFFFFFFFFu, lane == 0 && poll_give_up(t0, err))) {
            failed = true;
            break;
          }
          __nanosleep(256);  // the acts come from other SMs' gate/up phase
        }
        if (failed) break;
        // accumulator starts: -8 * 2^-20 * (sum of the group's 32 acts) of
        // columns 2c and 2c + 1, from the fragments (quad g holds column g)
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
          const float2 h0 = h2_to_f2(ba[gi].x), h1 = h2_to_f2(ba[gi].y);
          const float2 h2 = h2_to_f2(ba[gi].z), h3 = h2_to_f2(ba[gi].w);
          float sm = ((h0.x + h0.y) + (h1.x + h1.y)) * 0.0625f + ((h2.x + h2.y) + (h3.x + h3.y));
          sm += __shfl_xor_sync(0xFFFFFFFFu, sm, 1);
          sm += __shfl_xor_sync(0xFFFFFFFFu, sm, 2);
          cs0[gi] = -8.0f / kTwo20 * __shfl_sync(0xFFFFFFFFu, sm, 8 * c);
          cs1[gi] = -8.0f / kTwo20 * __shfl_sync(0xFFFFFFFFu, sm, 8 * c + 4);
        }
      }
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_st[rs], par, err))) {
        failed = true;
        break;
      }
      if (s < 8) stamp(24 + s);  // debug: warp 0 sees stage s's data (and acts)
      float* pbase = p.partial + static_cast<size_t>(slot) * T * D * NC + ch;
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const int k = warp + kWarps * j;
        if (k < sg.n) {
          const int rb = 16 * k + 8 * (m & 1) + r8;
          const uint32_t addr =
              sbase + static_cast<uint32_t>(rb) * 32u +
              ((static_cast<uint32_t>(m >> 1) ^ ((static_cast<uint32_t>(rb) >> 2) & 1u)) << 4);
          uint32_t q0, q1, q2, q3;
          ldsm_x4(addr, q0, q1, q2, q3);
          float d0[4], d1[4];
          mma_group(d0, q0, q1, ba[0], cs0[0], cs1[0]);
          mma_group(d1, q2, q3, ba[1], cs0[1], cs1[1]);
          const float2 sa = h2_to_f2(sreg[j][0]);
          const float2 sb = h2_to_f2(sreg[j][1]);
          const int d = 16 * (sg.a + k) + g;
          if (2 * c < T) {
            float* o = pbase + (static_cast<size_t>(2 * c) * D + d) * NC;
            o[0] = fmaf(sa.y, d1[0], sa.x * d0[0]);
            o[8 * NC] = fmaf(sb.y, d1[2], sb.x * d0[2]);
          }
          if (2 * c + 1 < T) {
            float* o = pbase + (static_cast<size_t>(2 * c + 1) * D + d) * NC;
            o[0] = fmaf(sa.y, d1[1], sa.x * d0[1]);
            o[8 * NC] = fmaf(sb.y, d1[3], sb.x * d0[3]);
          }
        }
      }
    }
    if (s < 7) stamp(12 + s);  // debug: warp 0 done with stage s
    // release the stage to the reduction warp (which refills its ring slot)
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_rel[rs]);
  }
  if (waves && !failed) {
    // 1. the slots this warp brings in (j = warp, warp + 15, ...): once the
    // reduction warp's copy of a slot's tagged act words has landed, every
    // word must carry this launch's tag (else the slot is copied again);
    // then its acts and accumulator starts (in the order the rows-owned
    // regime sums them) are unpacked next to the words and the slot is
    // released
    const uint32_t sbytes = static_cast<uint32_t>(F) * 4u;  // F / 2 words
    for (int j = warp; j < nslots && !failed; j += kWarps) {
      uint32_t par = 0;
      const unsigned long long t0 = global_timer_ns();
      for (;;) {
        if (!__all_sync(0xFFFFFFFFu, mbar_wait_inl(&bar_ld[j], par, err))) {
          failed = true;
          break;
        }
        par ^= 1u;
        if (kPhaseStamps && lane == 0 && p.stamps && j < 8) stamp_at(p.stamps, bid * kStamps + 48 + j);  // debug
        const unsigned long long* wv = wstg + static_cast<size_t>(j) * (F / 2);
        bool ok = true;
        for (int w = lane; w < F / 2; w += 32) ok &= static_cast<uint32_t>(wv[w] >> 32) == tag;
        if (__all_sync(0xFFFFFFFFu, ok)) break;
        if (__any_sync(0xFFFFFFFFu, lane == 0 && poll_give_up(t0, err))) {
          failed = true;
          break;
        }
        fence_async_shared();  // (this warp's reads of the copy come first)
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_ld[j], sbytes);
          bulk_load(wstg + static_cast<size_t>(j) * (F / 2), p.hact + static_cast<size_t>(j) * (F / 2),
                    sbytes, &bar_ld[j]);
        }
      }
      if (failed) {
        if (lane == 0) drain_wait(&bar_ld[j], par);  // a copy still in flight lands first
        break;
      }
      const unsigned long long* wv = wstg + static_cast<size_t>(j) * (F / 2);
      uint32_t* a32 = reinterpret_cast<uint32_t*>(wact + static_cast<size_t>(j) * F8);
      for (int w = lane; w < F / 2; w += 32) a32[w] = static_cast<uint32_t>(wv[w]);
      __syncwarp();
      for (int grp = lane; grp < F / 32; grp += 32)
        wast[static_cast<size_t>(j) * (F / 32) + grp] =
            -8.0f / kTwo20 * group_act_sum(wact + static_cast<size_t>(j) * F8 + 4 * grp);
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar_slot[j]);
        if (kPhaseStamps && p.stamps && j < 8) stamp_at(p.stamps, bid * kStamps + 32 + j);  // debug: slot in
      }
    }
    // 2. this warp's down units, slot by slot, as the slots come in
    // (the waits suspend in hardware: a spinning warp would take issue
    // slots from the reduction warp that brings the slots in)
    stamp(41);  // debug: warp 0's slots brought in
    if (!__all_sync(0xFFFFFFFFu, mbar_sleep(&bar_down, 0, err))) failed = true;
    stamp(42);  // debug: warp 0 sees the down rows
    int dbg_k = 0;
    for (int j = 0; j < nslots && !failed; ++j) {
      const int u = ((warp - j * wU) % kAllWarps + kAllWarps) % kAllWarps;
      if (u >= wU) continue;
      if (!__all_sync(0xFFFFFFFFu, mbar_sleep(&bar_slot[j], 0, err))) {
        failed = true;
        break;
      }
      if (dbg_k < 6) stamp(56 + 2 * dbg_k);  // debug: warp 0's unit k starts
      wave_unit(wrow, j, u / kParts, u % kParts, wact, wast, lane);
      if (dbg_k < 6) stamp(57 + 2 * dbg_k);  // debug: and ends
      ++dbg_k;
    }
    stamp(23);  // debug: warp 0's down units done
  }
  } else {
    // the reduction and refill warp: for every stage, once all compute warps
    // have released it, reduce a gate/up block's partials (in warp order),
    // publish its acts, and request the stage that reuses the ring slot
    // (gate/up stages come first; once the last is published, this CTA
    // flags its acts as out)
    int ngu = 0;
    while (ngu < nst && (s_stage[ngu].kind_slot >> 8) == 0) ++ngu;
    if (ngu == 0 && lane == 0 && !waves) {
      st_relaxed_u32(p.gdone + bid, tag);
      __threadfence();
    }
    for (int s = 0; s < nst && !failed; ++s) {
      const Stage sg = s_stage[s];
      const int rs = s % NS;
      uint8_t* base = ring + static_cast<uint32_t>(rs) * L.sb;
      const uint32_t par = static_cast<uint32_t>(s / NS) & 1u;
      const int slot = sg.kind_slot & 0xFF;
      const bool down = (sg.kind_slot >> 8) != 0;
      const float* rd = red + static_cast<uint32_t>(rs) * kWarps * L.red_words;
      if (!__all_sync(0xFFFFFFFFu, mbar_sleep(&bar_rel[rs], par, err))) {
        failed = true;
        break;
      }
      if (!down) {
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        const uint32_t RW = L.red_words;
        if (T == 1) {
          if (c == 0)
            for (int w = 0; w < kWarps; ++w) {
              v[0] += rd[w * RW + 2 * g];
              v[2] += rd[w * RW + 2 * g + 1];
            }
        } else if (T == 2) {
          if (c == 0)
            for (int w = 0; w < kWarps; ++w) {
              const float4 q = *reinterpret_cast<const float4*>(rd + w * RW + 4 * g);
              v[0] += q.x; v[1] += q.y; v[2] += q.z; v[3] += q.w;
            }
        } else {
          if (c < 2)
            for (int w = 0; w < kWarps; ++w) {
              const float4 q = *reinterpret_cast<const float4*>(rd + w * RW + 4 * (2 * g + c));
              v[0] += q.x; v[1] += q.y; v[2] += q.z; v[3] += q.w;
            }
        }
        // rows g: gate f (v0, v1) and up f (v2, v3) of columns 2c, 2c + 1
        const float a0 = gate_act_fast(p.act, v[0] * kTwo20) * (v[2] * kTwo20);
        const float a1 = gate_act_fast(p.act, v[1] * kTwo20) * (v[3] * kTwo20);
        float col[8];
        const int n = lane & 7, src_c = n >> 1;
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
          const float s0 = __shfl_sync(0xFFFFFFFFu, a0, gg * 4 + src_c);
          const float s1 = __shfl_sync(0xFFFFFFFFu, a1, gg * 4 + src_c);
          col[gg] = (n & 1) ? s1 : s0;
        }
        float hs = 0.0f;
        const uint4 fr = op_chunk(col, &hs);
        const int blk = 8 * sg.chunk + sg.a;
        if (waves) {
          // four tagged words, no fence: the readers check every tag
          if (lane == 0) {
            unsigned long long* o = p.hact + (static_cast<size_t>(slot) * F8 + blk) * 4;
            const unsigned long long tg = static_cast<unsigned long long>(tag) << 32;
            st_relaxed_u64(o + 0, tg | fr.x);
            st_relaxed_u64(o + 1, tg | fr.y);
            st_relaxed_u64(o + 2, tg | fr.z);
            st_relaxed_u64(o + 3, tg | fr.w);
          }
          __syncwarp();
          if (kPhaseStamps && s < 8 && lane == 0 && p.stamps) stamp_at(p.stamps, bid * kStamps + 48 + s);  // debug

        } else if (lane < T) {
          // four (tag, half2) words: a reader that sees this launch's tag in
          // a word sees that word's data (no fence, no separate flag)
          unsigned long long* o = p.hact + ((static_cast<size_t>(slot) * T + lane) * F8 + blk) * 4;
          const unsigned long long tg = static_cast<unsigned long long>(tag) << 32;
          st_relaxed_u64(o + 0, tg | fr.x);
          st_relaxed_u64(o + 1, tg | fr.y);
          st_relaxed_u64(o + 2, tg | fr.z);
          st_relaxed_u64(o + 3, tg | fr.w);
        }
        __syncwarp();
      }
      if (s == ngu - 1 && !waves) {
        // the block's act words, then the flag: a fence on each side, so that
        // both leave this SM now rather than whenever its store queue drains
        // (once per CTA, on this warp only)
        __threadfence();
        __syncwarp();
        if (lane == 0) {
          st_relaxed_u32(p.gdone + bid, tag);
          __threadfence();
          if (kPhaseStamps && p.stamps) stamp_at(p.stamps, bid * kStamps + 11);  // debug: acts out
        }
        __syncwarp();
      }
      if (s + NS < nst) {
        issue_stage(p, L, s_stage[s + NS], s_slot_expert, base, &bar_st[rs], lane);
        if (lane == 0) ++s_issued[rs];
      }
    }
    if (waves && !failed && lane == 0) {
      // every stage is released, so the ring is free: each slot's tagged act
      // words in one bulk copy, all requested at once (the compute warps
      // check, unpack and release them)
      if (kPhaseStamps && p.stamps) stamp_at(p.stamps, bid * kStamps + 40);  // debug: loads start
      const uint32_t sbytes = static_cast<uint32_t>(F) * 4u;  // F / 2 words
      for (int j = 0; j < nslots; ++j) {
        mbar_arrive_expect_tx(&bar_ld[j], sbytes);
        bulk_load(wstg + static_cast<size_t>(j) * (F / 2), p.hact + static_cast<size_t>(j) * (F / 2),
                  sbytes, &bar_ld[j]);
      }
    }
    // then this warp runs down units too (the round goes over all 16
    // warps: a CTA of 20 rows and eight slots gives every warp one unit)
    if (waves && !failed) {
      if (!__all_sync(0xFFFFFFFFu, mbar_sleep(&bar_down, 0, err))) failed = true;
      for (int j = 0; j < nslots && !failed; ++j) {
        const int u = ((warp - j * wU) % kAllWarps + kAllWarps) % kAllWarps;
        if (u >= wU) continue;
        if (!__all_sync(0xFFFFFFFFu, mbar_sleep(&bar_slot[j], 0, err))) {
          failed = true;
          break;
        }
        wave_unit(wrow, j, u / kParts, u % kParts, wact, wast, lane);
      }
    }
  }

  if (failed && lane == 0) atomicOr(&s_failed, 1);
  __syncthreads();
  stamp(5);
  if (s_failed) {
    // let this CTA's own copies land before it exits; the host clears the
    // signals after reading the error word
    if (tid == 0) {
      for (int i = 0; i < NS; ++i)
        if (s_issued[i] > 0) drain_wait(&bar_st[i], static_cast<uint32_t>(s_issued[i] - 1) & 1u);
      if (s_down_issued) drain_wait(&bar_down, 0);
    }
    return;
  }

  if (waves) {
    // ---------------- this CTA's rows of y (one token) ----------------
    // v = the K parts of a row added in order; y = residual + gate *
    // shared + sum over ranks (ascending) w * v.  As with owned rows, the
    // next launch's grid counter is cleared all the same.
    if (bid == 0 && tid == 0) sig->gcount[(tag & 1u) ^ 1u] = 0u;
    for (int q = tid; q < wnr; q += kThreads) {
      auto vs = [&](int j) {
        float v = 0.0f;
#pragma unroll
        for (int kp = 0; kp < kParts; ++kp) v += sv_w[(static_cast<size_t>(kp) * (K + 1) + j) * 32 + q];
        return v * kTwo20;
      };
      const int d = wr0 + q;
      float y = q == tid ? wres : (p.residual ? p.residual[d] : 0.0f);
      if (p.has_shared) {
        const float v = vs(nslots - 1);
        y = p.has_gate ? fmaf(s_gate[0], v, y) : y + v;
      }
      for (int r = 0; r < K; ++r) y = fmaf(s_w[0][r], vs(r), y);
      if (p.y_f32)
        reinterpret_cast<float*>(p.y)[d] = y;
      else
        reinterpret_cast<__nv_bfloat16*>(p.y)[d] = __float2bfloat16_rn(y);
    }
    stamp(7);
    if (tid == 0) sig->epoch[bid] = tag;  // read by this CTA's next launch
    return;
  }

  if (rows_owned(T)) {
    // ---------------- this CTA's rows of y, combined here ----------------
    // y = residual + gate * shared + sum over ranks (ascending) w * v.  No
    // grid counter is used; the next launch's counter is still cleared, as
    // every launch that passes its grid barrier does, since the next launch
    // may be one of the kernels that counts on it starting at zero.
    if (bid == 0 && tid == 0) sig->gcount[(tag & 1u) ^ 1u] = 0u;
    const uint32_t ntl = static_cast<uint32_t>(D / 16);
    const int t0 = static_cast<int>((ntl * static_cast<uint32_t>(bid)) / static_cast<uint32_t>(G));
    const int t1 = static_cast<int>((ntl * static_cast<uint32_t>(bid + 1)) / static_cast<uint32_t>(G));
    const int RWS = 16 * (t1 - t0);
    // v of (slot, token, row): its K parts added in order, in place of part 0
    for (int q = tid; q < nslots * T * RWS; q += kThreads) {
      float v = 0.0f;
#pragma unroll
      for (int kp = 0; kp < kParts; ++kp) v += sv[static_cast<size_t>(kp) * nslots * T * RWS + q];
      sv[q] = v * kTwo20;
    }
    __syncthreads();
    auto vsum = [&](int sl, int t, int rl) {
      return sv[(static_cast<size_t>(sl) * T + t) * RWS + rl];
    };
    for (int q = tid; q < T * RWS; q += kThreads) {
      const int t = q / RWS, rl = q - t * RWS, d = 16 * t0 + rl;
      float y = p.residual ? p.residual[static_cast<size_t>(t) * D + d] : 0.0f;
      if (p.has_shared) {
        const float v = vsum(nslots - 1, t, rl);
        y = p.has_gate ? fmaf(s_gate[t], v, y) : y + v;
      }
      for (int r = 0; r < K; ++r) {
        const int sl = fast1 ? r : s_pos_slot[s_pair_pos[t * K + r]];
        y = fmaf(s_w[t][r], vsum(sl, t, rl), y);
      }
      if (p.y_f32)
        reinterpret_cast<float*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] = y;
      else
        reinterpret_cast<__nv_bfloat16*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] =
            __float2bfloat16_rn(y);
    }
    stamp(7);
    if (tid == 0) sig->epoch[bid] = tag;  // read by this CTA's next launch
    return;
  }

  // ---------------- every partial of the grid ----------------
  if (tid == 0) {
    uint32_t* ctr = &sig->gcount[tag & 1u];
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    const unsigned long long t0 = global_timer_ns();
    bool ok = true;
    for (uint32_t spin = 0; ld_acquire_u32(ctr) < static_cast<uint32_t>(G); ++spin) {
      if ((spin & 63u) == 63u && poll_give_up(t0, err)) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
    s_failed = ok ? 0 : 1;
    if (ok && bid == 0) sig->gcount[(tag & 1u) ^ 1u] = 0u;
  }
  __syncthreads();
  stamp(6);
  if (s_failed) return;

  // ---------------- combine this CTA's share of y ----------------
  // v[t][r] = sum over chunks of the rank's slot partials (fixed order), then
  // y = residual + gate * shared + sum over ranks (ascending) w * v
  {
    const int d0 = (bid * D) / G, d1 = ((bid + 1) * D) / G, nd = d1 - d0;
    const int R = K + (p.has_shared ? 1 : 0);
    // v = sum over the rank's slot's chunks, in chunk order; a (token, rank,
    // d) row of NC partials is contiguous
    float* sv = reinterpret_cast<float*>(ring);  // [T][R][nd]
    for (int q = tid; q < T * R * nd; q += kThreads) {
      const int tr = q / nd, dl = q - tr * nd, t = tr / R, r = tr - t * R;
      const int sl = r < K ? (fast1 ? r : s_pos_slot[s_pair_pos[t * K + r]]) : nslots - 1;
      const float* src = p.partial + ((static_cast<size_t>(sl) * T + t) * D + d0 + dl) * NC;
      float v = 0.0f;
      for (int c0 = 0; c0 < NC; c0 += 16) {
        float part[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) part[u] = c0 + u < NC ? __ldcg(src + c0 + u) : 0.0f;
#pragma unroll
        for (int u = 0; u < 16; ++u) v += part[u];
      }
      sv[q] = v * kTwo20;
    }
    __syncthreads();
    for (int q = tid; q < T * nd; q += kThreads) {
      const int t = q / nd, dl = q - t * nd, d = d0 + dl;
      float y = p.residual ? p.residual[static_cast<size_t>(t) * D + d] : 0.0f;
      if (p.has_shared) {
        const float v = sv[(t * R + K) * nd + dl];
        y = p.has_gate ? fmaf(s_gate[t], v, y) : y + v;
      }
      for (int r = 0; r < K; ++r) y = fmaf(s_w[t][r], sv[(t * R + r) * nd + dl], y);
      if (p.y_f32)
        reinterpret_cast<float*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] = y;
      else
        reinterpret_cast<__nv_bfloat16*>(p.y)[static_cast<size_t>(t) * p.y_stride + d] =
            __float2bfloat16_rn(y);
    }
  }
  stamp(7);
  if (tid == 0) sig->epoch[bid] = tag;  // read by this CTA's next launch
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
size_t stream_smem_limit() {
  static size_t limit = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    const void* kernels[5] = {reinterpret_cast<const void*>(decode_stream_kernel<1, false>),
                              reinterpret_cast<const void*>(decode_stream_kernel<1, true>),
                              reinterpret_cast<const void*>(decode_stream_kernel<2, false>),
                              reinterpret_cast<const void*>(decode_stream_kernel<3, false>),
                              reinterpret_cast<const void*>(decode_stream_kernel<4, false>)};
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

// Ring stages for this shape within the shared memory limit (0: does not fit).
int ring_slots_for(int T, int D, int F, int K, int G, bool waves = false) {
  const size_t lim = stream_smem_limit();
  for (int ns = kMaxRing; ns >= 2; --ns)
    if (make_plan(T, D, F, K, G, ns, waves).total <= lim) return ns;
  return 0;
}

// Whether one router-routed token can run in waves: a CTA's rows of y in two
// 16-row tiles, the whole plan in shared memory with room for the router
// rows and order keys, and the slots' acts in the ring after the stages.
bool waves_ok(int D, int F, int K, int E, int G) {
  if (F / 64 < kParts) return false;
  if (4 * ((D / 4 + G - 1) / G) > 32) return false;
  if ((static_cast<long long>(K + 1) * (F / 8) + G - 1) / G > kMaxStages) return false;
  const int ns = ring_slots_for(1, D, F, K, G, true);
  if (ns < 2) return false;
  const Plan L = make_plan(1, D, F, K, G, ns, true);
  // after the stages the ring holds every slot's act words, acts and
  // accumulator starts
  const uint64_t acts = static_cast<uint64_t>(K + 1) * (static_cast<uint64_t>(F) * 6u + (F / 32) * 4u);
  return 2u * static_cast<uint32_t>(D) * 4u + static_cast<uint32_t>(E) * 4u <=
             static_cast<uint32_t>(ns) * L.sb &&
         acts <= static_cast<uint64_t>(ns) * L.sb;
}

// An upper bound of the stages of one CTA's share (largest slot count).
long long max_stages_bound(int T, int D, int F, int K, int E, int has_shared, int G, uint32_t sd,
                           uint32_t sb) {
  const long long nslots = std::min(T * K, E) + (has_shared ? 1 : 0);
  const long long ng = nslots * (F / 8), nd = D / 16, ndt = nslots * (F / 64) * nd;
  const long long gshare = (ng + G - 1) / G, dshare = (ndt + G - 1) / G;
  if (rows_owned(T)) {
    // whole down rows of every slot, packed slots per stage
    const long long ntmax = (nd + G - 1) / G;
    const long long sbb = ntmax * 16 * (F / 2 + F / 16);
    const long long per = sbb > 0 ? std::min<long long>(32, static_cast<long long>(sb) / sbb) : 1;
    if (per < 1) return kMaxStages + 1;
    return gshare + 1 + (nslots + per - 1) / per;
  }
  return gshare + dshare / sd + dshare / nd + 3;
}

bool encode_down(CUtensorMap* map, const void* base, uint64_t F, uint64_t D, uint64_t n,
                 uint64_t nstride, uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {F / 2, D, n};
  const cuuint64_t strides[2] = {F / 2, nstride};
  const cuuint32_t box[3] = {32, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The partial sums of one launch.  The tagged act words live apart, in a
// region zeroed at allocation and after an error, so that no stale word can
// carry a later launch's tag.
// Gate (or up) codes [E][F][D/2] bytes as 8-row boxes laid out
// [D/256 chunks][8 rows][128 bytes] with the 128-byte swizzle (dims: byte in
// chunk, row, chunk, expert).
bool encode_rows8(CUtensorMap* map, const void* base, uint64_t D, uint64_t F, uint64_t n,
                  uint64_t nstride) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {128, F, D / 256, n};
  const cuuint64_t strides[3] = {D / 2, 128, nstride};
  const cuuint32_t box[4] = {128, 8, static_cast<cuuint32_t>(D / 256), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct ScratchLayout {
  size_t partial, total;
};

ScratchLayout scratch_layout(int T, int D, int F, int K) {
  const size_t slots = static_cast<size_t>(T * K + 1);
  ScratchLayout s;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = (o + bytes + 255) / 256 * 256;
    return at;
  };
  s.partial = take(slots * (F / 64) * T * static_cast<size_t>(D) * 4);
  s.total = o;
  return s;
}

}  // namespace

bool encode_decode_maps(const ExpertSet& ex, int D, int F, int E, DecodeMaps* out) {
  const uint64_t est = ex.stride ? ex.stride : static_cast<uint64_t>(F) * D;
  const uint8_t* rb = ex.base + ex.off.down_w;
  if (!encode_down(&out->down128, rb, F, D, static_cast<uint64_t>(E), est, kDownBox) ||
      !encode_down(&out->down16, rb, F, D, static_cast<uint64_t>(E), est, 16) ||
      !encode_rows8(&out->gate8, ex.base + ex.off.gate_w, D, F, static_cast<uint64_t>(E), est) ||
      !encode_rows8(&out->up8, ex.base + ex.off.up_w, D, F, static_cast<uint64_t>(E), est))
    return false;
  if (ex.shared) {
    const uint8_t* sb = ex.shared + ex.shared_off.down_w;
    const uint64_t sst = static_cast<uint64_t>(F) * D * 2;
    return encode_down(&out->sdown128, sb, F, D, 1, sst, kDownBox) &&
           encode_down(&out->sdown16, sb, F, D, 1, sst, 16) &&
           encode_rows8(&out->sgate8, ex.shared + ex.shared_off.gate_w, D, F, 1, sst) &&
           encode_rows8(&out->sup8, ex.shared + ex.shared_off.up_w, D, F, 1, sst);
  }
  out->sdown128 = out->down128;
  out->sdown16 = out->down16;
  out->sgate8 = out->gate8;
  out->sup8 = out->up8;
  return true;
}

bool decode_stream_supported(int T, int D, int F, int K, int E, int has_gate, int has_shared,
                             int num_sms) {
  if (T < 1 || T > kMaxTok || T * K > kMaxPairs || K > kMaxK || E > 256 || E % 4 ||
      E + has_gate > 2 * num_sms || num_sms > kMaxCtas)
    return false;
  if (D % 64 || D > 4096 || D < 128 || F % 64 || F > 4096) return false;
  const int ns = ring_slots_for(T, D, F, K, num_sms);
  if (ns < 2) return false;
  const Plan L = make_plan(T, D, F, K, num_sms, ns);
  if (L.sd < 1) return false;
  // router rows and order keys live in the ring before the first copy
  if (2u * static_cast<uint32_t>(D) * 4u + static_cast<uint32_t>(T * E) * 4u >
      static_cast<uint32_t>(ns) * L.sb)
    return false;
  // the final combine stages every partial of a CTA's share in the ring
  const size_t nd = static_cast<size_t>((D + num_sms - 1) / num_sms);
  const size_t R = static_cast<size_t>(K + (has_shared ? 1 : 0));
  if (static_cast<size_t>(T) * R * nd * 4 > static_cast<size_t>(ns) * L.sb) return false;
  if (D % 256 || D / 256 > 16) return false;  // 8-row boxes of D/256 128-byte chunks
  if (D / 64 > 3 * kWarps) return false;       // at most 3 pairs of groups per compute warp
  return max_stages_bound(T, D, F, K, E, has_shared, num_sms, L.sd, L.sb) <= kMaxStages;
}

size_t decode_stream_scratch_bytes(int T, int D, int F, int K) {
  return scratch_layout(T, D, F, K).total;
}

// [kMaxCtas] per-CTA "acts out" tags, then the tagged act words
size_t decode_stream_flag_bytes(int T, int F, int K) {
  return kMaxCtas * 4 + static_cast<size_t>(T * K + 1) * T * (F / 8) * 32;
}

cudaError_t launch_decode_stream(const DecodeFusedArgs& a, const DecodeMaps& maps, void* scratch,
                                 void* flags, cudaStream_t s) {
  if (!decode_stream_supported(a.T, a.D, a.F, a.K, a.E, a.has_gate, a.has_shared, a.num_sms))
    return cudaErrorInvalidValue;
  const bool waves = a.T == 1 && a.ids_in == nullptr && waves_ok(a.D, a.F, a.K, a.E, a.num_sms);
  const int ns = ring_slots_for(a.T, a.D, a.F, a.K, a.num_sms, waves);
  const Plan L = make_plan(a.T, a.D, a.F, a.K, a.num_sms, ns, waves);
  const ScratchLayout sl = scratch_layout(a.T, a.D, a.F, a.K);
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  StreamParams p{};
  p.maps = maps;
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
  p.gdone = static_cast<uint32_t*>(flags);
  p.hact = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(flags) + kMaxCtas * 4);
  p.partial = reinterpret_cast<float*>(sc + sl.partial);
  p.counters = a.counters;
  p.ids_out = a.ids_out;
  p.w_out = a.w_out;
  p.w16_out = a.w16_out;
  p.pairs_out = a.pairs_out;
  p.err = a.err;
  p.stamps = a.stamps;
  p.smem_bytes = L.total;
  p.ring_slots = ns;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeCooperative;
  attrs[0].val.cooperative = a.cooperative ? 1 : 0;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = a.allow_pdl ? 1 : 0;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  switch (a.T) {
    case 1:
      return waves ? cudaLaunchKernelEx(&cfg, decode_stream_kernel<1, true>, p)
                   : cudaLaunchKernelEx(&cfg, decode_stream_kernel<1, false>, p);
    case 2: return cudaLaunchKernelEx(&cfg, decode_stream_kernel<2, false>, p);
    case 3: return cudaLaunchKernelEx(&cfg, decode_stream_kernel<3, false>, p);
    default: return cudaLaunchKernelEx(&cfg, decode_stream_kernel<4, false>, p);
  }
}

}  // namespace tsg
