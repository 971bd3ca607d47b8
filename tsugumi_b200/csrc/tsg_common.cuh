// tsg_common.cuh -- device helpers shared by the MoE kernels (sm_100a only).
//
// Inline-PTX wrappers for mbarriers, bulk and tensor copies (TMA), and the
// 5th-generation tensor core (tcgen05: TMEM allocation, UMMA issue, commit,
// TMEM loads).  Every wait on an mbarrier is bounded: after kWaitLimitNs of
// global time it records TSG_DEVERR_TIMEOUT in the launch's error word and
// returns false, so a broken pipeline ends the kernel instead of hanging the
// GPU.  No multicast form of any copy is used anywhere in this library.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <unordered_set>

#define TSG_DEV __device__ __forceinline__

// Bits of the per-context device error word (read back by tsg_sync).
enum : uint32_t {
  TSG_DEVERR_TIMEOUT = 1u,   // a bounded wait ran out
  TSG_DEVERR_BOUNDS = 2u,    // an index failed its range check; access skipped
  TSG_DEVERR_METADATA = 4u,  // routing metadata failed validation
  TSG_DEVERR_DUPLICATE = 8u, // duplicate (token, rank) pair
};

// Opts a kernel into the largest dynamic shared memory once per process, so
// launches (including those recorded into a CUDA graph) set no attributes.
inline cudaError_t allow_max_smem_ptr(const void* k) {
  static std::mutex mu;
  static std::unordered_set<const void*> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(k)) return cudaSuccess;
  // the opt-in limit covers static + dynamic shared memory together
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa;
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, k);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - static_cast<int>(fa.sharedSizeBytes));
  if (e == cudaSuccess) done.insert(k);
  return e;
}
template <typename Kern>
inline cudaError_t allow_max_smem(Kern k) {
  return allow_max_smem_ptr(reinterpret_cast<const void*>(k));
}

// One second: far above any legitimate pipeline stall of these kernels.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

TSG_DEV int imin(int a, int b) { return a < b ? a : b; }
TSG_DEV uint32_t umin32(uint32_t a, uint32_t b) { return a < b ? a : b; }

TSG_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

TSG_DEV unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

TSG_DEV void flag_error(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

TSG_DEV bool error_raised(const uint32_t* err) {
  return err && (*(volatile const uint32_t*)err) != 0u;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
TSG_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

TSG_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

TSG_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

TSG_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One try of a phase: the thread may be suspended until the phase completes
// or kTryWaitHintNs pass.  The bound is explicit: without one the suspend
// limit is the system's choice, and a wait loop that checks its clock between
// tries could then overrun its own limit by far.
constexpr uint32_t kTryWaitHintNs = 10000u;
TSG_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kTryWaitHintNs)
      : "memory");
  return ok != 0u;
}

// Non-blocking test of a phase (for a look ahead that must not stall).
TSG_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (and flags TSG_DEVERR_TIMEOUT) when the limit runs out, or when
// another thread of the launch has already flagged an error.  The spin is
// kept out of line so that every call site costs a few instructions of code.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, uint32_t* err) {
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
TSG_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, err);
}

// As mbar_wait, but each try suspends the thread in hardware (up to
// kSuspendHintNs, or until the phase completes) instead of spinning, so a
// warp that waits for a long time takes no issue slots from the warps that
// work.  For pipelines with many waiting warps per SM.
constexpr uint32_t kSuspendHintNs = 1000000u;
TSG_DEV bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0u;
}
static __device__ __noinline__ bool mbar_sleep_slow(uint64_t* bar, uint32_t parity, uint32_t* err) {
  const unsigned long long t0 = global_timer_ns();
  while (!mbar_try_wait_suspend(bar, parity)) {
    if (error_raised(err)) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      flag_error(err, TSG_DEVERR_TIMEOUT);
      return false;
    }
  }
  return true;
}
TSG_DEV bool mbar_sleep(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_sleep_slow(bar, parity, err);
}

// ---------------------------------------------------------------------------
// Bulk (1-D) and tensor (TMA) copies, global -> shared, no multicast.
// ---------------------------------------------------------------------------
// Both addresses 16-byte aligned, bytes a multiple of 16.
TSG_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

TSG_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

TSG_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0, int32_t c1,
                         int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

TSG_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy writes to shared memory that the tensor core (async proxy)
// will read must be fenced before the consumer is signalled.
TSG_DEV void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM and UMMA (cta_group::1)
// ---------------------------------------------------------------------------
TSG_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
TSG_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
TSG_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
TSG_DEV void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
TSG_DEV void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulate.  One
// thread issues.  The disable-output-lane mask is all zero.
TSG_DEV void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T.  A is M=128 rows in TMEM lanes 0-127,
// K packed two fp16 per 32-bit column (element 2c in the low half of column
// c), so one K=16 step reads 8 columns from `a_tmem`.
TSG_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One 64-wide k-step as four K=16 MMAs issued from a single asm block, A in
// TMEM (columns a_tmem, +8, +16, +24) and B in a 128-byte-swizzled smem tile
// (descriptor b_desc, advanced by 32 bytes per K=16).  Issuing the four with
// their operands already in distinct registers lets them leave the issuing
// thread back to back; issued one by one with address arithmetic in between,
// each waits for the previous one's operands to be consumed.
TSG_DEV void umma_f16_ts_k64(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                             uint32_t accumulate) {
  const uint64_t b1 = b_desc + 2u, b2 = b_desc + 4u, b3 = b_desc + 6u;
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t.reg .b32 a1, a2, a3;\n\t"
      "setp.ne.b32 p0, %4, 0;\n\t"
      "setp.eq.b32 p1, %4, %4;\n\t"
      "add.u32 a1, %1, 8;\n\t"
      "add.u32 a2, %1, 16;\n\t"
      "add.u32 a3, %1, 24;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], %5, %3, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], %6, %3, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], %7, %3, p1;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "l"(b1), "l"(b2), "l"(b3)
      : "memory");
}

// Arrive on an mbarrier once every UMMA issued so far by this thread is done.
TSG_DEV void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 TMEM lanes x 32 bits, 16 consecutive columns per thread.
TSG_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
TSG_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The store counterpart: 16 consecutive columns of this thread's lane.  The
// warp may only address its own lane quarter (32 * (warp % 4)).
TSG_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
TSG_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// 128-byte swizzle layout: rows of 128 bytes (64 fp16 of K), 8-row atoms of
// 1024 bytes stacked densely (stride-dimension offset 1024 B), 16-byte chunk
// index XOR (row % 8).  The tile base must be 1024-byte aligned.  Field
// positions: start address >> 4 in [0,14), leading offset >> 4 in [16,30)
// (unused for swizzled K-major, set to 1), stride offset >> 4 in [32,46),
// version 1 in [46,48), layout type in [61,64) with SWIZZLE_128B = 2.
TSG_DEV uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp16 A and B (format 0), fp32 D
// (format 1 in [4,6)), both K-major, N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t m, uint32_t n) {
  return (1u << 4) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Byte offset of element (row, k) inside a SW128 K-major tile of 64-wide rows
// (k in [0, 64), 2-byte elements).
TSG_DEV uint32_t sw128_offset(uint32_t row, uint32_t k) {
  const uint32_t chunk = (k >> 3) ^ (row & 7u);
  return row * 128u + chunk * 16u + (k & 7u) * 2u;
}

// ---------------------------------------------------------------------------
// Number formats
// ---------------------------------------------------------------------------
TSG_DEV float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// The 8 nibbles of a 32-bit code word as floats 1 + q/16 (q the unsigned
// code), by placing (0x80 | q << 3) into the top mantissa byte of 1.0f.
// The caller recovers (q - 8) * x sums as 16 * sum(f * x) - 24 * sum(x).
// Element order: out[j] is element j of the word (low nibble of byte j/2 for
// even j).
TSG_DEV void nibbles_to_f32_plus1(uint32_t w, float (&out)[8]) {
  const uint32_t lo = ((w << 3) & 0x78787878u) | 0x80808080u;  // even elements
  const uint32_t hi = ((w >> 1) & 0x78787878u) | 0x80808080u;  // odd elements
  out[0] = __uint_as_float(__byte_perm(lo, 0x3Fu, 0x4055u));
  out[1] = __uint_as_float(__byte_perm(hi, 0x3Fu, 0x4055u));
  out[2] = __uint_as_float(__byte_perm(lo, 0x3Fu, 0x4155u));
  out[3] = __uint_as_float(__byte_perm(hi, 0x3Fu, 0x4155u));
  out[4] = __uint_as_float(__byte_perm(lo, 0x3Fu, 0x4255u));
  out[5] = __uint_as_float(__byte_perm(hi, 0x3Fu, 0x4255u));
  out[6] = __uint_as_float(__byte_perm(lo, 0x3Fu, 0x4355u));
  out[7] = __uint_as_float(__byte_perm(hi, 0x3Fu, 0x4355u));
}

// The 8 nibbles of a code word dequantised to fp16 with one rounding:
// out[i] = half2((q_2i - 8) * s, (q_2i+1 - 8) * s).  A byte permute places
// code byte i in both halves next to 0x64; masking keeps the low nibble in
// the low half (fp16 1024 + q) and the high nibble in the high half (fp16
// 1024 + 16 q).  One fma with (1, 1/16) and (-1032, -72) gives q - 8 exactly
// in both halves, and one multiply by the scale rounds once.
TSG_DEV void nibbles_to_f16x2_scaled(uint32_t w, __half2 s2, uint32_t (&out)[4]) {
  const __half2 mul = __halves2half2(__float2half_rn(1.0f), __float2half_rn(0.0625f));
  const __half2 add = __halves2half2(__float2half_rn(-1032.0f), __float2half_rn(-72.0f));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t sel = 0x4040u | (static_cast<uint32_t>(i) << 8) | static_cast<uint32_t>(i);
    const uint32_t pr = __byte_perm(w, 0x64u, sel) & 0xFFF0FF0Fu;
    __half2 h = *reinterpret_cast<const __half2*>(&pr);
    h = __hmul2(__hfma2(h, mul, add), s2);
    out[i] = *reinterpret_cast<uint32_t*>(&h);
  }
}

TSG_DEV float gelu_tanh_f(float x) {
  const float inner = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}
TSG_DEV float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// The same two activations for epilogues that evaluate thousands per
// thread: 0.5 x (1 + tanh(y)) = x / (1 + exp(-2y)) exactly, evaluated with
// the hardware exponential and a fast divide (relative error ~1e-6, far
// below the fp16 rounding of the result).  exp overflowing to +inf for very
// negative x gives x / inf = -0, the limit.
TSG_DEV float gelu_tanh_fast(float x) {
  const float y = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return __fdividef(x, 1.0f + __expf(-2.0f * y));
}
TSG_DEV float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
TSG_DEV float gate_act_fast(int act, float g) { return act == 1 ? silu_fast(g) : gelu_tanh_fast(g); }
TSG_DEV float gate_act(int act, float g) { return act == 1 ? silu_f(g) : gelu_tanh_f(g); }

TSG_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
