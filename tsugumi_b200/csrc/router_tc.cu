// router_tc.cu -- the prefill router logits on tcgen05, exact to fp32.
//
// Reference behaviour: the router GEMM of the prefill path
// (Sources/Tsugumi/Metal/Prefill/prefill.metal:719-794, router logits
// x · W^T with the effective scale folded into W) -- raw dot products of
// every token row with every fp32 router row; the norm factor, bias and
// top-K are applied afterwards by router_topk_kernel (router.cu).
//
// The token rows are bf16 and the router rows fp32.  Every fp32 value w is
// the exact sum of three bf16 values (hi = bf16(w), mid = bf16(w - hi),
// lo = w - hi - mid, which has at most 8 significant bits left), and a
// product of two bf16 values is exact in fp32.  So three bf16 MMAs per
// k-step (x·hi + x·mid + x·lo) into one fp32 accumulator give the fp32 dot
// product up to the order of the additions, the same freedom the split-K
// SIMT kernel already takes.  The three planes are made once per layer.
//
// One CTA per (128 router rows, 128 tokens, K split); 4 warps: lane 0 of
// warp 0 feeds a three-stage TMA ring (three 128-row weight boxes and one
// 128-row token box per 64-wide k-step, 128-byte swizzle, no multicast),
// lane 0 of warp 1 issues twelve MMAs per k-step (M=128 router rows,
// N=128 tokens, K=16) into three 128-column TMEM accumulators, one per
// plane, and all four warps then add them (small terms first) and drain
// their TMEM lane quarter into logits_raw[split][token][row].
// Every wait is bounded.
#include <cuda_bf16.h>

#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kRM = 128;      // router rows per CTA (MMA M)
constexpr int kRN = 128;      // tokens per CTA (MMA N)
constexpr int kRK = 64;       // K per stage
constexpr int kRStages = 3;
constexpr int kPlaneBytes = kRM * kRK * 2;     // one 128 x 64 bf16 box
constexpr int kRStageBytes = 3 * kPlaneBytes + kRN * kRK * 2;
constexpr int kRThreads = 128;
constexpr uint32_t kRTmemCols = 512;  // three 128-column accumulators (hi, mid, lo)

struct RtArgs {
  int T, E, E_pad, ksteps_total, ksteps_per_split;
  float* out;  // logits_raw [ksplit][T][E]
  uint32_t* err;
};

// Four K=16 bf16 MMAs of one 64-wide k-step, both operands in 128-byte
// swizzled shared memory (descriptors advance 32 bytes per K=16).
TSG_DEV void umma_ss_k64(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %3, 0;\n\t"
      "setp.eq.b32 p1, %3, %3;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %4, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %6, %4, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %8, %4, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %9, %10, %4, p1;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(accumulate), "r"(idesc), "l"(a_desc + 2), "l"(b_desc + 2),
      "l"(a_desc + 4), "l"(b_desc + 4), "l"(a_desc + 6), "l"(b_desc + 6)
      : "memory");
}

// kind::f16 instruction descriptor with bf16 A and B (format 1 in [7,10) and
// [10,13)), fp32 D, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(uint32_t m, uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__global__ void __launch_bounds__(kRThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                     const RtArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kRStages], empty[kRStages], done;
  __shared__ uint32_t tmem_base;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - smem_u32(smem_raw));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kRN, m0 = blockIdx.y * kRM, split = blockIdx.z;
  const int k0 = split * a.ksteps_per_split;
  const int k1 = min(a.ksteps_total, k0 + a.ksteps_per_split);
  const int nk = k1 - k0;

  if (tid == 0) {
    for (int s = 0; s < kRStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, kRTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = tmem_base;

  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&map_w);
    prefetch_tensormap(&map_x);
    bool ok = true;
    int issued = 0;
    for (int k = 0; k < nk && ok; ++k, ++issued) {
      const int s = k % kRStages;
      if (!mbar_sleep(&empty[s], ((k / kRStages) & 1u) ^ 1u, a.err)) { ok = false; break; }
      uint8_t* st = g + s * kRStageBytes;
      mbar_arrive_expect_tx(&full[s], kRStageBytes);
      const int kx = (k0 + k) * kRK;
      for (int pl = 0; pl < 3; ++pl)
        tma_load_2d(st + pl * kPlaneBytes, &map_w, &full[s], kx, pl * a.E_pad + m0);
      tma_load_2d(st + 3 * kPlaneBytes, &map_x, &full[s], kx, n0);
    }
    for (int q = (issued > kRStages ? issued - kRStages : 0); q < issued; ++q)
      mbar_sleep(&full[q % kRStages], (q / kRStages) & 1u, a.err);
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = umma_idesc_bf16(kRM, kRN);
    bool ok = true;
    for (int k = 0; k < nk; ++k) {
      const int s = k % kRStages;
      if (!mbar_sleep(&full[s], (k / kRStages) & 1u, a.err)) { ok = false; break; }
      tc_fence_after_sync();
      const uint32_t st = smem_u32(g + s * kRStageBytes);
      const uint64_t db = umma_desc_sw128(st + 3 * kPlaneBytes);
      // one accumulator per plane: the hi, mid and lo products each meet
      // terms of their own size, and are added in the epilogue
#pragma unroll
      for (int pl = 0; pl < 3; ++pl)
        umma_ss_k64(tmem + pl * kRN, umma_desc_sw128(st + pl * kPlaneBytes), db, idesc,
                    k > 0 ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    if (ok) umma_commit(&done);
  }
  __syncwarp();

  // epilogue: warp q drains TMEM lanes 32q.. (router rows m0 + 32q + lane);
  // a split with no k-steps writes zero partial sums
  const bool ok = nk <= 0 || __all_sync(0xffffffffu, mbar_sleep(&done, 0, a.err)) != 0;
  tc_fence_after_sync();
  const int row = m0 + 32 * warp + lane;
  float* out = a.out + static_cast<size_t>(split) * a.T * a.E;
  for (int c0 = 0; ok && c0 < kRN; c0 += 16) {
    uint32_t rh[16], rm[16], rl[16];
    if (nk > 0) {
      const uint32_t ta = tmem + (static_cast<uint32_t>(32 * warp) << 16) + c0;
      tmem_ld16(ta, rh);
      tmem_ld16(ta + kRN, rm);
      tmem_ld16(ta + 2 * kRN, rl);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) rh[j] = rm[j] = rl[j] = 0u;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int t = n0 + c0 + j;
      const float v = (__uint_as_float(rl[j]) + __uint_as_float(rm[j])) + __uint_as_float(rh[j]);
      if (t < a.T && row < a.E) out[static_cast<size_t>(t) * a.E + row] = v;
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kRTmemCols);
  }
}

// hi / mid / lo bf16 planes of the fp32 router rows, rows >= E zero.
__global__ void split_router_kernel(const float* w, int E, int D, int E_pad, __nv_bfloat16* out) {
  const size_t n = static_cast<size_t>(E_pad) * D;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / D;
    const float v = row < static_cast<size_t>(E) ? w[i] : 0.0f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(mid);
    out[i] = hi;
    out[n + i] = mid;
    out[2 * n + i] = __float2bfloat16_rn(r2);
  }
}

bool encode_bf16_rows(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                      uint64_t stride_elems, uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {stride_elems * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int router_tc_pad(int E) { return (E + kRM - 1) / kRM * kRM; }

cudaError_t launch_split_router(const float* w, int E, int D, void* planes, cudaStream_t s) {
  const int E_pad = router_tc_pad(E);
  split_router_kernel<<<256, 256, 0, s>>>(w, E, D, E_pad, static_cast<__nv_bfloat16*>(planes));
  return cudaGetLastError();
}

bool router_tc_usable(const RouterParams& p) {
  // T >= 128: the token box is never taller than the token matrix
  return p.w_bf16x3 != nullptr && p.T >= kRN && p.D % kRK == 0 && p.x_stride % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0;
}

int router_tc_ksplit(int T, int E, int D) {
  const int mt = (T + kRN - 1) / kRN, et = router_tc_pad(E) / kRM;
  const int ksteps = D / kRK;
  int ksplit = 1;
  // enough CTAs for the SMs, each with at least 4 k-steps
  while (mt * et * ksplit * 2 <= 148 && ksplit * 2 <= 8 && ksteps / (ksplit * 2) >= 4) ksplit *= 2;
  return ksplit;
}

cudaError_t launch_router_tc(const RouterParams& p, const RouteBuffers& rb, int ksplit,
                             cudaStream_t s) {
  const int E_pad = router_tc_pad(p.E);
  CUtensorMap mw, mx;
  if (!encode_bf16_rows(&mw, p.w_bf16x3, 3ull * E_pad, p.D, p.D, kRM) ||
      !encode_bf16_rows(&mx, p.x, p.T, p.D, p.x_stride, kRN))
    return cudaErrorInvalidValue;
  RtArgs a;
  a.T = p.T;
  a.E = p.E;
  a.E_pad = E_pad;
  a.ksteps_total = p.D / kRK;
  a.ksteps_per_split = (a.ksteps_total + ksplit - 1) / ksplit;
  a.out = rb.logits_raw;
  a.err = rb.err;
  cudaError_t e = allow_max_smem(router_tc_kernel);
  if (e != cudaSuccess) return e;
  const size_t smem = 1024 + static_cast<size_t>(kRStages) * kRStageBytes;
  dim3 grid((p.T + kRN - 1) / kRN, E_pad / kRM, ksplit);
  router_tc_kernel<<<grid, kRThreads, smem, s>>>(mw, mx, a);
  return cudaGetLastError();
}

}  // namespace tsg
