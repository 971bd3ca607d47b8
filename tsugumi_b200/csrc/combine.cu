// combine.cu -- the weighted combine / unpermute of the prefill regime.
//
// Reference behaviour: prefill_moe_reduce_token_major
// (Sources/Tsugumi/Metal/Prefill/prefill.metal:796-817) and the decode phase-2
// sum (Metal/MoE/moe.metal:651-687): for every token and output column,
// h2[t, d] = sum over ranks r ascending of fma(w[t, r], partial[t, r, d]),
// starting from the residual -- in the Qwen layer the residual is the shared
// branch, sigmoid(w_s . x) * shared(x) (QwenForwardRunner.swift:1548-1612).
// Here the routed partials sit in expert-sorted order and pair_pos maps each
// (token, rank) to its sorted row, so the kernel is also the unpermute.
#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

// One thread per (token, 8 consecutive columns).
__global__ void __launch_bounds__(256) combine_kernel(CombineParams p) {
  const int groups = p.D / 8;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int t = blockIdx.y;
  if (idx >= groups || t >= p.T) return;
  const int d0 = idx * 8;
  float acc[8];
  if (p.residual) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = p.residual[static_cast<size_t>(t) * p.D + d0 + j];
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  }
  if (p.has_shared) {
    float gate = 1.0f;
    if (p.gate_raw) {  // shared-gate logit, raw dot times the row's norm factor
      const float z = p.gate_raw[t] * p.inv_rms[t];
      gate = 1.0f / (1.0f + __expf(-z));
    }
    const uint4 v = *reinterpret_cast<const uint4*>(
        p.partials + static_cast<size_t>(p.T * p.K + t) * p.D + d0);
    const __half2* h2 = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __half22float2(h2[q]);
      acc[2 * q] = fmaf(gate, f.x, acc[2 * q]);
      acc[2 * q + 1] = fmaf(gate, f.y, acc[2 * q + 1]);
    }
  }
  for (int r = 0; r < p.K; ++r) {
    const uint32_t pos = p.pair_pos[t * p.K + r];
    const float w = p.weights[t * p.K + r];
    const uint4 v = *reinterpret_cast<const uint4*>(p.partials + static_cast<size_t>(pos) * p.D + d0);
    const __half2* h2 = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __half22float2(h2[q]);
      acc[2 * q] = fmaf(w, f.x, acc[2 * q]);
      acc[2 * q + 1] = fmaf(w, f.y, acc[2 * q + 1]);
    }
  }
  if (p.y_f32) {
    float* y = reinterpret_cast<float*>(p.y) + static_cast<size_t>(t) * p.y_stride + d0;
    *reinterpret_cast<float4*>(y) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(y + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  } else {
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      o[q] = *reinterpret_cast<uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.y) +
                              static_cast<size_t>(t) * p.y_stride + d0) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The reference's token-major reduce, as is: partials [(t*K + r)*D + d] fp16.
__global__ void reduce_token_major_kernel(const __half* partials, const float* w, int T, int K,
                                          int D, void* h2, int h2_f32) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  const int t = blockIdx.y;
  if (d >= D || t >= T) return;
  float acc = 0.0f;
  for (int r = 0; r < K; ++r)
    acc = fmaf(w[t * K + r], __half2float(partials[(static_cast<size_t>(t) * K + r) * D + d]), acc);
  if (h2_f32) reinterpret_cast<float*>(h2)[static_cast<size_t>(t) * D + d] = acc;
  else reinterpret_cast<__half*>(h2)[static_cast<size_t>(t) * D + d] = __float2half_rn(acc);
}

}  // namespace

cudaError_t launch_combine(const CombineParams& p, cudaStream_t s) {
  if (p.D % 8 || p.T <= 0) return p.T <= 0 ? cudaSuccess : cudaErrorInvalidValue;
  const int groups = p.D / 8;
  dim3 grid((groups + 255) / 256, p.T);
  combine_kernel<<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_reduce_token_major(const __half* partials, const float* w, int T, int K, int D,
                                      void* h2, int h2_f32, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  dim3 grid((D + 255) / 256, T);
  reduce_token_major_kernel<<<grid, 256, 0, s>>>(partials, w, T, K, D, h2, h2_f32);
  return cudaGetLastError();
}

}  // namespace tsg
