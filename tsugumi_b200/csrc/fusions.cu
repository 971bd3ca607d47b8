// The norms and residuals on either side of Gemma's MoE block, fused into one
// row pass each: the reference's fused_post_attn_setup and fused_layer_tail
// (Sources/Tsugumi/Metal/Fusions/fused.metal:190-267, :269-374), with the
// dense branch's post-norm (RealForwardRunner.swift:3236-3242, rmsnorm with a
// BF16 weight) folded into the tail.  The reference rounds each stored
// intermediate to fp16; here the activations are bf16, rounded at the same
// points.  One CTA of 256 threads per token; D <= 4096.

#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

constexpr int kFuseThreads = 256;

TSG_DEV float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
TSG_DEV uint16_t bf16b(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

// Sum over the CTA (every thread gets it).
TSG_DEV float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();  // (red is reused by consecutive calls)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int w = 0; w < kFuseThreads / 32; ++w) s += red[w];
  return s;
}

TSG_DEV float inv_rms(float sumsq, int D, float eps) {
  return rsqrtf(sumsq / static_cast<float>(D) + eps);
}

// hidden += post_attn_norm(attn); then the block's three inputs from the
// normalised hidden row: router_x = h^, routed_x = h^ w_pre_ffn2,
// dense_x = h^ w_pre_ffn (fused_post_attn_setup).
__global__ void __launch_bounds__(kFuseThreads) gemma_setup_kernel(
    uint16_t* hidden, uint32_t h_stride, const uint16_t* attn, uint32_t a_stride, int D,
    GemmaNorms n, uint16_t* router_x, uint16_t* routed_x, uint16_t* dense_x) {
  __shared__ float red[kFuseThreads / 32];
  extern __shared__ float hrow[];  // [D]
  const int t = blockIdx.x, tid = threadIdx.x;
  uint16_t* hr = hidden + static_cast<size_t>(t) * h_stride;
  const uint16_t* ar = attn + static_cast<size_t>(t) * a_stride;
  float ss = 0.0f;
  for (int i = tid; i < D; i += kFuseThreads) {
    const float a = bf16_bits_to_f32(ar[i]);
    ss = fmaf(a, a, ss);
  }
  const float inv_a = inv_rms(block_sum(ss, red), D, n.eps);
  ss = 0.0f;
  for (int i = tid; i < D; i += kFuseThreads) {
    const float a = bf16r(bf16_bits_to_f32(ar[i]) * inv_a * bf16_bits_to_f32(n.post_attn[i]));
    const float h = bf16r(bf16_bits_to_f32(hr[i]) + a);
    hrow[i] = h;
    hr[i] = bf16b(h);
    ss = fmaf(h, h, ss);
  }
  const float inv_h = inv_rms(block_sum(ss, red), D, n.eps);
  const size_t o = static_cast<size_t>(t) * D;
  for (int i = tid; i < D; i += kFuseThreads) {
    const float x = hrow[i] * inv_h;
    router_x[o + i] = bf16b(x);
    routed_x[o + i] = bf16b(x * bf16_bits_to_f32(n.pre_ffn2[i]));
    dense_x[o + i] = bf16b(x * bf16_bits_to_f32(n.pre_ffn[i]));
  }
}

// h1 = post_dense_norm(dense out); t = post_routed_norm(routed out);
// h12 = h1 + t; hidden = (hidden + post_ffn_norm(h12)) * layer_scalar
// (fused_layer_tail, with the dense branch's post-norm first).
__global__ void __launch_bounds__(kFuseThreads) gemma_tail_kernel(
    const float* h2, const float* h1, uint16_t* hidden, uint32_t h_stride, int D, GemmaNorms n) {
  __shared__ float red[kFuseThreads / 32];
  extern __shared__ float row[];  // [D]: h1n, then h12
  const int t = blockIdx.x, tid = threadIdx.x;
  const size_t o = static_cast<size_t>(t) * D;
  float s1 = 0.0f, s2 = 0.0f;
  for (int i = tid; i < D; i += kFuseThreads) {
    const float a = h1 ? h1[o + i] : 0.0f, b = h2[o + i];
    s1 = fmaf(a, a, s1);
    s2 = fmaf(b, b, s2);
  }
  const float inv1 = h1 ? inv_rms(block_sum(s1, red), D, n.eps) : 0.0f;
  const float inv2 = inv_rms(block_sum(s2, red), D, n.eps);
  float ss = 0.0f;
  for (int i = tid; i < D; i += kFuseThreads) {
    const float d1 = h1 ? bf16r(h1[o + i] * inv1 * bf16_bits_to_f32(n.post_dense[i])) : 0.0f;
    const float r = bf16r(h2[o + i] * inv2 * bf16_bits_to_f32(n.post_routed[i]));
    const float h12 = bf16r(d1 + r);
    row[i] = h12;
    ss = fmaf(h12, h12, ss);
  }
  const float inv12 = inv_rms(block_sum(ss, red), D, n.eps);
  const float scale = bf16r(n.layer_scalar);
  uint16_t* hr = hidden + static_cast<size_t>(t) * h_stride;
  for (int i = tid; i < D; i += kFuseThreads) {
    const float f = bf16r(row[i] * inv12 * bf16_bits_to_f32(n.post_ffn[i]));
    hr[i] = bf16b(bf16r(bf16_bits_to_f32(hr[i]) + f) * scale);
  }
}

}  // namespace

cudaError_t launch_gemma_setup(uint16_t* hidden, uint32_t h_stride, const uint16_t* attn,
                               uint32_t a_stride, int T, int D, const GemmaNorms& n,
                               uint16_t* router_x, uint16_t* routed_x, uint16_t* dense_x,
                               cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (D <= 0 || D > 4096) return cudaErrorInvalidValue;
  gemma_setup_kernel<<<T, kFuseThreads, static_cast<size_t>(D) * 4, s>>>(
      hidden, h_stride, attn, a_stride, D, n, router_x, routed_x, dense_x);
  return cudaGetLastError();
}

cudaError_t launch_gemma_tail(const float* h2, const float* h1, uint16_t* hidden, uint32_t h_stride,
                              int T, int D, const GemmaNorms& n, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (D <= 0 || D > 4096) return cudaErrorInvalidValue;
  gemma_tail_kernel<<<T, kFuseThreads, static_cast<size_t>(D) * 4, s>>>(h2, h1, hidden, h_stride,
                                                                         D, n);
  return cudaGetLastError();
}

}  // namespace tsg
