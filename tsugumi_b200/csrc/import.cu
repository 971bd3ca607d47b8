// Import of one int4 matrix of a .moepack expert blob into this library's
// layout, on the device.
//
// A .moepack expert carries each projection in the MLX affine layout
// (MoEPackPackedExpertsLayoutV1.swift, RepackPlanner.swift:440-470): codes as
// U32 words [rows][cols / 8] (element k of a row in bits 4 (k % 8) of word
// k / 8), BF16 scales [rows][cols / group] and, unless the blob is `sym`,
// BF16 biases.  The kernels here read codes as bytes (low nibble = even
// element: the same bytes, little-endian) and one fp16 scale per 32-group, and
// implement the symmetric scheme w = s (q - 8).  The import is exact or
// fails:
//   * every BF16 scale must be an fp16 value (a BF16 value has 8 significant
//     bits, so it is one whenever its exponent is in fp16's range -- the
//     case for int4 group scales), converted without rounding;
//   * a group of g > 32 elements gives its scale to each of its g / 32
//     32-groups (the same products);
//   * biases, when given, must be -8 x scale as a BF16 bit pattern, the
//     identity of the symmetric scheme (MoEPackAffineV1.swift:14-26).
// A failure is recorded in the context's error word (code 10: scale, code
// 11: bias; value: the group index) and reported by tsg_sync.

#include "tsg_common.cuh"
#include "tsg_kernels.cuh"

namespace tsg {
namespace {

TSG_DEV void record_import_error(uint32_t* err, uint32_t code, uint32_t value) {
  if (!err) return;
  atomicOr(err, TSG_DEVERR_METADATA);
  if (atomicCAS(err + 1, 0u, code) == 0u) err[2] = value;
}

// -8 x scale in BF16 from BF16 bits, rounded to nearest even (a power-of-two
// product: exact for every finite scale).
TSG_DEV uint16_t symmetric_bias_bits(uint16_t s) {
  const float v = __uint_as_float(static_cast<uint32_t>(s) << 16) * -8.0f;
  const uint32_t b = __float_as_uint(v);
  return static_cast<uint16_t>((b + 0x7FFFu + ((b >> 16) & 1u)) >> 16);
}

__global__ void import_codes_kernel(const uint4* src, uint4* dst, size_t n16) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

__global__ void import_scales_kernel(const uint16_t* scales, const uint16_t* biases, int rows,
                                     int groups_in, int per, __half* out, uint32_t* err) {
  const size_t n = static_cast<size_t>(rows) * groups_in;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint16_t sb = scales[i];
    const float s = __uint_as_float(static_cast<uint32_t>(sb) << 16);
    const __half h = __float2half_rn(s);
    if (__half2float(h) != s) record_import_error(err, 10u, static_cast<uint32_t>(i));
    if (biases && biases[i] != symmetric_bias_bits(sb))
      record_import_error(err, 11u, static_cast<uint32_t>(i));
    for (int k = 0; k < per; ++k) out[i * per + k] = h;
  }
}

}  // namespace

cudaError_t launch_import_int4(const void* codes, const uint16_t* scales, const uint16_t* biases,
                               int rows, int cols, int group, void* out_codes, __half* out_scales,
                               uint32_t* err, cudaStream_t s) {
  if (rows <= 0 || cols <= 0 || cols % 32 || group % 32 || cols % group)
    return cudaErrorInvalidValue;
  const size_t bytes = static_cast<size_t>(rows) * cols / 2;
  if (bytes % 16 || (reinterpret_cast<uintptr_t>(codes) | reinterpret_cast<uintptr_t>(out_codes)) & 15u)
    return cudaErrorInvalidValue;
  import_codes_kernel<<<592, 256, 0, s>>>(static_cast<const uint4*>(codes),
                                          static_cast<uint4*>(out_codes), bytes / 16);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  import_scales_kernel<<<592, 256, 0, s>>>(scales, biases, rows, cols / group, group / 32,
                                           out_scales, err);
  return cudaGetLastError();
}

}  // namespace tsg
