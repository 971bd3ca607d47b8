// int4_mma.cuh -- int4 weights dequantised in registers for mma.sync
// m16n8k16 (fp16 operands, fp32 accumulate), shared by the register-resident
// decode kernels.
//
// A thread of the MMA (lane = 4 g + c) reads one whole 32-element group of
// a weight row with one 16-byte load -- group 4 s + c of a super-group s of
// 4 groups -- so each MMA mixes the four groups of a super-group; the token
// operand follows the same permutation of K (within each 8 elements:
// (x0,x4), (x2,x6), (x1,x5), (x3,x7)), so the dot products are unchanged.
// A code word holds elements e0..e7 (e_{2i} in the low nibble of byte i);
// (w & 0x000F000F) | 0x64006400 is the fp16 pair (1024 + q0, 1024 + q4), the
// 0x00F000F0 mask gives (1024 + 16 q1, 1024 + 16 q5), the same on w >> 8
// gives elements 2, 6 and 3, 7; subtracting 1032 (or 1152) is exact, and a
// multiply by the group's scale (or scale / 16) rounds once: fp16 s (q - 8).
#pragma once

#include <cuda_fp16.h>

#include "tsg_common.cuh"

namespace tsg {

TSG_DEV void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (a & b) | c in one instruction.
TSG_DEV uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

TSG_DEV uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
TSG_DEV __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// A code word as four scaled fp16 pairs s (q - 8):
// p[0] = (e0,e4), p[1] = (e2,e6), p[2] = (e1,e5), p[3] = (e3,e7).
// s2 = (s, s), s16 = (s / 16, s / 16).
TSG_DEV void dequant_word(uint32_t w, __half2 s2, __half2 s16, uint32_t (&p)[4]) {
  const uint32_t w8 = w >> 8;
  const __half2 lo_off = bits_h2(0x64086408u);  // (1032, 1032)
  const __half2 hi_off = bits_h2(0x64806480u);  // (1152, 1152)
  p[0] = h2_bits(__hmul2(__hsub2(bits_h2(and_or(w, 0x000F000Fu, 0x64006400u)), lo_off), s2));
  p[1] = h2_bits(__hmul2(__hsub2(bits_h2(and_or(w8, 0x000F000Fu, 0x64006400u)), lo_off), s2));
  p[2] = h2_bits(__hmul2(__hsub2(bits_h2(and_or(w, 0x00F000F0u, 0x64006400u)), hi_off), s16));
  p[3] = h2_bits(__hmul2(__hsub2(bits_h2(and_or(w8, 0x00F000F0u, 0x64006400u)), hi_off), s16));
}

TSG_DEV void scale_pair(const __half* s, __half2* s2, __half2* s16) {
  const __half h = *s;
  *s2 = __halves2half2(h, h);
  *s16 = __hmul2(*s2, bits_h2(0x2C002C00u));  // (s / 16, s / 16), exact
}

// Eight consecutive fp16 values (one 16-byte load, natural order) as the B
// fragment chunk of the permuted K order: (x0,x4), (x2,x6), (x1,x5), (x3,x7).
TSG_DEV uint4 frag_from_row(uint4 v) {
  return make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.y, v.w, 0x5410),
                    __byte_perm(v.x, v.z, 0x7632), __byte_perm(v.y, v.w, 0x7632));
}

}  // namespace tsg
