// int4_mma.cuh — INT4 page consumption on the tensor cores (mma.sync) for
// the paged decode kernel.
//
// The decode of one query row is not a dense contraction, but doing its two
// skinny products on the tensor pipe removes most of the per-element ALU work
// that makes a CUDA-core INT4 loop issue-bound:
//   * scores (m16n8k32, s8 x s8 -> s32, exact): A = K codes as the signed
//     bytes 16 (code - 8) (16 tokens x 32 dims per mma, two ALU ops per four
//     codes), B = q rounded to 16-bit integers and split into two signed
//     bytes (hi, lo), one column per (scale group, half).  The integer sums
//     are exact; the per-(token, group) fp16 scales and the q scale are
//     applied once per token after the mma.
//   * P.V (m16n8k16, fp16, fp32 accumulation): O[d] += sum_tok
//     (code-8)[tok][d] * p[tok] * scale[tok][group(d)] with the 16 dims of a
//     block as rows of A (V codes) and B column g = p * scale of group g.
//     Nibbles become fp16 with the 0x6400 exponent trick: the half with bits
//     0x6400 | n is 1024 + n exactly; subtracting 1032 gives n - 8 exactly
//     (the offset is removed before the products, so the long fp32
//     accumulation over the context carries no large common term).
// Reduction dims (k) may be permuted freely as long as both operands use the
// same permutation; the permutations used make the shared-memory reads
// conflict-free.
#pragma once
#include "common.cuh"

namespace memopt {
namespace int4mma {

__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d = (a & b) | c and d = (a & b) ^ c as one three-input logic op.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Half2 (n_a - 8, n_b - 8) of the nibbles at bits [0,4) and [16,20) of x
// (k_f16 = 0x64006400): the half 0x6400 | n is 1024 + n exactly.
__device__ __forceinline__ uint32_t lo_pair(uint32_t x, uint32_t k_f16) {
  uint32_t h = and_or(x, 0x000F000Fu, k_f16);
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), __half2half2(__ushort_as_half(0x6408)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Half2 (n_a - 8, n_b - 8) of the nibbles at bits [4,8) and [20,24) of x:
// the half 0x6400 | n << 4 is 1024 + 16 n, and (1024 + 16 n) / 16 - 72 = n - 8
// with a single exact fma.
__device__ __forceinline__ uint32_t hi_pair(uint32_t x, uint32_t k_f16) {
  uint32_t h = and_or(x, 0x00F000F0u, k_f16);
  const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), __half2half2(__ushort_as_half(0x2C00)),
                            __half2half2(__ushort_as_half(0xD480)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Integer product m16n8k32, signed 8-bit operands, exact int32 accumulation.
__device__ __forceinline__ void mma_s8(int c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four codes of a word as signed bytes 16 (n - 8) (k_s8 = 0x80808080):
// placing the nibble in the high half of a byte and flipping its top bit gives
// the two's complement of 16 (n - 8) exactly.  Even elements (low nibbles) /
// odd elements (high nibbles).
__device__ __forceinline__ uint32_t s8x16_even(uint32_t w, uint32_t k_s8) { return and_xor(w << 4, 0xF0F0F0F0u, k_s8); }
__device__ __forceinline__ uint32_t s8x16_odd(uint32_t w, uint32_t k_s8) { return and_xor(w, 0xF0F0F0F0u, k_s8); }

// Half2 (1024 + n_a, 1024 + n_b) of the nibbles at bits [0,4) and [16,20),
// and (1024 + 16 n_a, 1024 + 16 n_b) of those at [4,8) and [20,24): one logic
// op each, the offsets are removed after the products.
__device__ __forceinline__ uint32_t lo_raw(uint32_t x, uint32_t k_f16) { return and_or(x, 0x000F000Fu, k_f16); }
__device__ __forceinline__ uint32_t hi_raw(uint32_t x, uint32_t k_f16) { return and_or(x, 0x00F000F0u, k_f16); }

// 2^x with the hardware approximation (relative error ~2^-22; -inf -> 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace int4mma
}  // namespace memopt
