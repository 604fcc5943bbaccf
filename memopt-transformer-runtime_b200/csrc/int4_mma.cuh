// int4_mma.cuh — INT4 page consumption on the tensor cores (mma.sync
// m16n8k16, fp16 operands, fp32 accumulation) for the paged decode kernel.
//
// The decode of one query row is not a dense contraction, but doing its two
// skinny products on the tensor pipe removes most of the per-element ALU work
// that makes a CUDA-core INT4 loop issue-bound:
//   * scores: S[tok] = sum_d (code-8)[tok][d] * q[d] for the 16 tokens of an
//     m-tile.  A = codes (16 tokens x 16 dims per mma), B = q with column 0
//     holding the dims of scale group 0 and column 1 those of group 1, so one
//     mma yields both per-group partial dots; the fp32 per-(token, group)
//     scales are applied after the mma.  Products are exact: (code-8) and q
//     are fp16 values, (code-8) a small integer.
//   * P.V: O[d] += sum_tok P'[tok] (code-8)[tok][d] with A row 0 = p*scale of
//     group 0 and row 1 = p*scale of group 1 (fp16), B = V codes.
// Nibbles become fp16 with the 0x6400 exponent trick: the half with bits
// 0x6400 | n is 1024 + n exactly; subtracting 1032 gives n - 8 exactly.
// Reduction dims (k) may be permuted freely as long as both operands use
// the same permutation; the permutations below make every shared-memory
// access conflict-free.
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

// Same product when rows 8..15 of A are zero: only rows 0..7 of D are kept
// (d0, d1 accumulate in place), rows 8..15 go to scratch outputs and their
// accumulator inputs are a shared zero, so no register moves are needed.
__device__ __forceinline__ void mma16816_top(float& d0, float& d1, const uint32_t a[4], uint32_t b0, uint32_t b1) {
  float x2, x3;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%10,%10};"
      : "+f"(d0), "+f"(d1), "=f"(x2), "=f"(x3)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// Half2 (n_a - 8, n_b - 8) of the nibbles at bits [0,4) and [16,20) of x.
__device__ __forceinline__ uint32_t lo_pair(uint32_t x) {
  uint32_t h = (x & 0x000F000Fu) | 0x64006400u;  // 1024 + n, exactly
  const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), __half2half2(__ushort_as_half(0x6408)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Half2 (n_a - 8, n_b - 8) of the nibbles at bits [4,8) and [20,24) of x:
// the half 0x6400 | n << 4 is 1024 + 16 n, and (1024 + 16 n) / 16 - 72 = n - 8
// with a single exact fma.
__device__ __forceinline__ uint32_t hi_pair(uint32_t x) {
  uint32_t h = (x & 0x00F000F0u) | 0x64006400u;
  const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), __half2half2(__ushort_as_half(0x2C00)),
                            __half2half2(__ushort_as_half(0xD480)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace int4mma
}  // namespace memopt
