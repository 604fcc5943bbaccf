// int4.cuh — group-64 symmetric INT4 arithmetic shared by the standalone
// quantizer and the fused write_cache.
//
// Per group (reference src/csrc/quantization.cu:129-202):
//   absmax = max |x|            (fmaxf semantics: NaN inputs are ignored)
//   scale  = absmax > 0 ? absmax / 7.0f : 1.0f       (IEEE fp32 division)
//   q      = clamp((int)roundf(x / scale) + 8, 0, 15) (roundf: ties away)
//   byte i = q[2i] | q[2i+1] << 4                      (low nibble = even)
// A group of 64 fp16 values is handled by 4 consecutive lanes, 16 values
// (32 bytes) each; lanes 4k..4k+3 must all be present for the shuffles.
#pragma once
#include "common.cuh"

namespace memopt {

__device__ __forceinline__ void unpack_half8(const uint4& v, float f[8]) {
  const __half2* h2 = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h2[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ float int4_scale_from_absmax(float absmax) {
  return (absmax > 0.f) ? (absmax / 7.0f) : 1.0f;
}

// One code, bit-exact with the reference.  The C-style float->int conversion
// is cvt.rzi.s32.f32 (saturating, NaN -> 0), exactly as in the reference.
__device__ __forceinline__ uint32_t int4_code(float x, float scale) {
  int iq = static_cast<int>(roundf(x / scale)) + 8;
  return static_cast<uint32_t>(min(max(iq, 0), 15));
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Max with NaN propagation: NaN if either input is NaN (fmaxf would skip it).
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// absmax / 7 for a finite absmax m >= 0 without the division routine:
// q0 = m * fp32(1/7) followed by one residual correction step
// q = fma(fma(-q0, 7, m), fp32(1/7), q0) (Markstein's correction for
// division by a constant: P. Markstein, "IA-64 and Elementary Functions",
// Prentice Hall 2000, ch. 8) is the correctly rounded quotient for every
// finite fp16 value m (checked exhaustively over all 31743 positive finite
// fp16 values against the IEEE fp32 quotient; m is the max of |fp16| inputs).
// 1.0 for an all-zero group, as in the reference.
__device__ __forceinline__ float int4_scale_div7(float m) {
  float scale = 1.0f;
  if (m > 0.f) {
    const float r7 = 0.142857149f;  // fp32(1/7)
    const float q0 = __fmul_rn(m, r7);
    scale = __fmaf_rn(__fmaf_rn(-q0, 7.0f, m), r7, q0);
  }
  return scale;
}

// The lane's 16 codes of a group of 64 shared by 4 consecutive lanes (16
// elements each, given as two 16-byte vectors a, b in element order) and the
// group's scale, bit-identical to int4_scale_from_absmax(absmax) and
// int4_code.  Returned as two code words (byte i = code 2i | code 2i+1 << 4).
// The group max is taken on the fp16 pairs (exact; NaN propagates), a group
// holding a NaN or an infinity takes the reference path.  Otherwise, with
// q = x * rcp(scale) (exact product, within 2e-6 of x / scale, |q| <= 7 +
// rounding), fma(x, rcp, 2^23 + 8) puts 8 + rint(q) in the low byte of its
// bit pattern; rint (ties to even) and the reference's roundf (ties away)
// of x / scale can only differ when q is within 1.6e-5 of a half-integer,
// which |q - rint(q)| shows, and then those codes are recomputed with the
// exact division.  Bytes are gathered with byte permutes and the two nibbles
// of each output byte joined by one shift-add.
__device__ __forceinline__ uint2 int4_quant16(const uint4& a, const uint4& b, float& scale_out) {
  const __half2* ha = reinterpret_cast<const __half2*>(&a);
  const __half2* hb = reinterpret_cast<const __half2*>(&b);
  __half2 m2 = __habs2(ha[0]);
#pragma unroll
  for (int i = 1; i < 4; ++i) m2 = __hmax2_nan(m2, __habs2(ha[i]));
#pragma unroll
  for (int i = 0; i < 4; ++i) m2 = __hmax2_nan(m2, __habs2(hb[i]));
  float m = fmax_nan(__low2float(m2), __high2float(m2));
  m = fmax_nan(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmax_nan(m, __shfl_xor_sync(0xffffffffu, m, 2));
  float f[16];
  unpack_half8(a, f);
  unpack_half8(b, f + 8);
  uint32_t w0 = 0, w1 = 0;
  if (!(m < INFINITY)) {  // NaN or inf in the group (uniform over its 4 lanes)
    float am = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) am = fmaxf(am, fabsf(f[j]));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    const float scale = int4_scale_from_absmax(am);
    scale_out = scale;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      w0 |= int4_code(f[j], scale) << (4 * j);
      w1 |= int4_code(f[8 + j], scale) << (4 * j);
    }
    return make_uint2(w0, w1);
  }
  const float scale = int4_scale_div7(m);
  scale_out = scale;
  const float rinv = rcp_approx(scale);
  constexpr float kMagic = 8388616.0f;  // 2^23 + 8
  constexpr float kNearHalf = 0.5f - 1.6e-5f;
  uint32_t u[16];
  float dmax = 0.f;
  const uint64_t rinv2 = f32x2_pack(rinv, rinv), magic2 = f32x2_pack(kMagic, kMagic);
#pragma unroll
  for (int j = 0; j < 16; j += 2) {
    // Per element (two at a time, packed fp32 ops; each lane of a packed op
    // rounds as the scalar one): t = RN(x rinv + 2^23 + 8) = 2^23 + 8 +
    // rint(x rinv) (unit spacing there); d = RN(x rinv - rint(x rinv)), the
    // distance to the chosen integer.
    const uint64_t x2 = f32x2_pack(f[j], f[j + 1]);
    const uint64_t t2 = f32x2_fma(x2, rinv2, magic2);
    const uint64_t d2 = f32x2_fma(x2, rinv2, f32x2_sub(magic2, t2));
    float t0, t1, d0, d1;
    f32x2_unpack(t2, t0, t1);
    f32x2_unpack(d2, d0, d1);
    u[j] = __float_as_uint(t0);
    u[j + 1] = __float_as_uint(t1);
    dmax = fmaxf(dmax, fmaxf(fabsf(d0), fabsf(d1)));
  }
  if (dmax >= kNearHalf) {
    // Rare per lane (about 0.8% of lanes on N(0,1) data, mostly exact ties
    // x / scale = n + 1/2), but it diverges the warp: only the flagged
    // elements take the exact division, and the low byte of u[j] is patched.
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float t = __fmaf_rn(f[j], rinv, kMagic);
      if (fabsf(__fmaf_rn(f[j], rinv, kMagic - t)) >= kNearHalf)
        u[j] = (u[j] & 0xFFFFFF00u) | int4_code(f[j], scale);
    }
  }
  // low byte of u[j] = code j
  const uint32_t e0 = __byte_perm(__byte_perm(u[0], u[2], 0x0040), __byte_perm(u[4], u[6], 0x0040), 0x5410);
  const uint32_t o0 = __byte_perm(__byte_perm(u[1], u[3], 0x0040), __byte_perm(u[5], u[7], 0x0040), 0x5410);
  const uint32_t e1 = __byte_perm(__byte_perm(u[8], u[10], 0x0040), __byte_perm(u[12], u[14], 0x0040), 0x5410);
  const uint32_t o1 = __byte_perm(__byte_perm(u[9], u[11], 0x0040), __byte_perm(u[13], u[15], 0x0040), 0x5410);
  return make_uint2((o0 << 4) + e0, (o1 << 4) + e1);
}

// INT4 page layout helpers (one page per (block, head)):
//   [K codes BS*D/2 | V codes BS*D/2 | K scales BS*(D/64) fp16 | V scales]
// K row pos holds byte i = q[2i] | q[2i+1] << 4 at byte i.  The V row holds
// the same bytes, but for D == 128 byte i sits at i ^ 32 when bit 1 of pos is
// set (the decode reads rows t and t+2 of a tile in one shared-memory
// instruction; the exchange puts them in different banks).  K scales are
// [BS][D/64]; V scales, per 16-token tile, [D/64][16] with token r of the
// tile at slot 2(r & 3) + ((r >> 2) & 1) + 8(r >> 3), which puts the tokens
// (t, t+4) and (t+8, t+12) that one decode lane pairs next to each other.
__host__ __device__ __forceinline__ int int4_vrow_swizzle(int pos, int byte, int head_dim) {
  return (head_dim == 128 && (pos & 2)) ? (byte ^ 32) : byte;
}
__host__ __device__ __forceinline__ int int4_vscale_index(int pos, int group, int groups) {
  const int r = pos & 15;
  return ((pos >> 4) * groups + group) * 16 + 2 * (r & 3) + ((r >> 2) & 1) + 8 * (r >> 3);
}

}  // namespace memopt
