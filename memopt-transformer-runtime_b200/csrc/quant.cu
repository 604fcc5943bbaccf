// quant.cu — standalone INT4 quantize / dequantize over a flat fp16 tensor.
//
// Replaces quantize_int4_kernel / dequantize_int4_kernel
// (reference src/csrc/quantization.cu:104-203 and 232-270).  The reference
// launches one 64-thread CTA per 128-byte group; here 8 lanes share a group
// (16-byte vector loads, one 32-bit code word per lane) and a grid sized to
// the SM count strides over all groups, so the kernels are HBM-bound.
#include "int4.cuh"

namespace memopt {
namespace {

constexpr int kQuantThreads = 256;

// One lane = 16 consecutive elements (32 bytes in, 8 bytes of codes out),
// 4 lanes per group.
// At most 64 registers: four 256-thread CTAs per SM.  The next warp-stride's
// 32 bytes per lane are loaded while the current ones are converted and
// stored, so every lane keeps a load in flight.
__global__ void __launch_bounds__(kQuantThreads, 4)
quantize_int4_kernel(const uint4* __restrict__ in, uint2* __restrict__ codes,
                     float* __restrict__ scales, int64_t num_pairs) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // Every lane of a warp runs the same number of iterations (the loop runs
  // over whole warps) so the group shuffles always see all 32 lanes.
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t warp_first = first & ~int64_t(31);
  int64_t c = warp_first + (threadIdx.x & 31);
  uint4 a = make_uint4(0, 0, 0, 0), b = a;
  if (c < num_pairs) {
    a = ld_stream_v4(in + 2 * c);
    b = ld_stream_v4(in + 2 * c + 1);
  }
  for (int64_t base = warp_first; base < num_pairs; base += stride) {
    const int64_t cn = c + stride;
    uint4 an = make_uint4(0, 0, 0, 0), bn = an;
    if (cn < num_pairs) {
      an = ld_stream_v4(in + 2 * cn);
      bn = ld_stream_v4(in + 2 * cn + 1);
    }
    float scale;
    const uint2 w = int4_quant16(a, b, scale);
    if (c < num_pairs) {
      codes[c] = w;
      if ((c & 3) == 0) scales[c >> 2] = scale;
    }
    a = an;
    b = bn;
    c = cn;
  }
}

// One lane = one code word (8 outputs, one 16-byte store).
__global__ void __launch_bounds__(kQuantThreads)
dequantize_int4_kernel(const uint32_t* __restrict__ codes, const float* __restrict__ scales,
                       uint4* __restrict__ out, int64_t num_chunks) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < num_chunks;
       c += stride) {
    const uint32_t w = __ldg(codes + c);
    const float s = __ldg(scales + (c >> 3));
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int lo = static_cast<int>((w >> (8 * k)) & 0xF);
      const int hi = static_cast<int>((w >> (8 * k + 4)) & 0xF);
      // Reference: __float2half(static_cast<float>(q - 8) * scale).
      __half2 h = __halves2half2(__float2half_rn(static_cast<float>(lo - 8) * s),
                                 __float2half_rn(static_cast<float>(hi - 8) * s));
      ow[k] = *reinterpret_cast<uint32_t*>(&h);
    }
    out[c] = o;
  }
}

int grid_for(int64_t chunks) {
  const int64_t want = (chunks + kQuantThreads - 1) / kQuantThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace memopt

using namespace memopt;

extern "C" int memopt_quantize_int4(const void* input_f16, int64_t numel, int group_size,
                                    uint8_t* packed, float* scales, void* stream) {
  if (group_size != 64)
    return fail(MEMOPT_ERR_INVALID_ARG, "quantize_kv_cache_int4: group_size must equal 64");
  if (numel < 0 || numel % 64 != 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "quantize_kv_cache_int4: numel must be a multiple of 64");
  if (numel == 0) return MEMOPT_OK;
  if (!input_f16 || !packed || !scales)
    return fail(MEMOPT_ERR_INVALID_ARG, "quantize_kv_cache_int4: null pointer");
  if (!aligned16(input_f16) || (reinterpret_cast<uintptr_t>(packed) & 7u))
    return fail(MEMOPT_ERR_INVALID_ARG,
                "quantize_kv_cache_int4: input must be 16-byte aligned, packed 8-byte aligned");
  const int64_t pairs = numel / 16;
  quantize_int4_kernel<<<grid_for(pairs), kQuantThreads, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4*>(input_f16), reinterpret_cast<uint2*>(packed), scales, pairs);
  MEMOPT_LAUNCH_CHECK("quantize_int4_kernel launch");
  return MEMOPT_OK;
}

extern "C" int memopt_dequantize_int4(const uint8_t* packed, const float* scales, int64_t numel,
                                      int group_size, void* output_f16, void* stream) {
  if (group_size != 64)
    return fail(MEMOPT_ERR_INVALID_ARG, "dequantize_kv_cache_int4: group_size must equal 64");
  if (numel < 0) return fail(MEMOPT_ERR_INVALID_ARG, "dequantize_kv_cache_int4: negative numel");
  const int64_t groups = numel / 64;
  if (groups == 0) return MEMOPT_OK;
  if (!packed || !scales || !output_f16)
    return fail(MEMOPT_ERR_INVALID_ARG, "dequantize_kv_cache_int4: null pointer");
  if (!aligned16(output_f16) || (reinterpret_cast<uintptr_t>(packed) & 3u))
    return fail(MEMOPT_ERR_INVALID_ARG,
                "dequantize_kv_cache_int4: output must be 16-byte aligned, packed 4-byte aligned");
  const int64_t chunks = groups * 8;
  dequantize_int4_kernel<<<grid_for(chunks), kQuantThreads, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint32_t*>(packed), scales, reinterpret_cast<uint4*>(output_f16), chunks);
  MEMOPT_LAUNCH_CHECK("dequantize_int4_kernel launch");
  return MEMOPT_OK;
}
