// write_cache.cu — scatter of new K/V tokens into the paged pool.
//
// Replaces write_cache_kernel (reference src/csrc/kv_cache.cu:228-260): the
// reference moves one 2-byte element per thread with one CTA per token.  Here
// one warp owns a token row and moves it with 16-byte vector accesses (a token
// row of the reference layout [block, pos, head, dim] is contiguous in both
// the input and the pool), several loads in flight per lane.
//
// The INT4 variant quantises while it writes (no reference counterpart for
// the fusion; the per-group arithmetic follows quantization.cu:129-202) into
// the INT4 page format: one contiguous page per (block, head) holding
// [K codes | V codes | K scales | V scales], so a decode step moves each page
// with a single bulk copy.
#include "int4.cuh"

namespace memopt {
namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kUnroll = 4;

__device__ __forceinline__ bool slot_ok(int32_t slot, int64_t num_slots) {
  return slot >= 0 && static_cast<int64_t>(slot) < num_slots;
}

// Token rows of `chunks` 16-byte pieces; one warp per token.
__global__ void __launch_bounds__(kWarpsPerCta * 32)
write_cache_f16_kernel(const uint4* __restrict__ keys, const uint4* __restrict__ values,
                       const int32_t* __restrict__ slots, int64_t num_tokens, int chunks,
                       uint4* __restrict__ kpool, uint4* __restrict__ vpool, int64_t num_slots,
                       int32_t* __restrict__ bad) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerCta;
  for (int64_t t = warp; t < num_tokens; t += nwarps) {
    const int32_t slot = __ldg(slots + t);
    if (!slot_ok(slot, num_slots)) {
      if (lane == 0 && bad) atomicAdd(bad, 1);
      continue;
    }
    const uint4* ksrc = keys + t * chunks;
    const uint4* vsrc = values + t * chunks;
    uint4* kdst = kpool + static_cast<int64_t>(slot) * chunks;
    uint4* vdst = vpool + static_cast<int64_t>(slot) * chunks;
    for (int c0 = lane; c0 < chunks; c0 += 32 * kUnroll) {
      uint4 kv[kUnroll], vv[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32;
        if (c < chunks) {
          kv[u] = ld_stream_v4(ksrc + c);
          vv[u] = ld_stream_v4(vsrc + c);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32;
        if (c < chunks) {
          kdst[c] = kv[u];
          vdst[c] = vv[u];
        }
      }
    }
  }
}

// Generic element-wise scatter for rows that are not a multiple of 16 bytes
// or not 16-byte aligned.
__global__ void write_cache_f16_scalar_kernel(const __half* __restrict__ keys,
                                              const __half* __restrict__ values,
                                              const int32_t* __restrict__ slots,
                                              int64_t num_tokens, int row,
                                              __half* __restrict__ kpool,
                                              __half* __restrict__ vpool, int64_t num_slots,
                                              int32_t* __restrict__ bad) {
  for (int64_t t = blockIdx.x; t < num_tokens; t += gridDim.x) {
    const int32_t slot = slots[t];
    if (!slot_ok(slot, num_slots)) {
      if (threadIdx.x == 0 && bad) atomicAdd(bad, 1);
      continue;
    }
    for (int i = threadIdx.x; i < row; i += blockDim.x) {
      kpool[static_cast<int64_t>(slot) * row + i] = keys[t * row + i];
      vpool[static_cast<int64_t>(slot) * row + i] = values[t * row + i];
    }
  }
}

// One warp per token; 4 lanes per 64-element group (16 elements = two
// 16-byte vectors each), 8 groups per warp step.  A lane stores 8 bytes of K
// codes and 8 of V codes (a group's 32-byte code row is written whole by its
// 4 lanes); the group's first lane stores the two fp16 scales.  head_dim is
// a template parameter (64 or 128), so the group -> (head, group in head)
// split is a shift; other multiples of 64 take D = 0 (run-time division).
constexpr int kInt4WriteWarps = 8;

template <int D>
__global__ void __launch_bounds__(kInt4WriteWarps * 32, 3)
write_cache_int4_kernel(const uint4* __restrict__ keys, const uint4* __restrict__ values,
                        const int32_t* __restrict__ slots, int64_t num_tokens, int num_heads,
                        int head_dim_rt, int block_size, int64_t num_slots,
                        uint8_t* __restrict__ pages, int64_t page_bytes, int32_t* __restrict__ bad) {
  const int head_dim = D > 0 ? D : head_dim_rt;
  const int lane = threadIdx.x & 31;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kInt4WriteWarps + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kInt4WriteWarps;
  const int gpr = head_dim / 64;                // groups per (token, head)
  const int chunks = num_heads * head_dim / 8;  // 16-byte chunks per token row
  const int64_t codes_bytes = static_cast<int64_t>(block_size) * (head_dim / 2);
  const int64_t scale_bytes = static_cast<int64_t>(block_size) * gpr * 2;
  for (int64_t t = warp; t < num_tokens; t += nwarps) {
    const int32_t slot = __ldg(slots + t);
    if (!slot_ok(slot, num_slots)) {
      if (lane == 0 && bad) atomicAdd(bad, 1);
      continue;
    }
    const int64_t blk = slot / block_size;
    const int pos = slot - static_cast<int32_t>(blk * block_size);
    const uint4* ksrc = keys + t * chunks;
    const uint4* vsrc = values + t * chunks;
    uint8_t* page0 = pages + blk * num_heads * page_bytes;
    const int64_t row = static_cast<int64_t>(pos) * (head_dim / 2);
    // chunks is a multiple of 8 (head_dim % 64 == 0): a group's 4 lanes are
    // all live or all idle, and every lane runs the same trip count.
    for (int c0 = 0; c0 < chunks; c0 += 64) {
      const int c = c0 + 2 * lane;
      uint4 ka = make_uint4(0, 0, 0, 0), kb = ka, va = ka, vb = ka;
      if (c < chunks) {
        ka = ld_stream_v4(ksrc + c);
        kb = ld_stream_v4(ksrc + c + 1);
        va = ld_stream_v4(vsrc + c);
        vb = ld_stream_v4(vsrc + c + 1);
      }
      float sk, sv;
      const uint2 wk = int4_quant16(ka, kb, sk);
      const uint2 wv = int4_quant16(va, vb, sv);
      if (c < chunks) {
        const int g = c >> 3;  // group within the token row
        const int h = D == 128 ? (g >> 1) : (D == 64 ? g : g / gpr);
        const int gi = g - h * gpr;
        uint8_t* page = page0 + h * page_bytes;
        const int byte = gi * 32 + (c & 7) * 4;  // logical byte of the row (c even: 8-byte aligned)
        *reinterpret_cast<uint2*>(page + row + byte) = wk;
        *reinterpret_cast<uint2*>(page + codes_bytes + row + int4_vrow_swizzle(pos, byte, head_dim)) = wv;
        if ((c & 7) == 0) {
          __half* ks = reinterpret_cast<__half*>(page + 2 * codes_bytes);
          __half* vs = reinterpret_cast<__half*>(page + 2 * codes_bytes + scale_bytes);
          ks[pos * gpr + gi] = __float2half_rn(sk);
          vs[int4_vscale_index(pos, gi, gpr)] = __float2half_rn(sv);
        }
      }
    }
  }
}

int grid_for_tokens(int64_t num_tokens) {
  const int64_t want = (num_tokens + kWarpsPerCta - 1) / kWarpsPerCta;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace memopt

using namespace memopt;

extern "C" int memopt_write_cache_f16(const void* keys, const void* values,
                                      const int32_t* slot_mapping, int64_t num_tokens,
                                      int num_heads, int head_dim, void* key_pool,
                                      void* value_pool, int64_t num_blocks, int block_size,
                                      int32_t* bad_slot_count, void* stream) {
  if (num_tokens < 0 || num_heads <= 0 || head_dim <= 0 || num_blocks < 0 || block_size <= 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "write_cache: invalid geometry");
  if (block_size % 16 != 0)
    return fail(MEMOPT_ERR_UNSUPPORTED, "write_cache_int4: block_size must be a multiple of 16");
  if (num_tokens == 0) return MEMOPT_OK;
  if (!keys || !values || !slot_mapping || !key_pool || !value_pool)
    return fail(MEMOPT_ERR_INVALID_ARG, "write_cache: null pointer");
  const int64_t num_slots = num_blocks * block_size;
  const int row = num_heads * head_dim;
  cudaStream_t s = as_stream(stream);
  if (row % 8 == 0 && aligned16(keys) && aligned16(values) && aligned16(key_pool) &&
      aligned16(value_pool)) {
    write_cache_f16_kernel<<<grid_for_tokens(num_tokens), kWarpsPerCta * 32, 0, s>>>(
        reinterpret_cast<const uint4*>(keys), reinterpret_cast<const uint4*>(values), slot_mapping,
        num_tokens, row / 8, reinterpret_cast<uint4*>(key_pool), reinterpret_cast<uint4*>(value_pool),
        num_slots, bad_slot_count);
  } else {
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    write_cache_f16_scalar_kernel<<<static_cast<int>(num_tokens < cap ? num_tokens : cap), 256, 0, s>>>(
        reinterpret_cast<const __half*>(keys), reinterpret_cast<const __half*>(values), slot_mapping,
        num_tokens, row, reinterpret_cast<__half*>(key_pool), reinterpret_cast<__half*>(value_pool),
        num_slots, bad_slot_count);
  }
  MEMOPT_LAUNCH_CHECK("write_cache_f16 launch");
  return MEMOPT_OK;
}

extern "C" size_t memopt_int4_page_bytes(int block_size, int head_dim) {
  if (block_size <= 0 || head_dim <= 0 || head_dim % 64 != 0) return 0;
  return static_cast<size_t>(block_size) * head_dim + static_cast<size_t>(block_size) * (head_dim / 64) * 4;
}

extern "C" int memopt_write_cache_int4(const void* keys, const void* values,
                                       const int32_t* slot_mapping, int64_t num_tokens,
                                       int num_heads, int head_dim, uint8_t* kv_pages,
                                       int64_t num_blocks, int block_size,
                                       int32_t* bad_slot_count, void* stream) {
  if (num_tokens < 0 || num_heads <= 0 || head_dim <= 0 || num_blocks < 0 || block_size <= 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "write_cache_int4: invalid geometry");
  if (head_dim % 64 != 0)
    return fail(MEMOPT_ERR_UNSUPPORTED, "write_cache_int4: head_dim must be a multiple of 64");
  if (num_tokens == 0) return MEMOPT_OK;
  if (!keys || !values || !slot_mapping || !kv_pages)
    return fail(MEMOPT_ERR_INVALID_ARG, "write_cache_int4: null pointer");
  if (!aligned16(keys) || !aligned16(values) || !aligned16(kv_pages))
    return fail(MEMOPT_ERR_INVALID_ARG, "write_cache_int4: misaligned pointer");
  const int64_t want = (num_tokens + kInt4WriteWarps - 1) / kInt4WriteWarps;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 3;
  const int grid = static_cast<int>(want < cap ? want : cap);
  auto kern = head_dim == 128 ? write_cache_int4_kernel<128>
                              : (head_dim == 64 ? write_cache_int4_kernel<64> : write_cache_int4_kernel<0>);
  kern<<<grid, kInt4WriteWarps * 32, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4*>(keys), reinterpret_cast<const uint4*>(values), slot_mapping,
      num_tokens, num_heads, head_dim, block_size, num_blocks * block_size, kv_pages,
      static_cast<int64_t>(memopt_int4_page_bytes(block_size, head_dim)), bad_slot_count);
  MEMOPT_LAUNCH_CHECK("write_cache_int4 launch");
  return MEMOPT_OK;
}
