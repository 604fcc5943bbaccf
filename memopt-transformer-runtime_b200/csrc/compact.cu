// compact.cu — exact sink-aware top-k eviction with physical compaction.
//
// No reference counterpart: the reference's evict_tokens picks a threshold by
// 32 bisection steps, evicts nothing at all when sinks are present, zeroes
// only part of an evicted row and never releases a page (kv_cache.cu:714-1014).
// This operator delivers the memory saving that eviction is meant to give,
// for one shared decision per sequence (pages hold every head of a token, so
// only a decision shared across heads can free pages):
//   * token score = sum over heads of scores[b, h, t] (fp32, heads in order);
//   * tokens t < num_sink_tokens are always kept; tokens at or past the
//     context length, or on a page whose table entry is < 0 or >= num_blocks,
//     are never kept (they hold no data);
//   * keep = max(1, min(L, ceil(r * L))) with L the number of valid tokens
//     (the reference's keep formula); the keep tokens with the largest scores
//     survive, ties broken by lower token index, NaN ranking lowest; the
//     selection is exact (radix select over order-preserving integer keys);
//   * the kept K/V rows (all heads) move in token order to positions
//     0..keep-1 over the sequence's valid pages; the block-table row becomes
//     those first ceil(keep / block_size) valid pages (then -1), the others
//     are reported as freed, and context_lens[b] becomes keep.
// Four launches: head sums (parallel over tokens), one CTA per sequence for
// the select + compaction indices, then a gather of the kept rows into the
// workspace and a scatter back (in place the moves would race: a token's
// destination can be an earlier token's source).
#include "common.cuh"
#include "memopt_b200.h"

namespace memopt {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kMaxLen = 32768;
constexpr int kVPT = kMaxLen / kSelThreads;  // 32 tokens per thread

__global__ void head_sum_kernel(const float* __restrict__ scores, int H, int max_len, float* __restrict__ sums) {
  const int b = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= max_len) return;
  const float* src = scores + static_cast<int64_t>(b) * H * max_len + t;
  float s = 0.f;
  for (int h = 0; h < H; ++h) s += __ldg(src + static_cast<int64_t>(h) * max_len);
  sums[static_cast<int64_t>(b) * max_len + t] = s;
}

// Order-preserving key of a float (larger float -> larger key); NaN -> 0.
__device__ __forceinline__ uint32_t score_key(float f) {
  if (f != f) return 0u;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ int block_excl_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();  // warp_sums may still be read by a previous scan
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  int w = lane < (kSelThreads / 32) ? warp_sums[lane] : 0;
  int winc = w;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, winc, o);
    if (lane >= o) winc += n;
  }
  const int woff = __shfl_sync(0xffffffffu, winc - w, warp);
  if (total) *total = __shfl_sync(0xffffffffu, winc, 31);
  return woff + incl - v;
}

__global__ void __launch_bounds__(kSelThreads, 1)
topk_select_kernel(const float* __restrict__ sums, int max_len, int32_t* __restrict__ bt, int MB,
                   int32_t* __restrict__ ctx_lens, int NB, int BS, float retain_ratio, int num_sinks,
                   int32_t* __restrict__ kept_idx, int32_t* __restrict__ kept_count,
                   int32_t* __restrict__ freed, int32_t* __restrict__ freed_count) {
  __shared__ int hist[256];
  __shared__ int warp_sums[32];
  __shared__ uint32_t sh_prefix;
  __shared__ int sh_remaining;
  const int b = blockIdx.x, tid = threadIdx.x;
  int32_t* btrow = bt + static_cast<int64_t>(b) * MB;
  const int L = min(max(ctx_lens[b], 0), max_len);
  const int t0 = tid * kVPT;

  // Valid tokens: below L and on a valid page.
  uint32_t key[kVPT];
  uint32_t valid = 0;  // bit i <-> token t0 + i
#pragma unroll
  for (int i = 0; i < kVPT; ++i) {
    const int t = t0 + i;
    key[i] = 0u;
    if (t < L) {
      const int lb = t / BS;
      const int pg = lb < MB ? btrow[lb] : -1;
      if (pg >= 0 && pg < NB) {
        valid |= 1u << i;
        key[i] = t < num_sinks ? 0xFFFFFFFFu : score_key(sums[static_cast<int64_t>(b) * max_len + t]);
      }
    }
  }
  int nvalid = 0;
  const int nval_thread = __popc(valid);
  block_excl_scan(nval_thread, warp_sums, &nvalid);
  const int keep = nvalid == 0 ? 0 : max(1, min(nvalid, static_cast<int>(ceilf(retain_ratio * static_cast<float>(nvalid)))));

  // Radix select of the keep-th largest key, 8 bits per pass from the top.
  if (tid == 0) {
    sh_prefix = 0u;
    sh_remaining = keep;
  }
  uint32_t prefix_mask = 0u;
  for (int pass = 0; pass < 4 && keep > 0; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = sh_prefix;
#pragma unroll
    for (int i = 0; i < kVPT; ++i)
      if (((valid >> i) & 1u) && (key[i] & prefix_mask) == prefix) atomicAdd(&hist[(key[i] >> shift) & 0xFFu], 1);
    __syncthreads();
    if (tid < 32) {
      // Warp 0: find the digit where the count from the top reaches remaining.
      const int rem = sh_remaining;
      int c[8];
      int part = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        c[k] = hist[255 - (tid * 8 + k)];
        part += c[k];
      }
      int incl = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += n;
      }
      int above = incl - part;  // count in digits higher than this lane's first
      int found_digit = -1, found_above = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (found_digit < 0 && above + c[k] >= rem) {
          found_digit = 255 - (tid * 8 + k);
          found_above = above;
        }
        above += c[k];
      }
      const unsigned m = __ballot_sync(0xffffffffu, found_digit >= 0);
      const int src = __ffs(m) - 1;
      const int dig = __shfl_sync(0xffffffffu, found_digit, src);
      const int abv = __shfl_sync(0xffffffffu, found_above, src);
      if (tid == 0) {
        sh_prefix = prefix | (static_cast<uint32_t>(dig) << shift);
        sh_remaining = rem - abv;
      }
    }
    prefix_mask |= 0xFFu << shift;
    __syncthreads();
  }
  const uint32_t T = sh_prefix;
  const int need_eq = sh_remaining;  // tokens with key == T to keep (the first ones)

  // Kept flags: key > T, or key == T within the first need_eq of them.
  uint32_t eq = 0;
#pragma unroll
  for (int i = 0; i < kVPT; ++i)
    if (((valid >> i) & 1u) && key[i] == T) eq |= 1u << i;
  const int eq_before = block_excl_scan(__popc(eq), warp_sums, nullptr);
  uint32_t kept = 0;
  int eq_rank = eq_before;
#pragma unroll
  for (int i = 0; i < kVPT; ++i) {
    if (!((valid >> i) & 1u) || keep == 0) continue;
    if (key[i] > T) {
      kept |= 1u << i;
    } else if ((eq >> i) & 1u) {
      if (eq_rank < need_eq) kept |= 1u << i;
      ++eq_rank;
    }
  }
  int total = 0;
  int pos = block_excl_scan(__popc(kept), warp_sums, &total);
  int32_t* kout = kept_idx + static_cast<int64_t>(b) * max_len;
#pragma unroll
  for (int i = 0; i < kVPT; ++i)
    if ((kept >> i) & 1u) kout[pos++] = t0 + i;
  for (int t = total + tid; t < max_len; t += kSelThreads) kout[t] = -1;

  // New block-table row: the first ceil(total / BS) valid pages, in order;
  // every other valid page is reported as freed.  (The table entries are
  // read into registers before any is rewritten.)
  const int need_pages = (total + BS - 1) / BS;
  int32_t* frow = freed + static_cast<int64_t>(b) * MB;
  constexpr int kPPT = 2;  // MB <= 2048 = kSelThreads * kPPT
  int pg[kPPT];
  int pvalid = 0;
#pragma unroll
  for (int k = 0; k < kPPT; ++k) {
    const int lb = tid * kPPT + k;
    pg[k] = lb < MB ? btrow[lb] : -1;
    if (pg[k] >= 0 && pg[k] < NB) ++pvalid;
  }
  int nvp = 0;
  int vrank = block_excl_scan(pvalid, warp_sums, &nvp);
  __syncthreads();  // all entries read
  for (int lb = tid; lb < MB; lb += kSelThreads) btrow[lb] = -1;
  for (int lb = tid; lb < MB; lb += kSelThreads) frow[lb] = -1;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kPPT; ++k) {
    if (pg[k] >= 0 && pg[k] < NB) {
      if (vrank < need_pages) btrow[vrank] = pg[k];
      else frow[vrank - need_pages] = pg[k];
      ++vrank;
    }
  }
  if (tid == 0) {
    kept_count[b] = total;
    freed_count[b] = max(0, nvp - need_pages);
    ctx_lens[b] = total;
  }
}

// One warp per kept row: gather (dir = 0: pool -> workspace) or scatter
// (dir = 1: workspace -> pool).  Rows are H*D fp16 = `chunks` 16-byte pieces.
__global__ void move_rows_kernel(const int32_t* __restrict__ kept_idx, const int32_t* __restrict__ kept_count,
                                 const int32_t* __restrict__ old_bt, const int32_t* __restrict__ new_bt, int MB,
                                 int max_len, int BS, uint4* __restrict__ kpool, uint4* __restrict__ vpool,
                                 uint4* __restrict__ ktmp, uint4* __restrict__ vtmp, int chunks, int dir) {
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= kept_count[b]) return;
  const int64_t trow = static_cast<int64_t>(b) * max_len + row;
  int64_t slot;
  if (dir == 0) {
    const int t = kept_idx[trow];
    slot = static_cast<int64_t>(old_bt[static_cast<int64_t>(b) * MB + t / BS]) * BS + t % BS;
  } else {
    slot = static_cast<int64_t>(new_bt[static_cast<int64_t>(b) * MB + row / BS]) * BS + row % BS;
  }
  uint4* kp = kpool + slot * chunks;
  uint4* vp = vpool + slot * chunks;
  uint4* kt = ktmp + trow * chunks;
  uint4* vt = vtmp + trow * chunks;
  for (int c = lane; c < chunks; c += 32) {
    if (dir == 0) {
      kt[c] = kp[c];
      vt[c] = vp[c];
    } else {
      kp[c] = kt[c];
      vp[c] = vt[c];
    }
  }
}

}  // namespace

extern "C" __attribute__((visibility("default"))) size_t memopt_evict_topk_workspace_size(int num_seqs, int max_len, int num_heads, int head_dim) {
  if (num_seqs <= 0 || max_len <= 0 || num_heads <= 0 || head_dim <= 0) return 0;
  const size_t rows = static_cast<size_t>(num_seqs) * max_len;
  const size_t mb = static_cast<size_t>(num_seqs) * (kMaxLen);  // old block-table copy (upper bound)
  return rows * 4 + mb * 4 + 2 * rows * num_heads * head_dim * 2 + 256;
}

extern "C" __attribute__((visibility("default"))) int memopt_evict_topk_compact(const float* scores, int num_seqs, int num_heads, int max_len,
                                         int32_t* block_tables, int max_blocks_per_seq, int32_t* context_lens,
                                         void* key_pool, void* value_pool, int pool_num_blocks, int block_size,
                                         int head_dim, float retain_ratio, int num_sink_tokens,
                                         int32_t* kept_idx, int32_t* kept_count, int32_t* freed_pages,
                                         int32_t* freed_count, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  if (!(retain_ratio > 0.f && retain_ratio <= 1.f))
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_compact: retain_ratio must be in (0, 1]");
  if (num_seqs < 0 || num_heads <= 0 || max_len < 0 || max_blocks_per_seq < 0 || pool_num_blocks < 0 ||
      block_size <= 0 || head_dim <= 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_compact: invalid geometry");
  if (max_len > kMaxLen) return fail(MEMOPT_ERR_UNSUPPORTED, "evict_topk_compact: max_len exceeds 32768");
  if (max_blocks_per_seq > 2 * kSelThreads)
    return fail(MEMOPT_ERR_UNSUPPORTED, "evict_topk_compact: more than 2048 blocks per sequence");
  if ((num_heads * head_dim) % 8 != 0)
    return fail(MEMOPT_ERR_UNSUPPORTED, "evict_topk_compact: num_heads * head_dim must be a multiple of 8");
  if (num_seqs == 0 || max_len == 0) return MEMOPT_OK;
  if (!scores || !block_tables || !context_lens || !key_pool || !value_pool || !kept_idx || !kept_count ||
      !freed_pages || !freed_count || !workspace)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_compact: null pointer");
  if ((reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool) |
       reinterpret_cast<uintptr_t>(workspace)) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_compact: pools and workspace must be 16-byte aligned");
  const size_t need = memopt_evict_topk_workspace_size(num_seqs, max_len, num_heads, head_dim);
  if (workspace_bytes < need) return fail(MEMOPT_ERR_WORKSPACE, "evict_topk_compact: workspace too small");
  cudaStream_t s = as_stream(stream);
  const size_t rows = static_cast<size_t>(num_seqs) * max_len;
  const int chunks = num_heads * head_dim / 8;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  uint4* ktmp = reinterpret_cast<uint4*>(w);
  uint4* vtmp = ktmp + rows * chunks;
  float* sums = reinterpret_cast<float*>(vtmp + rows * chunks);
  int32_t* old_bt = reinterpret_cast<int32_t*>(sums + rows);
  const size_t bt_bytes = static_cast<size_t>(num_seqs) * max_blocks_per_seq * 4;
  cudaError_t e = cudaMemcpyAsync(old_bt, block_tables, bt_bytes, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "evict_topk_compact: block-table copy");
  head_sum_kernel<<<dim3((max_len + 255) / 256, num_seqs), 256, 0, s>>>(scores, num_heads, max_len, sums);
  MEMOPT_LAUNCH_CHECK("head_sum_kernel launch");
  const int sinks = num_sink_tokens < 0 ? 0 : num_sink_tokens;
  topk_select_kernel<<<num_seqs, kSelThreads, 0, s>>>(sums, max_len, block_tables, max_blocks_per_seq, context_lens,
                                                      pool_num_blocks, block_size, retain_ratio, sinks, kept_idx,
                                                      kept_count, freed_pages, freed_count);
  MEMOPT_LAUNCH_CHECK("topk_select_kernel launch");
  const dim3 mgrid((max_len + 7) / 8, num_seqs);
  move_rows_kernel<<<mgrid, 256, 0, s>>>(kept_idx, kept_count, old_bt, block_tables, max_blocks_per_seq, max_len,
                                         block_size, static_cast<uint4*>(key_pool), static_cast<uint4*>(value_pool),
                                         ktmp, vtmp, chunks, 0);
  MEMOPT_LAUNCH_CHECK("move_rows_kernel (gather) launch");
  move_rows_kernel<<<mgrid, 256, 0, s>>>(kept_idx, kept_count, old_bt, block_tables, max_blocks_per_seq, max_len,
                                         block_size, static_cast<uint4*>(key_pool), static_cast<uint4*>(value_pool),
                                         ktmp, vtmp, chunks, 1);
  MEMOPT_LAUNCH_CHECK("move_rows_kernel (scatter) launch");
  return MEMOPT_OK;
}

}  // namespace memopt
