// evict.cu — Ada-KV eviction over the paged pool.
//
// evict_tokens: replaces evict_tokens_kernel (reference
// src/csrc/kv_cache.cu:640-1015).  Semantics reproduced exactly:
//   * scores of tokens t < num_sink_tokens are replaced by 1e38f (:723-726);
//   * keep = max(1, min(L, (int)ceilf(r * (float)L)))            (:754-755);
//   * min/max start at +1e38f / -1e38f and use fminf/fmaxf       (:758-803);
//   * if min >= max: thr = min - 1.0f, else 32 bisection steps
//     mid = lo + (hi - lo) * 0.5f (contracted to one fma, as nvcc does by
//     default), count(s >= mid) >= keep ? lo = mid : hi = mid; thr = lo;
//   * token t is evicted iff s < thr; of an evicted row only the elements
//     d = (t % 32) + 32k are zeroed in K and V (:937-973);
//   * the per-block vote counts only evicted tokens with t % 32 == 0 (:978),
//     so it can reach block_size only when block_size == 1 (:993-1014).
// The reference runs one 128-thread CTA per (seq, head) with the scores in
// shared memory and three barriers per bisection step; here one CTA keeps the
// scores in registers (<= 64 per thread) and runs no block-wide step per
// bisection: the steps' outcomes depend on the scores only through the
// keep-th largest comparable score, which bounds decide for most steps and an
// exact radix select gives for the rest, so the 32 steps are replayed on
// scalars.  The kept tokens are also stream-compacted into an ascending index
// list.
//
// evict_cache: replaces evict_cache_kernel (kv_cache.cu:379-483): per
// (physical block, head) the threshold is the keep-th largest score found by
// repeated arg-max (values <= -1e38f or NaN never win), keep =
// max(1, (int)(r * block_size)); rows with score < threshold are zeroed.
#include "common.cuh"

namespace memopt {
namespace {

// Scores per thread (VPT) are a multiple of 4: rows up to 1024 tokens use 256
// threads, up to 16384 tokens 1024 threads with 4..16 scores each, longer
// rows 512 threads holding 64 scores each (register budget 128 per thread).
constexpr int kMaxEvictLen = 32768;

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Order-preserving key of a float (x < y as floats <=> key(x) < key(y) as
// unsigned, -0 just below +0) and its inverse.
__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return b ^ (static_cast<uint32_t>(static_cast<int32_t>(b) >> 31) | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float(k ^ ((k & 0x80000000u) ? 0x80000000u : 0xFFFFFFFFu));
}

template <int VPT, int kEvictThreads>
__global__ void __launch_bounds__(kEvictThreads, 1)
evict_tokens_kernel(const float* __restrict__ scores, int num_seqs, int num_heads, int seq_len,
                    int32_t* __restrict__ block_tables, int max_blocks_per_seq,
                    int32_t* __restrict__ is_block_free, int total_pool_blocks,
                    __half* __restrict__ kpool, __half* __restrict__ vpool, int block_size,
                    int head_dim, float retain_ratio, int num_sinks,
                    int32_t* __restrict__ retained_idx, int32_t* __restrict__ retained_count) {
  static_assert(VPT % 4 == 0 && VPT <= 64, "VPT: multiple of 4, at most 64 (one 64-bit mask)");
  const int seq = blockIdx.x;
  const int head = blockIdx.y;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int L = seq_len;
  constexpr int kEvictWarps = kEvictThreads / 32;

  __shared__ float red_f[2][kEvictWarps];
  __shared__ int red_i[2][kEvictWarps];
  __shared__ int warp_tot[kEvictWarps];
  // Radix select: one histogram copy per lane (a warp's atomics never meet),
  // the bin totals and the chosen digit with the remaining rank.
  __shared__ int hist[256][32];
  __shared__ int bin_tot[256];
  __shared__ int sel_digit[2];

  // ---- load: warp w owns tokens [w*32*VPT, (w+1)*32*VPT); in round k lane
  // holds the 4 tokens chunk + 128 k + 4 lane .. +3, so every warp load and
  // every index store covers 512 contiguous bytes.  A lane's tokens ascend
  // with i, so its valid ones are the first nv.
  const float* src = scores + (static_cast<int64_t>(seq) * num_heads + head) * L;
  const int wbase = warp * (32 * VPT);
  auto tok = [&](int i) { return wbase + (i >> 2) * 128 + lane * 4 + (i & 3); };
  int nv = 0;
#pragma unroll
  for (int k = 0; k < VPT / 4; ++k) nv += min(4, max(0, L - tok(4 * k)));

  // Tokens past L hold NaN: fminf/fmaxf skip it and `s >= mid` / `s < thr`
  // are false for it, exactly how the reference treats a NaN score, so the
  // scans below need no bounds test (a real NaN score is never counted and
  // never evicted either).
  float v[VPT];
  const bool vec = (L % 4 == 0) && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
  if (vec) {
#pragma unroll
    for (int k = 0; k < VPT / 4; ++k) {
      float4 f = make_float4(NAN, NAN, NAN, NAN);
      const int t = tok(4 * k);
      if (t < L) f = __ldg(reinterpret_cast<const float4*>(src + t));
      v[4 * k] = f.x;
      v[4 * k + 1] = f.y;
      v[4 * k + 2] = f.z;
      v[4 * k + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPT; ++i) v[i] = i < nv ? __ldg(src + tok(i)) : NAN;
  }
  if (wbase < num_sinks) {
#pragma unroll
    for (int i = 0; i < VPT; ++i)
      if (tok(i) < num_sinks) v[i] = 1e38f;
  }

  // ---- min / max and this thread's count of comparable scores -----------
  float tmin = 1e38f, tmax = -1e38f;
  int ncmp = 0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    tmin = fminf(tmin, v[i]);
    tmax = fmaxf(tmax, v[i]);
    ncmp += (v[i] == v[i]) ? 1 : 0;
  }
  float gmin = tmin, gmax = tmax;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    gmin = fminf(gmin, __shfl_xor_sync(0xffffffffu, gmin, o));
    gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, o));
  }
  if (lane == 0) {
    red_f[0][warp] = gmin;
    red_f[1][warp] = gmax;
  }
  __syncthreads();
  gmin = lane < kEvictWarps ? red_f[0][lane] : 1e38f;
  gmax = lane < kEvictWarps ? red_f[1][lane] : -1e38f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    gmin = fminf(gmin, __shfl_xor_sync(0xffffffffu, gmin, o));
    gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, o));
  }

  // Exact keep-th largest comparable score of the block (keep <= the number
  // of comparable scores): radix select over order-preserving 32-bit keys,
  // four 8-bit digits from the most significant, each pass one histogram of
  // the digit over the keys that match the digits chosen so far.
  auto radix_select = [&](const float (&vals)[VPT], int rank) -> float {
    uint32_t prefix = 0, pmask = 0;
    int kk = rank;  // rank among the keys that match the prefix, from the top
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256 * 32; i += kEvictThreads) hist[i >> 5][i & 31] = 0;
      __syncthreads();
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const uint32_t key = order_key(vals[i]);
        if (vals[i] == vals[i] && (key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u][lane], 1);
      }
      __syncthreads();
      if (tid < 256) {
        int c = 0;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) c += hist[tid][(j + tid) & 31];  // rotated: no bank conflicts
        bin_tot[tid] = c;
      }
      __syncthreads();
      if (warp == 0) {
        // lane l holds digits 255 - 8l .. 248 - 8l, in descending order
        int c8[8], sum = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          c8[e] = bin_tot[255 - 8 * lane - e];
          sum += c8[e];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int n = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += n;
        }
        int above = incl - sum;  // keys with a larger digit than this lane's first
        if (above < kk && kk <= incl) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (above < kk && kk <= above + c8[e]) {
              sel_digit[0] = 255 - 8 * lane - e;
              sel_digit[1] = kk - above;
            }
            above += c8[e];
          }
        }
      }
      __syncthreads();
      prefix |= static_cast<uint32_t>(sel_digit[0]) << shift;
      pmask |= 255u << shift;
      kk = sel_digit[1];
      __syncthreads();  // sel_digit is written again by the next pass
    }
    return key_float(prefix);
  };

  // ---- threshold ---------------------------------------------------------
  const int keep = max(1, min(L, static_cast<int>(ceilf(retain_ratio * static_cast<float>(L)))));
  float thr;
  if (gmin >= gmax) {
    thr = gmin - 1.0f;
  } else {
    // count(s >= mid) >= keep holds exactly when w >= mid, w being the
    // keep-th largest comparable (non-NaN) score, and never when fewer than
    // keep scores are comparable.  So the 32 bisection steps depend on the
    // scores only through w and are replayed here on scalars with the same
    // fma.  Most steps are decided by bounds of w: w <= u (u = the largest
    // score below the maximum when fewer than keep scores equal the maximum,
    // else the maximum) and w >= gmin; only a midpoint inside (gmin, u]
    // needs w itself, found once by an exact radix select.
    float mx2 = -INFINITY;
    int neq = 0;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      neq += (v[i] == gmax) ? 1 : 0;
      if (v[i] < gmax) mx2 = fmaxf(mx2, v[i]);
    }
    int tot_cmp = ncmp, tot_eq = neq;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      tot_cmp += __shfl_xor_sync(0xffffffffu, tot_cmp, o);
      tot_eq += __shfl_xor_sync(0xffffffffu, tot_eq, o);
      mx2 = fmaxf(mx2, __shfl_xor_sync(0xffffffffu, mx2, o));
    }
    __syncthreads();  // every warp has read the min / max partials in red_f
    if (lane == 0) {
      red_i[0][warp] = tot_cmp;
      red_i[1][warp] = tot_eq;
      red_f[0][warp] = mx2;
    }
    __syncthreads();
    tot_cmp = lane < kEvictWarps ? red_i[0][lane] : 0;
    tot_eq = lane < kEvictWarps ? red_i[1][lane] : 0;
    mx2 = lane < kEvictWarps ? red_f[0][lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      tot_cmp += __shfl_xor_sync(0xffffffffu, tot_cmp, o);
      tot_eq += __shfl_xor_sync(0xffffffffu, tot_eq, o);
      mx2 = fmaxf(mx2, __shfl_xor_sync(0xffffffffu, mx2, o));
    }
    const float u = tot_eq < keep ? mx2 : gmax;
    bool have_w = false;
    float w = 0.f;
    float lo = gmin, hi = gmax;
#pragma unroll 1
    for (int it = 0; it < 32; ++it) {
      const float mid = __fmaf_rn(hi - lo, 0.5f, lo);
      bool ge;
      if (tot_cmp < keep || mid != mid || mid > u) {
        ge = false;
      } else if (mid <= gmin) {
        ge = true;
      } else {
        if (!have_w) {  // block-uniform: every input above is the same in all threads
          w = radix_select(v, keep);
          have_w = true;
        }
        ge = w >= mid;
      }
      if (ge) lo = mid; else hi = mid;
    }
    thr = lo;
  }

  // ---- evicted tokens as a bit mask (bit i <-> v[i]) -----------------------
  uint64_t ev = 0;
#pragma unroll
  for (int i = 0; i < VPT; ++i) ev |= static_cast<uint64_t>(v[i] < thr ? 1 : 0) << i;
  const int kept = nv - __popcll(ev);

  // ---- zero evicted rows (partial pattern) ---------------------------------
  const int64_t hd = static_cast<int64_t>(head_dim);
  const int64_t table_size = static_cast<int64_t>(num_seqs) * max_blocks_per_seq;
  for (uint64_t m = ev; m != 0; m &= m - 1) {
    const int i = __ffsll(static_cast<long long>(m)) - 1;
    const int t = tok(i);
    const int lb = t / block_size;
    const int pos = t - lb * block_size;
    const int64_t flat = static_cast<int64_t>(seq) * max_blocks_per_seq + lb;
    if (flat >= table_size) continue;
    const int phys = block_tables[flat];
    if (phys < 0 || phys >= total_pool_blocks) continue;
    const int64_t base = ((static_cast<int64_t>(phys) * block_size + pos) * num_heads + head) * hd;
    for (int d = t & 31; d < head_dim; d += 32) {
      kpool[base + d] = __float2half_rn(0.f);
      vpool[base + d] = __float2half_rn(0.f);
    }
  }
  if (block_size == 1) {
    // Only here can a block's vote reach block_size: token t == lb, counted
    // when t % 32 == 0.  Votes follow every zeroing of this CTA.
    __syncthreads();
    for (uint64_t m = ev; m != 0; m &= m - 1) {
      const int t = tok(__ffsll(static_cast<long long>(m)) - 1);
      if ((t & 31) != 0) continue;
      const int64_t flat = static_cast<int64_t>(seq) * max_blocks_per_seq + t;
      if (flat >= table_size) continue;
      const int phys = block_tables[flat];
      if (phys < 0 || phys >= total_pool_blocks) continue;
      const int prev = atomicAdd(is_block_free + phys, 1);
      if (prev + 1 == num_heads) block_tables[flat] = -1;
    }
  }

  // ---- stream compaction of kept token indices ---------------------------
  // Warp offsets come from a block scan of per-warp kept counts; inside a
  // warp the 128-token rounds are emitted in order with a lane scan each.
  if (retained_idx != nullptr || retained_count != nullptr) {
    const int wkept = warp_sum_i(kept);
    if (lane == 0) warp_tot[warp] = wkept;
    __syncthreads();
    const int wt = lane < kEvictWarps ? warp_tot[lane] : 0;
    int wincl = wt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wincl, o);
      if (lane >= o) wincl += n;
    }
    int out = __shfl_sync(0xffffffffu, wincl - wt, warp);
    const int total = __shfl_sync(0xffffffffu, wincl, 31);
    const int64_t pair = static_cast<int64_t>(seq) * num_heads + head;
    if (retained_idx != nullptr) {
      int32_t* dst = retained_idx + pair * L;
      const bool dst16 = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
      const uint64_t keepm = ~ev & (nv >= 64 ? ~0ull : ((1ull << nv) - 1ull));
#pragma unroll 1
      for (int k = 0; k < VPT / 4; ++k) {
        const uint32_t b = static_cast<uint32_t>(keepm >> (4 * k)) & 0xFu;
        const int n4 = __popc(b);
        const int t = tok(4 * k);
        if (__all_sync(0xffffffffu, b == 0xFu) && dst16 && (out & 3) == 0) {
          reinterpret_cast<int4*>(dst + out)[lane] = make_int4(t, t + 1, t + 2, t + 3);
          out += 128;
        } else {
          int incl = n4;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
          }
          int pos = out + incl - n4;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (b & (1u << j)) dst[pos++] = t + j;
          out += __shfl_sync(0xffffffffu, incl, 31);
        }
      }
      for (int t = total + tid; t < L; t += kEvictThreads) dst[t] = -1;
    }
    if (retained_count != nullptr && tid == 0) retained_count[pair] = total;
  }
}

// One warp per physical block: its lanes first find, per head, the rows to
// zero (the keep-th largest score by repeated arg-max, as below) as a row
// bit mask in shared memory, then zero the marked rows of all heads with
// 16-byte stores that cover each token row ([head][dim], contiguous) in
// order, so every store instruction writes 512 contiguous bytes.  Needs
// head_dim % 8 == 0 and 16-byte aligned pools.
constexpr int kEvictCacheWarps = 8;

template <int BS>
__global__ void __launch_bounds__(kEvictCacheWarps * 32)
evict_cache_rows_kernel(const float* __restrict__ scores, int num_blocks, int num_heads, int head_dim,
                        uint4* __restrict__ kpool, uint4* __restrict__ vpool, float retain_ratio) {
  extern __shared__ uint32_t row_masks_all[];  // kEvictCacheWarps x num_heads
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  uint32_t* masks = row_masks_all + w * num_heads;
  const int cph = head_dim / 8;        // 16-byte chunks per head row
  const int cpr = num_heads * cph;     // per token row
  int keep = max(1, static_cast<int>(retain_ratio * static_cast<float>(BS)));
  keep = min(keep, BS);
  for (int64_t blk = static_cast<int64_t>(blockIdx.x) * kEvictCacheWarps + w; blk < num_blocks;
       blk += static_cast<int64_t>(gridDim.x) * kEvictCacheWarps) {
    uint32_t any = 0;
    for (int h = lane; h < num_heads; h += 32) {
      float s[BS], wv[BS];
#pragma unroll
      for (int p = 0; p < BS; ++p) {
        s[p] = __ldg(scores + (blk * BS + p) * num_heads + h);
        wv[p] = s[p];
      }
      float thr = -1e38f;
      for (int k = 0; k < keep; ++k) {
        float best = -1e38f;
        int best_pos = -1;
#pragma unroll
        for (int p = 0; p < BS; ++p) {
          if (wv[p] > best) {
            best = wv[p];
            best_pos = p;
          }
        }
        thr = best;
#pragma unroll
        for (int p = 0; p < BS; ++p)
          if (p == best_pos) wv[p] = -1e38f;
      }
      uint32_t m = 0;
#pragma unroll
      for (int p = 0; p < BS; ++p) m |= (s[p] < thr) ? (1u << p) : 0u;
      masks[h] = m;
      any |= m;
    }
    any = __reduce_or_sync(0xffffffffu, any);
    __syncwarp();
    for (int p = 0; p < BS; ++p) {
      if (!((any >> p) & 1u)) continue;
      const int64_t base = (blk * BS + p) * cpr;
      for (int c = lane; c < cpr; c += 32) {
        if ((masks[c / cph] >> p) & 1u) {
          kpool[base + c] = make_uint4(0, 0, 0, 0);
          vpool[base + c] = make_uint4(0, 0, 0, 0);
        }
      }
    }
    __syncwarp();
  }
}

// One thread per (physical block, head); heads fastest for coalesced reads.
template <int BS>
__global__ void __launch_bounds__(256)
evict_cache_kernel(const float* __restrict__ scores, int num_blocks, int num_heads, int head_dim,
                   __half* __restrict__ kpool, __half* __restrict__ vpool, float retain_ratio) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(num_blocks) * num_heads) return;
  const int64_t blk = idx / num_heads;
  const int head = static_cast<int>(idx - blk * num_heads);
  float s[BS], w[BS];
#pragma unroll
  for (int p = 0; p < BS; ++p) {
    s[p] = __ldg(scores + (blk * BS + p) * num_heads + head);
    w[p] = s[p];
  }
  int keep = max(1, static_cast<int>(retain_ratio * static_cast<float>(BS)));
  keep = min(keep, BS);
  float thr = -1e38f;
  for (int k = 0; k < keep; ++k) {
    float best = -1e38f;
    int best_pos = -1;
#pragma unroll
    for (int p = 0; p < BS; ++p) {
      if (w[p] > best) {
        best = w[p];
        best_pos = p;
      }
    }
    thr = best;
#pragma unroll
    for (int p = 0; p < BS; ++p)
      if (p == best_pos) w[p] = -1e38f;
  }
  const int64_t hd = head_dim;
  const bool vec = (head_dim % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(kpool) | reinterpret_cast<uintptr_t>(vpool)) & 15u) == 0;
#pragma unroll
  for (int p = 0; p < BS; ++p) {
    if (!(s[p] < thr)) continue;
    const int64_t base = ((blk * BS + p) * num_heads + head) * hd;
    if (vec) {
      uint4* kd = reinterpret_cast<uint4*>(kpool + base);
      uint4* vd = reinterpret_cast<uint4*>(vpool + base);
      for (int c = 0; c < head_dim / 8; ++c) {
        kd[c] = make_uint4(0, 0, 0, 0);
        vd[c] = make_uint4(0, 0, 0, 0);
      }
    } else {
      for (int d = 0; d < head_dim; ++d) {
        kpool[base + d] = __float2half_rn(0.f);
        vpool[base + d] = __float2half_rn(0.f);
      }
    }
  }
}

// Any block size, no scratch: the repeated arg-max picks scores in
// descending order (ties by position), with scores <= -1e38f or NaN acting as
// -1e38f.  The keep-th pick is therefore the element whose rank
//   #{q : w'[q] > w'[p]} + #{q < p : w'[q] == w'[p]}
// equals keep-1, where w' is that normalised score.
__global__ void __launch_bounds__(256)
evict_cache_generic_kernel(const float* __restrict__ scores, int num_blocks, int block_size,
                           int num_heads, int head_dim, __half* __restrict__ kpool,
                           __half* __restrict__ vpool, float retain_ratio) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(num_blocks) * num_heads) return;
  const int64_t blk = idx / num_heads;
  const int head = static_cast<int>(idx - blk * num_heads);
  auto at = [&](int p) {
    const float x = scores[(blk * block_size + p) * num_heads + head];
    return (x > -1e38f) ? x : -1e38f;
  };
  int keep = max(1, static_cast<int>(retain_ratio * static_cast<float>(block_size)));
  keep = min(keep, block_size);
  float thr = -1e38f;
  for (int p = 0; p < block_size; ++p) {
    const float wp = at(p);
    int rank = 0;
    for (int q = 0; q < block_size; ++q) {
      const float wq = at(q);
      rank += (wq > wp) || (q < p && wq == wp);
    }
    if (rank == keep - 1) {
      thr = wp;
      break;
    }
  }
  for (int p = 0; p < block_size; ++p) {
    if (!(scores[(blk * block_size + p) * num_heads + head] < thr)) continue;
    const int64_t base = ((blk * block_size + p) * num_heads + head) * static_cast<int64_t>(head_dim);
    for (int d = 0; d < head_dim; ++d) {
      kpool[base + d] = __float2half_rn(0.f);
      vpool[base + d] = __float2half_rn(0.f);
    }
  }
}

}  // namespace
}  // namespace memopt

using namespace memopt;

extern "C" int memopt_evict_tokens(const float* scores, int num_seqs, int num_heads, int seq_len,
                                   int32_t* block_tables, int max_blocks_per_seq,
                                   int32_t* is_block_free, int total_pool_blocks, void* key_pool,
                                   void* value_pool, int pool_num_blocks, int block_size,
                                   int head_dim, float retain_ratio, int num_sink_tokens,
                                   int32_t* retained_idx, int32_t* retained_count, void* stream) {
  if (!(retain_ratio > 0.f && retain_ratio <= 1.f))
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_tokens: retain_ratio must be in (0, 1]");
  if (num_seqs < 0 || num_heads <= 0 || seq_len < 0 || max_blocks_per_seq < 0 ||
      total_pool_blocks < 0 || block_size <= 0 || head_dim <= 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_tokens: invalid geometry");
  if (total_pool_blocks > pool_num_blocks)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_tokens: is_block_free size > pool.num_blocks");
  if (seq_len > kMaxEvictLen)
    return fail(MEMOPT_ERR_UNSUPPORTED, "evict_tokens: seq_len exceeds 32768");
  if (num_seqs == 0 || seq_len == 0) return MEMOPT_OK;
  if (!scores || !block_tables || !is_block_free || !key_pool || !value_pool)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_tokens: null pointer");
  const int sinks = num_sink_tokens < 0 ? 0 : (num_sink_tokens > seq_len ? seq_len : num_sink_tokens);
  const dim3 grid(num_seqs, num_heads);
  cudaStream_t s = as_stream(stream);
  const int vpt1024 = (seq_len + 1023) / 1024;
#define MEMOPT_EVICT_LAUNCH(V, NT)                                                                \
  evict_tokens_kernel<V, NT><<<grid, NT, 0, s>>>(                                               \
      scores, num_seqs, num_heads, seq_len, block_tables, max_blocks_per_seq, is_block_free,     \
      total_pool_blocks, reinterpret_cast<__half*>(key_pool), reinterpret_cast<__half*>(value_pool), \
      block_size, head_dim, retain_ratio, sinks, retained_idx, retained_count)
  if (seq_len <= 1024) MEMOPT_EVICT_LAUNCH(4, 256);
  else if (vpt1024 <= 4) MEMOPT_EVICT_LAUNCH(4, 1024);
  else if (vpt1024 <= 8) MEMOPT_EVICT_LAUNCH(8, 1024);
  else if (vpt1024 <= 16) MEMOPT_EVICT_LAUNCH(16, 1024);
  else MEMOPT_EVICT_LAUNCH(64, 512);
#undef MEMOPT_EVICT_LAUNCH
  MEMOPT_LAUNCH_CHECK("evict_tokens launch");
  return MEMOPT_OK;
}

extern "C" int memopt_evict_cache(const float* scores, int num_blocks, int block_size,
                                  int num_heads, int head_dim, void* key_pool, void* value_pool,
                                  float retain_ratio, void* stream) {
  if (!(retain_ratio > 0.f && retain_ratio <= 1.f))
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_cache: retain_ratio must be in (0, 1]");
  if (num_blocks < 0 || block_size <= 0 || num_heads <= 0 || head_dim <= 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_cache: invalid geometry");
  if (num_blocks == 0) return MEMOPT_OK;
  if (!scores || !key_pool || !value_pool) return fail(MEMOPT_ERR_INVALID_ARG, "evict_cache: null pointer");
  const int64_t n = static_cast<int64_t>(num_blocks) * num_heads;
  const int grid = static_cast<int>((n + 255) / 256);
  cudaStream_t s = as_stream(stream);
  __half* k = reinterpret_cast<__half*>(key_pool);
  __half* v = reinterpret_cast<__half*>(value_pool);
  const bool rows_ok = head_dim % 8 == 0 && num_heads <= 2048 &&
                       ((reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool)) & 15u) == 0;
  if (rows_ok && (block_size == 16 || block_size == 32)) {
    const int64_t want = (num_blocks + kEvictCacheWarps - 1) / kEvictCacheWarps;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    const int g = static_cast<int>(want < cap ? want : cap);
    const size_t smem = static_cast<size_t>(kEvictCacheWarps) * num_heads * 4;
    uint4* k4 = reinterpret_cast<uint4*>(key_pool);
    uint4* v4 = reinterpret_cast<uint4*>(value_pool);
    if (smem > 48 * 1024) {
      cudaError_t e = block_size == 16
                          ? cudaFuncSetAttribute(evict_cache_rows_kernel<16>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem))
                          : cudaFuncSetAttribute(evict_cache_rows_kernel<32>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return cuda_fail(e, "evict_cache: shared-memory attribute");
    }
    if (block_size == 16)
      evict_cache_rows_kernel<16><<<g, kEvictCacheWarps * 32, smem, s>>>(scores, num_blocks, num_heads, head_dim,
                                                                          k4, v4, retain_ratio);
    else
      evict_cache_rows_kernel<32><<<g, kEvictCacheWarps * 32, smem, s>>>(scores, num_blocks, num_heads, head_dim,
                                                                          k4, v4, retain_ratio);
  } else if (block_size == 16) {
    evict_cache_kernel<16><<<grid, 256, 0, s>>>(scores, num_blocks, num_heads, head_dim, k, v, retain_ratio);
  } else if (block_size == 32) {
    evict_cache_kernel<32><<<grid, 256, 0, s>>>(scores, num_blocks, num_heads, head_dim, k, v, retain_ratio);
  } else if (block_size == 8) {
    evict_cache_kernel<8><<<grid, 256, 0, s>>>(scores, num_blocks, num_heads, head_dim, k, v, retain_ratio);
  } else {
    evict_cache_generic_kernel<<<grid, 256, 0, s>>>(scores, num_blocks, block_size, num_heads, head_dim,
                                                    k, v, retain_ratio);
  }
  MEMOPT_LAUNCH_CHECK("evict_cache launch");
  return MEMOPT_OK;
}
