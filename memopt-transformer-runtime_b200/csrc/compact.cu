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
// With heads sharded over G ranks, each rank sums its own heads
// (memopt_evict_topk_head_sum), the G partial rows are exchanged, and
// memopt_evict_topk_compact_parts ranks tokens by the fp32 sum of the parts in
// rank order: every rank takes the same decision and compacts the rows of
// its own heads.  With G = 1 this is exactly memopt_evict_topk_compact.
// Three launches: head sums (parallel over tokens), one CTA per sequence for
// the selection, the new block-table row and each kept row's source ordinal
// (its slot's position among the sequence's valid pages), then the kept rows
// move in place.  A row only moves forward (destination ordinal <= source
// ordinal), so the one hazard is overwriting a slot before the row that
// lives there has been read; the move kernel orders exactly those pairs.
#include <atomic>
#include <climits>

#include "common.cuh"
#include "int4.cuh"
#include "memopt_b200.h"

namespace memopt {
namespace {

constexpr int kSelThreads = 1024;
constexpr int kMaxLen = 32768;
constexpr int kVPT = kMaxLen / kSelThreads;  // 32 tokens per thread
// Kept rows moved by one CTA.  At 8 sequences x 32768 tokens x 8 KB rows
// (retain 0.75) one row per CTA moved the rows in 1.17 ms, 2 in 1.19 ms,
// 4 in 1.29 ms and 8 in 1.73 ms: small CTAs keep more copies in flight.
constexpr int kSegRows = 1;

// Flag-wait bound of the row movers and the test hook that withholds their
// "read" flags (memopt_evict_topk_set_test_hooks); defaults: kMaxPolls, off.
std::atomic<uint32_t> g_flag_polls{kMaxPolls};
std::atomic<int> g_withhold_flags{0};
constexpr int kMaxPagesBig = 16 * kSelThreads;   // streaming select: up to 16 table entries per thread
constexpr int kMoveSmemLimit = 200 * 1024;       // 2 * kSegRows rows staged in shared memory

// sums[b, t] = fp32 sum over i in order of src[b * b_stride + i * i_stride + t].
// Per-head scores [B, H, L] are (b_stride, i_stride) = (H*L, L); the partial
// sums of G ranks stacked as [G, B, L] are (L, B*L).  The sum starts at +0, so
// it is never -0 (the integer keys below order -0 below +0).
__global__ void head_sum_kernel(const float* __restrict__ src, int64_t b_stride, int64_t i_stride, int n_terms,
                                int max_len, float* __restrict__ sums) {
  const int b = blockIdx.y;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= max_len) return;
  const float* p = src + static_cast<int64_t>(b) * b_stride + t;
  float s = 0.f;
  for (int i = 0; i < n_terms; ++i) s += __ldg(p + static_cast<int64_t>(i) * i_stride);
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
                   int32_t* __restrict__ freed, int32_t* __restrict__ freed_count,
                   int32_t* __restrict__ src_ord, int32_t* __restrict__ seg_dep, int seg_stride) {
  __shared__ int hist[256];
  __shared__ int warp_sums[32];
  __shared__ int page_rank[2 * kSelThreads];  // rank of each valid page among the row's valid pages
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

  // Ranks of the valid pages (the new row is the first ceil(total / BS) of
  // them, in order).  The table entries are read into registers here, before
  // any is rewritten.
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
  const int vrank0 = block_excl_scan(pvalid, warp_sums, &nvp);
  {
    int v = vrank0;
#pragma unroll
    for (int k = 0; k < kPPT; ++k) {
      const int lb = tid * kPPT + k;
      if (lb < MB) page_rank[lb] = (pg[k] >= 0 && pg[k] < NB) ? v++ : -1;
    }
  }
  const int nseg = (total + kSegRows - 1) / kSegRows;
  int32_t* dep = seg_dep + static_cast<int64_t>(b) * seg_stride;
  for (int k = tid; k < nseg; k += kSelThreads) dep[k] = INT_MAX;
  __syncthreads();

  // Kept rows in token order.  Row `pos` moves from ordinal src (the token's
  // position among the valid pages' slots) to ordinal pos <= src.  A segment
  // of kSegRows destination rows may only be written after every row whose
  // source lies in it has been read: dep[segment] = the lowest segment with
  // such a row (those rows are consecutive, so they span at most that
  // segment and the next one).
  int32_t* kout = kept_idx + static_cast<int64_t>(b) * max_len;
  int32_t* oout = src_ord + static_cast<int64_t>(b) * max_len;
#pragma unroll
  for (int i = 0; i < kVPT; ++i) {
    if ((kept >> i) & 1u) {
      const int t = t0 + i;
      const int so = page_rank[t / BS] * BS + t % BS;
      kout[pos] = t;
      oout[pos] = so;
      if (so / kSegRows != pos / kSegRows) atomicMin(&dep[so / kSegRows], pos / kSegRows);
      ++pos;
    }
  }
  for (int t = total + tid; t < max_len; t += kSelThreads) kout[t] = -1;

  const int need_pages = (total + BS - 1) / BS;
  int32_t* frow = freed + static_cast<int64_t>(b) * MB;
  for (int lb = tid; lb < MB; lb += kSelThreads) btrow[lb] = -1;
  for (int lb = tid; lb < MB; lb += kSelThreads) frow[lb] = -1;
  __syncthreads();
  int vrank = vrank0;
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

// The same selection for long sequences (max_len > 32768 or more than 2048
// table entries): keys are recomputed from the token sums (L2-resident) in
// every pass instead of being held in registers, each thread owns a
// contiguous chunk of tokens (so block scans give token order), and the page
// ranks live in dynamic shared memory.  Same outputs as topk_select_kernel.
__global__ void __launch_bounds__(kSelThreads, 1)
topk_select_big_kernel(const float* __restrict__ sums, int max_len, int32_t* __restrict__ bt, int MB,
                       int32_t* __restrict__ ctx_lens, int NB, int BS, float retain_ratio, int num_sinks,
                       int32_t* __restrict__ kept_idx, int32_t* __restrict__ kept_count,
                       int32_t* __restrict__ freed, int32_t* __restrict__ freed_count,
                       int32_t* __restrict__ src_ord, int32_t* __restrict__ seg_dep, int seg_stride) {
  extern __shared__ int page_rank[];  // [MB]: rank among the row's valid pages, -1 if invalid
  __shared__ int hist[256];
  __shared__ int warp_sums[32];
  __shared__ uint32_t sh_prefix;
  __shared__ int sh_remaining;
  const int b = blockIdx.x, tid = threadIdx.x;
  int32_t* btrow = bt + static_cast<int64_t>(b) * MB;
  const int L = min(max(ctx_lens[b], 0), max_len);
  const float* srow = sums + static_cast<int64_t>(b) * max_len;

  // Page ranks: thread tid owns table entries [tid * PPT, tid * PPT + PPT).
  const int PPT = (MB + kSelThreads - 1) / kSelThreads;  // <= 16
  int pg[16];
  int pvalid = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const int lb = tid * PPT + k;
    pg[k] = (k < PPT && lb < MB) ? btrow[lb] : -1;
    if (pg[k] >= 0 && pg[k] < NB) ++pvalid;
  }
  int nvp = 0;
  const int vrank0 = block_excl_scan(pvalid, warp_sums, &nvp);
  {
    int v = vrank0;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int lb = tid * PPT + k;
      if (k < PPT && lb < MB) page_rank[lb] = (pg[k] >= 0 && pg[k] < NB) ? v++ : -1;
    }
  }
  __syncthreads();

  // Key of token t (< L): 0 = not a candidate (NaN keys are 0 too, as below).
  const int CH = (L + kSelThreads - 1) / kSelThreads;
  const int t_lo = min(tid * CH, L), t_hi = min(t_lo + CH, L);
  auto valid_tok = [&](int t) { return page_rank[t / BS] >= 0; };  // t < L <= max_len, t / BS < MB checked below
  auto key_of = [&](int t) -> uint32_t { return t < num_sinks ? 0xFFFFFFFFu : score_key(srow[t]); };
  const bool tbl_ok = (L + BS - 1) / BS <= MB;  // tokens on entries past the table are never valid
  auto in_table = [&](int t) { return tbl_ok || t / BS < MB; };

  int nv_thread = 0;
  for (int t = t_lo; t < t_hi; ++t) nv_thread += (in_table(t) && valid_tok(t)) ? 1 : 0;
  int nvalid = 0;
  block_excl_scan(nv_thread, warp_sums, &nvalid);
  const int keep = nvalid == 0 ? 0 : max(1, min(nvalid, static_cast<int>(ceilf(retain_ratio * static_cast<float>(nvalid)))));

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
    for (int t = t_lo; t < t_hi; ++t) {
      if (!(in_table(t) && valid_tok(t))) continue;
      const uint32_t k = key_of(t);
      if ((k & prefix_mask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFFu], 1);
    }
    __syncthreads();
    if (tid < 32) {
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
      int above = incl - part;
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
  const int need_eq = sh_remaining;

  int eq_thread = 0;
  for (int t = t_lo; t < t_hi; ++t)
    if (in_table(t) && valid_tok(t) && key_of(t) == T) ++eq_thread;
  const int eq_before = block_excl_scan(eq_thread, warp_sums, nullptr);
  auto kept_tok = [&](int t, int& eq_rank) -> bool {
    if (keep == 0 || !(in_table(t) && valid_tok(t))) return false;
    const uint32_t k = key_of(t);
    if (k > T) return true;
    if (k == T) return eq_rank++ < need_eq;
    return false;
  };
  int kept_thread = 0;
  {
    int er = eq_before;
    for (int t = t_lo; t < t_hi; ++t) kept_thread += kept_tok(t, er) ? 1 : 0;
  }
  int total = 0;
  int pos = block_excl_scan(kept_thread, warp_sums, &total);

  const int nseg = (total + kSegRows - 1) / kSegRows;
  int32_t* dep = seg_dep + static_cast<int64_t>(b) * seg_stride;
  for (int k = tid; k < nseg; k += kSelThreads) dep[k] = INT_MAX;
  __syncthreads();
  int32_t* kout = kept_idx + static_cast<int64_t>(b) * max_len;
  int32_t* oout = src_ord + static_cast<int64_t>(b) * max_len;
  {
    int er = eq_before;
    for (int t = t_lo; t < t_hi; ++t) {
      if (!kept_tok(t, er)) continue;
      const int so = page_rank[t / BS] * BS + t % BS;
      kout[pos] = t;
      oout[pos] = so;
      if (so / kSegRows != pos / kSegRows) atomicMin(&dep[so / kSegRows], pos / kSegRows);
      ++pos;
    }
  }
  for (int t = total + tid; t < max_len; t += kSelThreads) kout[t] = -1;

  const int need_pages = (total + BS - 1) / BS;
  int32_t* frow = freed + static_cast<int64_t>(b) * MB;
  __syncthreads();  // every table entry was read (pg[]) before any is rewritten
  for (int lb = tid; lb < MB; lb += kSelThreads) btrow[lb] = -1;
  for (int lb = tid; lb < MB; lb += kSelThreads) frow[lb] = -1;
  __syncthreads();
  int vrank = vrank0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    if (k < PPT && pg[k] >= 0 && pg[k] < NB) {
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

// In-place move of the kept rows, kSegRows rows per warp and kMoveWarps16
// warps per CTA (lane 0 of each warp issues its bulk copies).  CTAs take
// their consecutive segments in order from a ticket counter, so every lower
// segment of the same sequence is held by a warp of the same CTA or of an
// earlier ticket, resident or finished, when a segment waits on it.  A segment bulk-loads its moving rows (K and V)
// into shared memory, publishes "read" in flags[ticket], waits until the
// (at most two) segments whose rows read its destination slots have
// published, then bulk-stores its rows.  Reads never wait, so every wait
// ends; each is still bounded, recording 1 in ctrl[1] if it gives up.
// Rows whose source is already their destination are not touched.
constexpr int kMoveWarps16 = 4;  // fp16 move: segments (warps) per CTA, one ticket per CTA

__global__ void __launch_bounds__(32 * kMoveWarps16) move_rows_inplace_kernel(
    const int32_t* __restrict__ kept_idx, const int32_t* __restrict__ src_ord,
    const int32_t* __restrict__ kept_count, const int32_t* __restrict__ seg_dep,
    const int32_t* __restrict__ old_bt, const int32_t* __restrict__ new_bt, int MB, int max_len, int BS,
    int nseg, int total_segs, uint8_t* __restrict__ kpool, uint8_t* __restrict__ vpool, uint32_t row_bytes,
    int* ctrl, int* flags, int seg_stride, uint32_t flag_polls, int withhold_flags) {
  __shared__ int cta_ticket;
  if (threadIdx.x == 0) cta_ticket = atomicAdd(&ctrl[0], 1);
  __syncthreads();
  if ((threadIdx.x & 31) != 0) return;
  const int w = threadIdx.x >> 5;
  extern __shared__ __align__(128) uint8_t stage_all[];
  __shared__ __align__(8) uint64_t bars[kMoveWarps16];
  uint8_t* stage = stage_all + static_cast<size_t>(w) * 2 * kSegRows * row_bytes;
  uint64_t& bar = bars[w];
  const int ticket = cta_ticket * kMoveWarps16 + w;  // this warp's segment, in ticket order
  if (ticket >= total_segs) return;
  const int b = ticket / nseg, k = ticket % nseg;
  const int cnt = kept_count[b];
  const int r0 = k * kSegRows;
  if (r0 >= cnt) return;  // no segment waits on one past the kept rows
  const int nr = min(kSegRows, cnt - r0);
  const int64_t rb = static_cast<int64_t>(b) * max_len;
  const int32_t* obt = old_bt + static_cast<int64_t>(b) * MB;
  const int32_t* nbt = new_bt + static_cast<int64_t>(b) * MB;
  int64_t src[kSegRows], dst[kSegRows];
  uint32_t moving = 0, bytes = 0;
  for (int i = 0; i < nr; ++i) {
    const int row = r0 + i;
    const int t = kept_idx[rb + row];
    src[i] = (static_cast<int64_t>(obt[t / BS]) * BS + t % BS) * row_bytes;
    dst[i] = (static_cast<int64_t>(nbt[row / BS]) * BS + row % BS) * row_bytes;
    if (src_ord[rb + row] != row) {
      moving |= 1u << i;
      bytes += 2 * row_bytes;
    }
  }
  const uint32_t sbar = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
  const uint32_t sstage = static_cast<uint32_t>(__cvta_generic_to_shared(stage));
  if (moving) {
    mbar_init(sbar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(sbar, bytes);
    for (int i = 0; i < nr; ++i) {
      if (!((moving >> i) & 1u)) continue;
      bulk_g2s(sstage + (2 * i) * row_bytes, kpool + src[i], row_bytes, sbar);
      bulk_g2s(sstage + (2 * i + 1) * row_bytes, vpool + src[i], row_bytes, sbar);
    }
    bool landed = false;
    for (uint32_t polls = 0; polls <= kMaxPolls && !landed; ++polls) landed = mbar_try_wait(sbar, 0);
    if (!landed) {
      // The rows never arrived: this segment neither publishes "read" nor
      // stores (its sources stay where they are), records the failure, and
      // gives its copies in flight one more bounded wait before the CTA's
      // shared memory goes away.
      atomicExch(&ctrl[1], 1);
      for (uint32_t polls = 0; polls <= kMaxPolls && !mbar_try_wait(sbar, 0); ++polls) {
      }
      return;
    }
  }
  if (!withhold_flags)
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(flags + static_cast<int64_t>(b) * seg_stride + k), "r"(1) : "memory");
  if (!moving) return;
  const int d = seg_dep[static_cast<int64_t>(b) * seg_stride + k];
  for (int m = d; m < k && m <= d + 1; ++m) {
    const int* f = flags + static_cast<int64_t>(b) * seg_stride + m;
    uint32_t polls = 0;
    int v = 0;
    while (true) {
      asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v) break;
      if (++polls > flag_polls) {
        // A row at this segment's destination may still be unread: skip the
        // stores (the destination keeps its old contents) and record it.
        atomicExch(&ctrl[1], 1);
        return;
      }
      __nanosleep(64);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  for (int i = 0; i < nr; ++i) {
    if (!((moving >> i) & 1u)) continue;
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(kpool + dst[i]),
                 "r"(sstage + (2 * i) * row_bytes), "r"(row_bytes)
                 : "memory");
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(vpool + dst[i]),
                 "r"(sstage + (2 * i + 1) * row_bytes), "r"(row_bytes)
                 : "memory");
  }
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The same move on INT4 pages ([num_blocks][KVH][page bytes], layout of
// int4.cuh): a token row is, in each head's page, a K code row, a V code row
// (16-byte chunks exchanged in pairs on rows whose position has bit 1 set, at
// D = 128), the K scales and the V scales (slots permuted per 16-token tile),
// so the position-dependent parts are re-laid out for the destination.  One
// warp per row, kMoveWarps consecutive rows per CTA taken with one ticket: a
// row only waits for lower rows, held by warps of its own CTA or of a CTA that
// took an earlier ticket, all resident or finished.  The code rows go through
// shared memory by cp.async (four lanes per 64-byte row, so a warp
// instruction reads whole rows of several heads), the scales through
// registers; the read flag is published after the warp's copies landed.
constexpr int kMoveWarps = 8;  // rows (warps) per CTA of the INT4 move, one ticket per CTA

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <int D>
__global__ void __launch_bounds__(32 * kMoveWarps) move_rows_int4_kernel(
    const int32_t* __restrict__ kept_idx, const int32_t* __restrict__ src_ord,
    const int32_t* __restrict__ kept_count, const int32_t* __restrict__ seg_dep,
    const int32_t* __restrict__ old_bt, const int32_t* __restrict__ new_bt, int MB, int max_len, int BS,
    int nseg, int total_rows, uint8_t* __restrict__ pages, int KVH, int64_t page_bytes, int* ctrl, int* flags,
    int seg_stride, uint32_t flag_polls, int withhold_flags) {
  constexpr int G = D / 64;
  constexpr int CB = D / 2;       // code row bytes
  constexpr int LPR = CB / 16;    // lanes per code row (16 bytes each)
  constexpr int HPI = 32 / LPR;   // heads per warp instruction
  extern __shared__ __align__(128) uint8_t stage_rows[];  // per warp: KVH x (K row, V row) code bytes
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __shared__ int cta_ticket;
  // Scales of the rows this CTA moves, stored together once every warp has
  // passed its dependency wait: the CTA's rows are consecutive positions of
  // one destination page, so (when all move) their K scales are 32
  // contiguous bytes per head and their V scales 16 per group.
  __shared__ uint16_t s_sc[kMoveWarps][64][4];  // [row][head][K g0, K g1, V g0, V g1] (KVH <= 64)
  __shared__ int s_dp[kMoveWarps], s_dpos[kMoveWarps], s_ok[kMoveWarps];
  if (threadIdx.x == 0) cta_ticket = atomicAdd(&ctrl[0], 1);
  __syncthreads();
  const int ticket = cta_ticket * kMoveWarps + w;  // this warp's row, in ticket order
  // Returns true when the row was moved (its codes stored) and its scales,
  // left in s_sc, are to be stored at (s_dp, s_dpos).
  auto move_row = [&]() -> bool {
    if (ticket >= total_rows) return false;
    const int b = ticket / nseg, row = ticket % nseg;  // one row per segment
    if (row >= kept_count[b]) return false;
    const int64_t rb = static_cast<int64_t>(b) * max_len;
    int* my_flag = flags + static_cast<int64_t>(b) * seg_stride + row;
    if (src_ord[rb + row] == row) {  // already in place
      if (lane == 0 && !withhold_flags)
        asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(my_flag), "r"(1) : "memory");
      return false;
    }
    const int t = kept_idx[rb + row];
    const int sp = old_bt[static_cast<int64_t>(b) * MB + t / BS], spos = t % BS;
    const int dp = new_bt[static_cast<int64_t>(b) * MB + row / BS], dpos = row % BS;
    const int sswap = (D == 128 && (spos & 2)) ? 2 : 0, dswap = (D == 128 && (dpos & 2)) ? 2 : 0;
    uint8_t* stage = stage_rows + static_cast<size_t>(w) * KVH * 2 * CB;
    const uint32_t sst = static_cast<uint32_t>(__cvta_generic_to_shared(stage));
    // Lane -> (head hs of each group of HPI heads, 16-byte chunk c of its rows):
    // a warp instruction covers HPI whole code rows (coalesced 64-byte runs).
    const int hs = lane / LPR, c = lane % LPR;
    for (int h = hs; h < KVH; h += HPI) {
      const uint8_t* pg = pages + (static_cast<int64_t>(sp) * KVH + h) * page_bytes;
      cp_async16(sst + (2 * h) * CB + 16 * c, pg + spos * CB + 16 * c);
      cp_async16(sst + (2 * h + 1) * CB + 16 * c, pg + BS * CB + spos * CB + 16 * (c ^ sswap));  // logical chunk c
    }
    // Scales (2 G halves per head) through registers: lane h, h + 32.
    uint16_t ks[2][G], vs[2][G];
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      const int h = lane + 32 * hi;
      if (h >= KVH) continue;
      const uint8_t* pg = pages + (static_cast<int64_t>(sp) * KVH + h) * page_bytes;
      const uint16_t* ksp = reinterpret_cast<const uint16_t*>(pg + BS * D) + spos * G;
      const uint16_t* vsp = reinterpret_cast<const uint16_t*>(pg + BS * D + BS * G * 2);
      if constexpr (G == 2) {  // a position's two K scales are one aligned 4-byte word
        const uint32_t k2 = *reinterpret_cast<const uint32_t*>(ksp);
        ks[hi][0] = static_cast<uint16_t>(k2);
        ks[hi][1] = static_cast<uint16_t>(k2 >> 16);
      } else {
        ks[hi][0] = ksp[0];
      }
#pragma unroll
      for (int g = 0; g < G; ++g) vs[hi][g] = vsp[int4_vscale_index(spos, g, G)];
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
    int gave_up = 0;
    if (lane == 0) {
      __threadfence();
      if (!withhold_flags) asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(my_flag), "r"(1) : "memory");
      // Wait until the row that lives at this row's destination has been read.
      const int d = seg_dep[static_cast<int64_t>(b) * seg_stride + row];
      for (int m = d; m < row && m <= d + 1 && !gave_up; ++m) {
        const int* f = flags + static_cast<int64_t>(b) * seg_stride + m;
        uint32_t polls = 0;
        int v = 0;
        while (true) {
          asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
          if (v) break;
          if (++polls > flag_polls) {
            atomicExch(&ctrl[1], 1);
            gave_up = 1;
            break;
          }
          __nanosleep(64);
        }
      }
    }
    // After a give-up the row is not stored: its destination may still hold an
    // unread kept row.
    if (__shfl_sync(0xffffffffu, gave_up, 0)) return false;
    for (int h = hs; h < KVH; h += HPI) {
      uint8_t* pg = pages + (static_cast<int64_t>(dp) * KVH + h) * page_bytes;
      const uint4 kv = *reinterpret_cast<const uint4*>(stage + (2 * h) * CB + 16 * c);
      const uint4 vv = *reinterpret_cast<const uint4*>(stage + (2 * h + 1) * CB + 16 * c);
      *reinterpret_cast<uint4*>(pg + dpos * CB + 16 * c) = kv;
      *reinterpret_cast<uint4*>(pg + BS * CB + dpos * CB + 16 * (c ^ dswap)) = vv;
    }
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      const int h = lane + 32 * hi;
      if (h >= KVH) continue;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        s_sc[w][h][g] = ks[hi][g];
        s_sc[w][h][2 + g] = vs[hi][g];
      }
    }
    if (lane == 0) {
      s_dp[w] = dp;
      s_dpos[w] = dpos;
    }
    return true;
  };
  const bool moved = move_row();
  if (lane == 0) s_ok[w] = moved ? 1 : 0;
  __syncthreads();
  bool whole = (kMoveWarps == 8) && s_dpos[0] % 8 == 0;
#pragma unroll
  for (int r = 0; r < kMoveWarps; ++r)
    whole = whole && s_ok[r] && s_dp[r] == s_dp[0] && s_dpos[r] == s_dpos[0] + r;
  if (whole) {
    // Thread (head, part): part 0..G-1 the K scales of 4 rows each (16 B),
    // part G..2G-1 the 8 V scales of group part - G (16 B; per-tile slot order).
    const int h = threadIdx.x / (2 * G), part = threadIdx.x % (2 * G);
    if (threadIdx.x < KVH * 2 * G) {
      uint8_t* pg = pages + (static_cast<int64_t>(s_dp[0]) * KVH + h) * page_bytes;
      const int p0 = s_dpos[0];
      uint16_t v8[8];
      uint4* dst;
      if (part < G) {
        // K scales of positions p0 .. p0 + 7: [pos][G] halves; this thread's 8 halves
        const int first = part * (8 / G);  // G = 2: rows 0-3 or 4-7; G = 1: rows 0-7
#pragma unroll
        for (int e = 0; e < 8; ++e) v8[e] = s_sc[first + e / G][h][e % G];
        dst = reinterpret_cast<uint4*>(pg + BS * D + (p0 + first) * G * 2);
      } else {
        const int g = part - G;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          // p0 is a multiple of 8, so position p0 + r takes slot (p0 & 8) + this
          // of its 16-token tile (the order int4_vscale_index gives)
          v8[2 * (r & 3) + ((r >> 2) & 1)] = s_sc[r][h][2 + g];
        }
        dst = reinterpret_cast<uint4*>(pg + BS * D + BS * G * 2 + 2 * (((p0 >> 4) * G + g) * 16 + (p0 & 8)));
      }
      *dst = make_uint4(v8[0] | (static_cast<uint32_t>(v8[1]) << 16), v8[2] | (static_cast<uint32_t>(v8[3]) << 16),
                        v8[4] | (static_cast<uint32_t>(v8[5]) << 16), v8[6] | (static_cast<uint32_t>(v8[7]) << 16));
    }
  } else {
    for (int idx = threadIdx.x; idx < kMoveWarps * KVH; idx += blockDim.x) {
      const int r = idx / KVH, h = idx % KVH;
      if (!s_ok[r]) continue;
      uint8_t* pg = pages + (static_cast<int64_t>(s_dp[r]) * KVH + h) * page_bytes;
      uint16_t* ksp = reinterpret_cast<uint16_t*>(pg + BS * D) + s_dpos[r] * G;
      uint16_t* vsp = reinterpret_cast<uint16_t*>(pg + BS * D + BS * G * 2);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        ksp[g] = s_sc[r][h][g];
        vsp[int4_vscale_index(s_dpos[r], g, G)] = s_sc[r][h][2 + g];
      }
    }
  }
}

}  // namespace

// Workspace: old block tables, token sums, source ordinals, segment
// dependencies and flags, and the ticket / status words.  No K/V rows: the
// moves are in place.
static size_t topk_ws_layout(int num_seqs, int max_len, size_t* off_sums, size_t* off_ord, size_t* off_dep,
                             size_t* off_flags, size_t* off_ctrl) {
  const size_t S = static_cast<size_t>(num_seqs);
  const size_t bt_cap = static_cast<size_t>(max_len > 2 * kSelThreads ? max_len : 2 * kSelThreads);
  size_t o = S * bt_cap * 4;  // old block-table copy (max_blocks_per_seq <= max(2048, max_len))
  *off_sums = o;
  o += S * max_len * 4;
  *off_ord = o;
  o += S * max_len * 4;
  *off_dep = o;
  o += S * max_len * 4;  // one dependency and one flag per kept row (kSegRows == 1)
  *off_flags = o;
  o += S * max_len * 4;
  *off_ctrl = o;
  return o + 256;
}

extern "C" __attribute__((visibility("default"))) size_t memopt_evict_topk_workspace_size(int num_seqs, int max_len, int num_heads, int head_dim) {
  if (num_seqs <= 0 || max_len <= 0 || num_heads <= 0 || head_dim <= 0) return 0;
  size_t a, b, c, d, e;
  return topk_ws_layout(num_seqs, max_len, &a, &b, &c, &d, &e);
}

// int4: key_pool holds the INT4 pages [pool_num_blocks][num_heads][page
// bytes] and value_pool is unused.
static int topk_compact(const char* who, bool int4, const float* src, int64_t b_stride, int64_t i_stride, int n_terms,
                        int num_seqs, int num_heads, int max_len, int32_t* block_tables, int max_blocks_per_seq,
                        int32_t* context_lens, void* key_pool, void* value_pool, int pool_num_blocks,
                        int block_size, int head_dim, float retain_ratio, int num_sink_tokens, int32_t* kept_idx,
                        int32_t* kept_count, int32_t* freed_pages, int32_t* freed_count, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!(retain_ratio > 0.f && retain_ratio <= 1.f))
    return fail(MEMOPT_ERR_INVALID_ARG, std::string(who) + ": retain_ratio must be in (0, 1]");
  if (n_terms <= 0 || num_seqs < 0 || num_heads <= 0 || max_len < 0 || max_blocks_per_seq < 0 || pool_num_blocks < 0 ||
      block_size <= 0 || head_dim <= 0)
    return fail(MEMOPT_ERR_INVALID_ARG, std::string(who) + ": invalid geometry");
  if (max_blocks_per_seq > kMaxPagesBig)
    return fail(MEMOPT_ERR_UNSUPPORTED, std::string(who) + ": more than 16384 blocks per sequence");
  if (max_blocks_per_seq > 2 * kSelThreads && max_blocks_per_seq > max_len)
    return fail(MEMOPT_ERR_UNSUPPORTED, std::string(who) + ": more than max(2048, max_len) blocks per sequence");
  if (!int4 && (num_heads * head_dim) % 8 != 0)
    return fail(MEMOPT_ERR_UNSUPPORTED, std::string(who) + ": num_heads * head_dim must be a multiple of 8");
  if (int4 && !((head_dim == 64 || head_dim == 128) && block_size % 16 == 0 && num_heads <= 64))
    return fail(MEMOPT_ERR_UNSUPPORTED,
                std::string(who) + ": INT4 pages need head_dim 64 or 128, block_size % 16 == 0, <= 64 heads");
  if (num_seqs == 0 || max_len == 0) return MEMOPT_OK;
  if (int4) value_pool = key_pool;
  if (!src || !block_tables || !context_lens || !key_pool || !value_pool || !kept_idx || !kept_count ||
      !freed_pages || !freed_count || !workspace)
    return fail(MEMOPT_ERR_INVALID_ARG, std::string(who) + ": null pointer");
  if ((reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool) |
       reinterpret_cast<uintptr_t>(workspace)) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, std::string(who) + ": pools and workspace must be 16-byte aligned");
  const size_t need = memopt_evict_topk_workspace_size(num_seqs, max_len, num_heads, head_dim);
  if (workspace_bytes < need) return fail(MEMOPT_ERR_WORKSPACE, std::string(who) + ": workspace too small");
  cudaStream_t s = as_stream(stream);
  const uint32_t row_bytes = static_cast<uint32_t>(num_heads) * head_dim * 2;
  const size_t stage_bytes = static_cast<size_t>(2 * kSegRows) * row_bytes * kMoveWarps16;
  if (!int4 && stage_bytes > static_cast<size_t>(kMoveSmemLimit))
    return fail(MEMOPT_ERR_UNSUPPORTED, std::string(who) + ": num_heads * head_dim above " +
                                             std::to_string(kMoveSmemLimit / (4 * kSegRows * kMoveWarps16)));
  cudaError_t ea = cudaFuncSetAttribute(move_rows_inplace_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kMoveSmemLimit);
  if (ea != cudaSuccess) return cuda_fail(ea, "evict_topk: shared-memory attribute");
  size_t o_sums, o_ord, o_dep, o_flags, o_ctrl;
  topk_ws_layout(num_seqs, max_len, &o_sums, &o_ord, &o_dep, &o_flags, &o_ctrl);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  int32_t* old_bt = reinterpret_cast<int32_t*>(w);
  float* sums = reinterpret_cast<float*>(w + o_sums);
  int32_t* ord = reinterpret_cast<int32_t*>(w + o_ord);
  int32_t* dep = reinterpret_cast<int32_t*>(w + o_dep);
  int* flags = reinterpret_cast<int*>(w + o_flags);
  int* ctrl = reinterpret_cast<int*>(w + o_ctrl);
  const size_t bt_bytes = static_cast<size_t>(num_seqs) * max_blocks_per_seq * 4;
  cudaError_t e = cudaMemcpyAsync(old_bt, block_tables, bt_bytes, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, (std::string(who) + ": block-table copy").c_str());
  e = cudaMemsetAsync(flags, 0, static_cast<size_t>(num_seqs) * max_len * 4 + 256, s);
  if (e != cudaSuccess) return cuda_fail(e, (std::string(who) + ": clearing flags").c_str());
  head_sum_kernel<<<dim3((max_len + 255) / 256, num_seqs), 256, 0, s>>>(src, b_stride, i_stride, n_terms, max_len, sums);
  MEMOPT_LAUNCH_CHECK("head_sum_kernel launch");
  const int sinks = num_sink_tokens < 0 ? 0 : num_sink_tokens;
  if (max_len <= kMaxLen && max_blocks_per_seq <= 2 * kSelThreads) {
    topk_select_kernel<<<num_seqs, kSelThreads, 0, s>>>(sums, max_len, block_tables, max_blocks_per_seq,
                                                        context_lens, pool_num_blocks, block_size, retain_ratio, sinks,
                                                        kept_idx, kept_count, freed_pages, freed_count, ord, dep,
                                                        max_len);
    MEMOPT_LAUNCH_CHECK("topk_select_kernel launch");
  } else {
    const size_t psm = static_cast<size_t>(max_blocks_per_seq) * 4;
    cudaError_t eb = cudaFuncSetAttribute(topk_select_big_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          kMaxPagesBig * 4);
    if (eb != cudaSuccess) return cuda_fail(eb, "evict_topk: shared-memory attribute (select)");
    topk_select_big_kernel<<<num_seqs, kSelThreads, psm, s>>>(
        sums, max_len, block_tables, max_blocks_per_seq, context_lens, pool_num_blocks, block_size, retain_ratio, sinks,
        kept_idx, kept_count, freed_pages, freed_count, ord, dep, max_len);
    MEMOPT_LAUNCH_CHECK("topk_select_big_kernel launch");
  }
  const int nseg = (max_len + kSegRows - 1) / kSegRows;
  const uint32_t polls = g_flag_polls.load(std::memory_order_relaxed);
  const int withhold = g_withhold_flags.load(std::memory_order_relaxed);
  if (int4) {
    const int64_t pb = static_cast<int64_t>(block_size) * head_dim + static_cast<int64_t>(block_size) * (head_dim / 64) * 4;
    uint8_t* pages = static_cast<uint8_t*>(key_pool);
    const int rows_total = num_seqs * nseg;
    const int grid4 = (rows_total + kMoveWarps - 1) / kMoveWarps;
    const size_t smem4 = static_cast<size_t>(kMoveWarps) * num_heads * head_dim;  // 2 code rows of D/2 per head
    cudaError_t ea4 = head_dim == 128 ? cudaFuncSetAttribute(move_rows_int4_kernel<128>,
                                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024)
                                      : cudaFuncSetAttribute(move_rows_int4_kernel<64>,
                                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (ea4 != cudaSuccess) return cuda_fail(ea4, "evict_topk_int4: shared-memory attribute");
    if (head_dim == 128)
      move_rows_int4_kernel<128><<<grid4, 32 * kMoveWarps, smem4, s>>>(
          kept_idx, ord, kept_count, dep, old_bt, block_tables, max_blocks_per_seq, max_len, block_size, nseg,
          rows_total, pages, num_heads, pb, ctrl, flags, max_len, polls, withhold);
    else
      move_rows_int4_kernel<64><<<grid4, 32 * kMoveWarps, smem4, s>>>(
          kept_idx, ord, kept_count, dep, old_bt, block_tables, max_blocks_per_seq, max_len, block_size, nseg,
          rows_total, pages, num_heads, pb, ctrl, flags, max_len, polls, withhold);
    MEMOPT_LAUNCH_CHECK("move_rows_int4_kernel launch");
    return MEMOPT_OK;
  }
  const int segs = num_seqs * nseg;
  move_rows_inplace_kernel<<<(segs + kMoveWarps16 - 1) / kMoveWarps16, 32 * kMoveWarps16, stage_bytes, s>>>(
      kept_idx, ord, kept_count, dep, old_bt, block_tables, max_blocks_per_seq, max_len, block_size, nseg, segs,
      static_cast<uint8_t*>(key_pool), static_cast<uint8_t*>(value_pool), row_bytes, ctrl, flags, max_len, polls,
      withhold);
  MEMOPT_LAUNCH_CHECK("move_rows_inplace_kernel launch");
  return MEMOPT_OK;
}


extern "C" __attribute__((visibility("default"))) int memopt_evict_topk_compact(
    const float* scores, int num_seqs, int num_heads, int max_len, int32_t* block_tables, int max_blocks_per_seq,
    int32_t* context_lens, void* key_pool, void* value_pool, int pool_num_blocks, int block_size, int head_dim,
    float retain_ratio, int num_sink_tokens, int32_t* kept_idx, int32_t* kept_count, int32_t* freed_pages,
    int32_t* freed_count, void* workspace, size_t workspace_bytes, void* stream) {
  return topk_compact("evict_topk_compact", false, scores, static_cast<int64_t>(num_heads) * max_len, max_len, num_heads,
                      num_seqs, num_heads, max_len, block_tables, max_blocks_per_seq, context_lens, key_pool,
                      value_pool, pool_num_blocks, block_size, head_dim, retain_ratio, num_sink_tokens, kept_idx,
                      kept_count, freed_pages, freed_count, workspace, workspace_bytes, stream);
}

extern "C" __attribute__((visibility("default"))) int memopt_evict_topk_head_sum(const float* scores, int num_seqs,
                                                                                int num_heads, int max_len,
                                                                                float* sums, void* stream) {
  if (num_seqs < 0 || num_heads <= 0 || max_len < 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_head_sum: invalid geometry");
  if (num_seqs == 0 || max_len == 0) return MEMOPT_OK;
  if (!scores || !sums) return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_head_sum: null pointer");
  head_sum_kernel<<<dim3((max_len + 255) / 256, num_seqs), 256, 0, as_stream(stream)>>>(
      scores, static_cast<int64_t>(num_heads) * max_len, max_len, num_heads, max_len, sums);
  MEMOPT_LAUNCH_CHECK("head_sum_kernel launch");
  return MEMOPT_OK;
}

extern "C" __attribute__((visibility("default"))) int memopt_evict_topk_compact_parts(
    const float* partial_sums, int num_parts, int num_seqs, int max_len, int32_t* block_tables,
    int max_blocks_per_seq, int32_t* context_lens, void* key_pool, void* value_pool, int pool_num_blocks,
    int block_size, int num_heads, int head_dim, float retain_ratio, int num_sink_tokens, int32_t* kept_idx,
    int32_t* kept_count, int32_t* freed_pages, int32_t* freed_count, void* workspace, size_t workspace_bytes,
    void* stream) {
  return topk_compact("evict_topk_compact_parts", false, partial_sums, max_len, static_cast<int64_t>(num_seqs) * max_len,
                      num_parts, num_seqs, num_heads, max_len, block_tables, max_blocks_per_seq, context_lens,
                      key_pool, value_pool, pool_num_blocks, block_size, head_dim, retain_ratio, num_sink_tokens,
                      kept_idx, kept_count, freed_pages, freed_count, workspace, workspace_bytes, stream);
}

extern "C" __attribute__((visibility("default"))) int memopt_evict_topk_compact_int4(
    const float* scores, int num_seqs, int num_heads, int max_len, int32_t* block_tables, int max_blocks_per_seq,
    int32_t* context_lens, uint8_t* kv_pages, int pool_num_blocks, int block_size, int head_dim, float retain_ratio,
    int num_sink_tokens, int32_t* kept_idx, int32_t* kept_count, int32_t* freed_pages, int32_t* freed_count,
    void* workspace, size_t workspace_bytes, void* stream) {
  return topk_compact("evict_topk_compact_int4", true, scores, static_cast<int64_t>(num_heads) * max_len, max_len,
                      num_heads, num_seqs, num_heads, max_len, block_tables, max_blocks_per_seq, context_lens, kv_pages,
                      nullptr, pool_num_blocks, block_size, head_dim, retain_ratio, num_sink_tokens, kept_idx,
                      kept_count, freed_pages, freed_count, workspace, workspace_bytes, stream);
}

extern "C" __attribute__((visibility("default"))) int memopt_evict_topk_set_test_hooks(uint32_t flag_poll_limit,
                                                                                      int withhold_read_flags) {
  g_flag_polls.store(flag_poll_limit == 0 ? kMaxPolls : flag_poll_limit, std::memory_order_relaxed);
  g_withhold_flags.store(withhold_read_flags ? 1 : 0, std::memory_order_relaxed);
  return MEMOPT_OK;
}

extern "C" __attribute__((visibility("default"))) int memopt_evict_topk_status(const void* workspace, int num_seqs,
                                                                              int max_len, void* stream) {
  if (num_seqs < 0 || max_len < 0) return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_status: invalid geometry");
  if (num_seqs == 0 || max_len == 0) return MEMOPT_OK;
  if (!workspace) return fail(MEMOPT_ERR_INVALID_ARG, "evict_topk_status: null workspace");
  size_t o_sums, o_ord, o_dep, o_flags, o_ctrl;
  topk_ws_layout(num_seqs, max_len, &o_sums, &o_ord, &o_dep, &o_flags, &o_ctrl);
  int ctrl1 = 0;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(&ctrl1, static_cast<const uint8_t*>(workspace) + o_ctrl + 4, 4,
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "evict_topk_status: reading the status word");
  if (ctrl1 != 0)
    return fail(MEMOPT_ERR_TIMEOUT,
                "evict_topk: a row move gave up waiting; rows whose wait ran out were not stored, so the pool, "
                "block tables and lengths are only partly compacted (no kept row was overwritten before it was read)");
  return MEMOPT_OK;
}

}  // namespace memopt
