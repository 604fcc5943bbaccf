// decode_kernel.cuh — paged, block-skipping, split-K flash-decode for sm_100a.
//
// Semantics follow sparse_flash_attention_kernel (reference
// src/csrc/attention.cu:98-339): for query row (b, q, h) the visible tokens
// are [max(0, ctx_b - W), ctx_b) of every logical page whose block-table
// entry is >= 0; no causal mask; out = sum_t softmax_t * V_t, or 0 when no
// token is visible.  Pages whose entry is >= num_blocks are skipped as well
// (the reference would read out of bounds there).
//
// Execution model (independent of the reference's one-CTA-per-row loop):
//   * work item = (query row, chunk of <= 32 consecutive logical pages);
//     each WARP processes items grid-strided, with no CTA-wide barriers;
//   * every warp owns a ring of NS shared-memory stages; lane 0 streams the
//     K/V pages of its items (crossing item boundaries) into the ring with
//     the TMA engine (3-D tensor map for the fp16 pool, 1-D bulk copies for
//     the contiguous INT4 pages) and mbarrier completion;
//   * a lane owns 8 head dims; a page is consumed as rows of LPR = D/8 lanes,
//     dot products are finished by a transpose-reduction (one value per lane
//     after log2(LPR) butterfly rounds), the online softmax runs in the log2
//     domain (q pre-scaled by log2(e)/sqrt(D)) with exp2f;
//   * items of a row write (m, l, o[D]) partials; the last item to finish
//     (atomic ticket) merges them in chunk order, so results are
//     deterministic, and resets the ticket for the next call.
#pragma once
#include "common.cuh"
#include "int4_mma.cuh"

namespace memopt {
namespace decode {

struct Params {
  const __half* q;   // [B, QL, H, D]
  __half* out;       // [B, QL, H, D]
  const int32_t* bt;   // [B, MB]
  const int32_t* ctx;  // [B]
  // INT4 pool: one page of PAGE_RAW bytes per (block, head)
  const uint8_t* pages;
  // split-K workspace
  int32_t* tickets;  // [pairs]
  float2* ml;        // [pairs * n_chunks]
  float* po;         // [pairs * n_chunks * D]
  int B, QL, H, MB;
  int KVH;     // heads of the pool (divides H)
  int group;   // H / KVH: query heads per KV head (grouped-query attention)
  int causal;  // 1: query row i of QL sees tokens up to ctx - QL + i (extension)
  int64_t NB;
  int window;    // already clamped as in attention.cu:453-455
  float qscale;  // log2(e) / sqrt(D)
  // INT4 code conversion constants, passed at run time so that they stay in
  // registers and every (x & mask) | const or (x & mask) ^ const is a single
  // three-input logic op: 0x64006400 (fp16 1024 in both halves), 0x80808080.
  uint32_t magic_f16;
  uint32_t magic_s8;
  int chunk_pages;  // pages per item (walked in 32-page sub-windows)
  int n_chunks;
  int64_t total_items;
};

template <int D, int BS, bool INT4>
struct Cfg {
  static constexpr int LPR = D / 8;     // lanes per page row
  static constexpr int RPI = 32 / LPR;  // rows per warp instruction
  static constexpr int TPL = BS / RPI;  // rows (tokens) per lane per page
  static constexpr int DUP = LPR / TPL; // lanes holding the same score
  static constexpr int K_BYTES = INT4 ? BS * D / 2 : BS * D * 2;
  static constexpr int S_BYTES = INT4 ? BS * (D / 64) * 2 : 0;
  static constexpr int PAGE_RAW = 2 * K_BYTES + 2 * S_BYTES;  // one page (INT4: one (block, head) page)
  // INT4 with 16-token pages: a stage holds two pages (the two tiles of one
  // softmax step) behind one mbarrier, halving the per-page pipeline work.
  static constexpr int PPS = (INT4 && BS == 16) ? 2 : 1;
  static constexpr int STAGE_RAW = PPS * PAGE_RAW;
  static constexpr int STAGE = (STAGE_RAW + 127) / 128 * 128;
  // fp16 pages are large: 3 stages of 8 KB per warp, 2 CTAs (8 warps) per SM.
  // INT4 pages are small and their consumer is issue-latency bound: ~12 KB of
  // stages per warp (two 2-page stages at 16-token pages) and 4 CTAs
  // (16 warps) per SM at <= 128 registers; occupancy matters more here than
  // ring depth (3 CTAs with four 2-page stages per warp measured slower).
  static constexpr int WARP_BUDGET = INT4 ? 12288 : 24576;
  static constexpr int NS_RAW = WARP_BUDGET / STAGE;
  // INT4: largest power of two that fits (the ring index is then a mask;
  // per-page integer overhead matters at 2 KB pages).  fp16: as many as fit.
  static constexpr int NS_P2 = NS_RAW >= 16 ? 16 : NS_RAW >= 8 ? 8 : NS_RAW >= 4 ? 4 : 2;
  static constexpr int NS = INT4 ? NS_P2 : (NS_RAW < 2 ? 2 : (NS_RAW > 16 ? 16 : NS_RAW));
  static constexpr int NW = 4;            // warps per CTA
  static constexpr int MIN_BLOCKS = INT4 ? 4 : 2;
  static constexpr int BAR_BYTES = 1024;  // mbarriers
  static constexpr int SMEM = BAR_BYTES + NW * NS * STAGE;
  static_assert(TPL >= 1 && DUP >= 1, "unsupported geometry");
  static_assert(NW * NS * 8 <= BAR_BYTES, "barrier area too small");
};


template <int D, int BS, bool INT4>
__global__ void __launch_bounds__(Cfg<D, BS, INT4>::NW * 32, Cfg<D, BS, INT4>::MIN_BLOCKS)
paged_decode_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap, int32_t* __restrict__ err) {
  using C = Cfg<D, BS, INT4>;
  constexpr int NS = C::NS;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + wid * NS;
  uint8_t* stages = smem + C::BAR_BYTES + wid * NS * C::STAGE;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t st0 = smem_u32(stages);

  if (lane == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
    if (!INT4) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
  }
  __syncwarp();

  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * C::NW;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * C::NW + wid;

  // Decodes an item and ballots the valid pages of sub-window `sub` (32 pages)
  // of its chunk; `more` tells whether the chunk has pages beyond it.
  auto load_item = [&](int64_t item, int sub, uint32_t& mask, int& phys_lane, int& h, int& c_lo,
                       int& win_start, int& ctx, bool& more) {
    const int64_t pair = item / p.n_chunks;
    const int chunk = static_cast<int>(item - pair * p.n_chunks);
    h = static_cast<int>(pair % p.H) / p.group;  // the KV head this query head reads
    const int64_t bq = pair / p.H;
    const int b = static_cast<int>(bq / p.QL);
    ctx = __ldg(p.ctx + b);
    // Causal rows: row i of the QL query rows is the token at ctx - QL + i.
    if (p.causal) ctx = ctx - p.QL + static_cast<int>(bq - static_cast<int64_t>(b) * p.QL) + 1;
    win_start = (p.window < ctx) ? (ctx - p.window) : 0;
    int p_hi = 0;
    if (ctx > 0) p_hi = min((ctx + BS - 1) / BS, p.MB);
    const int p_lo = win_start / BS;
    const int k_lo = p_lo + chunk * p.chunk_pages;
    const int k_hi = min(k_lo + p.chunk_pages, p_hi);
    c_lo = k_lo + 32 * sub;
    const int c_hi = min(c_lo + 32, k_hi);
    more = c_lo + 32 < k_hi;
    const int page = c_lo + lane;
    phys_lane = -1;
    if (page < c_hi) phys_lane = __ldg(p.bt + static_cast<int64_t>(b) * p.MB + page);
    const bool ok = page < c_hi && phys_lane >= 0 && static_cast<int64_t>(phys_lane) < p.NB;
    mask = __ballot_sync(0xffffffffu, ok);
  };

  // phys2 >= 0: a second page into the same stage (INT4, PPS == 2).
  auto issue = [&](uint32_t seq, int phys, int phys2, int h) {
    const int s = static_cast<int>(seq % NS);
    const uint32_t bar = bar0 + 8 * s;
    const uint32_t dst = st0 + s * C::STAGE;
    fence_proxy_async_smem();
    if (!INT4) {
      mbar_arrive_expect_tx(bar, C::STAGE_RAW);
      tma_load_3d(dst, &kmap, 0, h, phys * BS, bar);
      tma_load_3d(dst + C::K_BYTES, &vmap, 0, h, phys * BS, bar);
    } else {
      mbar_arrive_expect_tx(bar, (C::PPS == 2 && phys2 >= 0) ? 2 * C::PAGE_RAW : C::PAGE_RAW);
      bulk_g2s(dst, p.pages + (static_cast<int64_t>(phys) * p.KVH + h) * C::PAGE_RAW, C::PAGE_RAW, bar);
      if (C::PPS == 2 && phys2 >= 0)
        bulk_g2s(dst + C::PAGE_RAW, p.pages + (static_cast<int64_t>(phys2) * p.KVH + h) * C::PAGE_RAW,
                 C::PAGE_RAW, bar);
    }
  };

  // ---------------- producer cursor (warp-uniform) ----------------------
  int64_t p_item = first - nwarps;  // advanced before first use
  int p_sub = 0;
  bool p_more = false;
  uint32_t p_mask = 0;
  int p_phys = -1;  // this lane's page entry for the producer's window
  int p_h = 0;
  uint32_t p_seq = 0;
  bool p_done = false;

  // Issues the next page of the warp's page stream (if any).
  auto produce = [&]() {
    while (!p_done && p_mask == 0) {
      if (p_more) {
        ++p_sub;
      } else {
        p_item += nwarps;
        p_sub = 0;
        if (p_item >= p.total_items) {
          p_done = true;
          break;
        }
      }
      int c_lo, ws, cx;
      load_item(p_item, p_sub, p_mask, p_phys, p_h, c_lo, ws, cx, p_more);
    }
    if (p_done) return;
    const int j = __ffs(p_mask) - 1;
    p_mask &= p_mask - 1;
    const int phys = __shfl_sync(0xffffffffu, p_phys, j);
    int phys2 = -1;
    if (C::PPS == 2 && p_mask != 0) {  // the consumer pairs pages the same way
      const int j2 = __ffs(p_mask) - 1;
      p_mask &= p_mask - 1;
      phys2 = __shfl_sync(0xffffffffu, p_phys, j2);
    }
    if constexpr (INT4) {
      // Warp-collective issue: one elected lane arms the stage's mbarrier and
      // starts the copies, with no divergent branch around it.
      const int s = static_cast<int>(p_seq % NS);
      const uint32_t bar = bar0 + 8 * s;
      const uint32_t dst = st0 + s * C::STAGE;
      const uint32_t bytes = (C::PPS == 2 && phys2 >= 0) ? 2 * C::PAGE_RAW : C::PAGE_RAW;
      const uint8_t* src1 = p.pages + (static_cast<int64_t>(phys) * p.KVH + p_h) * C::PAGE_RAW;
      const uint8_t* src2 = p.pages + (static_cast<int64_t>(phys2 >= 0 ? phys2 : phys) * p.KVH + p_h) * C::PAGE_RAW;
      const uint32_t two = (C::PPS == 2 && phys2 >= 0) ? 1u : 0u;
      asm volatile(
          "{\n\t.reg .pred pe, p2;\n\t"
          "elect.sync _|pe, 0xffffffff;\n\t"
          "setp.ne.and.u32 p2, %5, 0, pe;\n\t"
          "@pe fence.proxy.async.shared::cta;\n\t"
          "@pe mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t"
          "@pe cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%3], %6, [%0];\n\t"
          "@p2 cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%7], [%4], %6, [%0];\n\t"
          "}" ::"r"(bar), "r"(bytes), "r"(dst), "l"(src1), "l"(src2), "r"(two), "r"(static_cast<uint32_t>(C::PAGE_RAW)),
          "r"(dst + static_cast<uint32_t>(C::PAGE_RAW))
          : "memory");
    } else {
      if (lane == 0) issue(p_seq, phys, phys2, p_h);
    }
    ++p_seq;
  };

  for (int s = 0; s < NS; ++s) produce();

  // ---------------- consumer -------------------------------------------
  const int r = lane / C::LPR;   // fp16: row within a warp instruction
  const int cl = lane % C::LPR;  // fp16: 8-dim column chunk
  const int mg = lane >> 2;      // int4 (mma fragments): group id
  const int mt4 = lane & 3;      // int4 (mma fragments): thread in group
  constexpr int G = D / 64;      // int4 scale groups per row
  constexpr int NKB = D / 32;    // int4: k-blocks of the score mma (= P.V dim-block pairs)
  const uint32_t kF16 = p.magic_f16;
  const uint32_t kS8 = p.magic_s8;
  // INT4: this lane's byte offsets inside a page stage (tile 0).
  const int i4_grp = G > 1 ? (mg & 1) : 0;  // B column mg of P.V -> scale group (columns >= G unused)
  const uint32_t o_k = mg * (D / 2) + mt4 * (D / 8);                        // K row mg; row mg + 8 at + 8 D/2
  const uint32_t o_ks = 2 * C::K_BYTES + (mg * G + (G > 1 ? (mt4 & 1) : 0)) * 2;  // row mg + 8 at + 16 G
  const uint32_t o_v = C::K_BYTES + (D == 128 ? mt4 * 64 + 8 * (mg ^ ((mt4 & 2) ? 4 : 0)) : mt4 * 32 + 4 * mg);
  const uint32_t o_vs = 2 * C::K_BYTES + C::S_BYTES + i4_grp * 32 + 4 * mt4;
  uint32_t c_seq = 0;
  bool failed = false;

  for (int64_t item = first; item < p.total_items && !failed; item += nwarps) {
    uint32_t mask;
    int phys_lane, h, c_lo, win_start, ctx;
    bool more;
    int sub = 0;
    load_item(item, 0, mask, phys_lane, h, c_lo, win_start, ctx, more);
    const int64_t pair = item / p.n_chunks;

    float q[8];
    // INT4: B operand of the score mma (m16n8k32, s8).  q is rounded to 16-bit
    // integers q_int = rint(q / qsc) (|q_int| <= 32639) and split exactly as
    // q_int = 256 hi + lo with hi, lo in [-128, 127]; column n < 2G of B holds
    // part (n & 1 ? lo : hi) of the dims of scale group n >> 1.  Lane (mg, mt4)
    // of k-block kb covers word wi = NKB*mt4 + kb of a K row: its even
    // dims in b0, its odd dims in b1 (the A side splits the word the same way).
    uint32_t qb[INT4 ? NKB : 1][2];
    float sfac = 0.f;
    if constexpr (!INT4) {
      const uint4 qv = *reinterpret_cast<const uint4*>(p.q + pair * D + cl * 8);
      const __half2* q2 = reinterpret_cast<const __half2*>(&qv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(q2[i]);
        q[2 * i] = f.x * p.qscale;
        q[2 * i + 1] = f.y * p.qscale;
      }
    } else {
      const __half* qrow = p.q + pair * D;
      float am = 0.f;
#pragma unroll
      for (int e = lane; e < D; e += 32) am = fmaxf(am, fabsf(__half2float(qrow[e])));
#pragma unroll
      for (int mk = 16; mk >= 1; mk >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, mk));
      const float qsc = am > 0.f ? am / 32639.f : 1.f;
      const float qinv = am > 0.f ? 32639.f / am : 1.f;
      // score = sum_g ks_g * sum_d 16 (c - 8) q_int * qsc / 16, then * qscale
      sfac = qsc * 0.0625f * p.qscale;
      const bool part_lo = (mg & 1) != 0;
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) {
        const int wi = NKB * mt4 + kb;  // word of the K row: dims 8 wi .. 8 wi + 7
        const bool use = mg < 2 * G && (mg >> 1) == wi / 8;
#pragma unroll
        for (int odd = 0; odd < 2; ++odd) {
          uint32_t r = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int qi = __float2int_rn(__half2float(qrow[8 * wi + 2 * e + odd]) * qinv);
            const int lo = ((qi + 128) & 255) - 128;
            const int hi = (qi - lo) >> 8;
            r |= (static_cast<uint32_t>(part_lo ? lo : hi) & 0xFFu) << (8 * e);
          }
          qb[kb][odd] = use ? r : 0u;
        }
      }
    }
    float m = -INFINITY, l = 0.f;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.f;
    // INT4 P.V accumulators: (D/32) dim blocks x (low, high nibble) fragments.
    float acc[INT4 ? 2 * NKB : 1][4];
#pragma unroll
    for (int j = 0; j < (INT4 ? 2 * NKB : 1); ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    // INT4: the V codes enter the P.V mma as 1024 + c (low nibbles) and
    // 1024 + 16 c (high nibbles); wsum (same fragment layout) accumulates the
    // B column sums, and every kFlushSteps steps (and at the end of the item)
    // the offsets are removed: low -= 1032 wsum, high -= 1152 wsum (the high
    // fragments carry 16x the value).  Bounding the span keeps the common
    // offset in the fp32 accumulators small relative to the result.
    float wsum[4] = {0.f, 0.f, 0.f, 0.f};
    int since_flush = 0;
    constexpr int kFlushSteps = 4;
    auto flush_offsets = [&]() {
      if constexpr (INT4) {
#pragma unroll
        for (int j = 0; j < NKB; ++j) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * j][e] = fmaf(-1032.f, wsum[e], acc[2 * j][e]);
            acc[2 * j + 1][e] = fmaf(-1152.f, wsum[e], acc[2 * j + 1][e]);
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) wsum[e] = 0.f;
        since_flush = 0;
      }
    };

    // Warp-uniform bounded wait for stage `seq` (a completed phase stays observable).
    auto wait_stage = [&](uint32_t seq) -> bool {
      const int st = static_cast<int>(seq % NS);
      const uint32_t parity = (seq / NS) & 1u;
      uint32_t polls = 0;
      bool ready = mbar_try_wait(bar0 + 8 * st, parity);
      while (!__all_sync(0xffffffffu, ready) && ++polls < kMaxPolls) {
        if (!ready) ready = mbar_try_wait(bar0 + 8 * st, parity);
      }
      return __all_sync(0xffffffffu, ready);
    };

    for (;;) {  // 32-page sub-windows of the chunk
    if constexpr (!INT4) {
      while (mask != 0) {
        const int jpage = __ffs(mask) - 1;
        mask &= mask - 1;
        const int page = c_lo + jpage;
        if (!wait_stage(c_seq)) {
          failed = true;
          break;
        }
        const uint8_t* stg = stages + static_cast<int>(c_seq % NS) * C::STAGE;
        // ---- scores: lane partials for TPL rows, then transpose-reduce ----
        float val[C::TPL];
#pragma unroll
        for (int i = 0; i < C::TPL; ++i) {
          const int t = i * C::RPI + r;
          const uint4 kv = *reinterpret_cast<const uint4*>(stg + t * D * 2 + cl * 16);
          const __half2* k2 = reinterpret_cast<const __half2*>(&kv);
          float a = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(k2[e]);
            a = fmaf(q[2 * e], f.x, a);
            a = fmaf(q[2 * e + 1], f.y, a);
          }
          val[i] = a;
        }
        int idx = 0;
        {
          int n = C::TPL;
#pragma unroll
          for (int mk = C::LPR / 2; mk >= 1; mk >>= 1) {
            if (n > 1) {
              const int half = n / 2;
              const bool up = (lane & mk) != 0;
#pragma unroll
              for (int i = 0; i < (C::TPL + 1) / 2; ++i) {
                if (i < half) {
                  const float send = up ? val[i] : val[i + half];
                  const float keepv = up ? val[i + half] : val[i];
                  val[i] = keepv + __shfl_xor_sync(0xffffffffu, send, mk);
                }
              }
              if (up) idx += half;
              n = half;
            } else {
              val[0] += __shfl_xor_sync(0xffffffffu, val[0], mk);
            }
          }
        }
        const int tok = page * BS + idx * C::RPI + r;
        const float s2 = (tok >= win_start && tok < ctx) ? val[0] : -INFINITY;
        float mp = s2;
#pragma unroll
        for (int mk = 16; mk >= 1; mk >>= 1) mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, mk));
        const float m_new = fmaxf(m, mp);
        if (m_new != -INFINITY) {
          const float alpha = exp2f(m - m_new);
          const float pr = exp2f(s2 - m_new);
          const bool dup = (lane & (C::DUP - 1)) != 0;
          l = l * alpha + (dup ? 0.f : pr);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] *= alpha;
          m = m_new;
#pragma unroll
          for (int i = 0; i < C::TPL; ++i) {
            const int t = i * C::RPI + r;
            const float pi = __shfl_sync(0xffffffffu, pr, r * C::LPR + i * C::DUP);
            const uint4 vv = *reinterpret_cast<const uint4*>(stg + C::K_BYTES + t * D * 2 + cl * 16);
            const __half2* v2 = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(v2[e]);
              o[2 * e] = fmaf(pi, f.x, o[2 * e]);
              o[2 * e + 1] = fmaf(pi, f.y, o[2 * e + 1]);
            }
          }
        }
        __syncwarp();
        ++c_seq;
        produce();
      }
    } else {
      using namespace int4mma;
      // Whether every token of the pages in this sub-window is visible (the
      // usual case): then no tile needs per-token masking.
      const bool sub_interior = mask != 0 && (c_lo + __ffs(mask) - 1) * BS >= win_start &&
                                (c_lo + 32 - __clz(mask)) * BS <= ctx;
      // Two 16-token tiles per softmax step: both halves of a 32-token page,
      // or two consecutive 16-token pages of the item.
      while (mask != 0) {
        const int ja = __ffs(mask) - 1;
        mask &= mask - 1;
        const bool two_pages = (BS == 16) && (mask != 0);
        int jb = ja;
        if (two_pages) {
          jb = __ffs(mask) - 1;
          mask &= mask - 1;
        }
        if (!wait_stage(c_seq)) {
          failed = true;
          break;
        }
        {
        const uint32_t sa = st0 + static_cast<uint32_t>(c_seq % NS) * C::STAGE;
        const uint32_t sb = sa + C::PAGE_RAW;  // second page of the stage (BS == 16)
        const bool has2 = (BS == 32) || two_pages;
        // tile ti: stage base and the tile's index inside its page (BS == 32
        // pages hold two 16-token tiles).
        const uint32_t tb[2] = {sa, (BS == 32) ? sa : sb};
        const int tt[2] = {0, (BS == 32) ? 1 : 0};
        const int ttok[2] = {(c_lo + ja) * BS, (BS == 32) ? (c_lo + ja) * BS + 16 : (c_lo + jb) * BS};
        float slo[2], shi[2];
        // ---- scores: exact integer products on the tensor pipe ----
        // A = K codes as signed bytes 16 (c - 8) (rows: tokens mg, mg + 8),
        // B = q_int halves (qb); lane mt4 < G gets the group-mt4 sums.
#pragma unroll
        for (int ti = 0; ti < 2; ++ti) {
          // Without a second page the tile is still computed on the stage's
          // stale bytes and masked below: a branch here would keep the two
          // tiles' conversion and mma chains from interleaving.
          slo[ti] = -INFINITY;
          shi[ti] = -INFINITY;
          const uint32_t kr = tb[ti] + tt[ti] * 16 * (D / 2) + o_k;
          uint32_t w0[NKB], w1[NKB];
          if constexpr (D == 128) {
            const uint4 x0 = lds_v4(kr);
            const uint4 x1 = lds_v4(kr + 8 * (D / 2));
            w0[0] = x0.x; w0[1] = x0.y; w0[2] = x0.z; w0[3] = x0.w;
            w1[0] = x1.x; w1[1] = x1.y; w1[2] = x1.z; w1[3] = x1.w;
          } else {
            const uint2 x0 = lds_v2(kr);
            const uint2 x1 = lds_v2(kr + 8 * (D / 2));
            w0[0] = x0.x; w0[1] = x0.y;
            w1[0] = x1.x; w1[1] = x1.y;
          }
          const uint32_t ksa = tb[ti] + tt[ti] * 16 * G * 2 + o_ks;
          const float ks_lo = lds_f16_as_f32(ksa);
          const float ks_hi = lds_f16_as_f32(ksa + 16 * G);
          int c[4] = {0, 0, 0, 0};
#pragma unroll
          for (int kb = 0; kb < NKB; ++kb) {
            uint32_t a[4];
            a[0] = s8x16_even(w0[kb], kS8);
            a[1] = s8x16_even(w1[kb], kS8);
            a[2] = s8x16_odd(w0[kb], kS8);
            a[3] = s8x16_odd(w1[kb], kS8);
            mma_s8(c, a, qb[kb][0], qb[kb][1]);
          }
          // Lanes mt4 >= G compute a value that is never used: the two group
          // sums meet in lanes mt4 = 0, 1.
          float a_lo = ks_lo * static_cast<float>(c[0] * 256 + c[1]);
          float a_hi = ks_hi * static_cast<float>(c[2] * 256 + c[3]);
          if constexpr (G > 1) {
            a_lo += __shfl_xor_sync(0xffffffffu, a_lo, 1);
            a_hi += __shfl_xor_sync(0xffffffffu, a_hi, 1);
          }
          // Only lanes mt4 == 0 hold the scores from here on: they are the
          // only sources of the P.V operand, of l and of the step max (other
          // lanes' values are never read).
          a_lo *= sfac;
          a_hi *= sfac;
          const int tl = ttok[ti] + mg;
          const bool interior = sub_interior || (ttok[ti] >= win_start && ttok[ti] + 16 <= ctx);
          slo[ti] = (interior || (tl >= win_start && tl < ctx)) ? a_lo : -INFINITY;
          shi[ti] = (interior || (tl + 8 >= win_start && tl + 8 < ctx)) ? a_hi : -INFINITY;
          if (ti == 1 && !has2) slo[ti] = shi[ti] = -INFINITY;  // no second page: stale stage bytes
        }
        // Step max over the lanes that own scores (mt4 == 0), in one warp
        // reduction on an order-preserving integer image of the floats
        // (f >= 0: its bits; f < 0: bits ^ 0x7fffffff; the map is its own inverse).
        float mp = fmaxf(fmaxf(slo[0], shi[0]), fmaxf(slo[1], shi[1]));
        int mk = __float_as_int(mt4 == 0 ? mp : -INFINITY);
        mk ^= (mk >> 31) & 0x7fffffff;
        mk = __reduce_max_sync(0xffffffffu, mk);
        mk ^= (mk >> 31) & 0x7fffffff;
        mp = __int_as_float(mk);
        const float m_new = fmaxf(m, mp);
        {
          // Nothing visible yet: subtract 0 (every p is 0) and keep the
          // (zero) accumulators unscaled, so no branch skips the step.
          const float msub = m_new == -INFINITY ? 0.f : m_new;
          const float alpha = m == -INFINITY ? 1.f : ex2_approx(m - msub);
          m = m_new;
#pragma unroll
          for (int ti = 0; ti < 2; ++ti) {
            slo[ti] = ex2_approx(slo[ti] - msub);
            shi[ti] = ex2_approx(shi[ti] - msub);
          }
          const float psum = (slo[0] + shi[0]) + (slo[1] + shi[1]);
          l = l * alpha + (mt4 == 0 ? psum : 0.f);
          if (alpha != 1.f) {  // warp-uniform; skipped once the running max settles
#pragma unroll
            for (int j = 0; j < 2 * NKB; ++j) {
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[j][e] *= alpha;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) wsum[e] *= alpha;
          }
          // ---- P.V on the tensor pipe, dims as rows ----
          // A = V codes (c - 8) in fp16: rows = 16 dims of a block, k = the
          // tile's tokens with k (2t, 2t+1, 8+2t, 9+2t) <-> tokens (t, t+4,
          // t+8, t+12); B = p * scale with column g = scale group g.
          // Lane (mg, mt4) reads dims [D/8 * mg, D/8 * (mg + 1)) of those four
          // token rows; block j pairs bytes 2j, 2j+1 of that run: low nibbles
          // -> fragment (j, low) = dims D/8 mg + 4j + {0, 2}, high nibbles ->
          // (j, high) = dims D/8 mg + 4j + {1, 3}.
#pragma unroll
          for (int ti = 0; ti < 2; ++ti) {

            const uint32_t pk = pack_half2(slo[ti], shi[ti]);   // (p_mg, p_mg+8)
            const uint32_t u0 = __shfl_sync(0xffffffffu, pk, 4 * mt4);        // (p_t, p_t+8)
            const uint32_t u1 = __shfl_sync(0xffffffffu, pk, 4 * mt4 + 16);   // (p_t+4, p_t+12)
            const uint32_t p04 = __byte_perm(u0, u1, 0x5410);
            const uint32_t p8c = __byte_perm(u0, u1, 0x7632);
            const uint32_t vsa = tb[ti] + tt[ti] * G * 32 + o_vs;
            const uint32_t vs04 = lds_u32(vsa);
            const uint32_t vs8c = lds_u32(vsa + 16);
            const __half2 b0h = __hmul2(*reinterpret_cast<const __half2*>(&p04), *reinterpret_cast<const __half2*>(&vs04));
            const __half2 b1h = __hmul2(*reinterpret_cast<const __half2*>(&p8c), *reinterpret_cast<const __half2*>(&vs8c));
            // No second page: p = 0 but the stale scale may be NaN, so zero B itself
            // (the V code halves are finite by construction).
            const bool live = ti == 0 || has2;
            const uint32_t b0 = live ? *reinterpret_cast<const uint32_t*>(&b0h) : 0u;
            const uint32_t b1 = live ? *reinterpret_cast<const uint32_t*>(&b1h) : 0u;
            const uint32_t vr = tb[ti] + tt[ti] * 16 * (D / 2) + o_v;
            uint32_t T0[2], T4[2], Y0[2], Y4[2];
            if constexpr (D == 128) {
              // rows t, t+4, t+8, t+12 share bit 1 with t (folded into o_v)
              const uint2 r0 = lds_v2(vr);
              const uint2 r4 = lds_v2(vr + 4 * 64);
              const uint2 r8 = lds_v2(vr + 8 * 64);
              const uint2 rc = lds_v2(vr + 12 * 64);
              T0[0] = r0.x; T0[1] = r0.y; T4[0] = r4.x; T4[1] = r4.y;
              Y0[0] = r8.x; Y0[1] = r8.y; Y4[0] = rc.x; Y4[1] = rc.y;
            } else {
              T0[0] = lds_u32(vr);
              T4[0] = lds_u32(vr + 4 * 32);
              Y0[0] = lds_u32(vr + 8 * 32);
              Y4[0] = lds_u32(vr + 12 * 32);
              T0[1] = T4[1] = Y0[1] = Y4[1] = 0u;
            }
#pragma unroll
            for (int j = 0; j < NKB; ++j) {
              const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;
              const uint32_t x = __byte_perm(T0[j >> 1], T4[j >> 1], sel);  // tokens t | t+4
              const uint32_t y = __byte_perm(Y0[j >> 1], Y4[j >> 1], sel);  // tokens t+8 | t+12
              const uint32_t x8 = x >> 8, y8 = y >> 8;
              uint32_t a[4];
              a[0] = lo_raw(x, kF16); a[1] = lo_raw(x8, kF16); a[2] = lo_raw(y, kF16); a[3] = lo_raw(y8, kF16);
              mma16816(acc[2 * j], a, b0, b1);
              a[0] = hi_raw(x, kF16); a[1] = hi_raw(x8, kF16); a[2] = hi_raw(y, kF16); a[3] = hi_raw(y8, kF16);
              mma16816(acc[2 * j + 1], a, b0, b1);
            }
            {  // column sums of B: A = all ones
              const uint32_t ones[4] = {0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u};
              mma16816(wsum, ones, b0, b1);
            }
          }
        }
        if (++since_flush == kFlushSteps) flush_offsets();
        }
        __syncwarp();
        ++c_seq;
        produce();
      }
    }
    if (failed || !more) break;
    ++sub;
    load_item(item, sub, mask, phys_lane, h, c_lo, win_start, ctx, more);
    }
    if (failed) break;

    // ---- finish the item -------------------------------------------------
#pragma unroll
    for (int mk = 16; mk >= 1; mk >>= 1) l += __shfl_xor_sync(0xffffffffu, l, mk);
    // Each writing lane owns DPW contiguous output dims starting at dbase.
    constexpr int DPW = INT4 ? D / 8 : 8;
    float ov[DPW];
    int dbase = 0;
    bool writer = false;
    if constexpr (!INT4) {
#pragma unroll
      for (int mk = C::LPR; mk < 32; mk <<= 1) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += __shfl_xor_sync(0xffffffffu, o[j], mk);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ov[j] = o[j];
      dbase = cl * 8;
      writer = r == 0;
    } else {
      // Lane (mg, 0) holds dims D/8 mg + [0, D/8): fragment (j, hl) row mg
      // is dim D/8 mg + 4j + hl, row mg + 8 is + 2; column = scale group.
      flush_offsets();
      const int grp = (D / 8) * mg / 64;
#pragma unroll
      for (int j = 0; j < NKB; ++j) {
#pragma unroll
        for (int hl = 0; hl < 2; ++hl) {
          const float f = hl ? 0.0625f : 1.f;  // high fragments hold 16x
          ov[4 * j + hl] = f * (grp ? acc[2 * j + hl][1] : acc[2 * j + hl][0]);
          ov[4 * j + 2 + hl] = f * (grp ? acc[2 * j + hl][3] : acc[2 * j + hl][2]);
        }
      }
      dbase = (D / 8) * mg;
      writer = mt4 == 0;
    }

    if (p.n_chunks == 1) {
      if (writer) {
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
        for (int e = 0; e < DPW; e += 8) {
          uint4 hv;
          __half2* h2 = reinterpret_cast<__half2*>(&hv);
#pragma unroll
          for (int k = 0; k < 4; ++k) h2[k] = __floats2half2_rn(ov[e + 2 * k] * inv, ov[e + 2 * k + 1] * inv);
          *reinterpret_cast<uint4*>(p.out + pair * D + dbase + e) = hv;
        }
      }
      continue;
    }
    if (writer) {
      float4* dst = reinterpret_cast<float4*>(p.po + item * D + dbase);
#pragma unroll
      for (int e = 0; e < DPW / 4; ++e) dst[e] = make_float4(ov[4 * e], ov[4 * e + 1], ov[4 * e + 2], ov[4 * e + 3]);
    }
    if (lane == 0) p.ml[item] = make_float2(m, l);
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(p.tickets + pair, 1) == p.n_chunks - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
    // ---- merge the row's partials in chunk order ----
    const int64_t base = pair * p.n_chunks;
    float M = -INFINITY;
    for (int c = lane; c < p.n_chunks; c += 32) M = fmaxf(M, __ldcg(&p.ml[base + c].x));
#pragma unroll
    for (int mk = 16; mk >= 1; mk >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, mk));
    constexpr int DPL = D / 32;  // dims per lane in the merge
    float macc[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) macc[j] = 0.f;
    float L = 0.f;
    if (M != -INFINITY) {
      for (int c = 0; c < p.n_chunks; ++c) {
        const float2 mlc = __ldcg(&p.ml[base + c]);
        const float w = exp2f(mlc.x - M);
        L = fmaf(w, mlc.y, L);
        const float* src = p.po + (base + c) * D + lane * DPL;
#pragma unroll
        for (int j = 0; j < DPL; ++j) macc[j] = fmaf(w, __ldcg(src + j), macc[j]);
      }
    }
    const float inv = (L > 0.f) ? 1.f / L : 0.f;
#pragma unroll
    for (int j = 0; j < DPL; j += 2) {
      *reinterpret_cast<__half2*>(p.out + pair * D + lane * DPL + j) =
          __floats2half2_rn(macc[j] * inv, macc[j + 1] * inv);
    }
    if (lane == 0) p.tickets[pair] = 0;
  }

  if (failed) {
    if (lane == 0 && err) atomicExch(err, 1);
    // Drain the copies this warp still has in flight before leaving.
    for (; c_seq < p_seq; ++c_seq) {
      const int s = static_cast<int>(c_seq % NS);
      uint32_t polls = 0;
      while (!mbar_try_wait(bar0 + 8 * s, (c_seq / NS) & 1u) && ++polls < kMaxPolls) {
      }
    }
  }
}

}  // namespace decode
}  // namespace memopt
