// decode_mq4.cuh — multi-query paged decode over INT4 pages.
//
// Work items as in decode_mq.cuh: (sequence, KV head, tile of query rows,
// chunk of pages), every page staged once for all rows of the tile.  The
// arithmetic is that of the one-row INT4 decode kernel, widened to 8 query
// rows per tile:
//
// * scores on mma.sync m16n8k32 s8 (exact int32): the query row is rounded to
//   16-bit integers q_int = rint(q / qsc) (qsc = absmax / 32639, per row) and
//   split exactly as q_int = 256 hi + lo with hi, lo in [-128, 127].  The A
//   operand rows are (row r, hi) for r < 8 and (row r - 8, lo) for r >= 8, so
//   a lane holds both halves of one query row; B is the K code words as the
//   signed bytes 16 (c - 8) (tokens as columns).  Each 32-dim k-block lies in
//   one scale group and accumulates into that group's sums; the K scales are
//   applied per token after the products.  Column c of a tile's 8-token
//   n-block is token (c >> 1) + 4 (c & 1), so lane (g, t) ends up holding the
//   scores of tokens t, t+4, t+8, t+12 — the pairing the P.V operand needs.
// * P.V transposed, O^T[dims x rows] += V^T[dims x tokens] . P^T, on mma.sync
//   m16n8k16 f16: the V code bytes enter as 1024 + c (low nibbles) and
//   1024 + 16 c (high nibbles) fp16 halves (one logic op per pair), each
//   m16 block of dims inside one scale group, B = p * (V scale of the token,
//   that group) with the query rows as columns; the common offsets are
//   removed every few steps from an mma-accumulated column sum of B.
//
// Page layout and the V-row half swap are those written by write_cache
// (int4.cuh): the swap makes the reads of rows t, t+4, t+8, t+12 by the four
// lanes of a dim group free of bank conflicts.
#pragma once
#include "common.cuh"
#include "decode_mq.cuh"
#include "int4_mma.cuh"

namespace memopt {
namespace decode_mq4 {

using decode_mq::Params;  // rows per tile: 8 (Params::tiles = ceil(rows / 8))

template <int D, int BS>
struct Cfg {
  static constexpr int G = D / 64;                          // scale groups
  static constexpr int PAGE_RAW = BS * D + 2 * BS * G * 2;  // one (block, head) page
  static constexpr int STAGE = (PAGE_RAW + 127) / 128 * 128;
  static constexpr int V_CODES = BS * D / 2;
  static constexpr int K_SCALE = BS * D;               // [BS][G] fp16
  static constexpr int V_SCALE = BS * D + BS * G * 2;  // per 16-token tile [G][16], permuted
  static constexpr int NW = 4;
  static constexpr int WARP_BUDGET = 12288;
  static constexpr int NS_RAW = WARP_BUDGET / STAGE;
  static constexpr int NS = NS_RAW > 8 ? 8 : (NS_RAW < 2 ? 2 : NS_RAW);
  static constexpr int MIN_BLOCKS = 4;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int SMEM = BAR_BYTES + NW * NS * STAGE;
  static_assert(NW * NS * 8 <= BAR_BYTES, "barrier area too small");
};

template <int D, int BS>
__global__ void __launch_bounds__(Cfg<D, BS>::NW * 32, Cfg<D, BS>::MIN_BLOCKS)
paged_decode_mq4_kernel(const __grid_constant__ Params p, int32_t* __restrict__ err) {
  using C = Cfg<D, BS>;
  using namespace int4mma;
  constexpr int NS = C::NS;
  constexpr int G = C::G;
  constexpr int HALVES = BS / 16;
  constexpr int NKB = D / 32;  // k-blocks of the score mma (two per scale group at D = 128)
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + wid * NS;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t st0 = smem_u32(smem + C::BAR_BYTES + wid * NS * C::STAGE);

  if (lane == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * C::NW;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * C::NW + wid;
  auto row_end = [&](int ctx, int qi) { return p.causal ? ctx - p.QL + qi + 1 : ctx; };

  auto load_item = [&](int64_t item, int sub, uint32_t& mask, int& phys_lane, int& kvh, int& c_lo, bool& more) {
    const int64_t grp = item / p.n_chunks;
    const int chunk = static_cast<int>(item - grp * p.n_chunks);
    const int tile = static_cast<int>(grp % p.tiles);
    const int64_t bk = grp / p.tiles;
    kvh = static_cast<int>(bk % p.KVH);
    const int b = static_cast<int>(bk / p.KVH);
    const int ctx = __ldg(p.ctx + b);
    const int r0 = tile * 8;
    const int r1 = min(r0 + 8, p.rows) - 1;
    const int e_lo = row_end(ctx, r0 / p.group);
    const int e_hi = row_end(ctx, r1 / p.group);
    const int w_lo = p.window < e_lo ? e_lo - p.window : 0;
    int p_hi = 0;
    if (e_hi > 0) p_hi = min((e_hi + BS - 1) / BS, p.MB);
    const int p_lo = w_lo / BS;
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


  // ---------------- producer cursor (warp-uniform) ----------------------
  int64_t p_item = first - nwarps;
  int p_sub = 0;
  bool p_more = false;
  uint32_t p_mask = 0;
  int p_phys = -1;
  int p_kvh = 0;
  uint32_t p_seq = 0;
  int p_st = 0;  // p_seq % NS, kept incrementally (NS need not be a power of two)
  bool p_done = false;

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
      int c_lo;
      load_item(p_item, p_sub, p_mask, p_phys, p_kvh, c_lo, p_more);
    }
    if (p_done) return;
    const int j = __ffs(p_mask) - 1;
    p_mask &= p_mask - 1;
    const int phys = __shfl_sync(0xffffffffu, p_phys, j);
    {
      // Warp-collective issue: one elected lane arms the stage and starts the
      // copy, with no divergent branch around it.
      const int st = p_st;
      const uint32_t bar = bar0 + 8 * st;
      const uint8_t* src = p.pages + (static_cast<int64_t>(phys) * p.KVH + p_kvh) * C::PAGE_RAW;
      asm volatile(
          "{\n\t.reg .pred pe;\n\t"
          "elect.sync _|pe, 0xffffffff;\n\t"
          "@pe fence.proxy.async.shared::cta;\n\t"
          "@pe mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t"
          "@pe cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%3], %1, [%0];\n\t"
          "}" ::"r"(bar), "r"(static_cast<uint32_t>(C::PAGE_RAW)), "r"(st0 + st * C::STAGE), "l"(src)
          : "memory");
    }
    ++p_seq;
    p_st = p_st + 1 == NS ? 0 : p_st + 1;
  };

  for (int s = 0; s < NS; ++s) produce();

  auto wait_stage = [&](int st, uint32_t parity) -> bool {
    uint32_t polls = 0;
    bool ready = mbar_try_wait(bar0 + 8 * st, parity);
    while (!__all_sync(0xffffffffu, ready) && ++polls < kMaxPolls) {
      if (!ready) ready = mbar_try_wait(bar0 + 8 * st, parity);
    }
    return __all_sync(0xffffffffu, ready);
  };

  // ---------------- consumer -------------------------------------------
  const int g8 = lane >> 2;  // score fragments: query row; P.V fragments: dim group
  const int t4 = lane & 3;   // score fragments: token pair (t4, t4 + 4); P.V: query-row pair
  const uint32_t kF16 = p.magic_f16;
  const uint32_t kS8 = p.magic_s8;
  // K code row of this lane's B column: token (g8 >> 1) + 4 (g8 & 1) (+ 8 for
  // the second n-block); its words 2 t4, 2 t4 + 1 of each scale group.
  const int k_tok = (g8 >> 1) + 4 * (g8 & 1);
  const uint32_t o_k = k_tok * (D / 2) + 8 * t4;
  // V rows t4, t4+4, t4+8, t4+12 (same bit 1 as t4: one half-swap for all),
  // bytes 4 g8 (+ 32 for the second scale group) of each.
  const uint32_t o_v = C::V_CODES + t4 * (D / 2) + (D == 128 ? ((4 * g8) ^ ((t4 & 2) ? 32 : 0)) : 4 * g8);
  // V scales of tokens (t4, t4 + 4) and (t4 + 8, t4 + 12): adjacent halves.
  const uint32_t o_vs = C::V_SCALE + 4 * t4;
  uint32_t c_seq = 0;
  int c_st = 0;          // c_seq % NS
  uint32_t c_ph = 0;     // (c_seq / NS) & 1
  bool failed = false;

  for (int64_t item = first; item < p.total_items && !failed; item += nwarps) {
    const int64_t grp = item / p.n_chunks;
    const int chunk = static_cast<int>(item - grp * p.n_chunks);
    const int tile = static_cast<int>(grp % p.tiles);
    const int64_t bk = grp / p.tiles;
    const int kvh = static_cast<int>(bk % p.KVH);
    const int b = static_cast<int>(bk / p.KVH);
    const int ctx = __ldg(p.ctx + b);

    // Query row g8 of the tile (score side): visible tokens [rlo, rhi).
    const int gr = tile * 8 + g8;
    const bool rvalid = gr < p.rows;
    const int qi = rvalid ? gr / p.group : 0;
    const int64_t rpair = (static_cast<int64_t>(b) * p.QL + qi) * p.H + kvh * p.group + (rvalid ? gr - qi * p.group : 0);
    const int rend = row_end(ctx, qi);
    const int rlo = p.window < rend ? rend - p.window : 0;
    const int rhi = rvalid ? rend : 0;

    // q_int = rint(q / qsc) split into (hi, lo) signed bytes; k-block kb
    // (group kb / 2 at D = 128) uses word w = 8 (kb >> 1) + 2 t4 + (kb & 1):
    // k 4t4 + j <-> dim 8w + 2j, k 16 + 4t4 + j <-> dim 8w + 2j + 1.
    uint32_t qa[NKB][4];
    float sfac;
    {
      const __half* qrow = p.q + rpair * D;
      float am = 0.f;
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) {
        const int w = 8 * (kb >> 1) + 2 * t4 + (kb & 1);
        const uint4 v = rvalid ? __ldg(reinterpret_cast<const uint4*>(qrow + 8 * w)) : make_uint4(0, 0, 0, 0);
        const __half2* h2 = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h2[e]);
          am = fmaxf(am, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
      const float qsc = am > 0.f ? am / 32639.f : 1.f;
      const float qinv = am > 0.f ? 32639.f / am : 1.f;
      sfac = qsc * 0.0625f * p.qscale;  // score = sum_g ks_g * (16 (c - 8) . q_int) * qsc / 16, log2 domain
#pragma unroll
      for (int kb = 0; kb < NKB; ++kb) {
        const int w = 8 * (kb >> 1) + 2 * t4 + (kb & 1);
        const uint4 v = rvalid ? __ldg(reinterpret_cast<const uint4*>(qrow + 8 * w)) : make_uint4(0, 0, 0, 0);
        const __half* hv = reinterpret_cast<const __half*>(&v);
        uint32_t hi_e = 0, lo_e = 0, hi_o = 0, lo_o = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int odd = 0; odd < 2; ++odd) {
            const int qv = __float2int_rn(__half2float(hv[2 * j + odd]) * qinv);
            const int lo = ((qv + 128) & 255) - 128;
            const int hi = (qv - lo) >> 8;
            const uint32_t hb = (static_cast<uint32_t>(hi) & 0xFFu) << (8 * j);
            const uint32_t lb = (static_cast<uint32_t>(lo) & 0xFFu) << (8 * j);
            if (odd) {
              hi_o |= hb;
              lo_o |= lb;
            } else {
              hi_e |= hb;
              lo_e |= lb;
            }
          }
        }
        qa[kb][0] = hi_e;
        qa[kb][1] = lo_e;
        qa[kb][2] = hi_o;
        qa[kb][3] = lo_o;
      }
    }

    float m = -INFINITY, l = 0.f;  // row g8 (lanes of a quad agree on m; l is lane-partial)
    // O^T accumulators [group][byte pair][low, high nibble]: rows = dims
    // 8 g8 + 64 h + 4 bp + hl (+ 2 for fragment row g8 + 8), columns = query
    // rows 2 t4, 2 t4 + 1 of the tile.
    float acc[G][2][2][4];
    float wsum[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        wsum[h][e] = 0.f;
        acc[h][0][0][e] = acc[h][0][1][e] = acc[h][1][0][e] = acc[h][1][1][e] = 0.f;
      }
    }
    int since_flush = 0;
    constexpr int kFlushSteps = 4;
    auto flush_offsets = [&]() {
#pragma unroll
      for (int h = 0; h < G; ++h) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
#pragma unroll
          for (int bp = 0; bp < 2; ++bp) {
            acc[h][bp][0][e] = fmaf(-1032.f, wsum[h][e], acc[h][bp][0][e]);
            acc[h][bp][1][e] = fmaf(-1152.f, wsum[h][e], acc[h][bp][1][e]);
          }
          wsum[h][e] = 0.f;
        }
      }
      since_flush = 0;
    };

    uint32_t mask;
    int phys_lane, kvh_i, c_lo;
    bool more;
    int sub = 0;
    load_item(item, 0, mask, phys_lane, kvh_i, c_lo, more);
    for (;;) {
      while (mask != 0) {
        // One softmax step covers two 16-token tiles: both halves of a
        // 32-token page, or two 16-token pages of the sub-window.  Without a
        // second page the second tile is computed on the stage's stale bytes
        // and masked (scores -inf, P.V operand zero): a branch would keep the
        // two tiles' chains from interleaving.
        const int ja = __ffs(mask) - 1;
        mask &= mask - 1;
        int jb = -1;
        if (HALVES == 1 && mask != 0) {
          jb = __ffs(mask) - 1;
          mask &= mask - 1;
        }
        const int nst = (HALVES == 1 && jb >= 0) ? 2 : 1;  // ring stages this step
        const int c_st1 = c_st + 1 == NS ? 0 : c_st + 1;  // stage of c_seq + 1
        const uint32_t c_ph1 = c_st1 == 0 ? c_ph ^ 1u : c_ph;
        if (!wait_stage(c_st, c_ph) || (nst == 2 && !wait_stage(c_st1, c_ph1))) {
          failed = true;
          break;
        }
        const bool has_b = HALVES == 2 || jb >= 0;
        uint32_t tstg[2];
        int thalf[2], ttok[2];
        tstg[0] = st0 + static_cast<uint32_t>(c_st) * C::STAGE;
        thalf[0] = 0;
        ttok[0] = (c_lo + ja) * BS;
        if (HALVES == 2) {
          tstg[1] = tstg[0];
          thalf[1] = 1;
          ttok[1] = ttok[0] + 16;
        } else {
          tstg[1] = st0 + static_cast<uint32_t>(c_st1) * C::STAGE;
          thalf[1] = 0;
          ttok[1] = (c_lo + (jb >= 0 ? jb : ja)) * BS;
        }
        // ---- scores: exact integer products, both tiles ----
        int sacc[2][G][2][4];
#pragma unroll
        for (int ti = 0; ti < 2; ++ti) {
#pragma unroll
          for (int h = 0; h < G; ++h) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              sacc[ti][h][nt][0] = sacc[ti][h][nt][1] = sacc[ti][h][nt][2] = sacc[ti][h][nt][3] = 0;
              const uint2 w2 = lds_v2(tstg[ti] + (thalf[ti] * 16 + nt * 8) * (D / 2) + o_k + 32 * h);
#pragma unroll
              for (int sb = 0; sb < 2; ++sb) {
                const uint32_t w = sb ? w2.y : w2.x;
                mma_s8(sacc[ti][h][nt], qa[2 * h + sb], s8x16_even(w, kS8), s8x16_odd(w, kS8));
              }
            }
          }
        }
        // Both tiles present and inside every valid row's visible range: no
        // per-score mask (rows past the group's end hold q = 0; their
        // finite scores feed only their own, never written, columns).
        const int t_lo = min(ttok[0], ttok[1]), t_hi = max(ttok[0], ttok[1]) + 16;
        const bool interior = __all_sync(0xffffffffu, has_b && (!rvalid || (t_lo >= rlo && t_hi <= rhi)));
        float s[2][2][2];
#pragma unroll
        for (int ti = 0; ti < 2; ++ti) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int pos = thalf[ti] * 16 + nt * 8 + t4 + 4 * e;
              float v;
              if constexpr (G == 2) {
                const uint32_t k2 = lds_u32(tstg[ti] + C::K_SCALE + pos * 4);
                const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(&k2));
                v = fmaf(kf.x, static_cast<float>(sacc[ti][0][nt][e] * 256 + sacc[ti][0][nt][e + 2]),
                         kf.y * static_cast<float>(sacc[ti][1][nt][e] * 256 + sacc[ti][1][nt][e + 2]));
              } else {
                v = lds_f16_as_f32(tstg[ti] + C::K_SCALE + pos * 2) *
                    static_cast<float>(sacc[ti][0][nt][e] * 256 + sacc[ti][0][nt][e + 2]);
              }
              v *= sfac;
              if (interior) {
                s[ti][nt][e] = v;
              } else {
                const int tok = ttok[ti] + nt * 8 + t4 + 4 * e;
                const bool vis = (ti == 0 || has_b) && tok >= rlo && tok < rhi;
                s[ti][nt][e] = vis ? v : -INFINITY;
              }
            }
          }
        }
        // ---- online softmax for row g8 (one quad per row) ----
        float mx = fmaxf(fmaxf(fmaxf(s[0][0][0], s[0][0][1]), fmaxf(s[0][1][0], s[0][1][1])),
                         fmaxf(fmaxf(s[1][0][0], s[1][0][1]), fmaxf(s[1][1][0], s[1][1][1])));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m, mx);
        const float msub = mn == -INFINITY ? 0.f : mn;
        // A row that has seen nothing yet has zero accumulators: no rescale.
        const float corr = m == -INFINITY ? 1.f : ex2_approx(m - msub);
        m = mn;
        float psum = 0.f;
#pragma unroll
        for (int ti = 0; ti < 2; ++ti) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              s[ti][nt][e] = ex2_approx(s[ti][nt][e] - msub);
              psum += s[ti][nt][e];
            }
          }
        }
        l = fmaf(l, corr, psum);
        // The O^T columns of this lane are query rows 2 t4 and 2 t4 + 1.
        const float c0 = __shfl_sync(0xffffffffu, corr, 8 * t4);
        const float c1 = __shfl_sync(0xffffffffu, corr, 8 * t4 + 4);
        if (__any_sync(0xffffffffu, c0 != 1.f || c1 != 1.f)) {
#pragma unroll
          for (int h = 0; h < G; ++h) {
#pragma unroll
            for (int bp = 0; bp < 2; ++bp) {
#pragma unroll
              for (int hl = 0; hl < 2; ++hl) {
                acc[h][bp][hl][0] *= c0;
                acc[h][bp][hl][1] *= c1;
                acc[h][bp][hl][2] *= c0;
                acc[h][bp][hl][3] *= c1;
              }
            }
            wsum[h][0] *= c0;
            wsum[h][1] *= c1;
            wsum[h][2] *= c0;
            wsum[h][3] *= c1;
          }
        }
        // ---- P.V transposed: A = V codes (dims x tokens), B = p * V scale ----
#pragma unroll
        for (int ti = 0; ti < 2; ++ti) {
          const bool live = ti == 0 || has_b;
          const uint32_t p04 = pack_half2(s[ti][0][0], s[ti][0][1]);  // tokens (t4, t4 + 4)
          const uint32_t p8c = pack_half2(s[ti][1][0], s[ti][1][1]);  // tokens (t4 + 8, t4 + 12)
          const uint32_t vr = tstg[ti] + thalf[ti] * 16 * (D / 2) + o_v;
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const uint32_t vsa = tstg[ti] + o_vs + (thalf[ti] * G + h) * 32;
            const uint32_t vs04 = lds_u32(vsa);
            const uint32_t vs8c = lds_u32(vsa + 16);
            const __half2 b0h = __hmul2(*reinterpret_cast<const __half2*>(&p04), *reinterpret_cast<const __half2*>(&vs04));
            const __half2 b1h = __hmul2(*reinterpret_cast<const __half2*>(&p8c), *reinterpret_cast<const __half2*>(&vs8c));
            // A stale scale may be NaN: zero the operand of a missing tile.
            const uint32_t b0 = live ? *reinterpret_cast<const uint32_t*>(&b0h) : 0u;
            const uint32_t b1 = live ? *reinterpret_cast<const uint32_t*>(&b1h) : 0u;
            // Group h's 4 bytes of rows t4, t4+4, t4+8, t4+12 (the half swap
            // moves the second group's bytes by -32 on swapped rows).
            const uint32_t ho = (D == 128 && h == 1) ? ((t4 & 2) ? 0u - 32u : 32u) : 0u;
            const uint32_t T0 = lds_u32(vr + ho);
            const uint32_t T4 = lds_u32(vr + ho + 4 * (D / 2));
            const uint32_t Y0 = lds_u32(vr + ho + 8 * (D / 2));
            const uint32_t Y4 = lds_u32(vr + ho + 12 * (D / 2));
#pragma unroll
            for (int bp = 0; bp < 2; ++bp) {
              const uint32_t sel = bp ? 0x7632u : 0x5410u;
              const uint32_t x = __byte_perm(T0, T4, sel);  // bytes 2bp, 2bp+1 of tokens t4 | t4+4
              const uint32_t y = __byte_perm(Y0, Y4, sel);  // tokens t4+8 | t4+12
              const uint32_t x8 = x >> 8, y8 = y >> 8;
              uint32_t a[4];
              a[0] = lo_raw(x, kF16); a[1] = lo_raw(x8, kF16); a[2] = lo_raw(y, kF16); a[3] = lo_raw(y8, kF16);
              mma16816(acc[h][bp][0], a, b0, b1);
              a[0] = hi_raw(x, kF16); a[1] = hi_raw(x8, kF16); a[2] = hi_raw(y, kF16); a[3] = hi_raw(y8, kF16);
              mma16816(acc[h][bp][1], a, b0, b1);
            }
            const uint32_t ones[4] = {0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u};
            mma16816(wsum[h], ones, b0, b1);
          }
        }
        if (++since_flush == kFlushSteps) flush_offsets();
        __syncwarp();
        for (int k = 0; k < nst; ++k) {
          ++c_seq;
          if (++c_st == NS) {
            c_st = 0;
            c_ph ^= 1u;
          }
          produce();
        }
      }
      if (failed || !more) break;
      ++sub;
      load_item(item, sub, mask, phys_lane, kvh_i, c_lo, more);
    }
    if (failed) break;

    // ---- finish the item -------------------------------------------------
    flush_offsets();
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    // This lane writes query rows 2 t4 + cr (cr = 0, 1) of the tile, dims
    // 8 g8 + 64 h + [0, 8); their m and l live in quad 2 t4 + cr.
    float rl[2], rm[2];
    rl[0] = __shfl_sync(0xffffffffu, l, 8 * t4);
    rl[1] = __shfl_sync(0xffffffffu, l, 8 * t4 + 4);
    rm[0] = __shfl_sync(0xffffffffu, m, 8 * t4);
    rm[1] = __shfl_sync(0xffffffffu, m, 8 * t4 + 4);
    int64_t opair[2];
    bool ovalid[2];
#pragma unroll
    for (int cr = 0; cr < 2; ++cr) {
      const int orow = tile * 8 + 2 * t4 + cr;
      ovalid[cr] = orow < p.rows;
      const int oqi = ovalid[cr] ? orow / p.group : 0;
      opair[cr] = (static_cast<int64_t>(b) * p.QL + oqi) * p.H + kvh * p.group + (ovalid[cr] ? orow - oqi * p.group : 0);
    }
    auto dims8 = [&](int h, int cr, float v[8]) {
#pragma unroll
      for (int bp = 0; bp < 2; ++bp) {
        v[4 * bp + 0] = acc[h][bp][0][cr];
        v[4 * bp + 1] = acc[h][bp][1][cr] * 0.0625f;
        v[4 * bp + 2] = acc[h][bp][0][cr + 2];
        v[4 * bp + 3] = acc[h][bp][1][cr + 2] * 0.0625f;
      }
    };
    if (p.n_chunks == 1) {
#pragma unroll
      for (int cr = 0; cr < 2; ++cr) {
        if (!ovalid[cr]) continue;
        const float inv = rl[cr] > 0.f ? 1.f / rl[cr] : 0.f;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float v[8];
          dims8(h, cr, v);
          uint4 hv;
          __half2* h2 = reinterpret_cast<__half2*>(&hv);
#pragma unroll
          for (int k = 0; k < 4; ++k) h2[k] = __floats2half2_rn(v[2 * k] * inv, v[2 * k + 1] * inv);
          *reinterpret_cast<uint4*>(p.out + opair[cr] * D + 8 * g8 + 64 * h) = hv;
        }
      }
      continue;
    }
#pragma unroll
    for (int cr = 0; cr < 2; ++cr) {
      if (!ovalid[cr]) continue;
      const int64_t slot = opair[cr] * p.n_chunks + chunk;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float v[8];
        dims8(h, cr, v);
        float4* dst = reinterpret_cast<float4*>(p.po + slot * D + 8 * g8 + 64 * h);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
      if (g8 == 0) p.ml[slot] = make_float2(rm[cr], rl[cr]);
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(p.tickets + grp, 1) == p.n_chunks - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
    // ---- merge each row of the tile in chunk order ----
    const int nrows = min(8, p.rows - tile * 8);
    constexpr int DPL = D / 32;
    for (int rr = 0; rr < nrows; ++rr) {
      const int orow = tile * 8 + rr;
      const int oqi = orow / p.group;
      const int64_t pair = (static_cast<int64_t>(b) * p.QL + oqi) * p.H + kvh * p.group + (orow - oqi * p.group);
      const int64_t base = pair * p.n_chunks;
      float M = -INFINITY;
      for (int c = lane; c < p.n_chunks; c += 32) M = fmaxf(M, __ldcg(&p.ml[base + c].x));
#pragma unroll
      for (int mk = 16; mk >= 1; mk >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, mk));
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
      for (int j = 0; j < DPL; j += 2)
        *reinterpret_cast<__half2*>(p.out + pair * D + lane * DPL + j) =
            __floats2half2_rn(macc[j] * inv, macc[j + 1] * inv);
    }
    if (lane == 0) p.tickets[grp] = 0;
  }

  if (failed) {
    if (lane == 0 && err) atomicExch(err, 1);
    for (; c_seq < p_seq; ++c_seq) {
      const int s = static_cast<int>(c_seq % NS);
      uint32_t polls = 0;
      while (!mbar_try_wait(bar0 + 8 * s, (c_seq / NS) & 1u) && ++polls < kMaxPolls) {
      }
    }
  }
}

}  // namespace decode_mq4
}  // namespace memopt
