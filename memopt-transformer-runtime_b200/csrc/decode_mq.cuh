// decode_mq.cuh — multi-query paged decode: the query rows that read the same
// KV head share every page load.
//
// The rows of one (sequence, KV head) are the group's query heads (grouped-
// query attention: H / KVH of them) times the q_len query positions.  The
// one-row-per-item decode kernel streams each page once per row, so with
// 4 query heads per KV head it moves 4x the pool's bytes through the SMs.
// Here a work item is (sequence, KV head, tile of <= 16 of those rows, chunk
// of pages): the page is staged once and both products run on the tensor
// pipe with the rows as the M dimension of mma.sync m16n8k16 (fp16 inputs,
// fp32 accumulators):
//   S[16 rows x 16 tokens] = Q[16 x D] . K^T     (D/16 k-steps x 2 n-tiles)
//   O[16 rows x D]        += P[16 x 16] . V      (D/8 n-tiles, one k-step)
// P goes from the S accumulators to the A operand in registers (the C and A
// fragment layouts coincide), so no shared-memory round trip.
//
// Staging: a ring of 16-token stages per warp (a 32-token page is two
// stages), filled by the TMA engine from the fp16 pool through tensor maps
// with 64-dim boxes and 128-byte swizzle, so the ldmatrix reads of K (as the
// B operand) and V (transposed, as the B operand) are free of bank
// conflicts.  Items are taken grid-strided by warps; softmax runs in the
// log2 domain on the fp32 scores (q is not pre-scaled: the fp16 query is
// used exactly); split-K partials per row merge in chunk order as in the
// one-row kernel, so the result is deterministic.
//
// Semantics are those of the one-row kernel: tokens [max(0, c - W), c) of
// valid pages, c = ctx (or ctx - q_len + i + 1 for causal row i), rows with
// no visible token produce 0.
#pragma once
#include "common.cuh"
#include "int4_mma.cuh"

namespace memopt {
namespace decode_mq {

struct Params {
  const __half* q;     // [B, QL, H, D]
  __half* out;         // [B, QL, H, D]
  const int32_t* bt;   // [B, MB]
  const int32_t* ctx;  // [B]
  const uint8_t* pages;  // INT4 pool [NB, KVH, page bytes] (decode_mq4.cuh)
  int32_t* tickets;    // [B * KVH * tiles]
  float2* ml;          // [B * QL * H * n_chunks]  (per query row, as the one-row kernel)
  float* po;           // [B * QL * H * n_chunks * D]
  int B, QL, H, KVH, group, MB, causal;
  int64_t NB;
  int window;          // clamped
  float qscale;        // log2(e) / sqrt(D)
  uint32_t magic_f16;  // INT4 conversion constants kept in registers (0x64006400, 0x80808080)
  uint32_t magic_s8;
  int rows;            // group * QL query rows per (sequence, KV head)
  int tiles;           // ceil(rows / rows per tile)
  int chunk_pages;
  int n_chunks;
  int64_t total_items;
};

template <int D>
struct Cfg {
  static constexpr int REG = 16 * 128;          // one 64-dim region of 16 tokens (128-byte rows)
  static constexpr int NREG = D / 64;           // regions per K (and per V) stage half
  static constexpr int STAGE = 2 * NREG * REG;  // K regions then V regions
  static constexpr int NW = 4;                  // warps per CTA
  static constexpr int WARP_BUDGET = 24576;
  static constexpr int NS_RAW = WARP_BUDGET / STAGE;
  static constexpr int NS = NS_RAW > 8 ? 8 : NS_RAW;
  static constexpr int MIN_BLOCKS = 2;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int SMEM = BAR_BYTES + NW * NS * STAGE;
  static_assert(NS >= 2, "ring too shallow");
  static_assert(NW * NS * 8 <= BAR_BYTES, "barrier area too small");
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

template <int D, int BS>
__global__ void __launch_bounds__(Cfg<D>::NW * 32, Cfg<D>::MIN_BLOCKS)
paged_decode_mq_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, int32_t* __restrict__ err) {
  using C = Cfg<D>;
  constexpr int NS = C::NS;
  constexpr int HALVES = BS / 16;  // 16-token stages per page
  constexpr int KK = D / 16;       // k-steps of Q.K^T
  constexpr int NT = D / 8;        // n-tiles of P.V
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + wid * NS;
  const uint32_t bar0 = smem_u32(bars);
  const uint32_t st0 = smem_u32(smem + C::BAR_BYTES + wid * NS * C::STAGE);

  if (lane == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  __syncwarp();

  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * C::NW;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * C::NW + wid;

  // Context end of query position qi (causal rows end at their own token).
  auto row_end = [&](int ctx, int qi) { return p.causal ? ctx - p.QL + qi + 1 : ctx; };

  // Decodes an item and ballots the valid pages of 32-page sub-window `sub`.
  auto load_item = [&](int64_t item, int sub, uint32_t& mask, int& phys_lane, int& kvh, int& c_lo, bool& more) {
    const int64_t grp = item / p.n_chunks;
    const int chunk = static_cast<int>(item - grp * p.n_chunks);
    const int tile = static_cast<int>(grp % p.tiles);
    const int64_t bk = grp / p.tiles;
    kvh = static_cast<int>(bk % p.KVH);
    const int b = static_cast<int>(bk / p.KVH);
    const int ctx = __ldg(p.ctx + b);
    const int r0 = tile * 16;
    const int r1 = min(r0 + 16, p.rows) - 1;
    const int e_lo = row_end(ctx, r0 / p.group);  // earliest query position of the tile
    const int e_hi = row_end(ctx, r1 / p.group);  // latest
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

  // One 16-token stage: K then V, each as D/64 swizzled 64-dim boxes.
  auto issue = [&](uint32_t seq, int phys, int half, int kvh) {
    const int s = static_cast<int>(seq % NS);
    const uint32_t bar = bar0 + 8 * s;
    const uint32_t dst = st0 + s * C::STAGE;
    const int row = phys * BS + half * 16;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, C::STAGE);
#pragma unroll
    for (int g = 0; g < C::NREG; ++g) {
      tma_load_3d(dst + g * C::REG, &kmap, 64 * g, kvh, row, bar);
      tma_load_3d(dst + (C::NREG + g) * C::REG, &vmap, 64 * g, kvh, row, bar);
    }
  };

  // ---------------- producer cursor (warp-uniform) ----------------------
  int64_t p_item = first - nwarps;
  int p_sub = 0, p_half = HALVES;  // p_half == HALVES: take the next page
  bool p_more = false;
  uint32_t p_mask = 0;
  int p_phys = -1, p_page = -1;
  int p_kvh = 0;
  uint32_t p_seq = 0;
  bool p_done = false;

  auto produce = [&]() {
    if (p_done) return;
    if (p_half == HALVES) {
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
      p_page = __shfl_sync(0xffffffffu, p_phys, j);
      p_half = 0;
    }
    if (lane == 0) issue(p_seq, p_page, p_half, p_kvh);
    ++p_half;
    ++p_seq;
  };

  for (int s = 0; s < NS; ++s) produce();

  // ---------------- consumer -------------------------------------------
  const int g8 = lane >> 2;  // fragment row (and row + 8)
  const int t4 = lane & 3;   // fragment column pair
  // ldmatrix lane roles: matrix lane >> 3, row lane & 7.
  const int lm = lane >> 3, lr = lane & 7;
  // K (non-transposed): matrices (tokens 0-7 | 8-15) x (dims +0 | +8).
  const int k_tok = (lm >> 1) * 8 + lr, k_dhalf = lm & 1;
  // V (transposed): matrices (tokens 0-7 | 8-15) x (dims +0 | +8) in the order b0, b1 of
  // n-tile 2nn then of 2nn + 1.
  const int v_tok = (lm & 1) * 8 + lr, v_dhalf = lm >> 1;
  uint32_t c_seq = 0;
  bool failed = false;

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

  for (int64_t item = first; item < p.total_items && !failed; item += nwarps) {
    const int64_t grp = item / p.n_chunks;
    const int chunk = static_cast<int>(item - grp * p.n_chunks);
    const int tile = static_cast<int>(grp % p.tiles);
    const int64_t bk = grp / p.tiles;
    const int kvh = static_cast<int>(bk % p.KVH);
    const int b = static_cast<int>(bk / p.KVH);
    const int ctx = __ldg(p.ctx + b);

    // This lane's two fragment rows (g8, g8 + 8): visible tokens [rlo, rhi).
    int rlo[2], rhi[2];
    int64_t rpair[2];
    bool rvalid[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int gr = tile * 16 + g8 + 8 * hr;
      rvalid[hr] = gr < p.rows;
      const int qi = rvalid[hr] ? gr / p.group : 0;
      const int j = rvalid[hr] ? gr - qi * p.group : 0;
      rpair[hr] = (static_cast<int64_t>(b) * p.QL + qi) * p.H + kvh * p.group + j;
      const int e = row_end(ctx, qi);
      rlo[hr] = p.window < e ? e - p.window : 0;
      rhi[hr] = rvalid[hr] ? e : 0;
    }
    // Q as the A operand: a0/a2 row g8 (dims +2t4, +2t4+8), a1/a3 row g8 + 8.
    uint32_t qa[KK][4];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const __half* qrow = p.q + rpair[hr] * D + 2 * t4;
#pragma unroll
      for (int kk = 0; kk < KK; ++kk) {
        qa[kk][hr] = rvalid[hr] ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * kk)) : 0u;
        qa[kk][2 + hr] = rvalid[hr] ? __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 8)) : 0u;
      }
    }
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;

    uint32_t mask;
    int phys_lane, kvh_i, c_lo;
    bool more;
    int sub = 0;
    load_item(item, 0, mask, phys_lane, kvh_i, c_lo, more);
    for (;;) {
      while (mask != 0) {
        const int jpage = __ffs(mask) - 1;
        mask &= mask - 1;
        const int page = c_lo + jpage;
#pragma unroll 1
        for (int half = 0; half < HALVES; ++half) {
          if (!wait_stage(c_seq)) {
            failed = true;
            break;
          }
          const uint32_t stg = st0 + static_cast<uint32_t>(c_seq % NS) * C::STAGE;
          const int tok0 = page * BS + half * 16;
          // ---- S = Q K^T on the tensor pipe ----
          float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int kk = 0; kk < KK; ++kk) {
            const int ch = 2 * kk + k_dhalf;
            const uint32_t addr =
                stg + (ch >> 3) * C::REG + k_tok * 128 + (((ch & 7) ^ (k_tok & 7)) << 4);
            uint32_t b00, b01, b10, b11;
            ldsm_x4(addr, b00, b01, b10, b11);
            int4mma::mma16816(s[0], qa[kk], b00, b01);
            int4mma::mma16816(s[1], qa[kk], b10, b11);
          }
          // ---- scale, mask, online softmax (rows g8 and g8 + 8) ----
          const bool interior = tok0 >= rlo[0] && tok0 + 16 <= rhi[0] && tok0 >= rlo[1] && tok0 + 16 <= rhi[1];
          float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int hr = e >> 1;
              float x = s[nt][e] * p.qscale;
              if (!interior) {
                const int tok = tok0 + nt * 8 + 2 * t4 + (e & 1);
                if (tok < rlo[hr] || tok >= rhi[hr]) x = -INFINITY;
              }
              s[nt][e] = x;
              mx[hr] = fmaxf(mx[hr], x);
            }
          }
          float corr[2];
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
            mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
            const float mn = fmaxf(m[hr], mx[hr]);
            const float msub = mn == -INFINITY ? 0.f : mn;  // a row with nothing visible yet
            // A row that has seen nothing yet has zero accumulators: no rescale.
            corr[hr] = m[hr] == -INFINITY ? 1.f : int4mma::ex2_approx(m[hr] - msub);
            m[hr] = mn;
            mx[hr] = msub;
          }
          float rs[2] = {0.f, 0.f};
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float pe = int4mma::ex2_approx(s[nt][e] - mx[e >> 1]);
              s[nt][e] = pe;
              rs[e >> 1] += pe;
            }
          }
          l[0] = fmaf(l[0], corr[0], rs[0]);
          l[1] = fmaf(l[1], corr[1], rs[1]);
          if (__any_sync(0xffffffffu, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              o[nt][0] *= corr[0];
              o[nt][1] *= corr[0];
              o[nt][2] *= corr[1];
              o[nt][3] *= corr[1];
            }
          }
          // P as the A operand: the S fragments of tokens 0-7 and 8-15.
          uint32_t pa[4];
          pa[0] = int4mma::pack_half2(s[0][0], s[0][1]);
          pa[1] = int4mma::pack_half2(s[0][2], s[0][3]);
          pa[2] = int4mma::pack_half2(s[1][0], s[1][1]);
          pa[3] = int4mma::pack_half2(s[1][2], s[1][3]);
          // ---- O += P V (V transposed out of shared memory) ----
#pragma unroll
          for (int nn = 0; nn < D / 16; ++nn) {
            const int ch = 2 * nn + v_dhalf;
            const uint32_t addr = stg + (C::NREG + (ch >> 3)) * C::REG + v_tok * 128 +
                                  (((ch & 7) ^ (v_tok & 7)) << 4);
            uint32_t v0, v1, v2, v3;
            ldsm_x4_t(addr, v0, v1, v2, v3);
            int4mma::mma16816(o[2 * nn], pa, v0, v1);
            int4mma::mma16816(o[2 * nn + 1], pa, v2, v3);
          }
          ++c_seq;
          __syncwarp();
          produce();
        }
        if (failed) break;
      }
      if (failed || !more) break;
      ++sub;
      load_item(item, sub, mask, phys_lane, kvh_i, c_lo, more);
    }
    if (failed) break;

    // ---- finish the item -------------------------------------------------
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 1);
      l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 2);
    }
    if (p.n_chunks == 1) {
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        if (!rvalid[hr]) continue;
        const float inv = l[hr] > 0.f ? 1.f / l[hr] : 0.f;
        __half* orow = p.out + rpair[hr] * D + 2 * t4;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          *reinterpret_cast<__half2*>(orow + 8 * nt) =
              __floats2half2_rn(o[nt][2 * hr] * inv, o[nt][2 * hr + 1] * inv);
      }
      continue;
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      if (!rvalid[hr]) continue;
      const int64_t slot = rpair[hr] * p.n_chunks + chunk;
      float* dst = p.po + slot * D + 2 * t4;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float2*>(dst + 8 * nt) = make_float2(o[nt][2 * hr], o[nt][2 * hr + 1]);
      if (t4 == 0) p.ml[slot] = make_float2(m[hr], l[hr]);
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(p.tickets + grp, 1) == p.n_chunks - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
    // ---- merge each row of the tile in chunk order ----
    const int nrows = min(16, p.rows - tile * 16);
    constexpr int DPL = D / 32;
    for (int rr = 0; rr < nrows; ++rr) {
      const int gr = tile * 16 + rr;
      const int qi = gr / p.group;
      const int64_t pair = (static_cast<int64_t>(b) * p.QL + qi) * p.H + kvh * p.group + (gr - qi * p.group);
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

}  // namespace decode_mq
}  // namespace memopt
