// prefill.cu — multi-query / prefill path of dynamic_sparse_attention on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Semantics are those of attention.cu:98-339 (reference): every query row of
// sequence b sees the tokens [max(0, ctx_b - W), ctx_b) of the pages whose
// block-table entry is >= 0 (and < num_blocks here), with no causal mask, so
// all rows of a sequence share one key set and the work is a dense
// non-causal attention per (sequence, head).
//
// One CTA = (two 128-query tiles, head, sequence); keys are consumed in blocks
// of 64 tokens (64/BS pages) shared by both tiles.
//   * warps 9 and 10 stage Q once and K/V blocks by TMA (3-D tensor maps over
//     the query tensor and the fp16 pool, 128-byte swizzle, no multicast) into
//     rings of 3 K and 2 V stages;
//   * warp 8 issues the tcgen05.mma instructions (warp-uniform code, one lane
//     elected per instruction): per tile, S(j) = Q K(j)^T (M=128, N=64, K=D)
//     into one of two TMEM score buffers and O += P(j) V(j) (M=128, N=D,
//     K=64) with P read from tensor memory (the A operand) and V the MN-major
//     operand from shared memory;
//   * warps 0-3 (tile 0) and 4-7 (tile 1) run the softmax, one thread per
//     query row (= TMEM lane): it loads its 64 scores with tcgen05.ld,
//     releases the score buffer, runs the online softmax in the log2 domain,
//     writes P (fp16 pairs) over the first 32 columns of the same score
//     buffer with tcgen05.st and rescales its O row in TMEM only when its
//     running max grows by more than 2^8 (stale maxima below that bound keep
//     P <= 256, exact enough in fp16).
// With two score buffers per tile, S(j+2) and P.V(j) run on the tensor pipe
// while the softmax works on block j+1; S(j+2) overwrites P(j) only after
// P.V(j), issued before it by the same thread (tcgen05.mma instructions of
// one thread execute in order).  The two tiles' softmax warps share every SM
// sub-partition, tile 1 running about half a block behind tile 0 (it starts
// after P(0) of tile 0); no CTA-wide barrier is taken per block.  The
// epilogue divides O by the row sum and stores fp16.  Pages that are skipped
// (entry < 0 or >= num_blocks) are zero-filled in smem and masked; every
// mbarrier wait is bounded and reports through `err`.
#include <cmath>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "int4.cuh"
#include "tc.cuh"

namespace memopt {
namespace prefill {

struct Params {
  const int32_t* bt;
  const int32_t* ctx;
  __half* out;
  int B, QL, H, MB;
  int64_t NB;
  int window;
  float qscale;  // log2(e) / sqrt(D)
  int group;     // query heads per KV head (the pool has H / group heads)
  int causal;    // 1: query row i of QL is the token at ctx - QL + i (extension)
};

constexpr int kBN = 64;                // key tokens per block
constexpr int kTiles = 2;              // 128-row query tiles per CTA
constexpr int kRows = 128 * kTiles;    // query rows per CTA
constexpr int kBtCache = 1024;         // block-table entries cached in smem per CTA
constexpr int kNSK = 3, kNSV = 2;      // K and V ring depths
constexpr int kSoftmaxWarps = 4 * kTiles;
constexpr int kMmaWarp = kSoftmaxWarps, kLoadKWarp = kSoftmaxWarps + 1, kLoadVWarp = kSoftmaxWarps + 2;
constexpr int kThreads = 32 * (kSoftmaxWarps + 3);  // + MMA warp + K and V load warps

template <int D, int BS>
struct Cfg {
  static constexpr int HALVES = D / 64;
  static constexpr int PPB = kBN / BS;                 // pages per block
  static constexpr int Q_HALF = 128 * 128;             // 128 rows x 128 B
  static constexpr int KV_HALF = kBN * 128;            // 64 rows x 128 B
  static constexpr int Q_TILE = HALVES * Q_HALF;
  static constexpr int KV_STAGE = HALVES * KV_HALF;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + kTiles * Q_TILE;
  static constexpr int V_OFF = K_OFF + kNSK * KV_STAGE;
  static constexpr int BT_OFF = V_OFF + kNSV * KV_STAGE;
  static constexpr int SMEM = BT_OFF + 4 * kBtCache + 1024;  // + alignment slack
  static constexpr uint32_t PAGE_TX = 1u * HALVES * BS * 128u;  // bytes of one page of K (or V)
  static constexpr uint32_t IDESC_S = tc::idesc_f16(128, kBN, false, false);
  static constexpr uint32_t IDESC_PV = tc::idesc_f16(128, D, false, true);
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(kTiles * (2 * kBN + D) <= 512, "tensor memory columns");
};

#ifndef MEMOPT_PF_HINT_NS
#define MEMOPT_PF_HINT_NS 1000
#endif
// Bounded wait: at most 2^21 polls of at most MEMOPT_PF_HINT_NS each (about
// two seconds), then the caller records a failure.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity) {
  uint32_t polls = 0;
  while (!mbar_try_wait_hint(bar, parity, MEMOPT_PF_HINT_NS)) {
    if (++polls >= (1u << 21)) return false;
  }
  return true;
}

// Barriers (index: role):
//   0 Q staged (tx) | 1..3 K stage full (tx) | 4..5 V stage full (tx)
//   6..8 K stage free (commit after both tiles' S) | 9..10 V stage free
//   (commit after both tiles' P.V) | per tile t at 11 + 8t: +0..1 S buffer
//   full (commit), +2..3 S buffer read (4 softmax warps), +4..5 P buffer full
//   (4 softmax warps), +6..7 P.V done, P buffer free (commit).
// Block j uses K stage j % 3, V stage j % 2, S and P buffers j % 2; a waiter
// never lags a barrier by two phases (each next phase needs an action of the
// waiter itself first).
constexpr int kBars = 11 + 8 * kTiles;

#ifdef MEMOPT_PF_TRACE
__device__ unsigned long long g_pf_trace[12][512];
#define PF_TRACE(ev, j)                                                                   \
  do {                                                                                    \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (j) < 512) g_pf_trace[ev][(j)] = clock64(); \
  } while (0)
#else
#define PF_TRACE(ev, j) \
  do {                  \
  } while (0)
#endif

template <int D, int BS>
__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap qmap,
               const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
               int32_t* __restrict__ err) {
  using C = Cfg<D, BS>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[kBars];
  __shared__ uint32_t tmem_slot;
  __shared__ int fail_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(base);
  auto bar_at = [&](int i) { return smem_u32(&bars[i]); };
  auto bar_kfull = [&](int j) { return bar_at(1 + j % kNSK); };
  auto bar_vfull = [&](int j) { return bar_at(4 + j % kNSV); };
  auto bar_kfree = [&](int j) { return bar_at(6 + j % kNSK); };
  auto bar_vfree = [&](int j) { return bar_at(9 + j % kNSV); };
  auto bar_sfull = [&](int t, int j) { return bar_at(11 + 8 * t + (j & 1)); };
  auto bar_sfree = [&](int t, int j) { return bar_at(13 + 8 * t + (j & 1)); };
  auto bar_pfull = [&](int t, int j) { return bar_at(15 + 8 * t + (j & 1)); };
  auto bar_pfree = [&](int t, int j) { return bar_at(17 + 8 * t + (j & 1)); };
  auto ph_k = [](int j) { return static_cast<uint32_t>((j / kNSK) & 1); };
  auto ph_v = [](int j) { return static_cast<uint32_t>((j / kNSV) & 1); };
  auto ph_2 = [](int j) { return static_cast<uint32_t>((j >> 1) & 1); };

  const int hk = h / p.group;  // KV head of this query head
  const int ctx_seq = __ldg(p.ctx + b);
  // Visible tokens of query row qi: [ws_i, ctx_i), ctx_i = ctx (non-causal)
  // or ctx - QL + qi + 1 (causal), ws_i = max(0, ctx_i - window).  The CTA
  // stages the union over its rows; each softmax thread masks with its own.
  auto row_ctx = [&](int qi) { return p.causal ? ctx_seq - p.QL + qi + 1 : ctx_seq; };
  auto row_ws = [&](int c) { return (p.window < c) ? (c - p.window) : 0; };
  const int ctx = row_ctx(min(qt * kRows + kRows - 1, p.QL - 1));
  const int ws = row_ws(row_ctx(qt * kRows));
  const int p_hi = ctx > 0 ? min((ctx + BS - 1) / BS, p.MB) : 0;
  const int p_lo = ws / BS;
  const int nblocks = p_hi > p_lo ? (p_hi - p_lo + C::PPB - 1) / C::PPB : 0;

  if (tid == 0) {
    for (int i = 0; i < 11; ++i) mbar_init(bar_at(i), 1);
    for (int t = 0; t < kTiles; ++t) {
      for (int i = 0; i < 2; ++i) mbar_init(bar_at(11 + 8 * t + i), 1);
      for (int i = 2; i < 6; ++i) mbar_init(bar_at(11 + 8 * t + i), 4);
      for (int i = 6; i < 8; ++i) mbar_init(bar_at(11 + 8 * t + i), 1);
    }
    fence_mbar_init();
    fail_flag = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&tmem_slot), 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  // Tile t: score buffers at columns 256 t + {0, 64}, O at 256 t + 128.
  auto tS = [&](int t, int j) { return tmem + 256u * t + (j & 1) * kBN; };
  auto tO = [&](int t) { return tmem + 256u * t + 128u; };

  // The pages of this sequence's window are read once into smem (when they
  // fit), so per-block validity checks rarely wait on global memory.
  int32_t* s_bt = reinterpret_cast<int32_t*>(base + C::BT_OFF);
  const int npages = p_hi > p_lo ? p_hi - p_lo : 0;
  const bool bt_cached = npages <= kBtCache;
  if (bt_cached) {
    for (int i = tid; i < npages; i += kThreads) s_bt[i] = __ldg(p.bt + static_cast<int64_t>(b) * p.MB + p_lo + i);
  }
  __syncthreads();

  // Validity of the pages of block j, one bit per page (warp-collective).
  auto page_bits = [&](int j, int& phys) -> uint32_t {
    const int page = p_lo + j * C::PPB + lane;
    phys = -1;
    if (lane < C::PPB && page < p_hi)
      phys = bt_cached ? s_bt[page - p_lo] : __ldg(p.bt + static_cast<int64_t>(b) * p.MB + page);
    const bool ok = lane < C::PPB && page < p_hi && phys >= 0 && static_cast<int64_t>(phys) < p.NB;
    return __ballot_sync(0xffffffffu, ok);
  };

  if (warp == kLoadKWarp || warp == kLoadVWarp) {
    // ======================= TMA load warps (K, V) =======================
    // K and V are staged by separate warps so that a K stage never waits
    // behind the release of a V stage (and the reverse).
    const bool is_v = warp == kLoadVWarp;
    if (lane == 0) {
      prefetch_tensormap(is_v ? &vmap : &kmap);
      if (!is_v) prefetch_tensormap(&qmap);
    }
    // Stage K or V of block j, zero-filling skipped pages.
    auto stage = [&](int j) {
      const uint32_t bar = is_v ? bar_vfull(j) : bar_kfull(j);
      const int off = is_v ? C::V_OFF + (j % kNSV) * C::KV_STAGE : C::K_OFF + (j % kNSK) * C::KV_STAGE;
      int phys;
      const uint32_t mask = page_bits(j, phys);
      const uint32_t bad = ~mask & ((1u << C::PPB) - 1u);
      if (bad != 0) {
        for (int pg = 0; pg < C::PPB; ++pg) {
          if (!((bad >> pg) & 1u)) continue;
          for (int hh = 0; hh < C::HALVES; ++hh) {
            uint4* dst = reinterpret_cast<uint4*>(base + off + hh * C::KV_HALF + pg * BS * 128);
            for (int c = lane; c < BS * 8; c += 32) dst[c] = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(bar, __popc(mask) * C::PAGE_TX);
      __syncwarp();  // the transaction count is armed before any copy can land
      if ((mask >> lane) & 1u) {
        for (int hh = 0; hh < C::HALVES; ++hh)
          tma_load_3d(sbase + off + hh * C::KV_HALF + lane * BS * 128, is_v ? &vmap : &kmap, hh * 64, hk,
                      phys * BS, bar);
      }
    };
    bool ok = true;
    if (!is_v && nblocks > 0 && lane == 0) {
      mbar_arrive_expect_tx(bar_at(0), kTiles * C::Q_TILE);
      for (int t = 0; t < kTiles; ++t)
        for (int hh = 0; hh < C::HALVES; ++hh)
          tma_load_3d(sbase + C::Q_OFF + t * C::Q_TILE + hh * C::Q_HALF, &qmap, hh * 64, h,
                      b * p.QL + qt * kRows + t * 128, bar_at(0));
    }
    const int depth = is_v ? kNSV : kNSK;
    for (int j = 0; j < nblocks && ok; ++j) {
      // The stage of block j is free once both tiles' S(j-3) (K) or
      // P.V(j-2) (V) completed.
      if (j >= depth && lane == 0)
        ok = is_v ? wait_bar(bar_vfree(j - kNSV), ph_v(j - kNSV)) : wait_bar(bar_kfree(j - kNSK), ph_k(j - kNSK));
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      stage(j);
      if (lane == 0) PF_TRACE(is_v ? 2 : 3, j);
    }
    if (!ok && lane == 0) fail_flag = 1;
  } else if (warp == kMmaWarp) {
    // ============================== MMA warp ==============================
    // The whole warp runs this loop (waits included) with warp-uniform
    // operands; elect.sync inside mma_f16_elect / commit_elect issues each
    // instruction once.  Descriptors are built once; a k-step or stage
    // advances the 14-bit start address field by (byte offset >> 4) (all
    // offsets stay below 256 KB).
    bool ok = true;
    if (nblocks > 0) {
      uint64_t dq[kTiles];
#pragma unroll
      for (int t = 0; t < kTiles; ++t) dq[t] = tc::sdesc_sw128(sbase + C::Q_OFF + t * C::Q_TILE, 16, 1024);
      const uint64_t dk0 = tc::sdesc_sw128(sbase + C::K_OFF, 16, 1024);
      const uint64_t dv0 = tc::sdesc_sw128(sbase + C::V_OFF, C::KV_HALF, 1024);
      auto issue_s = [&](int t, int j) {
        const uint64_t dk = dk0 + static_cast<uint64_t>(((j % kNSK) * C::KV_STAGE) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          tc::mma_f16_elect(tS(t, j), dq[t] + static_cast<uint64_t>(((kk / 4) * C::Q_HALF + (kk % 4) * 32) >> 4),
                            dk + static_cast<uint64_t>(((kk / 4) * C::KV_HALF + (kk % 4) * 32) >> 4), C::IDESC_S,
                            kk > 0);
        }
        tc::commit_elect(bar_sfull(t, j));
      };
      auto issue_pv = [&](int t, int j) {
        const uint64_t dv = dv0 + static_cast<uint64_t>(((j % kNSV) * C::KV_STAGE) >> 4);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // A = P from tensor memory: columns 8 kk .. 8 kk + 7 of the score
          // buffer hold tokens 16 kk .. 16 kk + 15 as fp16 pairs.
          tc::mma_f16_tmem_a_elect(tO(t), tS(t, j) + 8u * kk, dv + static_cast<uint64_t>((kk * 2048) >> 4),
                                   C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc::commit_elect(bar_pfree(t, j));
      };
      auto wait_all = [&](uint32_t bar, uint32_t parity) { return __all_sync(0xffffffffu, wait_bar(bar, parity)); };
      // S(j) of both tiles into score buffer j % 2, the K stage released after.
      auto issue_s_both = [&](int j) -> bool {
        if (!wait_all(bar_kfull(j), ph_k(j))) return false;
        for (int t = 0; t < kTiles; ++t) {
          if (j >= 2 && !wait_all(bar_sfree(t, j - 2), ph_2(j - 2))) return false;  // buffer read
          tc::fence_after_sync();
          issue_s(t, j);
        }
        tc::commit_elect(bar_kfree(j));
        if (lane == 0) PF_TRACE(1, j);
        return true;
      };
      ok = wait_all(bar_at(0), 0);
      if (ok) ok = issue_s_both(0);
      if (ok && nblocks > 1) ok = issue_s_both(1);
      for (int j = 0; j < nblocks && ok; ++j) {
        ok = wait_all(bar_vfull(j), ph_v(j));
        for (int t = 0; t < kTiles && ok; ++t) {
          ok = wait_all(bar_pfull(t, j), ph_2(j));
          if (ok) {
            tc::fence_after_sync();
            issue_pv(t, j);
          }
        }
        if (!ok) break;
        tc::commit_elect(bar_vfree(j));
        if (lane == 0) PF_TRACE(0, j);
        if (j + 2 < nblocks) ok = issue_s_both(j + 2);
      }
      if (!ok && lane == 0) fail_flag = 1;
    }
    __syncwarp();
  } else {
    // =========================== softmax warps ===========================
    const int t = warp >> 2;                 // query tile
    const int row = (warp & 3) * 32 + lane;  // row within the tile = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int ctx_r = row_ctx(qt * kRows + t * 128 + row);  // this row's visible tokens
    const int ws_r = row_ws(ctx_r);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nblocks && ok; ++j) {
      if (j == 0 && t == 1) {
        // Tile 1 starts once tile 0 has stored P(0).  The two tiles then keep
        // that offset (S(j + 2) of both follows both P(j)), so one tile's
        // exponentials run while the other loads scores, takes the row max
        // or waits; started together, they stay in step and the exponential
        // unit idles in those phases.
        ok = __all_sync(0xffffffffu, wait_bar(bar_pfull(0, 0), 0));
        if (!ok) break;
      }
      ok = wait_bar(bar_sfull(t, j), ph_2(j));
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (tid == 0) PF_TRACE(4, j);
      if (tid == 128) PF_TRACE(7, j);
      tc::fence_after_sync();
      float s[kBN];
      {
        float va[32], vb[32];
        tc::ld32(tS(t, j) + lane_base, va);
        tc::ld32(tS(t, j) + lane_base + 32, vb);
        tc::wait_ld(va);
        tc::wait_ld(vb);  // nothing left in flight: orders the uses of vb
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = va[i];
          s[32 + i] = vb[i];
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree(t, j));
      int phys_unused;
      const uint32_t mask = page_bits(j, phys_unused);
      const int tok0 = (p_lo + j * C::PPB) * BS;
      const bool edge = mask != ((1u << C::PPB) - 1u) || tok0 < ws_r || tok0 + kBN > ctx_r;
      if (edge) {
#pragma unroll
        for (int i = 0; i < kBN; ++i) {
          const int tk = tok0 + i;
          const bool valid = ((mask >> (i / BS)) & 1u) && tk >= ws_r && tk < ctx_r;
          s[i] = valid ? s[i] : -INFINITY;
        }
      }
      float mxp[8];  // eight independent partial maxima (short dependency chains)
#pragma unroll
      for (int k = 0; k < 8; ++k) mxp[k] = s[k];
#pragma unroll
      for (int i = 8; i < kBN; ++i) mxp[i & 7] = fmaxf(mxp[i & 7], s[i]);
      float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                       fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      mx *= p.qscale;  // qscale > 0: the max of the scaled scores
      if (tid == 0) PF_TRACE(10, j);
      if (tid == 128) PF_TRACE(11, j);
      const float m_new = fmaxf(m_run, mx);
      float m_use = m_run, alpha = 1.f;
      bool rescale = false;
      if (m_run == -INFINITY) {
        m_use = m_new;  // nothing accumulated yet (all earlier p were 0)
      } else if (m_new > m_run + 8.f) {
        m_use = m_new;
        alpha = tc::ex2(m_run - m_new);
        rescale = true;
      }
      const float msub = (m_use == -INFINITY) ? 0.f : m_use;  // all-masked rows: every p = ex2(-inf) = 0
      // x = s qscale - msub two at a time (packed fp32 fma), p = 2^x, P in
      // fp16 pairs; the row sum adds exactly those fp16 values (fp16 pairs
      // over 4 steps each, then fp32), so l matches the P that P.V uses.
      const uint64_t qs2 = f32x2_pack(p.qscale, p.qscale), nm2 = f32x2_pack(-msub, -msub);
      __half2 hs[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) hs[k] = __float2half2_rn(0.f);
      uint32_t ph[kBN / 2];
#pragma unroll
      for (int i = 0; i < kBN / 2; ++i) {
        float x0, x1;
        f32x2_unpack(f32x2_fma(f32x2_pack(s[2 * i], s[2 * i + 1]), qs2, nm2), x0, x1);
        const __half2 hv = __floats2half2_rn(tc::ex2(x0), tc::ex2(x1));
        ph[i] = *reinterpret_cast<const uint32_t*>(&hv);
        hs[i & 7] = __hadd2(hs[i & 7], hv);
      }
      float psum = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float2 f = __half22float2(hs[k]);
        psum += f.x + f.y;
      }
      l_run = l_run * alpha + psum;
      m_run = m_use;
      if (tid == 0) PF_TRACE(6, j);
      if (tid == 128) PF_TRACE(9, j);
      if (__any_sync(0xffffffffu, rescale)) {
        // O holds P.V up to block j-1 only after P.V(j-1) completed.
        if (j >= 1 && ok) ok = wait_bar(bar_pfree(t, j - 1), ph_2(j - 1));
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          const uint32_t col = tO(t) + lane_base + c * 32;
          tc::ld32(col, v);
          tc::wait_ld(v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tc::st32(col, v);
        }
        tc::wait_st();
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      // P (64 fp16 values as 32 pairs) over the scores it replaces in the
      // tile's score buffer j % 2 (this thread's lane, columns 0-31): the
      // A operand of P.V(j).  S(j+2) reuses the buffer only after P.V(j),
      // issued before it by the same thread.
      {
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          lo[i] = ph[i];
          hi[i] = ph[16 + i];
        }
        tc::st16(tS(t, j) + lane_base, lo);
        tc::st16(tS(t, j) + lane_base + 16, hi);
        tc::wait_st();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_pfull(t, j));
      if (tid == 0) PF_TRACE(5, j);
      if (tid == 128) PF_TRACE(8, j);
    }
    // ---- epilogue ------------------------------------------------------------
    const int qi = qt * kRows + t * 128 + row;
    __half* orow = p.out + ((static_cast<int64_t>(b) * p.QL + qi) * p.H + h) * D;
    if (nblocks > 0 && ok) ok = wait_bar(bar_pfree(t, nblocks - 1), ph_2(nblocks - 1));
    ok = __all_sync(0xffffffffu, ok);
    tc::fence_after_sync();
    if (nblocks > 0 && ok) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        tc::ld32(tO(t) + lane_base + c * 32, v);
        tc::wait_ld(v);
        if (qi < p.QL) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint4 u;
            __half2* h2 = reinterpret_cast<__half2*>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              h2[e] = __floats2half2_rn(v[8 * k + 2 * e] * inv, v[8 * k + 2 * e + 1] * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * k) = u;
          }
        }
      }
    } else if (qi < p.QL) {
      // No visible token (or a failed wait): zero row, as attention.cu:334 does for l == 0.
      for (int c = 0; c < D / 8; ++c) reinterpret_cast<uint4*>(orow)[c] = make_uint4(0, 0, 0, 0);
    }
    if (!ok && lane == 0) fail_flag = 1;
  }
  tc::fence_before_sync();
  __syncthreads();
  if (fail_flag && tid == 0 && err) atomicExch(err, 2);
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

}  // namespace prefill

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_prefill() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D view [rows][H][D] of a row-major fp16 tensor; box = 64 dims x 1 head x
// box_rows rows, 128-byte swizzle (inner box extent is exactly 128 B).
int map_rows_sw128(CUtensorMap* map, const void* base, int64_t rows, int H, int D, int box_rows) {
  auto fn = encode_fn_prefill();
  if (!fn) return fail(MEMOPT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MEMOPT_ERR_CUDA, "cuTensorMapEncodeTiled (prefill) failed: " + std::to_string(static_cast<int>(r)));
  return MEMOPT_OK;
}

template <int D, int BS>
int launch_prefill(const prefill::Params& p, const void* query, const void* kpool, const void* vpool,
                   cudaStream_t s) {
  using C = prefill::Cfg<D, BS>;
  alignas(64) CUtensorMap qm, km, vm;
  int st = map_rows_sw128(&qm, query, static_cast<int64_t>(p.B) * p.QL, p.H, D, 128);
  if (st != MEMOPT_OK) return st;
  st = map_rows_sw128(&km, kpool, p.NB * BS, p.H / p.group, D, BS);
  if (st != MEMOPT_OK) return st;
  st = map_rows_sw128(&vm, vpool, p.NB * BS, p.H / p.group, D, BS);
  if (st != MEMOPT_OK) return st;
  auto kern = prefill::prefill_kernel<D, BS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill)");
  const dim3 grid((p.QL + prefill::kRows - 1) / prefill::kRows, p.H, p.B);
  kern<<<grid, prefill::kThreads, C::SMEM, s>>>(p, qm, km, vm, nullptr);
  MEMOPT_LAUNCH_CHECK("prefill_kernel launch");
  return MEMOPT_OK;
}

}  // namespace

#ifdef MEMOPT_PF_TRACE
extern "C" __attribute__((visibility("default"))) int memopt_prefill_trace(unsigned long long* host) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, prefill::g_pf_trace, sizeof(prefill::g_pf_trace)));
}
#endif

// ---- INT4 pools: pages dequantised into an fp16 paged scratch, then the
// fp16 prefill kernel.  This follows the reference's INT4 path
// (quantization.cu:371-428: dequantize_kv_cache_int4 into an fp16 cache,
// then fp16 attention): every K and V value is (code - 8) * its group's fp16
// scale, exact in fp32 and rounded once to fp16.
namespace {

// One CTA per (sequence, block-table slot, 4 KV heads), one warp per head.
// D/8 lanes cover one token row (each 8 dims: 4 code bytes in, one 16-byte
// fp16 store out), so a warp instruction writes 32/(D/8) whole rows of K or
// V; every value is (code - 8) * its group's fp16 scale.  Scratch page
// b * MB + i holds slot i of sequence b; its table entry is -1 where the slot
// is a hole (entry < 0 or >= NB) or lies past the sequence's context, which
// the prefill kernel skips exactly as it skips such entries of an fp16 pool.
template <int D, int BS>
__global__ void __launch_bounds__(128) int4_pages_to_f16_kernel(const uint8_t* __restrict__ pages,
                                                                const int32_t* __restrict__ bt,
                                                                const int32_t* __restrict__ ctx, int MB,
                                                                int64_t NB, int KVH, __half* __restrict__ k16,
                                                                __half* __restrict__ v16,
                                                                int32_t* __restrict__ bt16) {
  constexpr int G = D / 64;
  constexpr int LPR = D / 8;        // lanes per token row
  constexpr int RPI = 32 / LPR;     // rows per warp instruction
  constexpr int64_t kPage = static_cast<int64_t>(BS) * D + static_cast<int64_t>(BS) * G * 4;
  const int hq = (KVH + 3) / 4;
  const int i = blockIdx.x / hq, b = blockIdx.y;
  const int64_t slot = static_cast<int64_t>(b) * MB + i;
  const int c = __ldg(ctx + b);
  const int e = __ldg(bt + slot);
  const bool valid = e >= 0 && e < NB && c > 0 && i < (c + BS - 1) / BS;
  const int hg = blockIdx.x - i * hq;
  if (threadIdx.x == 0 && hg == 0) bt16[slot] = valid ? static_cast<int32_t>(slot) : -1;
  if (!valid) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int h = hg * 4 + warp;
  if (h >= KVH) return;
  const uint8_t* pg = pages + (static_cast<int64_t>(e) * KVH + h) * kPage;
  const __half* ks = reinterpret_cast<const __half*>(pg + BS * D);
  const __half* vs = reinterpret_cast<const __half*>(pg + BS * D + BS * G * 2);
  const int cl = lane % LPR;      // 8-dim chunk of the row: code bytes 4 cl .. 4 cl + 3
  const int g = cl / 8;           // its 64-dim scale group
#pragma unroll
  for (int r0 = 0; r0 < BS; r0 += RPI) {
    const int pos = r0 + lane / LPR;
    // V rows whose position has bit 1 set hold their two 32-byte halves swapped (D = 128)
    const int vb = (D == 128 && (pos & 2)) ? (4 * cl) ^ 32 : 4 * cl;
    const uint32_t kw = *reinterpret_cast<const uint32_t*>(pg + pos * (D / 2) + 4 * cl);
    const uint32_t vw = *reinterpret_cast<const uint32_t*>(pg + BS * (D / 2) + pos * (D / 2) + vb);
    const float sk = __half2float(ks[pos * G + g]);
    const float sv = __half2float(vs[int4_vscale_index(pos, g, G)]);
    const int64_t orow = ((slot * BS + pos) * KVH + h) * D + 8 * cl;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const uint32_t w = kv ? vw : kw;
      const float sc = kv ? sv : sk;
      uint32_t hv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {  // byte j: dims 2j (low nibble), 2j + 1 (high nibble)
        const uint32_t byte = (w >> (8 * j)) & 0xFFu;
        const __half2 pr = __floats2half2_rn(static_cast<float>(static_cast<int>(byte & 15u) - 8) * sc,
                                             static_cast<float>(static_cast<int>(byte >> 4) - 8) * sc);
        hv[j] = *reinterpret_cast<const uint32_t*>(&pr);
      }
      *reinterpret_cast<uint4*>((kv ? v16 : k16) + orow) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    }
  }
}

struct Int4Scratch {
  size_t k, v, bt, total;
};
Int4Scratch int4_scratch_layout(int B, int KVH, int D, int MB, int BS) {
  auto a256 = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  Int4Scratch l{};
  const size_t kv = a256(static_cast<size_t>(B) * MB * BS * KVH * D * 2);
  l.k = 0;
  l.v = kv;
  l.bt = 2 * kv;
  l.total = 2 * kv + a256(static_cast<size_t>(B) * MB * 4);
  return l;
}

}  // namespace

int prefill_f16(const void* query, const void* kpool, const void* vpool, const int32_t* bt, const int32_t* ctx,
                int B, int QL, int H, int KVH, int D, int MB, int64_t NB, int BS, int window_clamped, int causal,
                void* out, cudaStream_t s);

bool prefill_int4_supported(int D, int BS) { return (D == 64 || D == 128) && (BS == 16 || BS == 32); }

size_t prefill_int4_scratch_bytes(int B, int KVH, int D, int MB, int BS) {
  if (B <= 0 || KVH <= 0 || MB <= 0 || !prefill_int4_supported(D, BS)) return 0;
  return int4_scratch_layout(B, KVH, D, MB, BS).total;
}

// Called by memopt_paged_attention_int4_ex for q_len >= kPrefillMinRows;
// `scratch` (prefill_int4_scratch_bytes) is 256-byte aligned.
int prefill_int4(const void* query, const uint8_t* pages, const int32_t* bt, const int32_t* ctx, int B, int QL,
                 int H, int KVH, int D, int MB, int64_t NB, int BS, int window_clamped, int causal, void* out,
                 void* scratch, size_t scratch_bytes, cudaStream_t s) {
  if (!prefill_int4_supported(D, BS)) return fail(MEMOPT_ERR_UNSUPPORTED, "prefill_int4: unsupported (block_size, head_dim)");
  const Int4Scratch l = int4_scratch_layout(B, KVH, D, MB, BS);
  if (reinterpret_cast<uintptr_t>(scratch) & 255u)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention_int4: workspace must be 256-byte aligned");
  if (scratch == nullptr || scratch_bytes < l.total)
    return fail(MEMOPT_ERR_WORKSPACE, "dynamic_sparse_attention_int4: workspace too small for the fp16 page scratch "
                                      "(need " + std::to_string(l.total) + " bytes past the split workspace)");
  const int64_t nb16 = static_cast<int64_t>(B) * MB;
  if (B > 65535) return fail(MEMOPT_ERR_UNSUPPORTED, "prefill_int4: more than 65535 sequences");
  if (nb16 * BS > 0x7fffffffLL) return fail(MEMOPT_ERR_UNSUPPORTED, "prefill_int4: more than 2^31 scratch rows");
  uint8_t* base = static_cast<uint8_t*>(scratch);
  __half* k16 = reinterpret_cast<__half*>(base + l.k);
  __half* v16 = reinterpret_cast<__half*>(base + l.v);
  int32_t* bt16 = reinterpret_cast<int32_t*>(base + l.bt);
  if (static_cast<int64_t>(MB) * ((KVH + 3) / 4) > 0x7fffffffLL)
    return fail(MEMOPT_ERR_UNSUPPORTED, "prefill_int4: too many pages per sequence");
  const dim3 grid(MB * ((KVH + 3) / 4), B);
#define MEMOPT_INT4_GATHER(DD, BB)                                                                                int4_pages_to_f16_kernel<DD, BB><<<grid, 128, 0, s>>>(pages, bt, ctx, MB, NB, KVH, k16, v16, bt16)
  if (D == 128 && BS == 16) MEMOPT_INT4_GATHER(128, 16);
  else if (D == 128 && BS == 32) MEMOPT_INT4_GATHER(128, 32);
  else if (D == 64 && BS == 16) MEMOPT_INT4_GATHER(64, 16);
  else MEMOPT_INT4_GATHER(64, 32);
#undef MEMOPT_INT4_GATHER
  MEMOPT_LAUNCH_CHECK("int4_pages_to_f16_kernel launch");
  return prefill_f16(query, k16, v16, bt16, ctx, B, QL, H, KVH, D, MB, nb16, BS, window_clamped, causal, out, s);
}

// Called by memopt_paged_attention_f16 for q_len >= kPrefillMinRows.
int prefill_f16(const void* query, const void* kpool, const void* vpool, const int32_t* bt, const int32_t* ctx,
                int B, int QL, int H, int KVH, int D, int MB, int64_t NB, int BS, int window_clamped, int causal,
                void* out, cudaStream_t s) {
  prefill::Params p{};
  p.bt = bt;
  p.ctx = ctx;
  p.out = reinterpret_cast<__half*>(out);
  p.B = B;
  p.QL = QL;
  p.H = H;
  p.MB = MB;
  p.NB = NB;
  p.window = window_clamped;
  p.qscale = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  p.group = H / KVH;
  p.causal = causal ? 1 : 0;
  if (static_cast<int64_t>(B) * QL > 0x7fffffffLL || NB * BS > 0x7fffffffLL)
    return fail(MEMOPT_ERR_UNSUPPORTED, "prefill: more than 2^31 rows");
  if (D == 128 && BS == 16) return launch_prefill<128, 16>(p, query, kpool, vpool, s);
  if (D == 128 && BS == 32) return launch_prefill<128, 32>(p, query, kpool, vpool, s);
  if (D == 64 && BS == 16) return launch_prefill<64, 16>(p, query, kpool, vpool, s);
  if (D == 64 && BS == 32) return launch_prefill<64, 32>(p, query, kpool, vpool, s);
  return fail(MEMOPT_ERR_UNSUPPORTED, "prefill: unsupported (block_size, head_dim)");
}

}  // namespace memopt
