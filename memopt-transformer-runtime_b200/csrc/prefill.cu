// prefill.cu — multi-query / prefill path of dynamic_sparse_attention on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Semantics are those of attention.cu:98-339 (reference): every query row of
// sequence b sees the tokens [max(0, ctx_b - W), ctx_b) of the pages whose
// block-table entry is >= 0 (and < num_blocks here), with no causal mask, so
// all rows of a sequence share one key set and the work is a dense
// non-causal attention per (sequence, head).
//
// One CTA = (128-query tile, head, sequence), one warpgroup:
//   * Q tile [128 x D] and, per step, a K/V block of 128 tokens (128/BS
//     pages) are staged by TMA (3-D tensor maps over the query tensor and the
//     fp16 pool, 128-byte swizzle, no multicast) into 1024-B aligned smem;
//     K/V blocks are double-buffered;
//   * thread 0 issues S = Q K^T (M=128, N=128, K=D) into TMEM columns
//     [0,128), then O += P V (M=128, N=D, K=128 tokens; V is the MN-major
//     operand) into TMEM columns [128, 128+D); completion is tracked with
//     tcgen05.commit on mbarriers;
//   * each thread owns one query row (TMEM lane): it loads its S row with
//     tcgen05.ld, masks, runs the online softmax in the log2 domain, writes
//     P (fp16) to smem in the swizzled K-major layout, and rescales its O row
//     in TMEM only when its running max grows by more than 2^8 (stale maxima
//     below that bound keep P <= 256, exact enough in fp16);
//   * the epilogue divides O by the row sum and stores fp16 rows.
// Pages that are skipped (entry < 0 or >= num_blocks) are zero-filled in smem
// and masked; every mbarrier wait is bounded and reports through `err`.
#include <cmath>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

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
};

constexpr int kTileBytes = 128 * 128;  // 128 rows x 128 B (one 64-wide half)
constexpr int kBtCache = 4096;         // block-table entries cached in smem per CTA

template <int D, int BS>
struct Cfg {
  static constexpr int HALVES = D / 64;
  static constexpr int PPB = 128 / BS;                 // pages per 128-token block
  static constexpr int TILE = HALVES * kTileBytes;     // one 128-row tile (Q, K or V)
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = TILE;                   // K ring: 2 tiles
  static constexpr int V_OFF = K_OFF + 2 * TILE;       // V ring: 2 tiles
  static constexpr int P_OFF = V_OFF + 2 * TILE;       // P: 128 rows x 128 tokens fp16
  static constexpr int BT_OFF = P_OFF + 2 * kTileBytes;  // block-table window (kBtCache entries)
  static constexpr int SMEM = BT_OFF + 4 * 4096 + 1024;     // + alignment slack
  static constexpr uint32_t PAGE_TX = 1u * HALVES * BS * 128u;  // bytes of one page of K (or V)
  static constexpr uint32_t IDESC_S = tc::idesc_f16(128, 128, false, false);
  static constexpr uint32_t IDESC_PV = tc::idesc_f16(128, D, false, true);
};

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity) {
  uint32_t polls = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++polls >= kMaxPolls) return false;
  }
  return true;
}

// Warp-specialised: warps 0-7 run the softmax, two threads per query row
// (warp w handles row 32*(w%4)+lane, score columns [64*(w/4), +64) and O
// columns [(D/2)*(w/4), +D/2)); warp 8 stages Q/K/V with TMA and issues the
// MMAs.  Barriers: 0 = Q, 1..2 = K ring, 3..4 = V ring, 6 = S(j) done
// (commit), 7 = P.V(j) done (commit), 8 = S(j) read out of TMEM (8 arrivals,
// one per softmax warp), 9 = P(j) written and O rescaled (8 arrivals).
constexpr int kThreads = 288;
constexpr int kSoftmaxWarps = 8;

template <int D, int BS>
__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ Params p, const __grid_constant__ CUtensorMap qmap,
               const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
               int32_t* __restrict__ err) {
  using C = Cfg<D, BS>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[10];
  __shared__ uint32_t tmem_slot;
  __shared__ int fail_flag;
  __shared__ float red_max[2][2][128];  // [block parity][half][row]
  __shared__ float red_sum[2][128];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(base);
  const uint32_t sQ = sbase + C::Q_OFF, sP = sbase + C::P_OFF;
  auto bar_at = [&](int i) { return smem_u32(&bars[i]); };
  const uint32_t bar_q = bar_at(0), bar_s = bar_at(6), bar_o = bar_at(7), bar_sfree = bar_at(8),
                 bar_pready = bar_at(9);

  const int ctx = __ldg(p.ctx + b);
  const int ws = (p.window < ctx) ? (ctx - p.window) : 0;
  const int p_hi = ctx > 0 ? min((ctx + BS - 1) / BS, p.MB) : 0;
  const int p_lo = ws / BS;
  const int nblocks = p_hi > p_lo ? (p_hi - p_lo + C::PPB - 1) / C::PPB : 0;

  if (tid == 0) {
    for (int i = 0; i < 8; ++i) mbar_init(bar_at(i), 1);
    mbar_init(bar_sfree, kSoftmaxWarps);
    mbar_init(bar_pready, kSoftmaxWarps);
    fence_mbar_init();
    fail_flag = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(smem_u32(&tmem_slot), 256);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  // The pages of this sequence's window are read once into smem (when they
  // fit), so per-block validity checks never wait on global memory.
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

  if (warp == kSoftmaxWarps) {
    // =========================== producer warp ===========================
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    // Stage the K (is_v = false) or V pages of block j, zero-filling skipped pages.
    auto stage = [&](int j, bool is_v) {
      const int slot = j & 1;
      const uint32_t bar = is_v ? bar_at(3 + slot) : bar_at(1 + slot);
      const int off = (is_v ? C::V_OFF : C::K_OFF) + slot * C::TILE;
      int phys;
      const uint32_t mask = page_bits(j, phys);
      const uint32_t bad = ~mask & ((1u << C::PPB) - 1u);
      if (bad != 0) {
        for (int pg = 0; pg < C::PPB; ++pg) {
          if (!((bad >> pg) & 1u)) continue;
          for (int hh = 0; hh < C::HALVES; ++hh) {
            uint4* dst = reinterpret_cast<uint4*>(base + off + hh * kTileBytes + pg * BS * 128);
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
          tma_load_3d(sbase + off + hh * kTileBytes + lane * BS * 128, is_v ? &vmap : &kmap, hh * 64, h,
                      phys * BS, bar);
      }
    };
    auto issue_s = [&](int j) {
      const uint32_t sK = sbase + C::K_OFF + (j & 1) * C::TILE;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk / 4) * kTileBytes + (kk % 4) * 32;
        tc::mma_f16(tS, tc::sdesc_sw128(sQ + off, 16, 1024), tc::sdesc_sw128(sK + off, 16, 1024), C::IDESC_S,
                    kk > 0);
      }
      tc::commit(bar_s);
    };
    auto issue_pv = [&](int j) {
      const uint32_t sV = sbase + C::V_OFF + (j & 1) * C::TILE;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t aoff = (kk / 4) * kTileBytes + (kk % 4) * 32;
        tc::mma_f16(tO, tc::sdesc_sw128(sP + aoff, 16, 1024), tc::sdesc_sw128(sV + kk * 2048, kTileBytes, 1024),
                    C::IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
      }
      tc::commit(bar_o);
    };
    bool ok = true;
    if (nblocks > 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(bar_q, C::TILE);
        for (int hh = 0; hh < C::HALVES; ++hh)
          tma_load_3d(sQ + hh * kTileBytes, &qmap, hh * 64, h, b * p.QL + qt * 128, bar_q);
      }
      stage(0, false);
      stage(0, true);
      if (nblocks > 1) {
        stage(1, false);
        stage(1, true);
      }
      if (lane == 0) {
        ok = wait_bar(bar_q, 0) && wait_bar(bar_at(1), 0);
        if (ok) {
          tc::fence_after_sync();
          issue_s(0);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    for (int j = 0; j < nblocks && ok; ++j) {
      if (j + 1 < nblocks) {
        // S(j+1) needs S(j) read out of TMEM and K(j+1) staged.
        if (lane == 0) {
          ok = wait_bar(bar_sfree, j & 1) && wait_bar(bar_at(1 + ((j + 1) & 1)), ((j + 1) >> 1) & 1);
          if (ok) {
            tc::fence_after_sync();
            issue_s(j + 1);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (j + 2 < nblocks) stage(j + 2, false);  // S(j) has completed: K slot j & 1 is free
      }
      // P.V(j) needs P(j) written (which implies P.V(j-1) completed) and V(j) staged.
      if (lane == 0) {
        ok = wait_bar(bar_pready, j & 1) && wait_bar(bar_at(3 + (j & 1)), (j >> 1) & 1);
        if (ok) {
          tc::fence_after_sync();
          issue_pv(j);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      // P(j) ready implies P.V(j-1) completed: V slot (j+1)&1 is free for block j+1.
      if (j >= 1 && j + 1 < nblocks) stage(j + 1, true);
    }
    if (!ok && lane == 0) fail_flag = 1;
  } else {
    // =========================== softmax warps ===========================
    const int row = (warp & 3) * 32 + lane;  // query row = TMEM lane
    const int hf = warp >> 2;                // which half of the columns
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    auto sync_softmax = [] { asm volatile("bar.sync 1, 256;" ::: "memory"); };
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // Every softmax thread runs the same number of iterations (named barrier
    // below); failures are published in fail_flag and read after the barrier.
    for (int j = 0; j < nblocks; ++j) {
      ok = wait_bar(bar_s, j & 1);
      tc::fence_after_sync();
      float s[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        tc::ld32(tS + lane_base + hf * 64 + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = v[i];
      }
      tc::wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree);
      ok = __all_sync(0xffffffffu, ok);
      int phys_unused;
      const uint32_t mask = page_bits(j, phys_unused);
      const int tok0 = (p_lo + j * C::PPB) * BS + hf * 64;
      const uint32_t hmask = (mask >> (hf * 64 / BS)) & ((1u << (64 / BS)) - 1u);
      const bool edge = hmask != ((1u << (64 / BS)) - 1u) || tok0 < ws || tok0 + 64 > ctx;
      float mx = -INFINITY;
      if (edge) {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const int t = tok0 + i;
          const bool valid = ((hmask >> (i / BS)) & 1u) && t >= ws && t < ctx;
          s[i] = valid ? s[i] * p.qscale : -INFINITY;
          mx = fmaxf(mx, s[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          s[i] *= p.qscale;
          mx = fmaxf(mx, s[i]);
        }
      }
      // Row max over both halves (the two threads of a row reach the same decision).
      red_max[j & 1][hf][row] = mx;
      if (!ok) fail_flag = 1;
      sync_softmax();
      if (fail_flag) {
        ok = false;
        break;
      }
      mx = fmaxf(red_max[j & 1][0][row], red_max[j & 1][1][row]);
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
      float psum = 0.f;
      uint32_t ph[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = tc::ex2(s[2 * i] - msub);
        const float p1 = tc::ex2(s[2 * i + 1] - msub);
        psum += p0 + p1;
        const __half2 hv = __floats2half2_rn(p0, p1);
        ph[i] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      l_run = l_run * alpha + psum;  // partial row sum of this half
      m_run = m_use;
      // P.V(j-1) must be done before P and the O rows are touched.
      if (j > 0 && !wait_bar(bar_o, (j - 1) & 1)) fail_flag = 1;  // seen at the next barrier
      tc::fence_after_sync();
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          float v[32];
          const uint32_t col = tO + lane_base + hf * (D / 2) + c * 32;
          tc::ld32(col, v);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tc::st32(col, v);
        }
        tc::wait_st();
      }
      // This half's 64 P values -> smem half hf, K-major with 128-byte swizzle.
#pragma unroll
      for (int chunk = 0; chunk < 8; ++chunk) {
        uint8_t* dst = base + C::P_OFF + hf * kTileBytes + row * 128 + ((chunk ^ (row & 7)) * 16);
        *reinterpret_cast<uint4*>(dst) =
            make_uint4(ph[4 * chunk], ph[4 * chunk + 1], ph[4 * chunk + 2], ph[4 * chunk + 3]);
      }
      fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_pready);
    }
    // ---- epilogue ------------------------------------------------------------
    red_sum[hf][row] = l_run;
    sync_softmax();
    ok = ok && !fail_flag;
    const float l_tot = red_sum[0][row] + red_sum[1][row];
    const int qi = qt * 128 + row;
    __half* orow = p.out + ((static_cast<int64_t>(b) * p.QL + qi) * p.H + h) * D + hf * (D / 2);
    if (nblocks > 0 && ok) ok = wait_bar(bar_o, (nblocks - 1) & 1);
    ok = __all_sync(0xffffffffu, ok);
    tc::fence_after_sync();
    if (nblocks > 0 && ok) {
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        float v[32];
        tc::ld32(tO + lane_base + hf * (D / 2) + c * 32, v);
        tc::wait_ld();
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
      for (int c = 0; c < D / 16; ++c) reinterpret_cast<uint4*>(orow)[c] = make_uint4(0, 0, 0, 0);
    }
    if (!ok && lane == 0) fail_flag = 1;
  }
  tc::fence_before_sync();
  __syncthreads();
  if (fail_flag && tid == 0 && err) atomicExch(err, 2);
  if (warp == 0) tc::tmem_dealloc(tmem, 256);
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
  st = map_rows_sw128(&km, kpool, p.NB * BS, p.H, D, BS);
  if (st != MEMOPT_OK) return st;
  st = map_rows_sw128(&vm, vpool, p.NB * BS, p.H, D, BS);
  if (st != MEMOPT_OK) return st;
  auto kern = prefill::prefill_kernel<D, BS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill)");
  const dim3 grid((p.QL + 127) / 128, p.H, p.B);
  kern<<<grid, prefill::kThreads, C::SMEM, s>>>(p, qm, km, vm, nullptr);
  MEMOPT_LAUNCH_CHECK("prefill_kernel launch");
  return MEMOPT_OK;
}

}  // namespace

// Called by memopt_paged_attention_f16 for q_len >= kPrefillMinRows.
int prefill_f16(const void* query, const void* kpool, const void* vpool, const int32_t* bt, const int32_t* ctx,
                int B, int QL, int H, int D, int MB, int64_t NB, int BS, int window_clamped, void* out,
                cudaStream_t s) {
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
  if (static_cast<int64_t>(B) * QL > 0x7fffffffLL || NB * BS > 0x7fffffffLL)
    return fail(MEMOPT_ERR_UNSUPPORTED, "prefill: more than 2^31 rows");
  if (D == 128 && BS == 16) return launch_prefill<128, 16>(p, query, kpool, vpool, s);
  if (D == 128 && BS == 32) return launch_prefill<128, 32>(p, query, kpool, vpool, s);
  if (D == 64 && BS == 16) return launch_prefill<64, 16>(p, query, kpool, vpool, s);
  if (D == 64 && BS == 32) return launch_prefill<64, 32>(p, query, kpool, vpool, s);
  return fail(MEMOPT_ERR_UNSUPPORTED, "prefill: unsupported (block_size, head_dim)");
}

}  // namespace memopt
