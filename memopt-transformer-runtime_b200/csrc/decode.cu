// decode.cu — host side of dynamic_sparse_attention (paged decode path).
//
// Replaces the host dispatch of attention.cu:371-521: argument checks, window
// clamp (attention.cu:453-455), scale 1/sqrtf(D) (:460), and dispatch on
// (block_size, head_dim) in {16,32} x {64,128} (:494-507), but launches on the
// caller's stream (the reference used the legacy default stream).
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "decode_kernel.cuh"
#include "decode_mq.cuh"
#include "decode_mq4.cuh"


namespace memopt {

// prefill.cu: tcgen05 path for q_len >= kPrefillMinRows.
int prefill_f16(const void* query, const void* kpool, const void* vpool, const int32_t* bt, const int32_t* ctx,
                int B, int QL, int H, int KVH, int D, int MB, int64_t NB, int BS, int window_clamped, int causal,
                void* out, cudaStream_t s);
constexpr int kPrefillMinRows = 64;
// INT4 pools: pages dequantised into an fp16 scratch, then the same kernel.
bool prefill_int4_supported(int D, int BS);
size_t prefill_int4_scratch_bytes(int B, int KVH, int D, int MB, int BS);
int prefill_int4(const void* query, const uint8_t* pages, const int32_t* bt, const int32_t* ctx, int B, int QL,
                 int H, int KVH, int D, int MB, int64_t NB, int BS, int window_clamped, int causal, void* out,
                 void* scratch, size_t scratch_bytes, cudaStream_t s);

// One predicate for the workspace size and the dispatch: q_len >= 64 runs on
// the tcgen05 prefill kernel (no split-K workspace); MEMOPT_DISABLE_PREFILL=1
// forces the decode kernel (diagnostics).
bool use_prefill(int q_len) {
  static const bool disabled = [] {
    const char* e = std::getenv("MEMOPT_DISABLE_PREFILL");
    return e != nullptr && e[0] == '1';
  }();
  return q_len >= kPrefillMinRows && !disabled;
}

namespace {

using decode::Cfg;
using decode::Params;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 3-D view of an fp16 pool [NB*BS rows][H][D]: box = one head, BS rows.
int make_pool_map(CUtensorMap* map, const void* base, int64_t rows, int H, int D, int BS) {
  auto fn = encode_fn();
  if (!fn) return fail(MEMOPT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(D), 1, static_cast<cuuint32_t>(BS)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MEMOPT_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
  return MEMOPT_OK;
}

// The same view with 64-dim boxes of 16 rows and 128-byte swizzle (the
// multi-query kernel's ldmatrix layout).
int make_pool_map_sw(CUtensorMap* map, const void* base, int64_t rows, int H, int D) {
  auto fn = encode_fn();
  if (!fn) return fail(MEMOPT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {64, 1, 16};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MEMOPT_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
  return MEMOPT_OK;
}

int clamp_window(int window_size, int max_seq_len) {
  return (window_size <= 0 || window_size > max_seq_len) ? max_seq_len : window_size;
}

struct Split {
  int chunk_pages = 32;
  int n_chunks = 1;
};

// Chooses the page-chunk size: the item count is aimed at `twice_target` / 2
// items per fp16 warp slot of the machine (8 warps per SM), balancing the
// tail wave against per-item cost (split-K partials and their merge).  A
// chunk may span any number of pages (the kernel walks it in 32-page
// sub-windows), so calls with many query rows need no partials at all.
// Measured on B200: fp16 decode is fastest near 1.5 items per slot, the INT4
// kernel (16 warps per SM, cheaper items) near 4.
constexpr int kSplitF16 = 3;
constexpr int kSplitInt4 = 8;
// The INT4 multi-query kernel (costlier items: q hi/lo preparation, up to 8
// rows merged) measured best near 1.5 items per slot as well: at 32 query
// heads over 8 KV heads, batch 32 / 128, ctx 4096, 64 / 172 us against 84 /
// 177 us at the one-row INT4 target.
constexpr int kSplitMq4 = 3;
Split choose_split(int64_t pairs, int max_blocks_per_seq, int block_size, int window, int twice_target) {
  Split s;
  const int64_t wpages =
      window > 0 ? (static_cast<int64_t>(window) + block_size - 1) / block_size + 1 : 0;
  int max_pages = static_cast<int>(wpages < max_blocks_per_seq ? wpages : max_blocks_per_seq);
  if (max_pages < 1) max_pages = 1;
  const int64_t warp_slots = static_cast<int64_t>(sm_count()) * 2 * 4;
  const int64_t target = warp_slots * twice_target / 2;
  int64_t n = (target + pairs - 1) / pairs;
  // Keep at least 4 pages per item so partials stay a small share of traffic.
  const int max_chunks = max_pages >= 4 ? max_pages / 4 : 1;
  if (n > max_chunks) n = max_chunks;
  if (n < 1) n = 1;
  s.chunk_pages = static_cast<int>((max_pages + n - 1) / n);
  s.n_chunks = (max_pages + s.chunk_pages - 1) / s.chunk_pages;
  return s;
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

struct WsLayout {
  size_t tickets = 0, ml = 0, po = 0, total = 0;
};

WsLayout ws_layout(int64_t pairs, int n_chunks, int D) {
  WsLayout w;
  if (n_chunks <= 1) return w;
  w.tickets = 0;
  w.ml = align256(pairs * sizeof(int32_t));
  w.po = w.ml + align256(pairs * n_chunks * sizeof(float2));
  w.total = w.po + align256(static_cast<size_t>(pairs) * n_chunks * D * sizeof(float));
  return w;
}

// Multi-query decode: at least two query rows per KV head and a q_len below
// the prefill threshold.  INT4 calls of q_len >= 64 take the prefill path when its kernel supports
// (head_dim, block_size); otherwise, like every call below 64 rows with at
// least two query rows per KV head, the multi-query decode kernel.
bool use_prefill_int4(int q_len, int D, int BS) { return use_prefill(q_len) && prefill_int4_supported(D, BS); }

bool use_mq(bool int4, int q_len, int H, int KVH, int D, int BS) {
  const bool prefill = int4 ? use_prefill_int4(q_len, D, BS) : use_prefill(q_len);
  return !prefill && KVH > 0 && (H / KVH) * q_len >= 2;
}
// Query rows per tile: 16 on the fp16 pool, 8 on the INT4 pool (whose score
// mma holds each row's two integer halves as separate rows).
int mq_tile_rows(bool int4) { return int4 ? 8 : 16; }
int64_t mq_groups(int batch, int q_len, int H, int KVH, int tile_rows) {
  const int rows = (H / KVH) * q_len;
  return static_cast<int64_t>(batch) * KVH * ((rows + tile_rows - 1) / tile_rows);
}
// A tile's rows may span q_len - 1 extra tokens (causal rows end at their own
// token), so its chunks cover window + q_len - 1 tokens.
Split mq_split(bool int4, int batch, int q_len, int H, int KVH, int MB, int BS, int window) {
  return choose_split(mq_groups(batch, q_len, H, KVH, mq_tile_rows(int4)), MB, BS, window + q_len - 1,
                      int4 ? kSplitMq4 : kSplitF16);
}

template <int D, int BS>
int launch_mq4(const decode_mq::Params& p, cudaStream_t s) {
  using C = decode_mq4::Cfg<D, BS>;
  auto kern = decode_mq4::paged_decode_mq4_kernel<D, BS>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_mq4)");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t ctas_needed = (p.total_items + C::NW - 1) / C::NW;
  int per_sm = (227 * 1024) / C::SMEM;
  if (per_sm > C::MIN_BLOCKS) per_sm = C::MIN_BLOCKS;
  if (per_sm < 1) per_sm = 1;
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  const int grid = static_cast<int>(ctas_needed < cap ? ctas_needed : cap);
  kern<<<grid, C::NW * 32, C::SMEM, s>>>(p, nullptr);
  MEMOPT_LAUNCH_CHECK("paged_decode_mq4_kernel launch");
  return MEMOPT_OK;
}

template <int D, int BS>
int launch_mq(const decode_mq::Params& p, const CUtensorMap& km, const CUtensorMap& vm, cudaStream_t s) {
  using C = decode_mq::Cfg<D>;
  auto kern = decode_mq::paged_decode_mq_kernel<D, BS>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_mq)");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t ctas_needed = (p.total_items + C::NW - 1) / C::NW;
  int per_sm = (227 * 1024) / C::SMEM;
  if (per_sm > C::MIN_BLOCKS) per_sm = C::MIN_BLOCKS;
  if (per_sm < 1) per_sm = 1;
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  const int grid = static_cast<int>(ctas_needed < cap ? ctas_needed : cap);
  kern<<<grid, C::NW * 32, C::SMEM, s>>>(p, km, vm, nullptr);
  MEMOPT_LAUNCH_CHECK("paged_decode_mq_kernel launch");
  return MEMOPT_OK;
}

// Runs the multi-query kernel with the checks common_setup already made.
// key_pool == nullptr: the INT4 pool, pages in value_pool.
int run_mq(const Params& one, const void* key_pool, const void* value_pool, int D, int BS, void* ws,
           size_t ws_bytes, cudaStream_t s) {
  const bool int4 = key_pool == nullptr;
  decode_mq::Params p{};
  p.pages = int4 ? static_cast<const uint8_t*>(value_pool) : nullptr;
  p.q = one.q;
  p.out = one.out;
  p.bt = one.bt;
  p.ctx = one.ctx;
  p.B = one.B;
  p.QL = one.QL;
  p.H = one.H;
  p.KVH = one.KVH;
  p.group = one.group;
  p.MB = one.MB;
  p.causal = one.causal;
  p.NB = one.NB;
  p.window = one.window;
  p.qscale = one.qscale;
  p.magic_f16 = one.magic_f16;
  p.magic_s8 = one.magic_s8;
  p.rows = one.group * one.QL;
  p.tiles = (p.rows + mq_tile_rows(int4) - 1) / mq_tile_rows(int4);
  const Split sp = mq_split(int4, one.B, one.QL, one.H, one.KVH, one.MB, BS, one.window);
  p.chunk_pages = sp.chunk_pages;
  p.n_chunks = sp.n_chunks;
  p.total_items = mq_groups(one.B, one.QL, one.H, one.KVH, mq_tile_rows(int4)) * sp.n_chunks;
  const int64_t pairs = static_cast<int64_t>(one.B) * one.QL * one.H;
  const WsLayout w = ws_layout(pairs, sp.n_chunks, D);
  if (w.total > 0) {
    if (ws == nullptr || ws_bytes < w.total)
      return fail(MEMOPT_ERR_WORKSPACE, "dynamic_sparse_attention: workspace too small (need " +
                                            std::to_string(w.total) + " bytes)");
    uint8_t* base = reinterpret_cast<uint8_t*>(ws);
    p.tickets = reinterpret_cast<int32_t*>(base + w.tickets);
    p.ml = reinterpret_cast<float2*>(base + w.ml);
    p.po = reinterpret_cast<float*>(base + w.po);
  }
  alignas(64) CUtensorMap km, vm;
  if (int4) {
    if (D == 128 && BS == 16) return launch_mq4<128, 16>(p, s);
    if (D == 128 && BS == 32) return launch_mq4<128, 32>(p, s);
    if (D == 64 && BS == 16) return launch_mq4<64, 16>(p, s);
    if (D == 64 && BS == 32) return launch_mq4<64, 32>(p, s);
    return fail(MEMOPT_ERR_UNSUPPORTED, "dynamic_sparse_attention_int4: unsupported geometry");
  }
  const int64_t rows = one.NB * BS;
  int st = make_pool_map_sw(&km, key_pool, rows, one.KVH, D);
  if (st != MEMOPT_OK) return st;
  st = make_pool_map_sw(&vm, value_pool, rows, one.KVH, D);
  if (st != MEMOPT_OK) return st;
  if (D == 128 && BS == 16) return launch_mq<128, 16>(p, km, vm, s);
  if (D == 128 && BS == 32) return launch_mq<128, 32>(p, km, vm, s);
  if (D == 64 && BS == 16) return launch_mq<64, 16>(p, km, vm, s);
  if (D == 64 && BS == 32) return launch_mq<64, 32>(p, km, vm, s);
  return fail(MEMOPT_ERR_UNSUPPORTED, "dynamic_sparse_attention: unsupported geometry");
}

template <int D, int BS, bool INT4>
int launch(const Params& p, const CUtensorMap& km, const CUtensorMap& vm, int32_t* err,
           cudaStream_t s) {
  using C = Cfg<D, BS, INT4>;
  auto kern = decode::paged_decode_kernel<D, BS, INT4>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode)");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t ctas_needed = (p.total_items + C::NW - 1) / C::NW;
  int per_sm = (227 * 1024) / C::SMEM;
  if (per_sm > C::MIN_BLOCKS) per_sm = C::MIN_BLOCKS;
  if (per_sm < 1) per_sm = 1;
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  const int grid = static_cast<int>(ctas_needed < cap ? ctas_needed : cap);
  kern<<<grid, C::NW * 32, C::SMEM, s>>>(p, km, vm, err);
  MEMOPT_LAUNCH_CHECK("paged_decode_kernel launch");
  return MEMOPT_OK;
}

int unsupported(int BS, int D) {
  return fail(MEMOPT_ERR_UNSUPPORTED,
              "dynamic_sparse_attention: unsupported (block_size=" + std::to_string(BS) +
                  ", head_dim=" + std::to_string(D) +
                  "). Supported combinations: block_size in {16,32}, head_dim in {64,128}.");
}

template <bool INT4>
int dispatch(const Params& p, int D, int BS, const CUtensorMap& km, const CUtensorMap& vm,
             int32_t* err, cudaStream_t s) {
  if (D == 128 && BS == 16) return launch<128, 16, INT4>(p, km, vm, err, s);
  if (D == 128 && BS == 32) return launch<128, 32, INT4>(p, km, vm, err, s);
  if (D == 64 && BS == 16) return launch<64, 16, INT4>(p, km, vm, err, s);
  if (D == 64 && BS == 32) return launch<64, 32, INT4>(p, km, vm, err, s);
  return unsupported(BS, D);
}

int common_setup(Params& p, const void* query, const int32_t* bt, const int32_t* ctx, int batch,
                 int q_len, int H, int KVH, int D, int MB, int64_t NB, int BS, int max_seq_len, int window,
                 int causal, bool int4, void* out, void* ws, size_t ws_bytes) {
  if (batch < 0 || q_len < 0 || H < 0 || D < 0 || MB < 0 || NB < 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: negative size");
  if (KVH <= 0 || (H > 0 && H % KVH != 0))
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: num_kv_heads must divide num_heads");
  if (!((BS == 16 || BS == 32) && (D == 64 || D == 128))) return unsupported(BS, D);
  if ((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: query/out must be 16-byte aligned");
  p.q = reinterpret_cast<const __half*>(query);
  p.out = reinterpret_cast<__half*>(out);
  p.bt = bt;
  p.ctx = ctx;
  p.B = batch;
  p.QL = q_len;
  p.H = H;
  p.KVH = KVH;
  p.group = H > 0 ? H / KVH : 1;
  p.causal = causal ? 1 : 0;
  p.MB = MB;
  p.NB = NB;
  p.window = clamp_window(window, max_seq_len);
  p.qscale = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  p.magic_f16 = 0x64006400u;
  p.magic_s8 = 0x80808080u;
  const int64_t pairs = static_cast<int64_t>(batch) * q_len * H;
  const Split sp = choose_split(pairs, MB, BS, p.window, int4 ? kSplitInt4 : kSplitF16);
  p.chunk_pages = sp.chunk_pages;
  p.n_chunks = sp.n_chunks;
  p.total_items = pairs * sp.n_chunks;
  const WsLayout w = ws_layout(pairs, sp.n_chunks, D);
  p.tickets = nullptr;
  p.ml = nullptr;
  p.po = nullptr;
  if (w.total > 0) {
    if (ws == nullptr || ws_bytes < w.total)
      return fail(MEMOPT_ERR_WORKSPACE, "dynamic_sparse_attention: workspace too small (need " +
                                            std::to_string(w.total) + " bytes)");
    uint8_t* base = reinterpret_cast<uint8_t*>(ws);
    p.tickets = reinterpret_cast<int32_t*>(base + w.tickets);
    p.ml = reinterpret_cast<float2*>(base + w.ml);
    p.po = reinterpret_cast<float*>(base + w.po);
  }
  return MEMOPT_OK;
}

int zero_output(void* out, int batch, int q_len, int H, int D, void* stream) {
  // No page can be visible: every output row is 0 (attention.cu:334).
  cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(batch) * q_len * H * D * 2,
                                  as_stream(stream));
  return e == cudaSuccess ? MEMOPT_OK : cuda_fail(e, "dynamic_sparse_attention: zero output");
}

}  // namespace

int validate_attention_f16(const void* query, const void* key_pool, const void* value_pool, int batch, int q_len,
                           int H, int KVH, int D, int MB, int64_t NB, int BS, const void* out) {
  if (batch < 0 || q_len < 0 || H < 0 || D < 0 || MB < 0 || NB < 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: negative size");
  if (KVH <= 0 || (H > 0 && H % KVH != 0))
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: num_kv_heads must divide num_heads");
  if (!((BS == 16 || BS == 32) && (D == 64 || D == 128))) return unsupported(BS, D);
  if ((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: query/out must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool)) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: pools must be 16-byte aligned");
  if (NB * BS > 0x7fffffffLL)
    return fail(MEMOPT_ERR_UNSUPPORTED, "dynamic_sparse_attention: pool has more than 2^31 token rows");
  return MEMOPT_OK;
}

}  // namespace memopt

using namespace memopt;

extern "C" size_t memopt_paged_attention_workspace_size_ex(int batch, int q_len, int num_heads, int num_kv_heads,
                                                           int head_dim, int max_blocks_per_seq, int block_size,
                                                           int max_seq_len, int window_size) {
  if (batch <= 0 || q_len <= 0 || num_heads <= 0 || head_dim <= 0 || block_size <= 0) return 0;
  if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return 0;
  const int64_t pairs = static_cast<int64_t>(batch) * q_len * num_heads;
  // One size serves every path the call can take (fp16 one-row, INT4,
  // fp16 multi-query): the largest need.
  const int w = clamp_window(window_size, max_seq_len);
  size_t need = ws_layout(pairs, choose_split(pairs, max_blocks_per_seq, block_size, w, kSplitF16).n_chunks,
                          head_dim).total;
  const size_t b = ws_layout(pairs, choose_split(pairs, max_blocks_per_seq, block_size, w, kSplitInt4).n_chunks,
                             head_dim).total;
  if (b > need) need = b;
  for (int f = 0; f < 2; ++f) {
    if (!use_mq(f == 1, q_len, num_heads, num_kv_heads, head_dim, block_size)) continue;
    const size_t c = ws_layout(pairs,
                               mq_split(f == 1, batch, q_len, num_heads, num_kv_heads, max_blocks_per_seq,
                                        block_size, w).n_chunks,
                               head_dim).total;
    if (c > need) need = c;
  }
  return need;
}

extern "C" size_t memopt_paged_attention_int4_workspace_size_ex(int batch, int q_len, int num_heads,
                                                                int num_kv_heads, int head_dim,
                                                                int max_blocks_per_seq, int block_size,
                                                                int max_seq_len, int window_size) {
  const size_t split = memopt_paged_attention_workspace_size_ex(batch, q_len, num_heads, num_kv_heads, head_dim,
                                                                max_blocks_per_seq, block_size, max_seq_len,
                                                                window_size);
  if (batch <= 0 || q_len <= 0 || num_kv_heads <= 0 || !use_prefill_int4(q_len, head_dim, block_size)) return split;
  return align256(split) + prefill_int4_scratch_bytes(batch, num_kv_heads, head_dim, max_blocks_per_seq, block_size);
}

extern "C" size_t memopt_paged_attention_workspace_size(int batch, int q_len, int num_heads,
                                                        int head_dim, int max_blocks_per_seq,
                                                        int block_size, int max_seq_len,
                                                        int window_size) {
  return memopt_paged_attention_workspace_size_ex(batch, q_len, num_heads, num_heads, head_dim, max_blocks_per_seq,
                                                  block_size, max_seq_len, window_size);
}

extern "C" size_t memopt_paged_attention_ticket_bytes(int batch, int q_len, int num_heads) {
  if (batch <= 0 || q_len <= 0 || num_heads <= 0) return 0;
  return align256(static_cast<size_t>(batch) * q_len * num_heads * sizeof(int32_t));
}

extern "C" int memopt_paged_attention_f16_ex(const void* query, const void* key_pool,
                                             const void* value_pool, const int32_t* block_tables,
                                             const int32_t* context_lens, int batch, int q_len,
                                             int num_heads, int num_kv_heads, int head_dim,
                                             int max_blocks_per_seq, int64_t num_blocks, int block_size,
                                             int max_seq_len, int window_size, int causal, void* out,
                                             void* workspace, size_t workspace_bytes, void* stream) {
  Params p{};
  int st = common_setup(p, query, block_tables, context_lens, batch, q_len, num_heads, num_kv_heads, head_dim,
                        max_blocks_per_seq, num_blocks, block_size, max_seq_len, window_size, causal, false, out,
                        workspace, workspace_bytes);
  if (st != MEMOPT_OK) return st;
  if (p.total_items == 0) return MEMOPT_OK;
  if (num_blocks == 0 || max_blocks_per_seq == 0)
    return zero_output(out, batch, q_len, num_heads, head_dim, stream);
  if ((reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool)) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention: pools must be 16-byte aligned");
  if (num_blocks * block_size > 0x7fffffffLL)
    return fail(MEMOPT_ERR_UNSUPPORTED, "dynamic_sparse_attention: pool has more than 2^31 token rows");
  if (use_prefill(q_len))
    return prefill_f16(query, key_pool, value_pool, block_tables, context_lens, batch, q_len, num_heads,
                       num_kv_heads, head_dim, max_blocks_per_seq, num_blocks, block_size, p.window, causal, out,
                       as_stream(stream));
  if (use_mq(false, q_len, num_heads, num_kv_heads, head_dim, block_size))
    return run_mq(p, key_pool, value_pool, head_dim, block_size, workspace, workspace_bytes, as_stream(stream));
  alignas(64) CUtensorMap km, vm;
  st = make_pool_map(&km, key_pool, num_blocks * block_size, num_kv_heads, head_dim, block_size);
  if (st != MEMOPT_OK) return st;
  st = make_pool_map(&vm, value_pool, num_blocks * block_size, num_kv_heads, head_dim, block_size);
  if (st != MEMOPT_OK) return st;
  return dispatch<false>(p, head_dim, block_size, km, vm, nullptr, as_stream(stream));
}

extern "C" int memopt_paged_attention_f16(const void* query, const void* key_pool,
                                          const void* value_pool, const int32_t* block_tables,
                                          const int32_t* context_lens, int batch, int q_len,
                                          int num_heads, int head_dim, int max_blocks_per_seq,
                                          int64_t num_blocks, int block_size, int max_seq_len,
                                          int window_size, void* out, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  return memopt_paged_attention_f16_ex(query, key_pool, value_pool, block_tables, context_lens, batch, q_len,
                                       num_heads, num_heads, head_dim, max_blocks_per_seq, num_blocks, block_size,
                                       max_seq_len, window_size, 0, out, workspace, workspace_bytes, stream);
}

extern "C" int memopt_paged_attention_int4_ex(const void* query, const uint8_t* kv_pages,
                                              const int32_t* block_tables, const int32_t* context_lens,
                                              int batch, int q_len, int num_heads, int num_kv_heads,
                                              int head_dim, int max_blocks_per_seq, int64_t num_blocks,
                                              int block_size, int max_seq_len, int window_size, int causal,
                                              void* out, void* workspace, size_t workspace_bytes,
                                              void* stream) {
  Params p{};
  int st = common_setup(p, query, block_tables, context_lens, batch, q_len, num_heads, num_kv_heads, head_dim,
                        max_blocks_per_seq, num_blocks, block_size, max_seq_len, window_size, causal, true, out,
                        workspace, workspace_bytes);
  if (st != MEMOPT_OK) return st;
  if (p.total_items == 0) return MEMOPT_OK;
  if (num_blocks == 0 || max_blocks_per_seq == 0)
    return zero_output(out, batch, q_len, num_heads, head_dim, stream);
  if (reinterpret_cast<uintptr_t>(kv_pages) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, "dynamic_sparse_attention_int4: pages must be 16-byte aligned");
  p.pages = kv_pages;
  if (use_prefill_int4(q_len, head_dim, block_size)) {
    // The fp16 page scratch follows the split workspace (whose tickets stay zero).
    const size_t off = align256(memopt_paged_attention_workspace_size_ex(
        batch, q_len, num_heads, num_kv_heads, head_dim, max_blocks_per_seq, block_size, max_seq_len, window_size));
    if (workspace == nullptr || workspace_bytes < off)
      return fail(MEMOPT_ERR_WORKSPACE, "dynamic_sparse_attention_int4: workspace too small (size it with "
                                        "memopt_paged_attention_int4_workspace_size_ex)");
    return prefill_int4(query, kv_pages, block_tables, context_lens, batch, q_len, num_heads, num_kv_heads, head_dim,
                        max_blocks_per_seq, num_blocks, block_size, p.window, causal, out,
                        static_cast<uint8_t*>(workspace) + off, workspace_bytes - off, as_stream(stream));
  }
  if (use_mq(true, q_len, num_heads, num_kv_heads, head_dim, block_size))
    return run_mq(p, nullptr, kv_pages, head_dim, block_size, workspace, workspace_bytes, as_stream(stream));
  alignas(64) CUtensorMap dummy;
  std::memset(&dummy, 0, sizeof(dummy));
  return dispatch<true>(p, head_dim, block_size, dummy, dummy, nullptr, as_stream(stream));
}

extern "C" int memopt_paged_attention_int4(const void* query, const uint8_t* kv_pages,
                                           const int32_t* block_tables, const int32_t* context_lens,
                                           int batch, int q_len, int num_heads, int head_dim,
                                           int max_blocks_per_seq, int64_t num_blocks, int block_size,
                                           int max_seq_len, int window_size, void* out, void* workspace,
                                           size_t workspace_bytes, void* stream) {
  return memopt_paged_attention_int4_ex(query, kv_pages, block_tables, context_lens, batch, q_len, num_heads,
                                        num_heads, head_dim, max_blocks_per_seq, num_blocks, block_size,
                                        max_seq_len, window_size, 0, out, workspace, workspace_bytes, stream);
}
