// memopt_C.cpp — the Python module `memopt_C`, a thin PyTorch wrapper over the
// C-ABI in memopt_b200.h.
//
// Mirrors the reference binding src/csrc/extension.cpp:10-124 (same function
// names, argument names, defaults and RuntimeError behaviour), plus:
//   * get_key_pool / get_value_pool, which the reference's DynamicAttention
//     calls (src/memopt/attention.py:330-331) but the reference never exported;
//   * an INT4 page pool (init_pool(..., kv_format="int4")) fed by write_cache
//     with on-the-fly quantisation, read by dynamic_sparse_attention_int4
//     (one [K codes | V codes | K scales | V scales] page per (block, head));
//   * optional compaction outputs of evict_tokens.
// The pool tensors are allocated here (caching allocator, zero filled as in
// kv_cache.cu:135-141); the free-list lives in the C library.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "memopt_b200.h"

namespace {

struct Pool {
  std::mutex mu;
  bool int4 = false;
  torch::Tensor k, v;            // fp16 [NB, BS, H, D]
  torch::Tensor kvp;             // int4 pages uint8 [NB, H, page_bytes]
  int nb = 0, bs = 0, h = 0, d = 0;
  bool live = false;
};
Pool& P() {
  static Pool p;
  return p;
}

void check(int st, const char* what) {
  if (st != MEMOPT_OK) {
    TORCH_CHECK(false, what, ": ", memopt_last_error(), " (", memopt_status_string(st), ")");
  }
}

void* cur_stream() { return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream().stream()); }

bool aligned16(const torch::Tensor& t) { return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0; }

torch::Tensor aligned_contig(const torch::Tensor& t) {
  auto c = t.contiguous();
  if (c.numel() > 0 && !aligned16(c)) c = c.clone();
  return c;
}

void require_pool(const char* who) {
  TORCH_CHECK(P().live && memopt_pool_is_initialized(), who, ": pool not initialized; call init_pool first");
}

}  // namespace

std::string get_hello() { return "MemOpt C++ Backend Initialized (B200 sm_100a data plane)."; }

void init_pool(int num_blocks, int block_size, int num_heads, int head_dim, const std::string& kv_format) {
  auto& p = P();
  std::lock_guard<std::mutex> lk(p.mu);
  TORCH_CHECK(kv_format == "fp16" || kv_format == "int4", "init_pool: kv_format must be 'fp16' or 'int4'");
  const bool int4 = kv_format == "int4";
  if (p.live && memopt_pool_is_initialized() && p.nb == num_blocks && p.bs == block_size &&
      p.h == num_heads && p.d == head_dim && p.int4 == int4)
    return;  // idempotent (kv_cache.cu:116-122)
  // Any other call resets first, so a rejected geometry leaves no pool behind.
  p.live = false;
  p.k = p.v = p.kvp = torch::Tensor();
  memopt_pool_reset();
  check(memopt_pool_init(num_blocks, block_size, num_heads, head_dim), "init_pool");
  if (int4 && (head_dim % 64 != 0 || block_size % 16 != 0)) {
    memopt_pool_reset();
    TORCH_CHECK(false, "init_pool: kv_format='int4' needs head_dim % 64 == 0 and block_size % 16 == 0");
  }
  auto dev = torch::Device(torch::kCUDA, c10::cuda::current_device());
  if (!int4) {
    auto o = torch::TensorOptions().dtype(torch::kFloat16).device(dev);
    p.k = torch::zeros({num_blocks, block_size, num_heads, head_dim}, o);
    p.v = torch::zeros({num_blocks, block_size, num_heads, head_dim}, o);
  } else {
    auto ou = torch::TensorOptions().dtype(torch::kUInt8).device(dev);
    const int64_t pb = static_cast<int64_t>(memopt_int4_page_bytes(block_size, head_dim));
    p.kvp = torch::zeros({num_blocks, num_heads, pb}, ou);
  }
  p.nb = num_blocks;
  p.bs = block_size;
  p.h = num_heads;
  p.d = head_dim;
  p.int4 = int4;
  p.live = true;
}

int allocate_block() {
  const int r = memopt_pool_allocate_block();
  TORCH_CHECK(r != MEMOPT_ERR_NOT_INITIALIZED, "allocate_block: pool not initialized");
  return r;
}

void free_block(int block_idx) { check(memopt_pool_free_block(block_idx), "free_block"); }

int free_blocks_count() { return memopt_pool_free_blocks_count(); }

namespace {
// Strided views of the four regions of every INT4 page in stored order (the
// layout is documented at memopt_write_cache_int4 in memopt_b200.h).
std::vector<torch::Tensor> int4_views(const torch::Tensor& kvp, int bs, int d) {
  const int64_t nb = kvp.size(0), h = kvp.size(1), pb = kvp.size(2), g = d / 64;
  const int64_t codes = static_cast<int64_t>(bs) * (d / 2);
  auto kc = kvp.as_strided({nb, h, bs, d / 2}, {h * pb, pb, d / 2, 1}, kvp.storage_offset());
  auto vc = kvp.as_strided({nb, h, bs, d / 2}, {h * pb, pb, d / 2, 1}, kvp.storage_offset() + codes);
  auto k16 = kvp.view(torch::kFloat16);  // [nb, h, pb / 2]
  auto ks = k16.as_strided({nb, h, bs, g}, {h * pb / 2, pb / 2, g, 1}, k16.storage_offset() + codes);
  // V scales are stored per 16-token tile as [G][16] in a permuted token order.
  auto vs = k16.as_strided({nb, h, bs / 16, g, 16}, {h * pb / 2, pb / 2, g * 16, 16, 1},
                           k16.storage_offset() + codes + bs * g);
  return {kc, ks, vc, vs};
}
}  // namespace

std::pair<torch::Tensor, torch::Tensor> get_pool_tensors() {
  require_pool("get_pool_tensors");
  auto& p = P();
  if (p.int4) {
    auto v = int4_views(p.kvp, p.bs, p.d);
    return {v[0], v[2]};
  }
  return {p.k, p.v};
}
torch::Tensor get_key_pool() { return get_pool_tensors().first; }
torch::Tensor get_value_pool() { return get_pool_tensors().second; }

std::vector<torch::Tensor> get_int4_pool_tensors() {
  require_pool("get_int4_pool_tensors");
  auto& p = P();
  TORCH_CHECK(p.int4, "get_int4_pool_tensors: pool was initialised with kv_format='fp16'");
  return int4_views(p.kvp, p.bs, p.d);
}

torch::Tensor get_int4_pages() {
  require_pool("get_int4_pages");
  auto& p = P();
  TORCH_CHECK(p.int4, "get_int4_pages: pool was initialised with kv_format='fp16'");
  return p.kvp;
}

std::string pool_format() {
  require_pool("pool_format");
  return P().int4 ? "int4" : "fp16";
}

void write_cache(torch::Tensor keys, torch::Tensor values, torch::Tensor block_tables,
                 torch::Tensor slot_mapping) {
  (void)block_tables;  // accepted for API symmetry, as in kv_cache.cu:279-280
  require_pool("write_cache");
  auto& p = P();
  TORCH_CHECK(keys.dim() == 3, "write_cache: keys must be 3-D [num_tokens, num_heads, head_dim]");
  TORCH_CHECK(values.dim() == 3, "write_cache: values must be 3-D [num_tokens, num_heads, head_dim]");
  TORCH_CHECK(slot_mapping.dim() == 1, "write_cache: slot_mapping must be 1-D [num_tokens]");
  const int64_t T = keys.size(0);
  const int H = static_cast<int>(keys.size(1));
  const int D = static_cast<int>(keys.size(2));
  TORCH_CHECK(values.size(0) == T, "write_cache: keys/values token count mismatch");
  TORCH_CHECK(values.size(1) == H, "write_cache: keys/values num_heads mismatch");
  TORCH_CHECK(values.size(2) == D, "write_cache: keys/values head_dim mismatch");
  TORCH_CHECK(slot_mapping.size(0) == T, "write_cache: slot_mapping length != num_tokens");
  TORCH_CHECK(H == p.h, "write_cache: num_heads != pool.num_heads");
  TORCH_CHECK(D == p.d, "write_cache: head_dim != pool.head_dim");
  TORCH_CHECK(keys.scalar_type() == torch::kFloat16 && values.scalar_type() == torch::kFloat16,
              "write_cache: keys/values must be float16 (the pool dtype)");
  TORCH_CHECK(slot_mapping.scalar_type() == torch::kInt32, "write_cache: slot_mapping must be int32");
  TORCH_CHECK(keys.is_cuda() && values.is_cuda() && slot_mapping.is_cuda(),
              "write_cache: inputs must be CUDA tensors");
  if (T == 0) return;
  keys = aligned_contig(keys);
  values = aligned_contig(values);
  slot_mapping = slot_mapping.contiguous();
  const at::cuda::CUDAGuard g(keys.device());
  // MEMOPT_DEBUG_BOUNDS=1: count skipped out-of-range slots and raise (one
  // host sync per call).  Otherwise such tokens are skipped silently.
  static const bool debug = [] {
    const char* e = std::getenv("MEMOPT_DEBUG_BOUNDS");
    return e != nullptr && e[0] == '1';
  }();
  torch::Tensor bad;
  int32_t* badp = nullptr;
  if (debug) {
    bad = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(keys.device()));
    badp = bad.data_ptr<int32_t>();
  }
  int st;
  if (!p.int4) {
    st = memopt_write_cache_f16(keys.data_ptr(), values.data_ptr(), slot_mapping.data_ptr<int32_t>(), T, H,
                                D, p.k.data_ptr(), p.v.data_ptr(), p.nb, p.bs, badp, cur_stream());
  } else {
    st = memopt_write_cache_int4(keys.data_ptr(), values.data_ptr(), slot_mapping.data_ptr<int32_t>(), T, H,
                                 D, p.kvp.data_ptr<uint8_t>(), p.nb, p.bs, badp, cur_stream());
  }
  check(st, "write_cache");
  if (debug) {
    const int n = bad.item<int32_t>();
    TORCH_CHECK(n == 0, "write_cache: ", n, " slot_mapping entries out of bounds (skipped)");
  }
}

void evict_cache(torch::Tensor block_tables, torch::Tensor attention_scores, float retain_ratio,
                 int num_sink_tokens) {
  (void)block_tables;     // operates pool-wide (kv_cache.cu:493-496)
  (void)num_sink_tokens;  // ignored by the reference kernel (kv_cache.cu:390)
  TORCH_CHECK(P().live && memopt_pool_is_initialized(), "evict_cache: pool not initialized");
  auto& p = P();
  TORCH_CHECK(retain_ratio > 0.f && retain_ratio <= 1.f, "evict_cache: retain_ratio must be in (0, 1]");
  TORCH_CHECK(attention_scores.dim() == 3,
              "evict_cache: attention_scores must be 3-D [num_blocks, block_size, num_heads]");
  TORCH_CHECK(attention_scores.scalar_type() == torch::kFloat32, "evict_cache: attention_scores must be float32");
  TORCH_CHECK(!p.int4, "evict_cache: not supported on an int4 pool");
  const int nb = static_cast<int>(attention_scores.size(0));
  const int bs = static_cast<int>(attention_scores.size(1));
  const int h = static_cast<int>(attention_scores.size(2));
  TORCH_CHECK(nb <= p.nb, "evict_cache: attention_scores num_blocks > pool.num_blocks");
  TORCH_CHECK(bs == p.bs, "evict_cache: attention_scores block_size != pool.block_size");
  TORCH_CHECK(h == p.h, "evict_cache: attention_scores num_heads != pool.num_heads");
  TORCH_CHECK(attention_scores.is_cuda(), "evict_cache: attention_scores must be a CUDA tensor");
  attention_scores = attention_scores.contiguous();
  if (nb == 0) return;
  const at::cuda::CUDAGuard g(attention_scores.device());
  check(memopt_evict_cache(attention_scores.data_ptr<float>(), nb, bs, h, p.d, p.k.data_ptr(), p.v.data_ptr(),
                           retain_ratio, cur_stream()),
        "evict_cache");
}

pybind11::object evict_tokens(torch::Tensor attention_scores, torch::Tensor block_tables,
                              torch::Tensor is_block_free, float retain_ratio, int num_sink_tokens,
                              bool return_retained) {
  TORCH_CHECK(P().live && memopt_pool_is_initialized(), "evict_tokens: pool not initialized");
  auto& p = P();
  TORCH_CHECK(retain_ratio > 0.f && retain_ratio <= 1.f, "evict_tokens: retain_ratio must be in (0, 1]");
  TORCH_CHECK(attention_scores.dim() == 3,
              "evict_tokens: attention_scores must be 3-D [num_seqs, num_heads, seq_len]");
  TORCH_CHECK(attention_scores.scalar_type() == torch::kFloat32, "evict_tokens: attention_scores must be float32");
  TORCH_CHECK(block_tables.dim() == 2, "evict_tokens: block_tables must be 2-D [num_seqs, max_blocks_per_seq]");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt32, "evict_tokens: block_tables must be int32");
  TORCH_CHECK(is_block_free.dim() == 1, "evict_tokens: is_block_free must be 1-D [total_pool_blocks]");
  TORCH_CHECK(is_block_free.scalar_type() == torch::kInt32, "evict_tokens: is_block_free must be int32");
  TORCH_CHECK(!p.int4, "evict_tokens: not supported on an int4 pool");
  const int S = static_cast<int>(attention_scores.size(0));
  const int H = static_cast<int>(attention_scores.size(1));
  const int L = static_cast<int>(attention_scores.size(2));
  const int MB = static_cast<int>(block_tables.size(1));
  const int NBF = static_cast<int>(is_block_free.size(0));
  TORCH_CHECK(L <= 32768, "evict_tokens: seq_len exceeds the maximum (32768)");
  TORCH_CHECK(H == p.h, "evict_tokens: attention_scores num_heads != pool.num_heads");
  TORCH_CHECK(block_tables.size(0) == S, "evict_tokens: block_tables batch size != num_seqs");
  TORCH_CHECK(NBF <= p.nb, "evict_tokens: is_block_free size > pool.num_blocks");
  TORCH_CHECK(attention_scores.is_cuda() && block_tables.is_cuda() && is_block_free.is_cuda(),
              "evict_tokens: inputs must be CUDA tensors");
  torch::Tensor idx, cnt;
  if (return_retained) {
    auto o = torch::TensorOptions().dtype(torch::kInt32).device(attention_scores.device());
    // The kernel writes every element (kept indices, then -1 padding).
    idx = (S == 0 || L == 0) ? torch::full({S, H, L}, -1, o) : torch::empty({S, H, L}, o);
    cnt = (S == 0 || L == 0) ? torch::zeros({S, H}, o) : torch::empty({S, H}, o);
  }
  if (S == 0 || L == 0) {
    if (return_retained) return pybind11::make_tuple(idx, cnt);
    return pybind11::none();
  }
  // As in kv_cache.cu:1096-1098, non-contiguous tables are copied and the
  // mutation is applied to the copy.
  attention_scores = attention_scores.contiguous();
  block_tables = block_tables.contiguous();
  is_block_free = is_block_free.contiguous();
  const at::cuda::CUDAGuard g(attention_scores.device());
  check(memopt_evict_tokens(attention_scores.data_ptr<float>(), S, H, L, block_tables.data_ptr<int32_t>(), MB,
                            is_block_free.data_ptr<int32_t>(), NBF, p.k.data_ptr(), p.v.data_ptr(), p.nb, p.bs,
                            p.d, retain_ratio, num_sink_tokens,
                            return_retained ? idx.data_ptr<int32_t>() : nullptr,
                            return_retained ? cnt.data_ptr<int32_t>() : nullptr, cur_stream()),
        "evict_tokens");
  if (return_retained) return pybind11::make_tuple(idx, cnt);
  return pybind11::none();
}

// Exact top-k eviction with compaction (new operator; see memopt_b200.h).
// block_tables and context_lens must be contiguous CUDA int32 tensors: they
// are updated in place.  Returns (kept_idx [S, L], kept_count [S],
// freed_pages [S, MB], freed_count [S]).
pybind11::tuple evict_topk_compact(torch::Tensor attention_scores, torch::Tensor block_tables,
                                   torch::Tensor context_lens, float retain_ratio, int num_sink_tokens) {
  TORCH_CHECK(P().live && memopt_pool_is_initialized(), "evict_topk_compact: pool not initialized");
  auto& p = P();
  TORCH_CHECK(attention_scores.dim() == 3 && attention_scores.scalar_type() == torch::kFloat32,
              "evict_topk_compact: attention_scores must be float32 [num_seqs, num_heads, max_len]");
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.scalar_type() == torch::kInt32 && block_tables.is_contiguous(),
              "evict_topk_compact: block_tables must be a contiguous int32 [num_seqs, max_blocks_per_seq] tensor");
  TORCH_CHECK(context_lens.dim() == 1 && context_lens.scalar_type() == torch::kInt32 && context_lens.is_contiguous(),
              "evict_topk_compact: context_lens must be a contiguous int32 [num_seqs] tensor");
  TORCH_CHECK(attention_scores.is_cuda() && block_tables.is_cuda() && context_lens.is_cuda(),
              "evict_topk_compact: inputs must be CUDA tensors");
  const int S = static_cast<int>(attention_scores.size(0));
  const int H = static_cast<int>(attention_scores.size(1));
  const int L = static_cast<int>(attention_scores.size(2));
  const int MB = static_cast<int>(block_tables.size(1));
  TORCH_CHECK(H == p.h, "evict_topk_compact: num_heads != pool.num_heads");
  TORCH_CHECK(block_tables.size(0) == S && context_lens.size(0) == S, "evict_topk_compact: batch size mismatch");
  auto o = torch::TensorOptions().dtype(torch::kInt32).device(attention_scores.device());
  auto kept = torch::full({S, L}, -1, o);
  auto cnt = torch::zeros({S}, o);
  auto freed = torch::full({S, MB}, -1, o);
  auto fcnt = torch::zeros({S}, o);
  if (S == 0 || L == 0) return pybind11::make_tuple(kept, cnt, freed, fcnt);
  attention_scores = attention_scores.contiguous();
  const at::cuda::CUDAGuard g(attention_scores.device());
  const size_t wsb = memopt_evict_topk_workspace_size(S, L, H, p.d);
  auto ws = torch::empty({static_cast<int64_t>(wsb)}, o.dtype(torch::kUInt8));
  if (p.int4) {
    check(memopt_evict_topk_compact_int4(attention_scores.data_ptr<float>(), S, H, L, block_tables.data_ptr<int32_t>(),
                                         MB, context_lens.data_ptr<int32_t>(), p.kvp.data_ptr<uint8_t>(), p.nb, p.bs,
                                         p.d, retain_ratio, num_sink_tokens, kept.data_ptr<int32_t>(),
                                         cnt.data_ptr<int32_t>(), freed.data_ptr<int32_t>(), fcnt.data_ptr<int32_t>(),
                                         ws.data_ptr(), wsb, cur_stream()),
          "evict_topk_compact");
  } else {
    check(memopt_evict_topk_compact(attention_scores.data_ptr<float>(), S, H, L, block_tables.data_ptr<int32_t>(), MB,
                                    context_lens.data_ptr<int32_t>(), p.k.data_ptr(), p.v.data_ptr(), p.nb, p.bs, p.d,
                                    retain_ratio, num_sink_tokens, kept.data_ptr<int32_t>(), cnt.data_ptr<int32_t>(),
                                    freed.data_ptr<int32_t>(), fcnt.data_ptr<int32_t>(), ws.data_ptr(), wsb,
                                    cur_stream()),
          "evict_topk_compact");
  }
  // Synchronises: a row move whose bounded wait ran out is an error here.
  check(memopt_evict_topk_status(ws.data_ptr(), S, L, cur_stream()), "evict_topk_compact");
  return pybind11::make_tuple(kept, cnt, freed, fcnt);
}

// Head-sharded exact eviction, step 1: this rank's partial token scores
// (fp32 sum of its heads, in order), float32 [num_seqs, max_len].
torch::Tensor evict_topk_head_sum(torch::Tensor attention_scores) {
  TORCH_CHECK(attention_scores.is_cuda() && attention_scores.dim() == 3 &&
                  attention_scores.scalar_type() == torch::kFloat32,
              "evict_topk_head_sum: attention_scores must be a CUDA float32 [num_seqs, num_heads, max_len] tensor");
  attention_scores = attention_scores.contiguous();
  const int S = static_cast<int>(attention_scores.size(0));
  const int H = static_cast<int>(attention_scores.size(1));
  const int L = static_cast<int>(attention_scores.size(2));
  TORCH_CHECK(H > 0, "evict_topk_head_sum: no heads");
  const at::cuda::CUDAGuard g(attention_scores.device());
  auto sums = torch::empty({S, L}, attention_scores.options());
  check(memopt_evict_topk_head_sum(attention_scores.data_ptr<float>(), S, H, L, sums.data_ptr<float>(),
                                   cur_stream()),
        "evict_topk_head_sum");
  return sums;
}

// Head-sharded exact eviction, step 2: partial_sums float32 [G, num_seqs,
// max_len] (every rank's evict_topk_head_sum, in rank order) decide; this
// rank's pool (its heads) is compacted.  Same outputs and in-place updates as
// evict_topk_compact.
pybind11::tuple evict_topk_compact_parts(torch::Tensor partial_sums, torch::Tensor block_tables,
                                         torch::Tensor context_lens, float retain_ratio, int num_sink_tokens) {
  TORCH_CHECK(P().live && memopt_pool_is_initialized(), "evict_topk_compact_parts: pool not initialized");
  auto& p = P();
  TORCH_CHECK(!p.int4, "evict_topk_compact_parts: needs the fp16 pool");
  TORCH_CHECK(partial_sums.dim() == 3 && partial_sums.scalar_type() == torch::kFloat32,
              "evict_topk_compact_parts: partial_sums must be float32 [num_parts, num_seqs, max_len]");
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.scalar_type() == torch::kInt32 && block_tables.is_contiguous(),
              "evict_topk_compact_parts: block_tables must be a contiguous int32 [num_seqs, max_blocks_per_seq] "
              "tensor");
  TORCH_CHECK(context_lens.dim() == 1 && context_lens.scalar_type() == torch::kInt32 && context_lens.is_contiguous(),
              "evict_topk_compact_parts: context_lens must be a contiguous int32 [num_seqs] tensor");
  TORCH_CHECK(partial_sums.is_cuda() && block_tables.is_cuda() && context_lens.is_cuda(),
              "evict_topk_compact_parts: inputs must be CUDA tensors");
  const int G = static_cast<int>(partial_sums.size(0));
  const int S = static_cast<int>(partial_sums.size(1));
  const int L = static_cast<int>(partial_sums.size(2));
  const int MB = static_cast<int>(block_tables.size(1));
  TORCH_CHECK(G > 0, "evict_topk_compact_parts: no parts");
  TORCH_CHECK(block_tables.size(0) == S && context_lens.size(0) == S,
              "evict_topk_compact_parts: batch size mismatch");
  auto o = torch::TensorOptions().dtype(torch::kInt32).device(partial_sums.device());
  auto kept = torch::full({S, L}, -1, o);
  auto cnt = torch::zeros({S}, o);
  auto freed = torch::full({S, MB}, -1, o);
  auto fcnt = torch::zeros({S}, o);
  if (S == 0 || L == 0) return pybind11::make_tuple(kept, cnt, freed, fcnt);
  partial_sums = partial_sums.contiguous();
  const at::cuda::CUDAGuard g(partial_sums.device());
  const size_t wsb = memopt_evict_topk_workspace_size(S, L, p.h, p.d);
  auto ws = torch::empty({static_cast<int64_t>(wsb)}, o.dtype(torch::kUInt8));
  check(memopt_evict_topk_compact_parts(partial_sums.data_ptr<float>(), G, S, L, block_tables.data_ptr<int32_t>(),
                                        MB, context_lens.data_ptr<int32_t>(), p.k.data_ptr(), p.v.data_ptr(), p.nb,
                                        p.bs, p.h, p.d, retain_ratio, num_sink_tokens, kept.data_ptr<int32_t>(),
                                        cnt.data_ptr<int32_t>(), freed.data_ptr<int32_t>(),
                                        fcnt.data_ptr<int32_t>(), ws.data_ptr(), wsb, cur_stream()),
        "evict_topk_compact_parts");
  check(memopt_evict_topk_status(ws.data_ptr(), S, L, cur_stream()), "evict_topk_compact_parts");
  return pybind11::make_tuple(kept, cnt, freed, fcnt);
}

namespace {

void attn_checks(const torch::Tensor& query, const torch::Tensor& block_tables, const torch::Tensor& context_lens) {
  TORCH_CHECK(query.is_cuda(), "query must be a CUDA tensor");
  TORCH_CHECK(block_tables.is_cuda(), "block_tables must be a CUDA tensor");
  TORCH_CHECK(context_lens.is_cuda(), "context_lens must be a CUDA tensor");
  TORCH_CHECK(query.dim() == 4, "query must be 4-D [batch, q_len, num_heads, head_dim]");
  TORCH_CHECK(block_tables.dim() == 2, "block_tables must be 2-D [batch, max_blocks_per_seq]");
  TORCH_CHECK(context_lens.dim() == 1, "context_lens must be 1-D [batch]");
  TORCH_CHECK(query.scalar_type() == torch::kFloat16, "query must be fp16");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt32, "block_tables must be int32");
  TORCH_CHECK(context_lens.scalar_type() == torch::kInt32, "context_lens must be int32");
  TORCH_CHECK(query.is_contiguous(), "query must be contiguous");
  TORCH_CHECK(block_tables.is_contiguous(), "block_tables must be contiguous");
  TORCH_CHECK(context_lens.is_contiguous(), "context_lens must be contiguous");
  TORCH_CHECK(block_tables.size(0) == query.size(0), "block_tables batch dimension mismatch");
  TORCH_CHECK(context_lens.size(0) == query.size(0), "context_lens batch dimension mismatch");
  TORCH_CHECK(query.size(3) <= 128, "head_dim ", query.size(3), " must be <= ATTN_BLOCK_DIM (128)");
}

// Split-K scratch, cached per (device, stream) so that a decode step does no
// allocation and no clearing: the kernels leave the ticket prefix of the
// workspace zero when they finish, so it is cleared only when the buffer is
// new or when a call needs more ticket bytes than the previous call on that
// stream left zero (the previous call's partials follow its own tickets).
// Calls on one stream are ordered, so they can share the buffer; a failed
// call drops the entry (its tickets may not have been reset).
struct WsEntry {
  torch::Tensor buf;
  size_t zero_tickets = 0;  // bytes at the start known to be zero
};
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, WsEntry> g_ws;

torch::Tensor attn_workspace(const torch::Tensor& query, int KVH, int MB, int BS, int max_seq_len,
                             int window_size, size_t* bytes, bool int4 = false) {
  const int B = static_cast<int>(query.size(0)), QL = static_cast<int>(query.size(1));
  const int H = static_cast<int>(query.size(2)), D = static_cast<int>(query.size(3));
  *bytes = int4 ? memopt_paged_attention_int4_workspace_size_ex(B, QL, H, KVH, D, MB, BS, max_seq_len, window_size)
                : memopt_paged_attention_workspace_size_ex(B, QL, H, KVH, D, MB, BS, max_seq_len, window_size);
  if (*bytes == 0) return torch::Tensor();
  const size_t tb = memopt_paged_attention_ticket_bytes(B, QL, H);
  cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
  std::lock_guard<std::mutex> lk(g_ws_mu);
  WsEntry& e = g_ws[{static_cast<int>(query.get_device()), st}];
  if (!e.buf.defined() || static_cast<size_t>(e.buf.numel()) < *bytes) {
    e.buf = torch::empty({static_cast<int64_t>(*bytes)},
                         torch::TensorOptions().dtype(torch::kUInt8).device(query.device()));
    e.zero_tickets = 0;
  }
  if (tb > e.zero_tickets) C10_CUDA_CHECK(cudaMemsetAsync(e.buf.data_ptr(), 0, tb, st));
  e.zero_tickets = tb;
  return e.buf;
}

void drop_workspace(const torch::Tensor& query) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  g_ws.erase({static_cast<int>(query.get_device()), at::cuda::getCurrentCUDAStream().stream()});
}

// Attention status check that forgets the stream's cached workspace first.
void check_attn(int st, const char* what, const torch::Tensor& query) {
  if (st != MEMOPT_OK) drop_workspace(query);
  check(st, what);
}

}  // namespace

// Additions beyond the reference: the pool may hold fewer heads than the
// query (grouped-query attention: query head h reads pool head h / (H / KVH))
// and causal=True makes query row i the token at context_len - q_len + i.
torch::Tensor dynamic_sparse_attention(torch::Tensor query, torch::Tensor key_cache, torch::Tensor value_cache,
                                       torch::Tensor block_tables, torch::Tensor context_lens, int max_seq_len,
                                       int window_size, bool causal) {
  attn_checks(query, block_tables, context_lens);
  TORCH_CHECK(key_cache.is_cuda(), "key_cache must be a CUDA tensor");
  TORCH_CHECK(value_cache.is_cuda(), "value_cache must be a CUDA tensor");
  TORCH_CHECK(key_cache.dim() == 4, "key_cache must be 4-D [num_kv_blocks, block_size, num_heads, head_dim]");
  TORCH_CHECK(value_cache.dim() == 4, "value_cache must be 4-D [num_kv_blocks, block_size, num_heads, head_dim]");
  TORCH_CHECK(key_cache.scalar_type() == torch::kFloat16, "key_cache must be fp16");
  TORCH_CHECK(value_cache.scalar_type() == torch::kFloat16, "value_cache must be fp16");
  TORCH_CHECK(key_cache.is_contiguous(), "key_cache must be contiguous");
  TORCH_CHECK(value_cache.is_contiguous(), "value_cache must be contiguous");
  const int B = static_cast<int>(query.size(0)), QL = static_cast<int>(query.size(1));
  const int H = static_cast<int>(query.size(2)), D = static_cast<int>(query.size(3));
  const int BS = static_cast<int>(key_cache.size(1));
  const int MB = static_cast<int>(block_tables.size(1));
  const int KVH = static_cast<int>(key_cache.size(2));
  TORCH_CHECK(KVH > 0 && H % KVH == 0, "key_cache num_heads ", KVH, " does not divide query num_heads ", H);
  TORCH_CHECK(key_cache.size(3) == D, "key_cache head_dim ", key_cache.size(3), " != query head_dim ", D);
  TORCH_CHECK(value_cache.size(0) == key_cache.size(0), "value_cache num_kv_blocks mismatch");
  TORCH_CHECK(value_cache.size(1) == BS, "value_cache block_size mismatch");
  TORCH_CHECK(value_cache.size(2) == KVH, "value_cache num_heads mismatch");
  TORCH_CHECK(value_cache.size(3) == D, "value_cache head_dim mismatch");
  auto out = torch::empty_like(query);
  if (B == 0 || QL == 0 || H == 0 || D == 0) return out;
  const at::cuda::CUDAGuard g(query.device());
  auto q = aligned_contig(query);
  size_t wsb = 0;
  auto ws = attn_workspace(q, KVH, MB, BS, max_seq_len, window_size, &wsb);
  check_attn(memopt_paged_attention_f16_ex(q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
                                      block_tables.data_ptr<int32_t>(), context_lens.data_ptr<int32_t>(), B, QL, H,
                                      KVH, D, MB, key_cache.size(0), BS, max_seq_len, window_size, causal ? 1 : 0,
                                      out.data_ptr(), wsb ? ws.data_ptr() : nullptr, wsb, cur_stream()),
             "dynamic_sparse_attention", q);
  return out;
}

torch::Tensor dynamic_sparse_attention_int4(torch::Tensor query, torch::Tensor kv_pages, torch::Tensor block_tables,
                                            torch::Tensor context_lens, int max_seq_len, int window_size,
                                            bool causal) {
  attn_checks(query, block_tables, context_lens);
  TORCH_CHECK(kv_pages.is_cuda() && kv_pages.dim() == 3 && kv_pages.scalar_type() == torch::kUInt8 &&
                  kv_pages.is_contiguous(),
              "kv_pages must be a contiguous CUDA uint8 tensor [num_blocks, num_heads, page_bytes]");
  const int B = static_cast<int>(query.size(0)), QL = static_cast<int>(query.size(1));
  const int H = static_cast<int>(query.size(2)), D = static_cast<int>(query.size(3));
  const int KVH = static_cast<int>(kv_pages.size(1));
  TORCH_CHECK(KVH > 0 && H % KVH == 0, "kv_pages num_heads ", KVH, " does not divide query num_heads ", H);
  TORCH_CHECK(D % 64 == 0, "dynamic_sparse_attention_int4: head_dim must be a multiple of 64");
  const int64_t per_token = D + 4 * (D / 64);
  TORCH_CHECK(kv_pages.size(2) % per_token == 0, "kv_pages page_bytes ", kv_pages.size(2),
              " is not a whole number of tokens for head_dim ", D);
  const int BS = static_cast<int>(kv_pages.size(2) / per_token);
  const int MB = static_cast<int>(block_tables.size(1));
  auto out = torch::empty_like(query);
  if (B == 0 || QL == 0 || H == 0 || D == 0) return out;
  const at::cuda::CUDAGuard g(query.device());
  auto q = aligned_contig(query);
  size_t wsb = 0;
  auto ws = attn_workspace(q, KVH, MB, BS, max_seq_len, window_size, &wsb, true);
  check_attn(memopt_paged_attention_int4_ex(q.data_ptr(), kv_pages.data_ptr<uint8_t>(), block_tables.data_ptr<int32_t>(),
                                       context_lens.data_ptr<int32_t>(), B, QL, H, KVH, D, MB, kv_pages.size(0), BS,
                                       max_seq_len, window_size, causal ? 1 : 0, out.data_ptr(),
                                       wsb ? ws.data_ptr() : nullptr, wsb, cur_stream()),
             "dynamic_sparse_attention_int4", q);
  return out;
}

std::vector<torch::Tensor> quantize_kv_cache_int4(torch::Tensor cache, int group_size) {
  TORCH_CHECK(cache.is_cuda(), "quantize_kv_cache_int4: cache must be a CUDA tensor");
  TORCH_CHECK(cache.is_contiguous(), "quantize_kv_cache_int4: cache must be contiguous");
  TORCH_CHECK(cache.scalar_type() == torch::kFloat16, "quantize_kv_cache_int4: cache must be float16");
  TORCH_CHECK(group_size == 64, "quantize_kv_cache_int4: group_size must equal 64 (got ", group_size, ")");
  const int64_t n = cache.numel();
  TORCH_CHECK(n % group_size == 0, "quantize_kv_cache_int4: total_elements (", n,
              ") must be divisible by group_size (", group_size, ")");
  TORCH_CHECK(cache.dim() >= 1, "quantize_kv_cache_int4: cache must have at least one dimension");
  const int64_t last = cache.size(cache.dim() - 1);
  TORCH_CHECK(last % 2 == 0, "quantize_kv_cache_int4: last dimension (", last, ") must be even for INT4 packing");
  auto sizes = cache.sizes().vec();
  sizes.back() /= 2;
  auto packed = torch::empty(sizes, torch::TensorOptions().dtype(torch::kUInt8).device(cache.device()));
  auto scales = torch::empty({n / group_size}, torch::TensorOptions().dtype(torch::kFloat32).device(cache.device()));
  if (n == 0) return {packed, scales};
  const at::cuda::CUDAGuard g(cache.device());
  auto c = aligned_contig(cache);
  check(memopt_quantize_int4(c.data_ptr(), n, group_size, packed.data_ptr<uint8_t>(), scales.data_ptr<float>(),
                             cur_stream()),
        "quantize_kv_cache_int4");
  return {packed, scales};
}

torch::Tensor dequantize_kv_cache_int4(torch::Tensor q_cache, torch::Tensor scales, int group_size) {
  TORCH_CHECK(q_cache.is_cuda(), "dequantize_kv_cache_int4: q_cache must be a CUDA tensor");
  TORCH_CHECK(scales.is_cuda(), "dequantize_kv_cache_int4: scales must be a CUDA tensor");
  TORCH_CHECK(q_cache.is_contiguous(), "dequantize_kv_cache_int4: q_cache must be contiguous");
  TORCH_CHECK(scales.is_contiguous(), "dequantize_kv_cache_int4: scales must be contiguous");
  TORCH_CHECK(q_cache.scalar_type() == torch::kUInt8, "dequantize_kv_cache_int4: q_cache must be uint8");
  TORCH_CHECK(scales.scalar_type() == torch::kFloat32, "dequantize_kv_cache_int4: scales must be float32");
  TORCH_CHECK(group_size == 64, "dequantize_kv_cache_int4: group_size must equal 64");
  TORCH_CHECK(q_cache.dim() >= 1, "dequantize_kv_cache_int4: q_cache must have at least one dimension");
  auto sizes = q_cache.sizes().vec();
  sizes.back() *= 2;
  const int64_t n = q_cache.numel() * 2;
  const int64_t groups = n / group_size;
  TORCH_CHECK(scales.numel() == groups, "dequantize_kv_cache_int4: scales length (", scales.numel(),
              ") != expected num_groups (", groups, ")");
  // Elements past the last whole group are set to 0 (the reference leaves them unwritten).
  auto opts = torch::TensorOptions().dtype(torch::kFloat16).device(q_cache.device());
  auto out = (n % group_size == 0) ? torch::empty(sizes, opts) : torch::zeros(sizes, opts);
  if (groups == 0) return out;
  const at::cuda::CUDAGuard g(q_cache.device());
  auto qc = q_cache;
  if (reinterpret_cast<uintptr_t>(qc.data_ptr()) & 3u) qc = qc.clone();
  check(memopt_dequantize_int4(qc.data_ptr<uint8_t>(), scales.data_ptr<float>(), groups * group_size, group_size,
                               out.data_ptr(), cur_stream()),
        "dequantize_kv_cache_int4");
  return out;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  m.def("release_workspaces", [] {
    std::lock_guard<std::mutex> lk(g_ws_mu);
    g_ws.clear();
  }, "Drop the split-K workspaces cached per (device, stream) by dynamic_sparse_attention");
  m.def("get_hello", &get_hello, "Initial handshake function for MemOpt C++ extension");
  m.def("init_pool", &init_pool, "Allocate the paged KV cache pool tensors on GPU and seed the free-list",
        py::arg("num_blocks"), py::arg("block_size"), py::arg("num_heads"), py::arg("head_dim"),
        py::arg("kv_format") = std::string("fp16"));
  m.def("allocate_block", &allocate_block, "Pop one free block index from the pool free-list; returns -1 if exhausted");
  m.def("free_block", &free_block, "Return a block index to the pool free-list", py::arg("block_idx"));
  m.def("get_pool_tensors", &get_pool_tensors,
        "Return (key_pool, val_pool) GPU tensors of shape [num_blocks, block_size, num_heads, head_dim]");
  m.def("get_key_pool", &get_key_pool, "Return the key pool tensor");
  m.def("get_value_pool", &get_value_pool, "Return the value pool tensor");
  m.def("get_int4_pool_tensors", &get_int4_pool_tensors,
        "Return strided views [key_codes, key_scales, value_codes, value_scales] of an int4 pool");
  m.def("get_int4_pages", &get_int4_pages, "Return the int4 page tensor [num_blocks, num_heads, page_bytes]");
  m.def("pool_format", &pool_format, "'fp16' or 'int4'");
  m.def("free_blocks_count", &free_blocks_count, "Return the number of free blocks remaining in the pool");
  m.def("write_cache", &write_cache, "Scatter key/value tokens into the paged KV cache pool via slot_mapping",
        py::arg("keys"), py::arg("values"), py::arg("block_tables"), py::arg("slot_mapping"));
  m.def("evict_cache", &evict_cache, "Zero evicted token slots in the pool based on attention score ranking",
        py::arg("block_tables"), py::arg("attention_scores"), py::arg("retain_ratio"),
        py::arg("num_sink_tokens") = 4);
  m.def("evict_tokens", &evict_tokens, "Sequence-centric Ada-KV token eviction with block_table unlinking",
        py::arg("attention_scores"), py::arg("block_tables"), py::arg("is_block_free"), py::arg("retain_ratio"),
        py::arg("num_sink_tokens") = 4, py::arg("return_retained") = false);
  m.def("evict_topk_compact", &evict_topk_compact,
        "Exact sink-aware top-k eviction shared across heads, with compaction of the kept K/V rows",
        py::arg("attention_scores"), py::arg("block_tables"), py::arg("context_lens"), py::arg("retain_ratio"),
        py::arg("num_sink_tokens") = 4);
  m.def("evict_topk_head_sum", &evict_topk_head_sum,
        "Partial token scores of this rank's heads for head-sharded exact eviction", py::arg("attention_scores"));
  m.def("evict_topk_compact_parts", &evict_topk_compact_parts,
        "Exact top-k eviction on the rank-ordered sum of partial token scores, compacting this rank's pool",
        py::arg("partial_sums"), py::arg("block_tables"), py::arg("context_lens"), py::arg("retain_ratio"),
        py::arg("num_sink_tokens") = 4);
  m.def("dynamic_sparse_attention", &dynamic_sparse_attention, "Dynamic sparse/chunked attention over paged KV cache",
        py::arg("query"), py::arg("key_cache"), py::arg("value_cache"), py::arg("block_tables"),
        py::arg("context_lens"), py::arg("max_seq_len"), py::arg("window_size"), py::arg("causal") = false);
  m.def("dynamic_sparse_attention_int4", &dynamic_sparse_attention_int4,
        "Paged attention over an int4 pool with dequantisation fused into the loads", py::arg("query"),
        py::arg("kv_pages"), py::arg("block_tables"), py::arg("context_lens"), py::arg("max_seq_len"),
        py::arg("window_size"), py::arg("causal") = false);
  m.def("quantize_kv_cache_int4", &quantize_kv_cache_int4,
        "Quantize KV cache to packed INT4 (group-wise symmetric); returns [packed_uint8, scales_float32]",
        py::arg("cache"), py::arg("group_size"));
  m.def("dequantize_kv_cache_int4", &dequantize_kv_cache_int4, "Dequantize packed INT4 KV cache to FP16",
        py::arg("q_cache"), py::arg("scales"), py::arg("group_size"));
}
