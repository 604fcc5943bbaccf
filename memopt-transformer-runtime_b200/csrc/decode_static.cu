// decode_static.cu — paged decode for callers that must not allocate.
//
// Some hosts of this library cannot call cudaMalloc at the point where they
// run attention: an allocator-less C runtime (a game engine or inference
// server with its own arena), or code running where allocation would break
// a contract (inside a latency-critical step that forbids allocator calls).
// memopt_paged_attention_f16 needs split-K scratch that the caller normally
// provides; this entry point instead uses a fixed scratch array that lives in
// the library's device image, so the call itself allocates nothing.
//
// Limits and rules (also stated in include/memopt_b200.h):
//   * the scratch is kStaticScratchBytes (4 MiB) per device; every GPU on
//     which the library is loaded holds it until the process exits;
//   * a call whose split-K scratch would exceed it is rejected with
//     MEMOPT_ERR_WORKSPACE before any work is queued;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current).  CUDA
//     loads modules lazily, so that first call is also when the array's
//     4 MiB are committed on the device, and it can fail with out-of-memory;
//     make that first call at start-up, before any stream capture;
//   * arguments are validated before the scratch is touched: a rejected call
//     queues no work;
//   * every call shares the one array: calls that overlap on the GPU (e.g. on
//     two streams without ordering between them) race.  The ticket region,
//     which must start at zero, is cleared at the start of every call.
#include <mutex>
#include <string>

#include "common.cuh"

namespace memopt {
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;

static __device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_decode_scratch for the current device.  The symbol's
// name in host code is only a host-side handle, never a device pointer.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention_f16_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(MEMOPT_ERR_UNSUPPORTED, "paged_attention_f16_noalloc: device index beyond 63");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return cuda_fail(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                       "paged_attention_f16_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MEMOPT_OK;
}

}  // namespace
}  // namespace memopt

using namespace memopt;

extern "C" size_t memopt_paged_attention_noalloc_max_bytes(void) { return kStaticScratchBytes; }

extern "C" int memopt_paged_attention_f16_noalloc(const void* query, const void* key_pool,
                                                  const void* value_pool, const int32_t* block_tables,
                                                  const int32_t* context_lens, int batch, int q_len,
                                                  int num_heads, int head_dim, int max_blocks_per_seq,
                                                  int64_t num_blocks, int block_size, int max_seq_len,
                                                  int window_size, void* out, void* stream) {
  // Arguments are checked before the shared scratch is touched, so a call
  // that is rejected queues nothing.
  const int vst = validate_attention_f16(query, key_pool, value_pool, batch, q_len, num_heads, num_heads, head_dim,
                                         max_blocks_per_seq, num_blocks, block_size, out);
  if (vst != MEMOPT_OK) return vst;
  const size_t need = memopt_paged_attention_workspace_size(batch, q_len, num_heads, head_dim,
                                                            max_blocks_per_seq, block_size, max_seq_len,
                                                            window_size);
  if (need > kStaticScratchBytes)
    return fail(MEMOPT_ERR_WORKSPACE,
                "paged_attention_f16_noalloc: this call needs " + std::to_string(need) +
                    " bytes of split-K scratch; the static scratch holds " +
                    std::to_string(kStaticScratchBytes) + " bytes (use memopt_paged_attention_f16 "
                    "with a caller-provided workspace)");
  void* ws = nullptr;
  if (need > 0) {
    const int st = scratch_for_current_device(&ws);
    if (st != MEMOPT_OK) return st;
    const size_t tickets = memopt_paged_attention_ticket_bytes(batch, q_len, num_heads);
    const cudaError_t e = cudaMemsetAsync(ws, 0, tickets, as_stream(stream));
    if (e != cudaSuccess) return cuda_fail(e, "paged_attention_f16_noalloc: clearing tickets");
  }
  return memopt_paged_attention_f16(query, key_pool, value_pool, block_tables, context_lens, batch,
                                    q_len, num_heads, head_dim, max_blocks_per_seq, num_blocks,
                                    block_size, max_seq_len, window_size, out, ws, need, stream);
}
