// host.cu — error reporting, device queries and the page-pool free-list.
//
// The free-list restates the reference's KVCachePool bookkeeping
// (src/csrc/kv_cache.cu:83-201): a process-wide FIFO of free block indices
// guarded by a mutex, idempotent re-initialisation for identical geometry.
// Device memory is not owned here (the caller allocates the pool tensors).
#include <deque>
#include <mutex>
#include <string>

#include "common.cuh"

namespace memopt {

namespace {
thread_local std::string g_last_error;

struct PoolState {
  std::mutex mu;
  bool initialized = false;
  int num_blocks = 0, block_size = 0, num_heads = 0, head_dim = 0;
  std::deque<int> free_list;
};
PoolState& pool() {
  static PoolState p;
  return p;
}
}  // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  set_last_error(msg);
  return status;
}

int cuda_fail(cudaError_t err, const char* what) {
  set_last_error(std::string(what) + ": " + cudaGetErrorString(err));
  return MEMOPT_ERR_CUDA;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

const char* last_error_cstr() { return g_last_error.c_str(); }

}  // namespace memopt

using memopt::pool;

extern "C" {

int memopt_abi_version(void) { return 1; }

const char* memopt_status_string(int status) {
  switch (status) {
    case MEMOPT_OK: return "ok";
    case MEMOPT_ERR_INVALID_ARG: return "invalid argument";
    case MEMOPT_ERR_NOT_INITIALIZED: return "pool not initialized";
    case MEMOPT_ERR_UNSUPPORTED: return "unsupported configuration";
    case MEMOPT_ERR_CUDA: return "CUDA error";
    case MEMOPT_ERR_OUT_OF_RANGE: return "out of range";
    case MEMOPT_ERR_WORKSPACE: return "workspace too small";
    case MEMOPT_ERR_TIMEOUT: return "a bounded device wait ran out";
    default: return "unknown status";
  }
}

const char* memopt_last_error(void) { return memopt::last_error_cstr(); }

int memopt_pool_init(int num_blocks, int block_size, int num_heads, int head_dim) {
  auto& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (p.initialized && p.num_blocks == num_blocks && p.block_size == block_size &&
      p.num_heads == num_heads && p.head_dim == head_dim)
    return MEMOPT_OK;
  // Any failed re-initialisation leaves the pool uninitialised, so a later
  // write cannot silently land in the previous pool's geometry.
  p.initialized = false;
  p.free_list.clear();
  if (num_blocks <= 0) return memopt::fail(MEMOPT_ERR_INVALID_ARG, "init_pool: num_blocks must be > 0");
  if (block_size <= 0) return memopt::fail(MEMOPT_ERR_INVALID_ARG, "init_pool: block_size must be > 0");
  if (num_heads <= 0) return memopt::fail(MEMOPT_ERR_INVALID_ARG, "init_pool: num_heads must be > 0");
  if (head_dim <= 0) return memopt::fail(MEMOPT_ERR_INVALID_ARG, "init_pool: head_dim must be > 0");
  if (head_dim % 2 != 0)
    return memopt::fail(MEMOPT_ERR_INVALID_ARG, "init_pool: head_dim must be even for fp16 coalesced access");
  for (int i = 0; i < num_blocks; ++i) p.free_list.push_back(i);
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.num_heads = num_heads;
  p.head_dim = head_dim;
  p.initialized = true;
  return MEMOPT_OK;
}

void memopt_pool_reset(void) {
  auto& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  p.initialized = false;
  p.free_list.clear();
  p.num_blocks = p.block_size = p.num_heads = p.head_dim = 0;
}

int memopt_pool_is_initialized(void) {
  auto& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  return p.initialized ? 1 : 0;
}

int memopt_pool_config(int* num_blocks, int* block_size, int* num_heads, int* head_dim) {
  auto& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!p.initialized) return memopt::fail(MEMOPT_ERR_NOT_INITIALIZED, "pool not initialized");
  if (num_blocks) *num_blocks = p.num_blocks;
  if (block_size) *block_size = p.block_size;
  if (num_heads) *num_heads = p.num_heads;
  if (head_dim) *head_dim = p.head_dim;
  return MEMOPT_OK;
}

int memopt_pool_allocate_block(void) {
  auto& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!p.initialized)
    return memopt::fail(MEMOPT_ERR_NOT_INITIALIZED, "allocate_block: pool not initialized");
  if (p.free_list.empty()) return -1;
  int idx = p.free_list.front();
  p.free_list.pop_front();
  return idx;
}

int memopt_pool_free_block(int block_idx) {
  auto& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!p.initialized) return memopt::fail(MEMOPT_ERR_NOT_INITIALIZED, "free_block: pool not initialized");
  if (block_idx < 0 || block_idx >= p.num_blocks)
    return memopt::fail(MEMOPT_ERR_OUT_OF_RANGE, "free_block: block_idx out of range");
  p.free_list.push_back(block_idx);
  return MEMOPT_OK;
}

int memopt_pool_free_blocks_count(void) {
  auto& p = pool();
  std::lock_guard<std::mutex> lk(p.mu);
  return p.initialized ? static_cast<int>(p.free_list.size()) : 0;
}

}  // extern "C"
