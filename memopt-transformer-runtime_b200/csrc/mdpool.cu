// mdpool.cu — KV pages spread over several GPUs.
//
// The reference keeps one pool on one device (src/csrc/kv_cache.cu:97, "extend
// to multi-GPU via device_id key if needed"; README "Future Work": a block
// allocator spanning devices).  This file holds the host side of that
// extension and the one device kernel it needs:
//
//  * a page allocator over D devices (one FIFO free-list per device, as the
//    single-device pool): a page is (owner device, block).  Allocation takes
//    the preferred device's oldest free block and spills to the device with
//    the most free blocks (lowest index on ties) when the preferred one is
//    full, so a context can outgrow one GPU's HBM.  Every rank of an SPMD job
//    runs the same calls and keeps an identical copy;
//  * a gather plan: for the pages a home device needs, the local block ids
//    of the pages it owns, and for the others one copy each (deduplicated)
//    into consecutive staging blocks of the home pool, grouped by owner in
//    device order, so each peer's pages arrive as one contiguous run;
//  * memopt_copy_pages: dst[dst_ids[i]] = src[src_ids[i]] for whole pages on
//    one device (packing pages for a transfer, or unpacking them), 16-byte
//    vector copies, one warp per page.
// No kernel here reads another GPU's memory: pages cross between devices
// only through the caller's transfer (NCCL send/recv) of packed buffers.
#include <algorithm>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace memopt {
namespace {

struct MdPool {
  std::mutex mu;
  bool initialized = false;
  std::vector<std::deque<int>> free_list;
  std::vector<std::vector<uint8_t>> in_use;
};
MdPool& mdpool() {
  static MdPool p;
  return p;
}

constexpr int kMaxDevices = 64;
constexpr int kCopyWarps = 8;

__global__ void __launch_bounds__(kCopyWarps * 32)
copy_pages_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ src_ids, uint4* __restrict__ dst,
                  const int32_t* __restrict__ dst_ids, int n, int64_t page_vecs) {
  const int lane = threadIdx.x & 31;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kCopyWarps + (threadIdx.x >> 5); i < n;
       i += static_cast<int64_t>(gridDim.x) * kCopyWarps) {
    const int64_t s = src_ids ? __ldg(src_ids + i) : i;
    const int64_t d = dst_ids ? __ldg(dst_ids + i) : i;
    if (s < 0 || d < 0) continue;
    const uint4* sp = src + s * page_vecs;
    uint4* dp = dst + d * page_vecs;
    for (int64_t c = lane; c < page_vecs; c += 32 * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c + 32 * u < page_vecs) v[u] = ld_stream_v4(sp + c + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c + 32 * u < page_vecs) dp[c + 32 * u] = v[u];
    }
  }
}

}  // namespace
}  // namespace memopt

using memopt::fail;
using memopt::mdpool;

extern "C" {

int memopt_mdpool_init(int num_devices, const int* blocks_per_device) {
  auto& p = mdpool();
  std::lock_guard<std::mutex> lk(p.mu);
  p.initialized = false;
  p.free_list.clear();
  p.in_use.clear();
  if (num_devices <= 0 || num_devices > memopt::kMaxDevices)
    return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_init: num_devices must be in [1, 64]");
  if (!blocks_per_device) return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_init: null blocks_per_device");
  for (int d = 0; d < num_devices; ++d)
    if (blocks_per_device[d] < 0) return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_init: negative block count");
  p.free_list.resize(num_devices);
  p.in_use.resize(num_devices);
  for (int d = 0; d < num_devices; ++d) {
    for (int b = 0; b < blocks_per_device[d]; ++b) p.free_list[d].push_back(b);
    p.in_use[d].assign(blocks_per_device[d], 0);
  }
  p.initialized = true;
  return MEMOPT_OK;
}

void memopt_mdpool_reset(void) {
  auto& p = mdpool();
  std::lock_guard<std::mutex> lk(p.mu);
  p.initialized = false;
  p.free_list.clear();
  p.in_use.clear();
}

int memopt_mdpool_allocate(int preferred_device, int* device_out) {
  auto& p = mdpool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!p.initialized) return fail(MEMOPT_ERR_NOT_INITIALIZED, "mdpool_allocate: pool not initialized");
  const int nd = static_cast<int>(p.free_list.size());
  if (preferred_device < 0 || preferred_device >= nd)
    return fail(MEMOPT_ERR_OUT_OF_RANGE, "mdpool_allocate: preferred_device out of range");
  int d = preferred_device;
  if (p.free_list[d].empty()) {
    d = -1;
    size_t most = 0;
    for (int i = 0; i < nd; ++i)
      if (p.free_list[i].size() > most) {
        most = p.free_list[i].size();
        d = i;
      }
    if (d < 0) return -1;  // every device exhausted
  }
  const int blk = p.free_list[d].front();
  p.free_list[d].pop_front();
  p.in_use[d][blk] = 1;
  if (device_out) *device_out = d;
  return blk;
}

int memopt_mdpool_free(int device, int block) {
  auto& p = mdpool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!p.initialized) return fail(MEMOPT_ERR_NOT_INITIALIZED, "mdpool_free: pool not initialized");
  if (device < 0 || device >= static_cast<int>(p.free_list.size()))
    return fail(MEMOPT_ERR_OUT_OF_RANGE, "mdpool_free: device out of range");
  if (block < 0 || block >= static_cast<int>(p.in_use[device].size()))
    return fail(MEMOPT_ERR_OUT_OF_RANGE, "mdpool_free: block out of range");
  if (!p.in_use[device][block]) return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_free: block is already free");
  p.in_use[device][block] = 0;
  p.free_list[device].push_back(block);
  return MEMOPT_OK;
}

int memopt_mdpool_free_count(int device) {
  auto& p = mdpool();
  std::lock_guard<std::mutex> lk(p.mu);
  if (!p.initialized) return fail(MEMOPT_ERR_NOT_INITIALIZED, "mdpool_free_count: pool not initialized");
  if (device < 0 || device >= static_cast<int>(p.free_list.size()))
    return fail(MEMOPT_ERR_OUT_OF_RANGE, "mdpool_free_count: device out of range");
  return static_cast<int>(p.free_list[device].size());
}

int memopt_mdpool_plan(const int32_t* page_dev, const int32_t* page_blk, int n, int home_device,
                       int staging_base, int staging_capacity, int32_t* local_blk, int32_t* copy_src_dev,
                       int32_t* copy_src_blk, int32_t* copy_dst_blk, int* n_copies) {
  if (n < 0 || staging_base < 0 || staging_capacity < 0 || home_device < 0)
    return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_plan: negative argument");
  if (n > 0 && (!page_dev || !page_blk || !local_blk)) return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_plan: null table");
  if (!n_copies) return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_plan: null n_copies");
  // Unique remote pages, grouped by owner device (device order), first
  // appearance order within a device.
  std::map<std::pair<int, int>, int> slot_of;
  std::vector<std::pair<int, int>> remote;
  for (int i = 0; i < n; ++i) {
    if (page_blk[i] < 0 || page_dev[i] == home_device) continue;
    const std::pair<int, int> key(page_dev[i], page_blk[i]);
    if (slot_of.emplace(key, -1).second) remote.push_back(key);
  }
  std::stable_sort(remote.begin(), remote.end(),
                   [](const std::pair<int, int>& a, const std::pair<int, int>& b) { return a.first < b.first; });
  if (static_cast<int>(remote.size()) > staging_capacity)
    return fail(MEMOPT_ERR_WORKSPACE, "mdpool_plan: " + std::to_string(remote.size()) +
                                          " remote pages but only " + std::to_string(staging_capacity) +
                                          " staging blocks");
  if (!remote.empty() && (!copy_src_dev || !copy_src_blk || !copy_dst_blk))
    return fail(MEMOPT_ERR_INVALID_ARG, "mdpool_plan: null copy list");
  for (size_t k = 0; k < remote.size(); ++k) {
    slot_of[remote[k]] = staging_base + static_cast<int>(k);
    copy_src_dev[k] = remote[k].first;
    copy_src_blk[k] = remote[k].second;
    copy_dst_blk[k] = staging_base + static_cast<int>(k);
  }
  for (int i = 0; i < n; ++i) {
    if (page_blk[i] < 0) local_blk[i] = -1;
    else if (page_dev[i] == home_device) local_blk[i] = page_blk[i];
    else local_blk[i] = slot_of[std::make_pair(page_dev[i], page_blk[i])];
  }
  *n_copies = static_cast<int>(remote.size());
  return MEMOPT_OK;
}

int memopt_copy_pages(const void* src_pool, const int32_t* src_ids, void* dst_pool, const int32_t* dst_ids,
                      int num_pages, int64_t page_bytes, void* stream) {
  if (num_pages < 0 || page_bytes <= 0) return fail(MEMOPT_ERR_INVALID_ARG, "copy_pages: invalid size");
  if (page_bytes % 16 != 0) return fail(MEMOPT_ERR_UNSUPPORTED, "copy_pages: page_bytes must be a multiple of 16");
  if (num_pages == 0) return MEMOPT_OK;
  if (!src_pool || !dst_pool) return fail(MEMOPT_ERR_INVALID_ARG, "copy_pages: null pool");
  if ((reinterpret_cast<uintptr_t>(src_pool) | reinterpret_cast<uintptr_t>(dst_pool)) & 15u)
    return fail(MEMOPT_ERR_INVALID_ARG, "copy_pages: pools must be 16-byte aligned");
  const int64_t want = (num_pages + memopt::kCopyWarps - 1) / memopt::kCopyWarps;
  const int64_t cap = static_cast<int64_t>(memopt::sm_count()) * 8;
  memopt::copy_pages_kernel<<<static_cast<int>(want < cap ? want : cap), memopt::kCopyWarps * 32, 0,
                              memopt::as_stream(stream)>>>(
      static_cast<const uint4*>(src_pool), src_ids, static_cast<uint4*>(dst_pool), dst_ids, num_pages,
      page_bytes / 16);
  MEMOPT_LAUNCH_CHECK("copy_pages_kernel launch");
  return MEMOPT_OK;
}

}  // extern "C"
