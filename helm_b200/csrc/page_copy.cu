// Page gather into HBM: the device half of perform_streaming_attention's host-page prefetch
// (helm/runtime/kv_cache.py:412-423) and of the mixed-residency decode path.
//
// Pages evicted to pinned host memory are scattered over the host slab, so a layer's host pages
// rarely form long runs; one cudaMemcpyAsync per page then costs more host time than the
// transfer itself.  When the source is pinned host memory that the device can address (and the
// destination is device memory), one launch gathers every page instead: each CTA streams whole
// pages over the host link with 16-byte loads, many in flight.  Otherwise runs of consecutive ids
// are copied with cudaMemcpyAsync.
//
// The eviction side (helm_move_pages) is the batched form of the reference's page-by-page
// synchronous move_page copies (helm/runtime/kv_allocator.py:104-116): a batch of (source slot,
// destination slot) pairs, usually device -> pinned host, moved by one launch on a side stream,
// each CTA writing whole pages over the host link with 16-byte stores.
#include "common.cuh"

namespace helm {
namespace {

constexpr int kGatherIds = 4096;        // page ids carried by value per launch
constexpr int kGatherThreads = 256;
constexpr int kGatherMinRuns = 16;      // below this many runs, cudaMemcpyAsync is cheaper

struct GatherArgs {
  const uint4 *src;    // device-visible address of the host slab
  uint4 *dst;          // first destination page
  int64_t page_vec;    // 16-byte vectors per page
  int32_t n;
  int32_t ids[kGatherIds];
};

// One page, by the whole CTA: four 16-byte loads in flight per thread, then their stores.
__device__ __forceinline__ void copy_page(const uint4 *s, uint4 *d, int64_t page_vec) {
  int64_t v = threadIdx.x;
  for (; v + 3 * kGatherThreads < page_vec; v += 4 * kGatherThreads) {
    const uint4 x0 = s[v], x1 = s[v + kGatherThreads], x2 = s[v + 2 * kGatherThreads],
                x3 = s[v + 3 * kGatherThreads];
    d[v] = x0;
    d[v + kGatherThreads] = x1;
    d[v + 2 * kGatherThreads] = x2;
    d[v + 3 * kGatherThreads] = x3;
  }
  for (; v < page_vec; v += kGatherThreads) d[v] = s[v];
}

__global__ void __launch_bounds__(kGatherThreads) gather_pages_kernel(const __grid_constant__ GatherArgs a) {
  for (int i = blockIdx.x; i < a.n; i += gridDim.x)
    copy_page(a.src + (int64_t)a.ids[i] * a.page_vec, a.dst + (int64_t)i * a.page_vec, a.page_vec);
}

constexpr int kMoveIds = 2048;          // (src, dst) id pairs carried by value per launch

struct MoveArgs {
  const uint4 *src;    // device-visible base of the source slab
  uint4 *dst;          // device-visible base of the destination slab
  int64_t page_vec;
  int32_t n;
  int32_t src_ids[kMoveIds];
  int32_t dst_ids[kMoveIds];
};

__global__ void __launch_bounds__(kGatherThreads) move_pages_kernel(const __grid_constant__ MoveArgs a) {
  for (int i = blockIdx.x; i < a.n; i += gridDim.x)
    copy_page(a.src + (int64_t)a.src_ids[i] * a.page_vec, a.dst + (int64_t)a.dst_ids[i] * a.page_vec, a.page_vec);
}

// Device-visible address of [p, p + bytes) when it lies in pinned host memory mapped for the
// device (both ends checked, with the same mapping offset); null otherwise.
const void *mapped_host_range(const void *p, int64_t bytes) {
  cudaPointerAttributes a0{}, a1{};
  if (cudaPointerGetAttributes(&a0, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  const char *last = static_cast<const char *>(p) + bytes - 1;
  if (cudaPointerGetAttributes(&a1, last) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a0.type != cudaMemoryTypeHost || a1.type != cudaMemoryTypeHost || !a0.devicePointer || !a1.devicePointer)
    return nullptr;
  if (static_cast<const char *>(a1.devicePointer) - static_cast<const char *>(a0.devicePointer) != bytes - 1)
    return nullptr;
  return a0.devicePointer;
}

// Device-visible address of [p, p + bytes): itself for device memory, the mapping for pinned
// host memory, null otherwise.
const void *device_visible_range(const void *p, int64_t bytes) {
  cudaPointerAttributes a0{}, a1{};
  if (cudaPointerGetAttributes(&a0, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a0.type == cudaMemoryTypeDevice) {
    const char *last = static_cast<const char *>(p) + bytes - 1;
    if (cudaPointerGetAttributes(&a1, last) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    return a1.type == cudaMemoryTypeDevice && a1.device == a0.device ? p : nullptr;
  }
  return mapped_host_range(p, bytes);
}

bool is_device_memory(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice;
}

}  // namespace
}  // namespace helm

extern "C" int helm_copy_pages(void *dst_base, int64_t dst_first, const void *src_base, const int32_t *src_ids,
                               int32_t count, int64_t page_bytes, int32_t *copies_out, void *stream) {
  helm::NvtxRange nvtx_range_("helm_copy_pages");
  using namespace helm;
  if (copies_out) *copies_out = 0;
  if (count < 0 || page_bytes <= 0 || dst_first < 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "copy_pages: bad sizes count=%d page_bytes=%lld", count,
                (long long)page_bytes);
  if (count == 0) return HELM_OK;
  if (!dst_base || !src_base || !src_ids) return fail(HELM_ERR_INVALID_ARGUMENT, "copy_pages: null pointer");
  cudaStream_t st = as_stream(stream);
  int runs = 0, max_id = 0;
  for (int i = 0; i < count; ++i) {
    if (src_ids[i] < 0) return fail(HELM_ERR_INVALID_ARGUMENT, "copy_pages: negative page id %d", src_ids[i]);
    if (i == 0 || src_ids[i] != src_ids[i - 1] + 1) ++runs;
    if (src_ids[i] > max_id) max_id = src_ids[i];
  }
  char *dst0 = static_cast<char *>(dst_base) + dst_first * page_bytes;
  const bool aligned = page_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src_base) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(dst0) % 16) == 0;
  if (runs >= kGatherMinRuns && aligned) {
    const void *src_dev = mapped_host_range(src_base, ((int64_t)max_id + 1) * page_bytes);
    if (src_dev && is_device_memory(dst0) &&
        is_device_memory(dst0 + (int64_t)count * page_bytes - 1)) {
      GatherArgs a;
      a.src = static_cast<const uint4 *>(src_dev);
      a.page_vec = page_bytes / 16;
      int launches = 0;
      for (int b0 = 0; b0 < count; b0 += kGatherIds) {
        const int n = count - b0 < kGatherIds ? count - b0 : kGatherIds;
        a.dst = reinterpret_cast<uint4 *>(dst0 + (int64_t)b0 * page_bytes);
        a.n = n;
        for (int i = 0; i < n; ++i) a.ids[i] = src_ids[b0 + i];
        const int grid = n < 4 * num_sms() ? n : 4 * num_sms();
        gather_pages_kernel<<<grid, kGatherThreads, 0, st>>>(a);
        const int rc = check_launch("gather_pages_kernel");
        if (rc != HELM_OK) return rc;
        ++launches;
      }
      if (copies_out) *copies_out = launches;
      return HELM_OK;
    }
  }
  int copies = 0;
  int i = 0;
  while (i < count) {
    int j = i + 1;
    while (j < count && src_ids[j] == src_ids[j - 1] + 1) ++j;
    char *dst = dst0 + (int64_t)i * page_bytes;
    const char *src = static_cast<const char *>(src_base) + (int64_t)src_ids[i] * page_bytes;
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)(j - i) * page_bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "copy_pages: cudaMemcpyAsync: %s", cudaGetErrorString(e));
    ++copies;
    i = j;
  }
  if (copies_out) *copies_out = copies;
  return HELM_OK;
}

extern "C" int helm_move_pages(void *dst_base, const int32_t *dst_ids, const void *src_base, const int32_t *src_ids,
                               int32_t count, int64_t page_bytes, int64_t dst_pages, int64_t src_pages,
                               int32_t *copies_out, void *stream) {
  helm::NvtxRange nvtx_range_("helm_move_pages");
  using namespace helm;
  if (copies_out) *copies_out = 0;
  if (count < 0 || page_bytes <= 0 || dst_pages < 0 || src_pages < 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "move_pages: bad sizes count=%d page_bytes=%lld", count,
                (long long)page_bytes);
  if (count == 0) return HELM_OK;
  if (!dst_base || !src_base || !src_ids || !dst_ids)
    return fail(HELM_ERR_INVALID_ARGUMENT, "move_pages: null pointer");
  int runs = 0;
  for (int i = 0; i < count; ++i) {
    if (src_ids[i] < 0 || src_ids[i] >= src_pages)
      return fail(HELM_ERR_INVALID_ARGUMENT, "move_pages: source page %d outside [0, %lld)", src_ids[i],
                  (long long)src_pages);
    if (dst_ids[i] < 0 || dst_ids[i] >= dst_pages)
      return fail(HELM_ERR_INVALID_ARGUMENT, "move_pages: destination page %d outside [0, %lld)", dst_ids[i],
                  (long long)dst_pages);
    if (i == 0 || src_ids[i] != src_ids[i - 1] + 1 || dst_ids[i] != dst_ids[i - 1] + 1) ++runs;
  }
  cudaStream_t st = as_stream(stream);
  const bool aligned = page_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src_base) % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(dst_base) % 16) == 0;
  if (runs >= kGatherMinRuns && aligned) {
    const void *src_dev = device_visible_range(src_base, src_pages * page_bytes);
    void *dst_dev = const_cast<void *>(device_visible_range(dst_base, dst_pages * page_bytes));
    if (src_dev && dst_dev) {
      MoveArgs a;
      a.src = static_cast<const uint4 *>(src_dev);
      a.dst = static_cast<uint4 *>(dst_dev);
      a.page_vec = page_bytes / 16;
      int launches = 0;
      for (int b0 = 0; b0 < count; b0 += kMoveIds) {
        const int n = count - b0 < kMoveIds ? count - b0 : kMoveIds;
        a.n = n;
        for (int i = 0; i < n; ++i) {
          a.src_ids[i] = src_ids[b0 + i];
          a.dst_ids[i] = dst_ids[b0 + i];
        }
        const int grid = n < 4 * num_sms() ? n : 4 * num_sms();
        move_pages_kernel<<<grid, kGatherThreads, 0, st>>>(a);
        const int rc = check_launch("move_pages_kernel");
        if (rc != HELM_OK) return rc;
        ++launches;
      }
      if (copies_out) *copies_out = launches;
      return HELM_OK;
    }
  }
  int copies = 0;
  int i = 0;
  while (i < count) {
    int j = i + 1;
    while (j < count && src_ids[j] == src_ids[j - 1] + 1 && dst_ids[j] == dst_ids[j - 1] + 1) ++j;
    char *dst = static_cast<char *>(dst_base) + (int64_t)dst_ids[i] * page_bytes;
    const char *src = static_cast<const char *>(src_base) + (int64_t)src_ids[i] * page_bytes;
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)(j - i) * page_bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "move_pages: cudaMemcpyAsync: %s", cudaGetErrorString(e));
    ++copies;
    i = j;
  }
  if (copies_out) *copies_out = copies;
  return HELM_OK;
}
