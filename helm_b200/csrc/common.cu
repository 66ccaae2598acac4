// Host helpers shared by the helm_b200 entry points.
#include "common.cuh"
#include "tma.cuh"

#include <cstring>
#include <mutex>

namespace helm {

namespace {
thread_local char g_err[512] = {0};
}

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return HELM_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace helm

extern "C" int helm_abi_version(void) { return HELM_ABI_VERSION; }

extern "C" const char *helm_last_error(void) { return helm::g_err; }

extern "C" int helm_copy_pages(void *dst_base, int64_t dst_first, const void *src_base, const int32_t *src_ids,
                               int32_t count, int64_t page_bytes, int32_t *copies_out, void *stream) {
  using namespace helm;
  if (copies_out) *copies_out = 0;
  if (count < 0 || page_bytes <= 0 || dst_first < 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "copy_pages: bad sizes count=%d page_bytes=%lld", count,
                (long long)page_bytes);
  if (count == 0) return HELM_OK;
  if (!dst_base || !src_base || !src_ids) return fail(HELM_ERR_INVALID_ARGUMENT, "copy_pages: null pointer");
  cudaStream_t st = as_stream(stream);
  int copies = 0;
  int i = 0;
  while (i < count) {
    if (src_ids[i] < 0) return fail(HELM_ERR_INVALID_ARGUMENT, "copy_pages: negative page id %d", src_ids[i]);
    int j = i + 1;
    while (j < count && src_ids[j] == src_ids[j - 1] + 1) ++j;
    char *dst = static_cast<char *>(dst_base) + (dst_first + i) * page_bytes;
    const char *src = static_cast<const char *>(src_base) + (int64_t)src_ids[i] * page_bytes;
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)(j - i) * page_bytes, cudaMemcpyDefault, st);
    if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "copy_pages: cudaMemcpyAsync: %s", cudaGetErrorString(e));
    ++copies;
    i = j;
  }
  if (copies_out) *copies_out = copies;
  return HELM_OK;
}
