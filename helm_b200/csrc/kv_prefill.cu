// Prefill page writes: the device half of KVCacheManager.append_prefill
// (helm/runtime/kv_cache.py:55-85), which cuts a prompt's K/V into page-sized
// chunks and copies each chunk into its page.  Here one launch writes every
// chunk of a call: the (slot, first token, tokens) list of the pages rides in
// the kernel parameters, one CTA copies one (page, kv head) tile with 16-byte
// loads and stores, and, when the caller passes a device page-table row, the
// same launch writes the pages' table entries.
#include "common.cuh"

namespace helm {
namespace {

constexpr int kPrefillPages = 1024;  // pages carried by value per launch
constexpr int kPrefillThreads = 256;

struct PrefillArgs {
  const void *k_src, *v_src;
  int32_t src_dtype;
  int64_t src_head_stride, src_tok_stride;
  void *k_base, *v_base;
  int64_t page_stride, head_stride;
  int32_t num_pool_pages;
  int32_t kv_dtype;
  int32_t Hkv, D, P;
  int32_t n;
  int32_t *page_table, *page_used, *num_pages;
  int32_t first_index, pt_stride;
  int32_t vec;                          // 1: 16-byte copies (same dtype, aligned)
  int32_t *error_flag;
  int32_t pages[kPrefillPages][3];      // {pool slot, first token in the source, tokens}
};

__global__ void __launch_bounds__(kPrefillThreads) prefill_pages_kernel(const __grid_constant__ PrefillArgs a) {
  const int i = blockIdx.x, h = blockIdx.y;
  const int slot = a.pages[i][0], t0 = a.pages[i][1], nt = a.pages[i][2];
  pdl_trigger();
  pdl_wait();
  if (slot < 0 || slot >= a.num_pool_pages || nt < 0 || nt > a.P) {
    if (threadIdx.x == 0 && h == 0) flag_error(a.error_flag, HELM_DEVERR_PAGE_ID);
    return;
  }
  if (h == 0 && threadIdx.x == 0 && a.page_table) {
    const int li = a.first_index + i;
    if (li < 0 || li >= a.pt_stride) {
      flag_error(a.error_flag, HELM_DEVERR_NUM_PAGES);
    } else {
      a.page_table[li] = slot;
      a.page_used[li] = nt;
      if (i == a.n - 1 && a.num_pages[0] < li + 1) a.num_pages[0] = li + 1;
    }
  }
  const int64_t dst0 = (int64_t)slot * a.page_stride + (int64_t)h * a.head_stride;
  const int64_t src0 = (int64_t)h * a.src_head_stride + (int64_t)t0 * a.src_tok_stride;
  for (int kv = 0; kv < 2; ++kv) {
    const void *src = kv ? a.v_src : a.k_src;
    void *dst = kv ? a.v_base : a.k_base;
    if (a.vec) {
      const int es = a.kv_dtype == HELM_F32 ? 4 : 2;
      const int per = 16 / es;                     // elements per 16-byte vector
      const int vrow = a.D / per;
      for (int j = threadIdx.x; j < nt * vrow; j += blockDim.x) {
        const int t = j / vrow, c = j - t * vrow;
        const uint4 v = *reinterpret_cast<const uint4 *>(static_cast<const char *>(src) +
                                                          (src0 + (int64_t)t * a.src_tok_stride + c * per) * es);
        *reinterpret_cast<uint4 *>(static_cast<char *>(dst) + (dst0 + (int64_t)t * a.D + c * per) * es) = v;
      }
    } else {
      for (int j = threadIdx.x; j < nt * a.D; j += blockDim.x) {
        const int t = j / a.D, d = j - t * a.D;
        store_f(dst, a.kv_dtype, dst0 + (int64_t)t * a.D + d,
                load_f(src, a.src_dtype, src0 + (int64_t)t * a.src_tok_stride + d));
      }
    }
  }
}

}  // namespace
}  // namespace helm

extern "C" int helm_kv_write_pages(const helm_kv_prefill_params *p, void *stream) {
  helm::NvtxRange nvtx_range_("helm_kv_write_pages");
  using namespace helm;
  if (!p) return fail(HELM_ERR_INVALID_ARGUMENT, "kv_write_pages: params is null");
  if (p->count < 0 || p->Hkv <= 0 || p->D <= 0 || p->P <= 0 || p->num_pool_pages < 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_write_pages: bad sizes count=%d Hkv=%d D=%d P=%d", p->count, p->Hkv,
                p->D, p->P);
  if (p->count == 0) return HELM_OK;
  if (!p->k_src || !p->v_src || !p->k_base || !p->v_base || !p->pages)
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_write_pages: null pointer");
  for (int dt : {p->src_dtype, p->kv_dtype})
    if (dt != HELM_F32 && dt != HELM_F16 && dt != HELM_BF16)
      return fail(HELM_ERR_UNSUPPORTED, "kv_write_pages: dtype %d", dt);
  if (p->page_table && (!p->page_used || !p->num_pages))
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_write_pages: page_table needs page_used and num_pages");
  for (int i = 0; i < p->count; ++i) {
    const int32_t *e = p->pages + 3 * i;
    if (e[0] < 0 || e[0] >= p->num_pool_pages || e[1] < 0 || e[2] < 0 || e[2] > p->P)
      return fail(HELM_ERR_INVALID_ARGUMENT, "kv_write_pages: page %d = {slot %d, start %d, tokens %d} out of range", i,
                  e[0], e[1], e[2]);
  }
  const int es = dtype_size(p->kv_dtype);
  const uintptr_t al = reinterpret_cast<uintptr_t>(p->k_src) | reinterpret_cast<uintptr_t>(p->v_src) |
                       reinterpret_cast<uintptr_t>(p->k_base) | reinterpret_cast<uintptr_t>(p->v_base);
  const bool vec = p->src_dtype == p->kv_dtype && (al & 15) == 0 && (p->D * es) % 16 == 0 &&
                   (p->src_head_stride * es) % 16 == 0 && (p->src_tok_stride * es) % 16 == 0 &&
                   (p->page_stride * es) % 16 == 0 && (p->head_stride * es) % 16 == 0;
  cudaStream_t st = as_stream(stream);
  PrefillArgs a;
  a.k_src = p->k_src;
  a.v_src = p->v_src;
  a.src_dtype = p->src_dtype;
  a.src_head_stride = p->src_head_stride;
  a.src_tok_stride = p->src_tok_stride;
  a.k_base = p->k_base;
  a.v_base = p->v_base;
  a.page_stride = p->page_stride;
  a.head_stride = p->head_stride;
  a.num_pool_pages = p->num_pool_pages;
  a.kv_dtype = p->kv_dtype;
  a.Hkv = p->Hkv;
  a.D = p->D;
  a.P = p->P;
  a.pt_stride = p->page_table_stride;
  a.vec = vec ? 1 : 0;
  a.error_flag = p->error_flag;
  a.num_pages = p->num_pages;
  for (int b0 = 0; b0 < p->count; b0 += kPrefillPages) {
    const int n = p->count - b0 < kPrefillPages ? p->count - b0 : kPrefillPages;
    a.n = n;
    a.first_index = p->first_index + b0;
    a.page_table = p->page_table;
    a.page_used = p->page_used;
    for (int i = 0; i < n; ++i)
      for (int j = 0; j < 3; ++j) a.pages[i][j] = p->pages[3 * (b0 + i) + j];
    const cudaError_t e = launch_pdl(prefill_pages_kernel, dim3(n, p->Hkv), dim3(kPrefillThreads), 0, st, a);
    if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "kv_write_pages: launch: %s", cudaGetErrorString(e));
    const int rc = check_launch("prefill_pages_kernel");
    if (rc != HELM_OK) return rc;
  }
  return HELM_OK;
}
