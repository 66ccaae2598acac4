// KV slot append: the device half of KVCacheManager.append_decode
// (helm/runtime/kv_cache.py:87-113), which writes one token's K/V into the
// tail page and advances the page's used-token count.
#include "common.cuh"

namespace helm {

constexpr int kHostDestRows = 64;  // host-directed rows carried per launch

struct AppendArgs {
  const void *k_new, *v_new;
  int32_t src_dtype;
  void *k_base, *v_base;
  int64_t page_stride, head_stride;
  int32_t num_pool_pages;
  int32_t kv_dtype;
  int32_t B, Hkv, D, P;
  const int32_t *dest;
  int32_t *page_table, *page_used, *num_pages;
  int32_t pt_stride;
  const int32_t *spare_pages;
  int32_t *spare_next;
  int32_t spare_stride;
  int32_t *error_flag;
  int32_t b0;                          // first sequence of this launch
  int32_t use_hdest;
  int32_t hdest[kHostDestRows][3];     // host-directed rows, by value
};

// One CTA per sequence: thread 0 resolves the destination (page id, slot),
// then the CTA copies Hkv*D elements of K and of V.
__global__ void __launch_bounds__(256) kv_append_kernel(AppendArgs a) {
  __shared__ int s_pid, s_slot;
  const int b = a.b0 + blockIdx.x;
  if (threadIdx.x == 0) {
    int pid = -1, slot = -1;
    int32_t *pt = a.page_table ? a.page_table + (int64_t)b * a.pt_stride : nullptr;
    int32_t *pu = a.page_used ? a.page_used + (int64_t)b * a.pt_stride : nullptr;
    if (a.dest || a.use_hdest) {
      const int32_t *row = a.use_hdest ? a.hdest[blockIdx.x] : a.dest + 3 * b;
      pid = row[0];
      const int li = row[1];
      slot = row[2];
      const bool ok = pid >= 0 && pid < a.num_pool_pages && slot >= 0 && slot < a.P;
      if (!ok) {
        flag_error(a.error_flag, HELM_DEVERR_PAGE_ID);
        pid = -1;
      } else if (pt) {
        if (li < 0 || li >= a.pt_stride) {
          flag_error(a.error_flag, HELM_DEVERR_NUM_PAGES);
          pid = -1;
        } else {
          pt[li] = pid;
          pu[li] = slot + 1;
          if (a.num_pages[b] < li + 1) a.num_pages[b] = li + 1;
        }
      }
    } else {
      const int np = a.num_pages[b];
      const bool np_ok = np >= 0 && np <= a.pt_stride;
      const int u = (np_ok && np > 0) ? pu[np - 1] : a.P;
      if (!np_ok) {
        flag_error(a.error_flag, HELM_DEVERR_NUM_PAGES);
      } else if (u < a.P) {
        pid = pt[np - 1];
        slot = u;
        pu[np - 1] = u + 1;
      } else {
        const int j = a.spare_next ? a.spare_next[b] : a.spare_stride;
        if (j >= a.spare_stride || np >= a.pt_stride) {
          flag_error(a.error_flag, HELM_DEVERR_APPEND_FULL);
        } else {
          pid = a.spare_pages[(int64_t)b * a.spare_stride + j];
          a.spare_next[b] = j + 1;
          slot = 0;
          pt[np] = pid;
          pu[np] = 1;
          a.num_pages[b] = np + 1;
        }
      }
      if (pid >= a.num_pool_pages || (pid < 0 && slot >= 0)) {
        flag_error(a.error_flag, HELM_DEVERR_PAGE_ID);
        pid = -1;
      }
    }
    s_pid = pid;
    s_slot = slot;
  }
  __syncthreads();
  const int pid = s_pid, slot = s_slot;
  if (pid < 0) return;
  const int n = a.Hkv * a.D;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = i / a.D, d = i - h * a.D;
    const int64_t src = (int64_t)b * n + i;
    const int64_t dst = (int64_t)pid * a.page_stride + (int64_t)h * a.head_stride + (int64_t)slot * a.D + d;
    store_f(a.k_base, a.kv_dtype, dst, load_f(a.k_new, a.src_dtype, src));
    store_f(a.v_base, a.kv_dtype, dst, load_f(a.v_new, a.src_dtype, src));
  }
}

}  // namespace helm

extern "C" int helm_kv_append(const helm_kv_append_params *p, void *stream) {
  using namespace helm;
  if (!p) return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: params is null");
  if (p->B < 0 || p->Hkv <= 0 || p->D <= 0 || p->P <= 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: bad sizes B=%d Hkv=%d D=%d P=%d", p->B, p->Hkv, p->D, p->P);
  for (int dt : {p->src_dtype, p->kv_dtype})
    if (dt != HELM_F32 && dt != HELM_F16 && dt != HELM_BF16)
      return fail(HELM_ERR_UNSUPPORTED, "kv_append: dtype %d", dt);
  if (p->B == 0) return HELM_OK;
  if (!p->k_new || !p->v_new || !p->k_base || !p->v_base)
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: null data pointer");
  const bool directed = p->dest || p->dest_host;
  if (!directed && (!p->page_table || !p->page_used || !p->num_pages || !p->spare_pages || !p->spare_next))
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: device-directed mode needs page table and spare pages");
  if (directed && p->page_table && (!p->page_used || !p->num_pages))
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: page_table given without page_used/num_pages");
  AppendArgs a{};
  a.k_new = p->k_new;
  a.v_new = p->v_new;
  a.src_dtype = p->src_dtype;
  a.k_base = p->k_base;
  a.v_base = p->v_base;
  a.page_stride = p->page_stride;
  a.head_stride = p->head_stride;
  a.num_pool_pages = p->num_pool_pages;
  a.kv_dtype = p->kv_dtype;
  a.B = p->B;
  a.Hkv = p->Hkv;
  a.D = p->D;
  a.P = p->P;
  a.dest = p->dest_host ? nullptr : p->dest;
  a.page_table = p->page_table;
  a.page_used = p->page_used;
  a.num_pages = p->num_pages;
  a.pt_stride = p->page_table_stride;
  a.spare_pages = p->spare_pages;
  a.spare_next = p->spare_next;
  a.spare_stride = p->spare_stride;
  a.error_flag = p->error_flag;
  cudaStream_t st = as_stream(stream);
  if (!p->dest_host) {
    kv_append_kernel<<<p->B, 256, 0, st>>>(a);
    return check_launch("kv_append_kernel");
  }
  a.use_hdest = 1;
  for (int b0 = 0; b0 < p->B; b0 += kHostDestRows) {
    const int nb = p->B - b0 < kHostDestRows ? p->B - b0 : kHostDestRows;
    a.b0 = b0;
    for (int i = 0; i < nb; ++i)
      for (int j = 0; j < 3; ++j) a.hdest[i][j] = p->dest_host[3 * (b0 + i) + j];
    kv_append_kernel<<<nb, 256, 0, st>>>(a);
    int rc = check_launch("kv_append_kernel");
    if (rc != HELM_OK) return rc;
  }
  return HELM_OK;
}
