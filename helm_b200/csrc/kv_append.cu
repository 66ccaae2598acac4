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

// Destination of sequence b's new token: (page id, slot), with the page table updated; pid = -1
// (and an error bit) when the destination is invalid.  Run by one thread.
__device__ void resolve_dest(const AppendArgs &a, int b, int local, int &pid_out, int &slot_out) {
  int pid = -1, slot = -1;
  int32_t *pt = a.page_table ? a.page_table + (int64_t)b * a.pt_stride : nullptr;
  int32_t *pu = a.page_used ? a.page_used + (int64_t)b * a.pt_stride : nullptr;
  if (a.dest || a.use_hdest) {
    const int32_t *row = a.use_hdest ? a.hdest[local] : a.dest + 3 * b;
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
  pid_out = pid;
  slot_out = slot;
}

// One CTA per sequence: thread 0 resolves the destination (page id, slot) while every thread
// loads its share of the new token's K and V; then the CTA stores Hkv*D elements of each.
constexpr int kAppendPre = 4;   // elements of K (and of V) a thread holds across the barrier

__global__ void __launch_bounds__(256) kv_append_kernel(AppendArgs a) {
  __shared__ int s_pid, s_slot;
  const int b = a.b0 + blockIdx.x;
  // Programmatic dependent launch: only the launch overlaps the previous kernel.
  pdl_trigger();
  pdl_wait();
  const int n = a.Hkv * a.D;
  const bool pre = n <= kAppendPre * (int)blockDim.x;
  float kr[kAppendPre], vr[kAppendPre];
  if (pre) {
#pragma unroll
    for (int j = 0; j < kAppendPre; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      kr[j] = i < n ? load_f(a.k_new, a.src_dtype, (int64_t)b * n + i) : 0.f;
      vr[j] = i < n ? load_f(a.v_new, a.src_dtype, (int64_t)b * n + i) : 0.f;
    }
  }
  if (threadIdx.x == 0) resolve_dest(a, b, blockIdx.x, s_pid, s_slot);
  __syncthreads();
  const int pid = s_pid, slot = s_slot;
  if (pid < 0) return;
  const int64_t base = (int64_t)pid * a.page_stride + (int64_t)slot * a.D;
  if (pre) {
#pragma unroll
    for (int j = 0; j < kAppendPre; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      if (i < n) {
        const int h = i / a.D, d = i - h * a.D;
        const int64_t dst = base + (int64_t)h * a.head_stride + d;
        store_f(a.k_base, a.kv_dtype, dst, kr[j]);
        store_f(a.v_base, a.kv_dtype, dst, vr[j]);
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = i / a.D, d = i - h * a.D;
    const int64_t src = (int64_t)b * n + i;
    const int64_t dst = base + (int64_t)h * a.head_stride + d;
    store_f(a.k_base, a.kv_dtype, dst, load_f(a.k_new, a.src_dtype, src));
    store_f(a.v_base, a.kv_dtype, dst, load_f(a.v_new, a.src_dtype, src));
  }
}

// ---------------------------------------------------------------------------
// Decode prologue: per-head RMSNorm of q and k (Qwen3 q_norm / k_norm), rotary
// embedding of q and k (x*cos + rotate_half(x)*sin, rotate_half(x) =
// (-x[D/2:], x[:D/2])), q written out, k and v appended to the pool.
// Grid (sequences, 1 + ceil(Hq / 8)) of 8-warp CTAs, one warp per head:
//   y = 0   the sequence's append: thread 0 resolves the destination while the
//           warps normalise and rotate the k heads (and load the v heads) into
//           shared memory; after the barrier the CTA stores them into the slot;
//   y >= 1  eight query heads each, written to q_out.
// A head's loads (x, norm weights, cos, sin) are all issued before any of them
// is used, so each head costs one memory round trip.  Lane l owns the rotary
// pairs (d, d + D/2) for d = l, l + 32, ...
// ---------------------------------------------------------------------------
struct PrologueArgs {
  const void *q_in;
  void *q_out;
  int32_t Hq;
  int64_t q_stride, k_stride, v_stride;  // elements between sequences of q_in, k_new, v_new
  const void *q_norm_w, *k_norm_w;
  int32_t norm_dtype;
  float eps;
  const void *cos, *sin;
  int32_t cs_dtype;
  int64_t cs_stride;
  int32_t do_append;
};

constexpr int kMaxHalfPerLane = 4;  // D <= 256
constexpr int kProWarps = 8;

__device__ __forceinline__ void norm_rope_head(const void *src, int src_dt, int64_t src_off, const void *w,
                                               int w_dt, float eps, const void *cs_cos, const void *cs_sin,
                                               int cs_dt, int64_t cs_off, int D, int lane,
                                               float (&lo)[kMaxHalfPerLane], float (&hi)[kMaxHalfPerLane]) {
  const int half = D >> 1;
  float w0[kMaxHalfPerLane], w1[kMaxHalfPerLane], c0[kMaxHalfPerLane], c1[kMaxHalfPerLane];
  float s0[kMaxHalfPerLane], s1[kMaxHalfPerLane];
#pragma unroll
  for (int i = 0; i < kMaxHalfPerLane; ++i) {
    const int d = lane + 32 * i;
    const bool in = d < half;
    lo[i] = in ? load_f(src, src_dt, src_off + d) : 0.f;
    hi[i] = in ? load_f(src, src_dt, src_off + d + half) : 0.f;
    w0[i] = in && w ? load_f(w, w_dt, d) : 0.f;
    w1[i] = in && w ? load_f(w, w_dt, d + half) : 0.f;
    c0[i] = in && cs_cos ? load_f(cs_cos, cs_dt, cs_off + d) : 0.f;
    c1[i] = in && cs_cos ? load_f(cs_cos, cs_dt, cs_off + d + half) : 0.f;
    s0[i] = in && cs_cos ? load_f(cs_sin, cs_dt, cs_off + d) : 0.f;
    s1[i] = in && cs_cos ? load_f(cs_sin, cs_dt, cs_off + d + half) : 0.f;
  }
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxHalfPerLane; ++i)
      if (lane + 32 * i < half) ss = fmaf(lo[i], lo[i], fmaf(hi[i], hi[i], ss));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float r = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int i = 0; i < kMaxHalfPerLane; ++i) {
      lo[i] = lo[i] * r * w0[i];
      hi[i] = hi[i] * r * w1[i];
    }
  }
  if (cs_cos) {
#pragma unroll
    for (int i = 0; i < kMaxHalfPerLane; ++i) {
      const float x0 = lo[i], x1 = hi[i];
      lo[i] = x0 * c0[i] - x1 * s0[i];  // rotate_half: first half takes -x[d + D/2]
      hi[i] = x1 * c1[i] + x0 * s1[i];  // second half takes x[d]
    }
  }
}

__global__ void __launch_bounds__(kProWarps * 32) decode_prologue_kernel(AppendArgs a, PrologueArgs pr) {
  extern __shared__ float kv_stage[];   // [2 * Hkv][D]: k heads after norm + rope, then v heads
  __shared__ int s_pid, s_slot;
  const int b = a.b0 + blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = a.D, half = D >> 1;
  const int64_t cs_off = (int64_t)b * pr.cs_stride;
  pdl_trigger();
  pdl_wait();
  float lo[kMaxHalfPerLane], hi[kMaxHalfPerLane];
  if (blockIdx.y > 0) {  // query head: norm + rope -> q_out
    const int t = (blockIdx.y - 1) * kProWarps + warp;
    if (t >= pr.Hq) return;
    norm_rope_head(pr.q_in, a.src_dtype, (int64_t)b * pr.q_stride + (int64_t)t * D, pr.q_norm_w, pr.norm_dtype,
                   pr.eps, pr.cos, pr.sin, pr.cs_dtype, cs_off, D, lane, lo, hi);
    const int64_t o = ((int64_t)b * pr.Hq + t) * D;
#pragma unroll
    for (int i = 0; i < kMaxHalfPerLane; ++i) {
      const int d = lane + 32 * i;
      if (d < half) {
        store_f(pr.q_out, a.src_dtype, o + d, lo[i]);
        store_f(pr.q_out, a.src_dtype, o + d + half, hi[i]);
      }
    }
    return;
  }
  if (!pr.do_append) return;
  if (threadIdx.x == 0) resolve_dest(a, b, blockIdx.x, s_pid, s_slot);
  for (int t = warp; t < 2 * a.Hkv; t += kProWarps) {
    float *row = kv_stage + (int64_t)t * D;
    if (t < a.Hkv) {  // key head: norm + rope
      norm_rope_head(a.k_new, a.src_dtype, (int64_t)b * pr.k_stride + (int64_t)t * D, pr.k_norm_w, pr.norm_dtype,
                     pr.eps, pr.cos, pr.sin, pr.cs_dtype, cs_off, D, lane, lo, hi);
#pragma unroll
      for (int i = 0; i < kMaxHalfPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < half) {
          row[d] = lo[i];
          row[d + half] = hi[i];
        }
      }
    } else {  // value head: as given
      const int64_t src = (int64_t)b * pr.v_stride + (int64_t)(t - a.Hkv) * D;
      for (int d = lane; d < D; d += 32) row[d] = load_f(a.v_new, a.src_dtype, src + d);
    }
  }
  __syncthreads();
  const int pid = s_pid, slot = s_slot;
  if (pid < 0) return;
  const int64_t base = (int64_t)pid * a.page_stride + (int64_t)slot * D;
  for (int i = threadIdx.x; i < 2 * a.Hkv * D; i += blockDim.x) {
    const int t = i / D, d = i - t * D;
    const bool is_k = t < a.Hkv;
    const int64_t dst = base + (int64_t)(is_k ? t : t - a.Hkv) * a.head_stride + d;
    store_f(is_k ? a.k_base : a.v_base, a.kv_dtype, dst, kv_stage[i]);
  }
}

}  // namespace helm

namespace helm {
namespace {

int check_append(const helm_kv_append_params *p, bool need_data) {
  if (!p) return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: params is null");
  if (p->B < 0 || p->Hkv <= 0 || p->D <= 0 || p->P <= 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: bad sizes B=%d Hkv=%d D=%d P=%d", p->B, p->Hkv, p->D, p->P);
  for (int dt : {p->src_dtype, p->kv_dtype})
    if (dt != HELM_F32 && dt != HELM_F16 && dt != HELM_BF16)
      return fail(HELM_ERR_UNSUPPORTED, "kv_append: dtype %d", dt);
  if (p->B == 0 || !need_data) return HELM_OK;
  if (!p->k_new || !p->v_new || !p->k_base || !p->v_base)
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: null data pointer");
  const bool directed = p->dest || p->dest_host;
  if (!directed && (!p->page_table || !p->page_used || !p->num_pages || !p->spare_pages || !p->spare_next))
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: device-directed mode needs page table and spare pages");
  if (directed && p->page_table && (!p->page_used || !p->num_pages))
    return fail(HELM_ERR_INVALID_ARGUMENT, "kv_append: page_table given without page_used/num_pages");
  return HELM_OK;
}

AppendArgs append_args(const helm_kv_append_params *p) {
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
  return a;
}

// Launches `launch(a, blocks)` once, or once per kHostDestRows sequences with the host-directed
// rows carried by value.
template <typename F>
int launch_rows(const helm_kv_append_params *p, AppendArgs a, F launch, const char *what) {
  if (!p->dest_host) {
    launch(a, p->B);
    return check_launch(what);
  }
  a.use_hdest = 1;
  for (int b0 = 0; b0 < p->B; b0 += kHostDestRows) {
    const int nb = p->B - b0 < kHostDestRows ? p->B - b0 : kHostDestRows;
    a.b0 = b0;
    for (int i = 0; i < nb; ++i)
      for (int j = 0; j < 3; ++j) a.hdest[i][j] = p->dest_host[3 * (b0 + i) + j];
    launch(a, nb);
    int rc = check_launch(what);
    if (rc != HELM_OK) return rc;
  }
  return HELM_OK;
}

}  // namespace
}  // namespace helm

extern "C" int helm_kv_append(const helm_kv_append_params *p, void *stream) {
  helm::NvtxRange nvtx_range_("helm_kv_append");
  using namespace helm;
  int rc = check_append(p, true);
  if (rc != HELM_OK || p->B == 0) return rc;
  cudaStream_t st = as_stream(stream);
  return launch_rows(p, append_args(p), [&](const AppendArgs &a, int blocks) {
    launch_pdl(kv_append_kernel, dim3(blocks), dim3(256), 0, st, a);
  }, "kv_append_kernel");
}

extern "C" int helm_decode_prologue(const helm_decode_prologue_params *p, void *stream) {
  helm::NvtxRange nvtx_range_("helm_decode_prologue");
  using namespace helm;
  if (!p) return fail(HELM_ERR_INVALID_ARGUMENT, "decode_prologue: params is null");
  const helm_kv_append_params *ap = &p->append;
  int rc = check_append(ap, p->do_append != 0);
  if (rc != HELM_OK) return rc;
  if (ap->B == 0) return HELM_OK;
  if (p->Hq <= 0 || p->Hq % ap->Hkv != 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "decode_prologue: Hq=%d not a positive multiple of Hkv=%d", p->Hq, ap->Hkv);
  if (ap->D % 2 != 0 || ap->D > 2 * 32 * kMaxHalfPerLane)
    return fail(HELM_ERR_UNSUPPORTED, "decode_prologue: head dim %d (even, <= 256)", ap->D);
  if (!p->q_in || !p->q_out) return fail(HELM_ERR_INVALID_ARGUMENT, "decode_prologue: null q pointer");
  if ((p->cos == nullptr) != (p->sin == nullptr))
    return fail(HELM_ERR_INVALID_ARGUMENT, "decode_prologue: cos and sin go together");
  if ((p->q_norm_w == nullptr) != (p->k_norm_w == nullptr))
    return fail(HELM_ERR_INVALID_ARGUMENT, "decode_prologue: q_norm and k_norm weights go together");
  for (int dt : {p->norm_dtype, p->cs_dtype})
    if (dt != HELM_F32 && dt != HELM_F16 && dt != HELM_BF16)
      return fail(HELM_ERR_UNSUPPORTED, "decode_prologue: dtype %d", dt);
  PrologueArgs pr{};
  pr.q_in = p->q_in;
  pr.q_out = p->q_out;
  pr.Hq = p->Hq;
  pr.q_stride = p->q_stride;
  pr.k_stride = p->k_stride;
  pr.v_stride = p->v_stride;
  pr.q_norm_w = p->q_norm_w;
  pr.k_norm_w = p->k_norm_w;
  pr.norm_dtype = p->norm_dtype;
  pr.eps = p->eps;
  pr.cos = p->cos;
  pr.sin = p->sin;
  pr.cs_dtype = p->cs_dtype;
  pr.cs_stride = p->cs_stride;
  pr.do_append = p->do_append;
  const size_t smem = p->do_append ? sizeof(float) * 2 * (size_t)ap->Hkv * ap->D : 0;
  if (smem > 200 * 1024)
    return fail(HELM_ERR_UNSUPPORTED, "decode_prologue: 2*Hkv*D = %d staged values exceed 200 KB", 2 * ap->Hkv * ap->D);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(decode_prologue_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "decode_prologue: %s", cudaGetErrorString(e));
  }
  cudaStream_t st = as_stream(stream);
  const unsigned qblocks = (unsigned)((p->Hq + kProWarps - 1) / kProWarps);
  return launch_rows(ap, append_args(ap), [&](const AppendArgs &a, int blocks) {
    launch_pdl(decode_prologue_kernel, dim3(blocks, 1 + qblocks), dim3(kProWarps * 32), smem, st, a, pr);
  }, "decode_prologue_kernel");
}
