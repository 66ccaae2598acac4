// Paged decode attention with split-KV partials and a log-sum-exp merge.
//
// Semantics follow HELM's perform_streaming_attention
// (helm/runtime/kv_cache.py:318-442): one query token per sequence, K/V read
// page by page, online softmax with fp32 running max / sum / output, pages
// with zero used tokens skipped, GQA by q head -> kv head hq / (Hq/Hkv),
// output o / clamp(l, 1e-12) cast to the output dtype.
//
// Two kernels compute the same partial records:
//   * attn_generic_kernel: CUDA cores, any page size / head dim <= 256 /
//     dtype (fp32, fp16, bf16).  Used for fp32 pages and odd shapes.
//   * attn_tc_kernel: bf16/fp16 pages of 64 tokens x 128 dims.  A producer
//     warp streams each page's K and V tiles with TMA (cp.async.bulk.tensor,
//     128B swizzle) into a 3-stage shared-memory ring guarded by mbarriers;
//     four consumer warps each own 16 tokens of a page and compute
//     S^T = K Q^T and O^T += V^T P^T with m16n8k16 tensor-core MMAs (the GQA
//     group is the N=8 dimension), keeping the online softmax in registers
//     with warp-shuffle max/sum reductions.  P is fed to the PV product as a
//     hi+lo pair of 16-bit values so the weights keep ~16 mantissa bits.
#include "common.cuh"
#include "tma.cuh"

#include <atomic>
#include <mutex>
#include <utility>
#include <vector>

namespace helm {

struct AttnArgs {
  const void *q;
  const void *k_base;
  const void *v_base;
  int64_t page_stride;
  int64_t head_stride;
  int32_t num_pool_pages;
  const int32_t *page_table;
  const int32_t *page_used;
  const int32_t *num_pages;
  int32_t pt_stride;
  int32_t B, Hq, Hkv, D, P, gq;
  int32_t head_chunks;   // warp kernel: CTAs per (split, kv head, sequence) along the GQA group
  int32_t q_dtype, out_dtype;
  float scale_log2;      // softmax scale * log2(e)
  int32_t num_splits;
  float *rec;            // split records [S][B*Hq][D+2] (null: none)
  float *out_record;     // merged record when S == 1 (null: none)
  void *out;             // normalised output when S == 1 (null: none)
  int32_t *error_flag;
};

// Page range [lo, hi) of split s for a sequence of n pages: balanced integer
// division, so every split gets floor(n/S) or ceil(n/S) pages.
__device__ __forceinline__ void split_range(int n, int s, int S, int &lo, int &hi) {
  lo = (int)(((int64_t)n * s) / S);
  hi = (int)(((int64_t)n * (s + 1)) / S);
}

__device__ __forceinline__ int read_num_pages(const AttnArgs &a, int b) {
  int n = a.num_pages[b];
  if (n < 0 || n > a.pt_stride) {
    flag_error(a.error_flag, HELM_DEVERR_NUM_PAGES);
    n = n < 0 ? 0 : a.pt_stride;
  }
  return n;
}

// Writes the CTA's result for query head hq, dim d: the unnormalised record
// (split or merged) and/or the normalised output.
__device__ __forceinline__ void emit(const AttnArgs &a, int split, int b, int hq, int d,
                                     float m, float l, float o) {
  const int rows = a.B * a.Hq;
  const int row = b * a.Hq + hq;
  const int rl = a.D + 2;
  if (a.rec) {
    float *r = a.rec + ((int64_t)split * rows + row) * rl;
    r[d] = o;
    if (d == 0) { r[a.D] = m; r[a.D + 1] = l; }
  }
  if (a.out_record) {
    float *r = a.out_record + (int64_t)row * rl;
    r[d] = o;
    if (d == 0) { r[a.D] = m; r[a.D + 1] = l; }
  }
  if (a.out) {
    float v = l > 0.f ? o / l : 0.f;
    store_f(a.out, a.out_dtype, (int64_t)row * a.D + d, v);
  }
}

// ===========================================================================
// Generic CUDA-core kernel.
// grid (S, Hkv, B), 128 threads.  Warp w handles pages lo+w, lo+w+4, ...;
// inside a page, lane t owns token t0+t for the scores and dim lane+32i for
// the P.V accumulation.  Per-warp (m, l, o) live in shared memory and are
// merged across warps at the end.
// ===========================================================================
constexpr int kGenWarps = 4;
constexpr int kGenHeadChunk = 8;
constexpr int kGenMaxDPL = 8;  // dims per lane: D <= 256

template <typename KT>
__global__ void __launch_bounds__(128) attn_generic_kernel(AttnArgs a) {
  extern __shared__ float smem_g[];
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = a.gq, D = a.D;

  float *q_s = smem_g;                                  // [gq][D]
  float *o_s = q_s + gq * D;                            // [4][gq][D]
  float *p_s = o_s + kGenWarps * gq * D;                // [4][32][gq]
  float *m_s = p_s + kGenWarps * 32 * gq;               // [4][gq]
  float *l_s = m_s + kGenWarps * gq;                    // [4][gq]
  float *al_s = l_s + kGenWarps * gq;                   // [4][gq]

  for (int i = threadIdx.x; i < gq * D; i += blockDim.x) {
    int h = i / D, d = i - h * D;
    q_s[i] = load_f(a.q, a.q_dtype, ((int64_t)(b * a.Hq + g * gq + h)) * D + d);
  }
  for (int i = threadIdx.x; i < kGenWarps * gq * D; i += blockDim.x) o_s[i] = 0.f;
  for (int i = threadIdx.x; i < kGenWarps * gq; i += blockDim.x) {
    m_s[i] = -INFINITY;
    l_s[i] = 0.f;
  }
  __syncthreads();

  const int n = read_num_pages(a, b);
  int lo, hi;
  split_range(n, s, a.num_splits, lo, hi);
  const KT *kb = reinterpret_cast<const KT *>(a.k_base);
  const KT *vb = reinterpret_cast<const KT *>(a.v_base);
  float *o_w = o_s + warp * gq * D;
  float *p_w = p_s + warp * 32 * gq;
  float *m_w = m_s + warp * gq;
  float *l_w = l_s + warp * gq;
  float *al_w = al_s + warp * gq;
  const int dpl = (D + 31) / 32;

  for (int pi = lo + warp; pi < hi; pi += kGenWarps) {
    const int pid = a.page_table[(int64_t)b * a.pt_stride + pi];
    const int used = a.page_used[(int64_t)b * a.pt_stride + pi];
    if (pid < 0 || pid >= a.num_pool_pages) {
      flag_error(a.error_flag, HELM_DEVERR_PAGE_ID);
      continue;
    }
    if (used < 0 || used > a.P) {
      flag_error(a.error_flag, HELM_DEVERR_PAGE_USED);
      continue;
    }
    const KT *kp = kb + (int64_t)pid * a.page_stride + (int64_t)g * a.head_stride;
    const KT *vp = vb + (int64_t)pid * a.page_stride + (int64_t)g * a.head_stride;
    for (int t0 = 0; t0 < used; t0 += 32) {
      const int t = t0 + lane;
      const bool valid = t < used;
      const int nt = min(32, used - t0);
      for (int h0 = 0; h0 < gq; h0 += kGenHeadChunk) {
        const int hc = min(kGenHeadChunk, gq - h0);
        float sc[kGenHeadChunk];
#pragma unroll
        for (int j = 0; j < kGenHeadChunk; ++j) sc[j] = 0.f;
        if (valid) {
          const KT *kr = kp + (int64_t)t * D;
          for (int d = 0; d < D; ++d) {
            const float kv = Elem<KT>::to_f(kr[d]);
#pragma unroll
            for (int j = 0; j < kGenHeadChunk; ++j)
              if (j < hc) sc[j] = fmaf(q_s[(h0 + j) * D + d], kv, sc[j]);
          }
        }
#pragma unroll
        for (int j = 0; j < kGenHeadChunk; ++j) {
          if (j >= hc) break;
          float v = valid ? sc[j] * a.scale_log2 : -INFINITY;
          float mx = v;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          const float m_old = m_w[h0 + j];
          const float m_new = fmaxf(m_old, mx);
          const float alpha = rescale_weight(m_old, m_new);
          const float p = valid ? fast_exp2(v - m_new) : 0.f;
          float ps = p;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
          p_w[lane * gq + h0 + j] = p;
          __syncwarp();
          if (lane == 0) {
            l_w[h0 + j] = l_w[h0 + j] * alpha + ps;
            m_w[h0 + j] = m_new;
            al_w[h0 + j] = alpha;
          }
          __syncwarp();
        }
        // o[h][d] = o[h][d] * alpha[h] + sum_t p[t][h] * v[t][d]
        float acc[kGenHeadChunk][kGenMaxDPL];
#pragma unroll
        for (int j = 0; j < kGenHeadChunk; ++j)
#pragma unroll
          for (int i = 0; i < kGenMaxDPL; ++i) {
            const int d = lane + 32 * i;
            acc[j][i] = (j < hc && i < dpl && d < D) ? o_w[(h0 + j) * D + d] * al_w[h0 + j] : 0.f;
          }
        for (int tt = 0; tt < nt; ++tt) {
          const KT *vr = vp + (int64_t)(t0 + tt) * D;
          float vv[kGenMaxDPL];
#pragma unroll
          for (int i = 0; i < kGenMaxDPL; ++i) {
            const int d = lane + 32 * i;
            vv[i] = (i < dpl && d < D) ? Elem<KT>::to_f(vr[d]) : 0.f;
          }
#pragma unroll
          for (int j = 0; j < kGenHeadChunk; ++j) {
            if (j >= hc) break;
            const float p = p_w[tt * gq + h0 + j];
#pragma unroll
            for (int i = 0; i < kGenMaxDPL; ++i) acc[j][i] = fmaf(p, vv[i], acc[j][i]);
          }
        }
#pragma unroll
        for (int j = 0; j < kGenHeadChunk; ++j)
#pragma unroll
          for (int i = 0; i < kGenMaxDPL; ++i) {
            const int d = lane + 32 * i;
            if (j < hc && i < dpl && d < D) o_w[(h0 + j) * D + d] = acc[j][i];
          }
        __syncwarp();
      }
    }
  }
  __syncthreads();

  // Merge the four warps' partial states.
  for (int i = threadIdx.x; i < gq * D; i += blockDim.x) {
    const int h = i / D, d = i - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kGenWarps; ++w) M = fmaxf(M, m_s[w * gq + h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kGenWarps; ++w) {
      const float wt = rescale_weight(m_s[w * gq + h], M);
      L = fmaf(l_s[w * gq + h], wt, L);
      O = fmaf(o_s[(w * gq + h) * D + d], wt, O);
    }
    if (M == -INFINITY) { L = 0.f; O = 0.f; }
    emit(a, s, b, g * gq + h, d, M, L, O);
  }
}

// ===========================================================================
// Warp-per-token-octet kernel (CUDA cores): fp32 pages, and 16-bit pages the
// tensor-core kernels do not take, for D = 32*DPL (DPL 1..8) and GQA group <= 8.
//
// grid (S, Hkv, B), 128 threads.  Lane l owns dims [l*DPL, l*DPL + DPL) of
// every row, so a K or V row is one coalesced 32*DPL-element load per warp.
// The split's pages are cut into octets of 8 tokens; warp w takes octets w,
// w+4, ... of each page.  Per octet a warp loads the 8 K and 8 V rows at once
// (many loads in flight per warp), forms the 8 x GQ scores with a butterfly
// sum over the lanes, and updates its running (m, l, o) with one rescale per
// octet.  The four warps' states are merged in shared memory at the end.
// ===========================================================================
constexpr int kWWarps = 4;
constexpr int kOct = 8;

// Adds one arrival to a token-tagged counter word and returns the arrivals after it; a word that
// carries another call's token (stale, or never written) counts as zero.
__device__ __forceinline__ uint32_t tagged_arrive(uint64_t *word, uint32_t tok) {
  unsigned long long old = *reinterpret_cast<volatile unsigned long long *>(word);
  for (;;) {
    const uint32_t cnt = (uint32_t)(old >> 32) == tok ? (uint32_t)old : 0u;
    const unsigned long long nw = ((unsigned long long)tok << 32) | (cnt + 1u);
    const unsigned long long prev = atomicCAS(reinterpret_cast<unsigned long long *>(word), old, nw);
    if (prev == old) return cnt + 1u;
    old = prev;
  }
}

template <typename KT, int DPL> struct RowLoad;
template <int DPL> struct RowLoad<float, DPL> {
  __device__ __forceinline__ static void run(const float *p, float (&v)[DPL]) {
    if constexpr (DPL % 4 == 0) {
#pragma unroll
      for (int j = 0; j < DPL; j += 4) {
        const float4 x = __ldg(reinterpret_cast<const float4 *>(p + j));
        v[j] = x.x; v[j + 1] = x.y; v[j + 2] = x.z; v[j + 3] = x.w;
      }
    } else if constexpr (DPL % 2 == 0) {
#pragma unroll
      for (int j = 0; j < DPL; j += 2) {
        const float2 x = __ldg(reinterpret_cast<const float2 *>(p + j));
        v[j] = x.x; v[j + 1] = x.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < DPL; ++j) v[j] = __ldg(p + j);
    }
  }
};
template <typename T16, int DPL> struct RowLoad16 {
  __device__ __forceinline__ static void run(const T16 *p, float (&v)[DPL]) {
    if constexpr (DPL % 8 == 0) {
#pragma unroll
      for (int j = 0; j < DPL; j += 8) {
        const uint4 x = __ldg(reinterpret_cast<const uint4 *>(p + j));
        const T16 *h = reinterpret_cast<const T16 *>(&x);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j + i] = Elem<T16>::to_f(h[i]);
      }
    } else if constexpr (DPL % 4 == 0) {
#pragma unroll
      for (int j = 0; j < DPL; j += 4) {
        const uint2 x = __ldg(reinterpret_cast<const uint2 *>(p + j));
        const T16 *h = reinterpret_cast<const T16 *>(&x);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[j + i] = Elem<T16>::to_f(h[i]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < DPL; ++j) v[j] = Elem<T16>::to_f(p[j]);
    }
  }
};
template <int DPL> struct RowLoad<__half, DPL> : RowLoad16<__half, DPL> {};
template <int DPL> struct RowLoad<__nv_bfloat16, DPL> : RowLoad16<__nv_bfloat16, DPL> {};

size_t warp_smem_bytes(int GQ, int D) { return sizeof(float) * (size_t)kWWarps * GQ * (D + 2); }

template <typename KT, int DPL, int GQ>
__global__ void __launch_bounds__(kWWarps * 32) attn_warp_kernel(AttnArgs a) {
  extern __shared__ float smem_w[];   // [warps][GQ][D] o, then [warps][GQ] m, [warps][GQ] l
  constexpr int D = 32 * DPL;
  // blockIdx.y = (kv head g, head chunk): this CTA serves query heads [h0, h0 + gn) of g's group.
  const int s = blockIdx.x, g = blockIdx.y / a.head_chunks, b = blockIdx.z;
  const int h0 = (blockIdx.y - g * a.head_chunks) * GQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = a.gq, gn = min(GQ, gq - h0), hq0 = g * gq + h0;
  float *o_s = smem_w;
  float *m_s = o_s + kWWarps * GQ * D;
  float *l_s = m_s + kWWarps * GQ;

  pdl_trigger();
  pdl_wait();

  // q of the group, this lane's dims, pre-scaled into the base-2 logit domain.
  float q[GQ][DPL];
#pragma unroll
  for (int h = 0; h < GQ; ++h)
#pragma unroll
    for (int j = 0; j < DPL; ++j)
      q[h][j] = h < gn ? load_f(a.q, a.q_dtype, ((int64_t)b * a.Hq + hq0 + h) * D + lane * DPL + j) * a.scale_log2
                       : 0.f;
  float m[GQ], l[GQ], o[GQ][DPL];
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) o[h][j] = 0.f;
  }

  const int n = read_num_pages(a, b);
  int lo, hi;
  split_range(n, s, a.num_splits, lo, hi);
  const KT *kb = reinterpret_cast<const KT *>(a.k_base);
  const KT *vb = reinterpret_cast<const KT *>(a.v_base);
  for (int pi = lo; pi < hi; ++pi) {
    const int pid = a.page_table[(int64_t)b * a.pt_stride + pi];
    const int used = a.page_used[(int64_t)b * a.pt_stride + pi];
    if (pid < 0 || pid >= a.num_pool_pages) {
      if (lane == 0 && warp == 0) flag_error(a.error_flag, HELM_DEVERR_PAGE_ID);
      continue;
    }
    if (used < 0 || used > a.P) {
      if (lane == 0 && warp == 0) flag_error(a.error_flag, HELM_DEVERR_PAGE_USED);
      continue;
    }
    const KT *kp = kb + (int64_t)pid * a.page_stride + (int64_t)g * a.head_stride + lane * DPL;
    const KT *vp = vb + (int64_t)pid * a.page_stride + (int64_t)g * a.head_stride + lane * DPL;
    for (int t0 = warp * kOct; t0 < used; t0 += kWWarps * kOct) {
      const int nt = min(kOct, used - t0);
      float kr[kOct][DPL], vr[kOct][DPL];
#pragma unroll
      for (int t = 0; t < kOct; ++t) {
        if (t < nt) {
          RowLoad<KT, DPL>::run(kp + (int64_t)(t0 + t) * D, kr[t]);
          RowLoad<KT, DPL>::run(vp + (int64_t)(t0 + t) * D, vr[t]);
        } else {
#pragma unroll
          for (int j = 0; j < DPL; ++j) kr[t][j] = vr[t][j] = 0.f;
        }
      }
      // scores: lane partials over its dims, summed over the warp (every lane gets every score)
      float sc[GQ][kOct];
#pragma unroll
      for (int h = 0; h < GQ; ++h)
#pragma unroll
        for (int t = 0; t < kOct; ++t) {
          float acc = 0.f;
#pragma unroll
          for (int j = 0; j < DPL; ++j) acc = fmaf(q[h][j], kr[t][j], acc);
          sc[h][t] = acc;
        }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int h = 0; h < GQ; ++h)
#pragma unroll
          for (int t = 0; t < kOct; ++t) sc[h][t] += __shfl_xor_sync(0xffffffffu, sc[h][t], off);
#pragma unroll
      for (int h = 0; h < GQ; ++h) {
        if (h >= gn) break;
        float mx = m[h];
#pragma unroll
        for (int t = 0; t < kOct; ++t)
          if (t < nt) mx = fmaxf(mx, sc[h][t]);
        const float alpha = rescale_weight(m[h], mx);
        m[h] = mx;
        float ps = 0.f;
        float acc[DPL];
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[j] = o[h][j] * alpha;
#pragma unroll
        for (int t = 0; t < kOct; ++t) {
          const float p = t < nt ? fast_exp2(sc[h][t] - mx) : 0.f;
          ps += p;
#pragma unroll
          for (int j = 0; j < DPL; ++j) acc[j] = fmaf(p, vr[t][j], acc[j]);
        }
        l[h] = fmaf(l[h], alpha, ps);
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[h][j] = acc[j];
      }
    }
  }

  // merge the warps' states
#pragma unroll
  for (int h = 0; h < GQ; ++h) {
#pragma unroll
    for (int j = 0; j < DPL; ++j) o_s[(warp * GQ + h) * D + lane * DPL + j] = o[h][j];
    if (lane == 0) {
      m_s[warp * GQ + h] = m[h];
      l_s[warp * GQ + h] = l[h];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < gn * D; i += blockDim.x) {
    const int h = i / D, d = i - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWWarps; ++w) M = fmaxf(M, m_s[w * GQ + h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWWarps; ++w) {
      const float wt = rescale_weight(m_s[w * GQ + h], M);
      L = fmaf(l_s[w * GQ + h], wt, L);
      O = fmaf(o_s[(w * GQ + h) * D + d], wt, O);
    }
    if (M == -INFINITY) { L = 0.f; O = 0.f; }
    emit(a, s, b, hq0 + h, d, M, L, O);
  }
}

// ===========================================================================
// TMA + tensor-core kernel (bf16 / fp16 pages, P = 64, D = 128).
// ===========================================================================
namespace tc {

constexpr int P = 64;
constexpr int D = 128;
constexpr int kStages = 3;
constexpr int kHalfBytes = P * 128;            // 64 rows x 128 B (64 dims)
constexpr int kTileBytes = 2 * kHalfBytes;     // one K or V tile: 16 KB
constexpr int kStageBytes = 2 * kTileBytes;    // K + V: 32 KB
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  // Packs (x, y) and their rounding residuals as bf16x2.
  __device__ __forceinline__ static void split(float x, float y, uint32_t &hi, uint32_t &lo) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    float2 hf = __bfloat1622float2(h);
    __nv_bfloat162 l = __floats2bfloat162_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<uint32_t *>(&h);
    lo = *reinterpret_cast<uint32_t *>(&l);
  }
};
template <> struct Mma<__half> {
  __device__ __forceinline__ static void run(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static void split(float x, float y, uint32_t &hi, uint32_t &lo) {
    __half2 h = __floats2half2_rn(x, y);
    float2 hf = __half22float2(h);
    __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<uint32_t *>(&h);
    lo = *reinterpret_cast<uint32_t *>(&l);
  }
};

// Byte offset of 16-byte chunk `chunk` (0..15, i.e. dims 8*chunk..8*chunk+7)
// of row `row` inside one tile stored as two 64-dim halves with the TMA
// 128-byte swizzle (chunk index XOR row % 8 within each 128-byte row).
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  const int half = chunk >> 3, c = chunk & 7;
  return half * kHalfBytes + row * 128 + ((c ^ (row & 7)) << 4);
}

template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ int stage_used[kStages];
  __shared__ float m_x[kConsumerWarps][NT * 8];
  __shared__ float l_x[kConsumerWarps][NT * 8];

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = a.gq;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kConsumerWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const int n = read_num_pages(a, b);
  int lo, hi;
  split_range(n, s, a.num_splits, lo, hi);
  const int npages = hi - lo;
  const int32_t *pt = a.page_table + (int64_t)b * a.pt_stride;
  const int32_t *pu = a.page_used + (int64_t)b * a.pt_stride;

  if (warp == kConsumerWarps) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < npages && ok; ++i) {
        const int st = i % kStages;
        if (i >= kStages && !mbar_wait(&empty_bar[st], ((i / kStages) - 1) & 1)) {
          flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
          ok = false;
          break;
        }
        const int pid = pt[lo + i];
        int used = pu[lo + i];
        if (pid < 0 || pid >= a.num_pool_pages) {
          flag_error(a.error_flag, HELM_DEVERR_PAGE_ID);
          used = 0;
        } else if (used < 0 || used > P) {
          flag_error(a.error_flag, HELM_DEVERR_PAGE_USED);
          used = 0;
        }
        stage_used[st] = used;
        if (used > 0) {
          uint8_t *kd = smem + st * kStageBytes;
          uint8_t *vd = kd + kTileBytes;
          mbar_arrive_expect_tx(&full_bar[st], kStageBytes);
          tma_load_4d(kd, &tmK, &full_bar[st], 0, 0, g, pid);
          tma_load_4d(kd + kHalfBytes, &tmK, &full_bar[st], 64, 0, g, pid);
          tma_load_4d(vd, &tmV, &full_bar[st], 0, 0, g, pid);
          tma_load_4d(vd + kHalfBytes, &tmV, &full_bar[st], 64, 0, g, pid);
        } else {
          mbar_arrive(&full_bar[st]);
        }
        issued = i + 1;
      }
      // Before the CTA can exit, every copy it issued must have landed.
      const int first = issued > kStages ? issued - kStages : 0;
      for (int i = first; i < issued; ++i)
        if (!mbar_wait(&full_bar[i % kStages], (i / kStages) & 1)) flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
    }
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int r = lane >> 2, c = lane & 3;
  uint32_t qf[NT][8][2];
  {
    const T *qp = reinterpret_cast<const T *>(a.q) + ((int64_t)b * a.Hq + (int64_t)g * gq) * D;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int h = nt * 8 + r;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (h < gq) {
          qf[nt][j][0] = *reinterpret_cast<const uint32_t *>(qp + h * D + 16 * j + 2 * c);
          qf[nt][j][1] = *reinterpret_cast<const uint32_t *>(qp + h * D + 16 * j + 2 * c + 8);
        } else {
          qf[nt][j][0] = 0u;
          qf[nt][j][1] = 0u;
        }
      }
    }
  }
  float o[NT][8][4];
  float m_run[NT][2], l_run[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int dt = 0; dt < 8; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nt][dt][e] = 0.f;
    m_run[nt][0] = m_run[nt][1] = -INFINITY;
    l_run[nt][0] = l_run[nt][1] = 0.f;
  }

  const int row0 = warp * 16;  // this warp's 16 tokens of every page
  const int mi = lane >> 3, ri = lane & 7;
  bool alive = true;
  for (int i = 0; i < npages && alive; ++i) {
    const int st = i % kStages;
    if (!mbar_wait(&full_bar[st], (i / kStages) & 1)) {
      flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
      alive = false;
      break;
    }
    const int used = stage_used[st];
    const int nvalid = min(16, used - row0);
    if (nvalid > 0) {
      uint8_t *kt = smem + st * kStageBytes;
      uint8_t *vt = kt + kTileBytes;
      if (nvalid < 16) {
        // Rows past `used` hold stale data (possibly NaN bit patterns): zero
        // this warp's invalid V rows so that 0-weight x V stays 0.
        for (int idx = lane; idx < (16 - nvalid) * 16; idx += 32) {
          const int rr = row0 + nvalid + idx / 16;
          const int q16 = idx % 16;
          *reinterpret_cast<uint4 *>(vt + (q16 >> 3) * kHalfBytes + rr * 128 + (q16 & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
      const uint32_t kbase = smem_u32(kt), vbase = smem_u32(vt);
      // S^T[16 tok x 8 heads] = K[16 x 128] * Q^T[128 x 8]
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t a0, a1, a2, a3;
        const int row = row0 + ri + (mi & 1) * 8;
        ldsm_x4(kbase + tile_off(row, 2 * j + (mi >> 1)), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<T>::run(sc[nt], a0, a1, a2, a3, qf[nt][j][0], qf[nt][j][1]);
      }
      const bool v_lo = r < nvalid, v_hi = r + 8 < nvalid;
      uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float x0 = v_lo ? sc[nt][0] * a.scale_log2 : -INFINITY;
        const float x1 = v_lo ? sc[nt][1] * a.scale_log2 : -INFINITY;
        const float x2 = v_hi ? sc[nt][2] * a.scale_log2 : -INFINITY;
        const float x3 = v_hi ? sc[nt][3] * a.scale_log2 : -INFINITY;
        float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, off));
          t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, off));
        }
        const float mn0 = fmaxf(m_run[nt][0], t0), mn1 = fmaxf(m_run[nt][1], t1);
        const float al0 = rescale_weight(m_run[nt][0], mn0), al1 = rescale_weight(m_run[nt][1], mn1);
        m_run[nt][0] = mn0;
        m_run[nt][1] = mn1;
        const float p0 = v_lo ? fast_exp2(x0 - mn0) : 0.f;
        const float p1 = v_lo ? fast_exp2(x1 - mn1) : 0.f;
        const float p2 = v_hi ? fast_exp2(x2 - mn0) : 0.f;
        const float p3 = v_hi ? fast_exp2(x3 - mn1) : 0.f;
        l_run[nt][0] = fmaf(l_run[nt][0], al0, p0 + p2);
        l_run[nt][1] = fmaf(l_run[nt][1], al1, p1 + p3);
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          o[nt][dt][0] *= al0;
          o[nt][dt][1] *= al1;
          o[nt][dt][2] *= al0;
          o[nt][dt][3] *= al1;
        }
        uint32_t h01, l01, h23, l23;
        Mma<T>::split(p0, p1, h01, l01);
        Mma<T>::split(p2, p3, h23, l23);
        bh[nt][0] = movm_t(h01);
        bh[nt][1] = movm_t(h23);
        bl[nt][0] = movm_t(l01);
        bl[nt][1] = movm_t(l23);
      }
      // O^T[128 dims x 8 heads] += V^T[128 x 16 tok] * P^T[16 tok x 8 heads]
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        uint32_t a0, a1, a2, a3;
        const int row = row0 + ri + (mi >> 1) * 8;
        ldsm_x4_t(vbase + tile_off(row, 2 * dt + (mi & 1)), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          Mma<T>::run(o[nt][dt], a0, a1, a2, a3, bh[nt][0], bh[nt][1]);
          Mma<T>::run(o[nt][dt], a0, a1, a2, a3, bl[nt][0], bl[nt][1]);
        }
      }
      if (nvalid < 16) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[st]);
  }

  // l is a per-thread partial over this thread's rows: sum the 8 lanes that
  // share the same head pair.
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float v = l_run[nt][e];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      l_run[nt][e] = v;
    }

  // All consumer warps must be done with the stage buffers before they are
  // reused as merge scratch.
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
  float *o_x = reinterpret_cast<float *>(smem);  // [4][NT*8][128]
  constexpr int HN = NT * 8;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h0 = nt * 8 + 2 * c;
    if (r == 0) {
      m_x[warp][h0] = m_run[nt][0];
      m_x[warp][h0 + 1] = m_run[nt][1];
      l_x[warp][h0] = l_run[nt][0];
      l_x[warp][h0 + 1] = l_run[nt][1];
    }
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      const int d = dt * 16 + r;
      o_x[(warp * HN + h0) * D + d] = o[nt][dt][0];
      o_x[(warp * HN + h0 + 1) * D + d] = o[nt][dt][1];
      o_x[(warp * HN + h0) * D + d + 8] = o[nt][dt][2];
      o_x[(warp * HN + h0 + 1) * D + d + 8] = o[nt][dt][3];
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
  for (int idx = threadIdx.x; idx < gq * D; idx += kConsumerWarps * 32) {
    const int h = idx / D, d = idx - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, m_x[w][h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float wt = rescale_weight(m_x[w][h], M);
      L = fmaf(l_x[w][h], wt, L);
      O = fmaf(o_x[(w * HN + h) * D + d], wt, O);
    }
    if (M == -INFINITY) { L = 0.f; O = 0.f; }
    emit(a, s, b, g * gq + h, d, M, L, O);
  }
}

// ---------------------------------------------------------------------------
// Persistent, work-balanced variant (stream-K over pages).
//
// The work is the flat list of units u = (sequence b, kv head g, page i) in
// b-major, g, i order; CTA c of C owns units [c*U/C, (c+1)*U/C), so every CTA
// streams the same number of pages and its TMA pipeline stays full across
// (b, g) boundaries.  A maximal run of units of one (b, g) pair inside a CTA is
// a segment.  At a segment end the four consumer warps merge their states into
// one CTA record of the pair (through the just-consumed stage buffer, which is
// held back from the producer until then), store it at slot c + pair of the
// workspace (unique: a later CTA never starts at an earlier pair) and bump the
// pair's arrival counter.  The CTA that completes a pair's count merges all of
// its CTA records after finishing its own units (chunked online log-sum-exp,
// fixed CTA order), so a single launch yields the attention output.
// ---------------------------------------------------------------------------
constexpr int kMaxSeqs = 512;
constexpr int kMaxPending = 64;  // deferred merges per CTA

struct PersistArgs {
  float *rec_o;        // [C + pairs][gq][D]: CTA c's unnormalised o for pair p at slot c + p
  float *rec_ml;       // [C + pairs][gq][2]: its (m, l)
  uint64_t *counter;   // [pairs]: (call token << 32) | arrivals; a word with another token counts 0
  uint32_t token;      // this call's token (host-issued; a captured graph replays its own)
  int C;               // grid size
  // Fused cross-GPU exchange (xworld > 1).  Receive slots of every rank: [2][G][B*Hq][D+2] words
  // of 64 bits, each one value (o[0..D), m, l) in the low half and the call's epoch in the high
  // half, so a reader knows a word has arrived from the word itself (no fence, no flag).
  int xrank, xworld;
  uint64_t *xrecv[HELM_MAX_RANKS];
  uint64_t *xrecv_local;
  uint32_t *xsent;                  // [pairs]: exchanges done per pair (epoch of the next is +1)
  uint64_t xwait_ns;                // bound of each wait for peers' words
};

constexpr uint64_t kExchangeWaitNs = 2000000000ull;


__device__ __forceinline__ uint64_t ll_word(float v, uint32_t epoch) {
  return ((uint64_t)epoch << 32) | __float_as_uint(v);
}

__device__ __forceinline__ void st_volatile_v2_u64(uint64_t *p, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void ld_volatile_v2_u64(const uint64_t *p, uint64_t &a, uint64_t &b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ bool ll_ok(uint64_t w, uint32_t epoch) { return (uint32_t)(w >> 32) == epoch; }

// CTA owning unit u when U units are split over C CTAs as [c*U/C, (c+1)*U/C).
__device__ __forceinline__ int owner_cta(int64_t u, int64_t U, int C) {
  return (int)(((u + 1) * (int64_t)C - 1) / U);
}

template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 2)
    attn_tc_persistent_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                              AttnArgs a, PersistArgs pa) {
  constexpr int HN = NT * 8;        // padded heads per kv head
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ int stage_used[kStages];
  __shared__ int stage_pair[kStages];
  __shared__ int stage_last[kStages];
  __shared__ int seq_prefix[kMaxSeqs + 1];  // units before sequence b
  __shared__ int seq_pages[kMaxSeqs];
  __shared__ float m_x[kConsumerWarps][HN];
  __shared__ float l_x[kConsumerWarps][HN];
  __shared__ float mg_m[HN][32];    // merge chunk: maxima, then weights
  __shared__ float mg_l[HN][32];
  __shared__ float mg_M[HN], mg_L[HN], mg_A[HN];
  __shared__ int pending[kMaxPending];
  __shared__ int npending;
  __shared__ uint32_t xs_epoch;
  __shared__ int xs_dead;  // a wait of this CTA ran out: later exchanges do not wait again
  __shared__ uint64_t *xs_peer[HELM_MAX_RANKS];  // pa.xrecv (dynamic indexing of a kernel parameter array
                                                 // would copy it to local memory)

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int c = blockIdx.x;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int gq = a.gq, B = a.B, Hkv = a.Hkv;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], kConsumerWarps);
    }
    npending = 0;
    xs_dead = 0;
#pragma unroll
    for (int r = 0; r < HELM_MAX_RANKS; ++r) xs_peer[r] = pa.xrecv[r];
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmK)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmV)) : "memory");
  }
  // Launched with programmatic dependent launch: everything above overlapped the previous
  // kernel; page tables, q, the workspace and the outputs are touched only after it finished.
  pdl_trigger();
  pdl_wait();
  // Units per sequence and their prefix sums (warp 0: chunked scan).
  if (warp == 0) {
    const int per = (B + 31) / 32;
    int local = 0;
    for (int j = 0; j < per; ++j) {
      const int b = lane * per + j;
      if (b < B) {
        const int n = read_num_pages(a, b);
        seq_pages[b] = n;
        local += n * Hkv;
      }
    }
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - local;
    for (int j = 0; j < per; ++j) {
      const int b = lane * per + j;
      if (b < B) {
        seq_prefix[b] = run;
        run += seq_pages[b] * Hkv;
      }
    }
    if (lane == 31) seq_prefix[B] = incl;
  }
  __syncthreads();
  const int64_t U = seq_prefix[B];
  // With fewer units than CTAs only the first U CTAs work, so every working CTA owns >= 1 unit
  // and the CTAs between a pair's first and last owner all hold some of its units.
  const int C = U < (int64_t)pa.C ? (int)U : pa.C;
  int64_t u0 = 0, u1 = 0;
  if (c < C) {
    u0 = U * c / C;
    u1 = U * (c + 1) / C;
  }

  // (sequence, kv head) pair of unit u: the last b with seq_prefix[b] <= u (and pages > 0)
  auto unit_pair = [&](int64_t u) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seq_prefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    int b = lo;
    while (seq_pages[b] == 0 && b > 0) --b;
    return b * Hkv + (int)((u - seq_prefix[b]) / seq_pages[b]);
  };

  if (warp == kConsumerWarps) {
    // ------------------------------ producer ------------------------------
    // The 32 lanes decode and fetch the (page id, used, pair, last) of the next 32 units ahead of
    // time (double-buffered), so a freed stage gets its TMA issued without a dependent load.
    if (u1 > u0) {
      auto fetch = [&](int64_t u, int &pid, int &used, int &pair, int &last) {
        pid = -1;
        used = 0;
        pair = 0;
        last = 0;
        if (u >= u1) return;
        int lo = 0, hi = B - 1;  // last b with seq_prefix[b] <= u and pages > 0
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (seq_prefix[mid] <= u) lo = mid; else hi = mid - 1;
        }
        int b = lo;
        while (seq_pages[b] == 0 && b > 0) --b;
        const int n = seq_pages[b];
        const int rem = (int)(u - seq_prefix[b]);
        const int g = rem / n, pi = rem - g * n;
        pid = a.page_table[(int64_t)b * a.pt_stride + pi];
        used = a.page_used[(int64_t)b * a.pt_stride + pi];
        pair = b * Hkv + g;
        last = (pi == n - 1) || (u + 1 == u1);
      };
      int c_pid, c_used, c_pair, c_last;  // current batch of 32 units, one per lane
      int n_pid, n_used, n_pair, n_last;  // next batch
      fetch(u0 + lane, c_pid, c_used, c_pair, c_last);
      fetch(u0 + 32 + lane, n_pid, n_used, n_pair, n_last);
      int issued = 0;
      bool ok = true;
      const int64_t n_units = u1 - u0;
      for (int64_t i = 0; i < n_units; ++i) {
        const int k = (int)(i & 31);
        if (k == 0 && i > 0) {
          c_pid = n_pid;
          c_used = n_used;
          c_pair = n_pair;
          c_last = n_last;
          fetch(u0 + i + 32 + lane, n_pid, n_used, n_pair, n_last);
        }
        const int pid = __shfl_sync(0xffffffffu, c_pid, k);
        int used = __shfl_sync(0xffffffffu, c_used, k);
        const int pair = __shfl_sync(0xffffffffu, c_pair, k);
        const int last = __shfl_sync(0xffffffffu, c_last, k);
        const int st = (int)(i % kStages);
        if (lane == 0) {
          if (i >= kStages && !mbar_wait(&empty_bar[st], (uint32_t)(((i / kStages) - 1) & 1))) {
            flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
            ok = false;
          } else {
            if (pid < 0 || pid >= a.num_pool_pages) {
              flag_error(a.error_flag, HELM_DEVERR_PAGE_ID);
              used = 0;
            } else if (used < 0 || used > P) {
              flag_error(a.error_flag, HELM_DEVERR_PAGE_USED);
              used = 0;
            }
            stage_used[st] = used;
            stage_pair[st] = pair;
            stage_last[st] = last;
            if (used > 0) {
              const int g = pair % Hkv;
              uint8_t *kd = smem + st * kStageBytes;
              uint8_t *vd = kd + kTileBytes;
              mbar_arrive_expect_tx(&full_bar[st], kStageBytes);
              tma_load_4d(kd, &tmK, &full_bar[st], 0, 0, g, pid);
              tma_load_4d(kd + kHalfBytes, &tmK, &full_bar[st], 64, 0, g, pid);
              tma_load_4d(vd, &tmV, &full_bar[st], 0, 0, g, pid);
              tma_load_4d(vd + kHalfBytes, &tmV, &full_bar[st], 64, 0, g, pid);
            } else {
              mbar_arrive(&full_bar[st]);
            }
            issued = (int)i + 1;
          }
        }
        if (!__shfl_sync(0xffffffffu, (int)ok, 0)) break;
      }
      if (lane == 0) {
        const int first = issued > kStages ? issued - kStages : 0;
        for (int i = first; i < issued; ++i)
          if (!mbar_wait(&full_bar[i % kStages], (i / kStages) & 1)) flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
      }
    }
  } else {
    // ------------------------------ consumers -------------------------------
    const int r = lane >> 2, cq = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    const int row0 = warp * 16;
    uint32_t qf[NT][8][2];
    float o[NT][8][4];
    float m_run[NT][2], l_run[NT][2];
    int cur_pair = -1;

    auto load_q = [&](int pair) {
      const int b = pair / Hkv, g = pair - b * Hkv;
      const T *qp = reinterpret_cast<const T *>(a.q) + ((int64_t)b * a.Hq + (int64_t)g * gq) * D;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int h = nt * 8 + r;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          qf[nt][j][0] = h < gq ? *reinterpret_cast<const uint32_t *>(qp + h * D + 16 * j + 2 * cq) : 0u;
          qf[nt][j][1] = h < gq ? *reinterpret_cast<const uint32_t *>(qp + h * D + 16 * j + 2 * cq + 8) : 0u;
        }
      }
    };
    auto reset_state = [&]() {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int dt = 0; dt < 8; ++dt)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[nt][dt][e] = 0.f;
        m_run[nt][0] = m_run[nt][1] = -INFINITY;
        l_run[nt][0] = l_run[nt][1] = 0.f;
      }
    };
    reset_state();

    // Emits pair (b, g) from its rank-local record: mg_M / mg_L (per head) and acc (this thread's
    // float4 slice of o).  With the exchange on, the record first goes to every rank and the G
    // records are merged in rank order.
    auto exchange_emit = [&](int pair, int b, int g, const float4 (&acc)[HN / 4]) {
      constexpr int F4x = HN / 4;
      if (pa.xworld <= 1) {
#pragma unroll
        for (int e = 0; e < F4x; ++e) {
          const int idx4 = tid + e * kConsumerWarps * 32;
          if (idx4 < gq * (D / 4)) {
            const int h = idx4 / (D / 4), d = (idx4 - h * (D / 4)) * 4;
            const float M = mg_M[h];
            const float L = M == -INFINITY ? 0.f : mg_L[h];
            const float vals[4] = {acc[e].x, acc[e].y, acc[e].z, acc[e].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) emit(a, 0, b, g * gq + h, d + j, M, L, M == -INFINITY ? 0.f : vals[j]);
          }
        }
        return;
      }
      // Exchange: this rank's record of the pair goes to every other rank as 64-bit words
      // (value | epoch << 32), then the G records are merged in rank order (the own one from
      // registers), exactly as helm_lse_merge merges them.  Row layout (D + 2 words): o[4c], o[4c+1]
      // at words 2c, 2c+1; o[4c+2], o[4c+3] at D/2 + 2c, D/2 + 2c + 1; then m, l -- so a warp's
      // 16-byte stores (and the readers' loads) cover 512 contiguous bytes.  Slot parity (epoch & 1)
      // keeps call n+1's words from overwriting call n's before every reader is done: a rank
      // starts call n+1 only after its call n received every rank's words of call n, which each
      // rank sends after it finished reading call n-1.
      const int G = pa.xworld, R = pa.xrank;
      const int64_t rows = (int64_t)B * a.Hq;
      constexpr int XW = D + 2;
      if (tid == 0) {
        xs_epoch = pa.xsent[pair] + 1;
        if (*(volatile int *)a.error_flag == HELM_DEVERR_TIMEOUT) xs_dead = 1;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
      const uint32_t ep = xs_epoch;
      const int64_t slot_base = (int64_t)(ep & 1u) * G;
#pragma unroll
      for (int e = 0; e < F4x; ++e) {
        const int idx4 = tid + e * kConsumerWarps * 32;
        if (idx4 < gq * (D / 4)) {
          const int h = idx4 / (D / 4), cq = idx4 - h * (D / 4);
          const float M = mg_M[h];
          const bool empty = M == -INFINITY;
          const float4 v = empty ? make_float4(0.f, 0.f, 0.f, 0.f) : acc[e];
          const uint64_t w0 = ll_word(v.x, ep), w1 = ll_word(v.y, ep), w2 = ll_word(v.z, ep),
                         w3 = ll_word(v.w, ep);
          const uint64_t wm = ll_word(M, ep), wl = ll_word(empty ? 0.f : mg_L[h], ep);
          const int64_t off = ((slot_base + R) * rows + (int64_t)b * a.Hq + g * gq + h) * XW;
          for (int k = 1; k < G; ++k) {
            const int dst = R + k < G ? R + k : R + k - G;  // spread the first stores over peers
            uint64_t *row = xs_peer[dst] + off;
            st_volatile_v2_u64(row + 2 * cq, w0, w1);
            st_volatile_v2_u64(row + D / 2 + 2 * cq, w2, w3);
            if (cq == 0) st_volatile_v2_u64(row + D, wm, wl);
          }
        }
      }
#pragma unroll
      for (int e = 0; e < F4x; ++e) {
        const int idx4 = tid + e * kConsumerWarps * 32;
        if (idx4 < gq * (D / 4)) {
          const int h = idx4 / (D / 4), cq = idx4 - h * (D / 4);
          const int64_t row = (int64_t)b * a.Hq + g * gq + h;
          const float own_M = mg_M[h];
          const bool own_empty = own_M == -INFINITY;
          // Every rank's words of this thread's slice, loaded four ranks at a time (register
          // budget) and re-polled (bounded) until all carry this call's epoch.
          float m_t[HELM_MAX_RANKS], l_t[HELM_MAX_RANKS];
          float4 o_t[HELM_MAX_RANKS];
          bool ok = true;
          uint64_t t0 = 0;
          bool timed = false;
#pragma unroll
          for (int t_lo = 0; t_lo < HELM_MAX_RANKS; t_lo += 4) {
            while (ok) {
              bool all = true;
#pragma unroll
              for (int t = t_lo; t < t_lo + 4; ++t) {
                if (t < G && t != R) {
                  const uint64_t *src = pa.xrecv_local + ((slot_base + t) * rows + row) * XW;
                  uint64_t wm, wl, w0, w1, w2, w3;
                  ld_volatile_v2_u64(src + D, wm, wl);
                  ld_volatile_v2_u64(src + 2 * cq, w0, w1);
                  ld_volatile_v2_u64(src + D / 2 + 2 * cq, w2, w3);
                  m_t[t] = __uint_as_float((uint32_t)wm);
                  l_t[t] = __uint_as_float((uint32_t)wl);
                  o_t[t] = make_float4(__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1),
                                       __uint_as_float((uint32_t)w2), __uint_as_float((uint32_t)w3));
                  all = all && ll_ok(wm, ep) && ll_ok(wl, ep) && ll_ok(w0, ep) && ll_ok(w1, ep) &&
                        ll_ok(w2, ep) && ll_ok(w3, ep);
                } else {
                  m_t[t] = own_M;
                  l_t[t] = own_empty ? 0.f : mg_L[h];
                  o_t[t] = own_empty ? make_float4(0.f, 0.f, 0.f, 0.f) : acc[e];
                }
              }
              if (all) break;
              if (*(volatile int *)&xs_dead) {
                ok = false;
                break;
              }
              if (!timed) {
                t0 = global_ns();
                timed = true;
              } else if (global_ns() - t0 > pa.xwait_ns) {
                ok = false;
                break;
              }
            }
          }
          float M = -INFINITY;
#pragma unroll
          for (int t = 0; t < HELM_MAX_RANKS; ++t)
            if (t < G && ok) M = fmaxf(M, m_t[t]);
          float L = 0.f;
          float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int t = 0; t < HELM_MAX_RANKS; ++t) {
            if (t >= G || !ok) continue;
            const float w = rescale_weight(m_t[t], M);
            L = fmaf(l_t[t], w, L);
            O.x = fmaf(o_t[t].x, w, O.x);
            O.y = fmaf(o_t[t].y, w, O.y);
            O.z = fmaf(o_t[t].z, w, O.z);
            O.w = fmaf(o_t[t].w, w, O.w);
          }
          if (!ok) {
            flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
            xs_dead = 1;
          }
          const bool none = M == -INFINITY || !ok;
          const int d = cq * 4;
          const float vals[4] = {O.x, O.y, O.z, O.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) emit(a, 0, b, g * gq + h, d + j, M, none ? 0.f : L, none ? 0.f : vals[j]);
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
      if (tid == 0) pa.xsent[pair] = ep;
    };

    const int64_t n_units = u1 - u0;
    if (n_units > 0) {  // the first pair's q loads while the producer fetches page ids and K/V
      cur_pair = unit_pair(u0);
      load_q(cur_pair);
    }
    for (int64_t i = 0; i < n_units; ++i) {
      const int st = (int)(i % kStages);
      if (!mbar_wait(&full_bar[st], (uint32_t)((i / kStages) & 1))) {
        flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
        break;
      }
      const int used = stage_used[st];
      const int pair = stage_pair[st];
      const int last = stage_last[st];
      if (pair != cur_pair) {
        load_q(pair);
        cur_pair = pair;
      }
      const int nvalid = min(16, used - row0);
      uint8_t *kt = smem + st * kStageBytes;
      if (nvalid > 0) {
        uint8_t *vt = kt + kTileBytes;
        if (nvalid < 16) {
          for (int idx = lane; idx < (16 - nvalid) * 16; idx += 32) {
            const int rr = row0 + nvalid + idx / 16;
            const int q16 = idx % 16;
            *reinterpret_cast<uint4 *>(vt + (q16 >> 3) * kHalfBytes + rr * 128 + (q16 & 7) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          __syncwarp();
        }
        const uint32_t kbase = smem_u32(kt), vbase = smem_u32(vt);
        float sc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t a0, a1, a2, a3;
          const int row = row0 + ri + (mi & 1) * 8;
          ldsm_x4(kbase + tile_off(row, 2 * j + (mi >> 1)), a0, a1, a2, a3);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Mma<T>::run(sc[nt], a0, a1, a2, a3, qf[nt][j][0], qf[nt][j][1]);
        }
        const bool v_lo = r < nvalid, v_hi = r + 8 < nvalid;
        uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float x0 = v_lo ? sc[nt][0] * a.scale_log2 : -INFINITY;
          const float x1 = v_lo ? sc[nt][1] * a.scale_log2 : -INFINITY;
          const float x2 = v_hi ? sc[nt][2] * a.scale_log2 : -INFINITY;
          const float x3 = v_hi ? sc[nt][3] * a.scale_log2 : -INFINITY;
          float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, off));
            t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, off));
          }
          const float mn0 = fmaxf(m_run[nt][0], t0), mn1 = fmaxf(m_run[nt][1], t1);
          const float al0 = rescale_weight(m_run[nt][0], mn0), al1 = rescale_weight(m_run[nt][1], mn1);
          m_run[nt][0] = mn0;
          m_run[nt][1] = mn1;
          const float p0 = v_lo ? fast_exp2(x0 - mn0) : 0.f;
          const float p1 = v_lo ? fast_exp2(x1 - mn1) : 0.f;
          const float p2 = v_hi ? fast_exp2(x2 - mn0) : 0.f;
          const float p3 = v_hi ? fast_exp2(x3 - mn1) : 0.f;
          l_run[nt][0] = fmaf(l_run[nt][0], al0, p0 + p2);
          l_run[nt][1] = fmaf(l_run[nt][1], al1, p1 + p3);
          if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
              o[nt][dt][0] *= al0;
              o[nt][dt][1] *= al1;
              o[nt][dt][2] *= al0;
              o[nt][dt][3] *= al1;
            }
          }
          uint32_t h01, l01, h23, l23;
          Mma<T>::split(p0, p1, h01, l01);
          Mma<T>::split(p2, p3, h23, l23);
          bh[nt][0] = movm_t(h01);
          bh[nt][1] = movm_t(h23);
          bl[nt][0] = movm_t(l01);
          bl[nt][1] = movm_t(l23);
        }
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          uint32_t a0, a1, a2, a3;
          const int row = row0 + ri + (mi >> 1) * 8;
          ldsm_x4_t(vbase + tile_off(row, 2 * dt + (mi & 1)), a0, a1, a2, a3);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            Mma<T>::run(o[nt][dt], a0, a1, a2, a3, bh[nt][0], bh[nt][1]);
            Mma<T>::run(o[nt][dt], a0, a1, a2, a3, bl[nt][0], bl[nt][1]);
          }
        }
      }

      if (last) {
        // ---- segment end: merge the four warps into one CTA record of the pair ----
        // Every consumer warp is done with this stage's K/V (barrier), and the stage is not
        // released to the producer until the merge below has read it: use it as scratch.
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        float *sx = reinterpret_cast<float *>(kt);  // [4][HN][D]
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int h0 = nt * 8 + 2 * cq;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float v = l_run[nt][e];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            if (r == 0) {
              m_x[warp][h0 + e] = m_run[nt][e];
              l_x[warp][h0 + e] = v;
            }
          }
#pragma unroll
          for (int dt = 0; dt < 8; ++dt) {
            const int d = dt * 16 + r;
            sx[(warp * HN + h0) * D + d] = o[nt][dt][0];
            sx[(warp * HN + h0 + 1) * D + d] = o[nt][dt][1];
            sx[(warp * HN + h0) * D + d + 8] = o[nt][dt][2];
            sx[(warp * HN + h0 + 1) * D + d + 8] = o[nt][dt][3];
          }
        }
        reset_state();
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        float *rec_o = pa.rec_o + (int64_t)(c + pair) * gq * D;
        float *rec_ml = pa.rec_ml + (int64_t)(c + pair) * gq * 2;
        for (int idx4 = tid; idx4 < gq * (D / 4); idx4 += kConsumerWarps * 32) {
          const int h = idx4 / (D / 4), d = (idx4 - h * (D / 4)) * 4;
          float M = -INFINITY;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, m_x[w][h]);
          float L = 0.f;
          float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) {
            const float wt = rescale_weight(m_x[w][h], M);
            L = fmaf(l_x[w][h], wt, L);
            const float4 v = *reinterpret_cast<const float4 *>(sx + (w * HN + h) * D + d);
            O.x = fmaf(v.x, wt, O.x);
            O.y = fmaf(v.y, wt, O.y);
            O.z = fmaf(v.z, wt, O.z);
            O.w = fmaf(v.w, wt, O.w);
          }
          *reinterpret_cast<float4 *>(rec_o + h * D + d) = O;
          if (d == 0) {
            rec_ml[2 * h] = M;
            rec_ml[2 * h + 1] = L;
          }
        }
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        if (tid == 0) {
          const int b = pair / Hkv, g = pair - b * Hkv;
          const int64_t up = seq_prefix[b] + (int64_t)g * seq_pages[b];
          const int c0 = owner_cta(up, U, C), c1 = owner_cta(up + seq_pages[b] - 1, U, C);
          if (tagged_arrive(&pa.counter[pair], pa.token) == (uint32_t)(c1 - c0 + 1)) {
            // the last arrival of this call: leave the word at (token, 0) for the next call, which
            // starts after this grid has finished (a graph replay reuses the token)
            pa.counter[pair] = (unsigned long long)pa.token << 32;
            pending[npending++] = pair;
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      } else if (nvalid > 0 && nvalid < 16) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[st]);
    }

    // ---- deferred merges: pairs whose last CTA record this CTA wrote ----
    constexpr int F4 = HN / 4;  // float4 elements per thread: HN*D/4/128
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
    __threadfence();
    const int np = npending;
    for (int k = 0; k < np; ++k) {
      const int pair = pending[k];
      const int b = pair / Hkv, g = pair - b * Hkv;
      const int64_t up = seq_prefix[b] + (int64_t)g * seq_pages[b];
      const int c0 = owner_cta(up, U, C), c1 = owner_cta(up + seq_pages[b] - 1, U, C);
      const int nrec = c1 - c0 + 1;
      const float *ro = pa.rec_o + (int64_t)(c0 + pair) * gq * D;    // CTA c0+j: + j*gq*D
      const float *rml = pa.rec_ml + (int64_t)(c0 + pair) * gq * 2;  // CTA c0+j: + j*gq*2
      float4 acc[F4];
#pragma unroll
      for (int e = 0; e < F4; ++e) acc[e] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (tid < gq) {
        mg_M[tid] = -INFINITY;
        mg_L[tid] = 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
      for (int r0 = 0; r0 < nrec; r0 += 32) {
        const int nr = min(32, nrec - r0);
        for (int idx = tid; idx < gq * 32; idx += kConsumerWarps * 32) {
          const int h = idx >> 5, rr = idx & 31;
          if (rr < nr) {
            const float2 ml = __ldcg(reinterpret_cast<const float2 *>(rml + (int64_t)(r0 + rr) * gq * 2 + 2 * h));
            mg_m[h][rr] = ml.x;
            mg_l[h][rr] = ml.y;
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        if (tid < gq) {
          const int h = tid;
          float Mc = mg_M[h];
          for (int rr = 0; rr < nr; ++rr) Mc = fmaxf(Mc, mg_m[h][rr]);
          const float al = rescale_weight(mg_M[h], Mc);
          float L = mg_L[h] * al;
          for (int rr = 0; rr < nr; ++rr) {
            const float wr = rescale_weight(mg_m[h][rr], Mc);
            L = fmaf(mg_l[h][rr], wr, L);
            mg_m[h][rr] = wr;
          }
          mg_A[h] = al;
          mg_M[h] = Mc;
          mg_L[h] = L;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
#pragma unroll
        for (int e = 0; e < F4; ++e) {
          const int idx4 = tid + e * kConsumerWarps * 32;
          if (idx4 < gq * (D / 4)) {
            const int h = idx4 / (D / 4);
            const float al = mg_A[h];
            acc[e].x *= al;
            acc[e].y *= al;
            acc[e].z *= al;
            acc[e].w *= al;
          }
        }
#pragma unroll 4
        for (int rr = 0; rr < nr; ++rr) {
#pragma unroll
          for (int e = 0; e < F4; ++e) {
            const int idx4 = tid + e * kConsumerWarps * 32;
            if (idx4 < gq * (D / 4)) {
              const int h = idx4 / (D / 4);
              const float w = mg_m[h][rr];
              const float4 v = __ldcg(reinterpret_cast<const float4 *>(ro + (int64_t)(r0 + rr) * gq * D) + idx4);
              acc[e].x = fmaf(w, v.x, acc[e].x);
              acc[e].y = fmaf(w, v.y, acc[e].y);
              acc[e].z = fmaf(w, v.z, acc[e].z);
              acc[e].w = fmaf(w, v.w, acc[e].w);
            }
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
      }
      exchange_emit(pair, b, g, acc);
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
    }
    // Sequences without pages on this rank: an empty record (zeros when not exchanging).
    for (int pq = c; pq < B * Hkv; pq += gridDim.x) {
      const int b = pq / Hkv, g = pq - b * Hkv;
      if (seq_pages[b] != 0) continue;
      float4 acc[F4];
#pragma unroll
      for (int e = 0; e < F4; ++e) acc[e] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (tid < HN) {
        mg_M[tid] = -INFINITY;
        mg_L[tid] = 0.f;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
      exchange_emit(pq, b, g, acc);
      asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
    }
  }
}

}  // namespace tc

// ===========================================================================
// Log-sum-exp merge, split-parallel: one CTA of 8 warps per row, for an even D <= 256 and
// 8-byte-aligned records.  The (m, l) of every partial are read in one parallel pass; then warp w
// sums partials w, w + 8, ... over the whole row (float2 loads, a 512-byte record row per warp
// load), four partials in flight per lane; the eight warps' sums meet in shared memory.  Each
// row costs about three memory round trips whatever the number of partials, where the
// dim-per-thread kernel below walks the partials one load batch at a time.
// ===========================================================================
constexpr int kMergeWarps = 8;

__global__ void __launch_bounds__(kMergeWarps * 32) lse_merge_wide_kernel(const float *__restrict__ parts, int S,
                                                                         int64_t pstride, int rows, int D,
                                                                         void *out, int out_dtype,
                                                                         float *out_record) {
  constexpr int kChunk = 1024;
  __shared__ float w_s[kChunk];
  __shared__ float o_red[kMergeWarps][256];
  __shared__ float red[kMergeWarps];
  __shared__ float s_M, s_L;
  const int row = blockIdx.x;
  const int rl = D + 2, nv = D >> 1;
  const float *base = parts + (int64_t)row * rl;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_trigger();
  pdl_wait();
  float M = -INFINITY;
  for (int sp = tid; sp < S; sp += blockDim.x) M = fmaxf(M, base[sp * pstride + D]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  if (tid == 0) {
    float m = red[0];
    for (int w = 1; w < kMergeWarps; ++w) m = fmaxf(m, red[w]);
    s_M = m;
  }
  __syncthreads();
  M = s_M;
  float L = 0.f;
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  for (int c0 = 0; c0 < S; c0 += kChunk) {
    const int n = min(kChunk, S - c0);
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const float *p = base + (int64_t)(c0 + i) * pstride;
      const float w = rescale_weight(p[D], M);
      w_s[i] = w;
      L = fmaf(p[D + 1], w, L);
    }
    __syncthreads();
    if (M != -INFINITY) {
#pragma unroll 4
      for (int i = warp; i < n; i += kMergeWarps) {
        const float w = w_s[i];
        const float2 *src = reinterpret_cast<const float2 *>(base + (int64_t)(c0 + i) * pstride);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int v = lane + 32 * k;
          if (v < nv) {
            const float2 x = src[v];
            acc[k].x = fmaf(x.x, w, acc[k].x);
            acc[k].y = fmaf(x.y, w, acc[k].y);
          }
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int v = lane + 32 * k;
    if (v < nv) {
      o_red[warp][2 * v] = acc[k].x;
      o_red[warp][2 * v + 1] = acc[k].y;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  __syncthreads();
  if (lane == 0) red[warp] = L;
  __syncthreads();
  if (tid == 0) {
    float l = 0.f;
    for (int w = 0; w < kMergeWarps; ++w) l += red[w];
    s_L = M == -INFINITY ? 0.f : l;
  }
  __syncthreads();
  L = s_L;
  for (int d = tid; d < D; d += blockDim.x) {
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) O += o_red[w][d];
    if (M == -INFINITY) O = 0.f;
    if (out) store_f(out, out_dtype, (int64_t)row * D + d, L > 0.f ? O / L : 0.f);
    if (out_record) {
      float *rr = out_record + (int64_t)row * rl;
      rr[d] = O;
      if (d == 0) { rr[D] = M; rr[D + 1] = L; }
    }
  }
}

// ===========================================================================
// Log-sum-exp merge: one CTA per row (query head of a sequence).
// ===========================================================================
__global__ void __launch_bounds__(128) lse_merge_kernel(const float *__restrict__ parts, int S, int64_t pstride,
                                                       int rows, int D, void *out, int out_dtype,
                                                       float *out_record) {
  // One CTA per row.  The partials' (m, l) are read once, in parallel, and their weights
  // 2^(m_s - M) kept in shared memory (in chunks of kChunk partials); each thread then sums its
  // dims over the chunk's partials with independent loads.
  constexpr int kChunk = 1024;
  __shared__ float w_s[kChunk];
  __shared__ float red[4];
  __shared__ float s_M, s_L;
  const int row = blockIdx.x;
  const int rl = D + 2;
  const float *base = parts + (int64_t)row * rl;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_trigger();
  pdl_wait();
  // M = max_s m_s
  float M = -INFINITY;
  for (int sp = tid; sp < S; sp += blockDim.x) M = fmaxf(M, base[sp * pstride + D]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  if (tid == 0) s_M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  M = s_M;
  float L = 0.f;
  float O0 = 0.f, O1 = 0.f;   // dims tid and tid + 128 (D <= 256)
  for (int c0 = 0; c0 < S; c0 += kChunk) {
    const int n = min(kChunk, S - c0);
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const float *p = base + (int64_t)(c0 + i) * pstride;
      const float w = rescale_weight(p[D], M);
      w_s[i] = w;
      L = fmaf(p[D + 1], w, L);
    }
    __syncthreads();
    if (M != -INFINITY) {
      const float *src = base + (int64_t)c0 * pstride;
      if (tid < D) {
#pragma unroll 16
        for (int i = 0; i < n; ++i) O0 = fmaf(src[(int64_t)i * pstride + tid], w_s[i], O0);
      }
      if (tid + 128 < D) {
#pragma unroll 16
        for (int i = 0; i < n; ++i) O1 = fmaf(src[(int64_t)i * pstride + tid + 128], w_s[i], O1);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  __syncthreads();
  if (lane == 0) red[warp] = L;
  __syncthreads();
  if (tid == 0) s_L = M == -INFINITY ? 0.f : red[0] + red[1] + red[2] + red[3];
  __syncthreads();
  L = s_L;
  for (int k = 0; k < 2; ++k) {
    const int d = tid + 128 * k;
    if (d >= D) break;
    const float O = M == -INFINITY ? 0.f : (k ? O1 : O0);
    if (out) store_f(out, out_dtype, (int64_t)row * D + d, L > 0.f ? O / L : 0.f);
    if (out_record) {
      float *rr = out_record + (int64_t)row * rl;
      rr[d] = O;
      if (d == 0) { rr[D] = M; rr[D + 1] = L; }
    }
  }
}

// ===========================================================================
// Host side.
// ===========================================================================
namespace {


// 4-D map over the pool: (dim, token, kv head, page), box 64 x 64 x 1 x 1,
// 128-byte swizzle.  Encoded maps are cached (keyed by everything they encode), since
// a decode step calls with the same pool every layer.
struct MapKey {
  const void *base;
  int dtype, D, P, Hkv, pages;
  int64_t head_stride, page_stride;
  bool operator==(const MapKey &o) const {
    return base == o.base && dtype == o.dtype && D == o.D && P == o.P && Hkv == o.Hkv && pages == o.pages &&
           head_stride == o.head_stride && page_stride == o.page_stride;
  }
};

bool encode_pool_map(CUtensorMap *m, const void *base, int kv_dtype, const helm_paged_attn_params *p);

bool make_pool_map(CUtensorMap *m, const void *base, int kv_dtype, const helm_paged_attn_params *p) {
  constexpr int kSlots = 32;
  static std::mutex mu;
  static MapKey keys[kSlots];
  static CUtensorMap maps[kSlots];
  static int filled = 0, next = 0;
  const MapKey key{base, kv_dtype, p->D, p->P, p->Hkv, p->num_pool_pages, p->head_stride, p->page_stride};
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < filled; ++i)
      if (keys[i] == key) {
        *m = maps[i];
        return true;
      }
  }
  if (!encode_pool_map(m, base, kv_dtype, p)) return false;
  std::lock_guard<std::mutex> lock(mu);
  keys[next] = key;
  maps[next] = *m;
  next = (next + 1) % kSlots;
  if (filled < kSlots) ++filled;
  return true;
}

bool encode_pool_map(CUtensorMap *m, const void *base, int kv_dtype, const helm_paged_attn_params *p) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  const int es = dtype_size(kv_dtype);
  cuuint64_t gdim[4] = {(cuuint64_t)p->D, (cuuint64_t)p->P, (cuuint64_t)p->Hkv, (cuuint64_t)p->num_pool_pages};
  cuuint64_t gstr[3] = {(cuuint64_t)p->D * es, (cuuint64_t)p->head_stride * es, (cuuint64_t)p->page_stride * es};
  cuuint32_t box[4] = {64, 64, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, kv_dtype == HELM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void *>(base), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Token of one persistent-kernel call: tags its arrival counters, so that words left by any other
// call (or never written) count as zero and no counter has to be zeroed before a call.
uint32_t next_call_token() {
  static std::atomic<uint32_t> counter{0};
  uint32_t t = counter.fetch_add(1u, std::memory_order_relaxed) + 1u;
  return t ? t : counter.fetch_add(1u, std::memory_order_relaxed) + 1u;
}

// Debug switches, read on every call so that tests can flip them between calls (cheap: no
// allocation, a short environment scan).
bool env_flag(const char *name) {
  const char *v = getenv(name);
  return v && v[0] && v[0] != '0';
}

// cudaFuncSetAttribute once per (kernel, device).
template <typename K>
void ensure_smem_attr(K kernel, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<const void *, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  const void *key = reinterpret_cast<const void *>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  for (const auto &d : done)
    if (d.first == key && d.second == dev) return;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  done.emplace_back(key, dev);
}

bool tc_eligible(const helm_paged_attn_params *p) {
  if (!(p->kv_dtype == HELM_BF16 || p->kv_dtype == HELM_F16)) return false;
  if (p->q_dtype != p->kv_dtype) return false;
  if (p->D != tc::D || p->P != tc::P) return false;
  const int gq = p->Hq / p->Hkv;
  if (gq > 16) return false;
  if ((reinterpret_cast<uintptr_t>(p->k_base) & 15) || (reinterpret_cast<uintptr_t>(p->v_base) & 15)) return false;
  if ((reinterpret_cast<uintptr_t>(p->q) & 3)) return false;
  if ((p->page_stride % 8) || (p->head_stride % 8)) return false;
  if (p->num_pool_pages < 1) return false;
  if (env_flag("HELM_B200_FORCE_GENERIC")) return false;
  return true;
}

// The warp-per-octet kernel: D a multiple of 32 up to 256 (a lane owns D/32 consecutive elements
// of a row; D = 224 excepted), any GQA group: the group's query heads are served GQ at a time
// (GQ <= 8, GQ * D/32 <= 32 registers per row of state), one CTA per chunk of GQ heads.
struct WarpCfg {
  int GQ = 0;      // heads per CTA (a power of two)
  int chunks = 0;  // CTAs along the GQA group
};

WarpCfg warp_cfg(int gq, int D) {
  WarpCfg c;
  if (D <= 0 || D % 32 != 0 || D > 256 || D == 224 || gq <= 0) return c;
  const int dpl = D / 32;
  int cap = 8;
  while (cap * dpl > 32) cap >>= 1;
  int GQ = 1;
  while (GQ < gq && GQ < cap) GQ *= 2;
  c.GQ = GQ;
  c.chunks = (gq + GQ - 1) / GQ;
  return c;
}

bool warp_eligible(const helm_paged_attn_params *p) {
  if (env_flag("HELM_B200_FORCE_GENERIC")) return false;
  if (p->Hkv <= 0 || p->Hq % p->Hkv != 0) return false;
  const WarpCfg c = warp_cfg(p->Hq / p->Hkv, p->D);
  if (c.GQ == 0) return false;
  const int dpl = p->D / 32;
  const int es = dtype_size(p->kv_dtype);
  // the alignment of RowLoad's widest access for this row length
  int vb;
  if (es == 4) vb = dpl % 4 == 0 ? 16 : dpl % 2 == 0 ? 8 : 4;
  else vb = dpl % 8 == 0 ? 16 : dpl % 4 == 0 ? 8 : 2;
  const uintptr_t kb = reinterpret_cast<uintptr_t>(p->k_base), vbp = reinterpret_cast<uintptr_t>(p->v_base);
  return kb % vb == 0 && vbp % vb == 0 && (p->page_stride * es) % vb == 0 && (p->head_stride * es) % vb == 0;
}

// Launches the merge of S partial records (stride pstride floats) into out / out_record.
int launch_lse_merge(const float *parts, int S, int64_t pstride, int rows, int D, void *out, int out_dtype,
                     float *out_record, cudaStream_t st) {
  // Many rows already fill the GPU with one 128-thread CTA per row; the split-parallel kernel pays
  // where rows are few (decode batches, sharded exchanges) or the partials many.
  const bool wide = D % 2 == 0 && D <= 256 && pstride % 2 == 0 && (reinterpret_cast<uintptr_t>(parts) & 7) == 0 &&
                    (rows < 8 * num_sms() || S >= 64);
  const cudaError_t e = wide ? launch_pdl(lse_merge_wide_kernel, dim3(rows), dim3(kMergeWarps * 32), 0, st, parts, S,
                                          pstride, rows, D, out, out_dtype, out_record)
                             : launch_pdl(lse_merge_kernel, dim3(rows), dim3(128), 0, st, parts, S, pstride, rows, D,
                                          out, out_dtype, out_record);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "lse_merge: launch: %s", cudaGetErrorString(e));
  return check_launch(wide ? "lse_merge_wide_kernel" : "lse_merge_kernel");
}
int warp_ctas_per_sm(int kv_dtype, int D, int gq);

int resolve_splits(const helm_paged_attn_params *p) {
  if (p->num_splits > 0) return p->num_splits;
  if (!tc_eligible(p) && warp_eligible(p)) {
    // as many CTAs as are resident at once (the instantiation's registers decide: 2 to 4 per SM),
    // every CTA with at least one page: the whole grid runs in one wave with most of the call's
    // K/V in flight
    const int gq = p->Hq / p->Hkv;
    const int pairs = p->B * p->Hkv * warp_cfg(gq, p->D).chunks;
    if (pairs <= 0 || p->max_pages <= 1) return 1;
    const int per_sm = warp_ctas_per_sm(p->kv_dtype, p->D, gq);
    int S = (per_sm > 4 ? 4 : per_sm) * num_sms() / pairs;
    if (S < 1) S = 1;
    return S > p->max_pages ? p->max_pages : S;
  }
  const int pairs = p->B * p->Hkv;
  const int maxp = p->max_pages;
  if (maxp <= 1 || pairs <= 0) return 1;
  if (tc_eligible(p)) {
    // k splits per (sequence, kv head) pair, k the largest power of two with k * pairs <= two CTAs
    // per SM (one resident wave; power-of-two page counts then split evenly), or 2k when every split
    // still gets >= 64 pages.  Measured over 34 MB - 2.1 GB calls with 8 to 64 pairs against other
    // split counts and the persistent kernel: the fastest or within 3 % (32 pairs x 2048 pages:
    // 8 splits 309.9 us, 9 313.6, 16 304.5).
    int k = 1;
    while (2 * k * pairs <= 2 * num_sms()) k *= 2;
    int S = maxp / (2 * k) >= 64 ? 2 * k : k;
    if (S > maxp) S = maxp;
    return S < 1 ? 1 : S;
  }
  const int slots = num_sms() * 2;  // two resident CTAs per SM
  for (int waves = 4; waves >= 1; --waves) {
    int S = (waves * slots) / pairs;
    if (S < 1) continue;
    if (maxp / S >= 8 || (waves == 1 && S > 1)) return S > maxp ? maxp : S;
  }
  // Few (sequence, kv head) pairs and short sequences: still fill the GPU.
  int S = (slots + pairs - 1) / pairs;
  if (S > maxp) S = maxp;
  return S < 1 ? 1 : S;
}

// Launch plan.  The persistent kernel (one launch, C CTAs, stream-K over all pages, fused merge)
// runs tensor-core-eligible calls that ask for it (num_splits == -1) or that carry a cross-GPU
// exchange (which it fuses); every other call runs the split grid + the LSE merge, which has the
// lower fixed cost per call (10 vs 16 us) and the higher streaming rate (7.3 vs 7.0 TB/s).
struct Plan {
  bool persistent = false;
  int S = 1;          // split mode: splits
  int C = 0;          // persistent mode: CTAs
  int64_t rec_bytes = 0;
  int64_t ml_off = 0;
  int64_t counter_off = 0;
  int64_t bytes = 0;  // workspace needed
};

Plan make_plan(const helm_paged_attn_params *p, bool eligible) {
  Plan pl;
  const int rows = p->B * p->Hq;
  const int pairs_all = p->B * p->Hkv;
  const int64_t units_max = (int64_t)pairs_all * (p->max_pages > 0 ? p->max_pages : 1);
  // Up to two CTAs per SM, as k CTAs per (sequence, kv head) pair with k the largest power of two
  // that fits: with equal page counts the stream-K ranges then end on pair boundaries (no CTA closes
  // one pair's record and opens another's mid-stream) and, for power-of-two page counts, every CTA
  // gets the same number of pages.  Measured on 32 pairs x 256 pages: 296 CTAs 54.2 us, 288 (9 per
  // pair) 51.2 us, 256 (8 per pair) 50.4 us.
  int64_t Cp = (int64_t)num_sms() * 2;
  if (pairs_all > 0 && pairs_all <= Cp) {
    int64_t k = 1;
    while (2 * k * pairs_all <= Cp) k *= 2;
    Cp = k * pairs_all;
  }
  if (Cp > units_max) Cp = units_max;
  if (Cp < 1) Cp = 1;
  // a CTA covers at most units_max/C + 1 units, hence at most that many + 1 pairs
  const bool pending_ok = pairs_all <= tc::kMaxPending || units_max / Cp + 2 <= tc::kMaxPending;
  // Workspace layout: the CTA records then the tagged arrival counters (persistent path), or the
  // split records (split path).
  const bool sharded = p->exchange && p->exchange->world > 1;
  const bool records_only = !p->out && !p->out_record;
  const bool want = !records_only && (p->num_splits == -1 || (p->num_splits == 0 && sharded));
  if (want && eligible && p->B <= tc::kMaxSeqs && pending_ok && units_max < (1ll << 31) &&
      !env_flag("HELM_B200_NO_PERSISTENT")) {
    pl.persistent = true;
    const int pairs = pairs_all;
    pl.C = (int)Cp;
    const int gq = p->Hq / p->Hkv;
    const int64_t slots = pl.C + (int64_t)pairs;
    pl.rec_bytes = slots * gq * p->D * (int64_t)sizeof(float);                 // o
    pl.ml_off = (pl.rec_bytes + 255) / 256 * 256;
    pl.counter_off = (pl.ml_off + slots * gq * 2 * (int64_t)sizeof(float) + 255) / 256 * 256;
    pl.bytes = pl.counter_off + (int64_t)pairs * sizeof(uint64_t);
    return pl;
  }
  pl.S = resolve_splits(p);
  pl.bytes = (pl.S > 1 || records_only) ? (int64_t)pl.S * rows * (p->D + 2) * (int64_t)sizeof(float) : 0;
  return pl;
}

int validate(const helm_paged_attn_params *p) {
  if (!p) return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: params is null");
  if (p->B < 0 || p->Hq < 0 || p->Hkv <= 0 || p->D <= 0 || p->P <= 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: bad sizes B=%d Hq=%d Hkv=%d D=%d P=%d", p->B, p->Hq,
                p->Hkv, p->D, p->P);
  if (p->Hq % p->Hkv != 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: Hq=%d not a multiple of Hkv=%d", p->Hq, p->Hkv);
  if (p->D > 256) return fail(HELM_ERR_UNSUPPORTED, "paged_attn: head dim %d > 256", p->D);
  for (int dt : {p->q_dtype, p->kv_dtype, p->out_dtype})
    if (dt != HELM_F32 && dt != HELM_F16 && dt != HELM_BF16)
      return fail(HELM_ERR_UNSUPPORTED, "paged_attn: dtype %d not supported", dt);
  if (p->B > 0 && p->Hq > 0) {
    if (!p->q || !p->k_base || !p->v_base || !p->page_table || !p->page_used || !p->num_pages)
      return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: null input pointer");
    // no out and no out_record: records-only mode (the split records, left in the workspace)
    if (!p->out && !p->out_record && p->exchange && p->exchange->world > 1)
      return fail(HELM_ERR_UNSUPPORTED, "paged_attn: records-only mode has no fused exchange");
  }
  if (p->page_stride < 0 || p->head_stride < 0 || p->page_table_stride < 0 || p->max_pages < 0 ||
      p->num_pool_pages < 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: negative stride or count");
  if (p->max_pages > p->page_table_stride)
    return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: max_pages %d > page_table_stride %d", p->max_pages,
                p->page_table_stride);
  if (p->num_splits < -1) return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: num_splits %d < -1", p->num_splits);
  if (p->exchange && p->exchange->world > 1) {
    const helm_shard_exchange *x = p->exchange;
    if (x->world > HELM_MAX_RANKS || x->rank < 0 || x->rank >= x->world)
      return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: bad exchange rank %d / world %d", x->rank, x->world);
    if (!x->recv_local || !x->counters)
      return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: exchange buffers missing");
    if (x->recv_local != x->peer_recv[x->rank])
      return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: exchange recv_local != peer_recv[rank]");
    for (int r = 0; r < x->world; ++r) {
      if (!x->peer_recv[r])
        return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: exchange peer %d missing", r);
      if (reinterpret_cast<uintptr_t>(x->peer_recv[r]) % 16 != 0)
        return fail(HELM_ERR_INVALID_ARGUMENT, "paged_attn: exchange slots of rank %d not 16-byte aligned", r);
    }
    if (p->num_splits > 0)
      return fail(HELM_ERR_UNSUPPORTED, "paged_attn: the fused exchange needs num_splits 0 or -1");
  }
  return HELM_OK;
}

size_t generic_smem_bytes(int gq, int D) {
  return sizeof(float) * ((size_t)gq * D * (1 + kGenWarps) + (size_t)kGenWarps * 32 * gq + 3 * kGenWarps * gq);
}

template <typename KT>
int launch_generic(const AttnArgs &a, cudaStream_t st) {
  const size_t smem = generic_smem_bytes(a.gq, a.D);
  if (smem > 200 * 1024) return fail(HELM_ERR_UNSUPPORTED, "paged_attn: gq*D too large for the generic kernel");
  cudaFuncSetAttribute(attn_generic_kernel<KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(a.num_splits, a.Hkv, a.B);
  attn_generic_kernel<KT><<<grid, 128, smem, st>>>(a);
  return check_launch("attn_generic_kernel");
}

// query = false: launch; query = true: return how many CTAs of the instantiation fit on an SM
// (0 when no instantiation serves the shape).
template <typename KT, int DPL, int GQ>
int launch_warp_cfg(AttnArgs a, int chunks, cudaStream_t st, bool query) {
  const size_t smem = warp_smem_bytes(GQ, 32 * DPL);
  ensure_smem_attr(attn_warp_kernel<KT, DPL, GQ>, (int)smem);
  if (query) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_warp_kernel<KT, DPL, GQ>, kWWarps * 32, smem) !=
        cudaSuccess) {
      cudaGetLastError();
      return 1;
    }
    return n > 0 ? n : 1;
  }
  a.head_chunks = chunks;
  const cudaError_t e = launch_pdl(attn_warp_kernel<KT, DPL, GQ>, dim3(a.num_splits, a.Hkv * chunks, a.B),
                                   dim3(kWWarps * 32), smem, st, a);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "paged_attn: launch: %s", cudaGetErrorString(e));
  return check_launch("attn_warp_kernel");
}

template <typename KT, int DPL>
int launch_warp_d(const AttnArgs &a, cudaStream_t st, bool query) {
  const WarpCfg c = warp_cfg(a.gq, a.D);
  if (c.GQ == 1) return launch_warp_cfg<KT, DPL, 1>(a, c.chunks, st, query);
  if (c.GQ == 2) return launch_warp_cfg<KT, DPL, 2>(a, c.chunks, st, query);
  if constexpr (DPL <= 8) {
    if (c.GQ == 4) return launch_warp_cfg<KT, DPL, 4>(a, c.chunks, st, query);
  }
  if constexpr (DPL <= 4) {
    if (c.GQ == 8) return launch_warp_cfg<KT, DPL, 8>(a, c.chunks, st, query);
  }
  if (query) return 0;
  return fail(HELM_ERR_UNSUPPORTED, "paged_attn: GQA group %d at head dim %d", a.gq, a.D);
}

template <typename KT>
int launch_warp(const AttnArgs &a, cudaStream_t st, bool query = false) {
  switch (a.D) {
    case 32: return launch_warp_d<KT, 1>(a, st, query);
    case 64: return launch_warp_d<KT, 2>(a, st, query);
    case 96: return launch_warp_d<KT, 3>(a, st, query);
    case 128: return launch_warp_d<KT, 4>(a, st, query);
    case 160: return launch_warp_d<KT, 5>(a, st, query);
    case 192: return launch_warp_d<KT, 6>(a, st, query);
    case 256: return launch_warp_d<KT, 8>(a, st, query);
    default:
      if (query) return 0;
      return fail(HELM_ERR_UNSUPPORTED, "paged_attn: head dim %d on the warp kernel", a.D);
  }
}

int warp_ctas_per_sm(int kv_dtype, int D, int gq) {
  static std::mutex mu;
  static std::vector<std::pair<std::pair<int, int>, std::pair<int, int>>> cache;  // ((dtype, D), (gq, n))
  int dev = 0;
  cudaGetDevice(&dev);
  const int key = kv_dtype * 4096 + D, key2 = dev * 65536 + gq;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto &c : cache)
      if (c.first.first == key && c.first.second == key2) return c.second.first;
  }
  AttnArgs a{};
  a.D = D;
  a.gq = gq;
  int n = 0;
  switch (kv_dtype) {
    case HELM_F32: n = launch_warp<float>(a, nullptr, true); break;
    case HELM_F16: n = launch_warp<__half>(a, nullptr, true); break;
    default: n = launch_warp<__nv_bfloat16>(a, nullptr, true); break;
  }
  if (n < 1) n = 1;
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({{key, key2}, {n, 0}});
  return n;
}

template <typename T, int NT>
int launch_tc_persistent(const CUtensorMap &mk, const CUtensorMap &mv, const AttnArgs &a,
                         const tc::PersistArgs &pa, cudaStream_t st) {
  ensure_smem_attr(tc::attn_tc_persistent_kernel<T, NT>, tc::kSmemBytes);
  const cudaError_t e = launch_pdl(tc::attn_tc_persistent_kernel<T, NT>, dim3(pa.C), dim3(tc::kThreads),
                                   tc::kSmemBytes, st, mk, mv, a, pa);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "paged_attn: launch: %s", cudaGetErrorString(e));
  return check_launch("attn_tc_persistent_kernel");
}

template <typename T, int NT>
int launch_tc(const CUtensorMap &mk, const CUtensorMap &mv, const AttnArgs &a, cudaStream_t st) {
  ensure_smem_attr(tc::attn_tc_kernel<T, NT>, tc::kSmemBytes);
  dim3 grid(a.num_splits, a.Hkv, a.B);
  tc::attn_tc_kernel<T, NT><<<grid, tc::kThreads, tc::kSmemBytes, st>>>(mk, mv, a);
  return check_launch("attn_tc_kernel");
}

}  // namespace
}  // namespace helm

using namespace helm;

extern "C" int64_t helm_paged_attn_workspace_bytes(const helm_paged_attn_params *p, int32_t *num_splits_out) {
  if (validate(p) != HELM_OK) return -1;
  const Plan pl = make_plan(p, tc_eligible(p));
  if (num_splits_out) *num_splits_out = pl.persistent ? -1 : pl.S;
  return pl.bytes;
}

extern "C" int helm_paged_attn_decode(const helm_paged_attn_params *p, void *stream) {
  helm::NvtxRange nvtx_range_("helm_paged_attn_decode");
  int rc = validate(p);
  if (rc != HELM_OK) return rc;
  if (p->B == 0 || p->Hq == 0) return HELM_OK;
  cudaStream_t st = as_stream(stream);
  const bool eligible = tc_eligible(p);
  const Plan pl = make_plan(p, eligible);
  const int S = pl.persistent ? 1 : pl.S;
  const int rows = p->B * p->Hq;
  const int64_t need = pl.bytes;
  if (need > 0 && (!p->workspace || p->workspace_bytes < need))
    return fail(HELM_ERR_WORKSPACE, "paged_attn: workspace %lld bytes < %lld needed", (long long)p->workspace_bytes,
                (long long)need);

  AttnArgs a{};
  a.q = p->q;
  a.k_base = p->k_base;
  a.v_base = p->v_base;
  a.page_stride = p->page_stride;
  a.head_stride = p->head_stride;
  a.num_pool_pages = p->num_pool_pages;
  a.page_table = p->page_table;
  a.page_used = p->page_used;
  a.num_pages = p->num_pages;
  a.pt_stride = p->page_table_stride;
  a.B = p->B;
  a.Hq = p->Hq;
  a.Hkv = p->Hkv;
  a.D = p->D;
  a.P = p->P;
  a.gq = p->Hq / p->Hkv;
  a.q_dtype = p->q_dtype;
  a.out_dtype = p->out_dtype;
  a.scale_log2 = p->scale * kLog2e;
  a.num_splits = S;
  a.error_flag = p->error_flag;
  float *const records = p->workspace;
  const bool records_only = !p->out && !p->out_record;  // the split records are the output
  if (S > 1 || records_only) {
    a.rec = records;
  } else {
    a.out = p->out;
    a.out_record = p->out_record;
  }

  if (p->exchange && p->exchange->world > 1 && !pl.persistent)
    return fail(HELM_ERR_UNSUPPORTED,
                "paged_attn: the fused exchange needs the persistent kernel (bf16/fp16 q == kv, D=128, P=64, "
                "num_splits=0, B <= 512)");
  if (eligible) {
    CUtensorMap mk, mv;
    if (!make_pool_map(&mk, p->k_base, p->kv_dtype, p) || !make_pool_map(&mv, p->v_base, p->kv_dtype, p))
      return fail(HELM_ERR_CUDA, "paged_attn: cuTensorMapEncodeTiled failed");
    const bool two = a.gq > 8;
    if (pl.persistent) {
      tc::PersistArgs pa{};
      char *ws = reinterpret_cast<char *>(p->workspace);
      pa.rec_o = records;
      pa.rec_ml = reinterpret_cast<float *>(ws + pl.ml_off);
      pa.counter = reinterpret_cast<uint64_t *>(ws + pl.counter_off);
      pa.token = next_call_token();
      pa.C = pl.C;
      pa.xwait_ns = tc::kExchangeWaitNs;
      pa.xrank = 0;
      pa.xworld = 0;
      if (p->exchange && p->exchange->world > 1) {
        const helm_shard_exchange *x = p->exchange;
        pa.xrank = x->rank;
        pa.xworld = x->world;
        for (int r = 0; r < x->world; ++r) pa.xrecv[r] = reinterpret_cast<uint64_t *>(x->peer_recv[r]);
        pa.xrecv_local = reinterpret_cast<uint64_t *>(x->recv_local);
        pa.xsent = x->counters;
        if (x->wait_ns) pa.xwait_ns = x->wait_ns;
      }
      a.rec = nullptr;
      a.out = p->out;
      a.out_record = p->out_record;
      a.num_splits = 1;
      if (p->kv_dtype == HELM_BF16)
        return two ? launch_tc_persistent<__nv_bfloat16, 2>(mk, mv, a, pa, st)
                   : launch_tc_persistent<__nv_bfloat16, 1>(mk, mv, a, pa, st);
      return two ? launch_tc_persistent<__half, 2>(mk, mv, a, pa, st)
                 : launch_tc_persistent<__half, 1>(mk, mv, a, pa, st);
    }
    if (p->kv_dtype == HELM_BF16)
      rc = two ? launch_tc<__nv_bfloat16, 2>(mk, mv, a, st) : launch_tc<__nv_bfloat16, 1>(mk, mv, a, st);
    else
      rc = two ? launch_tc<__half, 2>(mk, mv, a, st) : launch_tc<__half, 1>(mk, mv, a, st);
  } else if (warp_eligible(p)) {
    switch (p->kv_dtype) {
      case HELM_F32: rc = launch_warp<float>(a, st); break;
      case HELM_F16: rc = launch_warp<__half>(a, st); break;
      default: rc = launch_warp<__nv_bfloat16>(a, st); break;
    }
  } else {
    switch (p->kv_dtype) {
      case HELM_F32: rc = launch_generic<float>(a, st); break;
      case HELM_F16: rc = launch_generic<__half>(a, st); break;
      default: rc = launch_generic<__nv_bfloat16>(a, st); break;
    }
  }
  if (rc != HELM_OK || S == 1 || records_only) return rc;
  return launch_lse_merge(records, S, (int64_t)rows * (p->D + 2), rows, p->D, p->out, p->out_dtype, p->out_record, st);
}

extern "C" int helm_lse_merge(const float *partials, int32_t num_partials, int64_t partial_stride, int32_t rows,
                              int32_t D, void *out, int32_t out_dtype, float *out_record, void *stream) {
  helm::NvtxRange nvtx_range_("helm_lse_merge");
  if (rows < 0 || D <= 0 || num_partials < 1 || partial_stride < (int64_t)rows * (D + 2))
    return fail(HELM_ERR_INVALID_ARGUMENT, "lse_merge: bad sizes rows=%d D=%d partials=%d stride=%lld", rows, D,
                num_partials, (long long)partial_stride);
  if (!partials || (!out && !out_record)) return fail(HELM_ERR_INVALID_ARGUMENT, "lse_merge: null pointer");
  if (D > 256) return fail(HELM_ERR_UNSUPPORTED, "lse_merge: head dim %d > 256", D);
  if (out && out_dtype != HELM_F32 && out_dtype != HELM_F16 && out_dtype != HELM_BF16)
    return fail(HELM_ERR_UNSUPPORTED, "lse_merge: dtype %d", out_dtype);
  if (rows == 0) return HELM_OK;
  return launch_lse_merge(partials, num_partials, partial_stride, rows, D, out, out_dtype, out_record,
                          as_stream(stream));
}

// ===========================================================================
// Allocation-free variant: split records in a file-scope device array.
// ===========================================================================
namespace helm {
namespace {

// Holds the split-KV records of helm_paged_attn_decode_noalloc.  Every GPU that
// loads this library reserves it (HELM_NOALLOC_SCRATCH_BYTES) until exit.
static __device__ __align__(256) float g_noalloc_scratch[HELM_NOALLOC_SCRATCH_BYTES / sizeof(float)];

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.  In host code the symbol itself is only a host-side stand-in,
// so the kernels must be given this address instead.
int noalloc_scratch(float **out) {
  static std::mutex mu;
  static float *addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "paged_attn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(HELM_ERR_UNSUPPORTED, "paged_attn_noalloc: device %d >= 64", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(HELM_ERR_CUDA, "paged_attn_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    addr[dev] = static_cast<float *>(p);
  }
  *out = addr[dev];
  return HELM_OK;
}

}  // namespace
}  // namespace helm

extern "C" int helm_paged_attn_decode_noalloc(const helm_paged_attn_params *p, void *stream) {
  helm::NvtxRange nvtx_range_("helm_paged_attn_decode_noalloc");
  using namespace helm;
  int rc = validate(p);
  if (rc != HELM_OK) return rc;
  if (p->B == 0 || p->Hq == 0) return HELM_OK;
  int S = resolve_splits(p);
  const int64_t cap = HELM_NOALLOC_SCRATCH_BYTES;
  const int64_t per_split = (int64_t)p->B * p->Hq * (p->D + 2) * (int64_t)sizeof(float);
  if (S > 1 && (int64_t)S * per_split > cap) {
    if (p->num_splits > 0)
      return fail(HELM_ERR_WORKSPACE,
                  "paged_attn_noalloc: %d splits x %lld bytes of records exceed the %lld-byte static scratch; "
                  "pass fewer splits (at most %lld) or use helm_paged_attn_decode with a workspace",
                  S, (long long)per_split, (long long)cap, (long long)(cap / per_split));
    S = (int)(cap / per_split);  // auto mode: as many splits as the scratch holds
    if (S < 1) S = 1;
  }
  helm_paged_attn_params q = *p;
  q.num_splits = S;
  q.workspace = nullptr;
  q.workspace_bytes = 0;
  if (S > 1) {
    rc = noalloc_scratch(&q.workspace);
    if (rc != HELM_OK) return rc;
    q.workspace_bytes = HELM_NOALLOC_SCRATCH_BYTES;
  }
  return helm_paged_attn_decode(&q, stream);
}

extern "C" int64_t helm_shard_exchange_bytes(int32_t world, int32_t rows, int32_t D, int64_t *recv_bytes_out,
                                             int64_t *flags_bytes_out, int64_t *counters_bytes_out) {
  using namespace helm;
  if (world < 1 || world > HELM_MAX_RANKS || rows < 0 || D <= 0) {
    fail(HELM_ERR_INVALID_ARGUMENT, "shard_exchange_bytes: bad sizes world=%d rows=%d D=%d", world, rows, D);
    return -1;
  }
  // receive slots [2][G][rows][D+2] words of 64 bits; no flags; counters sent[rows] (>= pairs).
  const int64_t recv = 2ll * world * rows * (D + 2) * (int64_t)sizeof(uint64_t);
  const int64_t flags = 0;
  const int64_t counters = (int64_t)rows * (int64_t)sizeof(uint32_t);
  if (recv_bytes_out) *recv_bytes_out = recv;
  if (flags_bytes_out) *flags_bytes_out = flags;
  if (counters_bytes_out) *counters_bytes_out = counters;
  return recv + flags + counters;
}
