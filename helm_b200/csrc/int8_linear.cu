// INT8 weight-only linear: y[m, n] = (sum_k x[m, k] * w[n, k]) * s[n] + bias[n].
//
// The GPU counterpart of HELM's CPU decode GEMV (helm/kernels/fp16_gemv.cpp:
// 45-100: one fp16 weight row dotted with x, fp32 accumulation, rows spread
// over threads), with the weight stored as int8 plus one scale per output
// channel.  Decode-sized M is HBM-bound: every weight byte is read once and
// used M times, so the kernel is built to keep as many weight bytes in flight
// as the SM allows and to spend as few instructions as possible per byte.
//
// Tensor-core formulation (mma.sync m16n8k16, fp32 accumulators): the weight
// rows are the 16-row A operand and the rows of x are the 8-column B operand
// (M <= 8 per n-tile, more n-tiles for larger M).  The reduction order inside
// a 256-wide K block is permuted so that every thread reads 64 contiguous
// weight bytes of each of its two rows (four 16-byte loads) and 128
// contiguous bytes of its x row: thread j of a quad owns k = 64j .. 64j+63 of
// the block, and MMA u of the block takes k = 64j + 4u + {0,1} as its
// fragment columns (2j, 2j+1) and 64j + 4u + {2,3} as (2j+8, 2j+9).  A and B
// use the same permutation, so the dot products are exact sums over the block.
//
// int8 -> fp16 is exact in two instructions per pair: the biased byte
// b ^ 0x80 is placed in the low mantissa byte of 1024.0 (0x64xx) and 1152 is
// subtracted.  For bf16 activations the pair goes through fp32 the same way
// (0x4B0000xx - (2^23 + 128)) and the high halves of the exact fp32 values
// are the bf16 values.  The per-channel scale and the bias are applied once
// per output in the epilogue.
//
// Data movement: one producer warp streams the weight rows of the CTA with TMA
// (2-D tensor map over W [N, K] int8, boxes of 128 k x 16*RT rows, 128-byte
// swizzle) into a ring of shared-memory stages guarded by full/empty
// mbarriers, so the bytes in flight are set by the ring size, not by
// registers; four consumer warps each take one 128-k box of every 512-k
// stage, convert their int8 fragments in registers and run the MMAs.  Their
// partial tiles are summed in shared memory at the end.  A CTA owns 16*RT rows
// over the whole K, with RT chosen so that every CTA is resident at once (the
// HBM stream then balances the CTAs by itself).  Every mbarrier wait is
// bounded (2 s); a wait that gives up sets HELM_DEVERR_TIMEOUT in the
// library's INT8 error word (helm_int8_linear_error) and the CTA finishes
// without writing its rows.  Launched with programmatic dependent launch: the
// producer starts on the weights while the previous kernel on the stream drains;
// the consumers wait for that kernel (griddepcontrol.wait) before reading x.
#include "common.cuh"
#include "tma.cuh"

#include <cstring>
#include <mutex>
#include <vector>

namespace helm {

namespace {

constexpr int kCWarps = 4;                       // consumer warps (default; 8 for long-K GEMVs),
                                                 // plus one producer warp; a stage is one 128-k box
                                                 // per consumer warp
constexpr int kBoxK = 128;                       // k per TMA box row (128-byte swizzle)
constexpr int kMaxStages = 16;

// Ring depth: the shared memory left per CTA when ceil(CTAs / SMs) CTAs share an SM (at most 3;
// the whole grid is resident at once), within 2..kMaxStages stages.  Few CTAs get deep rings,
// which is what keeps a short-N, long-K weight (few rows per SM) streaming at the HBM rate.
inline int ring_stages(int ctas, int sms, int stage_bytes, int other_bytes) {
  int per = (ctas + sms - 1) / sms;
  if (per < 1) per = 1;
  if (per > 3) per = 3;
  int budget = (226 * 1024) / per - other_bytes - 2048;
  if (budget > 200 * 1024) budget = 200 * 1024;
  int st = budget / stage_bytes;
  if (st > kMaxStages) st = kMaxStages;
  return st < 2 ? 2 : st;
}

__device__ int g_int8_error;  // HELM_DEVERR_* bits of the INT8 kernels (helm_int8_linear_error)

// Packed weights (helm_int8_pack_weight): W [N, K] as blocks of 16 rows x 128 k (2 KB), block
// (t, kb) at byte ((t * KB) + kb) * 2048 with KB = ceil(K / 128), each block laid out exactly as
// the 128-byte-swizzled TMA box lands in shared memory (row r at r * 128, 16-byte chunk c at
// (c ^ (r & 7)) * 16), zero-padded past N and K.  A row tile's k range is then contiguous: one
// bulk copy moves a whole stage of it.
constexpr int kPackBlock = 16 * kBoxK;   // bytes of one packed block

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__global__ void __launch_bounds__(256) pack_weight_kernel(const int8_t *__restrict__ w, int N, int K, int KB,
                                                          int8_t *__restrict__ out, int64_t chunks) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < chunks; i += (int64_t)gridDim.x * blockDim.x) {
    // destination chunk i: block (t, kb), row r, stored chunk q (holding source chunk q ^ (r & 7))
    const int q = (int)(i & 7), r = (int)((i >> 3) & 15);
    const int64_t blk = i >> 7;
    const int kb = (int)(blk % KB), t = (int)(blk / KB);
    const int row = t * 16 + r, k0 = kb * kBoxK + ((q ^ (r & 7)) << 4);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < N && k0 < K) v = *reinterpret_cast<const uint4 *>(w + (int64_t)row * K + k0);
    reinterpret_cast<uint4 *>(out)[i] = v;
  }
}


// Bytes (lo, hi) of `biased` (the int8 word xor 0x80808080) as an exact 16-bit pair of the
// activation type; SEL picks the two bytes (0x4140: bytes 0,1; 0x4342: bytes 2,3).
template <typename XT, uint32_t SEL> __device__ __forceinline__ uint32_t i8pair(uint32_t biased);

template <> __device__ __forceinline__ uint32_t i8pair<__half, 0x4140u>(uint32_t u) {
  uint32_t h = __byte_perm(u, 0x64646464u, 0x4140u), r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));  // (1024 + u) - 1152
  return r;
}
template <> __device__ __forceinline__ uint32_t i8pair<__half, 0x4342u>(uint32_t u) {
  uint32_t h = __byte_perm(u, 0x64646464u, 0x4342u), r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
  return r;
}

__device__ __forceinline__ uint32_t bf16pair_from_bytes(uint32_t u, uint32_t sel_lo, uint32_t sel_hi) {
  // fp32 (2^23 + u_byte) for both bytes, minus 2^23 + 128, exact; integers below 2^8 have zero
  // low 16 bits in fp32, so the high halves are the bf16 values.
  const uint32_t f0 = __byte_perm(u, 0x4B000000u, sel_lo);
  const uint32_t f1 = __byte_perm(u, 0x4B000000u, sel_hi);
  unsigned long long p = (static_cast<unsigned long long>(f1) << 32) | f0;
  const unsigned long long bias = (static_cast<unsigned long long>(0x4B000080u) << 32) | 0x4B000080u;
  asm("sub.rn.f32x2 %0, %0, %1;" : "+l"(p) : "l"(bias));
  return __byte_perm(static_cast<uint32_t>(p), static_cast<uint32_t>(p >> 32), 0x7632u);
}
template <> __device__ __forceinline__ uint32_t i8pair<__nv_bfloat16, 0x4140u>(uint32_t u) {
  return bf16pair_from_bytes(u, 0x7540u, 0x7541u);
}
template <> __device__ __forceinline__ uint32_t i8pair<__nv_bfloat16, 0x4342u>(uint32_t u) {
  return bf16pair_from_bytes(u, 0x7542u, 0x7543u);
}

template <typename XT>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// Grid (ceil(N / (16*RT)), ceil(M / (8*MT))), 160 threads.  Dynamic shared memory: the ring of
// ST stages (each, 1024-byte aligned: 4 weight boxes of 128 k x 16*RT rows, then 4 x boxes of
// 128 k x XR rows at 128-byte alignment) + kCWarps * RT * MT * 128 floats for the final sum.
template <typename XT, int RT, int MT, int CW>
__global__ void __launch_bounds__((CW + 1) * 32) int8_tma_kernel(const __grid_constant__ CUtensorMap tmW,
                                                            const __grid_constant__ CUtensorMap tmX,
                                                            const void *__restrict__ scale, int scale_dt,
                                                            const XT *__restrict__ bias, XT *__restrict__ y, int M,
                                                            int N, int K, int ST, int XR, int xbox_bytes, int glu,
                                                            const int8_t *__restrict__ wpk) {
  constexpr int kWBoxBytes = kBoxK * 16 * RT;
  constexpr int P = RT * MT * 128;  // floats of one warp's partial tile
  const int stage_bytes = (CW * (kWBoxBytes + xbox_bytes) + 1023) & ~1023;
  const uint32_t xtx = (uint32_t)(kBoxK * XR * sizeof(XT));  // bytes one x box brings
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages];
  __shared__ int any_fail;
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *red = reinterpret_cast<float *>(ring + (size_t)ST * stage_bytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_base = blockIdx.x * 16 * RT;
  const int m_base = blockIdx.y * 8 * MT;
  const int nst = (K + (CW * kBoxK) - 1) / (CW * kBoxK);
  // Weight tile (rt, box bx) of a stage: [bx][rt] for tensor-map boxes (one box spans the CTA's
  // 16*RT rows), [rt][bx] for packed blocks (one bulk copy per row tile spans its boxes).
  const int rt_stride = wpk ? CW * kPackBlock : kPackBlock;
  const int bx_stride = wpk ? kPackBlock : kWBoxBytes;
  const int KB = (K + kBoxK - 1) / kBoxK;
  const int n_tiles = (N + 15) / 16;
  auto wbox = [&](int slot, int bx) { return ring + (size_t)slot * stage_bytes + bx * bx_stride; };
  auto wtile = [&](int slot, int rt) { return ring + (size_t)slot * stage_bytes + rt * rt_stride; };
  auto xbox = [&](int slot, int bx) {
    return ring + (size_t)slot * stage_bytes + CW * kWBoxBytes + bx * xbox_bytes;
  };

  // Programmatic dependent launch: the next kernel on the stream may start its own prologue now;
  // it still waits (griddepcontrol.wait) for this grid to finish before reading what we write.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], CW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    any_fail = 0;
  }
  __syncthreads();

  if (warp == CW) {
    // ---------------- producer ----------------
    if (lane == 0) {
      bool ok = true;
      auto boxes_of = [&](int s) { return min(CW, (K - s * (CW * kBoxK) + kBoxK - 1) / kBoxK); };
      // The weights of the first stages go out before the previous kernel has finished (they
      // are never written by a preceding kernel of a decode step); x only after it has.
      const int pre = min(ST, nst);
      const int tiles = wpk ? max(0, min(RT, n_tiles - n_base / 16)) : RT;  // packed: tiles that exist
      auto load_w = [&](int slot, int s, int boxes) {
        if (wpk) {
          for (int rt = 0; rt < tiles; ++rt)
            bulk_load(wtile(slot, rt), wpk + ((int64_t)(n_base / 16 + rt) * KB + s * CW) * kPackBlock,
                      (uint32_t)(boxes * kPackBlock), &full_bar[slot]);
        } else {
          for (int bx = 0; bx < boxes; ++bx)
            tma_load_2d(wbox(slot, bx), &tmW, &full_bar[slot], s * (CW * kBoxK) + bx * kBoxK, n_base);
        }
      };
      auto stage_tx = [&](int boxes) {
        return (uint32_t)(boxes * ((wpk ? tiles * kPackBlock : kWBoxBytes) + xtx));
      };
      for (int s = 0; s < pre; ++s) {
        const int boxes = boxes_of(s);
        mbar_arrive_expect_tx(&full_bar[s], stage_tx(boxes));
        load_w(s, s, boxes);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int s = 0; s < pre; ++s)
        for (int bx = 0; bx < boxes_of(s); ++bx)
          tma_load_2d(xbox(s, bx), &tmX, &full_bar[s], s * (CW * kBoxK) + bx * kBoxK, m_base);
      for (int s = pre; s < nst; ++s) {
        const int slot = s % ST;
        if (!mbar_wait(&empty_bar[slot], (uint32_t)((s / ST - 1) & 1))) {
          atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
          ok = false;
          break;
        }
        const int boxes = boxes_of(s);
        mbar_arrive_expect_tx(&full_bar[slot], stage_tx(boxes));
        load_w(slot, s, boxes);
        for (int bx = 0; bx < boxes; ++bx)
          tma_load_2d(xbox(slot, bx), &tmX, &full_bar[slot], s * (CW * kBoxK) + bx * kBoxK, m_base);
      }
      // drain: the copies of the last stages land before this CTA can finish
      for (int s = max(0, nst - ST); s < nst && ok; ++s)
        if (!mbar_wait(&full_bar[s % ST], (uint32_t)((s / ST) & 1))) atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, j = lane & 3;
  float acc[RT][MT][4];
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int nt = 0; nt < MT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[rt][nt][e] = 0.f;

  for (int s = 0; s < nst; ++s) {
    const int slot = s % ST;
    const int kbox = s * (CW * kBoxK) + warp * kBoxK;
    if (!mbar_wait(&full_bar[slot], (uint32_t)((s / ST) & 1))) {
      atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
      any_fail = 1;
      break;
    }
    if (kbox < K) {
      const uint32_t box = smem_u32(wbox(slot, warp));  // row tile rt at + rt * rt_stride
      const uint32_t xb = smem_u32(xbox(slot, warp));
      // weights: rows g and g+8 of each row tile, 32 bytes each = 16-byte chunks 2j and 2j+1 of
      // the 128-byte row, stored at chunk ^ (row & 7) by the 128-byte swizzle
      uint4 wv[RT][2][2];
#pragma unroll
      for (int rt = 0; rt < RT; ++rt)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int r = rt * 16 + g + hr * 8;
#pragma unroll
          for (int c = 0; c < 2; ++c)
            wv[rt][hr][c] = lds128(box + rt * rt_stride + (r - rt * 16) * kBoxK + (((2 * j + c) ^ (r & 7)) << 4));
        }
#pragma unroll
      for (int nt = 0; nt < MT; ++nt) {
        // x: row nt*8 + g of the box (rows past XR are zero), k = 32j .. 32j+31 of the box
        const int r = nt * 8 + g;
        uint4 xl[4];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          xl[c] = r < XR ? lds128(xb + r * (kBoxK * (int)sizeof(XT)) + 64 * j + 16 * c) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {  // word u of the thread's 32 bytes: k = box + 32j + 4u + {0..3}
          const uint4 xa = xl[u >> 1];
          const uint32_t b0 = (u & 1) ? xa.z : xa.x;
          const uint32_t b1 = (u & 1) ? xa.w : xa.y;
#pragma unroll
          for (int rt = 0; rt < RT; ++rt) {
            const uint32_t w0 = (&wv[rt][0][u >> 2].x)[u & 3] ^ 0x80808080u;
            const uint32_t w1 = (&wv[rt][1][u >> 2].x)[u & 3] ^ 0x80808080u;
            mma16816<XT>(acc[rt][nt], i8pair<XT, 0x4140u>(w0), i8pair<XT, 0x4140u>(w1),
                         i8pair<XT, 0x4342u>(w0), i8pair<XT, 0x4342u>(w1), b0, b1);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[slot]);
  }

  // ---- sum the consumer warps' partial tiles (layout [warp][rt][nt][e][lane]) ----
#pragma unroll
  for (int rt = 0; rt < RT; ++rt)
#pragma unroll
    for (int nt = 0; nt < MT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp * P + ((rt * MT + nt) * 4 + e) * 32 + lane] = acc[rt][nt][e];
  asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
  if (any_fail) return;  // a stage never arrived: leave the rows unwritten (error word set)
  asm volatile("griddepcontrol.wait;" ::: "memory");  // y may still be read by the previous kernel
  if (glu) {
    // Gated unit: row tiles 2u and 2u+1 of W hold the gate and the up rows of outputs 16u..16u+15;
    // y[m, 16u + r] = silu(gate) * up, y [M, N/2].  The CTA owns whole tile pairs (RT even).
    const int half = N >> 1;
    for (int pos = threadIdx.x; pos < P; pos += CW * 32) {
      const int ln = pos & 31, e = (pos >> 5) & 3, tile = pos >> 7;
      const int rt = tile / MT, nt = tile - rt * MT;
      if (rt & 1) continue;
      const int pos_up = pos + MT * 128;  // same (nt, e, lane) of tile rt + 1
      float gv = 0.f, uv = 0.f;
#pragma unroll
      for (int wp = 0; wp < CW; ++wp) {
        gv += red[wp * P + pos];
        uv += red[wp * P + pos_up];
      }
      const int row = (ln >> 2) + ((e & 2) ? 8 : 0), col = (ln & 3) * 2 + (e & 1);
      const int ng = n_base + rt * 16 + row, nu = ng + 16, m = m_base + nt * 8 + col;
      if (nu < N && m < M) {
        gv *= load_f(scale, scale_dt, ng);
        uv *= load_f(scale, scale_dt, nu);
        if (bias) {
          gv += Elem<XT>::to_f(bias[ng]);
          uv += Elem<XT>::to_f(bias[nu]);
        }
        const float act = gv / (1.f + __expf(-gv));
        y[(int64_t)m * half + (ng >> 5) * 16 + (ng & 15)] = Elem<XT>::from_f(act * uv);
      }
    }
    return;
  }
  for (int pos = threadIdx.x; pos < P; pos += CW * 32) {
    float v = 0.f;
#pragma unroll
    for (int wp = 0; wp < CW; ++wp) v += red[wp * P + pos];
    const int ln = pos & 31, e = (pos >> 5) & 3, tile = pos >> 7;
    const int rt = tile / MT, nt = tile - rt * MT;
    const int row = (ln >> 2) + ((e & 2) ? 8 : 0), col = (ln & 3) * 2 + (e & 1);
    const int n = n_base + rt * 16 + row, m = m_base + nt * 8 + col;
    if (n < N && m < M) {
      v *= load_f(scale, scale_dt, n);
      if (bias) v += Elem<XT>::to_f(bias[n]);
      y[(int64_t)m * N + n] = Elem<XT>::from_f(v);
    }
  }
}

// 2-D map over W [N, K] int8: box 128 k x 16*RT rows, 128-byte swizzle, zero fill past the
// edges.  Encoded maps are cached (a model calls the same weights every step).
struct WMapKey {
  const void *w;
  int N, K, rows;
  bool operator==(const WMapKey &o) const { return w == o.w && N == o.N && K == o.K && rows == o.rows; }
};

bool weight_map(CUtensorMap *m, const int8_t *w, int N, int K, int rows) {
  constexpr size_t kSlots = 512;
  static std::mutex mu;
  static std::vector<std::pair<WMapKey, CUtensorMap>> cache;
  static size_t next = 0;
  const WMapKey key{w, N, K, rows};
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto &e : cache)
      if (e.first == key) {
        *m = e.second;
        return true;
      }
  }
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)N};
  cuuint64_t gstr[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {(cuuint32_t)kBoxK, (cuuint32_t)rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(w), gdim, gstr, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() < kSlots) {
    cache.emplace_back(key, *m);
  } else {
    cache[next] = {key, *m};
    next = (next + 1) % kSlots;
  }
  return true;
}

// 2-D map over x [M, K] (16-bit): box 128 k x XR rows, no swizzle, zero fill past the edges.
// Activations move between calls, so these maps are re-encoded when the pointer is new (small
// cache keyed by everything the map encodes).
bool act_map(CUtensorMap *m, const void *x, int xdt, int M, int K, int rows) {
  struct Key {
    const void *x;
    int dt, M, K, rows;
  };
  constexpr size_t kSlots = 64;
  static std::mutex mu;
  static std::vector<std::pair<Key, CUtensorMap>> cache;
  static size_t next = 0;
  const Key key{x, xdt, M, K, rows};
  auto same = [&](const Key &a) { return a.x == key.x && a.dt == key.dt && a.M == key.M && a.K == key.K && a.rows == key.rows; };
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto &e : cache)
      if (same(e.first)) {
        *m = e.second;
        return true;
      }
  }
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t gstr[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBoxK, (cuuint32_t)rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, xdt == HELM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void *>(x), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() < kSlots) {
    cache.emplace_back(key, *m);
  } else {
    cache[next] = {key, *m};
    next = (next + 1) % kSlots;
  }
  return true;
}

template <typename XT, int RT, int MT, int CW = kCWarps>
int launch_cfg(const void *x, int xdt, const int8_t *w, const void *scale, int sdt, const void *bias, void *y,
               int M, int N, int K, cudaStream_t st, int glu, const int8_t *wpk) {
  const int XR = M < 8 * MT ? M : 8 * MT;                          // x rows per box
  const int xbox_bytes = ((kBoxK * XR * (int)sizeof(XT)) + 127) & ~127;   // 128-byte aligned x boxes
  const int stage_bytes = (CW * (kBoxK * 16 * RT + xbox_bytes) + 1023) & ~1023;
  const int red_bytes = (int)sizeof(float) * CW * RT * MT * 128;
  const int ctas = ((N + 16 * RT - 1) / (16 * RT)) * ((M + 8 * MT - 1) / (8 * MT));
  const int ST = ring_stages(ctas, num_sms(), stage_bytes, red_bytes);
  const size_t smem = 1024 + (size_t)ST * stage_bytes + red_bytes;
  auto kern = int8_tma_kernel<XT, RT, MT, CW>;
  {
    static std::mutex mu;
    static std::vector<std::pair<int, size_t>> done;  // (device, bytes allowed)
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    size_t have = 0;
    for (const auto &d : done)
      if (d.first == dev) have = d.second;
    if (have < smem) {
      const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "int8_linear: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      done.emplace_back(dev, smem);
    }
  }
  CUtensorMap wmap, xmap;
  if (wpk) memset(&wmap, 0, sizeof(wmap));  // unused: the packed weights move by bulk copies
  if ((!wpk && !weight_map(&wmap, w, N, K, 16 * RT)) || !act_map(&xmap, x, xdt, M, K, XR))
    return fail(HELM_ERR_CUDA, "int8_linear: cuTensorMapEncodeTiled failed");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + 16 * RT - 1) / (16 * RT), (M + 8 * MT - 1) / (8 * MT));
  cfg.blockDim = dim3((CW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, wmap, xmap, scale, sdt, static_cast<const XT *>(bias),
                                           static_cast<XT *>(y), M, N, K, ST, XR, xbox_bytes, glu, wpk);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "int8_linear: launch: %s", cudaGetErrorString(e));
  return check_launch("int8_tma_kernel");
}

// Rows per CTA: the fewest row tiles (16 rows each, at most 4) for which every CTA is resident
// at once -- 3 CTAs per SM with one tile (64 KB ring), 2 with more (96 KB ring).
template <typename XT, int MT>
int launch_m(const void *x, int xdt, const int8_t *w, const void *scale, int sdt, const void *bias, void *y, int M, int N,
             int K, cudaStream_t st, int glu, const int8_t *wpk) {
  const int sms = num_sms();
  const int tiles = (N + 15) / 16;
  if (glu) {  // whole (gate, up) tile pairs per CTA
    if constexpr (MT >= 4) {
      return launch_cfg<XT, 2, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 1, wpk);
    } else {
      if (tiles <= 2 * 2 * sms) return launch_cfg<XT, 2, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 1, wpk);
      return launch_cfg<XT, 4, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 1, wpk);
    }
  }
  if constexpr (MT >= 4) {  // wide x tiles: one row tile per CTA (register budget)
    return launch_cfg<XT, 1, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 0, wpk);
  } else {
    // One row tile per CTA over a long K: eight consumer warps, 1024-k stages (half the stage
    // round trips of a 512-k ring for the same bytes in flight).  Measured: +27 % on
    // (4096, 12288); at K = 4096 it pays only for a single row of x (6144 x 4096: 7.7 -> 6.5 us
    // at M = 1, no change at M = 4 or 8).
    if (tiles <= 3 * sms && (K >= 8192 || (M == 1 && K >= 4096)))
      return launch_cfg<XT, 1, MT, 8>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 0, wpk);
    if (tiles <= 3 * sms) return launch_cfg<XT, 1, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 0, wpk);
    if (tiles <= 2 * 2 * sms) return launch_cfg<XT, 2, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 0, wpk);
    if (tiles <= 2 * 3 * sms) return launch_cfg<XT, 3, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 0, wpk);
    return launch_cfg<XT, 4, MT>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, 0, wpk);
  }
}

template <typename XT>
int launch(const void *x, int xdt, const int8_t *w, const void *scale, int sdt, const void *bias, void *y, int M, int N,
           int K, cudaStream_t st, int glu, const int8_t *wpk = nullptr) {
  if (M <= 8) return launch_m<XT, 1>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, glu, wpk);
  if (M <= 16) return launch_m<XT, 2>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, glu, wpk);
  if (M <= 32) return launch_m<XT, 4>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, glu, wpk);
  return launch_m<XT, 8>(x, xdt, w, scale, sdt, bias, y, M, N, K, st, glu, wpk);
}

int check_args(const void *x, int32_t x_dtype, const int8_t *w, const void *w_scale, int32_t scale_dtype, void *y,
               int32_t M, int32_t N, int32_t K, const char *what) {
  if (M < 0 || N < 0 || K <= 0) return fail(HELM_ERR_INVALID_ARGUMENT, "%s: bad sizes M=%d N=%d K=%d", what, M, N, K);
  if (K % 16) return fail(HELM_ERR_UNSUPPORTED, "%s: K=%d is not a multiple of 16", what, K);
  if (x_dtype != HELM_F16 && x_dtype != HELM_BF16) return fail(HELM_ERR_UNSUPPORTED, "%s: x dtype %d", what, x_dtype);
  if (scale_dtype != HELM_F16 && scale_dtype != HELM_BF16 && scale_dtype != HELM_F32)
    return fail(HELM_ERR_UNSUPPORTED, "%s: scale dtype %d", what, scale_dtype);
  if (M == 0 || N == 0) return HELM_OK;
  if (!x || !w || !w_scale || !y) return fail(HELM_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15)
    return fail(HELM_ERR_INVALID_ARGUMENT, "%s: x and w must be 16-byte aligned", what);
  if ((int64_t)M > 65535ll * 8) return fail(HELM_ERR_UNSUPPORTED, "%s: M=%d too large", what, M);
  return HELM_OK;
}

}  // namespace
}  // namespace helm

#include "int8_gemm_tc.cuh"

extern "C" int helm_int8_linear(const void *x, int32_t x_dtype, const int8_t *w, const void *w_scale,
                                int32_t scale_dtype, const void *bias, void *y, int32_t M, int32_t N, int32_t K,
                                void *stream) {
  helm::NvtxRange nvtx_range_("helm_int8_linear");
  using namespace helm;
  const int rc = check_args(x, x_dtype, w, w_scale, scale_dtype, y, M, N, K, "int8_linear");
  if (rc != HELM_OK || M == 0 || N == 0) return rc;
  cudaStream_t st = as_stream(stream);
  return x_dtype == HELM_F16 ? launch<__half>(x, x_dtype, w, w_scale, scale_dtype, bias, y, M, N, K, st, 0)
                             : launch<__nv_bfloat16>(x, x_dtype, w, w_scale, scale_dtype, bias, y, M, N, K, st, 0);
}

extern "C" int helm_int8_linear_glu(const void *x, int32_t x_dtype, const int8_t *w, const void *w_scale,
                                    int32_t scale_dtype, const void *bias, void *y, int32_t M, int32_t I, int32_t K,
                                    void *stream) {
  helm::NvtxRange nvtx_range_("helm_int8_linear_glu");
  using namespace helm;
  if (I < 0 || I % 16) return fail(HELM_ERR_UNSUPPORTED, "int8_linear_glu: I=%d is not a multiple of 16", I);
  const int rc = check_args(x, x_dtype, w, w_scale, scale_dtype, y, M, 2 * I, K, "int8_linear_glu");
  if (rc != HELM_OK || M == 0 || I == 0) return rc;
  cudaStream_t st = as_stream(stream);
  return x_dtype == HELM_F16 ? launch<__half>(x, x_dtype, w, w_scale, scale_dtype, bias, y, M, 2 * I, K, st, 1)
                             : launch<__nv_bfloat16>(x, x_dtype, w, w_scale, scale_dtype, bias, y, M, 2 * I, K, st, 1);
}

extern "C" int64_t helm_int8_packed_bytes(int32_t N, int32_t K) {
  if (N < 0 || K <= 0 || K % 16) return -1;
  return (int64_t)((N + 15) / 16) * ((K + 127) / 128) * helm::kPackBlock;
}

extern "C" int helm_int8_pack_weight(const int8_t *w, int32_t N, int32_t K, int8_t *packed, void *stream) {
  helm::NvtxRange nvtx_range_("helm_int8_pack_weight");
  using namespace helm;
  if (N < 0 || K <= 0) return fail(HELM_ERR_INVALID_ARGUMENT, "int8_pack_weight: bad sizes N=%d K=%d", N, K);
  if (K % 16) return fail(HELM_ERR_UNSUPPORTED, "int8_pack_weight: K=%d is not a multiple of 16", K);
  if (N == 0) return HELM_OK;
  if (!w || !packed) return fail(HELM_ERR_INVALID_ARGUMENT, "int8_pack_weight: null pointer");
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(packed)) & 15)
    return fail(HELM_ERR_INVALID_ARGUMENT, "int8_pack_weight: w and packed must be 16-byte aligned");
  const int KB = (K + kBoxK - 1) / kBoxK;
  const int64_t chunks = helm_int8_packed_bytes(N, K) / 16;
  const int64_t want = (chunks + 255) / 256;
  const int grid = (int)(want < 16 * num_sms() ? want : 16 * num_sms());
  pack_weight_kernel<<<grid, 256, 0, as_stream(stream)>>>(w, N, K, KB, packed, chunks);
  return check_launch("pack_weight_kernel");
}

extern "C" int helm_int8_linear_packed(const void *x, int32_t x_dtype, const int8_t *packed, const void *w_scale,
                                       int32_t scale_dtype, const void *bias, void *y, int32_t M, int32_t N, int32_t K,
                                       void *stream) {
  helm::NvtxRange nvtx_range_("helm_int8_linear_packed");
  using namespace helm;
  const int rc = check_args(x, x_dtype, packed, w_scale, scale_dtype, y, M, N, K, "int8_linear_packed");
  if (rc != HELM_OK || M == 0 || N == 0) return rc;
  cudaStream_t st = as_stream(stream);
  return x_dtype == HELM_F16 ? launch<__half>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, N, K, st, 0, packed)
                             : launch<__nv_bfloat16>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, N, K, st, 0,
                                                     packed);
}

extern "C" int helm_int8_linear_glu_packed(const void *x, int32_t x_dtype, const int8_t *packed, const void *w_scale,
                                           int32_t scale_dtype, const void *bias, void *y, int32_t M, int32_t I,
                                           int32_t K, void *stream) {
  helm::NvtxRange nvtx_range_("helm_int8_linear_glu_packed");
  using namespace helm;
  if (I < 0 || I % 16) return fail(HELM_ERR_UNSUPPORTED, "int8_linear_glu_packed: I=%d is not a multiple of 16", I);
  const int rc = check_args(x, x_dtype, packed, w_scale, scale_dtype, y, M, 2 * I, K, "int8_linear_glu_packed");
  if (rc != HELM_OK || M == 0 || I == 0) return rc;
  cudaStream_t st = as_stream(stream);
  return x_dtype == HELM_F16
             ? launch<__half>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, 2 * I, K, st, 1, packed)
             : launch<__nv_bfloat16>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, 2 * I, K, st, 1, packed);
}

extern "C" int helm_int8_linear_error(int32_t *flag_out, int32_t reset) {
  helm::NvtxRange nvtx_range_("helm_int8_linear_error");
  using namespace helm;
  if (!flag_out) return fail(HELM_ERR_INVALID_ARGUMENT, "int8_linear_error: null pointer");
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_int8_error, sizeof(int));
  if (e == cudaSuccess && reset && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_int8_error, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "int8_linear_error: %s", cudaGetErrorString(e));
  *flag_out = v;
  return HELM_OK;
}
