// INT8 weight-only GEMM for prefill-sized inputs on the 5th-generation tensor cores (tcgen05).
//
//   y[m, n] = (sum_k x[m, k] * w[n, k]) * s[n] + bias[n]
//
// with w int8 in the packed block layout of helm_int8_pack_weight and x bf16 / fp16.  It is the
// M > 64 companion of the decode GEMV (int8_linear.cu): the same arithmetic -- exact int8 -> 16-bit
// conversion, fp32 accumulation, the per-channel scale and the bias applied once per output -- as
// a dense contraction, so that prefill no longer builds a dequantised copy of the weight.
//
// The weight is the A operand and lives in tensor memory; x is the B operand in shared memory:
//   D[n, m] (128 channels x 256 tokens, fp32, tensor memory) += W[n, k] . x[m, k]
// CTA tile 128 output channels x 256 tokens; k in steps of 128 (one packed block column, eight
// MMAs of K = 16 per step, which halves the per-step barrier round trips of 64-k steps).  Each
// converted weight element feeds
// 256 tokens, and the converted weights go from registers to tensor memory (tcgen05.st) instead of
// through shared memory, which leaves shared memory to the x tiles and the int8 blocks.
//   x   (256 tokens x 128 k as two 64-k boxes, 64 KB, 3 deep)  shared memory, filled by TMA (128-byte
//                                            swizzle), released by the MMAs (tcgen05.commit);
//   W   (packed int8 block column: 128 channels x 128 k, 16 KB, 2 deep)  shared memory, filled by bulk
//                                            copies, released by the converters;
//   A   (converted 16-bit weights: 128 lanes x 64 columns per k step, 2 deep)  tensor memory, written
//                                            by the converters, released by the MMAs.
// Warp roles (576 threads):
//   warp 0      producer: TMA for x, bulk copies for the packed weight blocks;
//   warp 1      MMA issuer: one thread issues tcgen05.mma kind::f16 with A in tensor memory (M=128
//               channels, N=256 tokens, K=16; B = x, K-major 128-byte-swizzled descriptor; D in
//               tensor memory) eight times per k step, then tcgen05.commit to the x and A empty
//               barriers;
//   warps 2-17  converters, then the epilogue.  Warp w may address the tensor-memory lanes
//               32*(w%4)..+31, so thread (w, l) owns channel row 32*(w%4) + l.  The warps form two
//               groups of eight (two per lane quadrant, one per half of the 128 k); group g converts
//               the k steps j with j % 2 == g from W stage g into A stage g, so a conversion has
//               two k steps of MMA time to finish and no barrier is waited on two phases ahead.
//               A row's 64 int8 values of a half step (four 16-byte chunks of its packed block row)
//               become 32 words of exact 16-bit pairs, stored with tcgen05.st into the stage's
//               columns (column c holds k = 2c, 2c+1).  After the last k step the same threads read
//               their channel's accumulators (tcgen05.ld, 32 tokens at a time, 64 tokens a warp),
//               apply the channel's scale and bias and store y.
// Tensor memory: 512 columns -- the 128 x 256 accumulator in columns 0-255, the A ring in 256-383.
// Every mbarrier wait is bounded: a wait that gives up sets HELM_DEVERR_TIMEOUT in the library's
// INT8 error word; the CTA then skips its remaining work and its stores, waits (bounded) for the
// copies it issued, and frees its tensor memory.
// Included by int8_linear.cu (it shares that file's INT8 error word, g_int8_error).
#pragma once

namespace helm {
namespace {

constexpr int GCH = 128, GTK = 256, GK = 128;    // CTA tile: channels x tokens; k step (one block column)
// kWStages == kAStages == the number of converter groups: group g converts the k steps j with
// j % 2 == g from W stage g into A stage g, so no barrier is ever waited on two phases ahead.
constexpr int kXStages = 3, kWStages = 2, kAStages = 2;
constexpr int kXBoxBytes = GTK * 64 * 2;         // 32 KB: one 64-k TMA box of 256 token rows x 128 B
constexpr int kXStageBytes = 2 * kXBoxBytes;     // 64 KB: the k step's two boxes
constexpr int kWStageBytes = GCH * 128;          // 16 KB: 8 packed blocks (16 rows x 128 k)
constexpr int kGSmem = kXStages * kXStageBytes + kWStages * kWStageBytes + 1024;
constexpr int kConvWarps = 16;                  // four groups of four (one per tensor-memory lane quadrant)
constexpr int kGroupWarps = 8;                  // two per lane quadrant, one per half of the 128 k
constexpr int kGThreads = (2 + kConvWarps) * 32;
constexpr int kTmemCols = 512;
constexpr int kAccCol = 0, kACol0 = 256, kAStageCols = GK / 2;   // 64 columns of 16-bit pairs per k step

__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr) {
  // K-major, 128-byte swizzle: leading byte offset 1 (16 B, unused for this layout), stride byte
  // offset 1024 B (eight 128-byte rows), descriptor version 1, base offset 0 (1024-aligned atoms).
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

template <typename XT> struct UFmt;
template <> struct UFmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };
template <> struct UFmt<__half> { static constexpr uint32_t v = 0; };

// kind::f16 instruction descriptor: fp32 accumulator, A and B of type XT, both K-major,
// N = GTK tokens (n_dim = N >> 3), M = GCH channels (m_dim = M >> 4).
template <typename XT> __device__ __forceinline__ uint32_t umma_idesc() {
  return (1u << 4) | (UFmt<XT>::v << 7) | (UFmt<XT>::v << 10) | ((uint32_t)(GTK >> 3) << 17) |
         ((uint32_t)(GCH >> 4) << 24);
}

// D[tmem_d] (+)= A[tmem_a] . B[desc]^T, A read from tensor memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 16 consecutive 32-bit columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 int8 values -> 16 exact 16-bit values of XT, as two 16-byte chunks (the pairwise conversions
// of the decode GEMV: int8 -> fp16 / bf16 without rounding).
template <typename XT> __device__ __forceinline__ void cvt16(const uint4 &raw, uint4 &lo, uint4 &hi) {
  const uint32_t w[4] = {raw.x ^ 0x80808080u, raw.y ^ 0x80808080u, raw.z ^ 0x80808080u, raw.w ^ 0x80808080u};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = i8pair<XT, 0x4140u>(w[i]);
    o[2 * i + 1] = i8pair<XT, 0x4342u>(w[i]);
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

template <typename XT>
__global__ void __launch_bounds__(kGThreads, 1)
    int8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const int8_t *__restrict__ wpk,
                        const void *__restrict__ scale, int scale_dt, const XT *__restrict__ bias,
                        XT *__restrict__ y, int M, int N, int K) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t x_full[kXStages], x_empty[kXStages];
  __shared__ __align__(8) uint64_t w_full[kWStages], w_empty[kWStages];
  __shared__ __align__(8) uint64_t a_full[kAStages], a_empty[kAStages];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *x_ring = smem;
  uint8_t *w_ring = x_ring + kXStages * kXStageBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * GCH, m0 = blockIdx.y * GTK;
  const int KB = (K + 127) / 128;          // packed block columns
  const int NK = (K + GK - 1) / GK;        // k steps
  const int n_tiles = (N + 15) / 16;
  const int tiles = max(0, min(GCH / 16, n_tiles - n0 / 16));   // packed 16-row tiles that exist

  if (threadIdx.x == 0) {
    for (int s = 0; s < kXStages; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], kGroupWarps);       // the eight warps of the group converting it
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], kGroupWarps);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(&acc_bar, 1);
    failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  pdl_trigger();
  pdl_wait();

  auto give_up = [&]() {
    atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
    failed = 1;
  };

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int x_issued = 0, w_issued = 0;
      for (int j = 0; j < NK && !*reinterpret_cast<volatile int *>(&failed); ++j) {
        const int ws = j % kWStages;             // the packed block column of k step j
        if (j >= kWStages && !mbar_wait(&w_empty[ws], (uint32_t)((j / kWStages - 1) & 1))) {
          give_up();
          break;
        }
        mbar_arrive_expect_tx(&w_full[ws], (uint32_t)(tiles * 2048));
        for (int t = 0; t < tiles; ++t)
          bulk_g2s(w_ring + ws * kWStageBytes + t * 2048, wpk + ((int64_t)(n0 / 16 + t) * KB + j) * 2048, 2048,
                   &w_full[ws]);
        w_issued = j + 1;
        const int xs = j % kXStages;
        if (j >= kXStages && !mbar_wait(&x_empty[xs], (uint32_t)((j / kXStages - 1) & 1))) {
          give_up();
          break;
        }
        // the second 64-k box only where it starts inside K (a box wholly past the edge is not
        // loaded; the MMAs of the last step stop at K)
        const bool two = j * GK + 64 < K;
        mbar_arrive_expect_tx(&x_full[xs], (uint32_t)(two ? kXStageBytes : kXBoxBytes));
        tma_load_2d(x_ring + xs * kXStageBytes, &tmX, &x_full[xs], j * GK, m0);
        if (two) tma_load_2d(x_ring + xs * kXStageBytes + kXBoxBytes, &tmX, &x_full[xs], j * GK + 64, m0);
        x_issued = j + 1;
      }
      // the copies still in flight land before this CTA can finish
      for (int j = max(0, x_issued - kXStages); j < x_issued; ++j)
        if (!mbar_wait(&x_full[j % kXStages], (uint32_t)((j / kXStages) & 1))) give_up();
      for (int c = max(0, w_issued - kWStages); c < w_issued; ++c)
        if (!mbar_wait(&w_full[c % kWStages], (uint32_t)((c / kWStages) & 1))) give_up();  // c: k step
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc<XT>();
      for (int j = 0; j < NK; ++j) {
        const int xs = j % kXStages, as = j % kAStages;
        if (!mbar_wait(&x_full[xs], (uint32_t)((j / kXStages) & 1)) ||
            !mbar_wait(&a_full[as], (uint32_t)((j / kAStages) & 1))) {
          give_up();
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t b0 = smem_u32(x_ring + xs * kXStageBytes);
        const uint32_t a0 = tmem + (uint32_t)(kACol0 + as * kAStageCols);
        const int nkk = min(GK / 16, (K - j * GK) / 16);   // K is a multiple of 16
#pragma unroll
        for (int kk = 0; kk < GK / 16; ++kk)       // k 16*kk: box kk/4, 32-byte column (kk%4) of its rows
          if (kk < nkk)
            umma_f16_ts(tmem + kAccCol, a0 + kk * 8, umma_smem_desc(b0 + (kk >> 2) * kXBoxBytes + (kk & 3) * 32),
                        idesc, (j | kk) != 0);
        umma_commit(&x_empty[xs]);
        umma_commit(&a_empty[as]);
      }
      umma_commit(&acc_bar);
    }
  } else {
    // ---------------- converters ----------------
    // Group g (warps 2+4g .. 5+4g, one per lane quadrant) converts k steps g, g+4, g+8, ... into
    // A stage g, so each group has four k steps of MMA time for one conversion.
    const int quad = warp & 3;                 // the tensor-memory lanes this warp may address
    const int grp = (warp - 2) >> 3;           // k steps j with j % 2 == grp; W and A stage grp
    const int half = ((warp - 2) >> 2) & 1;    // which 64 k of the step
    const int r = quad * 32 + lane;            // channel row of the tile
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const uint32_t a_addr = tmem + lane_addr + (uint32_t)(kACol0 + grp * kAStageCols + half * 32);
    for (int j = grp; j < NK; j += kAStages) {
      const int ws = j % kWStages;
      // Read and convert the int8 block column as soon as it lands, release the W stage, and only
      // then wait for the MMAs to free A stage grp: the conversion overlaps the running MMAs, and
      // only the tensor-memory stores sit between an A stage's release and its refill.
      if (!mbar_wait(&w_full[ws], (uint32_t)((j / kWStages) & 1))) {
        give_up();
        break;
      }
      const uint8_t *row = w_ring + ws * kWStageBytes + (r >> 4) * 2048 + (r & 15) * 128;
      uint4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)             // logical 16-value chunk 4*half + i of the row (its swizzled slot)
        v[i] = *reinterpret_cast<const uint4 *>(row + (((4 * half + i) ^ (r & 7)) << 4));
      uint32_t w[2][16];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint4 q0, q1, q2, q3;
        cvt16<XT>(v[2 * h], q0, q1);
        cvt16<XT>(v[2 * h + 1], q2, q3);
        const uint32_t t[16] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w,
                                q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
#pragma unroll
        for (int e = 0; e < 16; ++e) w[h][e] = t[e];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&w_empty[ws]);   // the warp's reads of the stage are done
      if (j >= kAStages && !mbar_wait(&a_empty[grp], (uint32_t)((j / kAStages - 1) & 1))) {
        give_up();
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      tmem_st16(a_addr, w[0]);
      tmem_st16(a_addr + 16u, w[1]);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[grp]);
    }
    // ---------------- epilogue ----------------
    if (!mbar_wait(&acc_bar, 0u)) {
      give_up();
    } else {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int n = n0 + r;
      const float sc = n < N ? load_f(scale, scale_dt, n) : 0.f;
      const float bi = (bias && n < N) ? Elem<XT>::to_f(bias[n]) : 0.f;
      const bool store = n < N && !*reinterpret_cast<volatile int *>(&failed);
      constexpr int kCols = GTK / (kConvWarps / 4);   // token columns per warp
      const int slot = grp * 2 + half;                // the quadrant's four warps split the 256 tokens
#pragma unroll 1
      for (int c0 = slot * kCols; c0 < slot * kCols + kCols; c0 += 32) {
        float acc[32];
        tmem_ld32(tmem + lane_addr + (uint32_t)(kAccCol + c0), acc);
        if (!store) continue;
        XT *dst = y + (int64_t)(m0 + c0) * N + n;
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          if (m0 + c0 + jj < M) dst[(int64_t)jj * N] = Elem<XT>::from_f(fmaf(acc[jj], sc, bi));
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// 2-D map over x [M, K] (16-bit): box 64 k x 256 tokens, 128-byte swizzle, zero fill past the edges.
bool x_map_sw128(CUtensorMap *m, const void *x, int xdt, int M, int K) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t gstr[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)GTK};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, xdt == HELM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
             const_cast<void *>(x), gdim, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename XT>
int launch_gemm(const void *x, int xdt, const int8_t *wpk, const void *scale, int sdt, const void *bias, void *y,
                int M, int N, int K, cudaStream_t st) {
  {
    static std::mutex mu;
    static std::vector<int> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    bool have = false;
    for (int d : done) have = have || d == dev;
    if (!have) {
      const cudaError_t e =
          cudaFuncSetAttribute(int8_gemm_tc_kernel<XT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem);
      if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "int8_gemm: cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      done.push_back(dev);
    }
  }
  CUtensorMap xm;
  if (!x_map_sw128(&xm, x, xdt, M, K)) return fail(HELM_ERR_CUDA, "int8_gemm: cuTensorMapEncodeTiled failed");
  const dim3 grid((N + GCH - 1) / GCH, (M + GTK - 1) / GTK);
  const cudaError_t e = launch_pdl(int8_gemm_tc_kernel<XT>, grid, dim3(kGThreads), kGSmem, st, xm, wpk, scale, sdt,
                                   static_cast<const XT *>(bias), static_cast<XT *>(y), M, N, K);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "int8_gemm: launch: %s", cudaGetErrorString(e));
  return check_launch("int8_gemm_tc_kernel");
}

}  // namespace
}  // namespace helm

extern "C" int helm_int8_gemm_packed(const void *x, int32_t x_dtype, const int8_t *packed, const void *w_scale,
                                     int32_t scale_dtype, const void *bias, void *y, int32_t M, int32_t N, int32_t K,
                                     void *stream) {
  helm::NvtxRange nvtx_range_("helm_int8_gemm_packed");
  using namespace helm;
  if (M < 0 || N < 0 || K <= 0) return fail(HELM_ERR_INVALID_ARGUMENT, "int8_gemm: bad sizes M=%d N=%d K=%d", M, N, K);
  if (K % 16) return fail(HELM_ERR_UNSUPPORTED, "int8_gemm: K=%d is not a multiple of 16", K);
  if (x_dtype != HELM_F16 && x_dtype != HELM_BF16) return fail(HELM_ERR_UNSUPPORTED, "int8_gemm: x dtype %d", x_dtype);
  if (scale_dtype != HELM_F16 && scale_dtype != HELM_BF16 && scale_dtype != HELM_F32)
    return fail(HELM_ERR_UNSUPPORTED, "int8_gemm: scale dtype %d", scale_dtype);
  if (M == 0 || N == 0) return HELM_OK;
  if (!x || !packed || !w_scale || !y) return fail(HELM_ERR_INVALID_ARGUMENT, "int8_gemm: null pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(packed)) & 15)
    return fail(HELM_ERR_INVALID_ARGUMENT, "int8_gemm: x and packed must be 16-byte aligned");
  if ((int64_t)(M + GTK - 1) / GTK > 65535) return fail(HELM_ERR_UNSUPPORTED, "int8_gemm: M=%d too large", M);
  cudaStream_t st = as_stream(stream);
  return x_dtype == HELM_F16 ? launch_gemm<__half>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, N, K, st)
                             : launch_gemm<__nv_bfloat16>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, N, K,
                                                          st);
}
