// INT8 weight-only GEMM for prefill-sized inputs on the 5th-generation tensor cores (tcgen05).
//
//   y[m, n] = (sum_k x[m, k] * w[n, k]) * s[n] + bias[n]
//
// with w int8 in the packed block layout of helm_int8_pack_weight and x bf16 / fp16.  It is the
// M > 64 companion of the decode GEMV (int8_linear.cu): the same arithmetic -- exact int8 -> 16-bit
// conversion, fp32 accumulation, the per-channel scale and the bias applied once per output -- as
// a dense contraction, so that prefill no longer builds a dequantised copy of the weight.
//
// CTA tile 128 (tokens) x 128 (output channels), k in stages of 128 (one packed block column).
// Warp roles (192 threads):
//   warp 0      TMA producer: x tile (two 64-k boxes, 128-byte swizzle) and the eight packed
//               16-row weight blocks of the stage (bulk copies) into a 2-stage ring;
//   warps 1-4   converters, then the epilogue: each stage's int8 block is rewritten as 16-bit
//               values in the canonical K-major 128-byte-swizzled layout the tensor core reads
//               (exact: |w| <= 127), then fence.proxy.async and an mbarrier arrive; after the
//               last stage they read the fp32 accumulators back from tensor memory
//               (tcgen05.ld, one 32-lane quadrant per warp), apply scale and bias, store y;
//   warp 5      MMA issuer: one elected thread issues tcgen05.mma kind::f16 (M=128, N=128,
//               K=16, A = x, B = w, both K-major from shared memory descriptors, D in tensor
//               memory) for the 8 k-steps of a stage and releases the stage with tcgen05.commit.
// Tensor memory: 128 columns (the 128 x 128 fp32 accumulator), allocated by warp 0.
// Every mbarrier wait is bounded: a wait that gives up sets HELM_DEVERR_TIMEOUT in the library's
// INT8 error word; the CTA then skips its remaining work, waits (bounded) for the copies it
// issued and frees its tensor memory.
// Included by int8_linear.cu (it shares that file's INT8 error word, g_int8_error).
#pragma once

namespace helm {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int kGStages = 2;
constexpr int kAtomBytes = 128 * 128;                 // 128 rows x 64 16-bit values (128 B)
constexpr int kABytes = 2 * kAtomBytes;               // x tile: two k atoms
constexpr int kBBytes = 2 * kAtomBytes;               // converted weight tile
constexpr int kWBytes = BN * BK;                      // eight packed 16 x 128 int8 blocks
constexpr int kGStageBytes = kABytes + kBBytes + kWBytes;
constexpr int kGSmem = kGStages * kGStageBytes + 1024;
constexpr int kGThreads = 192;
constexpr int kTmemCols = 128;

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
// N = 128 (n_dim = N >> 3), M = 128 (m_dim = M >> 4).
template <typename XT> __device__ __forceinline__ uint32_t umma_idesc() {
  return (1u << 4) | (UFmt<XT>::v << 7) | (UFmt<XT>::v << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
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

// 16 int8 values -> 16 exact 16-bit values of XT, as two 16-byte chunks.
template <typename XT> __device__ __forceinline__ void cvt16(const int4 &raw, uint4 &lo, uint4 &hi) {
  const int8_t *b = reinterpret_cast<const int8_t *>(&raw);
  XT o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = Elem<XT>::from_f((float)b[i]);
  lo = *reinterpret_cast<const uint4 *>(&o[0]);
  hi = *reinterpret_cast<const uint4 *>(&o[8]);
}

template <typename XT>
__global__ void __launch_bounds__(kGThreads, 1)
    int8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const int8_t *__restrict__ wpk,
                        const void *__restrict__ scale, int scale_dt, const XT *__restrict__ bias,
                        XT *__restrict__ y, int M, int N, int K) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kGStages];
  __shared__ __align__(8) uint64_t ready_bar[kGStages];
  __shared__ __align__(8) uint64_t empty_bar[kGStages];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int KB = (K + BK - 1) / BK;
  const int n_tiles = (N + 15) / 16;
  auto a_tile = [&](int s) { return smem + (size_t)s * kGStageBytes; };
  auto b_tile = [&](int s) { return smem + (size_t)s * kGStageBytes + kABytes; };
  auto w_raw = [&](int s) { return smem + (size_t)s * kGStageBytes + kABytes + kBBytes; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&ready_bar[s], 4);
      mbar_init(&empty_bar[s], 1);
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

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const int tiles = max(0, min(BN / 16, n_tiles - n0 / 16));
      int issued = 0;
      for (int i = 0; i < KB; ++i) {
        const int s = i % kGStages;
        if (i >= kGStages && !mbar_wait(&empty_bar[s], (uint32_t)((i / kGStages - 1) & 1))) {
          atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
          failed = 1;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], (uint32_t)(kABytes + tiles * 2048));
        tma_load_2d(a_tile(s), &tmX, &full_bar[s], i * BK, m0);
        tma_load_2d(a_tile(s) + kAtomBytes, &tmX, &full_bar[s], i * BK + 64, m0);
        for (int t = 0; t < tiles; ++t)
          bulk_g2s(w_raw(s) + t * 2048, wpk + ((int64_t)(n0 / 16 + t) * KB + i) * 2048, 2048, &full_bar[s]);
        issued = i + 1;
      }
      // the copies of the last stages land before this CTA can finish
      for (int i = max(0, issued - kGStages); i < issued; ++i)
        if (!mbar_wait(&full_bar[i % kGStages], (uint32_t)((i / kGStages) & 1))) atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
    }
  } else if (warp <= 4) {
    // ---------------- converters ----------------
    const int tc = threadIdx.x - 32;  // 0..127
    for (int i = 0; i < KB; ++i) {
      const int s = i % kGStages;
      if (!mbar_wait(&full_bar[s], (uint32_t)((i / kGStages) & 1))) {
        atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
        failed = 1;
        break;
      }
      const uint8_t *raw = w_raw(s);
      uint8_t *bt = b_tile(s);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = tc + 128 * j;          // packed chunk: row r (0..127), stored position p
        const int r = q >> 3, p = q & 7;
        const int lc = p ^ (r & 7);          // logical 16-value chunk: k = 16*lc .. 16*lc + 15
        const int4 v = *reinterpret_cast<const int4 *>(raw + (r >> 4) * 2048 + (r & 15) * 128 + p * 16);
        uint4 lo, hi;
        cvt16<XT>(v, lo, hi);
        uint8_t *atom = bt + (lc >> 2) * kAtomBytes + r * 128;
        const int c0 = 2 * (lc & 3);
        *reinterpret_cast<uint4 *>(atom + (((c0) ^ (r & 7)) << 4)) = lo;
        *reinterpret_cast<uint4 *>(atom + (((c0 + 1) ^ (r & 7)) << 4)) = hi;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready_bar[s]);
    }
    // ---------------- epilogue ----------------
    if (!mbar_wait(&acc_bar, 0u)) {
      atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
      failed = 1;
    } else {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int quad = warp & 3;
      const int m = m0 + quad * 32 + lane;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float acc[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, acc);
        if (m < M && !*reinterpret_cast<volatile int *>(&failed)) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = n0 + c0 + j;
            if (n < N) {
              float v = acc[j] * load_f(scale, scale_dt, n);
              if (bias) v += Elem<XT>::to_f(bias[n]);
              y[(int64_t)m * N + n] = Elem<XT>::from_f(v);
            }
          }
        }
      }
    }
  } else {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = umma_idesc<XT>();
      bool ok = true;
      for (int i = 0; i < KB && ok; ++i) {
        const int s = i % kGStages;
        if (!mbar_wait(&full_bar[s], (uint32_t)((i / kGStages) & 1)) ||
            !mbar_wait(&ready_bar[s], (uint32_t)((i / kGStages) & 1))) {
          atomicOr(&g_int8_error, HELM_DEVERR_TIMEOUT);
          failed = 1;
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a0 = smem_u32(a_tile(s)), b0 = smem_u32(b_tile(s));
#pragma unroll
        for (int j = 0; j < BK / 16; ++j) {
          const uint32_t off = (uint32_t)((j >> 2) * kAtomBytes + (j & 3) * 32);
          umma_f16(tmem, umma_smem_desc(a0 + off), umma_smem_desc(b0 + off), idesc, (i | j) != 0);
        }
        umma_commit(&empty_bar[s]);
      }
      umma_commit(&acc_bar);
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// 2-D map over x [M, K] (16-bit): box 64 k x 128 rows, 128-byte swizzle, zero fill past the edges.
bool x_map_sw128(CUtensorMap *m, const void *x, int xdt, int M, int K) {
  auto enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t gstr[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)BM};
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
  const dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
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
  if ((int64_t)(M + BM - 1) / BM > 65535) return fail(HELM_ERR_UNSUPPORTED, "int8_gemm: M=%d too large", M);
  cudaStream_t st = as_stream(stream);
  return x_dtype == HELM_F16 ? launch_gemm<__half>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, N, K, st)
                             : launch_gemm<__nv_bfloat16>(x, x_dtype, packed, w_scale, scale_dtype, bias, y, M, N, K,
                                                          st);
}
