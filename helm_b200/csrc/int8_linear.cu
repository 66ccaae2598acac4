// INT8 weight-only linear: y[m, n] = (sum_k x[m, k] * w[n, k]) * s[n] + bias[n].
//
// The GPU counterpart of HELM's CPU decode GEMV (helm/kernels/fp16_gemv.cpp:
// 45-100, one fp16 weight row dotted with x, fp32 accumulation, rows spread
// over threads), with the weight stored as int8 plus one scale per output
// channel.  Decode-sized M (<= 8 per pass) runs on the CUDA cores: each warp
// streams 4 weight rows with 16-byte loads, dequantises the int8 bytes in
// registers (byte -> float through the 2^23 exponent trick, no I2F), and
// accumulates with packed fp32x2 FMAs; the per-channel scale is applied once
// per output in the epilogue.
#include "common.cuh"

namespace helm {

namespace {

constexpr int kRowsPerWarp = 4;
constexpr int kWarps = 8;
constexpr int kRowsPerBlock = kRowsPerWarp * kWarps;

__device__ __forceinline__ uint4 ld_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned long long f2u(float2 v) {
  return (static_cast<unsigned long long>(__float_as_uint(v.y)) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 u2f(unsigned long long u) {
  return make_float2(__uint_as_float(static_cast<uint32_t>(u)), __uint_as_float(static_cast<uint32_t>(u >> 32)));
}

// acc += a * b on both lanes of an fp32 pair.
__device__ __forceinline__ void ffma2(unsigned long long &acc, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

// Four signed bytes of `word` -> two fp32 pairs, exactly.  Each byte b is
// biased to b+128 in [0, 255], placed in the low mantissa byte of 2^23, and
// the float 2^23 + 128 is subtracted.
__device__ __forceinline__ void i8x4_to_f2x2(uint32_t word, unsigned long long &p01, unsigned long long &p23) {
  const uint32_t u = word ^ 0x80808080u;
  const uint32_t f0 = __byte_perm(u, 0x4B000000u, 0x7540);
  const uint32_t f1 = __byte_perm(u, 0x4B000000u, 0x7541);
  const uint32_t f2 = __byte_perm(u, 0x4B000000u, 0x7542);
  const uint32_t f3 = __byte_perm(u, 0x4B000000u, 0x7543);
  const unsigned long long bias = f2u(make_float2(8388736.f, 8388736.f));
  unsigned long long a = (static_cast<unsigned long long>(f1) << 32) | f0;
  unsigned long long c = (static_cast<unsigned long long>(f3) << 32) | f2;
  asm("sub.f32x2 %0, %0, %1;" : "+l"(a) : "l"(bias));
  asm("sub.f32x2 %0, %0, %1;" : "+l"(c) : "l"(bias));
  p01 = a;
  p23 = c;
}

template <typename XT> __device__ __forceinline__ unsigned long long x2_to_f2(uint32_t v);
template <> __device__ __forceinline__ unsigned long long x2_to_f2<__half>(uint32_t v) {
  return f2u(__half22float2(*reinterpret_cast<__half2 *>(&v)));
}
template <> __device__ __forceinline__ unsigned long long x2_to_f2<__nv_bfloat16>(uint32_t v) {
  return (static_cast<unsigned long long>(v & 0xffff0000u) << 32) | (v << 16);
}

template <typename XT, int MB>
__global__ void __launch_bounds__(256) int8_gemv_kernel(const XT *__restrict__ x, const int8_t *__restrict__ w,
                                                        const void *__restrict__ scale, int scale_dt,
                                                        const XT *__restrict__ bias, XT *__restrict__ y, int M,
                                                        int N, int K) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kRowsPerBlock + warp * kRowsPerWarp;
  const int m0 = blockIdx.y * MB;
  if (n0 >= N) return;
  const int mcount = min(MB, M - m0);

  unsigned long long acc[kRowsPerWarp][MB];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int m = 0; m < MB; ++m) acc[r][m] = 0ull;

  for (int k = lane * 16; k < K; k += 32 * 16) {
    uint4 wv[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
      wv[r] = (n0 + r < N) ? ld_stream(w + (int64_t)(n0 + r) * K + k) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      unsigned long long xf[MB][4];
#pragma unroll
      for (int m = 0; m < MB; ++m) {
        if (m < mcount) {
          const uint4 xv = __ldg(reinterpret_cast<const uint4 *>(x + (int64_t)(m0 + m) * K + k + 8 * half));
          xf[m][0] = x2_to_f2<XT>(xv.x);
          xf[m][1] = x2_to_f2<XT>(xv.y);
          xf[m][2] = x2_to_f2<XT>(xv.z);
          xf[m][3] = x2_to_f2<XT>(xv.w);
        } else {
          xf[m][0] = xf[m][1] = xf[m][2] = xf[m][3] = 0ull;
        }
      }
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        unsigned long long wf[4];
        i8x4_to_f2x2(half ? wv[r].z : wv[r].x, wf[0], wf[1]);
        i8x4_to_f2x2(half ? wv[r].w : wv[r].y, wf[2], wf[3]);
#pragma unroll
        for (int m = 0; m < MB; ++m)
#pragma unroll
          for (int j = 0; j < 4; ++j) ffma2(acc[r][m], wf[j], xf[m][j]);
      }
    }
  }

#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int n = n0 + r;
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      const float2 p = u2f(acc[r][m]);
      float v = p.x + p.y;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0 && n < N && m < mcount) {
        v *= load_f(scale, scale_dt, n);
        if (bias) v += Elem<XT>::to_f(bias[n]);
        y[(int64_t)(m0 + m) * N + n] = Elem<XT>::from_f(v);
      }
    }
  }
}

template <typename XT>
int launch(const void *x, const int8_t *w, const void *scale, int sdt, const void *bias, void *y, int M, int N,
           int K, cudaStream_t st) {
  const XT *xp = static_cast<const XT *>(x);
  const XT *bp = static_cast<const XT *>(bias);
  XT *yp = static_cast<XT *>(y);
  const int gx = (N + kRowsPerBlock - 1) / kRowsPerBlock;
  if (M == 1) {
    int8_gemv_kernel<XT, 1><<<dim3(gx, 1), 256, 0, st>>>(xp, w, scale, sdt, bp, yp, M, N, K);
  } else if (M == 2) {
    int8_gemv_kernel<XT, 2><<<dim3(gx, 1), 256, 0, st>>>(xp, w, scale, sdt, bp, yp, M, N, K);
  } else if (M <= 4) {
    int8_gemv_kernel<XT, 4><<<dim3(gx, 1), 256, 0, st>>>(xp, w, scale, sdt, bp, yp, M, N, K);
  } else {
    int8_gemv_kernel<XT, 8><<<dim3(gx, (M + 7) / 8), 256, 0, st>>>(xp, w, scale, sdt, bp, yp, M, N, K);
  }
  return check_launch("int8_gemv_kernel");
}

}  // namespace
}  // namespace helm

extern "C" int helm_int8_linear(const void *x, int32_t x_dtype, const int8_t *w, const void *w_scale,
                                int32_t scale_dtype, const void *bias, void *y, int32_t M, int32_t N, int32_t K,
                                void *stream) {
  using namespace helm;
  if (M < 0 || N < 0 || K <= 0) return fail(HELM_ERR_INVALID_ARGUMENT, "int8_linear: bad sizes M=%d N=%d K=%d", M, N, K);
  if (K % 16) return fail(HELM_ERR_UNSUPPORTED, "int8_linear: K=%d is not a multiple of 16", K);
  if (x_dtype != HELM_F16 && x_dtype != HELM_BF16) return fail(HELM_ERR_UNSUPPORTED, "int8_linear: x dtype %d", x_dtype);
  if (scale_dtype != HELM_F16 && scale_dtype != HELM_BF16 && scale_dtype != HELM_F32)
    return fail(HELM_ERR_UNSUPPORTED, "int8_linear: scale dtype %d", scale_dtype);
  if (M == 0 || N == 0) return HELM_OK;
  if (!x || !w || !w_scale || !y) return fail(HELM_ERR_INVALID_ARGUMENT, "int8_linear: null pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15)
    return fail(HELM_ERR_INVALID_ARGUMENT, "int8_linear: x and w must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  return x_dtype == HELM_F16 ? launch<__half>(x, w, w_scale, scale_dtype, bias, y, M, N, K, st)
                             : launch<__nv_bfloat16>(x, w, w_scale, scale_dtype, bias, y, M, N, K, st);
}
