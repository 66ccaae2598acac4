// Fused RMSNorm over the last dimension: y = w * cast(x * rsqrt(mean(x^2) + eps)), one CTA per
// row.  The cast to x's dtype before the weight multiply follows the HF RMSNorm modules the
// decoders use (Qwen3RMSNorm / Qwen2RMSNorm / LlamaRMSNorm: fp32 statistics, normalised value
// cast back to the input dtype, then scaled by the weight), which an eager decode step runs as
// five separate kernels.
#include "common.cuh"

namespace helm {
namespace {

constexpr int kNormThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const T *__restrict__ x, int64_t x_stride,
                                                               const void *__restrict__ w, int w_dt,
                                                               T *__restrict__ y, int64_t y_stride, int dim,
                                                               float eps) {
  __shared__ float red[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const T *xr = x + row * x_stride;
  T *yr = y + row * y_stride;
  float ss = 0.f;
  for (int i = threadIdx.x; i < dim; i += kNormThreads) {
    const float v = Elem<T>::to_f(xr[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += kNormThreads) {
    const float n = Elem<T>::to_f(Elem<T>::from_f(Elem<T>::to_f(xr[i]) * r));
    yr[i] = Elem<T>::from_f(load_f(w, w_dt, i) * n);
  }
}

}  // namespace
}  // namespace helm

extern "C" int helm_rmsnorm(const void *x, int32_t x_dtype, int64_t x_stride, const void *w, int32_t w_dtype,
                            void *y, int64_t y_stride, int64_t rows, int32_t dim, float eps, void *stream) {
  helm::NvtxRange nvtx_range_("helm_rmsnorm");
  using namespace helm;
  if (rows < 0 || dim <= 0) return fail(HELM_ERR_INVALID_ARGUMENT, "rmsnorm: bad sizes rows=%lld dim=%d",
                                        (long long)rows, dim);
  if (rows == 0) return HELM_OK;
  if (!x || !w || !y) return fail(HELM_ERR_INVALID_ARGUMENT, "rmsnorm: null pointer");
  if (x_stride < dim || y_stride < dim) return fail(HELM_ERR_INVALID_ARGUMENT, "rmsnorm: row stride < dim");
  if (rows > 0x7fffffffll) return fail(HELM_ERR_UNSUPPORTED, "rmsnorm: too many rows");
  if (w_dtype != HELM_F32 && w_dtype != HELM_F16 && w_dtype != HELM_BF16)
    return fail(HELM_ERR_UNSUPPORTED, "rmsnorm: weight dtype %d", w_dtype);
  cudaStream_t st = as_stream(stream);
  const dim3 grid((unsigned)rows);
  switch (x_dtype) {
    case HELM_BF16:
      rmsnorm_kernel<__nv_bfloat16><<<grid, kNormThreads, 0, st>>>(
          static_cast<const __nv_bfloat16 *>(x), x_stride, w, w_dtype, static_cast<__nv_bfloat16 *>(y), y_stride,
          dim, eps);
      break;
    case HELM_F16:
      rmsnorm_kernel<__half><<<grid, kNormThreads, 0, st>>>(static_cast<const __half *>(x), x_stride, w, w_dtype,
                                                             static_cast<__half *>(y), y_stride, dim, eps);
      break;
    case HELM_F32:
      rmsnorm_kernel<float><<<grid, kNormThreads, 0, st>>>(static_cast<const float *>(x), x_stride, w, w_dtype,
                                                            static_cast<float *>(y), y_stride, dim, eps);
      break;
    default:
      return fail(HELM_ERR_UNSUPPORTED, "rmsnorm: dtype %d", x_dtype);
  }
  return check_launch("rmsnorm_kernel");
}
