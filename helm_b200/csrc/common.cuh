// Shared device/host helpers for the helm_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <cstdarg>
#include <utility>

#include <nvtx3/nvToolsExt.h>

#include "../../include/helm_b200.h"

namespace helm {

// ---------------------------------------------------------------------------
// Host-side error reporting (thread-local message behind helm_last_error()).
// ---------------------------------------------------------------------------
void set_error(const char *fmt, ...);
int fail(int code, const char *fmt, ...);
int check_launch(const char *what);

inline int dtype_size(int dt) {
  switch (dt) {
    case HELM_F32: return 4;
    case HELM_F16: return 2;
    case HELM_BF16: return 2;
    case HELM_I8: return 1;
    default: return 0;
  }
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms();  // SM count of the current device (cached per device)

// NVTX range around one C-ABI call (named after the entry point), recorded when the environment
// sets HELM_B200_NVTX=1 (read once): the kernel families then show as named ranges in a profiler
// timeline.  Off, it costs one branch.
bool nvtx_enabled();
struct NvtxRange {
  bool on;
  explicit NvtxRange(const char *name) : on(nvtx_enabled()) {
    if (on) nvtxRangePushA(name);
  }
  ~NvtxRange() {
    if (on) nvtxRangePop();
  }
  NvtxRange(const NvtxRange &) = delete;
  NvtxRange &operator=(const NvtxRange &) = delete;
};

// ---------------------------------------------------------------------------
// Element conversions.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};
template <> struct Elem<__half> {
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float load_f(const void *base, int dt, int64_t i) {
  switch (dt) {
    case HELM_F16: return __half2float(reinterpret_cast<const __half *>(base)[i]);
    case HELM_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(base)[i]);
    default: return reinterpret_cast<const float *>(base)[i];
  }
}

__device__ __forceinline__ void store_f(void *base, int dt, int64_t i, float v) {
  switch (dt) {
    case HELM_F16: reinterpret_cast<__half *>(base)[i] = __float2half_rn(v); break;
    case HELM_BF16: reinterpret_cast<__nv_bfloat16 *>(base)[i] = __float2bfloat16_rn(v); break;
    default: reinterpret_cast<float *>(base)[i] = v; break;
  }
}

// 2^x on the special-function unit (MUFU.EX2); ex2(-inf) == 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Weight 2^(m_part - m_total) of a partial with running max m_part, exact 0
// for an empty partial (m_part == -inf) and 1 when both maxima are -inf.
__device__ __forceinline__ float rescale_weight(float m_part, float m_total) {
  if (m_part == -INFINITY) return m_total == -INFINITY ? 1.f : 0.f;
  return fast_exp2(m_part - m_total);
}

__device__ __forceinline__ void flag_error(int32_t *flag, int bits) {
  if (flag) atomicOr(flag, bits);
}

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with launch_pdl() may start
// while the previous kernel on the stream is still running: it must call
// pdl_wait() before reading anything an earlier kernel writes (and before
// writing anything an earlier kernel may still read).  pdl_trigger() lets the
// next kernel on the stream start its own prologue early.  Both are no-ops in a
// kernel launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace helm
