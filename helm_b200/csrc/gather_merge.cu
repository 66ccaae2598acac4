// Cross-GPU exchange of attention records + log-sum-exp merge (KV sequence sharding).
// The input is this rank's merged record per row, or the split records of the attention's split
// path, which each CTA then merges for its rows before the exchange (one launch in place of
// helm_lse_merge + the exchange).
//
// Every rank holds a contiguous range of each sequence's pages and produces a
// merged record [rows][D+2] = (o, m, l) per (sequence, query head).  This
// kernel replaces an NCCL all-gather followed by a merge kernel: each CTA owns
// a block of rows; it stores its rows directly into every rank's receive
// buffer over NVLink (CUDA IPC mappings, plain P2P stores), publishes them
// with a release increment of a per-(source rank, row block) counter in the
// destination's flag array, waits (bounded) until every source rank's
// counter for its block has advanced, and merges the G records of each of its
// rows in fixed rank order, so every rank computes the identical output.
//
// All bookkeeping is device-resident and monotonic: sent[block] counts this
// rank's calls, seen[src][block] the calls consumed from src, and the receive
// slot of a call is its count's parity.  A slot is rewritten two calls later,
// which cannot happen before its reader has consumed it (the writer's next
// call needs the reader's record of the intervening call).  No host epochs
// and no resets, so the launch can be replayed from a CUDA graph.
#include "common.cuh"

#include <cstring>

namespace helm {
namespace {

constexpr int kRowsPerBlock = 8;
constexpr int kThreads = 256;                // one warp per row of a block
constexpr int kMaxD = 256;                   // head dim limit when merging split records here
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait

struct GatherArgs {
  int rank, world, rows, D, nblocks;
  const float *record;
  float *recv[HELM_MAX_RANKS];        // receive buffer of each rank (this process's mapping)
  uint32_t *flags[HELM_MAX_RANKS];    // flag array of each rank
  float *recv_local;
  uint32_t *flags_local;
  uint32_t *sent;
  uint32_t *seen;
  void *out;
  int out_dtype;
  float *out_record;
  int32_t *error_flag;
  uint64_t wait_ns;
  int S;                              // > 1: `record` holds S split records, pstride floats apart
  int64_t pstride;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_relaxed_sys_add(uint32_t *p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__global__ void __launch_bounds__(kThreads) gather_merge_kernel(GatherArgs a) {
  __shared__ uint32_t s_sent;
  __shared__ uint32_t s_slot[HELM_MAX_RANKS];
  __shared__ int s_ok;
  const int rb = blockIdx.x;
  const int row0 = rb * kRowsPerBlock;
  const int nrows = min(kRowsPerBlock, a.rows - row0);
  const int rl = a.D + 2;
  const int G = a.world;
  // Launched with programmatic dependent launch: the CTAs may be resident before the attention
  // that writes `record` has finished; everything below runs after it has.
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    s_sent = a.sent[rb];
    s_ok = 1;
  }
  __syncthreads();
  // 0) with split records: merge this block's rows first (warp w merges row row0 + w over the S
  //    splits in split order, lane l the dims l, l + 32, ...) into shared memory
  __shared__ __align__(16) float rec_s[kRowsPerBlock * (kMaxD + 2)];
  const float *src = a.record + (int64_t)row0 * rl;
  if (a.S > 1) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < nrows) {
      const float *base = a.record + (int64_t)(row0 + warp) * rl;
      float M = -INFINITY;
      for (int sp = lane; sp < a.S; sp += 32) M = fmaxf(M, base[sp * a.pstride + a.D]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.f, O[kMaxD / 32];
#pragma unroll
      for (int k = 0; k < kMaxD / 32; ++k) O[k] = 0.f;
#pragma unroll 4
      for (int sp = 0; sp < a.S; ++sp) {
        const float *pp = base + sp * a.pstride;
        const float w = rescale_weight(pp[a.D], M);
        L = fmaf(pp[a.D + 1], w, L);
#pragma unroll
        for (int k = 0; k < kMaxD / 32; ++k) {
          const int d = lane + 32 * k;
          if (d < a.D) O[k] = fmaf(pp[d], w, O[k]);
        }
      }
      float *r = rec_s + warp * rl;
#pragma unroll
      for (int k = 0; k < kMaxD / 32; ++k) {
        const int d = lane + 32 * k;
        if (d < a.D) r[d] = M == -INFINITY ? 0.f : O[k];
      }
      if (lane == 0) {
        r[a.D] = M;
        r[a.D + 1] = M == -INFINITY ? 0.f : L;
      }
    }
    __syncthreads();
    src = rec_s;
  }
  // 1) push this rank's rows into every rank's receive slot (sent parity, source = this rank);
  //    16-byte stores when the block is 16-byte aligned (rows*(D+2) floats per block)
  const int n = nrows * rl;
  const uint32_t slot = s_sent & 1u;
  const bool vec = ((n & 3) == 0) && ((((int64_t)row0 * rl) & 3) == 0) && ((((int64_t)a.rows * rl) & 3) == 0);
  for (int dst = 0; dst < G; ++dst) {
    float *d = a.recv[dst] + (((int64_t)slot * G + a.rank) * a.rows + row0) * rl;
    if (vec) {
      const float4 *s4 = reinterpret_cast<const float4 *>(src);
      float4 *d4 = reinterpret_cast<float4 *>(d);
      for (int i = threadIdx.x; i < n / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
      for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = src[i];
    }
  }
  __syncthreads();
  // Publish: after the barrier, one thread per destination fences at system scope (making the
  // whole block's stores visible) and bumps that destination's counter.
  if (threadIdx.x < G) {
    __threadfence_system();
    red_relaxed_sys_add(a.flags[threadIdx.x] + a.rank * a.nblocks + rb, 1u);
  }
  if (threadIdx.x == 0) a.sent[rb] = s_sent + 1;
  // 2) wait until every source's counter for this block covers the call we consume next
  if (threadIdx.x < G) {
    const int s = threadIdx.x;
    const uint32_t want = a.seen[s * a.nblocks + rb] + 1;
    const uint32_t *f = a.flags_local + s * a.nblocks + rb;
    bool ok = ld_acquire_sys(f) >= want;
    if (!ok) {
      const uint64_t t0 = now_ns();
      while (true) {
        if (ld_acquire_sys(f) >= want) {
          ok = true;
          break;
        }
        if (now_ns() - t0 > a.wait_ns) break;
      }
    }
    if (!ok) {
      flag_error(a.error_flag, HELM_DEVERR_TIMEOUT);
      atomicExch(&s_ok, 0);
    }
    s_slot[s] = (want - 1) & 1u;
  }
  __syncthreads();
  __threadfence();
  // 3) merge the G records of each row in rank order
  for (int idx = threadIdx.x; idx < nrows * a.D; idx += blockDim.x) {
    const int r = idx / a.D, dd = idx - r * a.D;
    const int row = row0 + r;
    float M = -INFINITY;
    for (int s = 0; s < G; ++s) {
      const float *rec = a.recv_local + (((int64_t)s_slot[s] * G + s) * a.rows + row) * rl;
      M = fmaxf(M, __ldcg(rec + a.D));
    }
    float L = 0.f, O = 0.f;
    for (int s = 0; s < G; ++s) {
      const float *rec = a.recv_local + (((int64_t)s_slot[s] * G + s) * a.rows + row) * rl;
      const float w = rescale_weight(__ldcg(rec + a.D), M);
      L = fmaf(__ldcg(rec + a.D + 1), w, L);
      O = fmaf(__ldcg(rec + dd), w, O);
    }
    if (M == -INFINITY) { L = 0.f; O = 0.f; }
    if (!s_ok) O = 0.f;
    if (a.out) store_f(a.out, a.out_dtype, (int64_t)row * a.D + dd, L > 0.f ? O / L : 0.f);
    if (a.out_record) {
      float *rr = a.out_record + (int64_t)row * rl;
      rr[dd] = O;
      if (dd == 0) { rr[a.D] = M; rr[a.D + 1] = L; }
    }
  }
  __syncthreads();
  // 4) mark the consumed call
  if (threadIdx.x < G) a.seen[threadIdx.x * a.nblocks + rb] += 1;
}

}  // namespace
}  // namespace helm

extern "C" int64_t helm_gather_merge_state_bytes(int32_t world, int32_t rows, int32_t D, int64_t *recv_bytes_out,
                                                  int64_t *flags_bytes_out, int64_t *counters_bytes_out) {
  using namespace helm;
  if (world < 1 || world > HELM_MAX_RANKS || rows < 0 || D <= 0) {
    fail(HELM_ERR_INVALID_ARGUMENT, "gather_merge: bad sizes world=%d rows=%d D=%d", world, rows, D);
    return -1;
  }
  const int64_t nblocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  const int64_t recv = 2ll * world * rows * (D + 2) * (int64_t)sizeof(float);
  const int64_t flags = (int64_t)world * nblocks * (int64_t)sizeof(uint32_t);
  const int64_t counters = (1 + (int64_t)world) * nblocks * (int64_t)sizeof(uint32_t);
  if (recv_bytes_out) *recv_bytes_out = recv;
  if (flags_bytes_out) *flags_bytes_out = flags;
  if (counters_bytes_out) *counters_bytes_out = counters;
  return recv + flags + counters;
}

extern "C" int helm_gather_merge(const helm_gather_merge_params *p, void *stream) {
  helm::NvtxRange nvtx_range_("helm_gather_merge");
  using namespace helm;
  if (!p) return fail(HELM_ERR_INVALID_ARGUMENT, "gather_merge: params is null");
  if (p->world < 1 || p->world > HELM_MAX_RANKS || p->rank < 0 || p->rank >= p->world || p->rows < 0 || p->D <= 0)
    return fail(HELM_ERR_INVALID_ARGUMENT, "gather_merge: bad rank/world/sizes");
  if (p->rows == 0) return HELM_OK;
  if (!p->record || !p->recv_local || !p->flags_local || !p->counters || (!p->out && !p->out_record))
    return fail(HELM_ERR_INVALID_ARGUMENT, "gather_merge: null pointer");
  for (int r = 0; r < p->world; ++r)
    if (!p->peer_recv[r] || !p->peer_flags[r]) return fail(HELM_ERR_INVALID_ARGUMENT, "gather_merge: null peer");
  if (p->out && p->out_dtype != HELM_F32 && p->out_dtype != HELM_F16 && p->out_dtype != HELM_BF16)
    return fail(HELM_ERR_UNSUPPORTED, "gather_merge: dtype %d", p->out_dtype);
  if (p->num_partials < 0) return fail(HELM_ERR_INVALID_ARGUMENT, "gather_merge: num_partials %d", p->num_partials);
  if (p->num_partials > 1) {
    if (p->D > kMaxD) return fail(HELM_ERR_UNSUPPORTED, "gather_merge: split records need D <= %d", kMaxD);
    if (p->partial_stride < (int64_t)p->rows * (p->D + 2))
      return fail(HELM_ERR_INVALID_ARGUMENT, "gather_merge: partial_stride %lld < rows*(D+2)",
                  (long long)p->partial_stride);
  }
  GatherArgs a{};
  a.rank = p->rank;
  a.world = p->world;
  a.rows = p->rows;
  a.D = p->D;
  a.nblocks = (p->rows + kRowsPerBlock - 1) / kRowsPerBlock;
  a.record = p->record;
  for (int r = 0; r < p->world; ++r) {
    a.recv[r] = p->peer_recv[r];
    a.flags[r] = p->peer_flags[r];
  }
  a.recv_local = p->recv_local;
  a.flags_local = p->flags_local;
  a.sent = p->counters;
  a.seen = p->counters + a.nblocks;
  a.out = p->out;
  a.out_dtype = p->out_dtype;
  a.out_record = p->out_record;
  a.error_flag = p->error_flag;
  a.wait_ns = p->wait_ns ? p->wait_ns : kWaitNs;
  a.S = p->num_partials;
  a.pstride = p->partial_stride;
  const cudaError_t e = launch_pdl(gather_merge_kernel, dim3(a.nblocks), dim3(kThreads), 0, as_stream(stream), a);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "gather_merge: launch: %s", cudaGetErrorString(e));
  return check_launch("gather_merge_kernel");
}

// ---- CUDA IPC helpers --------------------------------------------------------------------

extern "C" int helm_ipc_export(const void *ptr, void *handle_out, int64_t *offset_out) {
  helm::NvtxRange nvtx_range_("helm_ipc_export");
  using namespace helm;
  if (!ptr || !handle_out || !offset_out) return fail(HELM_ERR_INVALID_ARGUMENT, "ipc_export: null pointer");
  // The handle names the whole allocation that contains ptr; report ptr's offset in it.
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess || attr.type != cudaMemoryTypeDevice)
    return fail(HELM_ERR_INVALID_ARGUMENT, "ipc_export: not a device pointer");
  void *base = nullptr;
  size_t size = 0;
  // cuMemGetAddressRange through the runtime's driver entry point (no libcuda link needed).
  using GetRange = int (*)(unsigned long long *, size_t *, unsigned long long);
  static GetRange get_range = nullptr;
  if (!get_range) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(HELM_ERR_CUDA, "ipc_export: cuMemGetAddressRange unavailable");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  unsigned long long b = 0;
  if (get_range(&b, &size, reinterpret_cast<unsigned long long>(ptr)) != 0)
    return fail(HELM_ERR_CUDA, "ipc_export: cuMemGetAddressRange failed");
  base = reinterpret_cast<void *>(b);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "ipc_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<const char *>(ptr) - static_cast<const char *>(base);
  return HELM_OK;
}

extern "C" int helm_ipc_import(const void *handle, int64_t offset, void **ptr_out, void **base_out) {
  helm::NvtxRange nvtx_range_("helm_ipc_import");
  using namespace helm;
  if (!handle || !ptr_out || !base_out) return fail(HELM_ERR_INVALID_ARGUMENT, "ipc_import: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "ipc_import: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *base_out = base;
  *ptr_out = static_cast<char *>(base) + offset;
  return HELM_OK;
}

extern "C" int helm_ipc_close(void *base) {
  helm::NvtxRange nvtx_range_("helm_ipc_close");
  using namespace helm;
  if (!base) return HELM_OK;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return fail(HELM_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(e));
  return HELM_OK;
}
