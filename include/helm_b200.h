/*
 * helm_b200.h -- C ABI of the B200 decode hot path (paged decode attention,
 * split-KV log-sum-exp merge, INT8 weight-only linear, KV-slot append).
 *
 * Every entry point takes plain pointers, sizes and a cudaStream_t (passed as
 * void* so that the header needs no CUDA include), never allocates device or
 * host memory, and returns an int status (HELM_OK == 0).  On a non-zero
 * status, helm_last_error() returns a thread-local message.  Device-side
 * index checks never trap: they record a code in the optional int
 * `error_flag` (device memory) and skip the offending page or row.
 *
 * The reference (HELM, Python + one CPU C++ kernel) has no C ABI of its own;
 * each declaration names the reference interface it replaces (file:line,
 * paths inside the HELM project).
 */
#ifndef HELM_B200_H
#define HELM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HELM_ABI_VERSION 4
#define HELM_MAX_RANKS 8

/* ---- status codes ------------------------------------------------------- */
enum {
  HELM_OK = 0,
  HELM_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad stride */
  HELM_ERR_UNSUPPORTED = 2,      /* dtype / shape combination not implemented */
  HELM_ERR_WORKSPACE = 3,        /* caller's workspace smaller than required */
  HELM_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed */
};

/* ---- device-side error flag bits (written with atomicOr) ---------------- */
enum {
  HELM_DEVERR_PAGE_ID = 1,     /* page id outside [0, num_pool_pages) */
  HELM_DEVERR_PAGE_USED = 2,   /* page_used outside [0, page_size] */
  HELM_DEVERR_NUM_PAGES = 4,   /* num_pages outside [0, page_table_stride] */
  HELM_DEVERR_TIMEOUT = 8,     /* a bounded mbarrier wait gave up */
  HELM_DEVERR_APPEND_FULL = 16 /* kv append found no spare page */
};

/* ---- element types ------------------------------------------------------ */
typedef enum {
  HELM_F32 = 0,
  HELM_F16 = 1,
  HELM_BF16 = 2,
  HELM_I8 = 3
} helm_dtype;

/* Returns HELM_ABI_VERSION of the loaded library. */
int helm_abi_version(void);

/* Thread-local text of the last non-zero status returned on this thread. */
const char *helm_last_error(void);

/* ---- paged decode attention -------------------------------------------- */
/*
 * Replaces perform_streaming_attention (helm/runtime/kv_cache.py:318-442) and
 * the decode SDPA calls of _decode_batched (helm/runtime/kv_offload.py:126,160).
 *
 * Layout.  One query token per sequence: q is [B, Hq, D] contiguous.  KV
 * pages live in a pool addressed by int32 page ids.  Element (page p, kv head
 * h, token t, dim d) of K is at k_base + p*page_stride + h*head_stride + t*D +
 * d (element units; V likewise from v_base).  The reference page tensor
 * [1, Hkv, P, D] (helm/runtime/kv_allocator.py:26-28) is exactly one page of
 * this layout with head_stride = P*D.
 *
 * Sequence b attends over pages page_table[b*page_table_stride + i] for
 * i < num_pages[b], using the first page_used[...] tokens of each page.  A page
 * with 0 used tokens is skipped (kv_cache.py:350-351); a sequence with no
 * tokens yields zeros (kv_cache.py:353-354).  Query head hq reads kv head
 * hq / (Hq/Hkv) (the repeat_interleave mapping of kv_cache.py:356-363).
 *
 * Split-KV.  The page list of each (sequence, kv head) is cut into
 * num_splits contiguous ranges; each range yields one partial record per
 * query head: float rec[D+2] = { o[0..D-1], m, l }, where m is the running
 * max of the base-2 logits s*scale*log2(e), l = sum 2^(logit-m) and o the
 * unnormalised sum of 2^(logit-m) * v.  An empty range has m = -inf, l = 0,
 * o = 0.  Records are stored [split][B*Hq][D+2] in `workspace`.
 *
 * Output.  When `out` is non-null the records are merged (helm_lse_merge
 * semantics) into out [B, Hq, D] of out_dtype; when `out_record` is non-null
 * the merged but unnormalised record [B*Hq][D+2] is also written, for a later
 * cross-GPU merge.  With num_splits == 1 and only `out` requested, no
 * workspace is touched.  With neither `out` nor `out_record` (records-only
 * mode, split path only, no fused exchange) the call writes its split records
 * to the workspace and stops there; helm_lse_merge or helm_gather_merge
 * (num_partials) merges them.
 *
 * Paths.  The split path runs a grid of (splits, kv heads, sequences) CTAs
 * and then the LSE merge; the persistent path runs one launch of two CTAs per
 * SM that stream-K over every (sequence, kv head, page) unit and merge inside
 * the kernel, and is the one that carries the fused cross-GPU exchange.
 *
 * Workspace.  The single-launch (persistent) path keeps per-CTA records and
 * per-(sequence, kv head) arrival counters there.  The counters are tagged
 * with a token the library issues per call, so no call needs them zeroed: a
 * fresh workspace, or one a split-path call or a timed-out call wrote over, is
 * valid as it is.  The kernels are launched with programmatic dependent launch
 * and touch the workspace only after the previous kernel on the stream has
 * finished, so consecutive calls on one stream may share one workspace.
 */
/* Cross-GPU exchange fused into helm_paged_attn_decode (KV sequence sharding).
 * With params.exchange set, each rank's pages are its share of every sequence:
 * the CTA that completes a (sequence, kv head) pair's rank-local merge stores
 * the pair's record into every other rank's receive slot over NVLink (CUDA IPC
 * mappings) as 64-bit words (value | epoch << 32, so no fence or flag is
 * needed), waits (bounded by wait_ns, default 2 s) for the other ranks' words of that pair and
 * merges the records in rank order, so `out` / `out_record` hold the
 * attention over the whole sequence on every rank, bit-identical across ranks.
 * Buffers: per rank one receive buffer of helm_shard_exchange_bytes()
 * (zeroed once, 16-byte aligned, shared through helm_ipc_export /
 * helm_ipc_import) and local counters (zeroed once).  Every rank makes the
 * same sequence of calls with the same B, Hq, Hkv, D, each call starting
 * after the previous one on the stream has finished.  peer_flags /
 * flags_local are unused (flags_bytes is 0).  No counterpart in the reference
 * (single-process). */
typedef struct {
  int32_t rank, world;
  float *peer_recv[HELM_MAX_RANKS];      /* receive slots of rank r, as mapped here */
  uint32_t *peer_flags[HELM_MAX_RANKS];  /* unused; may be null */
  float *recv_local;                     /* == peer_recv[rank] */
  uint32_t *flags_local;                 /* unused; may be null */
  uint32_t *counters;                    /* local */
  uint64_t wait_ns;                      /* bound of each wait for peers; 0 = 2 s */
} helm_shard_exchange;

/* Sizes for rows = B*Hq records of D dims: receive slots, flags (0), local counters. */
int64_t helm_shard_exchange_bytes(int32_t world, int32_t rows, int32_t D, int64_t *recv_bytes_out,
                                  int64_t *flags_bytes_out, int64_t *counters_bytes_out);

typedef struct {
  const void *q;          /* [B, Hq, D], q_dtype */
  const void *k_base;     /* pool base of K, kv_dtype */
  const void *v_base;     /* pool base of V, kv_dtype */
  int64_t page_stride;    /* elements between consecutive page ids */
  int64_t head_stride;    /* elements between kv heads inside a page */
  int32_t num_pool_pages; /* valid page ids: [0, num_pool_pages) */
  const int32_t *page_table; /* [B, page_table_stride] page ids (device) */
  const int32_t *page_used;  /* [B, page_table_stride] used tokens (device) */
  const int32_t *num_pages;  /* [B] listed pages per sequence (device) */
  int32_t page_table_stride;
  int32_t max_pages;      /* host-side upper bound of num_pages[b] */
  int32_t B, Hq, Hkv, D, P;
  int32_t q_dtype, kv_dtype, out_dtype; /* helm_dtype */
  float scale;            /* softmax scale; reference default 1/sqrt(D) */
  int32_t num_splits;     /* >= 1: that many splits; 0: automatic (the split
                             path with about one resident wave of CTAs, or the
                             persistent kernel when `exchange` spans several
                             GPUs); -1: the persistent single-launch kernel
                             (bf16/fp16, P=64, D=128 calls; others as 0) */
  float *workspace;       /* split records, may be null if not needed */
  int64_t workspace_bytes;
  void *out;              /* [B, Hq, D] out_dtype, or null */
  float *out_record;      /* [B*Hq, D+2] merged record, or null */
  int32_t *error_flag;    /* device int, optional */
  const helm_shard_exchange *exchange; /* null, or the fused cross-GPU exchange */
} helm_paged_attn_params;

/* Bytes of workspace helm_paged_attn_decode needs for these params, after
 * resolving num_splits == 0.  Writes the split count it will use to
 * *num_splits_out when non-null: >= 1 for the split path, -1 for the
 * persistent kernel (pass it back as num_splits to keep that plan). */
int64_t helm_paged_attn_workspace_bytes(const helm_paged_attn_params *p,
                                        int32_t *num_splits_out);

int helm_paged_attn_decode(const helm_paged_attn_params *p, void *stream);

/* ---- paged decode attention without any allocation --------------------- */
/*
 * No counterpart in the reference: an extra entry point for callers that
 * cannot allocate device memory themselves -- for example a plugin whose host
 * application owns the whole device-memory budget, or a foreign-language
 * caller that has no CUDA allocator to obtain a workspace from.
 *
 * Same contract as helm_paged_attn_decode, except that p->workspace and
 * p->workspace_bytes are ignored: the split-KV records go to a static device
 * array of HELM_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds
 * until the process exits.  Nothing is allocated or freed.  With
 * num_splits == 0 the split count is capped to what the array holds; an
 * explicit num_splits whose records (num_splits * B*Hq*(D+2)*4 bytes) exceed
 * it is rejected with HELM_ERR_WORKSPACE.
 *
 * The first call on a device looks up the array's device address (with that
 * device current) and so should come before any stream capture.  All calls in
 * the process share the one array per device and it keeps the previous
 * call's records: calls whose executions overlap on the GPU (different
 * streams, or several host threads) race on it and must be serialised by the
 * caller.  The caller still owns q, the pool, the page tables and the output.
 */
#define HELM_NOALLOC_SCRATCH_BYTES (8u << 20)

int helm_paged_attn_decode_noalloc(const helm_paged_attn_params *p, void *stream);

/* ---- log-sum-exp merge of partial records -------------------------------- */
/*
 * No single reference counterpart: it performs, across page ranges (and
 * across GPUs after an all-gather), the rescale-and-add of the online softmax
 * at helm/runtime/kv_cache.py:402-410,431-441 and the final
 * o / clamp(l, 1e-12) of kv_cache.py:441.
 *
 * partials: num_partials blocks of `rows` records of D+2 floats, block i at
 * partials + i*partial_stride (floats).  out [rows, D] of out_dtype (null to
 * skip); out_record [rows, D+2] receives the merged record (null to skip).
 */
int helm_lse_merge(const float *partials, int32_t num_partials,
                   int64_t partial_stride, int32_t rows, int32_t D,
                   void *out, int32_t out_dtype, float *out_record,
                   void *stream);

/* ---- INT8 weight-only linear -------------------------------------------- */
/*
 * Replaces helm_fp16_linear (helm/kernels/fp16_gemv.cpp:105-157) and
 * fp16_linear (helm/kernels/__init__.py:55-88) on the GPU, with INT8 weights:
 *   y[m, n] = (sum_k x[m, k] * w[n, k]) * w_scale[n] + bias[n]
 * x [M, K] (F16 or BF16), w [N, K] int8 row-major, w_scale [N] (F16, BF16 or
 * F32), bias [N] (same dtype as x) or null, y [M, N] of x_dtype.  fp32
 * accumulation.  Any M >= 1; K must be a multiple of 16; x and w 16-byte
 * aligned.  The weight streams through a TMA + mbarrier ring; the call encodes
 * (and caches) a tensor map over w on its first use.  The kernel is launched
 * with programmatic dependent launch: it starts reading w while the previous
 * kernel on the stream may still be running (x is read only after that kernel
 * has finished), so w must not be written by the kernel launched immediately
 * before this call on the same stream -- weights written on the device need an
 * event or any other launch in between.
 */
int helm_int8_linear(const void *x, int32_t x_dtype, const int8_t *w,
                     const void *w_scale, int32_t scale_dtype,
                     const void *bias, void *y, int32_t M, int32_t N,
                     int32_t K, void *stream);

/* Gated INT8 linear (SwiGLU MLP front half) in one launch:
 *   y[m, j] = silu(g[m, j]) * u[m, j],  g = x . Wg^T * sg + bg,  u = x . Wu^T * su + bu
 * for j < I.  w [2I, K] int8 holds the gate and up rows interleaved in tiles of
 * 16 rows: rows 32t..32t+15 are gate rows 16t..16t+15 and rows 32t+16..32t+31
 * the up rows 16t..16t+15; w_scale [2I] and bias [2I] (or null) follow the same
 * order.  y [M, I] of x_dtype; I a multiple of 16; otherwise the contract of
 * helm_int8_linear (fp32 accumulation, silu in fp32, one rounding to x_dtype).
 * No counterpart in the reference's kernels: it fuses the decoder MLP's
 * gate_proj, up_proj and act_fn(gate) * up (transformers' Qwen3MLP / LlamaMLP
 * forward, run around the patched attention). */
int helm_int8_linear_glu(const void *x, int32_t x_dtype, const int8_t *w,
                         const void *w_scale, int32_t scale_dtype,
                         const void *bias, void *y, int32_t M, int32_t I,
                         int32_t K, void *stream);

/* Packed INT8 weights.  helm_int8_pack_weight rewrites w [N, K] int8 row-major
 * (K a multiple of 16, both pointers 16-byte aligned) into `packed`, of
 * helm_int8_packed_bytes(N, K) bytes (-1 for bad sizes): blocks of 16 rows x
 * 128 k, block (t, kb) at byte (t * ceil(K/128) + kb) * 2048, each block in
 * the 128-byte-swizzled order the kernel reads (row r at r*128, 16-byte chunk
 * c at (c ^ (r & 7)) * 16), zero past N and K.  One row tile's k range is then
 * contiguous in memory, so the kernel streams it with one bulk copy per stage
 * instead of one 2-D box per 128 k.  helm_int8_linear_packed and
 * helm_int8_linear_glu_packed are helm_int8_linear / helm_int8_linear_glu on
 * such weights (same results bit for bit; the GLU row interleaving is applied
 * before packing).  No counterpart in the reference (a storage layout of the
 * INT8 weights that replace its fp16 ones). */
int64_t helm_int8_packed_bytes(int32_t N, int32_t K);
int helm_int8_pack_weight(const int8_t *w, int32_t N, int32_t K, int8_t *packed,
                          void *stream);
int helm_int8_linear_packed(const void *x, int32_t x_dtype, const int8_t *packed,
                            const void *w_scale, int32_t scale_dtype,
                            const void *bias, void *y, int32_t M, int32_t N,
                            int32_t K, void *stream);
int helm_int8_linear_glu_packed(const void *x, int32_t x_dtype,
                                const int8_t *packed, const void *w_scale,
                                int32_t scale_dtype, const void *bias, void *y,
                                int32_t M, int32_t I, int32_t K, void *stream);

/* Prefill-sized INT8 weight-only GEMM on the tcgen05 tensor cores: the result
 * of helm_int8_linear_packed for any M (meant for M > 64, where the GEMV's
 * one-pass design stops paying), computed as a dense contraction: 128 x 128
 * output tiles, the packed int8 weight converted exactly to x's 16-bit type
 * in shared memory, x and the converted weight read by tcgen05.mma from
 * shared memory, fp32 accumulators in tensor memory, scale and bias applied
 * in the epilogue.  Same arguments and alignment rules as
 * helm_int8_linear_packed.  Replaces the dequantise-then-dense-GEMM prefill
 * path of the INT8 linear (no counterpart in the reference, whose linear is
 * the fp16 GEMV helm/kernels/fp16_gemv.cpp:105-157). */
int helm_int8_gemm_packed(const void *x, int32_t x_dtype, const int8_t *packed,
                          const void *w_scale, int32_t scale_dtype,
                          const void *bias, void *y, int32_t M, int32_t N,
                          int32_t K, void *stream);

/* HELM_DEVERR_* bits raised by the INT8 kernels since the last reset (a bounded
 * wait of the weight pipeline that gave up: HELM_DEVERR_TIMEOUT; the rows of
 * that CTA are then left unwritten).  Synchronises with the device; reset != 0
 * clears the word.  No counterpart in the reference. */
int helm_int8_linear_error(int32_t *flag_out, int32_t reset);

/* ---- KV append ------------------------------------------------------------ */
/*
 * Replaces the slot writes of KVCacheManager.append_decode
 * (helm/runtime/kv_cache.py:103-110): writes one new token per sequence,
 * k_new/v_new [B, Hkv, D] (src_dtype, converted to kv_dtype), into the pool.
 *
 * Host-directed mode (dest or dest_host non-null): int32 [B, 3] rows
 * {page id, index of that page in the sequence's page list, token slot}, in
 * device memory (dest) or in host memory (dest_host, copied into the kernel
 * parameters at launch, so the caller may reuse it as soon as the call
 * returns).  The kernel writes the token and, when page_table is non-null,
 * also sets page_table[b][idx] = page id, page_used[b][idx] = slot+1 and
 * num_pages[b] = max(num_pages[b], idx+1).
 *
 * Device-directed mode (both null): the kernel reads the tail page of each
 * sequence from page_table/page_used/num_pages; when the tail is full it takes
 * the next id from spare_pages[b*spare_stride + spare_next[b]++] (bounded by
 * spare_stride, else HELM_DEVERR_APPEND_FULL), so a whole decode loop can run
 * without a host round trip (and be captured in a CUDA graph).
 */
typedef struct {
  const void *k_new;  /* [B, Hkv, D] */
  const void *v_new;  /* [B, Hkv, D] */
  int32_t src_dtype;
  void *k_base;
  void *v_base;
  int64_t page_stride;
  int64_t head_stride;
  int32_t num_pool_pages;
  int32_t kv_dtype;
  int32_t B, Hkv, D, P;
  const int32_t *dest;   /* [B, 3] device array, or null */
  const int32_t *dest_host; /* [B, 3] host array, or null */
  int32_t *page_table;   /* [B, page_table_stride] */
  int32_t *page_used;
  int32_t *num_pages;
  int32_t page_table_stride;
  const int32_t *spare_pages; /* [B, spare_stride] (device-directed mode) */
  int32_t *spare_next;        /* [B] */
  int32_t spare_stride;
  int32_t *error_flag;
} helm_kv_append_params;

int helm_kv_append(const helm_kv_append_params *p, void *stream);

/* ---- Prefill page writes ---------------------------------------------------- */
/*
 * Replaces the per-page chunk copies of KVCacheManager.append_prefill
 * (helm/runtime/kv_cache.py:55-85): writes `count` page-sized chunks of a
 * prompt's K/V into the pool in one launch.  k_src / v_src hold one sequence's
 * K and V, element (kv head h, token t, dim d) at h*src_head_stride +
 * t*src_tok_stride + d (src_dtype, converted to kv_dtype).  pages is a HOST
 * array int32 [count][3] of {pool slot, first source token, tokens} (tokens <=
 * P); chunk i lands in tokens 0.. of its slot.  With page_table non-null (one
 * sequence's device row: page_table / page_used of page_table_stride entries
 * and its num_pages word), entry first_index + i is set to {slot, tokens} and
 * num_pages is raised to first_index + count.  Ids are checked on the host.
 */
typedef struct {
  const void *k_src, *v_src;
  int32_t src_dtype;
  int64_t src_head_stride, src_tok_stride;
  void *k_base, *v_base;
  int64_t page_stride, head_stride;
  int32_t num_pool_pages;
  int32_t kv_dtype;
  int32_t Hkv, D, P;
  const int32_t *pages;   /* host [count][3] */
  int32_t count;
  int32_t *page_table, *page_used, *num_pages;  /* optional device table row */
  int32_t page_table_stride, first_index;
  int32_t *error_flag;
} helm_kv_prefill_params;

int helm_kv_write_pages(const helm_kv_prefill_params *p, void *stream);

/* ---- Decode prologue (fused) ---------------------------------------------- */
/*
 * The attention forward's decode prologue in one launch (kv_offload.py:244-249
 * + append_decode, kv_cache.py:87-113): per-head RMSNorm of q and k with the
 * q_norm / k_norm weights (Qwen3; null weights = none), the rotary embedding
 * x*cos + rotate_half(x)*sin of q and k (null cos/sin = none), q written to
 * q_out [B, Hq, D] (contiguous, append.src_dtype), and -- with do_append -- k
 * and v written into the pool exactly as helm_kv_append places them (host- or
 * device-directed).  q_in / append.k_new / append.v_new are the raw
 * projections [B, H, D] with row strides q_stride / k_stride / v_stride
 * elements; cos / sin [B, D] with row stride cs_stride.  fp32 arithmetic.
 */
typedef struct {
  helm_kv_append_params append;
  const void *q_in;
  void *q_out;
  int32_t Hq;
  int64_t q_stride, k_stride, v_stride;
  const void *q_norm_w, *k_norm_w;
  int32_t norm_dtype;
  float eps;
  const void *cos, *sin;
  int32_t cs_dtype;
  int64_t cs_stride;
  int32_t do_append;
} helm_decode_prologue_params;

int helm_decode_prologue(const helm_decode_prologue_params *p, void *stream);

/* ---- RMSNorm (fused) ------------------------------------------------------ */
/*
 * y[r] = w * cast(x[r] * rsqrt(mean(x[r]^2) + eps)) for rows r < rows of dim
 * elements (row strides in elements), x / y of x_dtype (F32/F16/BF16), w of
 * w_dtype: the decoders' RMSNorm modules (Qwen3RMSNorm etc., used around the
 * patched attention) in one launch.  No counterpart in the reference's kernels.
 */
int helm_rmsnorm(const void *x, int32_t x_dtype, int64_t x_stride, const void *w, int32_t w_dtype,
                 void *y, int64_t y_stride, int64_t rows, int32_t dim, float eps, void *stream);

/* ---- KV sequence sharding: cross-GPU record exchange + merge ------------- */
/*
 * No reference counterpart (HELM has no multi-GPU path): with each sequence's
 * pages split across `world` GPUs, every rank computes a merged record
 * [rows][D+2] (helm_paged_attn_decode's out_record) over its pages; this call
 * exchanges the records over NVLink and merges them (helm_lse_merge semantics,
 * fixed rank order) into out [rows, D] on every rank.
 *
 * Each rank owns one exchange buffer of helm_gather_merge_state_bytes():
 * recv_bytes of receive slots followed by flags_bytes of flags, zeroed once
 * before the first call and shared with the other ranks through CUDA IPC
 * (helm_ipc_export / helm_ipc_import).  peer_recv[r] / peer_flags[r] are rank
 * r's buffer parts as mapped in this process (this rank's own entries are its
 * local pointers).  `counters` (counters_bytes, zeroed once) stays local.
 * Every rank must make the same sequence of calls with the same rows and D.
 * Waits for peers are bounded (wait_ns, default 2 s); a wait that gives up
 * sets HELM_DEVERR_TIMEOUT in error_flag and leaves zeros in the affected rows.
 */
typedef struct {
  int32_t rank, world, rows, D;
  const float *record;                  /* [rows][D+2], this rank's */
  float *peer_recv[HELM_MAX_RANKS];
  uint32_t *peer_flags[HELM_MAX_RANKS];
  float *recv_local;
  uint32_t *flags_local;
  uint32_t *counters;
  void *out;                            /* [rows, D] or null */
  int32_t out_dtype;
  float *out_record;                    /* [rows, D+2] or null */
  int32_t *error_flag;
  uint64_t wait_ns;                     /* bound of each wait for peers; 0 = 2 s */
  int32_t num_partials;                 /* 0 or 1: `record` is the merged record; > 1:
                                           `record` holds num_partials split records
                                           (helm_paged_attn_decode's workspace in records-
                                           only mode), partial_stride floats apart, merged
                                           here before the exchange (D <= 256) */
  int64_t partial_stride;
} helm_gather_merge_params;

int64_t helm_gather_merge_state_bytes(int32_t world, int32_t rows, int32_t D, int64_t *recv_bytes_out,
                                      int64_t *flags_bytes_out, int64_t *counters_bytes_out);

int helm_gather_merge(const helm_gather_merge_params *p, void *stream);

/* CUDA IPC: export the allocation containing a device pointer (64-byte handle
 * + the pointer's offset in it); import a peer's handle (returns the pointer
 * and the mapping base to close). */
int helm_ipc_export(const void *ptr, void *handle_out, int64_t *offset_out);
int helm_ipc_import(const void *handle, int64_t offset, void **ptr_out, void **base_out);
int helm_ipc_close(void *base);

/* ---- page gather (host pages -> HBM staging) ------------------------------ */
/*
 * Replaces the per-page H2D prefetch of perform_streaming_attention
 * (helm/runtime/kv_cache.py:412-423): copies `count` pages of page_bytes
 * bytes each from src_base + src_ids[i]*page_bytes (pinned host or device
 * memory) to dst_base + (dst_first + i)*page_bytes on `stream`.  When the ids
 * form many runs, the source is pinned host memory the device can address and
 * the destination is device memory, one gather kernel copies every page
 * (16-byte loads over the host link); otherwise runs of consecutive ids are
 * copied with one cudaMemcpyAsync each.  src_ids is a HOST array.  Returns the
 * number of launches / copies issued in *copies_out.
 */
int helm_copy_pages(void *dst_base, int64_t dst_first, const void *src_base,
                    const int32_t *src_ids, int32_t count, int64_t page_bytes,
                    int32_t *copies_out, void *stream);

/* ---- batched page migration (eviction copies) ----------------------------- */
/*
 * Replaces the per-page synchronous copies of KVAllocator.move_page
 * (helm/runtime/kv_allocator.py:104-116) for a whole batch of evictions:
 * copies `count` pages of page_bytes bytes, src_base + src_ids[i]*page_bytes ->
 * dst_base + dst_ids[i]*page_bytes, on `stream`.  src_ids / dst_ids are HOST
 * arrays; every id must lie in [0, src_pages) / [0, dst_pages) (the slabs'
 * page capacities), else HELM_ERR_INVALID_ARGUMENT and nothing is copied.
 * When the pairs form many runs and both slabs are device-addressable (device
 * memory, or pinned host memory mapped for the device), one kernel moves every
 * page (16-byte loads and stores); otherwise runs consecutive in both lists
 * are copied with one cudaMemcpyAsync each.  *copies_out receives the number
 * of launches / copies issued.
 */
int helm_move_pages(void *dst_base, const int32_t *dst_ids, const void *src_base,
                    const int32_t *src_ids, int32_t count, int64_t page_bytes,
                    int64_t dst_pages, int64_t src_pages, int32_t *copies_out,
                    void *stream);

#ifdef __cplusplus
}
#endif

#endif /* HELM_B200_H */
