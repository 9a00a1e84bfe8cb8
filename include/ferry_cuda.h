/*
 * ferry_cuda.h -- C ABI of the B200-native sparse KV-cache miss-stream decode
 * path (libferry_cuda.so, built for sm_100a).
 *
 * The reference (clearleo126/ferry) has no FFI layer: its hot path is
 * header-only C++ called in-process. Each entry point below names the
 * reference interface whose job it takes over (path:line inside the reference
 * project). All functions return an int status (FERRY_OK or a FERRY_E_* code)
 * and never exit the process -- unlike the reference, whose CUDA_CHECK exits
 * (src/common/cuda_check.cuh:9-17) and whose trace loader aborts
 * (src/workloads/miss_trace.cuh:64-71). ferry_last_error() gives the message.
 *
 * Units and layout
 *   page unit   one (request, layer, kv_head, page): 16 tokens x 128 dims, K
 *               then V, fp16 -> 8192 bytes. The reference's unit is a 4-token
 *               "C4" block over all kv heads (src/workloads/missstream.cuh:66);
 *               per-head pages are what per-head top-k selection needs.
 *   lane        one (request, layer, kv_head); global lane index
 *               (req * num_layers + layer) * kv_heads + head. A step over a
 *               batch of n_req requests works on n_req * num_layers * kv_heads
 *               batch lanes a = (i * num_layers + layer) * kv_heads + head.
 *   q / out     [n_req][num_layers][q_heads][128]; q fp16, out fp32.
 *   host pool   pinned, device-mapped host memory of pool_units page units;
 *               lane l, page p lives in unit (l * max_pages + p) % pool_units
 *               (modulo addressing, as the reference's host slab does:
 *               src/runtime/wla_multigpu.cuh:323-332).
 *
 * Threading: one ferry_ctx per GPU, used from one host thread at a time. All
 * per-step calls are asynchronous on the caller's stream; pointers named d_*
 * are device pointers on the ctx's device.
 */
#ifndef FERRY_CUDA_H
#define FERRY_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FERRY_OK 0
#define FERRY_E_INVAL 1   /* bad argument or configuration */
#define FERRY_E_OOM 2     /* device or pinned allocation failed */
#define FERRY_E_TIMEOUT 3 /* a bounded device wait ran out */
#define FERRY_E_CUDA 4    /* CUDA runtime error (message in ferry_last_error) */
#define FERRY_E_STATE 5   /* call out of order (e.g. no host pool registered) */
#define FERRY_E_RANGE 6   /* a kernel saw an out-of-range index and skipped it */

#define FERRY_KV_F16 0

#define FERRY_LRU_DISTINCT 1 /* selections of a lane hold no duplicates */

typedef struct ferry_cfg {
  int num_requests; /* request slots R */
  int num_layers;   /* L */
  int q_heads;      /* Hq */
  int kv_heads;     /* Hkv; q_heads % kv_heads == 0, group <= 8 */
  int head_dim;     /* must be 128 */
  int page_tokens;  /* must be 16 */
  int max_pages;    /* N: pages per lane context (<= 16384) */
  int cache_pages;  /* C: HBM cache slots per lane */
  int top_k;        /* k: selected pages per lane, k <= C */
  int kv_dtype;     /* FERRY_KV_F16 */
} ferry_cfg;

typedef struct ferry_ctx ferry_ctx;
typedef struct ferry_lru ferry_lru;

/* Last error message of the calling thread ("" when none). */
const char* ferry_last_error(void);
/* Library version (major * 100 + minor). */
int ferry_version(void);

/* ---- context ------------------------------------------------------------
 * Replaces the per-GPU state the reference builds in the WlaMultiGpuCtx
 * constructor (src/runtime/wla_multigpu.cuh:435-623: d_cache_/d_out_ per GPU,
 * LRU mirrors lru_dq_/lru_set_) and in run_miss_workload
 * (src/workloads/kv_exec.cuh:64-102). The ctx owns the HBM page cache, page
 * tables, LRU state, page summaries and scratch. */
int ferry_ctx_create(int device, const ferry_cfg* cfg, ferry_ctx** out);
int ferry_ctx_destroy(ferry_ctx* ctx);
/* Synchronises the ctx's device and reports any error a kernel recorded
 * (FERRY_E_TIMEOUT / FERRY_E_RANGE); clears the record. */
int ferry_ctx_check(ferry_ctx* ctx);

/* Pinned, device-mapped host memory (cudaHostAlloc mapped|portable); the
 * caller owns it and frees it with ferry_host_free. */
int ferry_host_alloc(size_t bytes, void** out);
int ferry_host_free(void* p);

/* Register the host KV pool (pinned + mapped; the caller keeps ownership and
 * must keep it alive). Replaces the reference's pinned host slab h_slab_
 * (src/runtime/wla_multigpu.cuh:533-544; src/workloads/kv_exec.cuh:78-86).
 * Allocates the per-unit page summaries (pool_units x 128 fp32). */
int ferry_kv_register(ferry_ctx* ctx, void* host_pool, size_t bytes);

/* Fill n_units page units starting at unit0 of dst (device or mapped host
 * memory) with the seeded procedural KV (Irwin-Hall N(0,1) -> fp16). Input
 * generator for tests and benches; no reference counterpart (the reference
 * fills its slab from mt19937, src/runtime/wla_multigpu.cuh:535-543). */
int ferry_kv_generate(void* stream, uint64_t seed, uint64_t unit0, int64_t n_units,
                      void* dst);

/* Page summaries (fp32 mean of the 16 keys, token order) of pool units
 * [unit0, unit0 + n_units), read from the registered host pool. The reference
 * computes page statistics only offline in torch
 * (tools/capture_miss_trace.py:139-147). */
int ferry_page_summary_update(ferry_ctx* ctx, void* stream, int64_t unit0, int64_t n_units);

/* Start (or restart) requests: set their context length in pages and empty
 * their lanes' cache state. d_req_ids / d_n_pages: n device ints. Replaces the
 * per-request LRU state creation of replay_miss_stream
 * (src/workloads/missstream.cuh:107-114) and kv_handoff(carry=false)
 * (src/runtime/wla_multigpu.cuh:1970-1987). */
int ferry_requests_begin(ferry_ctx* ctx, void* stream, const int32_t* d_req_ids,
                         const int32_t* d_n_pages, int n);

/* ---- the four hot-path steps --------------------------------------------- */

/* Top-k page selection: score = q . mean-key summary per kv head (max over
 * the GQA group), top-k descending with ties to the lower page id, output
 * ascending by page id. d_sel: [n_req*L*Hkv][k]; d_n_sel: [n_req*L*Hkv].
 * Replaces Selector.on_layer (tools/capture_miss_trace.py:128-159) and the
 * synthetic selector of replay_miss_stream (src/workloads/missstream.cuh:118-133). */
int ferry_select_topk(ferry_ctx* ctx, void* stream, const uint16_t* d_q,
                      const int32_t* d_req_ids, int n_req, int32_t* d_sel, int32_t* d_n_sel);

/* Miss detection against the HBM page cache: exact sequential LRU per lane in
 * selection order, page table and slot assignment updated on device.
 * Outputs per batch lane (row stride k): d_item_slot (cache slot of each
 * selected page), d_miss_page / d_miss_slot (misses in selection order),
 * d_n_miss; d_is_miss may be NULL. Replaces kv_touch
 * (src/runtime/wla_multigpu.cuh:1937-1962) and the LRU of replay_miss_stream
 * (src/workloads/missstream.cuh:137-161). */
int ferry_detect_misses(ferry_ctx* ctx, void* stream, const int32_t* d_req_ids, int n_req,
                        const int32_t* d_sel, const int32_t* d_n_sel, int32_t* d_item_slot,
                        int32_t* d_miss_page, int32_t* d_miss_slot, int32_t* d_n_miss,
                        uint8_t* d_is_miss);

/* Miss gather: copy every missed page unit from the registered host pool
 * (device-initiated 128-bit reads over the host link) into its cache slot.
 * Replaces the run-merge + HostStagedChannel::submit refill path
 * (src/runtime/wla_multigpu.cuh:2527-2604, src/comm/host_staged_channel.cpp:43-74). */
int ferry_gather_misses(ferry_ctx* ctx, void* stream, const int32_t* d_req_ids, int n_req,
                        const int32_t* d_miss_page, const int32_t* d_miss_slot,
                        const int32_t* d_n_miss);

/* Paged sparse decode attention over the selected pages (fp32 accumulation,
 * softmax scale 1/sqrt(128)). Uses ctx-owned scratch for split-K partials.
 * Replaces the stand-in wla_attn_kernel / attn_kernel
 * (src/runtime/wla_multigpu.cuh:96-103, src/workloads/kv_exec.cuh:30-37). */
int ferry_sparse_decode(ferry_ctx* ctx, void* stream, const uint16_t* d_q,
                        const int32_t* d_req_ids, int n_req, const int32_t* d_item_slot,
                        const int32_t* d_n_sel, float* d_out);

/* Allocation-free variant of ferry_sparse_decode. No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc -- a serving
 * engine that gives all of HBM to its own KV arena or caching allocator at
 * start-up, or a decode loop on the latency-critical path where cudaMalloc's
 * implicit device synchronisation would stall every stream. It needs no ctx:
 * the caller passes the page cache (d_cache, num_requests * lanes_per_req *
 * cache_pages page units, lane-major) and its geometry (group = q heads per kv
 * head) plus the same q / req_ids / item_slot / n_sel / out as
 * ferry_sparse_decode, on the current device. Scratch is a fixed 4 MiB
 * __device__ array inside the library (held by every GPU that loads it until
 * exit): at most 16384 lanes per call, and batches whose split-K partials do
 * not fit are rejected with FERRY_E_INVAL. The first call on a device looks up
 * the array's address (call it once before any stream capture). Calls share
 * the array, so calls that overlap on the GPU race; out-of-range ids are
 * skipped, not reported. */
int ferry_sparse_decode_noalloc(void* stream, const void* d_cache, int cache_pages,
                                int num_requests, int lanes_per_req, int group, int top_k,
                                const uint16_t* d_q, const int32_t* d_req_ids, int n_req,
                                const int32_t* d_item_slot, const int32_t* d_n_sel,
                                float* d_out);

/* One decode step = select -> detect -> gather -> attention on ctx-owned
 * workspace. Replaces exec_step mode C (src/runtime/wla_multigpu.cuh:2527-2604)
 * and run_miss_workload mode C (src/workloads/kv_exec.cuh:187-292). */
int ferry_decode_step(ferry_ctx* ctx, void* stream, const uint16_t* d_q,
                      const int32_t* d_req_ids, int n_req, float* d_out);

/* Read (and optionally zero) the ctx counters: stats[0] = page units gathered,
 * stats[1] = gather bytes. Synchronous. */
int ferry_stats_read(ferry_ctx* ctx, uint64_t* stats, int reset);

/* Copy ctx device state to host for checking (synchronous).
 * which: 0 cache bytes, 1 page_slot, 2 lru order, 3 lru size, 4 summaries,
 * 5 ctx pages, 6 decode-step workspace (sel | n_sel | item_slot | miss_page |
 * miss_slot | n_miss, each sized for num_requests). */
int ferry_debug_read(ferry_ctx* ctx, int which, size_t offset, size_t bytes, void* host_dst);

/* ---- standalone LRU lanes (generic miss detector) -------------------------
 * The same device kernel as ferry_detect_misses on its own state, for any lane
 * count / capacity / id domain -- e.g. the reference's per-(request, layer)
 * block stream with duplicates (src/workloads/missstream.cuh:104-170). */
int ferry_lru_create(int device, int lanes, int capacity, int ids, ferry_lru** out);
int ferry_lru_destroy(ferry_lru* lru);
/* d_lane_ids / d_reset (nullable) / d_n_sel: n entries; d_sel and outputs have
 * row stride k. flags: FERRY_LRU_DISTINCT skips duplicate tracking. */
int ferry_lru_touch(ferry_lru* lru, void* stream, const int32_t* d_lane_ids,
                    const uint8_t* d_reset, int n, const int32_t* d_sel, int k,
                    const int32_t* d_n_sel, int flags, uint8_t* d_is_miss,
                    int32_t* d_item_slot, int32_t* d_miss_page, int32_t* d_miss_slot,
                    int32_t* d_n_miss);
/* Synchronous host copy of one lane: page_slot (ids ints), LRU order as slots
 * (capacity ints, first *size valid), size. */
int ferry_lru_read(ferry_lru* lru, int lane, int32_t* page_slot, int32_t* lru_slots,
                   int32_t* size);

#ifdef __cplusplus
}
#endif
#endif /* FERRY_CUDA_H */
