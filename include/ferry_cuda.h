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
 * per-step calls are asynchronous on the caller's stream, which must be a
 * stream of the ctx's device (calls switch to that device and restore the
 * caller's); pointers named d_* are device pointers on the ctx's device.
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

#define FERRY_KV_F16 0  /* page unit 8192 B: K[16][128] f16 | V[16][128] f16 */
#define FERRY_KV_E4M3 1 /* page unit 4112 B: K e4m3 | V e4m3 | k_scale f32 | v_scale f32 | 8 pad;
                           attention runs on tcgen05 tensor cores */

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
  int kv_dtype;     /* FERRY_KV_F16 or FERRY_KV_E4M3 */
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
 * memory) with the seeded procedural KV: Irwin-Hall N(0,1) values, rounded to
 * fp16 (FERRY_KV_F16) or quantised to e4m3 with per-page scale amax/448
 * (FERRY_KV_E4M3). Runs on the calling thread's current device, on `stream`
 * (a stream of that device). Input generator for tests and benches; no
 * reference counterpart (the reference fills its slab from mt19937,
 * src/runtime/wla_multigpu.cuh:535-543). */
int ferry_kv_generate(void* stream, uint64_t seed, uint64_t unit0, int64_t n_units,
                      void* dst, int kv_dtype);

/* Page summaries (fp32 mean of the 16 keys, token order) of pool units
 * [unit0, unit0 + n_units), read from the registered host pool. The reference
 * computes page statistics only offline in torch
 * (tools/capture_miss_trace.py:139-147). */
int ferry_page_summary_update(ferry_ctx* ctx, void* stream, int64_t unit0, int64_t n_units);

/* Start (or restart) requests: set their context length in pages, their home
 * in the host pool, and empty their lanes' cache state. d_req_ids / d_n_pages:
 * n device ints; d_pool_base: n device int64 (nullable) -- the pool unit of
 * the request's (lane 0, page 0); lane l of the request, page p is unit
 * (base + l * max_pages + p) % pool_units. NULL uses req * L * Hkv * max_pages.
 * Replaces the per-request LRU state creation of replay_miss_stream
 * (src/workloads/missstream.cuh:107-114), the slab offsets wla_slab_off
 * (src/runtime/wla_multigpu.cuh:323-332) and kv_handoff(carry=false)
 * (src/runtime/wla_multigpu.cuh:1970-1987). */
int ferry_requests_begin(ferry_ctx* ctx, void* stream, const int32_t* d_req_ids,
                         const int32_t* d_n_pages, const int64_t* d_pool_base, int n);

/* Decode appends: each decode step adds tokens to its request's context (the
 * reference's history grows every step, src/workloads/missstream.cuh:119). A
 * request's context is whole pages plus the tokens of a partial last page;
 * a page becomes selectable when its 16th token arrives -- the reference's
 * selector scores whole pages only (tools/capture_miss_trace.py:131-133) --
 * and its summary (mean row, or Quest bounds) is then computed from the pool
 * unit that holds it, which the caller must have written. A context that
 * reaches max_pages stops growing. ferry_requests_append grows the listed
 * (distinct) requests by `tokens` tokens, asynchronously on `stream`;
 * ferry_decode_appends(ctx, t) makes every ferry_decode_step append t tokens
 * to each request it decodes, after its attention (0, the default: fixed
 * contexts). ferry_requests_begin starts a context at whole pages. */
int ferry_requests_append(ferry_ctx* ctx, void* stream, const int32_t* d_req_ids, int n, int tokens);
int ferry_decode_appends(ferry_ctx* ctx, int tokens_per_step);
/* Pipelined ferry_decode_step: the batch is cut into `chunks` (1..16) runs of
 * requests; chunk i's selection and miss detection run on the caller's stream
 * while chunk i-1's gather runs on one of two streams of the ctx (alternating,
 * so that consecutive gathers overlap at their ends) and chunk i-2's
 * attention on a third, and the caller's stream waits for all of it before
 * the step returns control of it (appends, if any, follow on the caller's
 * stream). Selection and attention are HBM-bound, the gather host-link- or
 * NVLink-bound, so they overlap. Selections, miss lists, page tables and
 * gathered bytes are identical to chunks = 1 (the default); the attention
 * splits each chunk's pages over the GPU's warps by the chunk's size, so its
 * outputs can differ from an unchunked step's in the last bits (both within
 * the attention tolerance of the reference math). Call it before any stream capture: it creates the ctx's streams
 * and events on first use. No counterpart in the reference. */
int ferry_step_chunks(ferry_ctx* ctx, int chunks);

/* ---- the four hot-path steps --------------------------------------------- */

/* Selection rule of the ctx (set before ferry_kv_register; FERRY_E_STATE after).
 * FERRY_SELECT_MEAN (default): per lane (request, layer, kv head), score =
 *   q . mean-key page summary, max over the GQA group -- the benchmark's rule.
 * FERRY_SELECT_QUEST: the reference's Quest method, Selector.on_layer
 *   (tools/capture_miss_trace.py:139-147, 158-159): per-page key min/max,
 *   bound = sum_d max(q_d * kmax_d, q_d * kmin_d), max over the GQA group and
 *   then over the kv heads, top-k, ascending -- ONE page set per (request,
 *   layer), written to the rows of all its kv-head lanes. Page summaries then
 *   hold [kmin[128] | kmax[128]] fp32 rows (1 KiB per pool unit).
 * Both: ties to the lower page id; a lane with n <= k pages selects all. */
#define FERRY_SELECT_MEAN 0
#define FERRY_SELECT_QUEST 1
int ferry_select_mode(ferry_ctx* ctx, int mode);

/* Top-k page selection under the ctx's selection rule (ferry_select_mode;
 * default: score = q . mean-key summary per kv head, max over the GQA group),
 * top-k descending with ties to the lower page id, output ascending by page id. d_sel: [n_req*L*Hkv][k]; d_n_sel: [n_req*L*Hkv].
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
 * ferry_sparse_decode, on the current device.
 * The cache must hold fp16 page units of 8192 bytes (FERRY_KV_F16): the call
 * has no dtype argument and reads 8192 bytes per slot, so an e4m3 cache is
 * not supported. It runs the CUDA-core kernel at every group (1, 2, 4, 8);
 * ferry_sparse_decode uses tensor cores for groups above 1 and is ~3x faster
 * at group 8.
 * Scratch is a fixed 4 MiB __device__ array inside the library (held by every
 * GPU that loads it until exit): at most 16384 lanes per call, and batches
 * whose split-K partials do not fit are rejected with FERRY_E_INVAL (large
 * batches run with fewer warps so that they fit). The first call on a device
 * looks up the array's address (call it once before any stream capture).
 * Calls share the array, so calls that overlap on the GPU race.
 * Errors the kernel sees -- a timed-out copy wait, an out-of-range request id
 * or n_sel (that lane is skipped and its rows are zero), an out-of-range slot
 * (read as slot 0 of its lane) -- are recorded in an error word inside the
 * array; ferry_sparse_decode_noalloc_status synchronises `stream`, returns
 * FERRY_E_TIMEOUT / FERRY_E_RANGE for any error recorded since its last call
 * (FERRY_OK otherwise) and clears the word. It allocates nothing either. */
int ferry_sparse_decode_noalloc(void* stream, const void* d_cache, int cache_pages,
                                int num_requests, int lanes_per_req, int group, int top_k,
                                const uint16_t* d_q, const int32_t* d_req_ids, int n_req,
                                const int32_t* d_item_slot, const int32_t* d_n_sel,
                                float* d_out);
int ferry_sparse_decode_noalloc_status(void* stream);

/* One decode step = select -> detect -> gather -> attention on ctx-owned
 * workspace. Replaces exec_step mode C (src/runtime/wla_multigpu.cuh:2527-2604)
 * and run_miss_workload mode C (src/workloads/kv_exec.cuh:187-292). */
int ferry_decode_step(ferry_ctx* ctx, void* stream, const uint16_t* d_q,
                      const int32_t* d_req_ids, int n_req, float* d_out);

/* Read (and optionally zero) the ctx counters into stats[FERRY_NUM_STATS]:
 * [0] page units gathered (any source), [1] gather bytes, [2] page units
 * migrated in, [3] migration bytes, [4] units gathered from peer GPUs' owner
 * stores, [5] their bytes, [6] units gathered from this GPU's own store,
 * [7] their bytes (host-pool units = [0] - [4] - [6]). Synchronous. */
#define FERRY_NUM_STATS 8
int ferry_stats_read(ferry_ctx* ctx, uint64_t* stats, int reset);

/* Bounded wait on `stream` until *d_flag == value -- a flag another stream,
 * a peer GPU (through a mapped pointer) or the host sets. At most max_polls
 * polls about 100 ns apart; when they run out the ctx records
 * FERRY_E_TIMEOUT (reported by ferry_ctx_check), the kernel returns and the
 * stream and the ctx stay usable. No counterpart in the reference (its waits
 * are host-side and unbounded). */
int ferry_wait_flag(ferry_ctx* ctx, void* stream, const uint32_t* d_flag, uint32_t value, uint32_t max_polls);

/* Copy ctx device state to host for checking (synchronous).
 * which: 0 cache bytes, 1 page_slot, 2 lru order, 3 lru size, 4 summaries,
 * 5 ctx pages (R full-page counts, then R partial-page token counts), 6 decode-step workspace (sel | item_slot | miss_page |
 * miss_slot | n_sel | n_miss, each sized for num_requests), 7 request pool
 * bases (int64). */
int ferry_debug_read(ferry_ctx* ctx, int which, size_t offset, size_t bytes, void* host_dst);

/* ---- multi-GPU: request migration over NVLink ------------------------------
 * Replaces steal_from's transfer (src/runtime/wla_multigpu.cuh:1353-1468:
 * gather kernel -> D2H -> H2D through the host ring -> scatter kernel) and
 * kv_handoff (:1970-1987). A peer is another GPU's ctx of the same geometry,
 * mapped into this ctx's device: ferry_ctx_link for a ctx in this process
 * (enables peer access), or ferry_ctx_export (owner) + ferry_ctx_import
 * (thief) through CUDA IPC for one process per GPU. Migration runs on the
 * thief: it pulls each request's lane state (LRU order, slot table, page
 * table, context length) and its cache pages with 128-bit peer loads --
 * FERRY_MIGRATE_DELTA copies only resident slots (the reference's kv-mode
 * delta), FERRY_MIGRATE_FULL every slot, FERRY_MIGRATE_DROP none (context
 * length and pool home only) -- then marks the victim's request slot as
 * migrated (ferry_slot_states reads those marks). */
#define FERRY_MAX_PEERS 8
#define FERRY_CTX_HANDLE_BYTES 1024
#define FERRY_MIGRATE_FULL 0
#define FERRY_MIGRATE_DELTA 1
#define FERRY_MIGRATE_DROP 2 /* no pages: the request's lanes start cold on the thief and refill by
                                misses (the reference's kv-mode drop, wla_multigpu.cuh:129, 1314) */
int ferry_ctx_export(ferry_ctx* ctx, void* handle /* FERRY_CTX_HANDLE_BYTES */);
/* ---- page-owner stores
 * Pages sharded by page id across the GPUs of a job: rank `rank` of `world`
 * keeps in HBM every page unit (lane, p) with p % world == rank, for global
 * lanes [0, global_lanes), at store index lane * ceil(N / world) + p / world.
 * A lane's global id is req_base / N + its index in the request (the
 * request's pool home; the default home of slot r is r * L * Hkv * N). The
 * store holds the bytes of the procedural pool unit the host path would read,
 * (lane * N + p) mod pool_units (ferry_kv_generate's content).
 * ferry_gather_source selects where misses come from: FERRY_SRC_HOST (the
 * registered pinned host pool) or FERRY_SRC_OWNER (the owning rank's store:
 * this GPU's, or a peer's read over NVLink once mapped by ferry_ctx_link or
 * ferry_ctx_import after the peer created its store; pages of unmapped owners
 * or of lanes outside the store come from the host pool). Stores are created
 * before ferry_ctx_export so that the handle carries them.
 * FERRY_SRC_HOST_BULK reads the same host pool as FERRY_SRC_HOST with the
 * TMA engine (one 1-D bulk copy per page unit into shared memory, then a bulk
 * store into the slot) instead of 16-byte SM loads; the bytes moved are the
 * same.
 * No counterpart in the reference (it has no page ownership). */
#define FERRY_SRC_HOST 0
#define FERRY_SRC_OWNER 1
#define FERRY_SRC_HOST_BULK 2
int ferry_store_create(ferry_ctx* ctx, int world, int rank, int64_t global_lanes);
int ferry_store_fill(ferry_ctx* ctx, void* stream, uint64_t seed, uint64_t pool_units);
int ferry_gather_source(ferry_ctx* ctx, int source);
/* A job whose every page lives in an owner store needs no host pool
 * (configs[4] at full depth: 687 GB of e4m3 KV, 86 GB per GPU at 8 GPUs, which
 * fits the stores but not a pinned host pool). ferry_kv_register_stores takes
 * the place of ferry_kv_register after ferry_store_create: it allocates the
 * summary rows of `units` pool units (the same unit addressing, req_base +
 * lane * N + p mod units) and switches the gather source to FERRY_SRC_OWNER.
 * ferry_page_summary_from_stores then computes the summaries (mean rows, or
 * Quest bounds) of every page of the listed requests (after
 * ferry_requests_begin) from the bytes in their owners' stores -- this GPU's
 * or a peer's over NVLink, so every rank's store must be filled and linked
 * first; the rows equal what ferry_page_summary_update computes from a host
 * pool with the same content. Without a pool, a page whose owner is not
 * mapped is a range error (FERRY_E_RANGE from ferry_check_errors) and is not
 * copied; FERRY_SRC_HOST, ferry_page_summary_update and appends return
 * FERRY_E_STATE. */
int ferry_kv_register_stores(ferry_ctx* ctx, uint64_t units);
int ferry_page_summary_from_stores(ferry_ctx* ctx, void* stream, const int32_t* d_req_ids, int n);
int ferry_ctx_import(ferry_ctx* ctx, int peer_slot, const void* handle);
int ferry_ctx_link(ferry_ctx* ctx, int peer_slot, ferry_ctx* peer);
int ferry_migrate_requests(ferry_ctx* ctx, void* stream, int peer_slot, const int32_t* d_src_req,
                           const int32_t* d_dst_req, int n, int mode);
/* Synchronous copy of the R request-slot states (2 = migrated away by a peer);
 * clear_migrated resets those marks to 0 after reading. */
int ferry_slot_states(ferry_ctx* ctx, int32_t* host_out, int clear_migrated);

/* ---- multi-GPU: device-visible work-stealing deque --------------------------
 * Replaces the reference's host std::deque + mutex steal path
 * (src/runtime/wla_multigpu.cuh:1063-1506) and its device ring with unbounded
 * spins (src/queue/gpu_bounded_queue.cuh:70-198). Chase-Lev deque of 64-bit
 * tasks in the owner GPU's memory: the owner pushes and pops at the bottom,
 * any GPU that maps it steals from the top with a system-scope CAS. No call
 * waits on another party: a steal gives up after a bounded number of lost
 * races and reports the tasks it got. Results land in device memory on the
 * caller's stream (d_pushed / d_count / d_size). */
typedef struct ferry_deque ferry_deque;
int ferry_deque_create(int device, uint64_t capacity, ferry_deque** out);
int ferry_deque_destroy(ferry_deque* q);
int ferry_deque_push(ferry_deque* q, void* stream, const uint64_t* d_tasks, int n, int32_t* d_pushed);
int ferry_deque_pop(ferry_deque* q, void* stream, uint64_t* d_out, int max_n, int32_t* d_count);
int ferry_deque_steal(ferry_deque* q, void* stream, uint64_t* d_out, int max_n, int32_t* d_count);
int ferry_deque_size(ferry_deque* q, void* stream, int64_t* d_size);
/* Copy up to max_n tasks at the top -- the ones the next steals would take --
 * without taking them (a snapshot: concurrent pops and steals may change
 * them). Owner or peer view. Used by the steal policy to price candidates. */
int ferry_deque_peek(ferry_deque* q, void* stream, uint64_t* d_out, int max_n, int32_t* d_count);
/* IPC export (64-byte handle) / import of an owner's deque, and a
 * same-process view from another device (enables peer access). */
int ferry_deque_export(ferry_deque* q, void* handle64);
int ferry_deque_import(int device, const void* handle64, uint64_t capacity, ferry_deque** out);
int ferry_deque_peer_view(int device, ferry_deque* owner, ferry_deque** out);
/* Exactly-once check under contention (the twin of the reference's
 * bench_queue, src/benches/bench_queue.cu:26-123): one owner block pushes and
 * pops n_tasks while `thieves` blocks steal concurrently (cooperative launch);
 * reports tasks taken and how many task ids were not taken exactly once. */
int ferry_deque_stress(int device, uint64_t capacity, int n_tasks, int thieves, int batch,
                       uint64_t* taken, int32_t* dup_or_missing);

/* ---- page-ownership exchange between ranks (one process per GPU) ----
 * Replaces the reference's host-shared ownership state: the fair share's
 * global pending count read under the context mutex
 * (src/runtime/wla_multigpu.cuh:1518-1526, refreshed at tick boundaries
 * :829-864) and the LLX rebalancer's per-GPU load (:2084-2112). Each rank
 * contributes one fixed-size int32 row; ferry_exchange_ownership all-gathers
 * the rows of every rank (NCCL, loaded at run time: without libnccl.so.2 these
 * calls return FERRY_E_STATE). The path's only collective. */
#define FERRY_COMM_ID_BYTES 128
typedef struct ferry_comm ferry_comm;
/* Rank 0 makes the id and hands it to the other ranks out of band. */
int ferry_comm_unique_id(void* id /* FERRY_COMM_ID_BYTES */);
/* Collective over the `world` ranks: blocks until all of them call it. */
int ferry_comm_create(int device, int world, int rank, const void* id, ferry_comm** out);
int ferry_comm_destroy(ferry_comm* comm);
/* Ends every collective of `comm` still in flight (e.g. when a peer rank is
 * gone and the caller's deadline for an exchange passed); the comm is then
 * unusable: exchanges return FERRY_E_STATE, destroy frees the handle. May be
 * called from another host thread while an exchange is pending. */
int ferry_comm_abort(ferry_comm* comm);
/* d_all[world][row_ints] <- every rank's d_row[row_ints]; device memory on the
 * comm's device; asynchronous on `stream`. */
int ferry_exchange_ownership(ferry_comm* comm, void* stream, const int32_t* d_row, int row_ints,
                             int32_t* d_all);

/* ---- per-GPU executor with work stealing ----------------------------------
 * The host runtime of one GPU: the counterpart of the reference's exec thread
 * and WlaMultiGpuCtx tick/steal protocol (src/runtime/wla_multigpu.cuh:829-864
 * tick_begin/tick_end, :1063-1506 steal_from, :1518-1526 fair_share,
 * :2446-2704 exec loop). Work unit: a decode task (global request, local
 * slot, step) in the GPU's own deque (capacity >= ctx num_requests). A tick
 * reclaims slots of requests peers migrated away, admits pending arrivals,
 * pops up to max_batch tasks, and -- when this GPU holds fewer than its fair
 * share ceil(pending / world) -- steals min(steal_batch, size - fair,
 * size / 2 + 1) tasks from the peer deque with the largest excess and
 * migrates those requests over NVLink; then it runs ferry_decode_step on the
 * batch (queries gathered from d_q_table, [total_requests][q_table_steps][L][Hq]
 * [128] fp16, device memory or pinned mapped host memory) and pushes the next
 * steps back. Request r's home in
 * the host pool is r * L * Hkv * max_pages (every GPU registers a pool with
 * the same content). */
typedef struct ferry_exec ferry_exec;
typedef struct ferry_exec_cfg {
  int rank;           /* this GPU's rank */
  int world;          /* number of ranks */
  int max_batch;      /* tasks decoded per tick (<= ctx num_requests) */
  int steal_batch;    /* most tasks one steal takes (the reference's steal_batch, default 4) */
  int migrate_mode;   /* FERRY_MIGRATE_DELTA, FERRY_MIGRATE_FULL or FERRY_MIGRATE_DROP */
  int steps_per_req;  /* decode steps of every request */
  int total_requests; /* global request ids are [0, total_requests) */
  int q_table_steps;  /* query-table rows per request (0 = steps_per_req); step s reads
                         row s % q_table_steps */
} ferry_exec_cfg;
typedef struct ferry_tick_stats {
  int decoded;      /* tasks decoded this tick */
  int finished;     /* requests that finished */
  int stolen;       /* tasks stolen this tick */
  int stolen_from;  /* victim rank of that steal */
  int queued;       /* tasks pushed back */
  float tick_ms;    /* device time of the tick (CUDA events) */
  float mig_ms;     /* device time of this tick's migration kernels (0 without a steal) */
  int64_t mig_bytes; /* page bytes migrated in this tick */
} ferry_tick_stats;
int ferry_exec_create(ferry_ctx* ctx, ferry_deque* own, const ferry_exec_cfg* cfg,
                      const uint16_t* d_q_table, ferry_exec** out);
int ferry_exec_destroy(ferry_exec* x);
/* Peer rank's deque (an IPC import or a peer view) and its ctx peer slot
 * (already linked or imported into this executor's ctx). */
int ferry_exec_link_peer(ferry_exec* x, int peer_rank, int ctx_peer_slot, ferry_deque* peer_deque);
/* Queue arrivals for this GPU (host arrays); admitted when slots are free. */
int ferry_exec_admit(ferry_exec* x, const int32_t* h_global_req, const int32_t* h_n_pages, int n);
/* Unfinished requests across all GPUs, from the ownership exchange. */
int ferry_exec_set_global(ferry_exec* x, int64_t global_pending);
/* Global ids of the requests this GPU holds (the ownership table row). */
int ferry_exec_owned(ferry_exec* x, int32_t* h_out, int cap, int* n);
int ferry_exec_tick(ferry_exec* x, void* stream, ferry_tick_stats* out);
/* Decision log: open (path) or close (NULL) a binary file receiving one
 * record per steal this executor makes -- the tick, the water level seen
 * (fair share, own and victim queue sizes), planned and taken tasks, the
 * migration's bytes and device time, and per stolen request its step, slots
 * and resident page units (what delta migration moves). The counterpart of the
 * reference's FERRY_WLA_SNAPSHOT decision records (src/runtime/
 * wla_multigpu.cuh:667-788) for its offline counterfactual tool
 * (src/tools/wla_counterfact.cpp); ferry_b200/decisions.py reads the log and
 * prices the alternatives. Layout in executor.cu. */
int ferry_exec_log(ferry_exec* x, const char* path);
/* The attention output of the last tick: row i ([L][Hq][128] fp32) belongs to
 * the i-th task decoded in that tick, host_req[i] (nullable) its global
 * request. Copies min(decoded, cap_rows) rows device -> host_out on `stream`
 * (asynchronous; pinned host_out); n_out = rows. The reference's exec loop
 * keeps its outputs on the device (d_out_, wla_multigpu.cuh:2455-2468). */
int ferry_exec_output(ferry_exec* x, void* stream, float* host_out, int32_t* host_req, int cap_rows,
                      int* n_out);

/* Steal policy. cost_filter = 0 is the water-level steal alone (the
 * reference's policy C, wla_multigpu.cuh:1063-1506). cost_filter = 1 adds
 * its value filter (policy E, cost_filter_ok, wla_multigpu.cuh:942-1061):
 * candidates are the victim's next tasks (ferry_deque_peek), and the thief
 * takes the longest prefix with
 *     remaining_steps * step_ms >= margin * (cost_scale * live_bytes / link + fixed_ms)
 * where live_bytes are the request's resident cache pages (delta migration),
 * step_ms an EMA of this GPU's tick time (0.9 / 0.1, from 2 ms) and link the
 * migration bandwidth in GB/s -- the measured NVLink peer copy instead of the
 * reference's PCIe constant (kMigBWRefGbs = 16.6, :146). */
typedef struct ferry_steal_policy {
  int cost_filter;
  double margin;      /* reference default 2.0 */
  double cost_scale;  /* kappa, reference default 3.0 */
  double link_gbs;    /* migration bandwidth */
  double fixed_ms;    /* per-migration fixed cost (reference kMigDeltaFixedMs 0.06) */
} ferry_steal_policy;
int ferry_exec_policy(ferry_exec* x, const ferry_steal_policy* policy);
/* Load of this GPU: remaining decode steps summed over its requests, and the
 * request count (the rebalancer's usage, rebalance_llumnix,
 * wla_multigpu.cuh:2084-2112). */
int ferry_exec_usage(ferry_exec* x, int64_t* remaining_steps, int32_t* requests);
/* A rebalance order: at the next tick steal up to k (<= steal_batch) tasks
 * from victim_rank and migrate their requests, whatever the water level and
 * without the cost filter (the reference's rebalancer path). */
int ferry_exec_rebalance(ferry_exec* x, int victim_rank, int k);
/* The filter alone (host, no GPU): value_ms / cost_ms per candidate
 * (nullable) and the length of the accepted prefix. */
int ferry_steal_filter(const ferry_steal_policy* policy, int n, const int32_t* remain_steps,
                       const int64_t* live_bytes, double step_ms, double* value_ms, double* cost_ms,
                       int* n_accept);

/* ---- real selection traces (FMT1) ----------------------------------------
 * Replaces load_miss_trace (src/workloads/miss_trace.cuh:75-185): reads the
 * FMT1 trace of the reference's capture tool (tools/capture_miss_trace.py:
 * 316-317, 368-370), checks every header field against the run, remaps raw
 * block ids to dense ids in first-seen order and writes them in event order
 * (request, step, layer, k) to blocks_out (capacity entries; NULL = count
 * only). Returns the number of distinct ids and the largest per-request
 * distinct count (the slab capacity). A mismatch or truncation returns
 * FERRY_E_INVAL with the reason -- the reference exits the process instead. */
int ferry_trace_load(const char* path, int requests, int steps, int layers, int sel_blocks,
                     int kv_heads, int head_dim, int64_t* blocks_out, int64_t capacity,
                     int64_t* unique_out, int32_t* slab_blocks_out);

/* ---- topology and link probes ----------------------------------------------
 * Replaces probe_topology / probe_host_staged_bandwidth
 * (src/topo/topo.cpp:68-215). ferry_probe_topology: device count and, for
 * cap >= n, n x n matrices (row stride cap) of P2P access and native peer
 * atomics. ferry_probe_link: GB/s of a copy kernel on dst_dev reading `bytes`
 * from pinned host memory (src_dev = -1) or from peer device src_dev over
 * NVLink -- the access patterns of the miss gather and of migration. */
int ferry_probe_topology(int* n_dev, int32_t* p2p, int32_t* atomics, int cap);
int ferry_probe_link(int src_dev, int dst_dev, size_t bytes, int iters, double* gbs);

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

/* ---- group lanes: the reference's prefix-group-shared LRU mirror ----------
 * kv_touch keyed by (GPU, prefix group, layer) with cap_mode, ownership masks
 * and steal-time handoff (src/runtime/wla_multigpu.cuh:1867-2015). A group
 * lane is a ferry_lru lane that every member of a prefix group touches, in
 * request order (one launch per member: a launch must list each lane once).
 * ferry_lru_group_enable adds a capacity per lane (starting at the lru's
 * capacity) and an owner mask per resident page (one bit per member, the
 * reference's own_bit = 1 << (request % prefix_group), :1877-1879).
 *   ferry_lru_touch_owned   ferry_lru_touch (same outputs) whose row i ORs
 *                           d_bits[i] into the mask of every page it touches;
 *                           a page it inserts owns d_bits[i] alone (the
 *                           evicted page's mask is dropped: own_drop)
 *   ferry_lru_set_capacity  new capacities (1..capacity) of the listed lanes;
 *                           a lane above its new capacity is trimmed from its
 *                           LRU front (grp_trim, :1923-1935, cap_mode 1:
 *                           capacity = hot x resident members). Survivors at
 *                           slots >= the new capacity move, in LRU order, into
 *                           the freed slots below it, ascending, so the
 *                           occupied slots stay [0, size)
 *   ferry_lru_release       clear `bit` in every mask of the lanes (own_release)
 *   ferry_lru_count_owned   d_count[i]: pages of lane i whose mask is exactly
 *                           `bit` (kv_live_owned, :1912-1921)
 *   ferry_lru_handoff       a steal's hot-set handoff from src lanes to the
 *                           consumer's dst lanes (kv_handoff, :1970-1990):
 *                           FERRY_HANDOFF_DROP empties the dst lanes (src
 *                           unused); FERRY_HANDOFF_CARRY makes each dst lane a
 *                           copy of its src lane (same capacity; a src lane
 *                           larger than the dst lane's capacity is a range
 *                           error); FERRY_HANDOFF_OWNED merges the src pages
 *                           whose mask is exactly `bit` into the dst lane in
 *                           src LRU order -- a page already resident there
 *                           gains `bit` and keeps its place, otherwise the dst
 *                           lane evicts its front while full and appends it
 *                           (kv_handoff_owned, :1991-2015). src may live on a
 *                           peer GPU (read over NVLink).
 *   ferry_lru_read_owned    synchronous host copy of a lane's masks (capacity
 *                           entries, by slot) and its capacity
 * Range errors of these kernels are recorded in the lru's error word and
 * returned by ferry_lru_read. */
#define FERRY_HANDOFF_DROP 0
#define FERRY_HANDOFF_CARRY 1
#define FERRY_HANDOFF_OWNED 2
int ferry_lru_group_enable(ferry_lru* lru);
int ferry_lru_touch_owned(ferry_lru* lru, void* stream, const int32_t* d_lane_ids,
                          const uint8_t* d_reset, int n, const int32_t* d_sel, int k,
                          const int32_t* d_n_sel, int flags, const uint32_t* d_bits,
                          uint8_t* d_is_miss, int32_t* d_item_slot, int32_t* d_miss_page,
                          int32_t* d_miss_slot, int32_t* d_n_miss);
int ferry_lru_set_capacity(ferry_lru* lru, void* stream, const int32_t* d_lane_ids,
                           const int32_t* d_caps, int n);
int ferry_lru_release(ferry_lru* lru, void* stream, const int32_t* d_lane_ids, int n, uint32_t bit);
int ferry_lru_count_owned(ferry_lru* lru, void* stream, const int32_t* d_lane_ids, int n,
                          uint32_t bit, int32_t* d_count);
int ferry_lru_handoff(ferry_lru* dst, void* stream, const ferry_lru* src, const int32_t* d_src_lanes,
                      const int32_t* d_dst_lanes, int n, int mode, uint32_t bit);
int ferry_lru_read_owned(ferry_lru* lru, int lane, uint32_t* masks, int32_t* capacity);

/* ---- Workload B: the reference's synthetic task stream and executors ------
 * Tasks arrive open-loop with a payload on a source GPU and an FMA work count;
 * an executor moves the payloads to the compute GPU and runs the task kernel
 * (src/workloads/synthetic.cuh, src/workloads/baselines.cuh,
 * src/runtime/redistribute.cuh). Not the decode path: kept so that the
 * reference's Workload B drivers (src/benches/run_synthetic.cu) drop in.
 *
 * ferry_taskb_generate   generate_tasks (synthetic.cuh:83-173): the same
 *                        mt19937_64 draws in the same order, so a seed gives
 *                        the reference's stream; `trace_ticks` supplies the
 *                        arrivals of FERRY_TASKB_TRACE (the reference reads
 *                        them from FERRY_TRACE_CSV). `out` holds spec->total.
 * ferry_taskb_create     payload pool (n * payload bytes, the reference's
 *                        content: mt19937_64 seed 9, (rng() % 1000) / 8) on
 *                        src_dev; moved payloads, outputs and works on
 *                        dst_dev (make_ctx, baselines.cuh:82-111); peer
 *                        access dst -> src when the devices differ. One
 *                        payload size (a multiple of 16 bytes), ascending
 *                        arrivals.
 * ferry_taskb_run        one executor (run_baseline_a / run_baseline_b /
 *                        run_ferry_abl, baselines.cuh:139-409) over the
 *                        stream, arrivals replayed on the host clock at
 *                        tick_ms per tick; synchronous; fills the reference's
 *                        ExecStats. C's batches follow choose_batch
 *                        (baselines.cuh:127-137) with adaptive, else the fixed
 *                        max_mb; with overlap the kernel of a batch waits on
 *                        its move's event and up to pending_ahead batches are
 *                        in flight. Transports: FERRY_TASKB_P2P, a copy kernel
 *                        on dst reading src's HBM (over NVLink, or local);
 *                        FERRY_TASKB_HOST_STAGED, the reference's pinned ring
 *                        (HostStagedChannel, host_staged_channel.cpp:43-87).
 *                        The stats' timings are host milliseconds.
 * ferry_taskb_results    synchronous copy of the first n_floats outputs
 * ferry_taskb_reset      zero the moved payloads and outputs */
#define FERRY_TASKB_STEADY 0
#define FERRY_TASKB_BURSTY 1
#define FERRY_TASKB_SKEWED 2
#define FERRY_TASKB_TRACE 3
#define FERRY_TASKB_A 0
#define FERRY_TASKB_B 1
#define FERRY_TASKB_C 2
#define FERRY_TASKB_P2P 0
#define FERRY_TASKB_HOST_STAGED 1
typedef struct {
  int arrival;          /* FERRY_TASKB_STEADY / BURSTY / SKEWED / TRACE */
  int sparsity;         /* payload 0: 4 KB, 1: 16 KB, 2: 64 KB */
  int imbalanced;       /* work 0: uniform 100..200; 1: 20 % of tasks x8 */
  int num_gpus;         /* GPUs the dest field spreads over */
  uint64_t total;       /* tasks */
  double dest_hot_frac; /* the reference's default 0.8 */
  int dest_hot_cards;   /* <= 0: max(1, num_gpus / 5) */
  int pad;
} ferry_taskb_spec;
typedef struct {
  double arrive_t; /* ticks */
  uint64_t payload; /* bytes */
  int32_t work;
  int32_t dest;
} ferry_taskb_task;
typedef struct {
  int mode;      /* FERRY_TASKB_A / B / C */
  int transport; /* FERRY_TASKB_P2P / HOST_STAGED */
  int inner_scale;
  int stride;    /* B: tasks per segment (the reference's 64) */
  double tick_ms;
  uint64_t pending_ahead; /* C: batches in flight (4) */
  int adaptive;  /* C: 1 = choose_batch, 0 = fixed max_mb */
  int overlap;   /* C: 1 = kernels wait on events, 0 = move, compute, sync */
  double min_mb, max_mb, target_batches; /* AdaptiveBatchPolicy */
} ferry_taskb_params;
typedef struct {
  double makespan_ms, p50_ms, p99_ms, throughput, backlog_max, arrival_span_ms;
  uint64_t migrated_bytes, migrations;
} ferry_taskb_stats;
typedef struct ferry_taskb ferry_taskb;
int ferry_taskb_generate(const ferry_taskb_spec* spec, uint64_t seed, const double* trace_ticks,
                         ferry_taskb_task* out);
int ferry_taskb_create(int src_dev, int dst_dev, const ferry_taskb_task* tasks, uint64_t n, ferry_taskb** out);
int ferry_taskb_run(ferry_taskb* tb, const ferry_taskb_params* params, ferry_taskb_stats* stats);
int ferry_taskb_results(ferry_taskb* tb, float* host_out, uint64_t n_floats);
int ferry_taskb_reset(ferry_taskb* tb);
int ferry_taskb_destroy(ferry_taskb* tb);

#ifdef __cplusplus
}
#endif
#endif /* FERRY_CUDA_H */
