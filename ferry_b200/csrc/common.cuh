// common.cuh -- shared definitions of libferry_cuda.so (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "ferry_cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libferry_cuda is built for sm_100a (B200) only"
#endif

namespace ferry {

constexpr int kHeadDim = 128;
constexpr int kPageTokens = 16;
constexpr int kUnitElems = 2 * kPageTokens * kHeadDim;  // K[16][128] then V[16][128]
constexpr int kUnitBytes = kUnitElems * 2;              // fp16: 8192 bytes
// e4m3 unit: K[16][128] | V[16][128] (1 byte each) | k_scale f32 | v_scale f32 | 8 pad
constexpr int kUnitBytesF8 = kUnitElems + 16;           // 4112 bytes
constexpr int kMaxGroup = 8;
constexpr int kMaxPages = 16384;
// Shared memory of one LRU lane (one warp of the miss-detect kernel): old
// order, slot table, touch marks (cap ints each), five k-int work lists and k
// flag bytes. A lane must fit one block's 227 KiB.
constexpr size_t kLruLaneSmemMax = 227 * 1024;
inline int lru_lane_ints(int cap, int k) { return ((3 * cap + 5 * k) + (k + 3) / 4 + 3) & ~3; }
// selection scores a lane in chunks of about this many pages (one CTA each)
// once the lane is longer than two chunks
constexpr int kSelChunk = 1024;
__host__ __device__ constexpr int select_chunks(int max_pages) {
  return max_pages <= 2 * kSelChunk ? 1 : (max_pages + kSelChunk - 1) / kSelChunk;
}
// pages per chunk: a multiple of 8 (the scoring batch)
__host__ __device__ constexpr int select_chunk_pages(int max_pages, int nchunks) {
  return (((max_pages + nchunks - 1) / nchunks) + 7) & ~7;
}

// Device-side error record bits (ctx->d_err); read by ferry_ctx_check.
enum : uint32_t { kErrTimeout = 1u, kErrRange = 2u };

// Every spin on an mbarrier or flag gives up after this many polls, records
// kErrTimeout and lets the kernel return.
constexpr uint32_t kSpinLimit = 1u << 22;

// ---------------------------------------------------------------- host errors
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);

#define FERRY_TRY(call)                                        \
  do {                                                         \
    cudaError_t e__ = (call);                                  \
    if (e__ != cudaSuccess) return ferry::cuda_status(e__, #call); \
  } while (0)

// Switch to a device for the duration of a call and restore the caller's.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    ok = cudaSetDevice(dev) == cudaSuccess;
    if (!ok) set_error("cudaSetDevice(%d) failed", dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// count elements of T on the current device, every byte set to fill_byte
template <typename T>
int dev_alloc(T** p, size_t count, int fill_byte) {
  *p = nullptr;
  if (count == 0) return FERRY_OK;
  cudaError_t e = cudaMalloc((void**)p, count * sizeof(T));
  if (e != cudaSuccess) {
    *p = nullptr;
    return cuda_status(e, "cudaMalloc");
  }
  FERRY_TRY(cudaMemset(*p, fill_byte, count * sizeof(T)));
  return FERRY_OK;
}

// ---------------------------------------------------------------- device helpers
__device__ __forceinline__ void record_error(uint32_t* err, uint32_t bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// subsequent async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase: true when the phase completed, false
// (after recording kErrTimeout) when the poll budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  record_error(err, kErrTimeout);
  return false;
}

// Bounded wait on an mbarrier phase in which each probe may suspend the warp
// in hardware for up to hint_ns (woken early when the phase completes), so
// that waiting warps leave their issue slots to the working ones. The probe
// count is capped so the whole wait stays near a second.
template <uint32_t kHintNs>
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t* err) {
  constexpr uint32_t kProbes = (uint32_t)(1000000000ull / kHintNs);
  for (uint32_t i = 0; i < kProbes; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kHintNs)
        : "memory");
    if (ok) return true;
  }
  record_error(err, kErrTimeout);
  return false;
}

// 1-D bulk async copy global -> shared (TMA engine), completion signalled on
// the mbarrier as transaction bytes. dst, src 16-byte aligned; bytes % 16 == 0.
// Split-K / chunk completion count: one atomic add with acquire-release
// semantics at GPU scope. Issued by one thread after a barrier over the
// threads that stored the partials (the barrier orders their stores at CTA
// scope, the release publishes them at GPU scope), its acquire orders the
// other blocks' partials before the last block's loads of them.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// splitmix64 finaliser (Steele, Lea, Flood 2014).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace ferry

// ---------------------------------------------------------------- ctx
struct ferry_lru {
  int device = -1;
  int lanes = 0, cap = 0, ids = 0;
  int32_t* page_slot = nullptr;  // lanes * ids, -1 = absent
  int32_t* slot_page = nullptr;  // lanes * cap
  int32_t* order = nullptr;      // lanes * cap, LRU order as slots (front first)
  int32_t* size = nullptr;       // lanes
  uint32_t* err = nullptr;       // device error record
  // group lanes (group.cu): per-lane capacity and per-slot owner bits, null
  // until ferry_lru_group_enable
  int32_t* lane_cap = nullptr;   // lanes
  uint32_t* mask = nullptr;      // lanes * cap
};

// Another GPU's ctx buffers as this ctx's device sees them (peer mapping or
// CUDA IPC mapping); see peer.cu.
struct ferry_peer {
  bool ipc = false;
  int device = -1;
  uint8_t* cache = nullptr;
  int32_t* page_slot = nullptr;
  int32_t* slot_page = nullptr;
  int32_t* order = nullptr;
  int32_t* size = nullptr;
  int32_t* ctx_pages = nullptr;
  int32_t* slot_state = nullptr;
  int64_t* req_base = nullptr;
  // the peer's page-owner store (null when it has none)
  uint8_t* store = nullptr;
  int own_world = 0, own_rank = -1;
  int64_t store_lanes = 0;
};

struct ferry_ctx {
  int device = -1;
  ferry_cfg cfg{};
  int group = 1;          // q heads per kv head
  int unit_bytes = ferry::kUnitBytes;  // 8192 (fp16) or 4112 (e4m3 + scales)
  int lanes_per_req = 0;  // L * Hkv
  int64_t lanes = 0;      // R * L * Hkv

  uint8_t* cache = nullptr;  // lanes * C units
  alignas(64) unsigned char cache_map[128] = {};  // TMA tensor map of the e4m3 cache
  ferry_lru lru;             // page tables + LRU order, lanes x (C, N)
  int32_t* ctx_pages = nullptr;  // 2R: full pages of each request's context, then the tokens of
                                 // its partial last page (0..15; decode appends)
  int append_tokens = 0;         // tokens ferry_decode_step appends per request (0 = fixed context)
  // pipelined step (ferry_step_chunks): request chunks whose selection and
  // miss detection run on the caller's stream, gathers alternately on `side`
  // and `side3`, attention on `side2`
  int step_chunks = 1;
  cudaStream_t side = nullptr, side2 = nullptr, side3 = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  cudaEvent_t ev_sel[16] = {};  // chunk i's misses are known
  cudaEvent_t ev_gat[16] = {};  // chunk i's pages are in their slots
  int64_t* req_base = nullptr;   // R: pool unit of the request's (lane 0, page 0)

  // host pool
  bool stores_only = false;       // summaries without a host pool; misses from owner stores only
  uint8_t* pool_dev = nullptr;  // device-visible address of the pinned pool
  uint64_t pool_units = 0;
  float* summ = nullptr;  // pool_units * summ_row: mean rows (128) or Quest [kmin | kmax] rows (256)
  int summ_row = ferry::kHeadDim;
  int select_mode = FERRY_SELECT_MEAN;
  uint32_t* quest_keys = nullptr;  // R * L * max_pages order keys (Quest mode)
  uint32_t* quest_done = nullptr;  // R * L chunk counters (Quest mode)

  // decode-step workspace (sized for R requests)
  int32_t* ws = nullptr;
  int32_t *ws_sel = nullptr, *ws_nsel = nullptr, *ws_islot = nullptr, *ws_mpage = nullptr,
          *ws_mslot = nullptr, *ws_nmiss = nullptr;

  // selection chunk scratch (select_chunks(max_pages) > 1 only)
  uint32_t* sel_keys = nullptr;  // lanes * max_pages order keys
  uint32_t* sel_done = nullptr;  // lanes chunk counters

  // attention scratch
  float* part = nullptr;          // attention_partial_slots * group * kPartStride
  uint32_t* lane_done = nullptr;  // lanes
  uint32_t* grid_done = nullptr;  // 1

  uint32_t* err = nullptr;                // device error record
  unsigned long long* stats = nullptr;    // FERRY_NUM_STATS counters (ferry_stats_read)
  int32_t* slot_state = nullptr;          // R: 2 = request migrated away by a peer
  ferry_peer peers[FERRY_MAX_PEERS];
  int num_sms = 148;

  // page-owner store (store.cu): pages with page id % own_world == own_rank
  int own_world = 0, own_rank = -1, own_np = 0;  // own_np = ceil(N / own_world)
  int64_t store_lanes = 0;                        // global lanes covered
  uint8_t* store = nullptr;
  uint8_t* store_of[FERRY_MAX_PEERS + 1] = {};    // by owner rank (this GPU's own included)
  int gather_src = FERRY_SRC_HOST;
};

namespace ferry {
constexpr int kPartStride = 132;  // o[128], m, l, pad -> 16-byte rows

// Owner stores by rank (FERRY_SRC_OWNER) as a kernel argument; world == 0
// means host only.
struct OwnerMap {
  const uint8_t* store[FERRY_MAX_PEERS + 1];
  int world, self, own_np;
  int64_t store_lanes;
};

// kernels' launchers (one per .cu)
int launch_kv_generate(cudaStream_t st, uint64_t seed, uint64_t unit0, int64_t n_units, void* dst,
                       int kv_dtype);
int launch_summary(cudaStream_t st, const uint8_t* pool, int64_t unit0, int64_t n_units,
                   float* summ, int kv_dtype);
int launch_select(const ferry_ctx* c, cudaStream_t st, const uint16_t* q, const int32_t* req_ids,
                  int n_req, int32_t* sel, int32_t* n_sel);
// decode appends: grow each listed request's context by `tokens` tokens and
// compute the summary of every page that becomes full (kvgen.cu)
int launch_append(const ferry_ctx* c, cudaStream_t st, const int32_t* req_ids, int n, int tokens);
// summaries (mean rows or Quest bounds) of every page of the listed
// requests, read from the owner stores (kvgen.cu)
int launch_store_summary(const ferry_ctx* c, cudaStream_t st, const int32_t* req_ids, int n);
// Quest page bounds [kmin | kmax] of pool units (kvgen.cu)
int launch_minmax(cudaStream_t st, const uint8_t* pool, int64_t unit0, int64_t n_units, float* mm,
                  int kv_dtype);
// dynamic shared memory of the Quest selection kernel (select.cu)
size_t select_quest_smem(int q_heads, int max_pages);
int launch_lru(const ferry_lru* L, cudaStream_t st, const int32_t* lane_ids, const int32_t* req_ids,
               int lanes_per_req, const uint8_t* reset, int n, const int32_t* sel, int k,
               const int32_t* n_sel, int distinct, uint8_t* is_miss, int32_t* item_slot,
               int32_t* miss_page, int32_t* miss_slot, int32_t* n_miss, const uint32_t* bits = nullptr);
int launch_lru_reset(const ferry_lru* L, cudaStream_t st, const int32_t* req_ids, int n,
                     int lanes_per_req, const int32_t* n_pages, int32_t* ctx_pages,
                     const int64_t* pool_base, int64_t* req_base);
// shared: the gather runs beside other kernels (a pipelined step), so its
// grid leaves most of every SM to them
int launch_gather(const ferry_ctx* c, cudaStream_t st, const int32_t* req_ids, int n_req,
                  const int32_t* miss_page, const int32_t* miss_slot, const int32_t* n_miss,
                  bool shared = false);
void close_all_peers(ferry_ctx* c);
// owner store of rank `rank` of `world` (kvgen.cu)
int launch_store_fill(cudaStream_t st, uint64_t seed, int world, int rank, int N, int own_np, int64_t n_units,
                      uint64_t pool_units, uint8_t* dst, int kv_dtype);
// recompute store_of[] from the own store and the mapped peers (store.cu)
void refresh_store_map(ferry_ctx* c);
// partial slots the attention kernel needs for `lanes` lanes on `sms` SMs
size_t attention_partial_slots(int64_t lanes, int sms);
int launch_attention(const ferry_ctx* c, cudaStream_t st, const uint16_t* q,
                     const int32_t* req_ids, int n_req, const int32_t* item_slot,
                     const int32_t* n_sel, float* out);
// e4m3 KV path on tcgen05 tensor cores (attn_tc.cu)
int make_cache_tensor_map(ferry_ctx* c);
int launch_attention_tc(const ferry_ctx* c, cudaStream_t st, const uint16_t* q,
                        const int32_t* req_ids, int n_req, const int32_t* item_slot,
                        const int32_t* n_sel, float* out);

// 16-byte-vector copy of one page unit by one warp (unit_bytes % 16 == 0,
// <= 8192): all of a lane's loads are issued before its stores.
__device__ __forceinline__ void warp_copy_unit(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                               int unit_bytes, int t) {
  const int n16 = unit_bytes >> 4;
  uint4 r[kUnitBytes / (32 * 16)];
#pragma unroll
  for (int j = 0; j < kUnitBytes / (32 * 16); ++j) {
    const int v = t + 32 * j;
    if (v < n16) r[j] = ld_nc_v4(src + (size_t)v * 16);
  }
#pragma unroll
  for (int j = 0; j < kUnitBytes / (32 * 16); ++j) {
    const int v = t + 32 * j;
    if (v < n16) st_v4(dst + (size_t)v * 16, r[j]);
  }
}
}  // namespace ferry
