// ctx.cu -- C ABI of libferry_cuda.so: context lifecycle, host pool
// registration and the per-step entry points (ferry_cuda.h).
#include <cstdarg>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace ferry {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int cuda_status(cudaError_t e, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return e == cudaErrorMemoryAllocation ? FERRY_E_OOM : FERRY_E_CUDA;
}

namespace {

// Attention kernel choice: with one q head per kv head (G = 1) every loaded
// fp16 K/V element feeds a single multiply-add, so the CUDA-core kernel
// (attn.cu) is the faster one; with a GQA group, or fp8 KV, the tcgen05
// kernel (attn_tc.cu) runs the dense QK / PV tiles on the tensor cores.
int launch_attention_any(const ferry_ctx* c, cudaStream_t st, const uint16_t* q, const int32_t* req_ids, int n_req,
                         const int32_t* item_slot, const int32_t* n_sel, float* out) {
  if (c->cfg.kv_dtype == FERRY_KV_F16 && c->group == 1)
    return launch_attention(c, st, q, req_ids, n_req, item_slot, n_sel, out);
  return launch_attention_tc(c, st, q, req_ids, n_req, item_slot, n_sel, out);
}

// one thread polls the flag (acquire, system scope) with a short sleep
__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t value, uint32_t max_polls, uint32_t* err) {
  if (threadIdx.x != 0) return;
  for (uint32_t i = 0; i < max_polls; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v == value) return;
    __nanosleep(100);
  }
  record_error(err, kErrTimeout);
}



void free_lru_state(ferry_lru* L) {
  cudaFree(L->page_slot);
  cudaFree(L->slot_page);
  cudaFree(L->order);
  cudaFree(L->size);
  cudaFree(L->lane_cap);
  cudaFree(L->mask);
  L->page_slot = L->slot_page = L->order = L->size = L->lane_cap = nullptr;
  L->mask = nullptr;
}

int alloc_lru_state(ferry_lru* L, int64_t lanes, int cap, int ids, uint32_t* err) {
  L->lanes = (int)lanes;
  L->cap = cap;
  L->ids = ids;
  L->err = err;
  int rc;
  if ((rc = dev_alloc(&L->page_slot, (size_t)lanes * ids, 0xFF))) return rc;
  if ((rc = dev_alloc(&L->slot_page, (size_t)lanes * cap, 0xFF))) return rc;
  if ((rc = dev_alloc(&L->order, (size_t)lanes * cap, 0))) return rc;
  if ((rc = dev_alloc(&L->size, (size_t)lanes, 0))) return rc;
  return FERRY_OK;
}

void destroy_ctx(ferry_ctx* c) {
  if (!c) return;
  close_all_peers(c);
  cudaFree(c->slot_state);
  free_lru_state(&c->lru);
  cudaFree(c->cache);
  cudaFree(c->ctx_pages);
  cudaFree(c->req_base);
  cudaFree(c->summ);
  cudaFree(c->ws);
  cudaFree(c->part);
  cudaFree(c->lane_done);
  cudaFree(c->sel_keys);
  cudaFree(c->store);
  cudaFree(c->sel_done);
  cudaFree(c->quest_keys);
  cudaFree(c->quest_done);
  cudaFree(c->err);
  cudaFree(c->stats);
  for (cudaEvent_t& e : c->ev_sel)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t& e : c->ev_gat)
    if (e) cudaEventDestroy(e);
  if (c->ev_fork) cudaEventDestroy(c->ev_fork);
  if (c->ev_join) cudaEventDestroy(c->ev_join);
  if (c->side) cudaStreamDestroy(c->side);
  if (c->side2) cudaStreamDestroy(c->side2);
  if (c->side3) cudaStreamDestroy(c->side3);
  delete c;
}

int validate_cfg(const ferry_cfg* cfg) {
  if (!cfg) return set_error("cfg is NULL"), FERRY_E_INVAL;
  if (cfg->head_dim != kHeadDim) return set_error("head_dim must be 128"), FERRY_E_INVAL;
  if (cfg->page_tokens != kPageTokens) return set_error("page_tokens must be 16"), FERRY_E_INVAL;
  if (cfg->kv_dtype != FERRY_KV_F16 && cfg->kv_dtype != FERRY_KV_E4M3)
    return set_error("kv_dtype must be FERRY_KV_F16 or FERRY_KV_E4M3"), FERRY_E_INVAL;
  if (cfg->num_requests < 1 || cfg->num_layers < 1 || cfg->kv_heads < 1 || cfg->q_heads < 1)
    return set_error("num_requests, num_layers, q_heads, kv_heads must be >= 1"), FERRY_E_INVAL;
  if (cfg->q_heads % cfg->kv_heads)
    return set_error("q_heads %% kv_heads != 0"), FERRY_E_INVAL;
  const int g = cfg->q_heads / cfg->kv_heads;
  if (g != 1 && g != 2 && g != 4 && g != 8)
    return set_error("GQA group %d not in {1,2,4,8}", g), FERRY_E_INVAL;
  if (cfg->max_pages < 1 || cfg->max_pages > kMaxPages)
    return set_error("max_pages must be in [1, %d]", kMaxPages), FERRY_E_INVAL;
  if (cfg->cache_pages < 1 || cfg->top_k < 1 || cfg->top_k > cfg->cache_pages)
    return set_error("need 1 <= top_k <= cache_pages"), FERRY_E_INVAL;
  if ((size_t)lru_lane_ints(cfg->cache_pages, cfg->top_k) * 4 > kLruLaneSmemMax)
    return set_error("cache_pages %d with top_k %d need %zu bytes of shared memory per lane for miss "
                     "detection (max %zu)",
                     cfg->cache_pages, cfg->top_k, (size_t)lru_lane_ints(cfg->cache_pages, cfg->top_k) * 4,
                     kLruLaneSmemMax),
           FERRY_E_INVAL;
  return FERRY_OK;
}

}  // namespace
}  // namespace ferry

using namespace ferry;

extern "C" {

const char* ferry_last_error(void) { return g_last_error.c_str(); }
int ferry_version(void) { return 100; }

int ferry_ctx_create(int device, const ferry_cfg* cfg, ferry_ctx** out) {
  if (!out) return set_error("out is NULL"), FERRY_E_INVAL;
  *out = nullptr;
  int rc = validate_cfg(cfg);
  if (rc) return rc;
  int ndev = 0;
  FERRY_TRY(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_error("device %d out of range", device), FERRY_E_INVAL;
  DeviceGuard guard(device);
  if (!guard.ok) return FERRY_E_CUDA;
  auto* c = new ferry_ctx;
  c->device = device;
  c->cfg = *cfg;
  c->group = cfg->q_heads / cfg->kv_heads;
  c->lanes_per_req = cfg->num_layers * cfg->kv_heads;
  c->lanes = (int64_t)cfg->num_requests * c->lanes_per_req;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);

  const size_t R = cfg->num_requests, k = cfg->top_k;
  const size_t LH = c->lanes_per_req;
#define FERRY_CK(x)        \
  if ((rc = (x))) {        \
    destroy_ctx(c);        \
    return rc;             \
  }
  FERRY_CK(dev_alloc(&c->err, 1, 0));
  FERRY_CK(dev_alloc(&c->stats, FERRY_NUM_STATS, 0));
  FERRY_CK(dev_alloc(&c->slot_state, (size_t)cfg->num_requests, 0));
  c->unit_bytes = cfg->kv_dtype == FERRY_KV_E4M3 ? kUnitBytesF8 : kUnitBytes;
  FERRY_CK(dev_alloc(&c->cache, (size_t)c->lanes * cfg->cache_pages * c->unit_bytes, 0));
  // the tensor-core attention kernel reads the cache through a TMA tensor map
  if (cfg->kv_dtype == FERRY_KV_E4M3 || c->group > 1) FERRY_CK(make_cache_tensor_map(c));
  FERRY_CK(alloc_lru_state(&c->lru, c->lanes, cfg->cache_pages, cfg->max_pages, c->err));
  c->lru.device = device;
  FERRY_CK(dev_alloc(&c->ctx_pages, 2 * R, 0));
  FERRY_CK(dev_alloc(&c->req_base, R, 0));
  {
    // default home of request slot r in the host pool: units r*L*Hkv*N onwards
    std::vector<int64_t> base(R);
    for (size_t r = 0; r < R; ++r) base[r] = (int64_t)r * (int64_t)LH * cfg->max_pages;
    FERRY_TRY(cudaMemcpy(c->req_base, base.data(), R * 8, cudaMemcpyHostToDevice));
  }
  const size_t ws_ints = R * LH * (4 * k + 2);
  FERRY_CK(dev_alloc(&c->ws, ws_ints, 0));
  c->ws_sel = c->ws;
  c->ws_islot = c->ws_sel + R * LH * k;
  c->ws_mpage = c->ws_islot + R * LH * k;
  c->ws_mslot = c->ws_mpage + R * LH * k;
  c->ws_nsel = c->ws_mslot + R * LH * k;
  c->ws_nmiss = c->ws_nsel + R * LH;
  FERRY_CK(dev_alloc(&c->part, attention_partial_slots(c->lanes, c->num_sms) * c->group * kPartStride, 0));
  FERRY_CK(dev_alloc(&c->lane_done, (size_t)c->lanes, 0));
  if (select_chunks(cfg->max_pages) > 1) {
    FERRY_CK(dev_alloc(&c->sel_keys, (size_t)c->lanes * cfg->max_pages, 0));
    FERRY_CK(dev_alloc(&c->sel_done, (size_t)c->lanes, 0));
  }
#undef FERRY_CK
  FERRY_TRY(cudaDeviceSynchronize());
  *out = c;
  return FERRY_OK;
}

int ferry_ctx_destroy(ferry_ctx* c) {
  if (!c) return FERRY_OK;
  DeviceGuard guard(c->device);
  cudaDeviceSynchronize();
  destroy_ctx(c);
  return FERRY_OK;
}

int ferry_ctx_check(ferry_ctx* c) {
  if (!c) return set_error("ctx is NULL"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  FERRY_TRY(cudaDeviceSynchronize());
  uint32_t e = 0;
  FERRY_TRY(cudaMemcpy(&e, c->err, 4, cudaMemcpyDeviceToHost));
  if (!e) return FERRY_OK;
  FERRY_TRY(cudaMemset(c->err, 0, 4));
  FERRY_TRY(cudaMemset(c->lane_done, 0, (size_t)c->lanes * 4));
  if (c->sel_done) FERRY_TRY(cudaMemset(c->sel_done, 0, (size_t)c->lanes * 4));
  if (c->quest_done)
    FERRY_TRY(cudaMemset(c->quest_done, 0, (size_t)c->cfg.num_requests * c->cfg.num_layers * 4));
  if (e & kErrTimeout) return set_error("a device wait timed out"), FERRY_E_TIMEOUT;
  return set_error("a kernel saw an out-of-range index"), FERRY_E_RANGE;
}

int ferry_host_alloc(size_t bytes, void** out) {
  if (!out || bytes == 0) return set_error("bad arguments"), FERRY_E_INVAL;
  cudaError_t e = cudaHostAlloc(out, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) {
    *out = nullptr;
    return cuda_status(e, "cudaHostAlloc");
  }
  return FERRY_OK;
}

int ferry_host_free(void* p) {
  if (p) FERRY_TRY(cudaFreeHost(p));
  return FERRY_OK;
}

int ferry_kv_register(ferry_ctx* c, void* host_pool, size_t bytes) {
  if (!c || !host_pool || bytes < (size_t)c->unit_bytes || ((uintptr_t)host_pool & 15))
    return set_error("kv_register: need a 16-byte aligned pool of >= one page unit"), FERRY_E_INVAL;
  if (c->stores_only) return set_error("kv_register: the ctx runs without a host pool"), FERRY_E_STATE;
  DeviceGuard guard(c->device);
  void* dev = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(&dev, host_pool, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error("kv_register: pool is not pinned+mapped host memory (use ferry_host_alloc)"),
           FERRY_E_INVAL;
  }
  const uint64_t units = bytes / c->unit_bytes;
  float* summ = nullptr;
  int rc = dev_alloc(&summ, (size_t)units * c->summ_row, 0);
  if (rc) return rc;
  cudaFree(c->summ);
  c->summ = summ;
  c->pool_dev = (uint8_t*)dev;
  c->pool_units = units;
  return FERRY_OK;
}

int ferry_kv_register_stores(ferry_ctx* c, uint64_t units) {
  if (!c || units == 0) return set_error("kv_register_stores: bad arguments"), FERRY_E_INVAL;
  if (!c->store) return set_error("kv_register_stores: create the owner store first"), FERRY_E_STATE;
  if (c->pool_dev) return set_error("kv_register_stores: a host pool is registered"), FERRY_E_STATE;
  DeviceGuard guard(c->device);
  float* summ = nullptr;
  int rc = dev_alloc(&summ, (size_t)units * c->summ_row, 0);
  if (rc) return rc;
  cudaFree(c->summ);
  c->summ = summ;
  c->pool_units = units;
  c->stores_only = true;
  c->gather_src = FERRY_SRC_OWNER;
  return FERRY_OK;
}

static int check_batch(const ferry_ctx* c, const int32_t* req_ids, int n_req);

int ferry_page_summary_from_stores(ferry_ctx* c, void* stream, const int32_t* d_req_ids, int n) {
  int rc = check_batch(c, d_req_ids, n);
  if (rc) return rc;
  if (!c->store || !c->summ) return set_error("summary_from_stores: needs a store and summary rows"), FERRY_E_STATE;
  DeviceGuard guard(c->device);
  return launch_store_summary(c, (cudaStream_t)stream, d_req_ids, n);
}

int ferry_kv_generate(void* stream, uint64_t seed, uint64_t unit0, int64_t n_units, void* dst,
                      int kv_dtype) {
  return launch_kv_generate((cudaStream_t)stream, seed, unit0, n_units, dst, kv_dtype);
}

int ferry_page_summary_update(ferry_ctx* c, void* stream, int64_t unit0, int64_t n_units) {
  if (!c) return set_error("ctx is NULL"), FERRY_E_INVAL;
  if (!c->pool_dev) return set_error("no host pool registered"), FERRY_E_STATE;
  if (unit0 < 0 || n_units < 0 || (uint64_t)(unit0 + n_units) > c->pool_units)
    return set_error("summary range outside the pool"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  if (c->select_mode == FERRY_SELECT_QUEST)
    return launch_minmax((cudaStream_t)stream, c->pool_dev, unit0, n_units, c->summ, c->cfg.kv_dtype);
  return launch_summary((cudaStream_t)stream, c->pool_dev, unit0, n_units, c->summ, c->cfg.kv_dtype);
}

int ferry_select_mode(ferry_ctx* c, int mode) {
  if (!c) return set_error("ctx is NULL"), FERRY_E_INVAL;
  if (mode != FERRY_SELECT_MEAN && mode != FERRY_SELECT_QUEST)
    return set_error("select_mode: unknown mode %d", mode), FERRY_E_INVAL;
  if (c->pool_dev || c->stores_only)
    return set_error("select_mode: set it before ferry_kv_register"), FERRY_E_STATE;
  if (mode == FERRY_SELECT_QUEST) {
    if (select_quest_smem(c->cfg.q_heads, c->cfg.max_pages) > 200 * 1024)
      return set_error("select_mode: %d q heads and %d pages exceed the Quest kernel's shared memory",
                       c->cfg.q_heads, c->cfg.max_pages),
             FERRY_E_INVAL;
    DeviceGuard guard(c->device);
    const size_t groups = (size_t)c->cfg.num_requests * c->cfg.num_layers;
    if (!c->quest_keys) {
      int rc = dev_alloc(&c->quest_keys, groups * c->cfg.max_pages, 0);
      if (!rc) rc = dev_alloc(&c->quest_done, groups, 0);
      if (rc) {
        cudaFree(c->quest_keys);
        c->quest_keys = nullptr;
        return rc;
      }
    }
  }
  c->select_mode = mode;
  c->summ_row = mode == FERRY_SELECT_QUEST ? 2 * kHeadDim : kHeadDim;
  return FERRY_OK;
}

int ferry_requests_begin(ferry_ctx* c, void* stream, const int32_t* d_req_ids,
                         const int32_t* d_n_pages, const int64_t* d_pool_base, int n) {
  if (!c || n < 0 || n > c->cfg.num_requests || (n && (!d_req_ids || !d_n_pages)))
    return set_error("requests_begin: bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  return launch_lru_reset(&c->lru, (cudaStream_t)stream, d_req_ids, n, c->lanes_per_req, d_n_pages,
                          c->ctx_pages, d_pool_base, c->req_base);
}

static int check_batch(const ferry_ctx* c, const int32_t* req_ids, int n_req) {
  if (!c) return set_error("ctx is NULL"), FERRY_E_INVAL;
  if (n_req < 0 || n_req > c->cfg.num_requests || (n_req && !req_ids))
    return set_error("batch of %d requests (max %d)", n_req, c->cfg.num_requests), FERRY_E_INVAL;
  return FERRY_OK;
}

int ferry_select_topk(ferry_ctx* c, void* stream, const uint16_t* d_q, const int32_t* d_req_ids,
                      int n_req, int32_t* d_sel, int32_t* d_n_sel) {
  int rc = check_batch(c, d_req_ids, n_req);
  if (rc) return rc;
  if (!c->summ) return set_error("no host pool registered (summaries missing)"), FERRY_E_STATE;
  if (n_req && (!d_q || !d_sel || !d_n_sel)) return set_error("select: NULL buffer"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  return launch_select(c, (cudaStream_t)stream, d_q, d_req_ids, n_req, d_sel, d_n_sel);
}

int ferry_detect_misses(ferry_ctx* c, void* stream, const int32_t* d_req_ids, int n_req,
                        const int32_t* d_sel, const int32_t* d_n_sel, int32_t* d_item_slot,
                        int32_t* d_miss_page, int32_t* d_miss_slot, int32_t* d_n_miss,
                        uint8_t* d_is_miss) {
  int rc = check_batch(c, d_req_ids, n_req);
  if (rc) return rc;
  DeviceGuard guard(c->device);
  return launch_lru(&c->lru, (cudaStream_t)stream, nullptr, d_req_ids, c->lanes_per_req, nullptr,
                    n_req * c->lanes_per_req, d_sel, c->cfg.top_k, d_n_sel, 1, d_is_miss,
                    d_item_slot, d_miss_page, d_miss_slot, d_n_miss);
}

int ferry_gather_misses(ferry_ctx* c, void* stream, const int32_t* d_req_ids, int n_req,
                        const int32_t* d_miss_page, const int32_t* d_miss_slot,
                        const int32_t* d_n_miss) {
  int rc = check_batch(c, d_req_ids, n_req);
  if (rc) return rc;
  if (n_req && (!d_miss_page || !d_miss_slot || !d_n_miss))
    return set_error("gather: NULL buffer"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  return launch_gather(c, (cudaStream_t)stream, d_req_ids, n_req, d_miss_page, d_miss_slot,
                       d_n_miss);
}

int ferry_sparse_decode(ferry_ctx* c, void* stream, const uint16_t* d_q, const int32_t* d_req_ids,
                        int n_req, const int32_t* d_item_slot, const int32_t* d_n_sel,
                        float* d_out) {
  int rc = check_batch(c, d_req_ids, n_req);
  if (rc) return rc;
  if (n_req && (!d_q || !d_item_slot || !d_n_sel || !d_out))
    return set_error("sparse_decode: NULL buffer"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  return launch_attention_any(c, (cudaStream_t)stream, d_q, d_req_ids, n_req, d_item_slot, d_n_sel, d_out);
}

int ferry_decode_step(ferry_ctx* c, void* stream, const uint16_t* d_q, const int32_t* d_req_ids,
                      int n_req, float* d_out) {
  int rc = check_batch(c, d_req_ids, n_req);
  if (rc) return rc;
  if (!c->summ || !(c->pool_dev || c->stores_only)) return set_error("no host pool registered"), FERRY_E_STATE;
  if (n_req && (!d_q || !d_out)) return set_error("decode_step: NULL buffer"), FERRY_E_INVAL;
  if (c->append_tokens > 0 && !c->pool_dev)
    return set_error("decode_step: appends read the new pages from the host pool"), FERRY_E_STATE;
  DeviceGuard guard(c->device);
  cudaStream_t st = (cudaStream_t)stream;
  const int LH = c->lanes_per_req, k = c->cfg.top_k;
  const size_t qrow = (size_t)c->cfg.num_layers * c->cfg.q_heads * kHeadDim;  // q / out elements per request
  const int nch = std::min(c->step_chunks, n_req);
  if (nch <= 1 || !c->side) {
    if ((rc = launch_select(c, st, d_q, d_req_ids, n_req, c->ws_sel, c->ws_nsel))) return rc;
    if ((rc = launch_lru(&c->lru, st, nullptr, d_req_ids, LH, nullptr, n_req * LH, c->ws_sel, k, c->ws_nsel, 1,
                         nullptr, c->ws_islot, c->ws_mpage, c->ws_mslot, c->ws_nmiss)))
      return rc;
    if ((rc = launch_gather(c, st, d_req_ids, n_req, c->ws_mpage, c->ws_mslot, c->ws_nmiss))) return rc;
    if ((rc = launch_attention_any(c, st, d_q, d_req_ids, n_req, c->ws_islot, c->ws_nsel, d_out))) return rc;
  } else {
    // Requests [s0, s0 + n) form chunk i. Chunk i's selection and miss
    // detection (HBM- and latency-bound) run on the caller's stream while
    // chunk i-1's gather (host- or NVLink-bound) runs on `side` or `side3`
    // (alternating, so that a chunk's gather starts while the previous one
    // drains and the link has no gap) and chunk i-2's attention on `side2`.
    // Chunks own disjoint lanes and their own rows of the workspace; kernels
    // of one kind that share scratch (selection chunk keys, attention
    // partials) stay on one stream each; gathers share only atomic counters.
    const int per = (n_req + nch - 1) / nch;
    FERRY_TRY(cudaEventRecord(c->ev_fork, st));
    FERRY_TRY(cudaStreamWaitEvent(c->side, c->ev_fork, 0));
    FERRY_TRY(cudaStreamWaitEvent(c->side2, c->ev_fork, 0));
    FERRY_TRY(cudaStreamWaitEvent(c->side3, c->ev_fork, 0));
    for (int i = 0, s0 = 0; s0 < n_req; ++i, s0 += per) {
      const int n = std::min(per, n_req - s0);
      const size_t l0 = (size_t)s0 * LH;
      const int32_t* ids = d_req_ids + s0;
      if ((rc = launch_select(c, st, d_q + (size_t)s0 * qrow, ids, n, c->ws_sel + l0 * k, c->ws_nsel + l0)))
        return rc;
      if ((rc = launch_lru(&c->lru, st, nullptr, ids, LH, nullptr, n * LH, c->ws_sel + l0 * k, k, c->ws_nsel + l0,
                           1, nullptr, c->ws_islot + l0 * k, c->ws_mpage + l0 * k, c->ws_mslot + l0 * k,
                           c->ws_nmiss + l0)))
        return rc;
      cudaStream_t gs = (i & 1) ? c->side3 : c->side;
      FERRY_TRY(cudaEventRecord(c->ev_sel[i], st));
      FERRY_TRY(cudaStreamWaitEvent(gs, c->ev_sel[i], 0));
      if ((rc = launch_gather(c, gs, ids, n, c->ws_mpage + l0 * k, c->ws_mslot + l0 * k, c->ws_nmiss + l0, true)))
        return rc;
      FERRY_TRY(cudaEventRecord(c->ev_gat[i], gs));
      FERRY_TRY(cudaStreamWaitEvent(c->side2, c->ev_gat[i], 0));
      if ((rc = launch_attention_any(c, c->side2, d_q + (size_t)s0 * qrow, ids, n, c->ws_islot + l0 * k,
                                     c->ws_nsel + l0, d_out + (size_t)s0 * qrow)))
        return rc;
    }
    // side2's last attention follows every chunk's gather (each attention
    // waited for its own)
    FERRY_TRY(cudaEventRecord(c->ev_join, c->side2));
    FERRY_TRY(cudaStreamWaitEvent(st, c->ev_join, 0));
  }
  // the token decoded in this step joins its request's context
  return c->append_tokens > 0 ? launch_append(c, st, d_req_ids, n_req, c->append_tokens) : FERRY_OK;
}

int ferry_step_chunks(ferry_ctx* c, int chunks) {
  if (!c || chunks < 1 || chunks > 16) return set_error("step_chunks: 1..16 chunks"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  if (chunks > 1 && !c->side) {
    FERRY_TRY(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking));
    FERRY_TRY(cudaStreamCreateWithFlags(&c->side2, cudaStreamNonBlocking));
    FERRY_TRY(cudaStreamCreateWithFlags(&c->side3, cudaStreamNonBlocking));
    FERRY_TRY(cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming));
    FERRY_TRY(cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming));
    for (cudaEvent_t& e : c->ev_sel) FERRY_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (cudaEvent_t& e : c->ev_gat) FERRY_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  c->step_chunks = chunks;
  return FERRY_OK;
}

int ferry_requests_append(ferry_ctx* c, void* stream, const int32_t* d_req_ids, int n, int tokens) {
  int rc = check_batch(c, d_req_ids, n);
  if (rc) return rc;
  if (tokens < 0) return set_error("requests_append: negative token count"), FERRY_E_INVAL;
  if (!c->summ || !c->pool_dev) return set_error("no host pool registered"), FERRY_E_STATE;
  DeviceGuard guard(c->device);
  return launch_append(c, (cudaStream_t)stream, d_req_ids, n, tokens);
}

int ferry_decode_appends(ferry_ctx* c, int tokens_per_step) {
  if (!c || tokens_per_step < 0) return set_error("decode_appends: bad arguments"), FERRY_E_INVAL;
  c->append_tokens = tokens_per_step;
  return FERRY_OK;
}

int ferry_wait_flag(ferry_ctx* c, void* stream, const uint32_t* d_flag, uint32_t value, uint32_t max_polls) {
  if (!c || !d_flag) return set_error("wait_flag: bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  wait_flag_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(d_flag, value, max_polls, c->err);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_stats_read(ferry_ctx* c, uint64_t* stats, int reset) {
  if (!c || !stats) return set_error("bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  FERRY_TRY(cudaDeviceSynchronize());
  FERRY_TRY(cudaMemcpy(stats, c->stats, 8 * FERRY_NUM_STATS, cudaMemcpyDeviceToHost));
  if (reset) FERRY_TRY(cudaMemset(c->stats, 0, 8 * FERRY_NUM_STATS));
  return FERRY_OK;
}

int ferry_debug_read(ferry_ctx* c, int which, size_t offset, size_t bytes, void* host_dst) {
  if (!c || !host_dst) return set_error("bad arguments"), FERRY_E_INVAL;
  const uint8_t* base = nullptr;
  size_t size = 0;
  const size_t R = c->cfg.num_requests, LH = c->lanes_per_req, k = c->cfg.top_k;
  switch (which) {
    case 0: base = c->cache; size = (size_t)c->lanes * c->cfg.cache_pages * c->unit_bytes; break;
    case 1: base = (uint8_t*)c->lru.page_slot; size = (size_t)c->lanes * c->cfg.max_pages * 4; break;
    case 2: base = (uint8_t*)c->lru.order; size = (size_t)c->lanes * c->cfg.cache_pages * 4; break;
    case 3: base = (uint8_t*)c->lru.size; size = (size_t)c->lanes * 4; break;
    case 4: base = (uint8_t*)c->summ; size = (size_t)c->pool_units * c->summ_row * 4; break;
    case 5: base = (uint8_t*)c->ctx_pages; size = 2 * R * 4; break;
    case 6: base = (uint8_t*)c->ws; size = R * LH * (4 * k + 2) * 4; break;
    case 7: base = (uint8_t*)c->req_base; size = R * 8; break;
    default: return set_error("debug_read: unknown buffer %d", which), FERRY_E_INVAL;
  }
  if (!base || offset > size || bytes > size - offset)
    return set_error("debug_read: range outside buffer %d", which), FERRY_E_INVAL;
  DeviceGuard guard(c->device);
  FERRY_TRY(cudaDeviceSynchronize());
  FERRY_TRY(cudaMemcpy(host_dst, base + offset, bytes, cudaMemcpyDeviceToHost));
  return FERRY_OK;
}

int ferry_lru_create(int device, int lanes, int capacity, int ids, ferry_lru** out) {
  if (!out || lanes < 1 || capacity < 1 || ids < 1) return set_error("bad arguments"), FERRY_E_INVAL;
  *out = nullptr;
  DeviceGuard guard(device);
  if (!guard.ok) return FERRY_E_CUDA;
  auto* L = new ferry_lru;
  L->device = device;
  uint32_t* err = nullptr;
  int rc = dev_alloc(&err, 1, 0);
  if (!rc) rc = alloc_lru_state(L, lanes, capacity, ids, err);
  if (rc) {
    free_lru_state(L);
    cudaFree(err);
    delete L;
    return rc;
  }
  *out = L;
  return FERRY_OK;
}

int ferry_lru_destroy(ferry_lru* L) {
  if (!L) return FERRY_OK;
  DeviceGuard guard(L->device);
  cudaDeviceSynchronize();
  free_lru_state(L);
  cudaFree(L->err);
  delete L;
  return FERRY_OK;
}

int ferry_lru_touch(ferry_lru* L, void* stream, const int32_t* d_lane_ids, const uint8_t* d_reset,
                    int n, const int32_t* d_sel, int k, const int32_t* d_n_sel, int flags,
                    uint8_t* d_is_miss, int32_t* d_item_slot, int32_t* d_miss_page,
                    int32_t* d_miss_slot, int32_t* d_n_miss) {
  if (!L || n < 0 || (n && !d_lane_ids)) return set_error("bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(L->device);
  return launch_lru(L, (cudaStream_t)stream, d_lane_ids, nullptr, 1, d_reset, n, d_sel, k, d_n_sel,
                    (flags & FERRY_LRU_DISTINCT) ? 1 : 0, d_is_miss, d_item_slot, d_miss_page,
                    d_miss_slot, d_n_miss);
}

int ferry_lru_read(ferry_lru* L, int lane, int32_t* page_slot, int32_t* lru_slots, int32_t* size) {
  if (!L || lane < 0 || lane >= L->lanes || !page_slot || !lru_slots || !size)
    return set_error("bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(L->device);
  FERRY_TRY(cudaDeviceSynchronize());
  uint32_t e = 0;
  FERRY_TRY(cudaMemcpy(&e, L->err, 4, cudaMemcpyDeviceToHost));
  FERRY_TRY(cudaMemcpy(page_slot, L->page_slot + (size_t)lane * L->ids, (size_t)L->ids * 4,
                       cudaMemcpyDeviceToHost));
  FERRY_TRY(cudaMemcpy(lru_slots, L->order + (size_t)lane * L->cap, (size_t)L->cap * 4,
                       cudaMemcpyDeviceToHost));
  FERRY_TRY(cudaMemcpy(size, L->size + lane, 4, cudaMemcpyDeviceToHost));
  if (e) {
    cudaMemset(L->err, 0, 4);
    return set_error("a kernel saw an out-of-range index"), FERRY_E_RANGE;
  }
  return FERRY_OK;
}

}  // extern "C"
