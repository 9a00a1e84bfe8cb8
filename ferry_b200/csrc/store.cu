// store.cu -- page-owner stores: the pages of a job sharded across its GPUs
// by page id (page p of every lane lives on rank p % world), so that a miss
// can be served from the owner's HBM over NVLink instead of the host link.
// The reference has no page ownership; its misses always come from host
// memory through HostStagedChannel (src/comm/host_staged_channel.cpp:43-74).
#include "common.cuh"

using namespace ferry;

namespace ferry {
void refresh_store_map(ferry_ctx* c) {
  for (auto& p : c->store_of) p = nullptr;
  if (c->own_world <= 0) return;
  if (c->own_rank >= 0 && c->own_rank <= FERRY_MAX_PEERS) c->store_of[c->own_rank] = c->store;
  for (const ferry_peer& p : c->peers)
    if (p.store && p.own_world == c->own_world && p.store_lanes == c->store_lanes && p.own_rank >= 0 &&
        p.own_rank < c->own_world && p.own_rank != c->own_rank)
      c->store_of[p.own_rank] = p.store;
}
}  // namespace ferry

namespace {
struct Guard {
  int prev = -1;
  explicit Guard(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~Guard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

extern "C" {

int ferry_store_create(ferry_ctx* c, int world, int rank, int64_t global_lanes) {
  if (!c || world < 1 || world > FERRY_MAX_PEERS + 1 || rank < 0 || rank >= world || global_lanes <= 0)
    return set_error("store_create: bad arguments"), FERRY_E_INVAL;
  if (c->store) return set_error("store_create: the ctx already has a store"), FERRY_E_STATE;
  const int N = c->cfg.max_pages;
  const int own_np = (N + world - 1) / world;
  const size_t bytes = (size_t)global_lanes * own_np * c->unit_bytes;
  Guard g(c->device);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return set_error("store_create: %zu bytes do not fit", bytes), FERRY_E_OOM;
  }
  FERRY_TRY(e);
  c->store = (uint8_t*)p;
  c->own_world = world;
  c->own_rank = rank;
  c->own_np = own_np;
  c->store_lanes = global_lanes;
  refresh_store_map(c);
  return FERRY_OK;
}

int ferry_store_fill(ferry_ctx* c, void* stream, uint64_t seed, uint64_t pool_units) {
  if (!c || !c->store || pool_units == 0) return set_error("store_fill: no store or bad arguments"), FERRY_E_INVAL;
  Guard g(c->device);
  return launch_store_fill((cudaStream_t)stream, seed, c->own_world, c->own_rank, c->cfg.max_pages, c->own_np,
                           c->store_lanes * c->own_np, pool_units, c->store, c->cfg.kv_dtype);
}

int ferry_gather_source(ferry_ctx* c, int source) {
  if (!c || (source != FERRY_SRC_HOST && source != FERRY_SRC_OWNER && source != FERRY_SRC_HOST_BULK))
    return set_error("gather_source: bad arguments"), FERRY_E_INVAL;
  if (source == FERRY_SRC_OWNER && !c->store)
    return set_error("gather_source: owner gathers need ferry_store_create first"), FERRY_E_STATE;
  if (source != FERRY_SRC_OWNER && c->stores_only)
    return set_error("gather_source: no host pool (ferry_kv_register_stores)"), FERRY_E_STATE;
  c->gather_src = source;
  return FERRY_OK;
}

}  // extern "C"
