// peer.cu -- request migration between GPUs: the thief pulls a stolen
// request's whole device state from the victim's memory over NVLink.
//
// Replaces the reference's migration path (steal_from's delta/full transfer,
// src/runtime/wla_multigpu.cuh:1353-1468: victim-side gather kernel -> D2H ->
// H2D through the pinned ring -> consumer-side scatter kernel, with index
// tables uploaded from the host). Here one stream on the thief GPU runs:
//   1. migrate_meta_kernel  warp per lane: empty the destination lane, copy
//      size, LRU order and slot table, rebuild the page table entries of the
//      resident pages, copy the request's context length;
//   2. migrate_pages_kernel warp per 8 KiB page unit, 16 outstanding 16-byte
//      peer loads per lane: the resident slots [0, size) of every lane
//      (delta, the reference's kv-mode delta) or all slots (full); none for
//      drop (the reference's kv-mode drop, wla_multigpu.cuh:1314: the
//      request's lanes start cold on the thief and refill by misses);
//   3. release_kernel       marks the victim's request slot as migrated
//      (system-scope release store) so the victim's host can reuse it.
// The victim's memory is reached through a direct peer mapping (same process,
// cudaDeviceEnablePeerAccess) or a CUDA IPC mapping (one process per GPU).
// Only plain loads read peer memory -- no TMA, no multicast.
#include <cstring>

#include "common.cuh"

namespace ferry {

constexpr int kPeerBufs = 8;  // cache, page_slot, slot_page, order, size, ctx_pages, slot_state, req_base

struct PeerHandle {  // what ferry_ctx_export writes (FERRY_CTX_HANDLE_BYTES)
  uint32_t magic;
  int32_t device;
  ferry_cfg cfg;
  cudaIpcMemHandle_t mem[kPeerBufs];
  // page-owner store (has_store == 0: none)
  int32_t has_store, own_world, own_rank, pad;
  int64_t store_lanes;
  cudaIpcMemHandle_t store_mem;
};
static_assert(sizeof(PeerHandle) <= FERRY_CTX_HANDLE_BYTES, "handle too large");
constexpr uint32_t kPeerMagic = 0x46455259u;  // "FERY"

namespace {

__device__ __forceinline__ void st_release_sys_i32(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct MigArgs {
  // peer (source)
  const uint8_t* p_cache;
  const int32_t* p_slot_page;
  const int32_t* p_order;
  const int32_t* p_size;
  const int32_t* p_ctx_pages;
  const int64_t* p_req_base;
  int32_t* p_slot_state;
  // local (destination)
  uint8_t* cache;
  int32_t* page_slot;
  int32_t* slot_page;
  int32_t* order;
  int32_t* size;
  int32_t* ctx_pages;
  int64_t* req_base;
  const int32_t* src_req;
  const int32_t* dst_req;
  int n;
  int lanes_per_req;
  int R;
  int C;
  int N;
  int full;
  int drop;  // FERRY_MIGRATE_DROP: state only, the destination lanes start cold
  int unit_bytes;
  unsigned long long* stats;
  uint32_t* err;
};

__global__ void __launch_bounds__(256) migrate_meta_kernel(MigArgs A) {
  const int t = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= A.n * A.lanes_per_req) return;
  const int i = w / A.lanes_per_req, l = w % A.lanes_per_req;
  const int sr = A.src_req[i], dr = A.dst_req[i];
  if (sr < 0 || sr >= A.R || dr < 0 || dr >= A.R) {
    if (t == 0) record_error(A.err, kErrRange);
    return;
  }
  const int64_t sl = (int64_t)sr * A.lanes_per_req + l, dl = (int64_t)dr * A.lanes_per_req + l;
  int32_t* ps = A.page_slot + dl * A.N;
  // empty the destination lane
  int dsz = A.size[dl];
  if (dsz < 0 || dsz > A.C) dsz = A.C;
  for (int s = t; s < dsz; s += 32) {
    const int pg = A.slot_page[dl * A.C + s];
    if (pg >= 0 && pg < A.N) ps[pg] = -1;
  }
  __syncwarp();
  int ssz = A.drop ? 0 : A.p_size[sl];
  if (ssz < 0 || ssz > A.C) {
    if (t == 0) record_error(A.err, kErrRange);
    ssz = 0;
  }
  for (int s = t; s < ssz; s += 32) {
    const int pg = A.p_slot_page[sl * A.C + s];
    A.slot_page[dl * A.C + s] = pg;
    A.order[dl * A.C + s] = A.p_order[sl * A.C + s];
    if (pg >= 0 && pg < A.N) ps[pg] = s;
  }
  if (t == 0) {
    A.size[dl] = ssz;
    if (l == 0) {
      A.ctx_pages[dr] = A.p_ctx_pages[sr];
      A.ctx_pages[A.R + dr] = A.p_ctx_pages[A.R + sr];  // tokens of the partial last page
      A.req_base[dr] = A.p_req_base[sr];  // the request keeps its home in the host pool
    }
  }
}

__global__ void __launch_bounds__(256) migrate_pages_kernel(MigArgs A) {
  const int t = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t total = (int64_t)A.n * A.lanes_per_req * A.C;
  uint32_t copied = 0;
  for (int64_t f = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); f < total; f += nw) {
    const int s = (int)(f % A.C);
    const int64_t il = f / A.C;
    const int i = (int)(il / A.lanes_per_req), l = (int)(il % A.lanes_per_req);
    const int sr = A.src_req[i], dr = A.dst_req[i];
    if (sr < 0 || sr >= A.R || dr < 0 || dr >= A.R) continue;
    const int64_t sl = (int64_t)sr * A.lanes_per_req + l, dl = (int64_t)dr * A.lanes_per_req + l;
    if (!A.full && s >= A.size[dl]) continue;  // delta: resident slots only
    const uint8_t* src = A.p_cache + ((size_t)sl * A.C + s) * A.unit_bytes;
    uint8_t* dst = A.cache + ((size_t)dl * A.C + s) * A.unit_bytes;
    warp_copy_unit(src, dst, A.unit_bytes, t);
    ++copied;
  }
  if (t == 0 && copied && A.stats) {
    atomicAdd(&A.stats[2], (unsigned long long)copied);
    atomicAdd(&A.stats[3], (unsigned long long)copied * A.unit_bytes);
  }
}

__global__ void release_kernel(MigArgs A) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= A.n) return;
  const int sr = A.src_req[i];
  if (sr >= 0 && sr < A.R && A.p_slot_state) st_release_sys_i32(A.p_slot_state + sr, 2);
}

}  // namespace
}  // namespace ferry

using namespace ferry;

namespace {
struct DevGuard2 {
  int prev = -1;
  explicit DevGuard2(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~DevGuard2() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

bool same_geometry(const ferry_cfg& a, const ferry_cfg& b) {
  return a.num_requests == b.num_requests && a.num_layers == b.num_layers &&
         a.q_heads == b.q_heads && a.kv_heads == b.kv_heads && a.max_pages == b.max_pages &&
         a.cache_pages == b.cache_pages && a.top_k == b.top_k && a.kv_dtype == b.kv_dtype;
}

void close_peer(ferry_peer& p) {
  if (p.ipc) {
    void* bufs[kPeerBufs] = {p.cache, p.page_slot, p.slot_page, p.order,
                             p.size,  p.ctx_pages, p.slot_state, p.req_base};
    for (void* b : bufs)
      if (b) cudaIpcCloseMemHandle(b);
    if (p.store) cudaIpcCloseMemHandle(p.store);
  }
  p = ferry_peer{};
}
}  // namespace

namespace ferry {
void close_all_peers(ferry_ctx* c) {
  for (auto& p : c->peers) close_peer(p);
  refresh_store_map(c);
}
}  // namespace ferry

extern "C" {

int ferry_ctx_export(ferry_ctx* c, void* handle) {
  if (!c || !handle) return set_error("ctx_export: bad arguments"), FERRY_E_INVAL;
  DevGuard2 g(c->device);
  PeerHandle h{};
  h.magic = kPeerMagic;
  h.device = c->device;
  h.cfg = c->cfg;
  const void* bufs[kPeerBufs] = {c->cache,    c->lru.page_slot, c->lru.slot_page, c->lru.order,
                                 c->lru.size, c->ctx_pages,     c->slot_state,    c->req_base};
  for (int i = 0; i < kPeerBufs; ++i) FERRY_TRY(cudaIpcGetMemHandle(&h.mem[i], (void*)bufs[i]));
  if (c->store) {
    h.has_store = 1;
    h.own_world = c->own_world;
    h.own_rank = c->own_rank;
    h.store_lanes = c->store_lanes;
    FERRY_TRY(cudaIpcGetMemHandle(&h.store_mem, c->store));
  }
  std::memset(handle, 0, FERRY_CTX_HANDLE_BYTES);
  std::memcpy(handle, &h, sizeof h);
  return FERRY_OK;
}

int ferry_ctx_import(ferry_ctx* c, int peer_slot, const void* handle) {
  if (!c || !handle || peer_slot < 0 || peer_slot >= FERRY_MAX_PEERS)
    return set_error("ctx_import: bad arguments"), FERRY_E_INVAL;
  PeerHandle h;
  std::memcpy(&h, handle, sizeof h);
  if (h.magic != kPeerMagic) return set_error("ctx_import: not a ctx handle"), FERRY_E_INVAL;
  if (!same_geometry(h.cfg, c->cfg)) return set_error("ctx_import: peer geometry differs"), FERRY_E_INVAL;
  DevGuard2 g(c->device);
  close_peer(c->peers[peer_slot]);
  void* p[kPeerBufs] = {};
  for (int i = 0; i < kPeerBufs; ++i) {
    cudaError_t e = cudaIpcOpenMemHandle(&p[i], h.mem[i], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaIpcCloseMemHandle(p[j]);
      return cuda_status(e, "cudaIpcOpenMemHandle");
    }
  }
  void* st = nullptr;
  if (h.has_store) {
    cudaError_t e = cudaIpcOpenMemHandle(&st, h.store_mem, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < kPeerBufs; ++j) cudaIpcCloseMemHandle(p[j]);
      return cuda_status(e, "cudaIpcOpenMemHandle (store)");
    }
  }
  ferry_peer& q = c->peers[peer_slot];
  q.ipc = true;
  q.device = h.device;
  q.store = (uint8_t*)st;
  q.own_world = h.has_store ? h.own_world : 0;
  q.own_rank = h.has_store ? h.own_rank : -1;
  q.store_lanes = h.has_store ? h.store_lanes : 0;
  q.cache = (uint8_t*)p[0];
  q.page_slot = (int32_t*)p[1];
  q.slot_page = (int32_t*)p[2];
  q.order = (int32_t*)p[3];
  q.size = (int32_t*)p[4];
  q.ctx_pages = (int32_t*)p[5];
  q.slot_state = (int32_t*)p[6];
  q.req_base = (int64_t*)p[7];
  refresh_store_map(c);
  return FERRY_OK;
}

int ferry_ctx_link(ferry_ctx* c, int peer_slot, ferry_ctx* peer) {
  if (!c || !peer || peer_slot < 0 || peer_slot >= FERRY_MAX_PEERS)
    return set_error("ctx_link: bad arguments"), FERRY_E_INVAL;
  if (!same_geometry(peer->cfg, c->cfg)) return set_error("ctx_link: peer geometry differs"), FERRY_E_INVAL;
  DevGuard2 g(c->device);
  if (peer->device != c->device) {
    int can = 0;
    FERRY_TRY(cudaDeviceCanAccessPeer(&can, c->device, peer->device));
    if (!can) return set_error("device %d cannot access device %d", c->device, peer->device), FERRY_E_INVAL;
    cudaError_t e = cudaDeviceEnablePeerAccess(peer->device, 0);
    if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return cuda_status(e, "cudaDeviceEnablePeerAccess");
    cudaGetLastError();
  }
  close_peer(c->peers[peer_slot]);
  ferry_peer& q = c->peers[peer_slot];
  q.ipc = false;
  q.device = peer->device;
  q.cache = peer->cache;
  q.page_slot = peer->lru.page_slot;
  q.slot_page = peer->lru.slot_page;
  q.order = peer->lru.order;
  q.size = peer->lru.size;
  q.ctx_pages = peer->ctx_pages;
  q.slot_state = peer->slot_state;
  q.req_base = peer->req_base;
  q.store = peer->store;
  q.own_world = peer->own_world;
  q.own_rank = peer->own_rank;
  q.store_lanes = peer->store_lanes;
  refresh_store_map(c);
  return FERRY_OK;
}

int ferry_migrate_requests(ferry_ctx* c, void* stream, int peer_slot, const int32_t* d_src_req,
                           const int32_t* d_dst_req, int n, int mode) {
  if (!c || peer_slot < 0 || peer_slot >= FERRY_MAX_PEERS || n < 0 || (n && (!d_src_req || !d_dst_req)) ||
      (mode != FERRY_MIGRATE_FULL && mode != FERRY_MIGRATE_DELTA && mode != FERRY_MIGRATE_DROP))
    return set_error("migrate_requests: bad arguments"), FERRY_E_INVAL;
  const ferry_peer& p = c->peers[peer_slot];
  if (!p.cache) return set_error("migrate_requests: peer slot %d is not linked", peer_slot), FERRY_E_STATE;
  if (n == 0) return FERRY_OK;
  DevGuard2 g(c->device);
  MigArgs A{};
  A.p_cache = p.cache;
  A.p_slot_page = p.slot_page;
  A.p_order = p.order;
  A.p_size = p.size;
  A.p_ctx_pages = p.ctx_pages;
  A.p_slot_state = p.slot_state;
  A.p_req_base = p.req_base;
  A.req_base = c->req_base;
  A.cache = c->cache;
  A.page_slot = c->lru.page_slot;
  A.slot_page = c->lru.slot_page;
  A.order = c->lru.order;
  A.size = c->lru.size;
  A.ctx_pages = c->ctx_pages;
  A.src_req = d_src_req;
  A.dst_req = d_dst_req;
  A.n = n;
  A.lanes_per_req = c->lanes_per_req;
  A.R = c->cfg.num_requests;
  A.C = c->cfg.cache_pages;
  A.N = c->cfg.max_pages;
  A.full = mode == FERRY_MIGRATE_FULL;
  A.drop = mode == FERRY_MIGRATE_DROP;
  A.unit_bytes = c->unit_bytes;
  A.stats = c->stats;
  A.err = c->err;
  cudaStream_t st = (cudaStream_t)stream;
  const int lanes = n * c->lanes_per_req;
  migrate_meta_kernel<<<(lanes + 7) / 8, 256, 0, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  if (!A.drop) {
    const int64_t items = (int64_t)lanes * A.C;
    const int64_t blocks = std::min<int64_t>((items + 7) / 8, (int64_t)c->num_sms * 16);
    migrate_pages_kernel<<<(unsigned)blocks, 256, 0, st>>>(A);
    FERRY_TRY(cudaGetLastError());
  }
  release_kernel<<<(n + 127) / 128, 128, 0, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_slot_states(ferry_ctx* c, int32_t* host_out, int clear_migrated) {
  if (!c || !host_out) return set_error("slot_states: bad arguments"), FERRY_E_INVAL;
  DevGuard2 g(c->device);
  FERRY_TRY(cudaDeviceSynchronize());
  const size_t R = c->cfg.num_requests;
  FERRY_TRY(cudaMemcpy(host_out, c->slot_state, R * 4, cudaMemcpyDeviceToHost));
  if (clear_migrated)
    for (size_t r = 0; r < R; ++r)
      if (host_out[r] == 2) FERRY_TRY(cudaMemset(c->slot_state + r, 0, 4));
  return FERRY_OK;
}

}  // extern "C"
