// gather.cu -- miss gather: missed page units from the pinned host pool (or a
// peer GPU's memory) into their HBM cache slots.
//
// The reference moves misses with host-driven cudaMemcpyAsync through a
// pinned ring (HostStagedChannel::submit, src/comm/host_staged_channel.cpp:43-74)
// after sorting and run-merging them on the CPU
// (src/runtime/wla_multigpu.cuh:2544-2593). Here the GPU pulls the pages
// itself: one warp per missed page unit, 16 outstanding 16-byte loads per lane
// (the whole 8 KiB unit in flight per warp), then 16 coalesced stores. The
// copy is index-driven straight from the miss list, so there is no host hop,
// no run merging and no per-run launch.
#include "common.cuh"

namespace ferry {
namespace {

__global__ void __launch_bounds__(256) gather_kernel(
    const uint8_t* __restrict__ pool, uint64_t pool_units, uint8_t* __restrict__ cache, int N,
    int C, const int32_t* __restrict__ req_ids, int lanes_per_req, int64_t lanes_total,
    int n_lanes, const int32_t* __restrict__ miss_page, const int32_t* __restrict__ miss_slot,
    const int32_t* __restrict__ n_miss, int k, const int64_t* __restrict__ req_base, int unit_bytes,
    const __grid_constant__ OwnerMap own, unsigned long long* stats, uint32_t* err) {
  const int t = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t total = (int64_t)n_lanes * k;
  uint32_t copied = 0, from_peer = 0, from_self = 0;
  for (int64_t f = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); f < total;
       f += nw) {
    const int a = (int)(f / k), i = (int)(f % k);
    if (i >= n_miss[a]) continue;  // warp-uniform
    const int page = miss_page[(size_t)a * k + i];
    const int slot = miss_slot[(size_t)a * k + i];
    const int req = req_ids[a / lanes_per_req];
    const int64_t gl = (int64_t)req * lanes_per_req + a % lanes_per_req;
    if (page < 0 || page >= N || slot < 0 || slot >= C || gl < 0 || gl >= lanes_total) {
      if (t == 0) record_error(err, kErrRange);
      continue;
    }
    const int64_t home = req_base[req] + (int64_t)(a % lanes_per_req) * N;  // global lane * N
    const uint8_t* src = nullptr;
    if (own.world > 0) {
      // the owner of page p is rank p % world; its store holds (lane, p) at
      // lane * own_np + p / world
      const int owner = page % own.world;
      const int64_t glane = home / N;
      if (glane >= 0 && glane < own.store_lanes && own.store[owner]) {
        src = own.store[owner] + ((size_t)glane * own.own_np + page / own.world) * unit_bytes;
        if (owner == own.self)
          ++from_self;
        else
          ++from_peer;
      }
    }
    if (!src) {
      if (!pool) {  // stores only: every owner must be mapped
        if (t == 0) record_error(err, kErrRange);
        continue;
      }
      src = pool + ((uint64_t)(home + page) % pool_units) * unit_bytes;
    }
    uint8_t* dst = cache + ((uint64_t)gl * C + slot) * unit_bytes;
    warp_copy_unit(src, dst, unit_bytes, t);
    ++copied;
  }
  if (t == 0 && copied && stats) {
    atomicAdd(&stats[0], (unsigned long long)copied);
    atomicAdd(&stats[1], (unsigned long long)copied * unit_bytes);
    if (from_peer) {
      atomicAdd(&stats[4], (unsigned long long)from_peer);
      atomicAdd(&stats[5], (unsigned long long)from_peer * unit_bytes);
    }
    if (from_self) {
      atomicAdd(&stats[6], (unsigned long long)from_self);
      atomicAdd(&stats[7], (unsigned long long)from_self * unit_bytes);
    }
  }
}

// Owner-store gathers (FERRY_SRC_OWNER): units whose owner store is
// mapped move by the TMA engine -- lane 0 of each warp streams them through
// a 2-stage shared-memory ring with 1-D bulk copies (load from the owner's
// store, this GPU's HBM or a peer's over NVLink; then a bulk store into the
// cache slot), one unit's load in flight while the previous one is stored.
// Units without a mapped owner fall back to a plain copy from the host pool
// (one 16-byte chunk per lane at a time: few registers, so that more warps,
// each an independent bulk-copy issuer, fit on an SM). With host_bulk
// (FERRY_SRC_HOST_BULK, own.world == 0) the host-pool units take the bulk
// ring too: the TMA engine reads each 8 KiB unit from the mapped pool as one
// copy instead of 512 16-byte SM loads.
constexpr int kGtMaxWarps = 16;
constexpr int kGtSmemBudget = 200 * 1024;

// bytes of one ring stage: the unit rounded up to 128
__host__ __device__ constexpr int gt_stride(int unit_bytes) { return (unit_bytes + 127) / 128 * 128; }
// shared memory of one warp: two stages and their barriers
constexpr int gt_warp_smem(int unit_bytes) { return 2 * gt_stride(unit_bytes) + 16; }

__device__ __forceinline__ void bulk_store(void* dst_global, const void* src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_global),
               "r"(smem_addr(src_smem)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// this thread's bulk stores have all finished reading shared memory
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(kGtMaxWarps * 32, 1) gather_store_kernel(
    const uint8_t* __restrict__ pool, uint64_t pool_units, uint8_t* __restrict__ cache, int N,
    int C, const int32_t* __restrict__ req_ids, int lanes_per_req, int64_t lanes_total,
    int n_lanes, const int32_t* __restrict__ miss_page, const int32_t* __restrict__ miss_slot,
    const int32_t* __restrict__ n_miss, int k, const int64_t* __restrict__ req_base, int unit_bytes,
    const __grid_constant__ OwnerMap own, bool host_bulk, unsigned long long* stats, uint32_t* err) {
  extern __shared__ __align__(128) uint8_t gsm[];
  const int t = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int stride = gt_stride(unit_bytes);
  uint8_t* ring = gsm + (size_t)warp * 2 * stride;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gsm + (size_t)nwarps * 2 * stride) + warp * 2;
  if (t == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const int64_t nw = (int64_t)gridDim.x * nwarps;
  const int64_t total = (int64_t)n_lanes * k;
  uint32_t copied = 0, from_peer = 0, from_self = 0;
  uint32_t it = 0;           // units this warp sent through the ring
  int pend = -1;             // stage whose load is still to be stored
  uint8_t* pend_dst = nullptr;
  bool ok = true;
  auto flush = [&]() {       // store the pending stage (lane 0)
    if (pend < 0) return;
    const uint32_t use = it - 1;  // the pending unit is the last one sent
    if (mbar_wait(&bars[pend], (use >> 1) & 1u, err))
      bulk_store(pend_dst, ring + pend * stride, (uint32_t)unit_bytes);
    else
      ok = false;
    pend = -1;
  };
  for (int64_t f = (int64_t)blockIdx.x * nwarps + warp; f < total && ok; f += nw) {
    const int a = (int)(f / k), i = (int)(f % k);
    if (i >= n_miss[a]) continue;  // warp-uniform
    const int page = miss_page[(size_t)a * k + i];
    const int slot = miss_slot[(size_t)a * k + i];
    const int req = req_ids[a / lanes_per_req];
    const int64_t gl = (int64_t)req * lanes_per_req + a % lanes_per_req;
    if (page < 0 || page >= N || slot < 0 || slot >= C || gl < 0 || gl >= lanes_total) {
      if (t == 0) record_error(err, kErrRange);
      continue;
    }
    const int64_t home = req_base[req] + (int64_t)(a % lanes_per_req) * N;  // global lane * N
    const int64_t glane = home / N;
    uint8_t* dst = cache + ((uint64_t)gl * C + slot) * unit_bytes;
    const uint8_t* src = nullptr;
    bool bulk = false;
    if (own.world > 0) {
      const int owner = page % own.world;
      if (glane >= 0 && glane < own.store_lanes && own.store[owner]) {
        src = own.store[owner] + ((size_t)glane * own.own_np + page / own.world) * unit_bytes;
        bulk = true;
        if (owner == own.self)
          ++from_self;
        else
          ++from_peer;
      }
    }
    if (!src && pool) {
      src = pool + ((uint64_t)(home + page) % pool_units) * unit_bytes;
      bulk = host_bulk;
    }
    if (!src) {  // stores only: every owner must be mapped
      if (t == 0) record_error(err, kErrRange);
      continue;
    }
    ++copied;
    if (bulk) {
      if (t == 0) {
        const int s = it & 1;
        bulk_wait_read();  // the store that last read stage s (the newest group) is done with it
        mbar_arrive_expect_tx(&bars[s], (uint32_t)unit_bytes);
        bulk_load(ring + s * stride, src, (uint32_t)unit_bytes, &bars[s]);
        ++it;
        const int ps = pend;
        uint8_t* pd = pend_dst;
        if (ps >= 0) {  // store the previous unit while this one loads
          if (mbar_wait(&bars[ps], ((it - 2) >> 1) & 1u, err))
            bulk_store(pd, ring + ps * stride, (uint32_t)unit_bytes);
          else
            ok = false;
        }
        pend = s;
        pend_dst = dst;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    } else {
      for (int v = t; v < (unit_bytes >> 4); v += 32) st_v4(dst + (size_t)v * 16, ld_nc_v4(src + (size_t)v * 16));
    }
  }
  if (t == 0) {
    if (ok) flush();
    // drain: loads still in flight land (bounded), stores complete
    if (!ok)
      for (uint32_t u = it >= 2 ? it - 2 : 0; u < it; ++u) mbar_wait(&bars[u & 1], (u >> 1) & 1u, nullptr);
    bulk_wait_all();
  }
  __syncwarp();
  if (t == 0 && copied && stats) {
    atomicAdd(&stats[0], (unsigned long long)copied);
    atomicAdd(&stats[1], (unsigned long long)copied * unit_bytes);
    if (from_peer) {
      atomicAdd(&stats[4], (unsigned long long)from_peer);
      atomicAdd(&stats[5], (unsigned long long)from_peer * unit_bytes);
    }
    if (from_self) {
      atomicAdd(&stats[6], (unsigned long long)from_self);
      atomicAdd(&stats[7], (unsigned long long)from_self * unit_bytes);
    }
  }
}

}  // namespace

int launch_gather(const ferry_ctx* c, cudaStream_t st, const int32_t* req_ids, int n_req,
                  const int32_t* miss_page, const int32_t* miss_slot, const int32_t* n_miss, bool shared) {
  if (n_req <= 0) return FERRY_OK;
  if (!c->pool_dev && !(c->stores_only && c->gather_src == FERRY_SRC_OWNER)) {
    set_error(c->stores_only ? "gather: a ctx without a host pool gathers from owner stores only"
                             : "gather: no host pool registered");
    return FERRY_E_STATE;
  }
  OwnerMap own{};
  if (c->gather_src == FERRY_SRC_OWNER && c->store) {
    own.world = c->own_world;
    own.self = c->own_rank;
    own.own_np = c->own_np;
    own.store_lanes = c->store_lanes;
    for (int r = 0; r <= FERRY_MAX_PEERS; ++r) own.store[r] = c->store_of[r];
  }
  const int n_lanes = n_req * c->lanes_per_req;
  const int64_t items = (int64_t)n_lanes * c->cfg.top_k;
  const bool host_bulk = c->gather_src == FERRY_SRC_HOST_BULK;
  if (own.world > 0 || host_bulk) {
    // shared: half the shared-memory budget, so that selection and attention
    // CTAs fit beside the ring on every SM
    const int budget = shared ? kGtSmemBudget / 2 : kGtSmemBudget;
    const int warps = std::max(1, std::min(kGtMaxWarps, budget / gt_warp_smem(c->unit_bytes)));
    const int smem = warps * gt_warp_smem(c->unit_bytes);
    FERRY_TRY(cudaFuncSetAttribute(gather_store_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int64_t blocks = std::min<int64_t>((items + warps - 1) / warps, (int64_t)c->num_sms);
    gather_store_kernel<<<(unsigned)blocks, warps * 32, smem, st>>>(
        c->pool_dev, c->pool_units, c->cache, c->cfg.max_pages, c->cfg.cache_pages, req_ids,
        c->lanes_per_req, c->lanes, n_lanes, miss_page, miss_slot, n_miss, c->cfg.top_k, c->req_base,
        c->unit_bytes, own, host_bulk, c->stats, c->err);
    FERRY_TRY(cudaGetLastError());
    return FERRY_OK;
  }
  // enough warps to keep the host link saturated, capped at 16 CTAs per SM;
  // beside other kernels 2 per SM (16 warps, a unit each in flight: far more
  // bytes in flight than the host link's latency needs)
  const int64_t blocks = std::min<int64_t>((items + 7) / 8, (int64_t)c->num_sms * (shared ? 2 : 16));
  gather_kernel<<<(unsigned)blocks, 256, 0, st>>>(
      c->pool_dev, c->pool_units, c->cache, c->cfg.max_pages, c->cfg.cache_pages, req_ids,
      c->lanes_per_req, c->lanes, n_lanes, miss_page, miss_slot, n_miss, c->cfg.top_k, c->req_base,
      c->unit_bytes, own, c->stats, c->err);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

}  // namespace ferry
