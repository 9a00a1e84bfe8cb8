// group.cu -- group lanes: the prefix-group-shared LRU of the reference's
// kv_touch, keyed per (GPU, prefix group, layer)
// (src/runtime/wla_multigpu.cuh:1867-2015), on the device LRU lanes.
//
// A group lane is an ordinary ferry_lru lane that every member of a prefix
// group touches (ferry_lru_touch_owned, members in request order). On top of
// the plain LRU it keeps
//   * a capacity per lane (cap_mode 1: wla_group_cap = hot x resident
//     members, src/workloads/missstream.cuh:91-94). Shrinking it trims the
//     lane from the LRU front (grp_trim, :1923-1935);
//   * an owner mask per resident page, one bit per group member (own_bit,
//     :1877-1879): a touch ORs the member's bit in, an eviction drops the
//     page's mask (own_drop), a departing member's bit is cleared everywhere
//     (own_release, :1896-1911);
//   * the steal-time handoff of a lane to another GPU's lane
//     (kv_handoff / kv_handoff_owned, :1970-2015): drop (the consumer starts
//     cold), carry (the consumer's lane becomes a copy), or owned (only pages
//     whose mask is exactly the moving member's bit are merged into the
//     consumer's lane, which evicts from its front as it fills).
//
// Slots. The device lanes keep a page table whose occupied slots are always
// [0, size): a miss takes slot `size` while the lane is not full, else the
// slot of the page it evicts. A trim keeps that invariant by compaction: the
// evicted front pages free their slots; survivors sitting at slots >= the new
// capacity move, in LRU order (front first), into the freed slots below it in
// ascending slot order, taking their owner masks along. (The reference keeps
// block ids in a deque and has no slots; the slot rules are this build's.)
#include <vector>

#include "common.cuh"

namespace ferry {
namespace {

// One warp per listed lane: trim to the new capacity with slot compaction,
// then record the capacity. Dynamic shared memory: 3 * cap ints per warp.
__global__ void __launch_bounds__(32) trim_kernel(int32_t* page_slot, int32_t* slot_page, int32_t* order,
                                                  int32_t* size, int32_t* lane_cap, uint32_t* mask, int lanes,
                                                  int cap, int ids, const int32_t* lane_ids,
                                                  const int32_t* caps, int n, uint32_t* err) {
  extern __shared__ int32_t tsm[];
  const int t = threadIdx.x, a = blockIdx.x;
  if (a >= n) return;
  const int lane = lane_ids[a], c = caps[a];
  if (lane < 0 || lane >= lanes || c < 1 || c > cap) {
    if (t == 0) record_error(err, kErrRange);
    return;
  }
  int32_t* ps = page_slot + (size_t)lane * ids;
  int32_t* sp = slot_page + (size_t)lane * cap;
  int32_t* od = order + (size_t)lane * cap;
  uint32_t* mk = mask + (size_t)lane * cap;
  const int sz = size[lane];
  if (sz < 0 || sz > cap) {
    if (t == 0) record_error(err, kErrRange);
    return;
  }
  if (sz <= c) {
    if (t == 0) lane_cap[lane] = c;
    return;
  }
  int32_t* o = tsm;            // the lane's order
  int32_t* freed = o + cap;    // freed[s] != 0: slot s < c was freed by the trim
  int32_t* fr = freed + cap;   // freed slots below c in ascending order
  const uint32_t lt = (1u << t) - 1u;
  const int e = sz - c;
  for (int j = t; j < sz; j += 32) o[j] = od[j];
  for (int s = t; s < c; s += 32) freed[s] = 0;
  __syncwarp();
  for (int j = t; j < e; j += 32) {  // the front e pages leave (own_drop with them)
    const int s = o[j];
    if (s < 0 || s >= cap) {
      record_error(err, kErrRange);
      continue;
    }
    const int pg = sp[s];
    if (pg >= 0 && pg < ids) ps[pg] = -1;
    sp[s] = -1;
    mk[s] = 0u;
    if (s < c) freed[s] = 1;
  }
  __syncwarp();
  int nf = 0;
  for (int s0 = 0; s0 < c; s0 += 32) {
    const int s = s0 + t;
    const bool f = s < c && freed[s];
    const uint32_t m = __ballot_sync(0xffffffffu, f);
    if (f) fr[nf + __popc(m & lt)] = s;
    nf += __popc(m);
  }
  __syncwarp();
  int nm = 0;
  for (int j0 = e; j0 < sz; j0 += 32) {  // survivors above the new capacity move down
    const int j = j0 + t;
    const int s = j < sz ? o[j] : -1;
    const bool mv = s >= c && s < cap;
    const uint32_t m = __ballot_sync(0xffffffffu, mv);
    if (mv) {
      const int r = nm + __popc(m & lt);
      if (r < nf) {
        const int f = fr[r], pg = sp[s];
        sp[f] = pg;
        if (pg >= 0 && pg < ids) ps[pg] = f;
        mk[f] = mk[s];
        sp[s] = -1;
        mk[s] = 0u;
        o[j] = f;
      } else {
        record_error(err, kErrRange);  // the occupied slots were not [0, size)
      }
    }
    nm += __popc(m);
  }
  __syncwarp();
  for (int j = e + t; j < sz; j += 32) od[j - e] = o[j];
  if (t == 0) {
    size[lane] = c;
    lane_cap[lane] = c;
  }
}

// own_release: clear `bit` in every resident page's mask of the listed lanes.
__global__ void release_kernel(uint32_t* mask, const int32_t* size, int lanes, int cap, const int32_t* lane_ids,
                               int n, uint32_t bit, uint32_t* err) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), t = threadIdx.x & 31;
  if (w >= n) return;
  const int lane = lane_ids[w];
  if (lane < 0 || lane >= lanes) {
    if (t == 0) record_error(err, kErrRange);
    return;
  }
  const int sz = min(max(size[lane], 0), cap);
  uint32_t* mk = mask + (size_t)lane * cap;
  for (int s = t; s < sz; s += 32) mk[s] &= ~bit;
}

// kv_live_owned per lane: resident pages whose mask is exactly `bit`.
__global__ void count_owned_kernel(const uint32_t* mask, const int32_t* size, int lanes, int cap,
                                   const int32_t* lane_ids, int n, uint32_t bit, int32_t* out, uint32_t* err) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), t = threadIdx.x & 31;
  if (w >= n) return;
  const int lane = lane_ids[w];
  if (lane < 0 || lane >= lanes) {
    if (t == 0) {
      record_error(err, kErrRange);
      out[w] = 0;
    }
    return;
  }
  const int sz = min(max(size[lane], 0), cap);
  const uint32_t* mk = mask + (size_t)lane * cap;
  int c = 0;
  for (int s = t; s < sz; s += 32) c += mk[s] == bit;
  c = __reduce_add_sync(0xffffffffu, c);
  if (t == 0) out[w] = c;
}

struct LaneRef {
  int32_t* page_slot;
  int32_t* slot_page;
  int32_t* order;
  int32_t* size;
  const int32_t* lane_cap;
  uint32_t* mask;
  int lanes, cap, ids;
};

// Drop (the consumer lane empties) and carry (it becomes a copy of the
// source lane, masks included): one warp per lane pair.
__global__ void handoff_copy_kernel(LaneRef src, LaneRef dst, const int32_t* src_lanes, const int32_t* dst_lanes,
                                    int n, int carry, uint32_t* err) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), t = threadIdx.x & 31;
  if (w >= n) return;
  const int dl = dst_lanes[w], sl = carry ? src_lanes[w] : 0;
  if (dl < 0 || dl >= dst.lanes || sl < 0 || sl >= src.lanes) {
    if (t == 0) record_error(err, kErrRange);
    return;
  }
  int32_t* dps = dst.page_slot + (size_t)dl * dst.ids;
  int32_t* dsp = dst.slot_page + (size_t)dl * dst.cap;
  int32_t* dod = dst.order + (size_t)dl * dst.cap;
  uint32_t* dmk = dst.mask + (size_t)dl * dst.cap;
  const int dsz = min(max(dst.size[dl], 0), dst.cap);
  if (!carry) {
    for (int s = t; s < dsz; s += 32) {
      const int pg = dsp[s];
      if (pg >= 0 && pg < dst.ids) dps[pg] = -1;
      dsp[s] = -1;
      dmk[s] = 0u;
    }
    __syncwarp();
    if (t == 0) dst.size[dl] = 0;
    return;
  }
  const int ssz = src.size[sl];
  const int dcap = dst.lane_cap ? dst.lane_cap[dl] : dst.cap;
  if (ssz < 0 || ssz > src.cap || ssz > dcap) {  // the copy would overfill the consumer lane
    if (t == 0) record_error(err, kErrRange);
    return;
  }
  const int32_t* sps = src.page_slot + (size_t)sl * src.ids;
  const int32_t* ssp = src.slot_page + (size_t)sl * src.cap;
  const int32_t* sod = src.order + (size_t)sl * src.cap;
  const uint32_t* smk = src.mask + (size_t)sl * src.cap;
  for (int i = t; i < dst.ids; i += 32) dps[i] = sps[i];
  for (int s = t; s < dst.cap; s += 32) {
    dsp[s] = s < ssz ? ssp[s] : -1;
    dmk[s] = s < ssz ? smk[s] : 0u;
    if (s < ssz) dod[s] = sod[s];
  }
  __syncwarp();
  if (t == 0) dst.size[dl] = ssz;
}

// kv_handoff_owned: one thread per lane pair walks the source lane from its
// LRU front; a page whose mask is exactly `bit` is merged into the consumer
// lane -- already resident there: the bit is ORed in and the page keeps its
// place; else the consumer evicts its front while full and appends the page
// with mask `bit`. The consumer's order is kept as a ring over its cap
// entries during the walk and rotated back to front-first at the end.
__global__ void handoff_owned_kernel(LaneRef src, LaneRef dst, const int32_t* src_lanes, const int32_t* dst_lanes,
                                     int n, uint32_t bit, uint32_t* err) {
  const int w = blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= n) return;
  const int sl = src_lanes[w], dl = dst_lanes[w];
  if (sl < 0 || sl >= src.lanes || dl < 0 || dl >= dst.lanes) {
    record_error(err, kErrRange);
    return;
  }
  const int32_t* ssp = src.slot_page + (size_t)sl * src.cap;
  const int32_t* sod = src.order + (size_t)sl * src.cap;
  const uint32_t* smk = src.mask + (size_t)sl * src.cap;
  int32_t* dps = dst.page_slot + (size_t)dl * dst.ids;
  int32_t* dsp = dst.slot_page + (size_t)dl * dst.cap;
  int32_t* dod = dst.order + (size_t)dl * dst.cap;
  uint32_t* dmk = dst.mask + (size_t)dl * dst.cap;
  const int ssz = src.size[sl], C = dst.cap;
  const int dcap = dst.lane_cap ? dst.lane_cap[dl] : C;
  int cnt = dst.size[dl], head = 0;
  if (ssz < 0 || ssz > src.cap || cnt < 0 || cnt > dcap || dcap < 1 || dcap > C) {
    record_error(err, kErrRange);
    return;
  }
  for (int j = 0; j < ssz; ++j) {
    const int s = sod[j];
    if (s < 0 || s >= src.cap) {
      record_error(err, kErrRange);
      return;
    }
    if (smk[s] != bit) continue;  // shared or dead pages stay behind
    const int pg = ssp[s];
    if (pg < 0 || pg >= dst.ids) {
      record_error(err, kErrRange);
      return;
    }
    const int d = dps[pg];
    if (d >= 0) {
      dmk[d] |= bit;
      continue;
    }
    int slot;
    if (cnt >= dcap) {  // evict the consumer's front; its slot takes the page
      slot = dod[head];
      head = head + 1 == C ? 0 : head + 1;
      --cnt;
      const int v = dsp[slot];
      if (v >= 0 && v < dst.ids) dps[v] = -1;
    } else {
      slot = cnt;  // the occupied slots are [0, cnt)
    }
    int tail = head + cnt;
    if (tail >= C) tail -= C;
    dod[tail] = slot;
    ++cnt;
    dsp[slot] = pg;
    dps[pg] = slot;
    dmk[slot] = bit;
  }
  if (head) {  // rotate the ring left by head: three reversals
    auto rev = [&](int lo, int hi) {
      for (--hi; lo < hi; ++lo, --hi) {
        const int32_t x = dod[lo];
        dod[lo] = dod[hi];
        dod[hi] = x;
      }
    };
    rev(0, head);
    rev(head, C);
    rev(0, C);
  }
  dst.size[dl] = cnt;
}

LaneRef lane_ref(const ferry_lru* L) {
  return LaneRef{L->page_slot, L->slot_page, L->order, L->size, L->lane_cap, L->mask, L->lanes, L->cap, L->ids};
}

int group_check(const ferry_lru* L, const char* what) {
  if (!L) {
    set_error("%s: lru is NULL", what);
    return FERRY_E_INVAL;
  }
  if (!L->mask || !L->lane_cap) {
    set_error("%s: call ferry_lru_group_enable first", what);
    return FERRY_E_STATE;
  }
  return FERRY_OK;
}

}  // namespace
}  // namespace ferry

using namespace ferry;

extern "C" {

int ferry_lru_group_enable(ferry_lru* L) {
  if (!L) return set_error("lru_group_enable: lru is NULL"), FERRY_E_INVAL;
  if (L->mask) return FERRY_OK;
  DeviceGuard guard(L->device);
  int32_t* caps = nullptr;
  uint32_t* mask = nullptr;
  int rc = dev_alloc(&caps, (size_t)L->lanes, 0);
  if (!rc) rc = dev_alloc(&mask, (size_t)L->lanes * L->cap, 0);
  if (rc) {
    cudaFree(caps);
    return rc;
  }
  std::vector<int32_t> h((size_t)L->lanes, L->cap);
  const cudaError_t e = cudaMemcpy(caps, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(caps);
    cudaFree(mask);
    return cuda_status(e, "lru_group_enable");
  }
  L->lane_cap = caps;
  L->mask = mask;
  return FERRY_OK;
}

int ferry_lru_touch_owned(ferry_lru* L, void* stream, const int32_t* d_lane_ids, const uint8_t* d_reset, int n,
                          const int32_t* d_sel, int k, const int32_t* d_n_sel, int flags, const uint32_t* d_bits,
                          uint8_t* d_is_miss, int32_t* d_item_slot, int32_t* d_miss_page, int32_t* d_miss_slot,
                          int32_t* d_n_miss) {
  int rc = group_check(L, "lru_touch_owned");
  if (rc) return rc;
  if (n < 0 || (n && (!d_lane_ids || !d_bits))) return set_error("lru_touch_owned: bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(L->device);
  return launch_lru(L, (cudaStream_t)stream, d_lane_ids, nullptr, 1, d_reset, n, d_sel, k, d_n_sel,
                    (flags & FERRY_LRU_DISTINCT) ? 1 : 0, d_is_miss, d_item_slot, d_miss_page, d_miss_slot,
                    d_n_miss, d_bits);
}

int ferry_lru_set_capacity(ferry_lru* L, void* stream, const int32_t* d_lane_ids, const int32_t* d_caps, int n) {
  int rc = group_check(L, "lru_set_capacity");
  if (rc) return rc;
  if (n < 0 || (n && (!d_lane_ids || !d_caps))) return set_error("lru_set_capacity: bad arguments"), FERRY_E_INVAL;
  if (n == 0) return FERRY_OK;
  const size_t smem = (size_t)3 * L->cap * 4;
  if (smem > kLruLaneSmemMax)
    return set_error("lru_set_capacity: capacity %d needs %zu bytes of shared memory", L->cap, smem), FERRY_E_INVAL;
  DeviceGuard guard(L->device);
  if (smem > 48 * 1024)
    FERRY_TRY(cudaFuncSetAttribute(trim_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  trim_kernel<<<(unsigned)n, 32, smem, (cudaStream_t)stream>>>(L->page_slot, L->slot_page, L->order, L->size,
                                                                 L->lane_cap, L->mask, L->lanes, L->cap, L->ids,
                                                                 d_lane_ids, d_caps, n, L->err);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_lru_release(ferry_lru* L, void* stream, const int32_t* d_lane_ids, int n, uint32_t bit) {
  int rc = group_check(L, "lru_release");
  if (rc) return rc;
  if (n < 0 || (n && !d_lane_ids)) return set_error("lru_release: bad arguments"), FERRY_E_INVAL;
  if (n == 0 || bit == 0) return FERRY_OK;
  DeviceGuard guard(L->device);
  release_kernel<<<(unsigned)((n + 7) / 8), 256, 0, (cudaStream_t)stream>>>(L->mask, L->size, L->lanes, L->cap,
                                                                              d_lane_ids, n, bit, L->err);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_lru_count_owned(ferry_lru* L, void* stream, const int32_t* d_lane_ids, int n, uint32_t bit,
                          int32_t* d_count) {
  int rc = group_check(L, "lru_count_owned");
  if (rc) return rc;
  if (n < 0 || (n && (!d_lane_ids || !d_count))) return set_error("lru_count_owned: bad arguments"), FERRY_E_INVAL;
  if (n == 0) return FERRY_OK;
  DeviceGuard guard(L->device);
  count_owned_kernel<<<(unsigned)((n + 7) / 8), 256, 0, (cudaStream_t)stream>>>(L->mask, L->size, L->lanes, L->cap,
                                                                                  d_lane_ids, n, bit, d_count, L->err);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_lru_handoff(ferry_lru* dst, void* stream, const ferry_lru* src, const int32_t* d_src_lanes,
                      const int32_t* d_dst_lanes, int n, int mode, uint32_t bit) {
  int rc = group_check(dst, "lru_handoff");
  if (rc) return rc;
  if (mode != FERRY_HANDOFF_DROP && (rc = group_check(src, "lru_handoff"))) return rc;
  if (n < 0 || (n && !d_dst_lanes) || (mode != FERRY_HANDOFF_DROP && n && !d_src_lanes) ||
      (mode != FERRY_HANDOFF_DROP && mode != FERRY_HANDOFF_CARRY && mode != FERRY_HANDOFF_OWNED) ||
      (mode == FERRY_HANDOFF_OWNED && bit == 0))
    return set_error("lru_handoff: bad arguments"), FERRY_E_INVAL;
  if (mode != FERRY_HANDOFF_DROP && (src->ids != dst->ids || (mode == FERRY_HANDOFF_CARRY && src->cap != dst->cap)))
    return set_error("lru_handoff: source and consumer lanes differ in ids or capacity"), FERRY_E_INVAL;
  if (n == 0) return FERRY_OK;
  DeviceGuard guard(dst->device);
  if (mode != FERRY_HANDOFF_DROP && src->device != dst->device) {
    int ok = 0;
    FERRY_TRY(cudaDeviceCanAccessPeer(&ok, dst->device, src->device));
    if (!ok) return set_error("lru_handoff: device %d cannot read device %d", dst->device, src->device), FERRY_E_INVAL;
    const cudaError_t e = cudaDeviceEnablePeerAccess(src->device, 0);
    if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return cuda_status(e, "lru_handoff");
    cudaGetLastError();
  }
  const LaneRef s = lane_ref(mode == FERRY_HANDOFF_DROP ? dst : src), d = lane_ref(dst);
  cudaStream_t st = (cudaStream_t)stream;
  if (mode == FERRY_HANDOFF_OWNED)
    handoff_owned_kernel<<<(unsigned)((n + 31) / 32), 32, 0, st>>>(s, d, d_src_lanes, d_dst_lanes, n, bit, dst->err);
  else
    handoff_copy_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(s, d, d_src_lanes, d_dst_lanes, n,
                                                                   mode == FERRY_HANDOFF_CARRY, dst->err);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_lru_read_owned(ferry_lru* L, int lane, uint32_t* masks, int32_t* capacity) {
  int rc = group_check(L, "lru_read_owned");
  if (rc) return rc;
  if (lane < 0 || lane >= L->lanes || !masks || !capacity) return set_error("lru_read_owned: bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(L->device);
  FERRY_TRY(cudaDeviceSynchronize());
  FERRY_TRY(cudaMemcpy(masks, L->mask + (size_t)lane * L->cap, (size_t)L->cap * 4, cudaMemcpyDeviceToHost));
  FERRY_TRY(cudaMemcpy(capacity, L->lane_cap + lane, 4, cudaMemcpyDeviceToHost));
  return FERRY_OK;
}

}  // extern "C"
