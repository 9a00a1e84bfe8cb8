// lru.cu -- miss detection against the HBM page cache (exact LRU per lane).
//
// Semantics (same as the reference deque LRU, src/workloads/missstream.cuh:137-161,
// processed in selection order): a hit moves the page to MRU; a miss evicts
// the LRU front when the lane holds `cap` pages, then appends the page. Slot
// rule: a miss takes slot `size` while the lane is not full, else the slot of
// the page it evicts. Per-lane state in HBM: page_slot[ids] (page -> slot or
// -1), slot_page[cap], order[cap] (slots, LRU front first), size.
//
// One warp per lane. The warp loads the lane's order and slot table plus the
// selection's page-table entries into shared memory (coalesced / gathered,
// several loads per thread in flight). A selection without duplicates (the
// decode step) is resolved warp-parallel and exactly, with ballot scans over
// the selection and the old order (see the comment at that path). Otherwise
// lane 0 replays the selection sequentially on shared memory only -- O(1) per
// item using two lazily-deleted queues: the old order (pointer p, an entry is
// live while its slot has not been touched this step) and this step's touch
// list (pointer q, an entry is live while it is its slot's latest touch). The
// warp then writes back the compacted order, slot table, page-table deltas
// (evictions first, then final residents), and the miss list.
#include "common.cuh"

namespace ferry {
namespace {

struct LruArgs {
  int32_t* page_slot;
  int32_t* slot_page;
  int32_t* order;
  int32_t* size;
  int lanes, cap, ids;
  const int32_t* lane_ids;  // nullable: derive from req_ids
  const int32_t* req_ids;
  int lanes_per_req;
  const uint8_t* reset;  // nullable
  int n;
  const int32_t* sel;
  int k;
  const int32_t* n_sel;
  int distinct;
  uint8_t* is_miss;  // nullable
  int32_t* item_slot;
  int32_t* miss_page;
  int32_t* miss_slot;
  int32_t* n_miss;
  uint32_t* err;
  int warp_ints;  // shared-memory ints per warp
  const int32_t* lane_cap;  // nullable: per-lane capacity (<= cap), group lanes
  uint32_t* mask;           // nullable: per-slot owner bits, group lanes
  const uint32_t* bits;     // nullable: the owner bit of each row's touches
};

constexpr int kLoadBatch = 8;
constexpr int kLruCtaMinCap = 128;  // lanes with more slots take the CTA-per-lane kernel
constexpr int kLruRounds = 8;  // fixpoint rounds before the serial replay takes over

// Owner bits of a group lane after one row's touches (the reference's
// own_ masks, wla_multigpu.cuh:1937-1962): a page the row inserted (its
// latest insertion, the slot's final resident) owns `bit` alone -- the mask
// of the page it evicted was dropped with it -- and a page it hit gains `bit`.
// Every slot an eviction frees is refilled by the miss that caused it, so no
// other slot changes. Threads th, th + nth, ... of the caller.
__device__ __forceinline__ void update_owner_masks(uint32_t* mk, uint32_t bit, const int32_t* sel_s,
                                                   const int32_t* islot, const uint8_t* mflag, const int32_t* spg,
                                                   int n, int th, int nth) {
  for (int i = th; i < n; i += nth)
    if (mflag[i] && spg[islot[i]] == sel_s[i]) mk[islot[i]] = bit;
  if (nth == 32)
    __syncwarp();
  else
    __syncthreads();
  for (int i = th; i < n; i += nth)
    if (!mflag[i] && sel_s[i] >= 0 && islot[i] >= 0 && spg[islot[i]] == sel_s[i]) atomicOr(mk + islot[i], bit);
}

__global__ void __launch_bounds__(256) lru_kernel(LruArgs A) {
  extern __shared__ int32_t smem_i[];
  const int t = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int a = blockIdx.x * (blockDim.x >> 5) + warp;
  if (a >= A.n) return;
  const int C = A.cap, k = A.k;
  int32_t* old = smem_i + (size_t)warp * A.warp_ints;
  int32_t* spg = old + C;
  int32_t* seq = spg + C;
  int32_t* sel_s = seq + C;
  int32_t* islot = sel_s + k;
  int32_t* prev = islot + k;
  int32_t* newl = prev + k;
  int32_t* evict = newl + k;
  uint8_t* mflag = reinterpret_cast<uint8_t*>(evict + k);
  const uint32_t lt = (1u << t) - 1u;

  const int64_t lane = A.lane_ids ? (int64_t)A.lane_ids[a]
                                  : (int64_t)A.req_ids[a / A.lanes_per_req] * A.lanes_per_req +
                                        a % A.lanes_per_req;
  int n = A.n_sel[a];
  if (lane < 0 || lane >= A.lanes || n < 0 || n > k) {
    if (t == 0) {
      record_error(A.err, kErrRange);
      A.n_miss[a] = 0;
    }
    for (int i = t; i < k; i += 32) {
      A.item_slot[(size_t)a * k + i] = -1;
      if (A.is_miss) A.is_miss[(size_t)a * k + i] = 0;
    }
    return;
  }
  int32_t* ps = A.page_slot + lane * A.ids;
  int32_t* sp = A.slot_page + lane * C;
  int32_t* od = A.order + lane * C;
  const int Ce = A.lane_cap ? min(max(A.lane_cap[lane], 1), C) : C;  // this lane's capacity
  int sz0 = A.size[lane];
  if (sz0 < 0 || sz0 > Ce) {
    if (t == 0) record_error(A.err, kErrRange);
    sz0 = 0;
  }
  const bool rst = A.reset && A.reset[a];

  // the lane's tables arrive in batches of kLoadBatch loads per thread in
  // flight (the tables are usually cold in L2 right after the selection)
  bool corrupt = false;
  for (int j0 = t; j0 < C; j0 += 32 * kLoadBatch) {
    int vo[kLoadBatch], vs[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int j = j0 + 32 * u;
      vo[u] = j < sz0 ? __ldcg(od + j) : 0;
      vs[u] = j < sz0 ? __ldcg(sp + j) : -1;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int j = j0 + 32 * u;
      if (j < C) {
        if (j < sz0) {
          if (vo[u] < 0 || vo[u] >= C) {
            corrupt = true;
            vo[u] = 0;
          }
          old[j] = vo[u];
        }
        spg[j] = vs[u];
        seq[j] = -1;
      }
    }
  }
  if (__any_sync(0xffffffffu, corrupt) && t == 0) record_error(A.err, kErrRange);
  __syncwarp();
  if (rst) {
    for (int s = t; s < sz0; s += 32) {
      const int pg = spg[s];
      if (pg >= 0 && pg < A.ids) ps[pg] = -1;
      spg[s] = -1;
      if (A.mask) A.mask[lane * C + s] = 0u;
    }
    sz0 = 0;
  }
  __syncwarp();
  bool bad = false;
  for (int i0 = t; i0 < n; i0 += 32 * kLoadBatch) {
    int vx[kLoadBatch], vp[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + 32 * u;
      vx[u] = i < n ? __ldcg(A.sel + (size_t)a * k + i) : -1;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + 32 * u;
      if (i < n && (vx[u] < 0 || vx[u] >= A.ids)) {
        bad = true;
        vx[u] = -1;
      }
      vp[u] = (vx[u] >= 0 && !rst) ? __ldcg(ps + vx[u]) : -1;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + 32 * u;
      if (i < n) {
        sel_s[i] = vx[u];
        islot[i] = vp[u];
      }
    }
  }
  if (__any_sync(0xffffffffu, bad) && t == 0) record_error(A.err, kErrRange);
  __syncwarp();
  if (!A.distinct) {
    for (int i = t; i < n; i += 32) {
      const int x = sel_s[i];
      int pj = -1;
      if (x >= 0)
        for (int j = i - 1; j >= 0; --j)
          if (sel_s[j] == x) {
            pj = j;
            break;
          }
      prev[i] = pj;
    }
    __syncwarp();
  }

  int p = 0, qn = 0, nn = 0, sz = sz0, ne = 0;
  bool done = false;
  // ---- distinct selections, warp-parallel. Times are ranks among the valid
  // items. Once the f free slots are used a miss evicts: eviction e happens
  // at the miss of rank f + e and takes the first old-order entry neither
  // evicted nor touched before that miss (a touched entry moved to MRU). An
  // old page evicted before its own touch in this step misses at that touch;
  // K, the set of such pages, is found by iteration. With K's misses added,
  // eviction e takes the e-th old entry that is untouched or in K; a round
  // then adds every touched entry the evictions reach before its touch,
  // drops every K entry touched no later than the eviction reaching it, and
  // drops K entries no eviction reaches. A round that changes nothing leaves
  // an assignment that agrees with every step of the sequential process (by
  // induction over time), so a hit keeps its slot and the r-th miss takes
  // slot sz0 + r while free slots last, else the slot of eviction r - f.
  // Evictions that would reach this step's touch list, or no fixed point
  // within kLruRounds, run the serial replay instead.
  // seq[s] = touch time of old slot s; -1 untouched; -(time + 2) in K.
  if (A.distinct) {
    int nv = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
      const int i = i0 + t;
      const int x = i < n ? sel_s[i] : -1;
      const int s = x >= 0 ? islot[i] : -1;
      const bool valid = x >= 0, hit = valid && s >= 0 && s < C && spg[s] == x;
      const uint32_t mv = __ballot_sync(0xffffffffu, valid);
      if (i < n) {
        if (!valid) islot[i] = -1;
        if (hit) seq[s] = nv + __popc(mv & lt);  // touched this step
        mflag[i] = valid && !hit;                // a page not resident before the step
      }
      nv += __popc(mv);
    }
    __syncwarp();
    const int f = max(0, Ce - sz0);
    int nmiss = 0, E = 0, jlast = -1;  // jlast: old position of eviction E - 1
    int kcount = 0;                    // entries in K
    bool ok = false;
    for (int round = 0; round < kLruRounds; ++round) {
      nmiss = 0;  // miss ranks (prev) and times (newl, scratch until the touch list)
      int tv = 0;
      for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + t;
        const bool valid = i < n && sel_s[i] >= 0;
        const bool ism = valid && (mflag[i] || seq[islot[i]] <= -2);
        const uint32_t mv = __ballot_sync(0xffffffffu, valid), mm = __ballot_sync(0xffffffffu, ism);
        if (ism) {
          const int r = nmiss + __popc(mm & lt);
          prev[i] = r;
          newl[r] = tv + __popc(mv & lt);
        }
        nmiss += __popc(mm);
        tv += __popc(mv);
      }
      __syncwarp();
      E = max(0, nmiss - f);
      int ucount = 0, kseen = 0, kadd = 0, kdrop = 0;  // kseen, kadd, kdrop: this thread's
      jlast = -1;
      for (int j0 = 0; j0 < sz0 && ucount < E; j0 += 32) {  // warp-uniform
        const int j = j0 + t;
        const int sl = j < sz0 ? old[j] : 0;
        const int tt = j < sz0 ? seq[sl] : 0;
        const bool cand = j < sz0 && (tt == -1 || tt <= -2);  // untouched or in K
        const uint32_t mu = __ballot_sync(0xffffffffu, cand);
        const int u = ucount + __popc(mu & lt);  // evictions ahead of j
        if (j < sz0 && u < E) {
          const int me = newl[f + u];  // time of the miss making eviction u
          if (cand) {
            evict[u] = sl;
            if (u == E - 1) jlast = j;
            if (tt <= -2) {
              ++kseen;
              if (-tt - 2 <= me) {  // touched before its eviction: a hit after all
                seq[sl] = -tt - 2;
                ++kdrop;
              }
            }
          } else if (tt > me) {  // evicted before its touch: joins K
            seq[sl] = -tt - 2;
            ++kadd;
          }
        }
        ucount += __popc(mu);
      }
      if (__any_sync(0xffffffffu, ucount < E)) break;  // evictions would reach the touch list
      jlast = __reduce_max_sync(0xffffffffu, jlast);
      kseen = __reduce_add_sync(0xffffffffu, kseen);
      kadd = __reduce_add_sync(0xffffffffu, kadd);
      kdrop = __reduce_add_sync(0xffffffffu, kdrop);
      if (kseen < kcount) {  // K entries past the last eviction are not evicted
        int d = 0;
        for (int j = jlast + 1 + t; j < sz0; j += 32) {
          const int sl = old[j], tt = seq[sl];
          if (tt <= -2) {
            seq[sl] = -tt - 2;
            ++d;
          }
        }
        kdrop += __reduce_add_sync(0xffffffffu, d);
      }
      kcount += kadd - kdrop;
      __syncwarp();
      if (kadd == 0 && kdrop == 0) {
        ok = true;
        break;
      }
    }
    if (ok) {
      for (int i = t; i < n; i += 32)  // K pages miss at their touch
        if (sel_s[i] >= 0 && !mflag[i] && seq[islot[i]] <= -2) mflag[i] = 1;
      __syncwarp();
      for (int i = t; i < n; i += 32)
        if (mflag[i]) {
          const int r = prev[i];
          int sl;
          if (r < f) {
            sl = sz0 + r;
          } else {
            sl = evict[r - f];
            evict[r - f] = spg[sl];
          }
          islot[i] = sl;
        }
      __syncwarp();
      int nv2 = 0;
      for (int i0 = 0; i0 < n; i0 += 32) {  // touch list in selection order
        const int i = i0 + t;
        const bool valid = i < n && sel_s[i] >= 0;
        const uint32_t mv = __ballot_sync(0xffffffffu, valid);
        if (valid) {
          const int tr = nv2 + __popc(mv & lt), sl = islot[i];
          newl[tr] = sl;
          seq[sl] = tr;
          if (mflag[i]) spg[sl] = sel_s[i];
        }
        nv2 += __popc(mv);
      }
      p = E > 0 ? jlast + 1 : 0;  // old entries ahead of p are evicted or touched
      nn = nv;
      sz = sz0 + min(nmiss, f);
      ne = E;
      done = true;
    } else {
      for (int i = t; i < n; i += 32)  // undo the hit marks for the serial replay
        if (sel_s[i] >= 0 && !mflag[i]) seq[islot[i]] = -1;
    }
    __syncwarp();
  }

  // ---- sequential replay on shared memory (lane 0)
  if (t == 0 && !done) {
    for (int i = 0; i < n; ++i) {
      const int x = sel_s[i];
      if (x < 0) {
        islot[i] = -1;
        mflag[i] = 0;
        continue;
      }
      int s = (!A.distinct && prev[i] >= 0) ? islot[prev[i]] : islot[i];
      const bool hit = s >= 0 && s < C && spg[s] == x;
      if (hit) {
        seq[s] = nn;
        newl[nn++] = s;
        islot[i] = s;
        mflag[i] = 0;
      } else {
        if (sz >= Ce) {
          while (p < sz0 && seq[old[p]] != -1) ++p;
          if (p < sz0) {
            s = old[p++];
          } else {
            while (qn < nn - 1 && seq[newl[qn]] != qn) ++qn;
            s = newl[qn++];
          }
          evict[ne++] = spg[s];
        } else {
          s = sz++;
        }
        spg[s] = x;
        seq[s] = nn;
        newl[nn++] = s;
        islot[i] = s;
        mflag[i] = 1;
      }
    }
  }
  __syncwarp();
  p = __shfl_sync(0xffffffffu, p, 0);
  qn = __shfl_sync(0xffffffffu, qn, 0);
  nn = __shfl_sync(0xffffffffu, nn, 0);
  sz = __shfl_sync(0xffffffffu, sz, 0);
  ne = __shfl_sync(0xffffffffu, ne, 0);

  // ---- new LRU order: live old entries, then live touch-list entries
  int outp = 0;
  for (int j0 = p; j0 < sz0; j0 += 32) {
    const int j = j0 + t;
    const bool live = j < sz0 && seq[old[j]] == -1;
    const uint32_t m = __ballot_sync(0xffffffffu, live);
    if (live) od[outp + __popc(m & lt)] = old[j];
    outp += __popc(m);
  }
  for (int j0 = qn; j0 < nn; j0 += 32) {
    const int j = j0 + t;
    const bool live = j < nn && seq[newl[j]] == j;
    const uint32_t m = __ballot_sync(0xffffffffu, live);
    if (live) od[outp + __popc(m & lt)] = newl[j];
    outp += __popc(m);
  }
  if (t == 0) A.size[lane] = sz;
  for (int i = t; i < n; i += 32)
    if (mflag[i]) sp[islot[i]] = spg[islot[i]];
  // page table: evictions first, then the final residents among the misses
  for (int e = t; e < ne; e += 32) {
    const int v = evict[e];
    if (v >= 0 && v < A.ids) ps[v] = -1;
  }
  __syncwarp();
  for (int i = t; i < n; i += 32)
    if (mflag[i]) {
      const int s = islot[i];
      if (spg[s] == sel_s[i]) ps[sel_s[i]] = s;
    }
  if (A.mask) update_owner_masks(A.mask + lane * C, A.bits ? A.bits[a] : 0u, sel_s, islot, mflag, spg, n, t, 32);

  // ---- outputs
  int nm = 0;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + t;
    const bool f = i < n && mflag[i];
    const uint32_t m = __ballot_sync(0xffffffffu, f);
    if (f) {
      const int r = nm + __popc(m & lt);
      A.miss_page[(size_t)a * k + r] = sel_s[i];
      A.miss_slot[(size_t)a * k + r] = islot[i];
    }
    nm += __popc(m);
  }
  for (int i = t; i < k; i += 32) {
    A.item_slot[(size_t)a * k + i] = i < n ? islot[i] : -1;
    if (A.is_miss) A.is_miss[(size_t)a * k + i] = i < n ? mflag[i] : 0;
  }
  if (t == 0) A.n_miss[a] = nm;
}


// ---------------------------------------------------------------------------
// CTA-per-lane variant for distinct selections (the decode step) on lanes of
// more than kLruCtaMinCap slots. The warp kernel above spends its time in one
// warp's dependent chain of chunked ballot scans (~9k instructions per lane at
// 1229 slots / 512 selected); here the lane's four warps share every loop:
// each chunk of 128 items is ranked by one block-ordered scan (ballot counts
// per warp through shared memory, one barrier), so the chain is ~4x shorter.
// Same algorithm and same results as the warp kernel's parallel path, with
// the same serial replay (thread 0) when it gives up.
#ifndef FERRY_LRU_CTA_WARPS
#define FERRY_LRU_CTA_WARPS 4
#endif
constexpr int kLruCtaWarps = FERRY_LRU_CTA_WARPS;  // warps sharing a lane (build-time tunable)
constexpr int kLruCtaThreads = kLruCtaWarps * 32;

// Exclusive ranks of two flags over one chunk (item order = thread order) and
// the chunk totals. One barrier; the double buffer lets the next call write
// while no thread can still be reading the same half (it passed this barrier).
__device__ __forceinline__ void cta_scan2(bool f0, bool f1, uint32_t (*buf)[2][kLruCtaWarps], int& par, int& r0,
                                          int& r1, int& t0, int& t1) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t m0 = __ballot_sync(0xffffffffu, f0), m1 = __ballot_sync(0xffffffffu, f1);
  if (lane == 0) {
    buf[par][0][warp] = __popc(m0);
    buf[par][1][warp] = __popc(m1);
  }
  __syncthreads();
  int b0 = 0, b1 = 0;
  t0 = t1 = 0;
#pragma unroll
  for (int w = 0; w < kLruCtaWarps; ++w) {
    const int c0 = (int)buf[par][0][w], c1 = (int)buf[par][1][w];
    if (w < warp) {
      b0 += c0;
      b1 += c1;
    }
    t0 += c0;
    t1 += c1;
  }
  const uint32_t lt = (1u << lane) - 1u;
  r0 = b0 + __popc(m0 & lt);
  r1 = b1 + __popc(m1 & lt);
  par ^= 1;
}

// Block sum and max (one barrier each, double-buffered like cta_scan2).
__device__ __forceinline__ int cta_sum(int v, int (*buf)[kLruCtaWarps], int& par) {
  v = __reduce_add_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) buf[par][threadIdx.x >> 5] = v;
  __syncthreads();
  int s = 0;
#pragma unroll
  for (int w = 0; w < kLruCtaWarps; ++w) s += buf[par][w];
  par ^= 1;
  return s;
}
__device__ __forceinline__ int cta_max(int v, int (*buf)[kLruCtaWarps], int& par) {
  v = __reduce_max_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) buf[par][threadIdx.x >> 5] = v;
  __syncthreads();
  int s = buf[par][0];
#pragma unroll
  for (int w = 1; w < kLruCtaWarps; ++w) s = max(s, buf[par][w]);
  par ^= 1;
  return s;
}

__global__ void __launch_bounds__(kLruCtaThreads) lru_cta_kernel(LruArgs A) {
  extern __shared__ int32_t smem_i[];
  __shared__ uint32_t sbuf[2][2][kLruCtaWarps];
  __shared__ int rbuf[2][kLruCtaWarps];
  __shared__ int s_state[5];
  const int tid = threadIdx.x, t = tid & 31;
  const int a = blockIdx.x;
  if (a >= A.n) return;
  const int C = A.cap, k = A.k;
  int32_t* old = smem_i;
  int32_t* spg = old + C;
  int32_t* seq = spg + C;
  int32_t* sel_s = seq + C;
  int32_t* islot = sel_s + k;
  int32_t* prev = islot + k;
  int32_t* newl = prev + k;
  int32_t* evict = newl + k;
  uint8_t* mflag = reinterpret_cast<uint8_t*>(evict + k);
  int spar = 0, rpar = 0;

  const int64_t lane = A.lane_ids ? (int64_t)A.lane_ids[a]
                                  : (int64_t)A.req_ids[a / A.lanes_per_req] * A.lanes_per_req +
                                        a % A.lanes_per_req;
  const int n = A.n_sel[a];
  if (lane < 0 || lane >= A.lanes || n < 0 || n > k) {
    if (tid == 0) {
      record_error(A.err, kErrRange);
      A.n_miss[a] = 0;
    }
    for (int i = tid; i < k; i += kLruCtaThreads) {
      A.item_slot[(size_t)a * k + i] = -1;
      if (A.is_miss) A.is_miss[(size_t)a * k + i] = 0;
    }
    return;
  }
  int32_t* ps = A.page_slot + lane * A.ids;
  int32_t* sp = A.slot_page + lane * C;
  int32_t* od = A.order + lane * C;
  const int Ce = A.lane_cap ? min(max(A.lane_cap[lane], 1), C) : C;  // this lane's capacity
  int sz0 = A.size[lane];
  if (sz0 < 0 || sz0 > Ce) {
    if (tid == 0) record_error(A.err, kErrRange);
    sz0 = 0;
  }
  const bool rst = A.reset && A.reset[a];

  // the lane's tables, kLoadBatch loads per thread in flight
  bool corrupt = false;
  for (int j0 = tid; j0 < C; j0 += kLruCtaThreads * kLoadBatch) {
    int vo[kLoadBatch], vs[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int j = j0 + kLruCtaThreads * u;
      vo[u] = j < sz0 ? __ldcg(od + j) : 0;
      vs[u] = j < sz0 ? __ldcg(sp + j) : -1;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int j = j0 + kLruCtaThreads * u;
      if (j < C) {
        if (j < sz0) {
          if (vo[u] < 0 || vo[u] >= C) {
            corrupt = true;
            vo[u] = 0;
          }
          old[j] = vo[u];
        }
        spg[j] = vs[u];
        seq[j] = -1;
      }
    }
  }
  if (__syncthreads_or(corrupt) && tid == 0) record_error(A.err, kErrRange);
  if (rst) {
    for (int s = tid; s < sz0; s += kLruCtaThreads) {
      const int pg = spg[s];
      if (pg >= 0 && pg < A.ids) ps[pg] = -1;
      spg[s] = -1;
      if (A.mask) A.mask[lane * C + s] = 0u;
    }
    sz0 = 0;
  }
  __syncthreads();
  bool bad = false;
  for (int i0 = tid; i0 < n; i0 += kLruCtaThreads * kLoadBatch) {
    int vx[kLoadBatch], vp[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + kLruCtaThreads * u;
      vx[u] = i < n ? __ldcg(A.sel + (size_t)a * k + i) : -1;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + kLruCtaThreads * u;
      if (i < n && (vx[u] < 0 || vx[u] >= A.ids)) {
        bad = true;
        vx[u] = -1;
      }
      vp[u] = (vx[u] >= 0 && !rst) ? __ldcg(ps + vx[u]) : -1;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + kLruCtaThreads * u;
      if (i < n) {
        sel_s[i] = vx[u];
        islot[i] = vp[u];
      }
    }
  }
  if (__syncthreads_or(bad) && tid == 0) record_error(A.err, kErrRange);

  // ---- the parallel exact path (see lru_kernel); seq[s] = touch time of old
  // slot s, -1 untouched, -(time + 2) in K
  int p = 0, qn = 0, nn = 0, sz = sz0, ne = 0;
  bool done = false;
  int nv = 0;
  for (int i0 = 0; i0 < n; i0 += kLruCtaThreads) {
    const int i = i0 + tid;
    const int x = i < n ? sel_s[i] : -1;
    const int s = x >= 0 ? islot[i] : -1;
    const bool valid = x >= 0, hit = valid && s >= 0 && s < C && spg[s] == x;
    int rv, r1, tv, t1;
    cta_scan2(valid, false, sbuf, spar, rv, r1, tv, t1);
    if (i < n) {
      if (!valid) islot[i] = -1;
      if (hit) seq[s] = nv + rv;
      mflag[i] = valid && !hit;
    }
    nv += tv;
  }
  __syncthreads();
  const int f = max(0, Ce - sz0);
  int nmiss = 0, E = 0, jlast = -1, kcount = 0;
  bool ok = false;
  for (int round = 0; round < kLruRounds; ++round) {
    nmiss = 0;
    int tvs = 0;
    for (int i0 = 0; i0 < n; i0 += kLruCtaThreads) {
      const int i = i0 + tid;
      const bool valid = i < n && sel_s[i] >= 0;
      const bool ism = valid && (mflag[i] || seq[islot[i]] <= -2);
      int rv, rm, tv, tm;
      cta_scan2(valid, ism, sbuf, spar, rv, rm, tv, tm);
      if (ism) {
        const int r = nmiss + rm;
        prev[i] = r;
        newl[r] = tvs + rv;
      }
      nmiss += tm;
      tvs += tv;
    }
    __syncthreads();
    E = max(0, nmiss - f);
    int ucount = 0, kseen = 0, kadd = 0, kdrop = 0, jl = -1;
    for (int j0 = 0; j0 < sz0 && ucount < E; j0 += kLruCtaThreads) {  // block-uniform
      const int j = j0 + tid;
      const int sl = j < sz0 ? old[j] : 0;
      const int tt = j < sz0 ? seq[sl] : 0;
      const bool cand = j < sz0 && (tt == -1 || tt <= -2);  // untouched or in K
      int rc, r1, tc, t1;
      cta_scan2(cand, false, sbuf, spar, rc, r1, tc, t1);
      const int u = ucount + rc;  // evictions ahead of j
      if (j < sz0 && u < E) {
        const int me = newl[f + u];  // time of the miss making eviction u
        if (cand) {
          evict[u] = sl;
          if (u == E - 1) jl = j;
          if (tt <= -2) {
            ++kseen;
            if (-tt - 2 <= me) {  // touched before its eviction: a hit after all
              seq[sl] = -tt - 2;
              ++kdrop;
            }
          }
        } else if (tt > me) {  // evicted before its touch: joins K
          seq[sl] = -tt - 2;
          ++kadd;
        }
      }
      ucount += tc;
    }
    if (ucount < E) break;  // evictions would reach the touch list (block-uniform)
    jlast = cta_max(jl, rbuf, rpar);
    kseen = cta_sum(kseen, rbuf, rpar);
    kadd = cta_sum(kadd, rbuf, rpar);
    kdrop = cta_sum(kdrop, rbuf, rpar);
    if (kseen < kcount) {  // K entries past the last eviction are not evicted
      int d = 0;
      for (int j = jlast + 1 + tid; j < sz0; j += kLruCtaThreads) {
        const int sl = old[j], tt = seq[sl];
        if (tt <= -2) {
          seq[sl] = -tt - 2;
          ++d;
        }
      }
      kdrop += cta_sum(d, rbuf, rpar);
    }
    kcount += kadd - kdrop;
    __syncthreads();
    if (kadd == 0 && kdrop == 0) {
      ok = true;
      break;
    }
  }
  __syncthreads();
  if (ok) {
    for (int i = tid; i < n; i += kLruCtaThreads)  // K pages miss at their touch
      if (sel_s[i] >= 0 && !mflag[i] && seq[islot[i]] <= -2) mflag[i] = 1;
    __syncthreads();
    for (int i = tid; i < n; i += kLruCtaThreads)
      if (mflag[i]) {
        const int r = prev[i];
        int sl;
        if (r < f) {
          sl = sz0 + r;
        } else {
          sl = evict[r - f];
          evict[r - f] = spg[sl];
        }
        islot[i] = sl;
      }
    __syncthreads();
    int nv2 = 0;
    for (int i0 = 0; i0 < n; i0 += kLruCtaThreads) {  // touch list in selection order
      const int i = i0 + tid;
      const bool valid = i < n && sel_s[i] >= 0;
      int rv, r1, tv, t1;
      cta_scan2(valid, false, sbuf, spar, rv, r1, tv, t1);
      if (valid) {
        const int tr = nv2 + rv, sl = islot[i];
        newl[tr] = sl;
        seq[sl] = tr;
        if (mflag[i]) spg[sl] = sel_s[i];
      }
      nv2 += tv;
    }
    p = E > 0 ? jlast + 1 : 0;
    nn = nv;
    sz = sz0 + min(nmiss, f);
    ne = E;
    done = true;
  } else {
    for (int i = tid; i < n; i += kLruCtaThreads)  // undo the hit marks for the serial replay
      if (sel_s[i] >= 0 && !mflag[i]) seq[islot[i]] = -1;
  }
  __syncthreads();

  // ---- sequential replay on shared memory (thread 0), as in lru_kernel
  if (tid == 0 && !done) {
    for (int i = 0; i < n; ++i) {
      const int x = sel_s[i];
      if (x < 0) {
        islot[i] = -1;
        mflag[i] = 0;
        continue;
      }
      int s = islot[i];
      const bool hit = s >= 0 && s < C && spg[s] == x;
      if (hit) {
        seq[s] = nn;
        newl[nn++] = s;
        islot[i] = s;
        mflag[i] = 0;
      } else {
        if (sz >= Ce) {
          while (p < sz0 && seq[old[p]] != -1) ++p;
          if (p < sz0) {
            s = old[p++];
          } else {
            while (qn < nn - 1 && seq[newl[qn]] != qn) ++qn;
            s = newl[qn++];
          }
          evict[ne++] = spg[s];
        } else {
          s = sz++;
        }
        spg[s] = x;
        seq[s] = nn;
        newl[nn++] = s;
        islot[i] = s;
        mflag[i] = 1;
      }
    }
  }
  if (tid == 0) {
    s_state[0] = p;
    s_state[1] = qn;
    s_state[2] = nn;
    s_state[3] = sz;
    s_state[4] = ne;
  }
  __syncthreads();
  p = s_state[0];
  qn = s_state[1];
  nn = s_state[2];
  sz = s_state[3];
  ne = s_state[4];

  // ---- new LRU order: live old entries, then live touch-list entries
  int outp = 0;
  for (int j0 = p; j0 < sz0; j0 += kLruCtaThreads) {
    const int j = j0 + tid;
    const bool live = j < sz0 && seq[old[j]] == -1;
    int rl, r1, tl, t1;
    cta_scan2(live, false, sbuf, spar, rl, r1, tl, t1);
    if (live) od[outp + rl] = old[j];
    outp += tl;
  }
  for (int j0 = qn; j0 < nn; j0 += kLruCtaThreads) {
    const int j = j0 + tid;
    const bool live = j < nn && seq[newl[j]] == j;
    int rl, r1, tl, t1;
    cta_scan2(live, false, sbuf, spar, rl, r1, tl, t1);
    if (live) od[outp + rl] = newl[j];
    outp += tl;
  }
  if (tid == 0) A.size[lane] = sz;
  for (int i = tid; i < n; i += kLruCtaThreads)
    if (mflag[i]) sp[islot[i]] = spg[islot[i]];
  // page table: evictions first, then the final residents among the misses
  for (int e = tid; e < ne; e += kLruCtaThreads) {
    const int v = evict[e];
    if (v >= 0 && v < A.ids) ps[v] = -1;
  }
  __syncthreads();
  for (int i = tid; i < n; i += kLruCtaThreads)
    if (mflag[i]) {
      const int s = islot[i];
      if (spg[s] == sel_s[i]) ps[sel_s[i]] = s;
    }
  if (A.mask) update_owner_masks(A.mask + lane * C, A.bits ? A.bits[a] : 0u, sel_s, islot, mflag, spg, n, tid,
                                 kLruCtaThreads);

  // ---- outputs
  int nm = 0;
  for (int i0 = 0; i0 < n; i0 += kLruCtaThreads) {
    const int i = i0 + tid;
    const bool fl = i < n && mflag[i];
    int rm, r1, tm, t1;
    cta_scan2(fl, false, sbuf, spar, rm, r1, tm, t1);
    if (fl) {
      const int r = nm + rm;
      A.miss_page[(size_t)a * k + r] = sel_s[i];
      A.miss_slot[(size_t)a * k + r] = islot[i];
    }
    nm += tm;
  }
  for (int i = tid; i < k; i += kLruCtaThreads) {
    A.item_slot[(size_t)a * k + i] = i < n ? islot[i] : -1;
    if (A.is_miss) A.is_miss[(size_t)a * k + i] = i < n ? mflag[i] : 0;
  }
  if (tid == 0) A.n_miss[a] = nm;
}

// Empty every lane of the listed requests and record their context length
// (ctx_pages holds the full pages of each request, then, R entries later, the
// tokens of its partial last page).
__global__ void __launch_bounds__(256) lru_reset_kernel(int32_t* page_slot, int32_t* slot_page,
                                                        int32_t* size, int lanes, int cap, int ids,
                                                        const int32_t* req_ids, int n,
                                                        int lanes_per_req, const int32_t* n_pages,
                                                        int32_t* ctx_pages, int max_pages,
                                                        const int64_t* pool_base, int64_t* req_base,
                                                        int max_requests, uint32_t* err) {
  const int t = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= n * lanes_per_req) return;
  const int i = w / lanes_per_req;
  const int64_t lane = (int64_t)req_ids[i] * lanes_per_req + w % lanes_per_req;
  if (lane < 0 || lane >= lanes) {
    if (t == 0) record_error(err, kErrRange);
    return;
  }
  int sz = size[lane];
  if (sz < 0 || sz > cap) sz = cap;
  int32_t* ps = page_slot + lane * ids;
  const int32_t* sp = slot_page + lane * cap;
  for (int s = t; s < sz; s += 32) {
    const int pg = sp[s];
    if (pg >= 0 && pg < ids) ps[pg] = -1;
  }
  if (t == 0) {
    size[lane] = 0;
    if (w % lanes_per_req == 0 && ctx_pages) {
      int np = n_pages[i];
      if (np < 0 || np > max_pages) {
        record_error(err, kErrRange);
        np = np < 0 ? 0 : max_pages;
      }
      ctx_pages[req_ids[i]] = np;
      ctx_pages[max_requests + req_ids[i]] = 0;  // no partial page yet
      if (req_base)
        req_base[req_ids[i]] = pool_base ? pool_base[i]
                                         : (int64_t)req_ids[i] * lanes_per_req * (int64_t)max_pages;
    }
  }
}

}  // namespace

int launch_lru(const ferry_lru* L, cudaStream_t st, const int32_t* lane_ids,
               const int32_t* req_ids, int lanes_per_req, const uint8_t* reset, int n,
               const int32_t* sel, int k, const int32_t* n_sel, int distinct, uint8_t* is_miss,
               int32_t* item_slot, int32_t* miss_page, int32_t* miss_slot, int32_t* n_miss,
               const uint32_t* bits) {
  if (n <= 0) return FERRY_OK;
  if (k <= 0 || !sel || !n_sel || !item_slot || !miss_page || !miss_slot || !n_miss) {
    set_error("lru: bad arguments");
    return FERRY_E_INVAL;
  }
  LruArgs A{};
  A.page_slot = L->page_slot;
  A.slot_page = L->slot_page;
  A.order = L->order;
  A.size = L->size;
  A.lanes = L->lanes;
  A.cap = L->cap;
  A.ids = L->ids;
  A.lane_ids = lane_ids;
  A.req_ids = req_ids;
  A.lanes_per_req = lanes_per_req;
  A.reset = reset;
  A.n = n;
  A.sel = sel;
  A.k = k;
  A.n_sel = n_sel;
  A.distinct = distinct;
  A.is_miss = is_miss;
  A.item_slot = item_slot;
  A.miss_page = miss_page;
  A.miss_slot = miss_slot;
  A.n_miss = n_miss;
  A.err = L->err;
  A.lane_cap = L->lane_cap;
  A.mask = L->mask;
  A.bits = bits;
  // old, spg, seq (cap each) + sel, islot, prev, newl, evict (k each) + k flag bytes
  A.warp_ints = lru_lane_ints(L->cap, k);
  const size_t per_warp = (size_t)A.warp_ints * 4;
  if (distinct && L->cap > kLruCtaMinCap && per_warp <= kLruLaneSmemMax) {
    // a CTA per lane (decode steps on long lanes)
    if (per_warp > 48 * 1024)
      FERRY_TRY(cudaFuncSetAttribute(lru_cta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)per_warp));
    lru_cta_kernel<<<(unsigned)n, kLruCtaThreads, per_warp, st>>>(A);
    FERRY_TRY(cudaGetLastError());
    return FERRY_OK;
  }
  int warps = (int)std::min<size_t>(8, std::max<size_t>(1, (96 * 1024) / per_warp));
  const size_t smem = per_warp * warps;
  if (smem > kLruLaneSmemMax) {
    set_error("lru: capacity %d / k %d need %zu bytes of shared memory per lane", L->cap, k,
              per_warp);
    return FERRY_E_INVAL;
  }
  if (smem > 48 * 1024)
    FERRY_TRY(cudaFuncSetAttribute(lru_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem));
  const unsigned grid = (unsigned)((n + warps - 1) / warps);
  lru_kernel<<<grid, warps * 32, smem, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_lru_reset(const ferry_lru* L, cudaStream_t st, const int32_t* req_ids, int n,
                     int lanes_per_req, const int32_t* n_pages, int32_t* ctx_pages,
                     const int64_t* pool_base, int64_t* req_base) {
  if (n <= 0) return FERRY_OK;
  const int warps = n * lanes_per_req;
  lru_reset_kernel<<<(warps + 7) / 8, 256, 0, st>>>(L->page_slot, L->slot_page, L->size, L->lanes,
                                                    L->cap, L->ids, req_ids, n, lanes_per_req,
                                                    n_pages, ctx_pages, L->ids, pool_base, req_base,
                                                    L->lanes / lanes_per_req, L->err);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

}  // namespace ferry
