// ferry_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// CPU restatement of the reference's sparse KV-cache miss-stream decode path
// (clearleo126/ferry) and of the per-kv-head page model this repository builds.
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
// arm load this library, and only as the checker or the timed CPU baseline.
// The product (ferry_b200/libferry_cuda.so) never links or calls it.
//
// Parity pins:
//  * replay_miss_stream / prefix sharing / mode-C gather plan are pinned against
//    the reference's own golden numbers (results/realtrace_20261021.md:19,
//    results/wla_7rep_20260930/wla_bursty_balanced_r1.log:3-9,
//    results/wla_pathdep_20261018/base_s42.log:12,14) and against the reference
//    headers compiled into oracle/_ref (ref_driver.cpp).
//  * The page-table LRU (orc_lru_*) reduces to the reference's deque LRU
//    (src/workloads/missstream.cuh:137-161) for the hit/miss sequence; the slot
//    rule and per-head keying are this build's own definitions.
//  * Selection (mean-key summary, q.summary, top-k) follows the benchmark
//    definition; the reference's only scoring code is torch
//    (tools/capture_miss_trace.py:128-159) and pins nothing bit-exactly, so
//    selection and attention parity are "unpinned" by any reference vector.
//
// Build: oracle/Makefile, with -ffp-contract=off so every fp32 operation below
// is exactly the one written.

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <deque>
#include <random>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

constexpr int kHeadDim = 128;
constexpr int kPageTokens = 16;
constexpr int kUnitElems = 2 * kPageTokens * kHeadDim;  // K[16][128] then V[16][128]

inline float h2f(uint16_t h) {
  _Float16 v;
  std::memcpy(&v, &h, 2);
  return (float)v;
}
inline uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;  // IEEE round-to-nearest-even, same as __float2half_rn
  uint16_t h;
  std::memcpy(&h, &v, 2);
  return h;
}

// splitmix64 finaliser (Steele, Lea, Flood 2014) -- the counter hash behind the
// procedural KV generator; the CUDA generator uses the identical integer steps.
inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace

extern "C" {

// ===========================================================================
// 1. Reference synthetic miss stream -- restates replay_miss_stream
//    (src/workloads/missstream.cuh:104-170): seeded mt19937_64, 66% reuse of the
//    previous step's selection (:127-128), else uniform over 64+8s blocks
//    (:118, :130); per-(req,layer) deque LRU of capacity hot_blocks (:137-161).
// ===========================================================================
struct OrcMissSpec {
  int num_requests, num_layers, steps, sel_blocks, hot_blocks, kv_heads, head_dim;
  int prefix_group, prefix_steps, cap_mode;
  uint64_t seed;
};

static inline uint64_t c4_bytes(const OrcMissSpec* sp) {
  // missstream.cuh:66: 4 tokens x (K,V) x kv_heads x head_dim x 2 B
  return (uint64_t)4 * 2 * sp->kv_heads * sp->head_dim * 2;
}

// blocks/is_miss: R*S*L*sel entries in event order (r, s, l, k), as the
// reference pushes them (missstream.cuh:116-140). totals = {selects, misses,
// miss_bytes}.
int orc_replay_miss_stream(const OrcMissSpec* sp, int64_t* blocks, uint8_t* is_miss,
                           uint64_t* totals) {
  const int R = sp->num_requests, L = sp->num_layers, S = sp->steps, G = sp->sel_blocks;
  std::mt19937_64 rng(sp->seed);
  std::vector<std::deque<uint64_t>> dq((size_t)R * L);
  std::vector<std::unordered_set<uint64_t>> st((size_t)R * L);
  std::vector<std::vector<uint64_t>> prev((size_t)R * L);
  uint64_t n_sel = 0, n_miss = 0, bytes = 0;
  size_t ev = 0;
  std::vector<uint64_t> sel;
  for (int r = 0; r < R; ++r)
    for (int s = 0; s < S; ++s) {
      const uint64_t hist = 64 + (uint64_t)s * 8;
      for (int l = 0; l < L; ++l) {
        auto& d = dq[(size_t)r * L + l];
        auto& set = st[(size_t)r * L + l];
        auto& pv = prev[(size_t)r * L + l];
        sel.clear();
        for (int i = 0; i < G; ++i) {
          uint64_t b;
          if (!pv.empty() && (double)(rng() % 1000) / 1000.0 < 0.66)
            b = pv[rng() % pv.size()];
          else
            b = rng() % hist;
          sel.push_back(b);
        }
        for (uint64_t b : sel) {
          ++n_sel;
          const bool hit = set.count(b) > 0;
          blocks[ev] = (int64_t)b;
          is_miss[ev] = hit ? 0 : 1;
          ++ev;
          if (hit) {
            d.erase(std::find(d.begin(), d.end(), b));
            d.push_back(b);
          } else {
            ++n_miss;
            bytes += c4_bytes(sp);
            if ((int)d.size() >= sp->hot_blocks) {
              set.erase(d.front());
              d.pop_front();
            }
            d.push_back(b);
            set.insert(b);
          }
        }
        pv = sel;
      }
    }
  totals[0] = n_sel;
  totals[1] = n_miss;
  totals[2] = bytes;
  return 0;
}

// Prefix sharing + group-LRU statistics -- restates wla_apply_prefix_sharing
// and wla_recompute_stats (src/runtime/wla_multigpu.cuh:359-372, :376-417) and
// wla_group_cap (src/workloads/missstream.cuh:91-94). Rewrites blocks in
// place; totals as above.
int orc_prefix_share_stats(const OrcMissSpec* sp, int64_t* blocks, uint64_t* totals) {
  const int R = sp->num_requests, L = sp->num_layers, S = sp->steps, G = sp->sel_blocks;
  if (sp->prefix_group <= 1) return -1;
  const size_t per_rs = (size_t)L * G;
  if (sp->prefix_steps > 0)
    for (int r = 0; r < R; ++r) {
      const int head = (r / sp->prefix_group) * sp->prefix_group;
      if (r == head) continue;
      for (int s = 0; s < std::min(sp->prefix_steps, S); ++s)
        std::memcpy(&blocks[((size_t)r * S + s) * per_rs],
                    &blocks[((size_t)head * S + s) * per_rs], per_rs * sizeof(int64_t));
    }
  const int ngrp = (R + sp->prefix_group - 1) / sp->prefix_group;
  std::vector<std::deque<int64_t>> dq((size_t)ngrp * L);
  std::vector<std::unordered_set<int64_t>> st((size_t)ngrp * L);
  uint64_t n_sel = 0, n_miss = 0, bytes = 0;
  for (int r = 0; r < R; ++r) {
    const int grp = r / sp->prefix_group;
    const int members = std::min(sp->prefix_group, R - grp * sp->prefix_group);
    const int cap = sp->cap_mode != 1 ? sp->hot_blocks
                                      : sp->hot_blocks * (members > 0 ? members : 1);
    for (int s = 0; s < S; ++s)
      for (int l = 0; l < L; ++l) {
        auto& d = dq[(size_t)grp * L + l];
        auto& set = st[(size_t)grp * L + l];
        for (int k = 0; k < G; ++k) {
          const int64_t b = blocks[((size_t)r * S + s) * per_rs + (size_t)l * G + k];
          ++n_sel;
          if (set.count(b)) {
            d.erase(std::find(d.begin(), d.end(), b));
            d.push_back(b);
          } else {
            ++n_miss;
            bytes += c4_bytes(sp);
            while ((int)d.size() >= cap) {
              set.erase(d.front());
              d.pop_front();
            }
            d.push_back(b);
            set.insert(b);
          }
        }
      }
  }
  totals[0] = n_sel;
  totals[1] = n_miss;
  totals[2] = bytes;
  return 0;
}

// AdaptiveBatchPolicy::choose_mb (src/runtime/adaptive_batch.cuh:31-36).
double orc_choose_mb(double pending_mb, double min_mb, double max_mb, double target) {
  double g = pending_mb / target;
  g = std::max(g, min_mb);
  g = std::min(g, max_mb);
  return g;
}

// Mode-C gather plan of one (request, step) -- restates exec_step mode C
// (src/runtime/wla_multigpu.cuh:2527-2604; 1-GPU twin
// src/workloads/kv_exec.cuh:187-292): sort misses by (layer, block), unique,
// adaptive batches, merge runs of consecutive blocks that do not cross the
// direct-mapped slot wrap. Returns segments (refill_events) and bytes.
int orc_gather_plan(const int* layers, const int64_t* blocks, int n, int hot_blocks,
                    uint64_t c4, uint64_t* segs_out, uint64_t* bytes_out) {
  std::vector<std::pair<int, int64_t>> m(n);
  for (int i = 0; i < n; ++i) m[i] = {layers[i], blocks[i]};
  std::sort(m.begin(), m.end());
  m.erase(std::unique(m.begin(), m.end()), m.end());
  uint64_t segs = 0, bytes = 0;
  size_t i0 = 0;
  while (i0 < m.size()) {
    const double pending_mb = (double)(m.size() - i0) * c4 / (1 << 20);
    const double gmb = orc_choose_mb(pending_mb, 1.0, 4.0, 4.0);
    const size_t take = std::min<size_t>(
        std::max<size_t>((size_t)(gmb * (1 << 20) / c4), 1), m.size() - i0);
    size_t k = 0;
    while (k < take) {
      const auto& m0 = m[i0 + k];
      size_t run = 1;
      while (k + run < take && m[i0 + k + run].first == m0.first &&
             m[i0 + k + run].second == m0.second + (int64_t)run)
        ++run;
      bytes += run * c4;  // wrapped runs are split per block; bytes are equal
      ++segs;
      k += run;
    }
    i0 += take;
  }
  *segs_out = segs;
  *bytes_out = bytes;
  return 0;
}

// ===========================================================================
// 2. Page-table LRU lanes (this build's miss-detect definition).
//    A lane is one (request, layer, kv_head) -- or one (request, layer) when
//    replaying the reference stream. Hit/miss sequence = the reference deque
//    LRU (missstream.cuh:137-161) processed in selection order: a hit moves the
//    page to MRU; a miss evicts the LRU front when size >= capacity, then
//    appends. Slot rule (new): a miss takes slot `size` while the cache is not
//    full, else the slot of the page it evicts; the page table maps page->slot.
// ===========================================================================
struct OrcLru {
  int lanes, cap, ids;
  std::vector<int32_t> page_slot;            // lanes*ids, -1 = absent
  std::vector<std::deque<int32_t>> order;    // LRU front .. MRU back (page ids)
  // group lanes: capacity per lane and owner masks keyed by page id (the
  // reference's own_ maps, src/runtime/wla_multigpu.cuh:1872-1916); empty
  // until orc_lru_group_enable
  std::vector<int> lane_cap;
  std::vector<std::unordered_map<int32_t, uint32_t>> own;
};

void* orc_lru_create(int lanes, int capacity, int ids) {
  auto* h = new OrcLru;
  h->lanes = lanes;
  h->cap = capacity;
  h->ids = ids;
  h->page_slot.assign((size_t)lanes * ids, -1);
  h->order.resize(lanes);
  return h;
}
void orc_lru_destroy(void* p) { delete (OrcLru*)p; }

// One step for n_active lanes. sel is n_active x k (row stride k); n_sel[i]
// items of row i are valid. reset[i] != 0 empties the lane first.
// Outputs (n_active x k): is_miss, item_slot, miss_page/miss_slot compacted per
// row in selection order, n_miss[i].
static int lru_step(OrcLru* h, int n_active, const int32_t* lane_ids, const uint8_t* reset,
                    const int32_t* sel, int k, const int32_t* n_sel, const uint32_t* bits,
                    uint8_t* is_miss, int32_t* item_slot, int32_t* miss_page, int32_t* miss_slot,
                    int32_t* n_miss) {
  const bool group = !h->lane_cap.empty();
  for (int a = 0; a < n_active; ++a) {
    const int lane = lane_ids[a];
    if (lane < 0 || lane >= h->lanes) return -1;
    int32_t* ps = &h->page_slot[(size_t)lane * h->ids];
    auto& dq = h->order[lane];
    const int cap = group ? h->lane_cap[lane] : h->cap;
    if (reset && reset[a]) {
      for (int32_t pg : dq) ps[pg] = -1;
      dq.clear();
      if (group) h->own[lane].clear();
    }
    int nm = 0;
    for (int i = 0; i < n_sel[a]; ++i) {
      const int32_t x = sel[(size_t)a * k + i];
      if (x < 0 || x >= h->ids) return -2;
      int32_t s = ps[x];
      const bool hit = s >= 0;
      if (hit) {
        dq.erase(std::find(dq.begin(), dq.end(), x));
        dq.push_back(x);
      } else {
        if ((int)dq.size() >= cap) {
          const int32_t v = dq.front();
          dq.pop_front();
          s = ps[v];
          ps[v] = -1;
          if (group) h->own[lane].erase(v);  // own_drop
        } else {
          s = (int32_t)dq.size();
        }
        dq.push_back(x);
        ps[x] = s;
        miss_page[(size_t)a * k + nm] = x;
        miss_slot[(size_t)a * k + nm] = s;
        ++nm;
      }
      is_miss[(size_t)a * k + i] = hit ? 0 : 1;
      item_slot[(size_t)a * k + i] = s;
      if (group && bits) h->own[lane][x] |= bits[a];  // kv_touch: the toucher needs it
    }
    n_miss[a] = nm;
  }
  return 0;
}

int orc_lru_step(void* p, int n_active, const int32_t* lane_ids, const uint8_t* reset,
                 const int32_t* sel, int k, const int32_t* n_sel, uint8_t* is_miss,
                 int32_t* item_slot, int32_t* miss_page, int32_t* miss_slot,
                 int32_t* n_miss) {
  return lru_step((OrcLru*)p, n_active, lane_ids, reset, sel, k, n_sel, nullptr, is_miss, item_slot,
                  miss_page, miss_slot, n_miss);
}

// ---- group lanes (kv_touch / grp_trim / own_* / kv_handoff of the reference,
// src/runtime/wla_multigpu.cuh:1867-2015) with this build's slot rules:
// occupied slots stay [0, size); a trim moves the survivors at slots >= the
// new capacity, in LRU order, into the freed slots below it, ascending.
int orc_lru_group_enable(void* p) {
  auto* h = (OrcLru*)p;
  if (h->lane_cap.empty()) {
    h->lane_cap.assign(h->lanes, h->cap);
    h->own.assign(h->lanes, {});
  }
  return 0;
}

int orc_lru_touch_owned(void* p, int n_active, const int32_t* lane_ids, const uint8_t* reset,
                        const int32_t* sel, int k, const int32_t* n_sel, const uint32_t* bits,
                        uint8_t* is_miss, int32_t* item_slot, int32_t* miss_page, int32_t* miss_slot,
                        int32_t* n_miss) {
  auto* h = (OrcLru*)p;
  if (h->lane_cap.empty()) return -3;
  return lru_step(h, n_active, lane_ids, reset, sel, k, n_sel, bits, is_miss, item_slot, miss_page,
                  miss_slot, n_miss);
}

// grp_trim (:1923-1935) after a capacity change (cap_mode 1)
int orc_lru_set_capacity(void* p, int n, const int32_t* lane_ids, const int32_t* caps) {
  auto* h = (OrcLru*)p;
  if (h->lane_cap.empty()) return -3;
  for (int a = 0; a < n; ++a) {
    const int lane = lane_ids[a], c = caps[a];
    if (lane < 0 || lane >= h->lanes || c < 1 || c > h->cap) return -1;
    h->lane_cap[lane] = c;
    auto& dq = h->order[lane];
    int32_t* ps = &h->page_slot[(size_t)lane * h->ids];
    std::vector<char> freed(c, 0);
    while ((int)dq.size() > c) {
      const int32_t v = dq.front();
      h->own[lane].erase(v);
      if (ps[v] < c) freed[ps[v]] = 1;
      ps[v] = -1;
      dq.pop_front();
    }
    std::vector<int32_t> fr;
    for (int s2 = 0; s2 < c; ++s2)
      if (freed[s2]) fr.push_back(s2);
    size_t r = 0;
    for (int32_t pg : dq)
      if (ps[pg] >= c) {
        if (r >= fr.size()) return -4;
        ps[pg] = fr[r++];
      }
  }
  return 0;
}

// own_release (:1896-1911)
int orc_lru_release(void* p, int n, const int32_t* lane_ids, uint32_t bit) {
  auto* h = (OrcLru*)p;
  if (h->lane_cap.empty()) return -3;
  for (int a = 0; a < n; ++a) {
    const int lane = lane_ids[a];
    if (lane < 0 || lane >= h->lanes) return -1;
    auto& m = h->own[lane];
    for (auto it = m.begin(); it != m.end();) {
      it->second &= ~bit;
      if (it->second == 0)
        it = m.erase(it);
      else
        ++it;
    }
  }
  return 0;
}

// kv_live_owned (:1912-1921), per lane
int orc_lru_count_owned(void* p, int n, const int32_t* lane_ids, uint32_t bit, int32_t* out) {
  auto* h = (OrcLru*)p;
  if (h->lane_cap.empty()) return -3;
  for (int a = 0; a < n; ++a) {
    const int lane = lane_ids[a];
    if (lane < 0 || lane >= h->lanes) return -1;
    int c = 0;
    for (int32_t pg : h->order[lane]) {
      auto it = h->own[lane].find(pg);
      c += (it != h->own[lane].end() && it->second == bit);
    }
    out[a] = c;
  }
  return 0;
}

// kv_handoff (:1970-1990) and kv_handoff_owned (:1991-2015); mode 0 drop,
// 1 carry, 2 owned
int orc_lru_handoff(void* pd, void* psrc, int n, const int32_t* src_lanes, const int32_t* dst_lanes, int mode,
                    uint32_t bit) {
  auto* d = (OrcLru*)pd;
  auto* sr = (OrcLru*)psrc;
  if (d->lane_cap.empty() || (mode != 0 && sr->lane_cap.empty())) return -3;
  for (int a = 0; a < n; ++a) {
    const int dl = dst_lanes[a];
    if (dl < 0 || dl >= d->lanes) return -1;
    int32_t* dps = &d->page_slot[(size_t)dl * d->ids];
    auto& ddq = d->order[dl];
    if (mode == 0) {
      for (int32_t pg : ddq) dps[pg] = -1;
      ddq.clear();
      d->own[dl].clear();
      continue;
    }
    const int sl = src_lanes[a];
    if (sl < 0 || sl >= sr->lanes) return -1;
    const int32_t* sps = &sr->page_slot[(size_t)sl * sr->ids];
    const auto& sdq = sr->order[sl];
    if (mode == 1) {
      if ((int)sdq.size() > d->lane_cap[dl]) return -5;
      for (int32_t pg : ddq) dps[pg] = -1;
      ddq = sdq;
      for (int32_t pg : ddq) dps[pg] = sps[pg];
      d->own[dl] = sr->own[sl];
      continue;
    }
    const int cap = d->lane_cap[dl];
    for (int32_t pg : sdq) {
      auto it = sr->own[sl].find(pg);
      if (it == sr->own[sl].end() || it->second != bit) continue;  // shared / dead: not moved
      if (dps[pg] >= 0) {
        d->own[dl][pg] |= bit;
        continue;
      }
      int32_t slot;
      if ((int)ddq.size() >= cap) {
        const int32_t v = ddq.front();
        ddq.pop_front();
        d->own[dl].erase(v);
        slot = dps[v];
        dps[v] = -1;
      } else {
        slot = (int32_t)ddq.size();
      }
      ddq.push_back(pg);
      dps[pg] = slot;
      d->own[dl][pg] |= bit;
    }
  }
  return 0;
}

// masks of one lane by slot (0 where no page or no owner) and its capacity
int orc_lru_owned_state(void* p, int lane, uint32_t* masks, int32_t* capacity) {
  auto* h = (OrcLru*)p;
  if (h->lane_cap.empty() || lane < 0 || lane >= h->lanes) return -1;
  const int32_t* ps = &h->page_slot[(size_t)lane * h->ids];
  std::memset(masks, 0, sizeof(uint32_t) * h->cap);
  for (const auto& kv : h->own[lane])
    if (ps[kv.first] >= 0) masks[ps[kv.first]] = kv.second;
  *capacity = h->lane_cap[lane];
  return 0;
}

// Full state of one lane: page_slot (ids entries), LRU order as slots
// (front..back), size.
int orc_lru_state(void* p, int lane, int32_t* page_slot, int32_t* lru_slots,
                  int32_t* size) {
  auto* h = (OrcLru*)p;
  const int32_t* ps = &h->page_slot[(size_t)lane * h->ids];
  std::memcpy(page_slot, ps, sizeof(int32_t) * h->ids);
  const auto& dq = h->order[lane];
  for (size_t j = 0; j < dq.size(); ++j) lru_slots[j] = ps[dq[j]];
  *size = (int32_t)dq.size();
  return 0;
}

// ===========================================================================
// 3. Procedural KV pool (synthetic input generator; identical integer steps in
//    ferry_b200/csrc/kvgen.cu). Element e of page unit u is an Irwin-Hall sum
//    of twelve 16-bit uniforms: z = (sum - 6*65536) / 65536, variance 1, range
//    [-6, 6], exact in fp32, rounded once to fp16.
// ===========================================================================
uint16_t orc_kv_elem(uint64_t seed, uint64_t unit, uint32_t e) {
  const uint64_t base = mix64(seed ^ mix64(unit * 4096ull + e));
  uint32_t acc = 0;
  for (int j = 0; j < 3; ++j) {
    const uint64_t h = mix64(base + (uint64_t)j);
    acc += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) +
           (uint32_t)((h >> 32) & 0xFFFF) + (uint32_t)(h >> 48);
  }
  const float z = (float)((int32_t)acc - 6 * 65536) * (1.0f / 65536.0f);
  return f2h(z);
}

int orc_kv_gen(uint64_t seed, uint64_t unit0, int64_t n_units, uint16_t* out) {
  for (int64_t u = 0; u < n_units; ++u)
    for (int e = 0; e < kUnitElems; ++e)
      out[u * kUnitElems + e] = orc_kv_elem(seed, unit0 + (uint64_t)u, (uint32_t)e);
  return 0;
}

// Same output, split over `threads` host threads by unit ranges.
int orc_kv_gen_mt(uint64_t seed, uint64_t unit0, int64_t n_units, uint16_t* out, int threads) {
  if (threads < 1) threads = 1;
  std::vector<std::thread> th;
  const int64_t per = (n_units + threads - 1) / threads;
  for (int i = 0; i < threads; ++i) {
    const int64_t b = i * per, e = std::min<int64_t>(n_units, b + per);
    if (b >= e) break;
    th.emplace_back([=] { orc_kv_gen(seed, unit0 + (uint64_t)b, e - b, out + b * kUnitElems); });
  }
  for (auto& x : th) x.join();
  return 0;
}

// ===========================================================================
// 4. Page summaries and top-k selection (benchmark definition).
//    summary[d] = (k_0[d] + k_1[d] + ... + k_15[d]) * (1/16), summed in token
//    order in fp32. score(page, head) = the 128-term dot product in the fixed
//    order: lane l in 0..31 forms q[4l]*s[4l], then fma-accumulates 4l+1..4l+3;
//    the 32 partials are combined by a butterfly (v_l += v_{l^off}, off = 16, 8,
//    4, 2, 1). GQA: max over the group's q heads. Top-k: descending by score,
//    ties to the lower page id, output ascending by page id -- the same
//    "topk(...).indices.sort()" shape as tools/capture_miss_trace.py:158-159.
// ===========================================================================
int orc_page_summary(const uint16_t* units, int64_t n_units, float* summ) {
  for (int64_t u = 0; u < n_units; ++u) {
    const uint16_t* K = units + u * kUnitElems;
    for (int d = 0; d < kHeadDim; ++d) {
      float acc = h2f(K[d]);
      for (int t = 1; t < kPageTokens; ++t) acc = acc + h2f(K[t * kHeadDim + d]);
      summ[u * kHeadDim + d] = acc * 0.0625f;
    }
  }
  return 0;
}

static inline float score_dot(const float* q, const float* s) {
  float v[32];
  for (int l = 0; l < 32; ++l) {
    float a = q[4 * l] * s[4 * l];
    a = std::fma(q[4 * l + 1], s[4 * l + 1], a);
    a = std::fma(q[4 * l + 2], s[4 * l + 2], a);
    a = std::fma(q[4 * l + 3], s[4 * l + 3], a);
    v[l] = a;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float w[32];
    for (int l = 0; l < 32; ++l) w[l] = v[l] + v[l ^ off];
    std::memcpy(v, w, sizeof v);
  }
  return v[0];
}

static inline uint32_t order_key(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// q: n_lanes x G x 128 fp16; summ: n_lanes x N x 128 fp32 (row stride N);
// n_pages[i] <= N valid pages. sel_out: n_lanes x k; n_sel_out = min(k, n_pages).
int orc_select_topk(const uint16_t* q, int G, const float* summ, int N,
                    const int32_t* n_pages, int n_lanes, int k, int32_t* sel_out,
                    int32_t* n_sel_out, float* scores_out) {
  std::vector<float> qf(G * kHeadDim);
  std::vector<std::pair<uint32_t, int32_t>> keys;
  for (int i = 0; i < n_lanes; ++i) {
    for (int j = 0; j < G * kHeadDim; ++j) qf[j] = h2f(q[(size_t)i * G * kHeadDim + j]);
    const int np = n_pages[i];
    keys.resize(np);
    for (int p = 0; p < np; ++p) {
      const float* s = summ + ((size_t)i * N + p) * kHeadDim;
      float best = score_dot(&qf[0], s);
      for (int g = 1; g < G; ++g) {
        const float v = score_dot(&qf[g * kHeadDim], s);
        best = v > best ? v : best;  // first head wins ties
      }
      if (scores_out) scores_out[(size_t)i * N + p] = best;
      keys[p] = {order_key(best), p};
    }
    const int kk = std::min(k, np);
    std::partial_sort(keys.begin(), keys.begin() + kk, keys.end(),
                      [](const auto& a, const auto& b) {
                        return a.first != b.first ? a.first > b.first : a.second < b.second;
                      });
    std::vector<int32_t> pick(kk);
    for (int j = 0; j < kk; ++j) pick[j] = keys[j].second;
    std::sort(pick.begin(), pick.end());
    for (int j = 0; j < kk; ++j) sel_out[(size_t)i * k + j] = pick[j];
    n_sel_out[i] = kk;
  }
  return 0;
}

// ===========================================================================
// 5. Sparse paged decode attention over the selected pages (no reference math
//    exists; standard softmax(q K^T * scale) V in double precision).
//    q: n_lanes x G x 128 fp16; pages: n_lanes x k units (row stride k) holding
//    the selected pages' K/V; out: n_lanes x G x 128.
// ===========================================================================
int orc_sparse_decode(const uint16_t* q, int G, const uint16_t* pages, const int32_t* n_sel,
                      int n_lanes, int k, float scale, float* out) {
  std::vector<double> logit;
  for (int i = 0; i < n_lanes; ++i)
    for (int g = 0; g < G; ++g) {
      const uint16_t* qh = q + ((size_t)i * G + g) * kHeadDim;
      const int ntok = n_sel[i] * kPageTokens;
      logit.assign(ntok, 0.0);
      double mx = -INFINITY;
      for (int p = 0; p < n_sel[i]; ++p) {
        const uint16_t* K = pages + ((size_t)i * k + p) * kUnitElems;
        for (int t = 0; t < kPageTokens; ++t) {
          double acc = 0.0;
          for (int d = 0; d < kHeadDim; ++d)
            acc += (double)h2f(qh[d]) * (double)h2f(K[t * kHeadDim + d]);
          acc *= scale;
          logit[p * kPageTokens + t] = acc;
          mx = std::max(mx, acc);
        }
      }
      double den = 0.0;
      double o[kHeadDim] = {0};
      for (int p = 0; p < n_sel[i]; ++p) {
        const uint16_t* V = pages + ((size_t)i * k + p) * kUnitElems + kPageTokens * kHeadDim;
        for (int t = 0; t < kPageTokens; ++t) {
          const double w = std::exp(logit[p * kPageTokens + t] - mx);
          den += w;
          for (int d = 0; d < kHeadDim; ++d) o[d] += w * (double)h2f(V[t * kHeadDim + d]);
        }
      }
      float* oh = out + ((size_t)i * G + g) * kHeadDim;
      for (int d = 0; d < kHeadDim; ++d) oh[d] = ntok ? (float)(o[d] / den) : 0.0f;
    }
  return 0;
}

// ===========================================================================
// 6. CPU pipeline for the timed baseline: select -> LRU miss detect -> memcpy
//    gather from the host pool -> attention, multi-threaded over lanes with
//    std::thread (the reference runs this path on host cores:
//    missstream.cuh:137-161 LRU, host_staged_channel.cpp:43-74 copies).
//    Attention here accumulates in fp32 (the timed baseline is the fp32 CPU
//    path; the double-precision checker above is separate).
// ===========================================================================
struct OrcPipe {
  int lanes, N, C, k, G, threads;
  const uint16_t* pool;     // lanes*N units (unit = lane*N + page) -- caller owns
  const float* summ;        // lanes*N*128
  std::vector<uint16_t> cache;  // lanes*C units
  OrcLru* lru;
};

void* orc_pipe_create(int lanes, int N, int C, int k, int G, const uint16_t* pool,
                      const float* summ, int threads) {
  auto* p = new OrcPipe;
  p->lanes = lanes; p->N = N; p->C = C; p->k = k; p->G = G;
  p->threads = threads > 0 ? threads : 1;
  p->pool = pool; p->summ = summ;
  p->cache.assign((size_t)lanes * C * kUnitElems, 0);
  p->lru = (OrcLru*)orc_lru_create(lanes, C, N);
  return p;
}
void orc_pipe_destroy(void* h) {
  auto* p = (OrcPipe*)h;
  orc_lru_destroy(p->lru);
  delete p;
}

// One decode step for n_active lanes: q is n_active x G x 128 fp16.
// Returns miss count; out is n_active x G x 128.
int64_t orc_pipe_step(void* h, int n_active, const int32_t* lane_ids, const uint8_t* reset,
                      const uint16_t* q, float scale, float* out, const int32_t* n_pages) {
  auto* p = (OrcPipe*)h;
  std::atomic<int> next{0};
  std::atomic<int64_t> misses{0};
  auto work = [&]() {
    const int k = p->k, G = p->G;
    std::vector<int32_t> sel(k), item_slot(k), mp(k), msl(k);
    std::vector<uint8_t> im(k);
    std::vector<float> qf(G * kHeadDim), logit(k * kPageTokens);
    std::vector<std::pair<uint32_t, int32_t>> keys(p->N);
    for (;;) {
      const int a = next.fetch_add(1);
      if (a >= n_active) break;
      const int lane = lane_ids[a];
      const uint16_t* qa = q + (size_t)a * G * kHeadDim;
      for (int j = 0; j < G * kHeadDim; ++j) qf[j] = h2f(qa[j]);
      const int np = n_pages ? std::max(0, std::min(p->N, n_pages[a])) : p->N;  // whole pages of the context
      for (int pg = 0; pg < np; ++pg) {
        const float* s = p->summ + ((size_t)lane * p->N + pg) * kHeadDim;
        float best = score_dot(&qf[0], s);
        for (int g = 1; g < G; ++g) {
        const float v = score_dot(&qf[g * kHeadDim], s);
        best = v > best ? v : best;  // first head wins ties
      }
        keys[pg] = {order_key(best), pg};
      }
      const int kk = std::min(k, np);
      std::partial_sort(keys.begin(), keys.begin() + kk, keys.begin() + np,
                        [](const auto& x, const auto& y) {
                          return x.first != y.first ? x.first > y.first : x.second < y.second;
                        });
      for (int j = 0; j < kk; ++j) sel[j] = keys[j].second;
      std::sort(sel.begin(), sel.begin() + kk);
      int32_t nm = 0, ns = kk;
      orc_lru_step(p->lru, 1, &lane, reset ? &reset[a] : nullptr, sel.data(), k, &ns,
                   im.data(), item_slot.data(), mp.data(), msl.data(), &nm);
      for (int j = 0; j < nm; ++j)
        std::memcpy(&p->cache[((size_t)lane * p->C + msl[j]) * kUnitElems],
                    p->pool + ((size_t)lane * p->N + mp[j]) * kUnitElems,
                    kUnitElems * sizeof(uint16_t));
      misses.fetch_add(nm);
      for (int g = 0; g < G; ++g) {
        const float* qh = &qf[g * kHeadDim];
        float mx = -INFINITY;
        for (int j = 0; j < kk; ++j) {
          const uint16_t* K = &p->cache[((size_t)lane * p->C + item_slot[j]) * kUnitElems];
          for (int t = 0; t < kPageTokens; ++t) {
            float acc = 0.f;
            for (int d = 0; d < kHeadDim; ++d) acc += qh[d] * h2f(K[t * kHeadDim + d]);
            acc *= scale;
            logit[j * kPageTokens + t] = acc;
            mx = std::max(mx, acc);
          }
        }
        float den = 0.f, o[kHeadDim] = {0};
        for (int j = 0; j < kk; ++j) {
          const uint16_t* V = &p->cache[((size_t)lane * p->C + item_slot[j]) * kUnitElems] +
                              kPageTokens * kHeadDim;
          for (int t = 0; t < kPageTokens; ++t) {
            const float w = std::exp(logit[j * kPageTokens + t] - mx);
            den += w;
            for (int d = 0; d < kHeadDim; ++d) o[d] += w * h2f(V[t * kHeadDim + d]);
          }
        }
        float* oh = out + ((size_t)a * G + g) * kHeadDim;
        for (int d = 0; d < kHeadDim; ++d) oh[d] = o[d] / den;
      }
    }
  };
  std::vector<std::thread> th;
  for (int t = 1; t < p->threads; ++t) th.emplace_back(work);
  work();
  for (auto& t : th) t.join();
  return misses.load();
}

// ===========================================================================
// 7. fp8 KV (benchmark definition: OCP e4m3 with a per-page fp32 scale).
//    e4m3: 1 sign, 4 exponent bits (bias 7), 3 mantissa bits, no infinities,
//    max finite 448, S.1111.111 = NaN. Encoding rounds to nearest, ties to
//    even, and saturates to +-448 (what cvt.rn.satfinite.e4m3x2.f32 does).
//    Page unit (4112 B): K[16][128] e4m3 | V[16][128] e4m3 | k_scale f32 |
//    v_scale f32 | 8 pad bytes. scale = amax / 448 over the page's K (resp.
//    V) values before quantisation; q = e4m3(z / scale).
// ===========================================================================
uint8_t orc_e4m3_encode(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  const uint8_t sign = (u >> 31) ? 0x80 : 0;
  const float a = std::fabs(x);
  if (std::isnan(x)) return 0x7F | sign;
  if (a >= 448.0f) return sign | 0x7E;  // satfinite
  // smallest subnormal 2^-9; values below 2^-10 (half of it) round to 0 or
  // to 2^-9 by ties-to-even at exactly 2^-10
  int e;
  std::frexp(a, &e);  // a = m * 2^e, m in [0.5, 1)
  int E = e - 1;      // a in [2^E, 2^(E+1))
  if (E < -6) E = -6;  // subnormal range: spacing 2^-9
  const float spacing = std::ldexp(1.0f, E - 3);
  float q = a / spacing;           // exact (power-of-two scaling)
  float r = std::nearbyint(q);     // ties to even (default rounding mode)
  float v = r * spacing;
  if (v >= 448.0f) return sign | 0x7E;
  if (v == 0.0f) return sign;
  int ev;
  const float mv = std::frexp(v, &ev);  // v = mv * 2^ev
  int Eb = ev - 1 + 7;
  if (Eb <= 0) {  // subnormal: v = mant * 2^-9
    const int mant = (int)std::ldexp(v, 9);
    return sign | (uint8_t)mant;
  }
  const int mant = (int)((mv * 2.0f - 1.0f) * 8.0f);
  return sign | (uint8_t)((Eb << 3) | mant);
}

float orc_e4m3_decode(uint8_t b) {
  const int s = b >> 7, E = (b >> 3) & 0xF, m = b & 7;
  if (E == 0xF && m == 7) return NAN;
  const float v = E == 0 ? std::ldexp((float)m, -9) : std::ldexp(1.0f + m / 8.0f, E - 7);
  return s ? -v : v;
}

static inline float kv_elem_f32(uint64_t seed, uint64_t unit, uint32_t e) {
  const uint64_t base = mix64(seed ^ mix64(unit * 4096ull + e));
  uint32_t acc = 0;
  for (int j = 0; j < 3; ++j) {
    const uint64_t h = mix64(base + (uint64_t)j);
    acc += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) +
           (uint32_t)((h >> 32) & 0xFFFF) + (uint32_t)(h >> 48);
  }
  return (float)((int32_t)acc - 6 * 65536) * (1.0f / 65536.0f);
}

constexpr int kUnitBytesF8 = 4112;

// n_units page units of 4112 bytes each
int orc_kv_gen_e4m3(uint64_t seed, uint64_t unit0, int64_t n_units, uint8_t* out) {
  for (int64_t u = 0; u < n_units; ++u) {
    uint8_t* dst = out + u * kUnitBytesF8;
    float scales[2];
    for (int half = 0; half < 2; ++half) {
      const uint32_t e0 = half * 2048;
      float amax = 0.f;
      for (int i = 0; i < 2048; ++i)
        amax = std::max(amax, std::fabs(kv_elem_f32(seed, unit0 + u, e0 + i)));
      const float scale = amax > 0.f ? amax / 448.0f : 1.0f;
      scales[half] = scale;
      for (int i = 0; i < 2048; ++i)
        dst[e0 + i] = orc_e4m3_encode(kv_elem_f32(seed, unit0 + u, e0 + i) / scale);
    }
    std::memcpy(dst + 4096, scales, 8);
    std::memset(dst + 4104, 0, 8);
  }
  return 0;
}

int orc_kv_gen_e4m3_mt(uint64_t seed, uint64_t unit0, int64_t n_units, uint8_t* out, int threads) {
  if (threads < 1) threads = 1;
  std::vector<std::thread> th;
  const int64_t per = (n_units + threads - 1) / threads;
  for (int i = 0; i < threads; ++i) {
    const int64_t b = i * per, e = std::min<int64_t>(n_units, b + per);
    if (b >= e) break;
    th.emplace_back([=] { orc_kv_gen_e4m3(seed, unit0 + (uint64_t)b, e - b, out + b * kUnitBytesF8); });
  }
  for (auto& x : th) x.join();
  return 0;
}

// dequantised K/V of n units into fp32 [n][2][16][128]
int orc_e4m3_unit_dequant(const uint8_t* units, int64_t n_units, float* out) {
  for (int64_t u = 0; u < n_units; ++u) {
    const uint8_t* p = units + u * kUnitBytesF8;
    float sc[2];
    std::memcpy(sc, p + 4096, 8);
    for (int i = 0; i < 4096; ++i) out[u * 4096 + i] = orc_e4m3_decode(p[i]) * sc[i / 2048];
  }
  return 0;
}

// summary[d] = (k_0[d] + ... + k_15[d]) * (1/16) over dequantised keys
// (each k_t[d] = float(e4m3) * k_scale, one rounding), token order.
int orc_page_summary_e4m3(const uint8_t* units, int64_t n_units, float* summ) {
  for (int64_t u = 0; u < n_units; ++u) {
    const uint8_t* K = units + u * kUnitBytesF8;
    float ks;
    std::memcpy(&ks, K + 4096, 4);
    for (int d = 0; d < kHeadDim; ++d) {
      float acc = orc_e4m3_decode(K[d]) * ks;
      for (int t = 1; t < kPageTokens; ++t) acc = acc + orc_e4m3_decode(K[t * kHeadDim + d]) * ks;
      summ[u * kHeadDim + d] = acc * 0.0625f;
    }
  }
  return 0;
}

// ===========================================================================
// 4b. Quest selection, the reference's Selector.on_layer method "quest"
//     (tools/capture_miss_trace.py:139-147, 158-159): per page and dim the min
//     and max of its keys; bound(head, page) = sum_d max(q_d*kmax_d, q_d*kmin_d);
//     score(page) = max over the GQA group, then over the kv heads (one page set
//     per layer); top-k by score, ascending output. Fixed arithmetic: products
//     rounded to fp32, max(a = q*kmax, b = q*kmin) = a >= b ? a : b, lane l sums
//     dims 4l..4l+3 in order, the 32 lane sums combine by the xor butterfly
//     (16, 8, 4, 2, 1); heads scanned kv head major, the first head wins ties;
//     top-k ties to the lower page id. min/max over tokens in token order
//     (a later token replaces only when strictly smaller / larger).
// ===========================================================================
static void minmax_rows(const float* K /* 16 x 128 */, float* mm) {
  for (int d = 0; d < kHeadDim; ++d) {
    float lo = K[d], hi = K[d];
    for (int t = 1; t < kPageTokens; ++t) {
      const float v = K[t * kHeadDim + d];
      lo = v < lo ? v : lo;
      hi = v > hi ? v : hi;
    }
    mm[d] = lo;
    mm[kHeadDim + d] = hi;
  }
}

int orc_page_minmax(const uint16_t* units, int64_t n_units, float* mm) {
  float K[kPageTokens * kHeadDim];
  for (int64_t u = 0; u < n_units; ++u) {
    for (int i = 0; i < kPageTokens * kHeadDim; ++i) K[i] = h2f(units[u * kUnitElems + i]);
    minmax_rows(K, mm + u * 2 * kHeadDim);
  }
  return 0;
}

int orc_page_minmax_e4m3(const uint8_t* units, int64_t n_units, float* mm) {
  float K[kPageTokens * kHeadDim];
  for (int64_t u = 0; u < n_units; ++u) {
    const uint8_t* p = units + u * kUnitBytesF8;
    float ks;
    std::memcpy(&ks, p + 4096, 4);
    for (int i = 0; i < kPageTokens * kHeadDim; ++i) K[i] = orc_e4m3_decode(p[i]) * ks;
    minmax_rows(K, mm + u * 2 * kHeadDim);
  }
  return 0;
}

static inline float quest_bound(const float* q, const float* mm) {
  float v[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.f;
    for (int j = 0; j < 4; ++j) {
      const int d = 4 * l + j;
      const float a = q[d] * mm[kHeadDim + d], b = q[d] * mm[d];
      const float m = a >= b ? a : b;
      acc = j == 0 ? m : acc + m;
    }
    v[l] = acc;
  }
  for (int off = 16; off >= 1; off >>= 1) {
    float w[32];
    for (int l = 0; l < 32; ++l) w[l] = v[l] + v[l ^ off];
    std::memcpy(v, w, sizeof v);
  }
  return v[0];
}

// q: n_grp x (Hkv * G) x 128 fp16 (head = kv head * G + g); mm: n_grp x Hkv x N
// rows of 256 fp32 [kmin | kmax]; n_pages[i] <= N. sel_out: n_grp x k;
// n_sel_out = min(k, n_pages); scores_out (nullable): n_grp x N.
int orc_select_quest(const uint16_t* q, int Hkv, int G, const float* mm, int N,
                     const int32_t* n_pages, int n_grp, int k, int32_t* sel_out,
                     int32_t* n_sel_out, float* scores_out) {
  const int Hq = Hkv * G;
  std::vector<float> qf((size_t)Hq * kHeadDim);
  std::vector<std::pair<uint32_t, int32_t>> keys;
  for (int i = 0; i < n_grp; ++i) {
    for (size_t j = 0; j < qf.size(); ++j) qf[j] = h2f(q[(size_t)i * Hq * kHeadDim + j]);
    const int np = n_pages[i];
    keys.resize(np);
    for (int p = 0; p < np; ++p) {
      float best = 0.f;
      for (int h = 0; h < Hkv; ++h) {
        const float* row = mm + (((size_t)i * Hkv + h) * N + p) * 2 * kHeadDim;
        for (int g = 0; g < G; ++g) {
          const float v = quest_bound(&qf[(size_t)(h * G + g) * kHeadDim], row);
          if ((h == 0 && g == 0) || v > best) best = v;
        }
      }
      if (scores_out) scores_out[(size_t)i * N + p] = best;
      keys[p] = {order_key(best), p};
    }
    const int kk = std::min(k, np);
    std::partial_sort(keys.begin(), keys.begin() + kk, keys.end(),
                      [](const auto& a, const auto& b) {
                        return a.first != b.first ? a.first > b.first : a.second < b.second;
                      });
    std::vector<int32_t> pick(kk);
    for (int j = 0; j < kk; ++j) pick[j] = keys[j].second;
    std::sort(pick.begin(), pick.end());
    for (int j = 0; j < k; ++j) sel_out[(size_t)i * k + j] = j < kk ? pick[j] : -1;
    n_sel_out[i] = kk;
  }
  return 0;
}

// ---- Workload B (src/workloads/baselines.cuh) -----------------------------
// The payload pool's content (baselines.cuh:86-89: mt19937_64 seed 9,
// (rng() % 1000) / 8 as float) and the task kernel (baselines.cuh:40-48:
// element i iterates v = fma(v, 1.0000001, 1e-7) works[i] * inner times) on
// the CPU, one correctly rounded fmaf per step as on the GPU.
void orc_taskb_payload(uint64_t n_floats, float* out) {
  std::mt19937_64 rng(9);
  for (uint64_t i = 0; i < n_floats; ++i) out[i] = (float)(rng() % 1000) / 8.0f;
}

void orc_taskb_compute(const float* in, float* out, uint64_t n, const int32_t* works, int inner) {
  for (uint64_t i = 0; i < n; ++i) {
    const int w = works[i] * inner;
    float v = in[i];
    for (int k = 0; k < w; ++k) v = std::fmaf(v, 1.0000001f, 1e-7f);
    out[i] = v;
  }
}

int orc_version(void) { return 2; }

}  // extern "C"
