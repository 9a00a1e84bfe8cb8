// select.cu -- top-k page selection by q . mean-key page summary.
//
// Scoring (phase 1) splits a lane (request, layer, kv_head) into chunks of
// kSelChunk pages, one CTA each, so the grid stays balanced however few lanes
// are long. A warp scores 8 pages per batch: lane l loads dims 4l..4l+3 of
// each fp32 summary row (one coalesced 512-byte row per warp load) and forms,
// per (page, q head), the partial q[4l]*s[4l] -> fma 4l+1..4l+3. The 32
// partials of up to 32 (page, head) values are summed together by one
// transpose-reduce whose additions are exactly those of the xor butterfly
// over 16, 8, 4, 2, 1 -- bit-identical to reducing each value alone, at one
// shuffle per value instead of five. The maximum over the GQA group is a
// lane tree in which the lower head wins ties (= the sequential scan "first
// head wins"). Every fp32 operation and its order is fixed, so any IEEE-754
// implementation of the same steps reproduces the selection bit for bit.
//
// The last CTA of a lane to finish (a per-lane counter; the sole CTA when the
// lane fits one chunk) holds all keys in shared memory and runs phase 2, a
// 4-pass 8-bit radix select of the k-th largest order-preserving key
// (warp-aggregated histogram atomics), and phase 3, emission in ascending
// page order of every page whose key is larger plus the lowest-id pages equal
// to it -- ties go to the lower page id.
#include "common.cuh"

namespace ferry {
namespace {

constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelBatch = 8;  // pages per warp per stage
constexpr int kSelStages = 3;
constexpr int kRowBytes = kHeadDim * 4;  // 512

// Ring geometry of a W-warp CTA: a stage holds 8 summary rows per warp.
// W = 8 (long lanes, chunked): 64-row / 32 KiB stages, 96 KiB ring, 2 CTAs
// per SM, block-level radix select. W = 4 (lanes of <= kSelSmallPages pages,
// one CTA each): 32-row / 16 KiB stages, 48 KiB ring, 4 CTAs per SM -- the
// whole batch in one wave with four lanes' loads in flight per SM -- and a
// warp-level select, so no CTA holds the SM through block barriers.
template <int W>
struct SelGeom {
  static constexpr int kThreads = W * 32;
  static constexpr int kStagePages = W * kSelBatch;
  static constexpr int kStageBytes = kStagePages * kRowBytes;
  static constexpr int kRingBytes = kSelStages * kStageBytes;
};
constexpr int kSelSmallPages = 1024;
static_assert(kMaxPages * 4 <= SelGeom<8>::kRingBytes, "keys of a lane must fit the ring");

template <int G>
struct SelShape {
  static constexpr int UR = (32 / G < kSelBatch) ? 32 / G : kSelBatch;  // pages per reduction
  static constexpr int NR = kSelBatch / UR;                            // reductions per batch
  static constexpr int V = UR * G;                                       // values per reduction
  static constexpr int T = V == 32 ? 5 : V == 16 ? 4 : 3;                // transposing levels
  static constexpr int S = 5 - T;  // lane l ends with value l >> S
};

// Sum over the 32 lanes of V independent values. Level j pairs lane l with
// l ^ (16 >> j), as the xor butterfly does; while more than one value is
// left the pair swaps halves, afterwards it is a plain butterfly step. Each
// addition has the same two operands as the butterfly's.
//
// The half swap needs no selects: lane l holds its values permuted,
// w[i] = value[i ^ m] with m = l >> (5 - log2 V), so at every level each lane
// keeps the lower half and sends the upper one (the partner's upper half
// holds the same values as this lane's lower half). Lane l returns value m.
template <int V>
__device__ __forceinline__ float transpose_reduce(float (&w)[V]) {
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const int o = 16 >> j;
    const int n = V >> j;
    if (n > 2) {
#pragma unroll
      for (int i = 0; i < n / 2; i += 2) {  // paired adds (same IEEE rounding per element)
        const float2 r = make_float2(__shfl_xor_sync(0xffffffffu, w[i + n / 2], o),
                                     __shfl_xor_sync(0xffffffffu, w[i + 1 + n / 2], o));
        const float2 sum = __fadd2_rn(make_float2(w[i], w[i + 1]), r);
        w[i] = sum.x;
        w[i + 1] = sum.y;
      }
    } else if (n == 2) {
      w[0] = __fadd_rn(w[0], __shfl_xor_sync(0xffffffffu, w[1], o));
    } else {
      w[0] = __fadd_rn(w[0], __shfl_xor_sync(0xffffffffu, w[0], o));
    }
  }
  return w[0];
}


__device__ __forceinline__ uint32_t lanemask_lt(int lane) { return (1u << lane) - 1u; }

// Shared state of topk_emit.
struct TopkSmem {
  uint32_t hist[256];
  uint32_t wcnt[2][kSelWarps];
  uint32_t s_prefix, s_krem;
};

// Top-k of np > k order keys in shared memory by one block of kSelThreads:
// phase 2, a 4-pass 8-bit radix select of the k-th largest key (warp-aggregated
// histogram atomics); phase 3, emission in ascending page order of every page
// whose key is larger plus the lowest-id pages equal to it (ties go to the
// lower page id). Writes out[0, k).
__device__ __forceinline__ void topk_emit(const uint32_t* keys, int np, int k, int32_t* out,
                                          TopkSmem& S) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* hist = S.hist;
  auto& wcnt = S.wcnt;
  // ---- phase 2: radix select of the k-th largest key
  uint32_t prefix = 0, mask = 0, krem = (uint32_t)k;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[tid] = 0;  // kSelThreads == 256 bins
    __syncthreads();
    for (int base = 0; base < np; base += kSelThreads) {  // block-uniform
      const int p = base + tid;
      const uint32_t key = p < np ? keys[p] : 0u;
      const bool act = p < np && (key & mask) == prefix;
      const uint32_t bin = act ? (key >> shift) & 255u : 256u;
      const uint32_t m = __match_any_sync(0xffffffffu, bin);
      if (act && lane == __ffs(m) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(m));
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[255 - (lane * 8 + j)];
        tot += c[j];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      const uint32_t excl = incl - tot;
      if (excl < krem && krem <= incl) {
        uint32_t run = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (run + c[j] >= krem) {
            S.s_prefix = prefix | ((uint32_t)(255 - (lane * 8 + j)) << shift);
            S.s_krem = krem - run;
            break;
          }
          run += c[j];
        }
      }
    }
    __syncthreads();
    prefix = S.s_prefix;
    krem = S.s_krem;
    mask |= 255u << shift;
  }
  const uint32_t T = prefix;

  // ---- phase 3: ordered emission; warp w owns pages [w * span, (w + 1) * span)
  const int span = ((np + kSelWarps * 32 - 1) / (kSelWarps * 32)) * 32;
  const int lo = warp * span, hi = min(np, lo + span);
  uint32_t ngt = 0, neq = 0;
  for (int base = lo; base < hi; base += 32) {  // warp-uniform
    const int p = base + lane;
    const uint32_t key = p < hi ? keys[p] : 0u;
    ngt += __popc(__ballot_sync(0xffffffffu, p < hi && key > T));
    neq += __popc(__ballot_sync(0xffffffffu, p < hi && key == T));
  }
  if (lane == 0) {
    wcnt[0][warp] = ngt;
    wcnt[1][warp] = neq;
  }
  __syncthreads();
  uint32_t gt_before = 0, eq_before = 0;
  for (int w = 0; w < warp; ++w) {
    gt_before += wcnt[0][w];
    eq_before += wcnt[1][w];
  }
  uint32_t pos = gt_before + min(eq_before, krem), eq_rank = eq_before;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    const uint32_t key = p < hi ? keys[p] : 0u;
    const bool gt = p < hi && key > T, eq = p < hi && key == T;
    const uint32_t meq = __ballot_sync(0xffffffffu, eq);
    const bool take = gt || (eq && eq_rank + __popc(meq & lanemask_lt(lane)) < krem);
    const uint32_t mt = __ballot_sync(0xffffffffu, take);
    if (take) out[pos + __popc(mt & lanemask_lt(lane))] = p;
    pos += __popc(mt);
    eq_rank += __popc(meq);
  }
}

// Top-k of np > k order keys (np <= kSelSmallPages, shared memory) by one
// warp, with the same result as topk_emit: the k-th largest key T is the
// largest t with #(key >= t) >= k, built from the top bit down (32 counting
// rounds over the kPer keys per lane held in registers); then every key > T
// and the lowest-id pages with key == T, emitted in ascending page order.
// Keys are order_key() values, never 0 for a real score (a real key has its
// top bit set or is the complement of a negative float's bits).
template <int kPer>  // keys per lane: np <= 32 * kPer
__device__ __forceinline__ void warp_topk(const uint32_t* keys, int np, int k, int32_t* out) {
  const int lane = threadIdx.x & 31;
  uint32_t kr[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int p = j * 32 + lane;
    kr[j] = p < np ? keys[p] : 0u;  // pages past np hold 0, below every real key
  }
  uint32_t T = 0;
#pragma unroll 1
  for (int b = 31; b >= 0; --b) {
    const uint32_t cand = T | (1u << b);
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) c += kr[j] >= cand ? 1u : 0u;  // cand > 0: padding never counts
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= (uint32_t)k) T = cand;
  }
  uint32_t gt = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) gt += kr[j] > T ? 1u : 0u;
  gt = __reduce_add_sync(0xffffffffu, gt);
  const uint32_t krem = (uint32_t)k - gt;  // keys equal to T that are taken
  uint32_t pos = 0, eq_rank = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int p = j * 32 + lane;
    const bool g = p < np && kr[j] > T, e = p < np && kr[j] == T;
    const uint32_t meq = __ballot_sync(0xffffffffu, e);
    const bool take = g || (e && eq_rank + __popc(meq & lanemask_lt(lane)) < krem);
    const uint32_t mt = __ballot_sync(0xffffffffu, take);
    if (take) out[pos + __popc(mt & lanemask_lt(lane))] = p;
    pos += __popc(mt);
    eq_rank += __popc(meq);
  }
}

struct SelArgs {
  const uint16_t* q;
  const int32_t* req_ids;
  int lanes_per_req;
  const int32_t* ctx_pages;
  const int64_t* req_base;
  const float* summ;
  uint64_t pool_units;
  int N, k, num_requests, nchunks;
  uint32_t* gkeys;  // [batch lanes][N] when nchunks > 1
  uint32_t* done;   // [batch lanes] chunk counters, back to 0 after each launch
  int32_t* sel_out;
  int32_t* n_sel_out;
  uint32_t* err;
};

template <int G, int W>
__global__ void __launch_bounds__(W * 32, W == 8 ? 2 : 4) select_kernel(SelArgs A) {
  using Sh = SelShape<G>;
  using SG = SelGeom<W>;
  constexpr int kThreads = SG::kThreads, kStagePages = SG::kStagePages, kStageBytes = SG::kStageBytes;
  // dynamic: the summary ring; keys after it (one chunk) or in it (after scoring)
  extern __shared__ __align__(128) uint8_t sel_smem[];
  uint8_t* ring = sel_smem;
  uint32_t* keys = reinterpret_cast<uint32_t*>(sel_smem + (A.nchunks > 1 ? 0 : SG::kRingBytes));
  __shared__ __align__(8) uint64_t bars[kSelStages];
  __shared__ TopkSmem tk;
  __shared__ uint32_t s_last;

  const int a = blockIdx.x / A.nchunks, chunk = blockIdx.x % A.nchunks;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int req = A.req_ids[a / A.lanes_per_req];
  const int k = A.k, N = A.N;
  int32_t* out = A.sel_out + (size_t)a * k;
  if (req < 0 || req >= A.num_requests) {  // every chunk of the lane takes this path
    if (tid == 0) {
      record_error(A.err, kErrRange);
      A.n_sel_out[a] = 0;
    }
    for (int j = tid; j < k; j += kThreads) out[j] = -1;
    return;
  }
  int np = A.ctx_pages[req];
  if (np < 0 || np > N) {
    if (tid == 0) record_error(A.err, kErrRange);
    np = np < 0 ? 0 : N;
  }

  // ---- phase 1: scores of this chunk's pages. Summary rows stream through a
  // kSelStages-deep ring of 64-row stages (cp.async.bulk, mbarrier-completed);
  // warp w scores rows 8w..8w+7 of each stage.
  {
    // this lane's value permutation (see transpose_reduce): page u ^ pm, head g ^ hm
    const int m = lane >> Sh::S, pm = m / G, hm = m % G;
    float qv[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint2 raw =
          *reinterpret_cast<const uint2*>(A.q + ((size_t)a * G + (g ^ hm)) * kHeadDim + lane * 4);
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      qv[g][0] = x.x; qv[g][1] = x.y; qv[g][2] = y.x; qv[g][3] = y.y;
    }
    // pool units of this lane: request home + lane-in-request * N (+ page)
    const uint64_t unit0 =
        (uint64_t)(A.req_base[req] + (int64_t)(a % A.lanes_per_req) * N) % A.pool_units;
    const int cs = select_chunk_pages(N, A.nchunks);
    const int c0 = chunk * cs, c1 = min(np, c0 + cs);
    const int n_st = c1 > c0 ? (c1 - c0 + kStagePages - 1) / kStagePages : 0;
    if (tid == 0) {
      for (int i = 0; i < kSelStages; ++i) mbar_init(&bars[i], 1);
      fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int it) {  // thread 0: stage `it` into buffer it % kSelStages
      const int pb = c0 + it * kStagePages, cnt = min(kStagePages, c1 - pb);
      uint8_t* dst = ring + (it % kSelStages) * kStageBytes;
      uint64_t* bar = &bars[it % kSelStages];
      mbar_arrive_expect_tx(bar, (uint32_t)(cnt * kRowBytes));
      uint64_t u = (unit0 + (uint64_t)pb) % A.pool_units;
      for (int d = 0; d < cnt;) {  // split where the pool wraps
        const uint64_t room = A.pool_units - u;
        const int run = (uint64_t)(cnt - d) < room ? cnt - d : (int)room;
        bulk_load(dst + d * kRowBytes, A.summ + u * kHeadDim, (uint32_t)(run * kRowBytes), bar);
        d += run;
        u = 0;
      }
    };
    if (tid == 0)
      for (int i = 0; i < kSelStages && i < n_st; ++i) issue(i);
    uint32_t* kdst = A.nchunks > 1 ? A.gkeys + (size_t)a * N : keys;
    for (int it = 0; it < n_st; ++it) {
      const int buf = it % kSelStages;
      const bool got = __all_sync(0xffffffffu, mbar_wait(&bars[buf], (uint32_t)((it / kSelStages) & 1), A.err));
      const int p0 = c0 + it * kStagePages + warp * kSelBatch;
      if (got && p0 < c1) {  // warp-uniform
        const uint8_t* rows = ring + buf * kStageBytes + warp * kSelBatch * kRowBytes + lane * 16;
#pragma unroll
        for (int r = 0; r < Sh::NR; ++r) {
          float v[Sh::V];
          float4 sv[Sh::UR];
#pragma unroll
          for (int u = 0; u < Sh::UR; ++u)
            sv[u] = *reinterpret_cast<const float4*>(rows + (r * Sh::UR + (u ^ pm)) * kRowBytes);
          // values x = 2i, 2i+1 in one paired FMA chain: heads g, g+1 of a
          // page (G >= 2), or pages u, u+1 (G = 1)
#pragma unroll
          for (int i = 0; i < Sh::V / 2; ++i) {
            const int x0 = 2 * i, x1 = 2 * i + 1;
            const float4 sa = sv[x0 / G], sb = sv[x1 / G];
            const float* qa = qv[x0 % G];
            const float* qb = qv[x1 % G];
            float2 acc = __fmul2_rn(make_float2(qa[0], qb[0]), make_float2(sa.x, sb.x));
            acc = __ffma2_rn(make_float2(qa[1], qb[1]), make_float2(sa.y, sb.y), acc);
            acc = __ffma2_rn(make_float2(qa[2], qb[2]), make_float2(sa.z, sb.z), acc);
            acc = __ffma2_rn(make_float2(qa[3], qb[3]), make_float2(sa.w, sb.w), acc);
            v[x0] = acc.x;
            v[x1] = acc.y;
          }
          float best = transpose_reduce<Sh::V>(v);
          // lane holds value m: page m / G, head m % G
#pragma unroll
          for (int b = 1; b < G; b <<= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, best, b << Sh::S);
            const bool right = (m & b) != 0;  // this lane carries the higher heads
            const float lo = right ? other : best, hi = right ? best : other;
            best = hi > lo ? hi : lo;  // the lower head wins ties
          }
          const int p = p0 + r * Sh::UR + pm;
          if (hm == 0 && (lane & ((1 << Sh::S) - 1)) == 0 && p < c1) kdst[p] = order_key(best);
        }
      }
      if (__syncthreads_or(!got)) {
        // a stage never completed: let the copies still in flight land, then leave
        if (tid == 0)
          for (int j = it; j < n_st && j < it + kSelStages; ++j)
            mbar_wait(&bars[j % kSelStages], (uint32_t)((j / kSelStages) & 1), nullptr);
        __syncthreads();
        return;
      }
      if (tid == 0 && it + kSelStages < n_st) issue(it + kSelStages);
    }
  }
  if (A.nchunks > 1) {
    __syncthreads();  // this chunk's keys are stored (CTA scope); the count publishes them
    if (tid == 0) s_last = atom_add_acq_rel_gpu(&A.done[a], 1u) == (uint32_t)(A.nchunks - 1);
    __syncthreads();
    if (!s_last) return;
    if (tid == 0) A.done[a] = 0;
    for (int p = tid; p < np; p += kThreads) keys[p] = __ldcg(A.gkeys + (size_t)a * N + p);
  }
  __syncthreads();

  if (np <= k) {
    for (int j = tid; j < k; j += kThreads) out[j] = j < np ? j : -1;
    if (tid == 0) A.n_sel_out[a] = np;
    return;
  }

  if constexpr (W == 8) {
    topk_emit(keys, np, k, out, tk);
  } else {
    if (warp != 0) return;
    if (np <= 256)
      warp_topk<8>(keys, np, k, out);
    else if (np <= 512)
      warp_topk<16>(keys, np, k, out);
    else
      warp_topk<32>(keys, np, k, out);
  }
  if (tid == 0) A.n_sel_out[a] = k;
}


// ---------------------------------------------------------------------------
// Quest selection (the reference's Selector.on_layer method "quest",
// tools/capture_miss_trace.py:139-147, 158-159): one page set per (request,
// layer) -- a "group lane" of Hkv kv-head lanes -- scored by
//   score(p) = max over kv heads h, group heads g of
//              sum_d max(q[h,g,d] * kmax[h,p,d], q[h,g,d] * kmin[h,p,d])
// over per-page key bounds (pool rows [kmin[128] | kmax[128]] fp32). Fixed
// arithmetic (the oracle's): products rounded to fp32, a >= b ? a : b with
// a = q*kmax, lane l sums dims 4l..4l+3 in order, the lanes combine by the
// xor butterfly 16, 8, 4, 2, 1; heads kv-head major, the first wins ties.
// A CTA scores a chunk of pages of one group lane, one page per warp at a
// time (all Hkv x G bounds of that page, four kv heads' bounds in flight);
// the last CTA of the group lane runs topk_emit and copies the page set into
// the rows of all Hkv lanes. A chunk holds about kQuestChunkRows (page, kv
// head) bound rows -- 16 pages at 32 kv heads, 64 at 8 -- so that many kv
// heads still spread over many CTAs.
constexpr int kQuestChunkRows = 512;
__host__ __device__ constexpr int quest_chunk_pages(int kv_heads) {
  return kQuestChunkRows / kv_heads < 8 ? 8 : (kQuestChunkRows / kv_heads > 64 ? 64 : kQuestChunkRows / kv_heads);
}

struct QuestArgs {
  const uint16_t* q;
  const int32_t* req_ids;
  int L, Hkv, G;
  const int32_t* ctx_pages;
  const int64_t* req_base;
  const float* mm;
  uint64_t pool_units;
  int N, k, num_requests, nchunks;
  uint32_t* gkeys;  // [batch group lanes][N]
  uint32_t* done;   // [batch group lanes], back to 0 after each launch
  int32_t* sel_out;
  int32_t* n_sel_out;
  uint32_t* err;
};

__device__ __forceinline__ float quest_term(float q, float lo, float hi) {
  const float a = __fmul_rn(q, hi), b = __fmul_rn(q, lo);
  return a >= b ? a : b;
}

__global__ void __launch_bounds__(kSelThreads) select_quest_kernel(QuestArgs A) {
  extern __shared__ __align__(16) uint8_t quest_smem[];
  const int Hq = A.Hkv * A.G;
  float* qs = reinterpret_cast<float*>(quest_smem);                          // Hq x 128
  uint32_t* keys = reinterpret_cast<uint32_t*>(quest_smem + (size_t)Hq * kHeadDim * 4);  // N
  __shared__ TopkSmem tk;
  __shared__ uint32_t s_last;
  const int ag = blockIdx.x / A.nchunks, chunk = blockIdx.x % A.nchunks;
  const int i = ag / A.L, layer = ag % A.L;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = A.k, N = A.N;
  int32_t* out0 = A.sel_out + (size_t)ag * A.Hkv * k;
  const int req = A.req_ids[i];
  if (req < 0 || req >= A.num_requests) {  // every chunk of the group lane takes this path
    if (tid == 0) record_error(A.err, kErrRange);
    for (int x = tid; x < A.Hkv * k; x += kSelThreads) out0[x] = -1;
    for (int h = tid; h < A.Hkv; h += kSelThreads) A.n_sel_out[(size_t)ag * A.Hkv + h] = 0;
    return;
  }
  int np = A.ctx_pages[req];
  if (np < 0 || np > N) {
    if (tid == 0) record_error(A.err, kErrRange);
    np = np < 0 ? 0 : N;
  }
  for (int x = tid; x < Hq * kHeadDim; x += kSelThreads)
    qs[x] = __half2float(__ushort_as_half(A.q[(size_t)ag * Hq * kHeadDim + x]));
  __syncthreads();
  const int cp = quest_chunk_pages(A.Hkv);
  const int c0 = chunk * cp, c1 = min(np, c0 + cp);
  uint32_t* kd = A.gkeys + (size_t)ag * N;
  const int64_t lane0 = A.req_base[req] + (int64_t)layer * A.Hkv * N;  // pool unit of (h = 0, p = 0)
  for (int p = c0 + warp; p < c1; p += kSelWarps) {  // warp-uniform
    float best = 0.f;
#pragma unroll 1
    for (int h0 = 0; h0 < A.Hkv; h0 += 4) {
      // the bounds of 4 kv heads in flight, then their scores in head order
      float4 lo[4], hi[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (h0 + u < A.Hkv) {
          const uint64_t unit = (uint64_t)(lane0 + (int64_t)(h0 + u) * N + p) % A.pool_units;
          lo[u] = __ldg(reinterpret_cast<const float4*>(A.mm + unit * 2 * kHeadDim) + lane);
          hi[u] = __ldg(reinterpret_cast<const float4*>(A.mm + unit * 2 * kHeadDim + kHeadDim) + lane);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int h = h0 + u;
        if (h >= A.Hkv) break;
#pragma unroll 1
        for (int g = 0; g < A.G; ++g) {
          const float4 qv = reinterpret_cast<const float4*>(qs + (size_t)(h * A.G + g) * kHeadDim)[lane];
          float v = quest_term(qv.x, lo[u].x, hi[u].x);
          v = __fadd_rn(v, quest_term(qv.y, lo[u].y, hi[u].y));
          v = __fadd_rn(v, quest_term(qv.z, lo[u].z, hi[u].z));
          v = __fadd_rn(v, quest_term(qv.w, lo[u].w, hi[u].w));
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
          if ((h == 0 && g == 0) || v > best) best = v;
        }
      }
    }
    if (lane == 0) kd[p] = order_key(best);
  }
  __syncthreads();  // this chunk's keys are stored (CTA scope); the count publishes them
  if (tid == 0) s_last = atom_add_acq_rel_gpu(&A.done[ag], 1u) == (uint32_t)(A.nchunks - 1);
  __syncthreads();
  if (!s_last) return;
  if (tid == 0) A.done[ag] = 0;
  for (int p = tid; p < np; p += kSelThreads) keys[p] = __ldcg(kd + p);
  __syncthreads();
  if (np <= k) {
    for (int j = tid; j < k; j += kSelThreads) out0[j] = j < np ? j : -1;
  } else {
    topk_emit(keys, np, k, out0, tk);
  }
  __syncthreads();  // out0 (global) written by this block is visible to the block
  for (int x = tid; x < (A.Hkv - 1) * k; x += kSelThreads) out0[k + x] = out0[x % k];
  for (int h = tid; h < A.Hkv; h += kSelThreads) A.n_sel_out[(size_t)ag * A.Hkv + h] = min(np, k);
}
}  // namespace

size_t select_quest_smem(int q_heads, int max_pages) {
  return (size_t)q_heads * kHeadDim * 4 + (size_t)max_pages * 4;
}

static int launch_select_quest(const ferry_ctx* c, cudaStream_t st, const uint16_t* q,
                               const int32_t* req_ids, int n_req, int32_t* sel, int32_t* n_sel) {
  QuestArgs A{};
  A.q = q;
  A.req_ids = req_ids;
  A.L = c->cfg.num_layers;
  A.Hkv = c->cfg.kv_heads;
  A.G = c->group;
  A.ctx_pages = c->ctx_pages;
  A.req_base = c->req_base;
  A.mm = c->summ;
  A.pool_units = c->pool_units;
  A.N = c->cfg.max_pages;
  A.k = c->cfg.top_k;
  A.num_requests = c->cfg.num_requests;
  A.nchunks = (A.N + quest_chunk_pages(A.Hkv) - 1) / quest_chunk_pages(A.Hkv);
  A.gkeys = c->quest_keys;
  A.done = c->quest_done;
  A.sel_out = sel;
  A.n_sel_out = n_sel;
  A.err = c->err;
  if (!A.gkeys || !A.done) {
    set_error("select: Quest scratch missing");
    return FERRY_E_STATE;
  }
  const size_t smem = select_quest_smem(c->cfg.q_heads, A.N);
  if (smem > 48 * 1024)
    FERRY_TRY(cudaFuncSetAttribute(select_quest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem));
  const unsigned grid = (unsigned)((int64_t)n_req * A.L * A.nchunks);
  select_quest_kernel<<<grid, kSelThreads, smem, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_select(const ferry_ctx* c, cudaStream_t st, const uint16_t* q,
                  const int32_t* req_ids, int n_req, int32_t* sel, int32_t* n_sel) {
  if (n_req <= 0) return FERRY_OK;
  if (c->select_mode == FERRY_SELECT_QUEST)
    return launch_select_quest(c, st, q, req_ids, n_req, sel, n_sel);
  SelArgs A{};
  A.q = q;
  A.req_ids = req_ids;
  A.lanes_per_req = c->lanes_per_req;
  A.ctx_pages = c->ctx_pages;
  A.req_base = c->req_base;
  A.summ = c->summ;
  A.pool_units = c->pool_units;
  A.N = c->cfg.max_pages;
  A.k = c->cfg.top_k;
  A.num_requests = c->cfg.num_requests;
  A.nchunks = select_chunks(A.N);
  A.gkeys = c->sel_keys;
  A.done = c->sel_done;
  A.sel_out = sel;
  A.n_sel_out = n_sel;
  A.err = c->err;
  if (A.nchunks > 1 && (!A.gkeys || !A.done)) {
    set_error("select: chunk scratch missing");
    return FERRY_E_STATE;
  }
  const unsigned grid = (unsigned)((int64_t)n_req * c->lanes_per_req * A.nchunks);
  const bool small = A.nchunks == 1 && A.N <= kSelSmallPages;
  const size_t smem = (small ? SelGeom<4>::kRingBytes : SelGeom<8>::kRingBytes) +
                      (A.nchunks > 1 ? 0 : (size_t)A.N * sizeof(uint32_t));
#define FERRY_SEL_CASE(GG)                                                                    \
  case GG: {                                                                                  \
    auto kern = small ? select_kernel<GG, 4> : select_kernel<GG, 8>;                          \
    if (smem > 48 * 1024)                                                                     \
      FERRY_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                     (int)smem));                                             \
    kern<<<grid, small ? 128 : 256, smem, st>>>(A);                                           \
    break;                                                                                    \
  }
  switch (c->group) {
    FERRY_SEL_CASE(1)
    FERRY_SEL_CASE(2)
    FERRY_SEL_CASE(4)
    FERRY_SEL_CASE(8)
    default:
      set_error("select: unsupported GQA group %d", c->group);
      return FERRY_E_INVAL;
  }
#undef FERRY_SEL_CASE
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

}  // namespace ferry
