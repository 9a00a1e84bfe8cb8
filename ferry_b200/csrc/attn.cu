// attn.cu -- paged sparse decode attention over the selected pages.
//
// Work split. The batch's selected pages are laid out flat, index
// x = lane * k + j (j < k; indices j >= n_sel[lane] are skipped). Warp w of nw
// owns the contiguous range [w*T/nw, (w+1)*T/nw), T = n_lanes * k, so every
// warp streams the same number of page slots (+-1) and no SM idles in a tail.
// A warp's range covers a few lane segments; each segment leaves one partial
// (o[128], m, l) in scratch slot lane + w (unique: ranges are ordered), and
// the warp that completes a lane's last segment (atomic count) combines its
// <= 32 partials -- one per warp lane -- into out.
//
// Streaming. Each warp owns a 2-stage shared-memory ring; a stage is one 8 KiB
// page unit filled by a single cp.async.bulk (TMA engine) completing on an
// mbarrier (bounded waits). The load cursor walks the same flat range one page
// ahead of compute, across lane boundaries. 2 stages keep the CTA at 64 KiB,
// 3 CTAs (12 warps) per SM.
//
// Math per page and q head (fp32 accumulation). Half-warp h = t>>4 handles the
// tokens of parity h; lane t owns dims 8*(t&15)..+8 (16-byte shared loads).
//   QK: 8 partial dots per lane; lane t loads token 2*(i ^ m)+h at step i,
//       m = (t&15)>>1, so the transpose-reduce over the half-warp (xor 8,4,2
//       keep the low half, then xor 1 sums) needs no selects: 4+2+1+1
//       shuffles leave token 2*m+h in lanes t and t^1.
//   softmax: online, base 2 (q pre-scaled by log2(e)/sqrt(128)), max over the
//       16 tokens by xor 2,4,8,16.
//   PV: p written to a 16-float shared slot per warp, read back as 2 float4,
//       8 tokens x 8 dims of FMA per lane; the two half-warps' o are summed
//       once per segment.
#include <mutex>

#include "common.cuh"

namespace ferry {
namespace {

// warps per CTA and bulk-copy stages per warp (build-time tunables)
#ifndef FERRY_ATTN_WARPS
#define FERRY_ATTN_WARPS 4
#endif
#ifndef FERRY_ATTN_STAGES
#define FERRY_ATTN_STAGES 2
#endif
constexpr int kAttnWarps = FERRY_ATTN_WARPS;
constexpr int kStages = FERRY_ATTN_STAGES;
constexpr uint32_t kFull = 0xffffffffu;
constexpr size_t kAttnSmem = (size_t)kAttnWarps * (kStages * kUnitBytes + kStages * 8 + 64);
// CTAs resident per SM: 228 KiB of shared memory per SM, 1 KiB reserved per CTA
constexpr int kAttnCtasPerSm = (int)((228u * 1024u) / (kAttnSmem + 1024u)) < 8
                                   ? (int)((228u * 1024u) / (kAttnSmem + 1024u))
                                   : 8;
static_assert(kAttnCtasPerSm >= 1, "attention ring does not fit an SM");

struct AttnArgs {
  const uint16_t* q;
  const int32_t* req_ids;
  int lanes_per_req;
  int n_lanes;
  int64_t lanes_total;
  const uint8_t* cache;
  int C;
  const int32_t* item_slot;
  const int32_t* n_sel;
  int k;
  int64_t T;  // n_lanes * k
  int nw;     // warps sharing the flat range
  float* part;
  uint32_t* lane_done;
  float* out;
  uint32_t* err;
  float qscale;
};

__device__ __forceinline__ void h8_to_f(const uint4& r, float* f) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

// end (exclusive, lane-relative) of the pages a warp processes in the lane
// starting at flat index base: its range end, the lane end, and n_sel
__device__ __forceinline__ int seg_end(int64_t x_hi, int64_t base, int k, int n) {
  int64_t e = x_hi - base;
  if (e > k) e = k;
  if (e > n) e = n;
  return (int)e;
}

// warp whose range holds flat index x
__device__ __forceinline__ int warp_of(int64_t x, int nw, int64_t T) {
  return (int)(((x + 1) * nw - 1) / T);
}

template <int G>
__global__ void __launch_bounds__(kAttnWarps * 32, kAttnCtasPerSm) attn_kernel(AttnArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, t = threadIdx.x & 31;
  const int w = blockIdx.x * kAttnWarps + warp;
  if (w >= A.nw) return;
  uint8_t* ring = smem + (size_t)warp * kStages * kUnitBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kAttnWarps * kStages * kUnitBytes) +
                   warp * kStages;
  float* psm = reinterpret_cast<float*>(smem + (size_t)kAttnWarps * (kStages * kUnitBytes + kStages * 8)) +
               warp * 16;
  const int64_t x_lo = (int64_t)w * A.T / A.nw, x_hi = (int64_t)(w + 1) * A.T / A.nw;
  if (x_lo >= x_hi) return;
  if (t == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const int k = A.k;
  const int h = t >> 4, d0 = 8 * (t & 15), m4 = (t & 15) >> 1;

  // valid pages of lane a (0 when its request id or n_sel is out of range)
  auto lane_pages = [&](int a, int64_t* unit0) -> int {
    const int64_t gl =
        (int64_t)A.req_ids[a / A.lanes_per_req] * A.lanes_per_req + a % A.lanes_per_req;
    const int n = A.n_sel[a];
    if (gl < 0 || gl >= A.lanes_total || n < 0 || n > k) {
      if (t == 0) record_error(A.err, kErrRange);
      return 0;
    }
    *unit0 = gl * A.C;
    return n;
  };

  // ---- load cursor
  int la = (int)(x_lo / k), lj = 0, lend = 0;
  int64_t lunit0 = 0;
  auto lane_begin = [&]() {
    const int n = lane_pages(la, &lunit0);
    const int64_t base = (int64_t)la * k;
    lj = (int)(max(x_lo, base) - base);
    lend = seg_end(x_hi, base, k, n);
  };
  lane_begin();
  uint32_t it_load = 0, it_use = 0;
  auto issue = [&]() {
    while ((int64_t)la * k < x_hi && lj >= lend) {
      ++la;
      if ((int64_t)la * k < x_hi) lane_begin();
    }
    if ((int64_t)la * k >= x_hi) return;
    if (t == 0) {
      int slot = A.item_slot[(size_t)la * k + lj];
      if (slot < 0 || slot >= A.C) {
        record_error(A.err, kErrRange);
        slot = 0;
      }
      const uint32_t s = it_load % kStages;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars[s], kUnitBytes);
      bulk_load(ring + (size_t)s * kUnitBytes, A.cache + (size_t)(lunit0 + slot) * kUnitBytes,
                kUnitBytes, &bars[s]);
    }
    ++lj;
    ++it_load;
  };
#pragma unroll
  for (int s = 0; s < kStages; ++s) issue();

  bool ok = true;
  // the next segment's lane inputs (request id, n_sel and, for small groups,
  // q) are loaded one segment ahead, so a segment starts without waiting on
  // them
  constexpr int kQPre = G <= 2 ? G : 1;
  const int a_first = (int)(x_lo / k);
  int nx_req = A.req_ids[a_first / A.lanes_per_req], nx_n = A.n_sel[a_first];
  uint4 nx_q[kQPre];
  if constexpr (G <= 2) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      nx_q[g] = *reinterpret_cast<const uint4*>(A.q + ((size_t)a_first * G + g) * kHeadDim + d0);
  }
  for (int a = a_first; (int64_t)a * k < x_hi && ok; ++a) {
    const int req_a = nx_req, nsel_a = nx_n;
    uint4 q_a[kQPre];
#pragma unroll
    for (int g = 0; g < kQPre; ++g) q_a[g] = nx_q[g];
    if ((int64_t)(a + 1) * k < x_hi) {  // lane a + 1 < n_lanes
      nx_req = A.req_ids[(a + 1) / A.lanes_per_req];
      nx_n = A.n_sel[a + 1];
      if constexpr (G <= 2) {
#pragma unroll
        for (int g = 0; g < G; ++g)
          nx_q[g] = *reinterpret_cast<const uint4*>(A.q + ((size_t)(a + 1) * G + g) * kHeadDim + d0);
      }
    }
    int n = nsel_a;
    {
      const int64_t gl = (int64_t)req_a * A.lanes_per_req + a % A.lanes_per_req;
      if (gl < 0 || gl >= A.lanes_total || n < 0 || n > k) {
        if (t == 0) record_error(A.err, kErrRange);
        n = 0;
      }
    }
    const int64_t base = (int64_t)a * k;
    const int jlo = (int)(max(x_lo, base) - base);
    const int jhi = seg_end(x_hi, base, k, n);
    float qv[G][8], mx[G], ls[G], o[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      uint4 raw;
      if constexpr (G <= 2)
        raw = q_a[g];
      else
        raw = *reinterpret_cast<const uint4*>(A.q + ((size_t)a * G + g) * kHeadDim + d0);
      h8_to_f(raw, qv[g]);
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        qv[g][d] *= A.qscale;
        o[g][d] = 0.f;
      }
      mx[g] = -INFINITY;
      ls[g] = 0.f;
    }
    for (int j = jlo; j < jhi; ++j) {
      const uint32_t s = it_use % kStages, par = (it_use / kStages) & 1u;
      if (!mbar_wait(&bars[s], par, A.err)) {
        ok = false;
        break;
      }
      const uint8_t* pg = ring + (size_t)s * kUnitBytes;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int tok = 2 * (i ^ m4) + h;
          float kf[8];
          h8_to_f(*reinterpret_cast<const uint4*>(pg + tok * 256 + d0 * 2), kf);
          float acc = qv[g][0] * kf[0];
#pragma unroll
          for (int d = 1; d < 8; ++d) acc = fmaf(qv[g][d], kf[d], acc);
          v[i] = acc;
        }
        float w4[4], w2[2];
#pragma unroll
        for (int i = 0; i < 4; ++i) w4[i] = v[i] + __shfl_xor_sync(kFull, v[4 + i], 8);
#pragma unroll
        for (int i = 0; i < 2; ++i) w2[i] = w4[i] + __shfl_xor_sync(kFull, w4[2 + i], 4);
        float sc = w2[0] + __shfl_xor_sync(kFull, w2[1], 2);
        sc += __shfl_xor_sync(kFull, sc, 1);  // token 2*m4 + h
        float pm = sc;
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 2));
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 4));
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 8));
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 16));
        const float mn = fmaxf(mx[g], pm);
        const float alpha = exp2f(mx[g] - mn);  // 0 on a segment's first page
        const float p = exp2f(sc - mn);
        ls[g] = ls[g] * alpha + ((t & 1) ? 0.f : p);
        mx[g] = mn;
        if (!(t & 1)) psm[h * 8 + m4] = p;  // slot of token 2*m4 + h
        __syncwarp();
        const float4 pa = *reinterpret_cast<const float4*>(psm + h * 8);
        const float4 pb = *reinterpret_cast<const float4*>(psm + h * 8 + 4);
        const float pt[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
        for (int d = 0; d < 8; ++d) o[g][d] *= alpha;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float vf[8];
          h8_to_f(*reinterpret_cast<const uint4*>(pg + kUnitBytes / 2 + (2 * i + h) * 256 + d0 * 2), vf);
#pragma unroll
          for (int d = 0; d < 8; ++d) o[g][d] = fmaf(pt[i], vf[d], o[g][d]);
        }
        __syncwarp();  // psm reused by the next head / page
      }
      ++it_use;
      issue();
    }
    if (!ok) break;
    // ---- partial of this lane segment: slot a + w
    const int wf = warp_of(base, A.nw, A.T);
    const int parts = warp_of(base + k - 1, A.nw, A.T) - wf + 1;
    float* pc = A.part + ((size_t)a + w) * G * kPartStride;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float lsum = ls[g];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) lsum += __shfl_xor_sync(kFull, lsum, off);
#pragma unroll
      for (int d = 0; d < 8; ++d) o[g][d] += __shfl_xor_sync(kFull, o[g][d], 16);
      if (t < 16) {
        float4* dst = reinterpret_cast<float4*>(pc + g * kPartStride + d0);
        dst[0] = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
        dst[1] = make_float4(o[g][4], o[g][5], o[g][6], o[g][7]);
      }
      if (t == 0) {
        pc[g * kPartStride + 128] = mx[g];
        pc[g * kPartStride + 129] = lsum;
      }
    }
    // the warp's partial stores, then one acq_rel count by lane 0: release
    // publishes them at GPU scope, acquire (for the last warp) orders the
    // other warps' partials before this warp's loads of them
    __syncwarp();
    uint32_t done = 0;
    if (t == 0) done = atom_add_acq_rel_gpu(&A.lane_done[a], 1u);
    done = __shfl_sync(kFull, done, 0);
    __syncwarp();
    if (done == (uint32_t)parts - 1) {
      // combine: lane j holds partial j's (m, l); the o loads are independent
      const float* pl = A.part + ((size_t)a + wf) * G * kPartStride;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float* pj = pl + ((size_t)t * G + g) * kPartStride;
        const bool have = t < parts;
        const float mj = have ? __ldcg(pj + 128) : -INFINITY;
        const float lj2 = have ? __ldcg(pj + 129) : 0.f;
        float M = mj;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(kFull, M, off));
        const float wj = (M == -INFINITY || mj == -INFINITY) ? 0.f : exp2f(mj - M);
        float L = lj2 * wj;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) L += __shfl_xor_sync(kFull, L, off);
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int jj = 0; jj < parts; ++jj) {
          const float wt = __shfl_sync(kFull, wj, jj);
          const float4 oj =
              __ldcg(reinterpret_cast<const float4*>(pl + ((size_t)jj * G + g) * kPartStride) + t);
          O.x = fmaf(oj.x, wt, O.x); O.y = fmaf(oj.y, wt, O.y);
          O.z = fmaf(oj.z, wt, O.z); O.w = fmaf(oj.w, wt, O.w);
        }
        const float inv = L > 0.f ? 1.f / L : 0.f;
        reinterpret_cast<float4*>(A.out + ((size_t)a * G + g) * kHeadDim)[t] =
            make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
      }
      if (t == 0) A.lane_done[a] = 0;
    }
  }
  if (!ok) {
    // drain this warp's copies still in flight (bounded), then leave
    while (it_use < it_load) {
      const uint32_t s = it_use % kStages, par = (it_use / kStages) & 1u;
      if (!mbar_wait(&bars[s], par, nullptr)) break;
      ++it_use;
    }
  }
}

// Warps that share the flat range: as many as fit resident, at least ~4 page
// slots each, and at most 31 per lane so a lane has <= 32 partials.
int attn_warps(int64_t T, int64_t n_lanes, int resident) {
  int64_t nw = std::min<int64_t>(resident, std::max<int64_t>(1, T / 4));
  nw = std::min<int64_t>(nw, std::max<int64_t>(1, 31 * n_lanes));
  if (nw >= kAttnWarps) nw = nw / kAttnWarps * kAttnWarps;
  return (int)nw;
}

template <int G>
int launch_g(const AttnArgs& A, cudaStream_t st) {
  FERRY_TRY(cudaFuncSetAttribute(attn_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kAttnSmem));
  const int blocks = (A.nw + kAttnWarps - 1) / kAttnWarps;
  attn_kernel<G><<<blocks, kAttnWarps * 32, kAttnSmem, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_attn(const AttnArgs& A, int group, cudaStream_t st) {
  switch (group) {
    case 1: return launch_g<1>(A, st);
    case 2: return launch_g<2>(A, st);
    case 4: return launch_g<4>(A, st);
    case 8: return launch_g<8>(A, st);
    default:
      set_error("attention: unsupported GQA group %d", group);
      return FERRY_E_INVAL;
  }
}

int resident_warps(int sms) { return sms * kAttnCtasPerSm * kAttnWarps; }

}  // namespace

size_t attention_partial_slots(int64_t lanes, int sms) { return (size_t)lanes + resident_warps(sms); }

int launch_attention(const ferry_ctx* c, cudaStream_t st, const uint16_t* q,
                     const int32_t* req_ids, int n_req, const int32_t* item_slot,
                     const int32_t* n_sel, float* out) {
  if (n_req <= 0) return FERRY_OK;
  AttnArgs A{};
  A.q = q;
  A.req_ids = req_ids;
  A.lanes_per_req = c->lanes_per_req;
  A.n_lanes = n_req * c->lanes_per_req;
  A.lanes_total = c->lanes;
  A.cache = c->cache;
  A.C = c->cfg.cache_pages;
  A.item_slot = item_slot;
  A.n_sel = n_sel;
  A.k = c->cfg.top_k;
  A.T = (int64_t)A.n_lanes * A.k;
  A.nw = attn_warps(A.T, A.n_lanes, resident_warps(c->num_sms));
  A.part = c->part;
  A.lane_done = c->lane_done;
  A.out = out;
  A.err = c->err;
  A.qscale = 1.4426950408889634f / sqrtf((float)kHeadDim);
  return launch_attn(A, c->group, st);
}

}  // namespace ferry

// ---------------------------------------------------------------------------
// Allocation-free attention entry point.
//
// Some callers cannot call cudaMalloc: a serving engine that hands all of HBM
// to its own KV arena or caching allocator at start-up (an extra cudaMalloc
// fails or fragments that pool), and a decode loop on the latency-critical
// path, where cudaMalloc's implicit device synchronisation would stall every
// stream. ferry_sparse_decode_noalloc serves them: it runs the fp16 CUDA-core
// attention kernel, but its split-K partials, per-lane counters and error word
// live in the fixed-size array below instead of a ctx allocation, and the call
// allocates nothing. The array is a file-scope __device__ object, so every GPU
// that loads this library holds its 4 MiB until the process exits.
//
// Layout of the array: [0, 64 KiB) per-lane completion counters (16384 lanes),
// [64 KiB, 4 MiB - 256) split-K partials, [4 MiB - 256, 4 MiB) the error word
// (kErrTimeout / kErrRange bits, sticky until ferry_sparse_decode_noalloc_status
// reads and clears it).
//
// Host code never passes g_noalloc_scratch itself to a kernel -- in host code
// that name is only a host-side stand-in for the symbol. The device address is
// looked up with cudaGetSymbolAddress the first time the entry point runs on
// a device (with that device current) and cached per device; do that first
// call before any stream capture. All calls share the array and it keeps the
// last call's contents: each call clears the counters it needs before its
// kernel, and calls that overlap on the GPU (different streams, or different
// host threads on one device) race on it.
// ---------------------------------------------------------------------------
namespace ferry {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocCounterBytes = 64u << 10;  // up to 16384 lanes of counters
constexpr size_t kNoAllocErrOffset = kNoAllocScratchBytes - 256;  // the error word

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("sparse_decode_noalloc: device %d out of range", dev);
    return FERRY_E_INVAL;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FERRY_OK;
}

}  // namespace
}  // namespace ferry

extern "C" int ferry_sparse_decode_noalloc(void* stream, const void* d_cache, int cache_pages,
                                           int num_requests, int lanes_per_req, int group,
                                           int top_k, const uint16_t* d_q,
                                           const int32_t* d_req_ids, int n_req,
                                           const int32_t* d_item_slot, const int32_t* d_n_sel,
                                           float* d_out) {
  using namespace ferry;
  if (cache_pages < 1 || num_requests < 1 || lanes_per_req < 1 || top_k < 1 ||
      top_k > cache_pages || (group != 1 && group != 2 && group != 4 && group != 8) ||
      n_req < 0 || n_req > num_requests) {
    set_error("sparse_decode_noalloc: bad geometry");
    return FERRY_E_INVAL;
  }
  if (n_req == 0) return FERRY_OK;
  if (!d_cache || !d_q || !d_req_ids || !d_item_slot || !d_n_sel || !d_out) {
    set_error("sparse_decode_noalloc: NULL buffer");
    return FERRY_E_INVAL;
  }
  const int64_t n_lanes = (int64_t)n_req * lanes_per_req;
  if (n_lanes * 4 > (int64_t)kNoAllocCounterBytes) {
    set_error("sparse_decode_noalloc: %lld lanes exceed the %zu-lane maximum", (long long)n_lanes,
              kNoAllocCounterBytes / 4);
    return FERRY_E_INVAL;
  }
  int dev = 0, sms = 148;
  FERRY_TRY(cudaGetDevice(&dev));
  FERRY_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  // partial slots = lanes + warps; use fewer warps when the array is the limit
  const size_t part_cap = kNoAllocErrOffset - kNoAllocCounterBytes;
  const size_t slot_bytes = (size_t)group * kPartStride * sizeof(float);
  const int64_t T = n_lanes * top_k;
  int nw = attn_warps(T, n_lanes, resident_warps(sms));
  const int64_t fit = (int64_t)(part_cap / slot_bytes) - n_lanes;
  if (fit < 1) {
    set_error("sparse_decode_noalloc: batch needs %zu bytes of partials; the fixed scratch "
              "holds %zu",
              (size_t)(n_lanes + 1) * slot_bytes, part_cap);
    return FERRY_E_INVAL;
  }
  if (nw > fit) nw = fit >= kAttnWarps ? (int)(fit / kAttnWarps * kAttnWarps) : (int)fit;
  void* base = nullptr;
  int rc = noalloc_scratch(dev, &base);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  uint32_t* lane_done = reinterpret_cast<uint32_t*>(base);
  float* part = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + kNoAllocCounterBytes);
  FERRY_TRY(cudaMemsetAsync(lane_done, 0, (size_t)n_lanes * 4, st));

  AttnArgs A{};
  A.q = d_q;
  A.req_ids = d_req_ids;
  A.lanes_per_req = lanes_per_req;
  A.n_lanes = (int)n_lanes;
  A.lanes_total = (int64_t)num_requests * lanes_per_req;
  A.cache = static_cast<const uint8_t*>(d_cache);
  A.C = cache_pages;
  A.item_slot = d_item_slot;
  A.n_sel = d_n_sel;
  A.k = top_k;
  A.T = T;
  A.nw = nw;
  A.part = part;
  A.lane_done = lane_done;
  A.out = d_out;
  // timed-out waits and out-of-range ids / n_sel / slots land in the array's
  // error word (ferry_sparse_decode_noalloc_status)
  A.err = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(base) + kNoAllocErrOffset);
  A.qscale = 1.4426950408889634f / sqrtf((float)kHeadDim);
  return launch_attn(A, group, st);
}

extern "C" int ferry_sparse_decode_noalloc_status(void* stream) {
  using namespace ferry;
  int dev = 0;
  FERRY_TRY(cudaGetDevice(&dev));
  void* base = nullptr;
  int rc = noalloc_scratch(dev, &base);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  uint32_t* err = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(base) + kNoAllocErrOffset);
  uint32_t e = 0;
  FERRY_TRY(cudaStreamSynchronize(st));
  FERRY_TRY(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, st));
  FERRY_TRY(cudaStreamSynchronize(st));
  if (!e) return FERRY_OK;
  FERRY_TRY(cudaMemsetAsync(err, 0, 4, st));
  FERRY_TRY(cudaStreamSynchronize(st));
  if (e & kErrTimeout) return set_error("sparse_decode_noalloc: a device wait timed out"), FERRY_E_TIMEOUT;
  return set_error("sparse_decode_noalloc: an out-of-range request id, n_sel or slot was seen"),
         FERRY_E_RANGE;
}
