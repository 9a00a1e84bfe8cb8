// attn.cu -- paged sparse decode attention over the selected pages.
//
// Work is split into chunks of `chunk_pages` selected pages of one lane
// (request, layer, kv_head); each warp walks a static stride of chunks and
// streams their pages through a 3-stage shared-memory ring, each stage filled
// by one 8 KiB cp.async.bulk (TMA engine) copy completing on an mbarrier. The
// load cursor runs up to 3 pages ahead across chunk boundaries, so a warp's
// copies never drain between chunks.
//
// Per page and q head (lane l owns dims 4l..4l+3):
//   logits  16 partial dots, then a transpose-reduce across the warp (8+4+2+1
//           shuffles + 1) leaves token t>>1 in lane t,
//   softmax online, base-2 (q pre-scaled by log2(e)/sqrt(128)),
//   PV      p of token tt broadcast from lane 2tt, fp32 FMA into 4 dims.
// Each chunk writes a partial (o[128], m, l) to scratch; the warp that
// finishes a lane's last chunk (atomic count) combines the partials and
// writes out[lane][g][128] in fp32.
#include <mutex>

#include "common.cuh"

namespace ferry {
namespace {

constexpr int kAttnWarps = 4;
constexpr int kStages = 3;
constexpr uint32_t kFull = 0xffffffffu;

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
  int chunk_pages;
  int cpl;
  int total;
  float* part;
  uint32_t* lane_done;
  float* out;
  uint32_t* err;
  float qscale;
};

__device__ __forceinline__ float2 h2f2(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

template <int G>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(AttnArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, t = threadIdx.x & 31;
  uint8_t* ring = smem + (size_t)warp * kStages * kUnitBytes;
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + (size_t)kAttnWarps * kStages * kUnitBytes) + warp * kStages;
  if (t == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int gw = blockIdx.x * kAttnWarps + warp;
  const int nw = gridDim.x * kAttnWarps;
  const int PC = A.chunk_pages;

  // ---- load cursor (runs ahead of compute, across chunks)
  int lc = gw, lp = 0, l_np = 0, l_base = 0;
  int64_t l_unit0 = 0;
  // pages of chunk c (0 when the lane's request id or n_sel is out of range)
  auto chunk_pages = [&](int c, int64_t* unit0) -> int {
    const int a = c / A.cpl, j = c % A.cpl;
    const int64_t gl =
        (int64_t)A.req_ids[a / A.lanes_per_req] * A.lanes_per_req + a % A.lanes_per_req;
    const int n = A.n_sel[a];
    if (gl < 0 || gl >= A.lanes_total || n < 0 || n > A.k) {
      if (t == 0 && j == 0) record_error(A.err, kErrRange);
      return 0;
    }
    *unit0 = gl * A.C;
    return max(0, min(PC, n - j * PC));
  };
  auto load_chunk = [&](int c) {
    l_np = chunk_pages(c, &l_unit0);
    l_base = (c / A.cpl) * A.k + (c % A.cpl) * PC;
  };
  if (lc < A.total) load_chunk(lc);
  uint32_t it_load = 0, it_use = 0;
  auto issue = [&]() {
    while (lc < A.total && lp >= l_np) {
      lc += nw;
      lp = 0;
      if (lc < A.total) load_chunk(lc);
    }
    if (lc >= A.total) return;
    if (t == 0) {
      int slot = A.item_slot[l_base + lp];
      if (slot < 0 || slot >= A.C) {
        record_error(A.err, kErrRange);
        slot = 0;
      }
      const uint32_t s = it_load % kStages;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars[s], kUnitBytes);
      bulk_load(ring + (size_t)s * kUnitBytes, A.cache + (size_t)(l_unit0 + slot) * kUnitBytes,
                kUnitBytes, &bars[s]);
    }
    ++lp;
    ++it_load;
  };
#pragma unroll
  for (int s = 0; s < kStages; ++s) issue();

  bool ok = true;
  for (int c = gw; c < A.total && ok; c += nw) {
    const int a = c / A.cpl;
    int64_t unit0_unused = 0;
    const int np = chunk_pages(c, &unit0_unused);
    float qv[G][4], m[G], l[G], o[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint2 raw = *reinterpret_cast<const uint2*>(A.q + ((size_t)a * G + g) * kHeadDim + t * 4);
      const float2 x = h2f2(raw.x), y = h2f2(raw.y);
      qv[g][0] = x.x * A.qscale; qv[g][1] = x.y * A.qscale;
      qv[g][2] = y.x * A.qscale; qv[g][3] = y.y * A.qscale;
      m[g] = -INFINITY; l[g] = 0.f;
      o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
    }
    for (int pp = 0; pp < np; ++pp) {
      const uint32_t s = it_use % kStages, par = (it_use / kStages) & 1u;
      if (!mbar_wait(&bars[s], par, A.err)) {
        ok = false;
        break;
      }
      const uint8_t* pg = ring + (size_t)s * kUnitBytes;
      const uint2* Kr = reinterpret_cast<const uint2*>(pg) + t;
      const uint2* Vr = reinterpret_cast<const uint2*>(pg + kUnitBytes / 2) + t;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v[16];
#pragma unroll
        for (int tt = 0; tt < 16; ++tt) {
          const uint2 kk = Kr[tt * 32];
          const float2 k01 = h2f2(kk.x), k23 = h2f2(kk.y);
          float acc = qv[g][0] * k01.x;
          acc = fmaf(qv[g][1], k01.y, acc);
          acc = fmaf(qv[g][2], k23.x, acc);
          v[tt] = fmaf(qv[g][3], k23.y, acc);
        }
        // transpose-reduce: token (t >> 1) ends in lanes t and t^1
        float w8[8], w4[4], w2[2];
        const bool b4 = t & 16, b3 = t & 8, b2 = t & 4, b1 = t & 2;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          w8[i] = (b4 ? v[8 + i] : v[i]) + __shfl_xor_sync(kFull, b4 ? v[i] : v[8 + i], 16);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          w4[i] = (b3 ? w8[4 + i] : w8[i]) + __shfl_xor_sync(kFull, b3 ? w8[i] : w8[4 + i], 8);
#pragma unroll
        for (int i = 0; i < 2; ++i)
          w2[i] = (b2 ? w4[2 + i] : w4[i]) + __shfl_xor_sync(kFull, b2 ? w4[i] : w4[2 + i], 4);
        float sc = (b1 ? w2[1] : w2[0]) + __shfl_xor_sync(kFull, b1 ? w2[0] : w2[1], 2);
        sc += __shfl_xor_sync(kFull, sc, 1);
        float pm = sc;
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 2));
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 4));
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 8));
        pm = fmaxf(pm, __shfl_xor_sync(kFull, pm, 16));
        const float mn = fmaxf(m[g], pm);
        const float alpha = exp2f(m[g] - mn);  // 0 on the first page (m = -inf)
        const float p = exp2f(sc - mn);
        l[g] = l[g] * alpha + ((t & 1) ? 0.f : p);
#pragma unroll
        for (int d = 0; d < 4; ++d) o[g][d] *= alpha;
        m[g] = mn;
#pragma unroll
        for (int tt = 0; tt < 16; ++tt) {
          const float pt = __shfl_sync(kFull, p, 2 * tt);
          const uint2 vv = Vr[tt * 32];
          const float2 v01 = h2f2(vv.x), v23 = h2f2(vv.y);
          o[g][0] = fmaf(pt, v01.x, o[g][0]);
          o[g][1] = fmaf(pt, v01.y, o[g][1]);
          o[g][2] = fmaf(pt, v23.x, o[g][2]);
          o[g][3] = fmaf(pt, v23.y, o[g][3]);
        }
      }
      __syncwarp();
      ++it_use;
      issue();
    }
    if (!ok) break;
    // ---- partial of this chunk
    float* pc = A.part + (size_t)c * G * kPartStride;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float ls = l[g];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) ls += __shfl_xor_sync(kFull, ls, off);
      reinterpret_cast<float4*>(pc + g * kPartStride)[t] = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
      if (t == 0) {
        pc[g * kPartStride + 128] = m[g];
        pc[g * kPartStride + 129] = ls;
      }
    }
    __threadfence();
    __syncwarp();
    uint32_t done = 0;
    if (t == 0) done = atomicAdd(&A.lane_done[a], 1u);
    done = __shfl_sync(kFull, done, 0);
    if (done == (uint32_t)A.cpl - 1) {
      __threadfence();
      const float* pl = A.part + (size_t)a * A.cpl * G * kPartStride;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float M = -INFINITY;
        for (int jj = 0; jj < A.cpl; ++jj) M = fmaxf(M, __ldcg(pl + ((size_t)jj * G + g) * kPartStride + 128));
        float L = 0.f;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
        if (M != -INFINITY) {
          for (int jj = 0; jj < A.cpl; ++jj) {
            const float* pj = pl + ((size_t)jj * G + g) * kPartStride;
            const float mj = __ldcg(pj + 128);
            if (mj == -INFINITY) continue;
            const float w = exp2f(mj - M);
            L = fmaf(__ldcg(pj + 129), w, L);
            const float4 oj = __ldcg(reinterpret_cast<const float4*>(pj) + t);
            O.x = fmaf(oj.x, w, O.x); O.y = fmaf(oj.y, w, O.y);
            O.z = fmaf(oj.z, w, O.z); O.w = fmaf(oj.w, w, O.w);
          }
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

}  // namespace

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
  A.chunk_pages = c->chunk_pages;
  A.cpl = c->chunks_per_lane;
  A.total = A.n_lanes * A.cpl;
  A.part = c->part;
  A.lane_done = c->lane_done;
  A.out = out;
  A.err = c->err;
  A.qscale = 1.4426950408889634f / sqrtf((float)kHeadDim);
  const size_t smem = (size_t)kAttnWarps * kStages * (kUnitBytes + 8);
  const int max_blocks = c->num_sms * 2;
  const int blocks = std::max(1, std::min(max_blocks, (A.total + kAttnWarps - 1) / kAttnWarps));
#define FERRY_ATTN_CASE(GG)                                                                   \
  case GG: {                                                                                  \
    FERRY_TRY(cudaFuncSetAttribute(attn_kernel<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   (int)smem));                                               \
    attn_kernel<GG><<<blocks, kAttnWarps * 32, smem, st>>>(A);                                \
    break;                                                                                    \
  }
  switch (c->group) {
    FERRY_ATTN_CASE(1)
    FERRY_ATTN_CASE(2)
    FERRY_ATTN_CASE(4)
    FERRY_ATTN_CASE(8)
    default:
      set_error("attention: unsupported GQA group %d", c->group);
      return FERRY_E_INVAL;
  }
#undef FERRY_ATTN_CASE
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

}  // namespace ferry

// ---------------------------------------------------------------------------
// Allocation-free attention entry point.
//
// Some callers cannot call cudaMalloc: a serving engine that hands all of HBM
// to its own KV arena or caching allocator at start-up (an extra cudaMalloc
// fails or fragments that pool), and a decode loop on the latency-critical
// path, where cudaMalloc's implicit device synchronisation would stall every
// stream. ferry_sparse_decode_noalloc serves them: it runs the same attention
// kernel, but its split-K partials and per-lane counters live in the
// fixed-size array below instead of a ctx allocation, and the call allocates
// nothing. The array is a file-scope __device__ object, so every GPU that
// loads this library holds its 4 MiB until the process exits.
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
  // chunking as in the ctx path, coarsened until the partials fit the array
  const size_t part_cap = kNoAllocScratchBytes - kNoAllocCounterBytes;
  const int64_t warps = (int64_t)sms * 2 * 4;
  int pc = 16;
  while (pc > 2 && n_lanes * ((top_k + pc - 1) / pc) < 4 * warps) pc >>= 1;
  auto need = [&](int p) {
    return (size_t)n_lanes * ((top_k + p - 1) / p) * group * kPartStride * sizeof(float);
  };
  while (need(pc) > part_cap && pc < top_k) pc *= 2;
  if (need(pc) > part_cap) {
    set_error("sparse_decode_noalloc: batch needs %zu bytes of partials; the fixed scratch "
              "holds %zu",
              need(pc), part_cap);
    return FERRY_E_INVAL;
  }
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
  A.chunk_pages = pc;
  A.cpl = (top_k + pc - 1) / pc;
  A.total = (int)(n_lanes * A.cpl);
  A.part = part;
  A.lane_done = lane_done;
  A.out = d_out;
  A.err = nullptr;  // no error word here: out-of-range ids are skipped, not reported
  A.qscale = 1.4426950408889634f / sqrtf((float)kHeadDim);
  const size_t smem = (size_t)kAttnWarps * kStages * (kUnitBytes + 8);
  const int blocks = std::max(1, std::min(sms * 2, (A.total + kAttnWarps - 1) / kAttnWarps));
  switch (group) {
#define FERRY_NOALLOC_CASE(GG)                                                                \
  case GG:                                                                                    \
    FERRY_TRY(cudaFuncSetAttribute(attn_kernel<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   (int)smem));                                               \
    attn_kernel<GG><<<blocks, kAttnWarps * 32, smem, st>>>(A);                                \
    break;
    FERRY_NOALLOC_CASE(1)
    FERRY_NOALLOC_CASE(2)
    FERRY_NOALLOC_CASE(4)
    FERRY_NOALLOC_CASE(8)
#undef FERRY_NOALLOC_CASE
  }
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}
