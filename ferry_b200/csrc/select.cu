// select.cu -- top-k page selection by q . mean-key page summary.
//
// One CTA per batch lane (request, layer, kv_head). Phase 1 scores every page
// of the lane's context: a warp per page, lane l holding dims 4l..4l+3 of the
// fp32 summary (one 16-byte load), dot product in the fixed order
// q[4l]*s[4l] -> fma 4l+1..4l+3 -> butterfly add over 16,8,4,2,1, and the
// maximum over the GQA group (first head wins ties). Phase 2 finds the k-th
// largest order-preserving key with a 4-pass 8-bit radix select in shared
// memory. Phase 3 emits, in ascending page order, every page whose key is
// larger plus the lowest-id pages equal to it -- ties go to the lower page id.
// Every fp32 operation and its order is fixed, so any IEEE-754 implementation
// of the same steps reproduces the selection bit for bit.
#include "common.cuh"

namespace ferry {
namespace {

constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;

__device__ __forceinline__ uint32_t block_excl_scan(bool flag, uint32_t* warp_tot,
                                                    uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t m = __ballot_sync(0xffffffffu, flag);
  const uint32_t below = __popc(m & ((1u << lane) - 1u));
  if (lane == 0) warp_tot[warp] = __popc(m);
  __syncthreads();
  uint32_t before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kSelWarps; ++w) {
    const uint32_t t = warp_tot[w];
    before += (w < warp) ? t : 0u;
    all += t;
  }
  __syncthreads();  // warp_tot reusable after this
  *total = all;
  return before + below;
}

template <int G>
__global__ void __launch_bounds__(kSelThreads) select_kernel(
    const uint16_t* __restrict__ q, const int32_t* __restrict__ req_ids, int lanes_per_req,
    const int32_t* __restrict__ ctx_pages, const int64_t* __restrict__ req_base,
    const float* __restrict__ summ, uint64_t pool_units,
    int N, int k, int num_requests, int32_t* __restrict__ sel_out,
    int32_t* __restrict__ n_sel_out, uint32_t* err) {
  extern __shared__ uint32_t keys[];  // N entries
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_tot[kSelWarps];
  __shared__ uint32_t s_prefix, s_krem;

  const int a = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int req = req_ids[a / lanes_per_req];
  int32_t* out = sel_out + (size_t)a * k;
  if (req < 0 || req >= num_requests) {
    if (threadIdx.x == 0) {
      record_error(err, kErrRange);
      n_sel_out[a] = 0;
    }
    for (int j = threadIdx.x; j < k; j += kSelThreads) out[j] = -1;
    return;
  }
  int np = ctx_pages[req];
  if (np < 0 || np > N) {
    if (threadIdx.x == 0) record_error(err, kErrRange);
    np = np < 0 ? 0 : N;
  }

  // ---- phase 1: scores
  float qv[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint2 raw =
        *reinterpret_cast<const uint2*>(q + ((size_t)a * G + g) * kHeadDim + lane * 4);
    const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    qv[g][0] = x.x; qv[g][1] = x.y; qv[g][2] = y.x; qv[g][3] = y.y;
  }
  // pool units of this lane: request home + lane-in-request * N (+ page)
  const uint64_t ubase = (uint64_t)(req_base[req] + (int64_t)(a % lanes_per_req) * N);
  constexpr int U = 4;
  for (int p0 = warp * U; p0 < np; p0 += kSelWarps * U) {
    float4 s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = p0 + u;
      if (p < np) {
        const uint64_t unit = (ubase + (uint64_t)p) % pool_units;
        s[u] = __ldg(reinterpret_cast<const float4*>(summ + unit * kHeadDim) + lane);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = p0 + u;
      if (p >= np) break;  // warp-uniform
      float best = 0.f;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v = __fmul_rn(qv[g][0], s[u].x);
        v = __fmaf_rn(qv[g][1], s[u].y, v);
        v = __fmaf_rn(qv[g][2], s[u].z, v);
        v = __fmaf_rn(qv[g][3], s[u].w, v);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
        best = (g == 0 || v > best) ? v : best;
      }
      if (lane == 0) keys[p] = order_key(best);
    }
  }
  __syncthreads();

  if (np <= k) {
    for (int j = threadIdx.x; j < k; j += kSelThreads) out[j] = j < np ? j : -1;
    if (threadIdx.x == 0) n_sel_out[a] = np;
    return;
  }

  // ---- phase 2: radix select of the k-th largest key
  uint32_t prefix = 0, mask = 0, krem = (uint32_t)k;
#pragma unroll 1
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[threadIdx.x] = 0;  // kSelThreads == 256 bins
    __syncthreads();
    for (int p = threadIdx.x; p < np; p += kSelThreads) {
      const uint32_t key = keys[p];
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
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
            s_prefix = prefix | ((uint32_t)(255 - (lane * 8 + j)) << shift);
            s_krem = krem - run;
            break;
          }
          run += c[j];
        }
      }
    }
    __syncthreads();
    prefix = s_prefix;
    krem = s_krem;
    mask |= 255u << shift;
  }
  const uint32_t T = prefix;

  // ---- phase 3: ordered emission
  uint32_t run_eq = 0, run_sel = 0;
  for (int base = 0; base < np; base += kSelThreads) {
    const int p = base + threadIdx.x;
    const uint32_t key = p < np ? keys[p] : 0u;
    const bool gt = p < np && key > T;
    const bool eq = p < np && key == T;
    uint32_t tot_eq, tot_sel;
    const uint32_t eq_rank = run_eq + block_excl_scan(eq, warp_tot, &tot_eq);
    const bool take = gt || (eq && eq_rank < krem);
    const uint32_t pos = run_sel + block_excl_scan(take, warp_tot, &tot_sel);
    if (take) out[pos] = p;
    run_eq += tot_eq;
    run_sel += tot_sel;
  }
  if (threadIdx.x == 0) n_sel_out[a] = k;
}

}  // namespace

int launch_select(const ferry_ctx* c, cudaStream_t st, const uint16_t* q,
                  const int32_t* req_ids, int n_req, int32_t* sel, int32_t* n_sel) {
  if (n_req <= 0) return FERRY_OK;
  const int N = c->cfg.max_pages, k = c->cfg.top_k;
  const unsigned grid = (unsigned)(n_req * c->lanes_per_req);
  const size_t smem = (size_t)N * sizeof(uint32_t);
#define FERRY_SEL_CASE(GG)                                                                    \
  case GG: {                                                                                  \
    auto kern = select_kernel<GG>;                                                            \
    if (smem > 48 * 1024)                                                                     \
      FERRY_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                     (int)smem));                                             \
    kern<<<grid, kSelThreads, smem, st>>>(q, req_ids, c->lanes_per_req, c->ctx_pages, c->req_base, c->summ, \
                                          c->pool_units, N, k, c->cfg.num_requests, sel,      \
                                          n_sel, c->err);                                     \
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
