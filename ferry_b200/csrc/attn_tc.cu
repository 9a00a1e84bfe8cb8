// attn_tc.cu -- fp8 (e4m3) KV sparse decode attention on the 5th-generation
// tensor cores (tcgen05 + TMEM), for grouped-query attention.
//
// With a GQA group of G q heads per kv head, every K/V element a lane streams
// feeds G multiply-adds, so the QK and PV products become dense tiles; this
// kernel runs them as tcgen05.mma with accumulators in tensor memory.
//
// One CTA of 4 warps (the 4 TMEM lane quadrants) walks lanes (request,
// layer, kv_head); per group of 8 selected pages = 128 tokens:
//   1. TMA: one cp.async.bulk per 4112-byte page unit (K e4m3 | V e4m3 |
//      k_scale | v_scale) into a staging buffer, mbarrier-completed; the
//      next group's copies are issued as soon as staging is converted.
//   2. convert: thread t takes token t, cvt.e4m3x2 -> f16x2 (exact), and
//      writes its K row and V row into canonical UMMA core-matrix layouts
//      (8 x 16-byte rows, SWIZZLE_NONE). The per-page scales stay out of the
//      tiles: k_scale multiplies the scores, v_scale multiplies P.
//   3. S = K Q^T: M = 128 tokens, N = 16 (q heads padded), K = 128 dims,
//      8 x tcgen05.mma kind::f16 (A K-major, B K-major), fp32 in TMEM.
//   4. tcgen05.ld 32x32b: thread t holds token t's 16 scores; online softmax
//      (base 2) per head with the group max reduced through shared memory.
//   5. O^T = V^T P'^T: M = 128 dims, N = 16, K = 128 tokens, A = V^T
//      MN-major, B = P' = p * v_scale (f16) K-major; tcgen05.ld gives thread
//      t dim t of every head, folded into register accumulators with the
//      softmax rescale.
// One elected thread issues the MMAs and commits them to an mbarrier; every
// wait is bounded (on timeout the kernel records FERRY_E_TIMEOUT, drains and
// frees its TMEM).
#include <cuda_fp8.h>

#include "common.cuh"

namespace ferry {
namespace {

constexpr int kTcThreads = 128;
constexpr int kTcPages = 8;          // pages per group: 8 x 16 = 128 tokens
constexpr int kTcN = 16;             // MMA N: q heads padded to 16
constexpr int kStageBytes = kTcPages * kUnitBytesF8;  // 32896
constexpr int kTileBytes = 128 * 128 * 2;            // 32768 (f16 128 x 128)
constexpr int kQPBytes = kTcN * 128 * 2;             // 4096
// shared-memory map (byte offsets, 1024-aligned tiles)
constexpr int kOffStage = 0;
constexpr int kOffK = 33792;                 // >= kStageBytes, 1024-aligned
constexpr int kOffV = kOffK + kTileBytes;    // 66560
constexpr int kOffQ = kOffV + kTileBytes;    // 99328
constexpr int kOffP = kOffQ + kQPBytes;      // 103424
constexpr int kOffRed = kOffP + kQPBytes;    // 107520: 4 warps x 16 heads f32
constexpr int kOffScale = kOffRed + 256;     // 8 pages x (k, v) f32
constexpr int kOffBar = kOffScale + 64;      // 2 mbarriers
constexpr int kOffTmem = kOffBar + 16;       // TMEM base address
constexpr int kTcSmem = kOffTmem + 16;       // 107872
static_assert(kOffK >= kOffStage + kStageBytes, "staging overlaps the K tile");
static_assert(2 * kTcSmem <= 228 * 1024, "two CTAs per SM must fit");
constexpr uint32_t kTmemCols = 32;           // S at cols [0,16), O at [16,32)

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  // SWIZZLE_NONE canonical layout, Blackwell descriptor version 1
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  return d;                // base_offset 0, lbo_mode 0, layout_type 0
}

// kind::f16 instruction descriptor: f32 accumulate, f16 A/B, M = 128, N = 16
__host__ __device__ constexpr uint32_t idesc_f16(bool a_mn_major) {
  return (1u << 4) | (a_mn_major ? (1u << 15) : 0u) | ((uint32_t)(kTcN >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// core-matrix byte offsets (8 rows x 16 B, rows = tokens / heads)
__device__ __forceinline__ uint32_t off_kmajor(int row, int col, int rows_per_chunk_block) {
  // K-major A/B: chunk c = col/8 blocks of (rows/8) core matrices
  return (uint32_t)((((col >> 3) * rows_per_chunk_block) + (row >> 3)) * 128 + (row & 7) * 16 + (col & 7) * 2);
}

struct TcArgs {
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
  float* out;
  uint32_t* err;
  float qscale;
};

template <int G>
__global__ void __launch_bounds__(kTcThreads, 2) attn_tc_kernel(TcArgs A) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* stage = smem + kOffStage;
  uint8_t* Kt = smem + kOffK;
  uint8_t* Vt = smem + kOffV;
  uint8_t* Qt = smem + kOffQ;
  uint8_t* Pt = smem + kOffP;
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  float* scl = reinterpret_cast<float*>(smem + kOffScale);
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);

  if (tid == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // zero Q and P tiles once: padded heads (rows >= G) stay zero
  for (int i = tid; i < (kQPBytes * 2) / 16; i += kTcThreads)
    reinterpret_cast<uint4*>(Qt)[i] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + 16;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t sK = smem_addr(Kt), sV = smem_addr(Vt), sQ = smem_addr(Qt), sP = smem_addr(Pt);
  constexpr uint32_t kIdQK = idesc_f16(false), kIdPV = idesc_f16(true);

  uint32_t ph_tma = 0, ph_mma = 0;
  bool ok = true;
  for (int a = blockIdx.x; a < A.n_lanes && ok; a += gridDim.x) {
    const int64_t gl = (int64_t)A.req_ids[a / A.lanes_per_req] * A.lanes_per_req + a % A.lanes_per_req;
    int n = A.n_sel[a];
    if (gl < 0 || gl >= A.lanes_total || n < 0 || n > A.k) {
      if (tid == 0) record_error(A.err, kErrRange);
      n = 0;
    }
    const uint8_t* lane_cache = A.cache + (size_t)gl * A.C * kUnitBytesF8;
    const int groups = (n + kTcPages - 1) / kTcPages;
    // q heads -> Q tile rows (raw f16; scaling is applied to the scores)
    for (int i = tid; i < G * 16; i += kTcThreads) {
      const int h = i >> 4, c = i & 15;  // 16 chunks of 8 dims per head
      const uint4 v = *reinterpret_cast<const uint4*>(A.q + ((size_t)a * G + h) * kHeadDim + c * 8);
      *reinterpret_cast<uint4*>(Qt + off_kmajor(h, c * 8, 2)) = v;
    }
    float m_run[G], l_thr[G], o_acc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      m_run[h] = -INFINITY;
      l_thr[h] = 0.f;
      o_acc[h] = 0.f;
    }
    auto issue_group = [&](int gi) {
      if (tid != 0 || gi >= groups) return;
      const int p0 = gi * kTcPages, np = min(kTcPages, n - p0);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(bar_tma, (uint32_t)(np * kUnitBytesF8));
      for (int p = 0; p < np; ++p) {
        int slot = A.item_slot[(size_t)a * A.k + p0 + p];
        if (slot < 0 || slot >= A.C) {
          record_error(A.err, kErrRange);
          slot = 0;
        }
        bulk_load(stage + p * kUnitBytesF8, lane_cache + (size_t)slot * kUnitBytesF8, kUnitBytesF8, bar_tma);
      }
    };
    issue_group(0);
    for (int gi = 0; gi < groups; ++gi) {
      const int np = min(kTcPages, n - gi * kTcPages);
      if (!mbar_wait(bar_tma, ph_tma, A.err)) {
        ok = false;
        break;
      }
      ph_tma ^= 1;
      // ---- convert token tid's K and V rows to f16 core matrices
      {
        const int t = tid, p = t >> 4, r = t & 15;
        const bool valid = p < np;
        const uint8_t* unit = stage + p * kUnitBytesF8;
#pragma unroll
        for (int part = 0; part < 2; ++part) {  // 0: K, 1: V
          const uint4* src = reinterpret_cast<const uint4*>(unit + part * 2048 + r * 128);
          uint8_t* dst_tile = part == 0 ? Kt : Vt;
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {  // 16 fp8 = 2 chunks of 8 dims
            // rotate the chunk order per token: 8 consecutive tokens (rows 128 B
            // apart) then hit 8 different bank groups
            const int c16 = (cc + t) & 7;
            uint4 raw = valid ? src[c16] : make_uint4(0, 0, 0, 0);
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
            uint32_t hx[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[j] & 0xFFFF), __NV_E4M3);
              const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[j] >> 16), __NV_E4M3);
              hx[2 * j] = (uint32_t)lo.x | ((uint32_t)lo.y << 16);
              hx[2 * j + 1] = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
            }
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const int d0 = c16 * 16 + half * 8;
              const uint32_t off = part == 0
                                       ? off_kmajor(t, d0, 16)                                            // K: rows = tokens
                                       : (uint32_t)((((t >> 3) * 16) + (d0 >> 3)) * 128 + (t & 7) * 16);  // V^T MN-major
              *reinterpret_cast<uint4*>(dst_tile + off) =
                  make_uint4(hx[4 * half], hx[4 * half + 1], hx[4 * half + 2], hx[4 * half + 3]);
            }
          }
        }
        if (tid < kTcPages) {
          float ks = 0.f, vs = 0.f;
          if (tid < np) {
            ks = *reinterpret_cast<const float*>(stage + tid * kUnitBytesF8 + 4096);
            vs = *reinterpret_cast<const float*>(stage + tid * kUnitBytesF8 + 4100);
          }
          scl[2 * tid] = ks;
          scl[2 * tid + 1] = vs;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      issue_group(gi + 1);  // staging is free again
      // ---- S = K Q^T
      if (tid == 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mma_f16(tmem_s, umma_desc(sK + j * 4096, 2048, 128), umma_desc(sQ + j * 512, 256, 128), kIdQK, j > 0);
        mma_commit(bar_mma);
      }
      if (!mbar_wait(bar_mma, ph_mma, A.err)) {
        ok = false;
        break;
      }
      ph_mma ^= 1;
      tc_fence_after();
      float s[16];
      tmem_ld16(tmem_s + lane_off, s);
      const int t = tid, p = t >> 4;
      const bool valid = p < np;
      const float ks = scl[2 * p] * A.qscale, vs = scl[2 * p + 1];
      float alpha[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float x = valid ? s[h] * ks : -INFINITY;
        s[h] = x;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
        if (lane == 0) red[warp * 16 + h] = x;
      }
      __syncthreads();
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float gm = fmaxf(fmaxf(red[h], red[16 + h]), fmaxf(red[32 + h], red[48 + h]));
        const float mn = fmaxf(m_run[h], gm);
        alpha[h] = exp2f(m_run[h] - mn);
        const float pv = valid ? exp2f(s[h] - mn) : 0.f;
        l_thr[h] = l_thr[h] * alpha[h] + pv;
        m_run[h] = mn;
        // P'^T tile (B of PV, K-major: rows = heads, 8 tokens per 16-byte row)
        *reinterpret_cast<__half*>(Pt + off_kmajor(h, t, 2)) = __float2half_rn(pv * vs);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      // ---- O^T = V^T P'^T
      if (tid == 0) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mma_f16(tmem_o, umma_desc(sV + j * 4096, 2048, 128), umma_desc(sP + j * 512, 256, 128), kIdPV, j > 0);
        mma_commit(bar_mma);
      }
      if (!mbar_wait(bar_mma, ph_mma, A.err)) {
        ok = false;
        break;
      }
      ph_mma ^= 1;
      tc_fence_after();
      float o[16];
      tmem_ld16(tmem_o + lane_off, o);  // thread tid = head dim tid
#pragma unroll
      for (int h = 0; h < G; ++h) o_acc[h] = o_acc[h] * alpha[h] + o[h];
      tc_fence_before();
      __syncthreads();  // S/O TMEM and red[] reusable
    }
    if (!ok) break;
    // ---- finish the lane: l over the 128 token-threads, then O / l
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float x = l_thr[h];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
      if (lane == 0) red[warp * 16 + h] = x;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float L = red[h] + red[16 + h] + red[32 + h] + red[48 + h];
      A.out[((size_t)a * G + h) * kHeadDim + tid] = (groups && L > 0.f) ? o_acc[h] / L : 0.f;
    }
    __syncthreads();
  }
  if (!ok) {
    // drain: a TMA group or an MMA may still be in flight (bounded waits,
    // results ignored) before the TMEM is released
    mbar_wait(bar_tma, ph_tma, nullptr);
    mbar_wait(bar_mma, ph_mma, nullptr);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

}  // namespace

int launch_attention_tc(const ferry_ctx* c, cudaStream_t st, const uint16_t* q, const int32_t* req_ids,
                        int n_req, const int32_t* item_slot, const int32_t* n_sel, float* out) {
  if (n_req <= 0) return FERRY_OK;
  TcArgs A{};
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
  A.out = out;
  A.err = c->err;
  A.qscale = 1.4426950408889634f / sqrtf((float)kHeadDim);
  const int blocks = std::max(1, std::min(A.n_lanes, c->num_sms * 2));
#define FERRY_TC_CASE(GG)                                                                         \
  case GG:                                                                                        \
    FERRY_TRY(cudaFuncSetAttribute(attn_tc_kernel<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   kTcSmem));                                                     \
    attn_tc_kernel<GG><<<blocks, kTcThreads, kTcSmem, st>>>(A);                                  \
    break;
  switch (c->group) {
    FERRY_TC_CASE(1)
    FERRY_TC_CASE(2)
    FERRY_TC_CASE(4)
    FERRY_TC_CASE(8)
    default:
      set_error("attention: unsupported GQA group %d", c->group);
      return FERRY_E_INVAL;
  }
#undef FERRY_TC_CASE
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

}  // namespace ferry
