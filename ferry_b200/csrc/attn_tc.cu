// attn_tc.cu -- sparse decode attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM): e4m3 KV with per-page scales
// (kind::f8f6f4), and fp16 KV with a GQA group (kind::f16).
//
// K and V bytes never pass through registers: per selected page 3-D TMA
// tensor copies (boxes of 128 B x 16 rows, SWIZZLE_128B) drop the page's K
// rows and V rows straight into the canonical UMMA layouts (fp16: two 64-dim
// blocks per tile), and the MMAs read them as they are. fp16 queries and
// softmax weights enter the f16 MMAs directly. For e4m3 they are re-encoded,
// each as three e4m3 terms with a power-of-two scale: x*a = t0 + t1/16 +
// t2/256 carries 12 significant bits (f16 has 11), so the products are as
// exact as with f16 operands; the terms are extra MMA columns (N = 3 x 8 rows,
// padded to 32).
//
// Work split. The batch's groups of 8 selected pages are laid out flat,
// x = lane * gpl + g (gpl = ceil(k / 8)); CTA c of nc owns the contiguous
// range [c*T/nc, (c+1)*T/nc). Each lane segment of a CTA leaves a partial
// (o[128], m, l) per q head in scratch slot lane + c; the CTA completing a
// lane's last segment (atomic count) combines them into out.
//
// A CTA is warp-specialized: warp 8 issues the TMA copies of a 3-stage ring
// (mbarrier full / empty per stage), warp 9 issues the MMAs, and warps 0-7 --
// two warpgroups over the same TMEM lanes, thread t of each = TMEM lane t =
// token t for S, dim t for O, each warpgroup taking half of the q heads --
// run the softmax. Per group of 128 tokens:
//   S = K Q^T      A = K tile K-major, B = Q (e4m3 terms or f16) K-major
//   softmax        base 2, per head; e4m3: k_scale applied to the scores
//   P              f16 weights, or p * v_scale as three e4m3 terms
//   O^T = V^T P^T  A = V tile read MN-major (dims contiguous), B = P MN-major
// S, P and O are double-buffered so the QK of the next group and the PV of
// the last one overlap the softmax. Every wait is bounded (probes suspend in
// hardware up to kWaitHintNs each, about a second in all; on timeout the
// kernel records FERRY_E_TIMEOUT, lets its copies and MMAs land and frees its
// TMEM).
#include <cuda.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace ferry {
namespace {

constexpr int kTcThreads = 320;  // warps 0-7 softmax (two warpgroups on the TMEM lanes), 8 TMA producer, 9 MMA issuer
constexpr int kSoftmaxWarps = 8;
constexpr int kTcPages = 8;      // pages per group: 128 tokens
constexpr int kTcStages = 3;
// each mbarrier probe may suspend a waiting warp this long (it wakes when the
// phase completes): idle roles stop taking issue slots from the softmax warps
constexpr uint32_t kWaitHintNs = 20000;
constexpr int kQP = 4096;            // the Q tile and each P tile
constexpr int kScl = kTcPages * 16;  // e4m3: 16 B per page (k_scale, v_scale, pad)
constexpr uint32_t kTmemCols = 128;  // S[2] at cols 0, 32; O[2] at 64, 96

// Shared-memory map for e4m3 (F8) or fp16 KV, from a 1024-aligned base. Stage
// s holds the K tile at s * kStage and the V tile kHalf after it: e4m3 128
// rows x 128 B each; fp16 two 64-dim blocks of 128 rows x 128 B each.
template <bool F8>
struct TcLayout {
  static constexpr int kHalf = F8 ? 128 * 128 : 2 * 128 * 128;
  static constexpr int kStage = 2 * kHalf;
  static constexpr int kOffQ = kTcStages * kStage;
  static constexpr int kOffP = kOffQ + kQP;
  static constexpr int kOffScl = kOffP + 2 * kQP;  // P double-buffered
  static constexpr int kUsed = kOffScl + (F8 ? kTcStages * kScl : 0);
  static constexpr int kSmem = kUsed + 1024;       // alignment slack
  static constexpr int kCtasPerSm = F8 ? 2 : 1;
};
static_assert(2 * (TcLayout<true>::kSmem + 1024) <= 228 * 1024, "two e4m3 CTAs per SM must fit");
static_assert(TcLayout<false>::kSmem + 1024 <= 228 * 1024, "one fp16 CTA per SM must fit");

// instruction descriptor, f32 accumulate, M = 128: kind::f8f6f4 e4m3 x e4m3
// with N = 32 (3 terms x 8 head rows, padded), or kind::f16 f16 x f16 with
// N = 16 (8 head rows, padded); the operand format codes are 0 in both
__host__ __device__ constexpr uint32_t idesc_tc(bool f8, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (a_mn_major ? (1u << 15) : 0u) | (b_mn_major ? (1u << 16) : 0u) |
         ((uint32_t)((f8 ? 32 : 16) >> 3) << 17) | ((128u >> 4) << 24);
}

template <bool F8>
__device__ __forceinline__ void mma_tc(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  if constexpr (F8)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

// byte offset of (row, col) in a K-major SWIZZLE_128B tile of 128-byte rows:
// 8-row atoms of 1024 B, 16-byte chunk index xor row % 8
__device__ __forceinline__ uint32_t sw128(int row, int col) {
  return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((col >> 4) ^ (row & 7)) << 4) | (col & 15)));
}

__device__ __forceinline__ uint8_t to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float from_e4m3(uint8_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3)));
}

// x (already scaled into [0, 448] in magnitude) as three e4m3 terms:
// x ~ t0 + t1/16 + t2/256
__device__ __forceinline__ void split3(float x, uint8_t* t) {
  t[0] = to_e4m3(x);
  const float r1 = (x - from_e4m3(t[0])) * 16.f;
  t[1] = to_e4m3(r1);
  t[2] = to_e4m3((r1 - from_e4m3(t[1])) * 16.f);
}

__device__ __forceinline__ float2 from_e4m3x2(__nv_fp8x2_storage_t v) {
  return __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(v, __NV_E4M3)));
}

// split3 of two values at once; each term is an e4m3 pair (.x in the low byte)
__device__ __forceinline__ void split3x2(float2 x, uint32_t& t0, uint32_t& t1, uint32_t& t2) {
  const __nv_fp8x2_storage_t a = __nv_cvt_float2_to_fp8x2(x, __NV_SATFINITE, __NV_E4M3);
  const float2 fa = from_e4m3x2(a);
  const float2 r1 = make_float2((x.x - fa.x) * 16.f, (x.y - fa.y) * 16.f);
  const __nv_fp8x2_storage_t b = __nv_cvt_float2_to_fp8x2(r1, __NV_SATFINITE, __NV_E4M3);
  const float2 fb = from_e4m3x2(b);
  const float2 r2 = make_float2((r1.x - fb.x) * 16.f, (r1.y - fb.y) * 16.f);
  const __nv_fp8x2_storage_t c = __nv_cvt_float2_to_fp8x2(r2, __NV_SATFINITE, __NV_E4M3);
  t0 = a;
  t1 = b;
  t2 = c;
}

// largest power of two s with amax * s <= 448 (1 when amax is not positive),
// from the exponent and mantissa bits: 448 = 1.75 * 2^8
__device__ __forceinline__ float pow2_scale(float amax) {
  if (!(amax > 0.f)) return 1.f;
  const int b = __float_as_int(amax);
  const int e = ((b >> 23) & 0xFF) - 127;
  const float m = __int_as_float((b & 0x007FFFFF) | 0x3F800000);
  int sh = (m <= 1.75f ? 8 : 7) - e;
  sh = sh > 127 ? 127 : (sh < -126 ? -126 : sh);
  return __int_as_float((sh + 127) << 23);
}


template <int G, bool F8>
__global__ void __launch_bounds__(kTcThreads, TcLayout<F8>::kCtasPerSm)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmap, TcArgs A) {
  using Lay = TcLayout<F8>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages];
  __shared__ __align__(8) uint64_t s_full[2], s_free[2], p_full[2], o_full[2], o_free[2], q_full;
  __shared__ float red[2][kSoftmaxWarps][8], qred[kSoftmaxWarps][8];
  __shared__ uint32_t tmem_slot, s_flag, s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  const int64_t x_lo = (int64_t)c * A.T / A.nc, x_hi = (int64_t)(c + 1) * A.T / A.nc;
  if (x_lo >= x_hi) return;
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t* Qt = smem + Lay::kOffQ;
  uint8_t* Pt = smem + Lay::kOffP;
  uint8_t* scl = smem + Lay::kOffScl;

  if (tid == 0) {
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&s_free[i], kSoftmaxWarps);  // one arrival per softmax warp
      mbar_init(&p_full[i], kSoftmaxWarps);
      mbar_init(&o_free[i], kSoftmaxWarps);
    }
    mbar_init(&q_full, kSoftmaxWarps);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // zero every tile once: rows the copies never fill (short groups, padded
  // heads and terms) must hold finite values, and zeros in P
  for (int i = tid; i < Lay::kUsed / 16; i += kTcThreads) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int k = A.k;

  // segment of lane a (no pages when its request id or n_sel is out of range)
  auto segment = [&](int a) {
    Seg sg;
    sg.a = a;
    const int64_t gl = (int64_t)A.req_ids[a / A.lanes_per_req] * A.lanes_per_req + a % A.lanes_per_req;
    int n = A.n_sel[a];
    if (gl < 0 || gl >= A.lanes_total || n < 0 || n > k) {
      if (tid == 0) record_error(A.err, kErrRange);
      n = 0;
    }
    sg.n = n;
    sg.unit0 = gl * A.C;
    const int64_t base = (int64_t)a * A.gpl;
    sg.glo = (int)(max(x_lo, base) - base);
    const int ng = (n + kTcPages - 1) / kTcPages;
    sg.ghi = (int)min(x_hi - base, (int64_t)ng);
    return sg;
  };
  const int a_lo = (int)(x_lo / A.gpl);
  auto in_range = [&](int a) { return (int64_t)a * A.gpl < x_hi; };

  // what each role leaves in flight, drained only when a wait gave up
  uint32_t prod_j = 0;           // producer: groups issued
  uint64_t* mma_last = nullptr;  // MMA issuer: barrier of its last commit
  uint32_t mma_par = 0;
  if (warp == kSoftmaxWarps) {
    // ================= producer: stage j of the group sequence into buffer j % 3
    uint32_t& j = prod_j;
    bool ok = true;
    for (int a = a_lo; in_range(a) && ok; ++a) {
      const Seg sg = segment(a);
      for (int g = sg.glo; g < sg.ghi; ++g, ++j) {
        const int s = j % kTcStages, np = min(kTcPages, sg.n - g * kTcPages);
        int slot = lane < np ? A.item_slot[(size_t)a * k + g * kTcPages + lane] : 0;
        if (j >= (uint32_t)kTcStages) ok = __all_sync(0xffffffffu, mbar_wait_sleep<kWaitHintNs>(&empty[s], ((j / kTcStages) - 1) & 1u, A.err));
        if (!ok) break;
        uint8_t* Ks = smem + s * Lay::kStage;
        if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(np * (F8 ? 2 * 2048 + 16 : 4 * 2048)));
        __syncwarp();
        if (lane < np) {
          if (slot < 0 || slot >= A.C) {
            record_error(A.err, kErrRange);
            slot = 0;
          }
          const int64_t unit = sg.unit0 + slot;
          if constexpr (F8) {
            tma_load_3d(Ks + lane * 2048, &tmap, 0, 0, (int)unit, &full[s]);                 // K rows
            tma_load_3d(Ks + Lay::kHalf + lane * 2048, &tmap, 0, 16, (int)unit, &full[s]);   // V rows
            bulk_load(scl + s * kScl + lane * 16, A.cache + (size_t)unit * kUnitBytesF8 + 4096, 16, &full[s]);
          } else {  // dims 0-63 and 64-127 of the K rows, then of the V rows
            tma_load_3d(Ks + lane * 2048, &tmap, 0, 0, (int)unit, &full[s]);
            tma_load_3d(Ks + 128 * 128 + lane * 2048, &tmap, 64, 0, (int)unit, &full[s]);
            tma_load_3d(Ks + Lay::kHalf + lane * 2048, &tmap, 0, 16, (int)unit, &full[s]);
            tma_load_3d(Ks + Lay::kHalf + 128 * 128 + lane * 2048, &tmap, 64, 16, (int)unit, &full[s]);
          }
        }
      }
    }
    if (!ok && lane == 0) atomicOr(&s_abort, 1u);
    __syncwarp();
  } else if (warp == kSoftmaxWarps + 1) {
    // ================= MMA issuer (one thread)
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_tc(F8, false, false), kIdPV = idesc_tc(F8, true, true);
      const uint32_t sQ = smem_addr(Qt);
      bool ok = true;
      uint64_t*& last_bar = mma_last;
      uint32_t& last_par = mma_par;
      auto issue_pv = [&](uint32_t i) {
        const int bi = i & 1, si = i % kTcStages;
        ok = ok && mbar_wait_sleep<kWaitHintNs>(&p_full[bi], (i >> 1) & 1u, A.err);
        if (ok && i >= 2) ok = mbar_wait_sleep<kWaitHintNs>(&o_free[bi], ((i >> 1) - 1) & 1u, A.err);
        if (!ok) return;
        tc_fence_after();
        const uint32_t sV = smem_addr(smem + si * Lay::kStage) + Lay::kHalf, sP = smem_addr(Pt + bi * kQP);
        // A = V read MN-major (dims contiguous; fp16: two 64-dim blocks 16 KiB
        // apart), B = P MN-major unswizzled; K steps of 32 (e4m3) / 16 (f16) tokens
        constexpr int kSteps = F8 ? 4 : 8;
#pragma unroll
        for (int jj = 0; jj < kSteps; ++jj)
          mma_tc<F8>(tmem + 64 + bi * 32, sw128_desc(sV + jj * (F8 ? 4096 : 2048), 128 * 128, 1024),
                     plain_desc(sP + jj * (F8 ? 1024 : 512), 256, 128), kIdPV, jj > 0);
        mma_commit(&o_full[bi]);
        mma_commit(&empty[si]);  // K and V of this stage are no longer read
        last_bar = &o_full[bi];
        last_par = (i >> 1) & 1u;
      };
      uint32_t j = 0, segs = 0;
      for (int a = a_lo; in_range(a) && ok; ++a) {
        const Seg sg = segment(a);
        for (int g = sg.glo; g < sg.ghi && ok; ++g, ++j) {
          const int s = j % kTcStages, b = j & 1;
          if (g == sg.glo) {
            if (j > 0) issue_pv(j - 1);  // the previous segment's last group first
            ok = ok && mbar_wait_sleep<kWaitHintNs>(&q_full, segs & 1u, A.err);
            ++segs;
          }
          ok = ok && mbar_wait_sleep<kWaitHintNs>(&full[s], (j / kTcStages) & 1u, A.err);
          if (ok && j >= 2) ok = mbar_wait_sleep<kWaitHintNs>(&s_free[b], ((j >> 1) - 1) & 1u, A.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sK = smem_addr(smem + s * Lay::kStage);
          // K steps of 32 B along the 128-B rows: 4 x K=32 (e4m3), or 2 dim
          // blocks x 4 x K=16 (f16, blocks 16 KiB apart in K and 2 KiB in Q)
#pragma unroll
          for (int kb = 0; kb < (F8 ? 1 : 2); ++kb)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj)
              mma_tc<F8>(tmem + b * 32, sw128_desc(sK + kb * 128 * 128 + jj * 32, 16, 1024),
                         sw128_desc(sQ + kb * 2048 + jj * 32, 16, 1024), kIdQK, (kb | jj) > 0);
          mma_commit(&s_full[b]);
          last_bar = &s_full[b];
          last_par = (j >> 1) & 1u;
          if (g > sg.glo) issue_pv(j - 1);
        }
      }
      if (ok && j > 0) issue_pv(j - 1);
      if (!ok) atomicOr(&s_abort, 1u);
    }
    __syncwarp();
  } else {
    // ================= softmax: warps 0-7, two warpgroups over the same 128
    // TMEM lanes (thread t = TMEM lane t = token t for S, dim t for O); each
    // warpgroup handles half of the q heads, h0 .. h0 + HG - 1
    constexpr int HG = (G + 1) / 2;
    const int wg = tid >> 7, t = tid & 127, h0 = wg * HG;
    const bool wg_on = h0 < G;  // false only for G == 1, warpgroup 1
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    uint32_t j = 0;
    bool ok = true;
    for (int a = a_lo; in_range(a) && ok; ++a) {
      const Seg sg = segment(a);
      const int glo = sg.glo, ghi = sg.ghi, n = sg.n;
      const int64_t base = (int64_t)a * A.gpl;
      float m_run[HG], l_thr[HG], o_acc[HG], qdiv[HG], alpha_prev[HG];
#pragma unroll
      for (int hh = 0; hh < HG; ++hh) {
        m_run[hh] = -INFINITY;
        l_thr[hh] = 0.f;
        o_acc[hh] = 0.f;
        qdiv[hh] = A.qscale;
        alpha_prev[hh] = 0.f;
      }
      float beta_prev = 1.f;
      if (glo < ghi && !F8) {
        // ---- Q of this lane as f16 rows (K-major, SWIZZLE_128B, two 64-dim
        // blocks 2 KiB apart): thread t = dim t
        if (wg_on)
#pragma unroll
          for (int hh = 0; hh < HG; ++hh)
            *reinterpret_cast<uint16_t*>(Qt + (t >> 6) * 2048 + sw128(h0 + hh, (t & 63) * 2)) =
                A.q[((size_t)a * G + h0 + hh) * kHeadDim + t];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full);
      }
      if (glo < ghi && F8) {
        // ---- Q terms of this lane: thread t = dim t; per-head power-of-two scale
        float qf[HG];
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
          qf[hh] = wg_on ? __half2float(__ushort_as_half(A.q[((size_t)a * G + h0 + hh) * kHeadDim + t])) : 0.f;
          float x = fabsf(qf[hh]);
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
          if (lane == 0) qred[warp][hh] = x;
        }
        softmax_bar_or(false);
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
          const float am = fmaxf(fmaxf(qred[wg * 4][hh], qred[wg * 4 + 1][hh]),
                                 fmaxf(qred[wg * 4 + 2][hh], qred[wg * 4 + 3][hh]));
          const float sc = pow2_scale(am);
          qdiv[hh] = A.qscale / sc;  // score = (S0 + S1/16 + S2/256) * k_scale * qdiv
          if (wg_on) {
            uint8_t tt[3];
            split3(qf[hh] * sc, tt);
#pragma unroll
            for (int jj = 0; jj < 3; ++jj) Qt[sw128(jj * 8 + h0 + hh, t)] = tt[jj];
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full);
      }
      // fold of group i's PV (buffer i & 1) into o_acc
      auto fold = [&](uint32_t i) {
        const int bi = i & 1;
        ok = __all_sync(0xffffffffu, mbar_wait_sleep<kWaitHintNs>(&o_full[bi], (i >> 1) & 1u, A.err));
        if (!ok) return;
        tc_fence_after();
        // thread t = head dim t; this warpgroup's heads only
        float o0[HG], o1[HG], o2[HG];
        tmem_ld_n<HG>(tmem + 64 + bi * 32 + lane_off + h0, o0);
        if constexpr (F8) {
          tmem_ld_n<HG>(tmem + 64 + bi * 32 + lane_off + 8 + h0, o1);
          tmem_ld_n<HG>(tmem + 64 + bi * 32 + lane_off + 16 + h0, o2);
        }
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[bi]);
        const float ib = __frcp_rn(beta_prev);  // exact: a power of two
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
          const float v = F8 ? (o0[hh] + o1[hh] * 0.0625f + o2[hh] * 0.00390625f) * ib : o0[hh];
          o_acc[hh] = o_acc[hh] * alpha_prev[hh] + v;
        }
      };
      for (int g = glo; g < ghi; ++g, ++j) {
        const int s = j % kTcStages, b = j & 1;
        const int np = min(kTcPages, n - g * kTcPages);
        // ---- S of this group (its buffer is released as soon as it is read)
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait_sleep<kWaitHintNs>(&s_full[b], (j >> 1) & 1u, A.err));  // a failed fold stays failed
        float s0[HG], s1[HG], s2[HG];
        if (ok) {
          tc_fence_after();
          // columns jj*8 + h: term jj of head h; this warpgroup's heads only
          tmem_ld_n<HG>(tmem + b * 32 + lane_off + h0, s0);
          if constexpr (F8) {
            tmem_ld_n<HG>(tmem + b * 32 + lane_off + 8 + h0, s1);
            tmem_ld_n<HG>(tmem + b * 32 + lane_off + 16 + h0, s2);
          }
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[b]);
          ok = mbar_wait_sleep<kWaitHintNs>(&full[s], (j / kTcStages) & 1u, A.err);  // the stage's scales
        }
        const int pg = t >> 4;
        const bool valid = pg < np;
        const float ks = F8 ? *reinterpret_cast<const float*>(scl + s * kScl + pg * 16) : 1.f;
        const float vs = F8 ? *reinterpret_cast<const float*>(scl + s * kScl + pg * 16 + 4) : 1.f;
        // weights against the running max of each head, taken as final when
        // no score of the group exceeds it: then the block update gives the
        // same max and alpha = ex2(0) = 1, bit for bit
        float x[HG], pf[HG];
        bool raise = false;
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
          const float sc = F8 ? (s0[hh] + s1[hh] * 0.0625f + s2[hh] * 0.00390625f) * ks : s0[hh];
          x[hh] = valid && ok && wg_on ? sc * qdiv[hh] : -INFINITY;
          raise |= x[hh] > m_run[hh];
          pf[hh] = valid && wg_on ? ex2(x[hh] - m_run[hh]) : 0.f;
        }
        // power-of-two scale of the weights: p * v_scale * beta <= 448 in this group
        float beta = 1.f;
        if constexpr (F8) {
          float vmax = lane < np ? *reinterpret_cast<const float*>(scl + s * kScl + (lane & 7) * 16 + 4) : 0.f;
          vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
          vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
          vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 4));
          beta = pow2_scale(__shfl_sync(0xffffffffu, vmax, 0));
        }
        float alpha[HG], pw[HG];
        if (softmax_bar_or(!ok || raise)) {
          // some score raises a running max (or a wait gave up): block
          // maximum per head of this warpgroup, lane l takes warp l / 8 of
          // the group, head l % 8
          float mx[HG];
#pragma unroll
          for (int hh = 0; hh < HG; ++hh) mx[hh] = x[hh];
          const float wm = warp_max_heads<HG>(mx, lane);  // head (lane >> (5 - log2 HG)) of the group
          if ((lane & ((32 / HG) - 1)) == 0) red[b][warp][lane / (32 / HG)] = wm;
          if (softmax_bar_or(!ok)) {
            ok = false;
            break;
          }
          float gmx = red[b][wg * 4 + ((lane >> 3) & 3)][lane & 7];
          gmx = fmaxf(gmx, __shfl_xor_sync(0xffffffffu, gmx, 8));
          gmx = fmaxf(gmx, __shfl_xor_sync(0xffffffffu, gmx, 16));
#pragma unroll
          for (int hh = 0; hh < HG; ++hh) {
            const float mn = fmaxf(m_run[hh], __shfl_sync(0xffffffffu, gmx, hh));
            alpha[hh] = ex2(m_run[hh] - mn);
            pf[hh] = valid && wg_on ? ex2(x[hh] - mn) : 0.f;
            m_run[hh] = mn;
          }
        } else {
#pragma unroll
          for (int hh = 0; hh < HG; ++hh) alpha[hh] = 1.f;
        }
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
          l_thr[hh] = l_thr[hh] * alpha[hh] + pf[hh];
          pw[hh] = pf[hh] * vs * beta;
        }
        // this token's row of P[b] (MN-major, no swizzle). e4m3: byte jj*8 + h
        // = term jj of head h; f16: element h. Each warpgroup writes its heads'
        // bytes; the rest of the row stays zero. P[b]'s last reader, the PV
        // two groups back, was folded a group ago.
        uint8_t* row = Pt + b * kQP + (t >> 3) * 256 + (t & 7) * 16;
        if (wg_on) {
          if constexpr (F8) {
            uint32_t tw[3] = {0, 0, 0};
#pragma unroll
            for (int i = 0; i < (HG + 1) / 2; ++i) {
              uint32_t t0, t1, t2;
              split3x2(make_float2(pw[2 * i], 2 * i + 1 < HG ? pw[2 * i + 1] : 0.f), t0, t1, t2);
              tw[0] |= t0 << (16 * i);
              tw[1] |= t1 << (16 * i);
              tw[2] |= t2 << (16 * i);
            }
#pragma unroll
            for (int jj = 0; jj < 3; ++jj) {
              uint8_t* dst = row + (jj >> 1) * 128 + (jj & 1) * 8 + h0;
              if (HG == 4) *reinterpret_cast<uint32_t*>(dst) = tw[jj];
              else if (HG == 2) *reinterpret_cast<uint16_t*>(dst) = (uint16_t)tw[jj];
              else *dst = (uint8_t)tw[jj];
            }
          } else {
            uint32_t w[2] = {0, 0};
#pragma unroll
            for (int i = 0; i < (HG + 1) / 2; ++i) {
              const __half2 hv = __floats2half2_rn(pw[2 * i], 2 * i + 1 < HG ? pw[2 * i + 1] : 0.f);
              w[i] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            uint8_t* dst = row + h0 * 2;
            if (HG == 4) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
            else if (HG == 2) *reinterpret_cast<uint32_t*>(dst) = w[0];
            else *reinterpret_cast<uint16_t*>(dst) = (uint16_t)w[0];
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
        // ---- fold the previous group's PV (a failure here ends the loop at
        // the next group's barrier, which every softmax warp reaches)
        if (g > glo && ok) fold(j - 1);
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) alpha_prev[hh] = alpha[hh];
        beta_prev = beta;
      }
      if (ok && glo < ghi) fold(j - 1);
      if (softmax_bar_or(!ok)) {
        ok = false;
        break;
      }
      // ---- partial of this lane segment: slot a + c
      const int cf = cta_of(base, A.nc, A.T);
      const int parts = cta_of(base + A.gpl - 1, A.nc, A.T) - cf + 1;
      float* pc = A.part + ((size_t)a + c) * G * kPartStride;
#pragma unroll
      for (int hh = 0; hh < HG; ++hh) {
        float l = l_thr[hh];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) qred[warp][hh] = l;
        if (wg_on) pc[(h0 + hh) * kPartStride + t] = o_acc[hh];
      }
      softmax_bar_or(false);
      if (wg_on && t < HG) {
        const int h = h0 + t;
        float mv = m_run[0];
#pragma unroll
        for (int hh = 1; hh < HG; ++hh) mv = t == hh ? m_run[hh] : mv;
        pc[h * kPartStride + 128] = mv;
        pc[h * kPartStride + 129] = qred[wg * 4][t] + qred[wg * 4 + 1][t] + qred[wg * 4 + 2][t] + qred[wg * 4 + 3][t];
      }
      // partial stores ordered by the softmax barrier, then one acq_rel count
      // by thread 0: release publishes them at GPU scope, acquire (for the
      // last CTA of the lane) orders the other CTAs' partials before the loads
      softmax_bar_or(false);
      if (tid == 0) s_flag = atom_add_acq_rel_gpu(&A.lane_done[a], 1u) == (uint32_t)(parts - 1);
      softmax_bar_or(false);
      if (s_flag && wg_on) {
        // combine: thread t = dim t of this warpgroup's heads
        const float* pl = A.part + ((size_t)a + cf) * G * kPartStride;
#pragma unroll
        for (int hh = 0; hh < HG; ++hh) {
          const int h = h0 + hh;
          float M = -INFINITY;
          for (int jj = 0; jj < parts; ++jj) M = fmaxf(M, __ldcg(pl + ((size_t)jj * G + h) * kPartStride + 128));
          float L = 0.f, O = 0.f;
          for (int jj = 0; jj < parts; ++jj) {
            const float* pj = pl + ((size_t)jj * G + h) * kPartStride;
            const float mj = __ldcg(pj + 128);
            const float wj = (M == -INFINITY || mj == -INFINITY) ? 0.f : exp2f(mj - M);
            L = fmaf(__ldcg(pj + 129), wj, L);
            O = fmaf(__ldcg(pj + t), wj, O);
          }
          A.out[((size_t)a * G + h) * kHeadDim + t] = L > 0.f ? O / L : 0.f;
        }
      }
      if (s_flag && tid == 0) A.lane_done[a] = 0;
      softmax_bar_or(false);  // qred / s_flag reusable
    }
    if (!ok && tid == 0) atomicOr(&s_abort, 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (s_abort) {
    // a wait gave up: let the copies and MMAs still in flight land (bounded)
    if (warp == kSoftmaxWarps && lane == 0)
      for (uint32_t i = prod_j > (uint32_t)kTcStages ? prod_j - kTcStages : 0; i < prod_j; ++i)
        mbar_wait_sleep<kWaitHintNs>(&full[i % kTcStages], (i / kTcStages) & 1u, nullptr);
    if (warp == kSoftmaxWarps + 1 && lane == 0 && mma_last) mbar_wait_sleep<kWaitHintNs>(mma_last, mma_par, nullptr);  // MMAs complete in order
    __syncthreads();
  }
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

// Tensor map over the cache as (dims, 32 rows, units): rows 0-15 of a unit
// are K, rows 16-31 V. e4m3: 128 B rows, unit stride 4112 B, boxes of 128 B x
// 16 rows; fp16: 256 B rows, unit stride 8192 B, boxes of 64 elements (128 B)
// x 16 rows. Boxes land SWIZZLE_128B in shared memory.
int make_cache_tensor_map(ferry_ctx* c) {
  auto fn = encode_fn();
  if (!fn) return set_error("cuTensorMapEncodeTiled unavailable"), FERRY_E_CUDA;
  const uint64_t units = (uint64_t)c->lanes * c->cfg.cache_pages;
  if (units == 0 || units > 0x7fffffffull) return set_error("cache too large for a tensor map"), FERRY_E_INVAL;
  const bool f8 = c->cfg.kv_dtype == FERRY_KV_E4M3;
  cuuint64_t dims[3] = {128, 32, units};
  cuuint64_t strides[2] = {f8 ? 128u : 256u, (cuuint64_t)(f8 ? kUnitBytesF8 : kUnitBytes)};
  cuuint32_t box[3] = {f8 ? 128u : 64u, 16, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  static_assert(sizeof(CUtensorMap) <= sizeof(c->cache_map), "tensor map storage");
  const CUresult r = fn(reinterpret_cast<CUtensorMap*>(c->cache_map),
                        f8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, c->cache, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error("cuTensorMapEncodeTiled failed (%d)", (int)r), FERRY_E_CUDA;
  return FERRY_OK;
}

int launch_attention_tc(const ferry_ctx* c, cudaStream_t st, const uint16_t* q, const int32_t* req_ids, int n_req,
                        const int32_t* item_slot, const int32_t* n_sel, float* out) {
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
  A.gpl = (A.k + kTcPages - 1) / kTcPages;
  A.T = (int64_t)A.n_lanes * A.gpl;
  const bool f8 = c->cfg.kv_dtype == FERRY_KV_E4M3;
  // resident CTAs, >= 2 groups each, <= 31 per lane (a lane combines <= 32 partials)
  int64_t nc = std::min<int64_t>((int64_t)c->num_sms * (f8 ? TcLayout<true>::kCtasPerSm : TcLayout<false>::kCtasPerSm),
                                 std::max<int64_t>(1, A.T / 2));
  nc = std::min<int64_t>(nc, 31 * (int64_t)A.n_lanes);
  if ((size_t)A.n_lanes + (size_t)nc > attention_partial_slots(c->lanes, c->num_sms))
    return set_error("attention: partial scratch too small"), FERRY_E_STATE;
  A.nc = (int)nc;
  A.part = c->part;
  A.lane_done = c->lane_done;
  A.out = out;
  A.err = c->err;
  A.qscale = 1.4426950408889634f / sqrtf((float)kHeadDim);
  const CUtensorMap* map = reinterpret_cast<const CUtensorMap*>(c->cache_map);
#define FERRY_TC_CASE(GG)                                                                                   \
  case GG:                                                                                                  \
    if (f8) {                                                                                               \
      FERRY_TRY(cudaFuncSetAttribute(attn_tc_kernel<GG, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                     TcLayout<true>::kSmem));                                               \
      attn_tc_kernel<GG, true><<<(unsigned)nc, kTcThreads, TcLayout<true>::kSmem, st>>>(*map, A);           \
    } else {                                                                                                \
      FERRY_TRY(cudaFuncSetAttribute(attn_tc_kernel<GG, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                     TcLayout<false>::kSmem));                                              \
      attn_tc_kernel<GG, false><<<(unsigned)nc, kTcThreads, TcLayout<false>::kSmem, st>>>(*map, A);         \
    }                                                                                                       \
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
