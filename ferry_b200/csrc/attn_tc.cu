// attn_tc.cu -- fp8 (e4m3) KV sparse decode attention on the 5th-generation
// tensor cores (tcgen05.mma kind::f8f6f4, accumulators in TMEM).
//
// K and V bytes never pass through registers: per selected page a 3-D TMA
// tensor copy (box 128 B x 16 rows, SWIZZLE_128B) drops the page's K rows and
// V rows straight into the canonical UMMA layouts, and the MMAs read them as
// e4m3. Only queries and softmax weights are re-encoded, each as three e4m3
// terms with a power-of-two scale: x*a = t0 + t1/16 + t2/256 carries 12
// significant bits (f16 has 11), so the products are as exact as with f16
// operands; the terms are extra MMA columns (N = 3 x 8 rows, padded to 32).
//
// Work split. The batch's groups of 8 selected pages are laid out flat,
// x = lane * gpl + g (gpl = ceil(k / 8)); CTA c of nc owns the contiguous
// range [c*T/nc, (c+1)*T/nc). Each lane segment of a CTA leaves a partial
// (o[128], m, l) per q head in scratch slot lane + c; the CTA completing a
// lane's last segment (atomic count) combines them into out.
//
// Per group (128 tokens; thread t = TMEM lane t = token t for S, dim t for O):
//   S = K Qt^T     A = K tile [128 tok][128 B] K-major, B = Q terms, 4 x K=32
//   softmax        base 2, per head; k_scale applied to the scores
//   P' = p*v_scale as three e4m3 terms (rows = head x term) -> P tile
//   O^T = V^T P'^T A = V tile read MN-major (dims contiguous), B = P tile
// A CTA keeps kTcStages groups in flight on mbarriers; every wait is bounded
// (on timeout the kernel records FERRY_E_TIMEOUT, lets its copies and MMAs
// land and frees its TMEM).
#include <cuda.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace ferry {
namespace {

constexpr int kTcThreads = 128;
constexpr int kTcPages = 8;                       // pages per group: 128 tokens
constexpr int kTcN = 32;                          // MMA N: 3 terms x 8 head rows, padded
constexpr int kTcStages = 3;
constexpr int kTile = 128 * 128;                  // 16 KiB: 128 rows x 128 B (e4m3)
constexpr int kQP = kTcN * 128;                   // 4 KiB: 32 rows x 128 B
constexpr int kScl = kTcPages * 16;               // 16 B per page: k_scale, v_scale, pad
// dynamic shared memory, from a 1024-aligned base
constexpr int kOffK = 0;                          // stage s: K at s * 2 * kTile, V after it
constexpr int kOffQ = kTcStages * 2 * kTile;      // 98304
constexpr int kOffP = kOffQ + kQP;
constexpr int kOffScl = kOffP + kQP;
constexpr int kTcSmemUsed = kOffScl + kTcStages * kScl;
constexpr int kTcSmem = kTcSmemUsed + 1024;       // alignment slack
static_assert(2 * (kTcSmem + 1024) <= 228 * 1024, "two CTAs per SM must fit");
constexpr uint32_t kTmemCols = 64;                // S at cols [0,32), O at [32,64)

// UMMA shared-memory descriptor without swizzle (layout type 0), version 1
__device__ __forceinline__ uint64_t plain_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// UMMA shared-memory descriptor, SWIZZLE_128B (layout type 2), version 1
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f8f6f4 instruction descriptor: e4m3 A and B, f32 accumulate, M = 128, N = 32
__host__ __device__ constexpr uint32_t idesc_f8(bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (a_mn_major ? (1u << 15) : 0u) | (b_mn_major ? (1u << 16) : 0u) |
         ((uint32_t)(kTcN >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 3-D tensor copy global -> shared (no multicast), completion on the mbarrier
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
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

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// maximum over the warp of G values per lane at once: levels pair lanes
// l ^ 16, l ^ 8, ...; while more than one value is left each pair swaps
// halves (the lane with the level's bit set keeps the upper half). Lane l
// returns the maximum of value l >> (5 - log2 G).
template <int G>
__device__ __forceinline__ float warp_max_heads(float (&v)[G], int lane) {
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const int o = 16 >> j;
    const int n = G >> j;
    if (n > 1) {
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = up ? v[i] : v[i + n / 2];
        const float keep = up ? v[i + n / 2] : v[i];
        v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, o));
      }
    } else {
      v[0] = fmaxf(v[0], __shfl_xor_sync(0xffffffffu, v[0], o));
    }
  }
  return v[0];
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
  int gpl;     // groups per lane: ceil(k / 8)
  int64_t T;   // n_lanes * gpl
  int nc;      // CTAs sharing the flat range
  float* part;
  uint32_t* lane_done;
  float* out;
  uint32_t* err;
  float qscale;  // log2(e) / sqrt(head_dim)
};

__device__ __forceinline__ int cta_of(int64_t x, int nc, int64_t T) { return (int)(((x + 1) * nc - 1) / T); }

template <int G>
__global__ void __launch_bounds__(kTcThreads, 2) attn_tc_kernel(const __grid_constant__ CUtensorMap tmap, TcArgs A) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kTcStages];
  __shared__ __align__(8) uint64_t bar_s, bar_o;
  __shared__ float red[4][8];
  __shared__ uint32_t tmem_slot, s_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  const int64_t x_lo = (int64_t)c * A.T / A.nc, x_hi = (int64_t)(c + 1) * A.T / A.nc;
  if (x_lo >= x_hi) return;
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t* Qt = smem + kOffQ;
  uint8_t* Pt = smem + kOffP;
  uint8_t* scl = smem + kOffScl;

  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) mbar_init(&full[s], 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // zero every tile once: rows the copies never fill (short groups, padded
  // heads) must hold finite values
  for (int i = tid; i < kTcSmemUsed / 16; i += kTcThreads) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot, tmem_s = tmem, tmem_o = tmem + 32;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  constexpr uint32_t kIdQK = idesc_f8(false, false), kIdPV = idesc_f8(true, true);
  const int k = A.k;

  // valid pages of lane a (0 when its request id or n_sel is out of range)
  auto lane_pages = [&](int a, int64_t* unit0) -> int {
    const int64_t gl = (int64_t)A.req_ids[a / A.lanes_per_req] * A.lanes_per_req + a % A.lanes_per_req;
    const int n = A.n_sel[a];
    if (gl < 0 || gl >= A.lanes_total || n < 0 || n > k) {
      if (tid == 0) record_error(A.err, kErrRange);
      return 0;
    }
    *unit0 = gl * A.C;
    return n;
  };

  // ---- producer (warp 0): a cursor over the same flat range, one group ahead
  // of the copies it issues; lane p holds the cache slot of page p of the
  // group under the cursor, loaded a group early so the copies never wait on it
  int la = (int)(x_lo / A.gpl), lg = 0, lgend = 0, lnp = 0, nslot = 0;
  int64_t lunit0 = 0;
  bool more = false;
  auto lane_begin = [&]() {
    lnp = lane_pages(la, &lunit0);
    const int64_t base = (int64_t)la * A.gpl;
    lg = (int)(max(x_lo, base) - base);
    const int64_t e = x_hi - base;
    const int ng = (lnp + kTcPages - 1) / kTcPages;
    lgend = (int)(e < ng ? e : ng);
  };
  auto advance = [&]() {  // to the next group with pages, then prefetch its slots
    while ((int64_t)la * A.gpl < x_hi && lg >= lgend) {
      ++la;
      if ((int64_t)la * A.gpl < x_hi) lane_begin();
    }
    more = (int64_t)la * A.gpl < x_hi;
    if (more) {
      const int p0 = lg * kTcPages;
      nslot = lane < min(kTcPages, lnp - p0) ? A.item_slot[(size_t)la * k + p0 + lane] : 0;
    }
  };
  uint32_t it_load = 0, it_use = 0;
  auto issue = [&]() {
    if (warp != 0 || !more) return;
    const int s = it_load % kTcStages;
    const int np = min(kTcPages, lnp - lg * kTcPages);
    uint8_t* Ks = smem + kOffK + s * 2 * kTile;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(np * (2 * 2048 + 16)));
    __syncwarp();
    if (lane < np) {
      int slot = nslot;
      if (slot < 0 || slot >= A.C) {
        record_error(A.err, kErrRange);
        slot = 0;
      }
      const int64_t unit = lunit0 + slot;
      tma_load_3d(Ks + lane * 2048, &tmap, 0, 0, (int)unit, &full[s]);           // K rows
      tma_load_3d(Ks + kTile + lane * 2048, &tmap, 0, 16, (int)unit, &full[s]);  // V rows
      bulk_load(scl + s * kScl + lane * 16, A.cache + (size_t)unit * kUnitBytesF8 + 4096, 16, &full[s]);
    }
    ++lg;
    ++it_load;
    advance();
  };
  if (warp == 0) {
    lane_begin();
    advance();
  }
  for (int s = 0; s < kTcStages; ++s) issue();

  uint32_t ph_s = 0, ph_o = 0;
  bool ok = true, mma_pending_s = false, mma_pending_o = false;
  const int t = tid;
  for (int a = (int)(x_lo / A.gpl); (int64_t)a * A.gpl < x_hi && ok; ++a) {
    int64_t unit0 = 0;
    const int n = lane_pages(a, &unit0);
    const int64_t base = (int64_t)a * A.gpl;
    const int glo = (int)(max(x_lo, base) - base);
    const int ng = (n + kTcPages - 1) / kTcPages;
    const int ghi = (int)min(x_hi - base, (int64_t)ng);
    float m_run[G], l_thr[G], o_acc[G], qdiv[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      m_run[h] = -INFINITY;
      l_thr[h] = 0.f;
      o_acc[h] = 0.f;
      qdiv[h] = 0.f;
    }
    if (glo < ghi) {
      // ---- Q terms of this lane: thread t = dim t; per-head power-of-two scale
      float qf[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        qf[h] = __half2float(__ushort_as_half(A.q[((size_t)a * G + h) * kHeadDim + t]));
        float x = fabsf(qf[h]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
        if (lane == 0) red[warp][h] = x;
      }
      __syncthreads();
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float am = fmaxf(fmaxf(red[0][h], red[1][h]), fmaxf(red[2][h], red[3][h]));
        const float sc = pow2_scale(am);
        qdiv[h] = A.qscale / sc;  // score = (S0 + S1/16 + S2/256) * k_scale * qdiv
        uint8_t tt[3];
        split3(qf[h] * sc, tt);
#pragma unroll
        for (int j = 0; j < 3; ++j) Qt[sw128(j * 8 + h, t)] = tt[j];
      }
      fence_proxy_async_smem();
      __syncthreads();  // red reusable; Q tile complete
    }
    for (int g = glo; g < ghi; ++g) {
      const int s = it_use % kTcStages;
      const uint32_t par = (it_use / kTcStages) & 1u;
      const int np = min(kTcPages, n - g * kTcPages);
      ok = mbar_wait(&full[s], par, A.err);
      if (__syncthreads_or(!ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sK = smem_addr(smem + kOffK + s * 2 * kTile), sV = sK + kTile;
      const uint32_t sQ = smem_addr(Qt), sP = smem_addr(Pt);
      // ---- S = K Q^T (4 K-steps of 32 dims)
      if (tid == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_f8(tmem_s, sw128_desc(sK + j * 32, 16, 1024), sw128_desc(sQ + j * 32, 16, 1024), kIdQK, j > 0);
        mma_commit(&bar_s);
      }
      mma_pending_s = true;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_s, ph_s, A.err));
      float sv[32];
      if (ok) {
        ph_s ^= 1;
        mma_pending_s = false;
        tc_fence_after();
        tmem_ld32(tmem_s + lane_off, sv);
      }
      const int pg = t >> 4;
      const bool valid = pg < np;
      const float ks = *reinterpret_cast<const float*>(scl + s * kScl + pg * 16);
      const float vs = *reinterpret_cast<const float*>(scl + s * kScl + pg * 16 + 4);
      float x[G], mx[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        x[h] = valid && ok ? (sv[h] + sv[8 + h] * 0.0625f + sv[16 + h] * 0.00390625f) * ks * qdiv[h] : -INFINITY;
        mx[h] = x[h];
      }
      {
        const float wm = warp_max_heads<G>(mx, lane);  // head (lane >> (5 - log2 G))
        if ((lane & ((32 / G) - 1)) == 0) red[warp][lane / (32 / G)] = wm;
      }
      // power-of-two scale of the weights: p * v_scale * beta <= 448 in this group
      float vmax = (lane & 31) < np ? *reinterpret_cast<const float*>(scl + s * kScl + (lane & 7) * 16 + 4) : 0.f;
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 4));
      const float beta = pow2_scale(__shfl_sync(0xffffffffu, vmax, 0));
      if (__syncthreads_or(!ok)) {
        ok = false;
        break;
      }
      // block maximum per head: lane l takes warp l / 8's value of head l % 8
      float gmx = red[lane >> 3][lane & 7];
      gmx = fmaxf(gmx, __shfl_xor_sync(0xffffffffu, gmx, 8));
      gmx = fmaxf(gmx, __shfl_xor_sync(0xffffffffu, gmx, 16));
      float alpha[G], pw[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float mn = fmaxf(m_run[h], __shfl_sync(0xffffffffu, gmx, h));
        alpha[h] = ex2(m_run[h] - mn);
        const float p = valid ? ex2(x[h] - mn) : 0.f;
        l_thr[h] = l_thr[h] * alpha[h] + p;
        m_run[h] = mn;
        pw[h] = p * vs * beta;
      }
      // this token's row of the P tile: byte j*8 + h = term j of head h
      uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int i = 0; i < (G + 1) / 2; ++i) {
        uint32_t t0, t1, t2;
        split3x2(make_float2(pw[2 * i], 2 * i + 1 < G ? pw[2 * i + 1] : 0.f), t0, t1, t2);
        const int sh = 16 * (i & 1);
        w[(i >> 1)] |= t0 << sh;
        w[2 + (i >> 1)] |= t1 << sh;
        w[4 + (i >> 1)] |= t2 << sh;
      }
      {
        uint8_t* row = Pt + (t >> 3) * 256 + (t & 7) * 16;
        *reinterpret_cast<uint4*>(row) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(row + 128) = make_uint4(w[4], w[5], w[6], w[7]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      // ---- O^T = V^T P'^T (4 K-steps of 32 tokens)
      if (tid == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_f8(tmem_o, sw128_desc(sV + j * 4096, kTile, 1024), plain_desc(sP + j * 1024, 256, 128), kIdPV, j > 0);
        mma_commit(&bar_o);
      }
      mma_pending_o = true;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_o, ph_o, A.err));
      if (ok) {
        ph_o ^= 1;
        mma_pending_o = false;
        tc_fence_after();
        float ov[32];
        tmem_ld32(tmem_o + lane_off, ov);  // thread t = head dim t
        const float ib = __frcp_rn(beta);  // exact: beta is a power of two
#pragma unroll
        for (int h = 0; h < G; ++h)
          o_acc[h] = o_acc[h] * alpha[h] + (ov[h] + ov[8 + h] * 0.0625f + ov[16 + h] * 0.00390625f) * ib;
      }
      ++it_use;
      tc_fence_before();
      if (__syncthreads_or(!ok)) {  // stage, S/O TMEM, P tile and red reusable
        ok = false;
        break;
      }
      issue();
    }
    if (!ok) break;
    // ---- partial of this lane segment: slot a + c
    const int cf = cta_of(base, A.nc, A.T);
    const int parts = cta_of(base + A.gpl - 1, A.nc, A.T) - cf + 1;
    float* pc = A.part + ((size_t)a + c) * G * kPartStride;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float l = l_thr[h];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) red[warp][h] = l;
      pc[h * kPartStride + t] = o_acc[h];
    }
    __syncthreads();
    if (tid < G) {
      pc[tid * kPartStride + 128] = m_run[tid];
      pc[tid * kPartStride + 129] = red[0][tid] + red[1][tid] + red[2][tid] + red[3][tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_flag = atomicAdd(&A.lane_done[a], 1u) == (uint32_t)(parts - 1);
    __syncthreads();
    if (s_flag) {
      // combine: thread t = dim t of every head
      __threadfence();
      const float* pl = A.part + ((size_t)a + cf) * G * kPartStride;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float M = -INFINITY;
        for (int j = 0; j < parts; ++j) M = fmaxf(M, __ldcg(pl + ((size_t)j * G + h) * kPartStride + 128));
        float L = 0.f, O = 0.f;
        for (int j = 0; j < parts; ++j) {
          const float* pj = pl + ((size_t)j * G + h) * kPartStride;
          const float mj = __ldcg(pj + 128);
          const float wj = (M == -INFINITY || mj == -INFINITY) ? 0.f : exp2f(mj - M);
          L = fmaf(__ldcg(pj + 129), wj, L);
          O = fmaf(__ldcg(pj + t), wj, O);
        }
        A.out[((size_t)a * G + h) * kHeadDim + t] = L > 0.f ? O / L : 0.f;
      }
      if (tid == 0) A.lane_done[a] = 0;
    }
    __syncthreads();  // red / s_flag reusable
  }
  if (!ok && tid == 0) {
    // let copies and MMAs still in flight land (bounded, results ignored)
    while (it_use < it_load) {
      mbar_wait(&full[it_use % kTcStages], (it_use / kTcStages) & 1u, nullptr);
      ++it_use;
    }
    if (mma_pending_s) mbar_wait(&bar_s, ph_s, nullptr);
    if (mma_pending_o) mbar_wait(&bar_o, ph_o, nullptr);
  }
  tc_fence_before();
  __syncthreads();
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

// Tensor map over the e4m3 cache: (128 B, 32 rows, units) with unit stride
// 4112 B; rows 0-15 of a unit are K, rows 16-31 V. Boxes of 128 B x 16 rows
// land SWIZZLE_128B in shared memory.
int make_cache_tensor_map(ferry_ctx* c) {
  auto fn = encode_fn();
  if (!fn) return set_error("cuTensorMapEncodeTiled unavailable"), FERRY_E_CUDA;
  const uint64_t units = (uint64_t)c->lanes * c->cfg.cache_pages;
  if (units == 0 || units > 0x7fffffffull) return set_error("cache too large for a tensor map"), FERRY_E_INVAL;
  cuuint64_t dims[3] = {128, 32, units};
  cuuint64_t strides[2] = {128, (cuuint64_t)kUnitBytesF8};
  cuuint32_t box[3] = {128, 16, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  static_assert(sizeof(CUtensorMap) <= sizeof(c->cache_map), "tensor map storage");
  const CUresult r = fn(reinterpret_cast<CUtensorMap*>(c->cache_map), CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, c->cache, dims,
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
  // resident CTAs, >= 2 groups each, <= 31 per lane (a lane combines <= 32 partials)
  int64_t nc = std::min<int64_t>((int64_t)c->num_sms * 2, std::max<int64_t>(1, A.T / 2));
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
#define FERRY_TC_CASE(GG)                                                                                  \
  case GG:                                                                                                 \
    FERRY_TRY(cudaFuncSetAttribute(attn_tc_kernel<GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem)); \
    attn_tc_kernel<GG><<<(unsigned)nc, kTcThreads, kTcSmem, st>>>(*map, A);                               \
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
