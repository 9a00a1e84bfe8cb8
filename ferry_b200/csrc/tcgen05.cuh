// tcgen05.cuh -- shared device helpers of the tensor-core attention kernels
// (attn_tc.cu, attn_tc16.cu): UMMA shared-memory descriptors, MMA commit and
// fences, TMA tensor loads, TMEM loads, the softmax-warp barrier and the
// flat work split. sm_100a only.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ferry {
namespace {

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

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 3-D tensor copy global -> shared (no multicast), completion on the mbarrier
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
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

// 8 consecutive f32 columns of this thread's TMEM lane (column a multiple of 8)
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// N consecutive f32 columns (N = 1, 2, 4 or 8) of this thread's TMEM lane
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, float* v) {
  if constexpr (N == 8) {
    tmem_ld8(taddr, v);
  } else if constexpr (N == 4) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
  } else if constexpr (N == 2) {
    uint32_t r[2];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr));
    v[0] = __uint_as_float(r[0]);
    v[1] = __uint_as_float(r[1]);
  } else {
    static_assert(N == 1, "tmem_ld_n: N is 1, 2, 4 or 8");
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
    v[0] = __uint_as_float(r);
  }
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// barrier among the 256 softmax threads only (named barrier 1); true when
// any of them passed `flag`
__device__ __forceinline__ bool softmax_bar_or(bool flag) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)flag)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Walk of a CTA's flat range, shared by its three roles: lane segments in
// order, each with its groups [glo, ghi) (pages present only).
struct Seg {
  int a, n, glo, ghi;
  int64_t unit0;
};


}  // namespace
}  // namespace ferry
