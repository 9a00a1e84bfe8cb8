// kvgen.cu -- procedural KV pool generator and page-summary kernels.
#include <cuda_fp8.h>

#include "common.cuh"

namespace ferry {

// Element e of page unit u: Irwin-Hall sum of twelve 16-bit uniforms drawn
// from three splitmix64 outputs, z = (sum - 6*65536) / 65536 (variance 1,
// exact in fp32).
__device__ __forceinline__ float kv_elem_f32(uint64_t seed, uint64_t unit, uint32_t e) {
  const uint64_t base = mix64(seed ^ mix64(unit * 4096ull + e));
  uint32_t acc = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint64_t h = mix64(base + (uint64_t)j);
    acc += (uint32_t)(h & 0xFFFF) + (uint32_t)((h >> 16) & 0xFFFF) +
           (uint32_t)((h >> 32) & 0xFFFF) + (uint32_t)(h >> 48);
  }
  return __fmul_rn((float)((int32_t)acc - 6 * 65536), 1.0f / 65536.0f);
}

namespace {

// fp16 pool: z rounded once to fp16
__device__ __forceinline__ uint16_t kv_elem(uint64_t seed, uint64_t unit, uint32_t e) {
  return __half_as_ushort(__float2half_rn(kv_elem_f32(seed, unit, e)));
}

// e4m3 unit by one warp (lane t). For K (elements 0..2047) and V
// (2048..4095): scale = amax / 448 of the unit's fp32 values (1 when all are
// zero), q = e4m3(z / scale), round to nearest even with saturation to +-448
// (cvt.rn.satfinite). Lane t owns 64 consecutive elements of each half.
__device__ __forceinline__ void gen_unit_e4m3(uint64_t seed, uint64_t unit, uint8_t* out, int t) {
    float scales[2];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t e0 = half * 2048 + t * 64;
      float amax = 0.f;
      for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(kv_elem_f32(seed, unit, e0 + i)));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float scale = amax > 0.f ? __fdiv_rn(amax, 448.0f) : 1.0f;
      scales[half] = scale;
#pragma unroll
      for (int v = 0; v < 4; ++v) {  // 4 x 16 bytes
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t word = 0;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const float z = kv_elem_f32(seed, unit, e0 + v * 16 + j * 4 + b);
            const __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(__fdiv_rn(z, scale), __NV_SATFINITE, __NV_E4M3);
            word |= (uint32_t)q << (8 * b);
          }
          w[j] = word;
        }
        *reinterpret_cast<uint4*>(out + e0 + v * 16) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    if (t == 0)
      *reinterpret_cast<uint4*>(out + 4096) =
          make_uint4(__float_as_uint(scales[0]), __float_as_uint(scales[1]), 0u, 0u);
}

// fp16 unit by one warp: lane t writes 16-byte vectors t, t + 32, ...
__device__ __forceinline__ void gen_unit_f16(uint64_t seed, uint64_t unit, uint8_t* out, int t) {
#pragma unroll 4
  for (int v = t; v < kUnitElems / 8; v += 32) {
    const uint32_t e0 = (uint32_t)v * 8;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = (uint32_t)__half_as_ushort(__float2half_rn(kv_elem_f32(seed, unit, e0 + 2 * j))) |
             ((uint32_t)__half_as_ushort(__float2half_rn(kv_elem_f32(seed, unit, e0 + 2 * j + 1))) << 16);
    reinterpret_cast<uint4*>(out)[v] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Owner store of rank `rank` of `world`: store index i holds page
// p = (i % own_np) * world + rank of global lane i / own_np, i.e. procedural
// unit (lane * N + p) mod pool_units; indices with p >= N stay zero.
__global__ void __launch_bounds__(256) store_fill_kernel(uint64_t seed, int world, int rank, int N, int own_np,
                                                         int64_t n_units, uint64_t pool_units, uint8_t* dst,
                                                         int unit_bytes, int e4m3) {
  const int t = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n_units; i += nw) {
    const int64_t lane = i / own_np;
    const int p = (int)(i % own_np) * world + rank;
    uint8_t* out = dst + (size_t)i * unit_bytes;
    if (p >= N) {
      for (int v = t; v < unit_bytes / 16; v += 32) reinterpret_cast<uint4*>(out)[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint64_t unit = ((uint64_t)lane * (uint64_t)N + (uint64_t)p) % pool_units;
    if (e4m3)
      gen_unit_e4m3(seed, unit, out, t);
    else
      gen_unit_f16(seed, unit, out, t);
  }
}

__global__ void __launch_bounds__(256) kv_generate_e4m3_kernel(uint64_t seed, uint64_t unit0,
                                                               int64_t n_units, uint8_t* dst) {
  const int t = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n_units; u += nw)
    gen_unit_e4m3(seed, unit0 + (uint64_t)u, dst + (size_t)u * kUnitBytesF8, t);
}

// e4m3 summary: summary[d] = (k_0[d] + ... + k_15[d]) * (1/16) with
// k_t[d] = float(e4m3) * k_scale (one rounding), in token order.
__global__ void __launch_bounds__(256) summary_e4m3_kernel(const uint8_t* __restrict__ pool, int64_t unit0,
                                                           int64_t n_units, float* __restrict__ summ) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n_units; u += warps) {
    const uint8_t* K = pool + (size_t)(unit0 + u) * kUnitBytesF8;
    const float ks = *reinterpret_cast<const float*>(K + 4096);
    float acc[4];
#pragma unroll
    for (int tt = 0; tt < kPageTokens; ++tt) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(K + tt * kHeadDim + lane * 4);
      const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xFFFF), __NV_E4M3);
      const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
      const float v[4] = {__half2float(__ushort_as_half(lo.x)), __half2float(__ushort_as_half(lo.y)),
                          __half2float(__ushort_as_half(hi.x)), __half2float(__ushort_as_half(hi.y))};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float kv = __fmul_rn(v[j], ks);
        acc[j] = tt == 0 ? kv : __fadd_rn(acc[j], kv);
      }
    }
    reinterpret_cast<float4*>(summ + (size_t)(unit0 + u) * kHeadDim)[lane] =
        make_float4(__fmul_rn(acc[0], 0.0625f), __fmul_rn(acc[1], 0.0625f), __fmul_rn(acc[2], 0.0625f),
                    __fmul_rn(acc[3], 0.0625f));
  }
}

// One thread writes 8 consecutive elements (one 16-byte store) so that
// destinations in mapped host memory see full-width PCIe writes.
__global__ void __launch_bounds__(256) kv_generate_kernel(uint64_t seed, uint64_t unit0,
                                                          int64_t n_vec, uint4* dst) {
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n_vec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t unit = unit0 + (uint64_t)(v / (kUnitElems / 8));
    const uint32_t e0 = (uint32_t)(v % (kUnitElems / 8)) * 8;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = (uint32_t)kv_elem(seed, unit, e0 + 2 * j) |
             ((uint32_t)kv_elem(seed, unit, e0 + 2 * j + 1) << 16);
    dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// summary[d] = (k_0[d] + ... + k_15[d]) * (1/16), token order, fp32. One warp
// per unit; lane l owns dims 4l..4l+3 (8-byte loads, 256 B per row).
__global__ void __launch_bounds__(256) summary_kernel(const uint8_t* __restrict__ pool,
                                                      int64_t unit0, int64_t n_units,
                                                      float* __restrict__ summ) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n_units;
       u += warps) {
    const uint8_t* K = pool + (size_t)(unit0 + u) * kUnitBytes;
    uint2 raw[kPageTokens];
#pragma unroll
    for (int t = 0; t < kPageTokens; ++t)
      raw[t] = *reinterpret_cast<const uint2*>(K + t * kHeadDim * 2 + lane * 8);
    float acc[4];
#pragma unroll
    for (int t = 0; t < kPageTokens; ++t) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw[t].x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw[t].y));
      if (t == 0) {
        acc[0] = a.x; acc[1] = a.y; acc[2] = b.x; acc[3] = b.y;
      } else {
        acc[0] = __fadd_rn(acc[0], a.x);
        acc[1] = __fadd_rn(acc[1], a.y);
        acc[2] = __fadd_rn(acc[2], b.x);
        acc[3] = __fadd_rn(acc[3], b.y);
      }
    }
    float4 s = make_float4(__fmul_rn(acc[0], 0.0625f), __fmul_rn(acc[1], 0.0625f),
                           __fmul_rn(acc[2], 0.0625f), __fmul_rn(acc[3], 0.0625f));
    reinterpret_cast<float4*>(summ + (size_t)(unit0 + u) * kHeadDim)[lane] = s;
  }
}


// Quest page bounds: per dim the min and max of the page's 16 keys, rows
// [kmin[128] | kmax[128]] fp32 (e4m3: dequantised keys, value * k_scale with
// one rounding). Tokens in order; a later token replaces only when strictly
// smaller / larger. One warp per unit; lane l owns dims 4l..4l+3.
template <bool F8>
__global__ void __launch_bounds__(256) minmax_kernel(const uint8_t* __restrict__ pool, int64_t unit0,
                                                     int64_t n_units, float* __restrict__ mm) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n_units; u += warps) {
    float lo[4], hi[4];
    if (F8) {
      const uint8_t* K = pool + (size_t)(unit0 + u) * kUnitBytesF8;
      const float ks = *reinterpret_cast<const float*>(K + 4096);
#pragma unroll
      for (int tt = 0; tt < kPageTokens; ++tt) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(K + tt * kHeadDim + lane * 4);
        const __half2_raw a = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xFFFF), __NV_E4M3);
        const __half2_raw b = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
        const float v[4] = {__half2float(__ushort_as_half(a.x)), __half2float(__ushort_as_half(a.y)),
                            __half2float(__ushort_as_half(b.x)), __half2float(__ushort_as_half(b.y))};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float kv = __fmul_rn(v[j], ks);
          lo[j] = (tt == 0 || kv < lo[j]) ? kv : lo[j];
          hi[j] = (tt == 0 || kv > hi[j]) ? kv : hi[j];
        }
      }
    } else {
      const uint8_t* K = pool + (size_t)(unit0 + u) * kUnitBytes;
#pragma unroll
      for (int tt = 0; tt < kPageTokens; ++tt) {
        const uint2 raw = *reinterpret_cast<const uint2*>(K + tt * kHeadDim * 2 + lane * 8);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        const float v[4] = {a.x, a.y, b.x, b.y};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lo[j] = (tt == 0 || v[j] < lo[j]) ? v[j] : lo[j];
          hi[j] = (tt == 0 || v[j] > hi[j]) ? v[j] : hi[j];
        }
      }
    }
    float4* row = reinterpret_cast<float4*>(mm + (size_t)(unit0 + u) * 2 * kHeadDim);
    row[lane] = make_float4(lo[0], lo[1], lo[2], lo[3]);
    row[32 + lane] = make_float4(hi[0], hi[1], hi[2], hi[3]);
  }
}

// ---- decode appends
// A decode step appends its token to the request's context. ctx_pages holds
// the full pages of each request and, R entries later, the tokens of its
// partial last page; a page joins the selectable context when its 16th token
// arrives (the reference's selector scores whole pages only,
// tools/capture_miss_trace.py:131-133), and its summary -- mean row or Quest
// bounds -- is computed then from the pool unit that holds it (the caller has
// written the page's K/V there). Warp per (request, lane) computes the new
// pages' summaries; a second kernel advances the counters.
struct AppendArgs {
  const int32_t* req_ids;
  int n, tokens, lanes_per_req, N, R;
  int32_t* ctx_pages;
  const int64_t* req_base;
  const uint8_t* pool;
  uint64_t pool_units;
  float* summ;
  int quest, f8;
  uint32_t* err;
};

// Summary row of the page unit at K (mean of its 16 keys, as summary_kernel)
// into row[128]; one warp, lane l owns dims 4l..4l+3.
__device__ __forceinline__ void summary_unit(const uint8_t* K, float* row, bool f8, int lane) {
  float acc[4];
  if (f8) {
    const float ks = *reinterpret_cast<const float*>(K + 4096);
#pragma unroll
    for (int tt = 0; tt < kPageTokens; ++tt) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(K + tt * kHeadDim + lane * 4);
      const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xFFFF), __NV_E4M3);
      const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
      const float v[4] = {__half2float(__ushort_as_half(lo.x)), __half2float(__ushort_as_half(lo.y)),
                          __half2float(__ushort_as_half(hi.x)), __half2float(__ushort_as_half(hi.y))};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float kv = __fmul_rn(v[j], ks);
        acc[j] = tt == 0 ? kv : __fadd_rn(acc[j], kv);
      }
    }
  } else {
#pragma unroll
    for (int tt = 0; tt < kPageTokens; ++tt) {
      const uint2 raw = *reinterpret_cast<const uint2*>(K + tt * kHeadDim * 2 + lane * 8);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      const float v[4] = {a.x, a.y, b.x, b.y};
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = tt == 0 ? v[j] : __fadd_rn(acc[j], v[j]);
    }
  }
  reinterpret_cast<float4*>(row)[lane] =
      make_float4(__fmul_rn(acc[0], 0.0625f), __fmul_rn(acc[1], 0.0625f), __fmul_rn(acc[2], 0.0625f),
                  __fmul_rn(acc[3], 0.0625f));
}

// Quest bounds of the page unit at K (as minmax_kernel) into row[256].
__device__ __forceinline__ void minmax_unit(const uint8_t* K, float* row, bool f8, int lane) {
  float lo[4], hi[4];
#pragma unroll
  for (int tt = 0; tt < kPageTokens; ++tt) {
    float v[4];
    if (f8) {
      const float ks = *reinterpret_cast<const float*>(K + 4096);
      const uint32_t w = *reinterpret_cast<const uint32_t*>(K + tt * kHeadDim + lane * 4);
      const __half2_raw a = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w & 0xFFFF), __NV_E4M3);
      const __half2_raw b = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w >> 16), __NV_E4M3);
      v[0] = __fmul_rn(__half2float(__ushort_as_half(a.x)), ks);
      v[1] = __fmul_rn(__half2float(__ushort_as_half(a.y)), ks);
      v[2] = __fmul_rn(__half2float(__ushort_as_half(b.x)), ks);
      v[3] = __fmul_rn(__half2float(__ushort_as_half(b.y)), ks);
    } else {
      const uint2 raw = *reinterpret_cast<const uint2*>(K + tt * kHeadDim * 2 + lane * 8);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo[j] = (tt == 0 || v[j] < lo[j]) ? v[j] : lo[j];
      hi[j] = (tt == 0 || v[j] > hi[j]) ? v[j] : hi[j];
    }
  }
  float4* r4 = reinterpret_cast<float4*>(row);
  r4[lane] = make_float4(lo[0], lo[1], lo[2], lo[3]);
  r4[32 + lane] = make_float4(hi[0], hi[1], hi[2], hi[3]);
}

__global__ void __launch_bounds__(256) append_summary_kernel(AppendArgs A) {
  const int t = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= A.n * A.lanes_per_req) return;
  const int i = w / A.lanes_per_req, l = w % A.lanes_per_req;
  const int r = A.req_ids[i];
  if (r < 0 || r >= A.R) {
    if (t == 0 && l == 0) record_error(A.err, kErrRange);
    return;
  }
  const int np = A.ctx_pages[r], tail = A.ctx_pages[A.R + r];
  if (np < 0 || np > A.N || tail < 0 || tail >= kPageTokens) {
    if (t == 0 && l == 0) record_error(A.err, kErrRange);
    return;
  }
  const int64_t np2 = min((int64_t)A.N, (int64_t)np + ((int64_t)tail + A.tokens) / kPageTokens);
  for (int64_t p = np; p < np2; ++p) {
    const uint64_t u = (uint64_t)(A.req_base[r] + (int64_t)l * A.N + p) % A.pool_units;
    const uint8_t* K = A.pool + (size_t)u * (A.f8 ? kUnitBytesF8 : kUnitBytes);
    if (A.quest)
      minmax_unit(K, A.summ + (size_t)u * 2 * kHeadDim, A.f8, t);
    else
      summary_unit(K, A.summ + (size_t)u * kHeadDim, A.f8, t);
  }
}

// ---- summaries read from the owner stores (no host pool)
// Page p of request r's lane l lives in the store of rank p % world, at index
// glane * own_np + p / world with glane = (req_base[r] + l * N) / N; its
// summary row goes to pool unit (req_base[r] + l * N + p) mod pool_units, the
// row ferry_page_summary_update would write from a host pool with the same
// content. One warp per (request, lane, page); pages whose owner store is
// not mapped are recorded as range errors and left alone.
struct StoreSumArgs {
  const int32_t* req_ids;
  int n, lanes_per_req, N, R;
  const int32_t* ctx_pages;
  const int64_t* req_base;
  OwnerMap own;
  int unit_bytes;
  uint64_t pool_units;
  float* summ;
  int quest, f8;
  uint32_t* err;
};

__global__ void __launch_bounds__(256) store_summary_kernel(const __grid_constant__ StoreSumArgs A) {
  const int t = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t total = (int64_t)A.n * A.lanes_per_req * A.N;
  for (int64_t f = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); f < total; f += nw) {
    const int p = (int)(f % A.N);
    const int64_t a = f / A.N;
    const int i = (int)(a / A.lanes_per_req), l = (int)(a % A.lanes_per_req);
    const int r = A.req_ids[i];
    if (r < 0 || r >= A.R) {
      if (t == 0 && l == 0 && p == 0) record_error(A.err, kErrRange);
      continue;
    }
    const int64_t home = A.req_base[r] + (int64_t)l * A.N;
    const int64_t glane = home / A.N;
    const int owner = p % A.own.world;
    if (glane < 0 || glane >= A.own.store_lanes || !A.own.store[owner]) {
      if (t == 0) record_error(A.err, kErrRange);
      continue;
    }
    const uint8_t* K = A.own.store[owner] + ((size_t)glane * A.own.own_np + p / A.own.world) * A.unit_bytes;
    const uint64_t u = (uint64_t)(home + p) % A.pool_units;
    if (A.quest)
      minmax_unit(K, A.summ + (size_t)u * 2 * kHeadDim, A.f8, t);
    else
      summary_unit(K, A.summ + (size_t)u * kHeadDim, A.f8, t);
  }
}

__global__ void append_state_kernel(AppendArgs A) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= A.n) return;
  const int r = A.req_ids[i];
  if (r < 0 || r >= A.R) return;
  const int np = A.ctx_pages[r], tail = A.ctx_pages[A.R + r];
  if (np < 0 || np > A.N || tail < 0 || tail >= kPageTokens) return;
  const int64_t tot = (int64_t)tail + A.tokens;
  const int64_t np2 = min((int64_t)A.N, (int64_t)np + tot / kPageTokens);
  A.ctx_pages[r] = (int32_t)np2;
  A.ctx_pages[A.R + r] = np2 >= A.N ? 0 : (int32_t)(tot % kPageTokens);  // a full context stops growing
}
}  // namespace

int launch_kv_generate(cudaStream_t st, uint64_t seed, uint64_t unit0, int64_t n_units,
                       void* dst, int kv_dtype) {
  if (n_units <= 0) return FERRY_OK;
  if (!dst || ((uintptr_t)dst & 15) || (kv_dtype != FERRY_KV_F16 && kv_dtype != FERRY_KV_E4M3)) {
    set_error("ferry_kv_generate: dst must be non-null and 16-byte aligned, dtype F16 or E4M3");
    return FERRY_E_INVAL;
  }
  // pinned host memory: write through its device-side alias
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, dst) == cudaSuccess && attr.type == cudaMemoryTypeHost &&
      attr.devicePointer)
    dst = attr.devicePointer;
  cudaGetLastError();
  if (kv_dtype == FERRY_KV_E4M3) {
    const int64_t blocks = std::min<int64_t>((n_units + 7) / 8, 148 * 16);
    kv_generate_e4m3_kernel<<<(unsigned)blocks, 256, 0, st>>>(seed, unit0, n_units, (uint8_t*)dst);
    FERRY_TRY(cudaGetLastError());
    return FERRY_OK;
  }
  const int64_t n_vec = n_units * (kUnitElems / 8);
  const int64_t blocks = std::min<int64_t>((n_vec + 255) / 256, 148 * 16);
  kv_generate_kernel<<<(unsigned)blocks, 256, 0, st>>>(seed, unit0, n_vec, (uint4*)dst);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_summary(cudaStream_t st, const uint8_t* pool, int64_t unit0, int64_t n_units,
                   float* summ, int kv_dtype) {
  if (n_units <= 0) return FERRY_OK;
  const int64_t blocks = std::min<int64_t>((n_units + 7) / 8, 148 * 16);
  if (kv_dtype == FERRY_KV_E4M3)
    summary_e4m3_kernel<<<(unsigned)blocks, 256, 0, st>>>(pool, unit0, n_units, summ);
  else
    summary_kernel<<<(unsigned)blocks, 256, 0, st>>>(pool, unit0, n_units, summ);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_append(const ferry_ctx* c, cudaStream_t st, const int32_t* req_ids, int n, int tokens) {
  if (n <= 0 || tokens <= 0) return FERRY_OK;
  AppendArgs A{};
  A.req_ids = req_ids;
  A.n = n;
  A.tokens = tokens;
  A.lanes_per_req = c->lanes_per_req;
  A.N = c->cfg.max_pages;
  A.R = c->cfg.num_requests;
  A.ctx_pages = c->ctx_pages;
  A.req_base = c->req_base;
  A.pool = c->pool_dev;
  A.pool_units = c->pool_units;
  A.summ = c->summ;
  A.quest = c->select_mode == FERRY_SELECT_QUEST;
  A.f8 = c->cfg.kv_dtype == FERRY_KV_E4M3;
  A.err = c->err;
  const int warps = n * c->lanes_per_req;
  append_summary_kernel<<<(warps + 7) / 8, 256, 0, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  append_state_kernel<<<(n + 127) / 128, 128, 0, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_store_summary(const ferry_ctx* c, cudaStream_t st, const int32_t* req_ids, int n) {
  if (n <= 0) return FERRY_OK;
  StoreSumArgs A{};
  A.req_ids = req_ids;
  A.n = n;
  A.lanes_per_req = c->lanes_per_req;
  A.N = c->cfg.max_pages;
  A.R = c->cfg.num_requests;
  A.ctx_pages = c->ctx_pages;
  A.req_base = c->req_base;
  A.own.world = c->own_world;
  A.own.self = c->own_rank;
  A.own.own_np = c->own_np;
  A.own.store_lanes = c->store_lanes;
  for (int r = 0; r <= FERRY_MAX_PEERS; ++r) A.own.store[r] = c->store_of[r];
  A.unit_bytes = c->unit_bytes;
  A.pool_units = c->pool_units;
  A.summ = c->summ;
  A.quest = c->select_mode == FERRY_SELECT_QUEST;
  A.f8 = c->cfg.kv_dtype == FERRY_KV_E4M3;
  A.err = c->err;
  const int64_t warps = (int64_t)n * c->lanes_per_req * c->cfg.max_pages;
  const int64_t blocks = std::min<int64_t>((warps + 7) / 8, (int64_t)c->num_sms * 16);
  store_summary_kernel<<<(unsigned)blocks, 256, 0, st>>>(A);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_minmax(cudaStream_t st, const uint8_t* pool, int64_t unit0, int64_t n_units, float* mm,
                  int kv_dtype) {
  if (n_units <= 0) return FERRY_OK;
  const int64_t blocks = std::min<int64_t>((n_units + 7) / 8, 148 * 16);
  if (kv_dtype == FERRY_KV_E4M3)
    minmax_kernel<true><<<(unsigned)blocks, 256, 0, st>>>(pool, unit0, n_units, mm);
  else
    minmax_kernel<false><<<(unsigned)blocks, 256, 0, st>>>(pool, unit0, n_units, mm);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int launch_store_fill(cudaStream_t st, uint64_t seed, int world, int rank, int N, int own_np, int64_t n_units,
                      uint64_t pool_units, uint8_t* dst, int kv_dtype) {
  if (n_units <= 0) return FERRY_OK;
  const int ub = kv_dtype == FERRY_KV_E4M3 ? kUnitBytesF8 : kUnitBytes;
  const int64_t blocks = std::min<int64_t>((n_units + 7) / 8, 148 * 16);
  store_fill_kernel<<<(unsigned)blocks, 256, 0, st>>>(seed, world, rank, N, own_np, n_units, pool_units, dst, ub,
                                                        kv_dtype == FERRY_KV_E4M3);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

}  // namespace ferry
