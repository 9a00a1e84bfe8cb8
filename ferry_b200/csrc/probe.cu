// probe.cu -- device/link discovery and link-peak probes.
//
// Counterpart of the reference's probe (src/topo/topo.cpp:12-215 enumerate /
// probe_topology / probe_host_staged_bandwidth, src/probe/main.cu:12-52),
// which measures P2P with cudaMemcpyPeerAsync and a host-staged ring. Here:
//   ferry_probe_topology   device count, P2P access and native peer atomics
//                          (the device deque's steal CAS needs them);
//   ferry_probe_link       GB/s of the two links the decode path uses:
//                          host -> device (pinned host memory read by a copy
//                          kernel, as the miss gather does) and peer -> device
//                          over NVLink (the migration copy kernel's access).
#include "common.cuh"

namespace ferry {
namespace {

__global__ void __launch_bounds__(256) pull_kernel(const uint8_t* __restrict__ src,
                                                   uint8_t* __restrict__ dst, int64_t n_units) {
  const int t = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t u = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); u < n_units; u += nw) {
    const uint8_t* s = src + u * kUnitBytes;
    uint8_t* d = dst + u * kUnitBytes;
    uint4 r[kUnitBytes / (32 * 16)];
#pragma unroll
    for (int j = 0; j < kUnitBytes / (32 * 16); ++j) r[j] = ld_nc_v4(s + (size_t)(t + 32 * j) * 16);
#pragma unroll
    for (int j = 0; j < kUnitBytes / (32 * 16); ++j) st_v4(d + (size_t)(t + 32 * j) * 16, r[j]);
  }
}

struct G {
  int prev = -1;
  explicit G(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~G() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace ferry

using namespace ferry;

extern "C" {

int ferry_probe_topology(int* n_dev, int32_t* p2p, int32_t* atomics, int cap) {
  if (!n_dev) return set_error("probe_topology: bad arguments"), FERRY_E_INVAL;
  int n = 0;
  FERRY_TRY(cudaGetDeviceCount(&n));
  *n_dev = n;
  if (!p2p || !atomics || cap < n) return FERRY_OK;
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < n; ++j) {
      int a = 0, at = 0;
      if (i != j) {
        FERRY_TRY(cudaDeviceCanAccessPeer(&a, i, j));
        FERRY_TRY(cudaDeviceGetP2PAttribute(&at, cudaDevP2PAttrNativeAtomicSupported, i, j));
      }
      p2p[i * cap + j] = a;
      atomics[i * cap + j] = at;
    }
  return FERRY_OK;
}

// src_dev = -1: pinned host memory; otherwise a peer device. The copy runs on
// dst_dev and reads the source directly (no copy engine).
int ferry_probe_link(int src_dev, int dst_dev, size_t bytes, int iters, double* gbs) {
  if (!gbs || iters < 1 || bytes < (size_t)kUnitBytes || src_dev == dst_dev)
    return set_error("probe_link: bad arguments"), FERRY_E_INVAL;
  const int64_t units = (int64_t)(bytes / kUnitBytes);
  bytes = (size_t)units * kUnitBytes;
  void* src = nullptr;
  void* src_dev_ptr = nullptr;
  void* dst = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int rc = FERRY_OK;
  auto fail = [&](cudaError_t e, const char* what) {
    rc = cuda_status(e, what);
  };
  {
    G g(dst_dev);
    cudaError_t e;
    if (src_dev < 0) {
      e = cudaHostAlloc(&src, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
      if (e != cudaSuccess) fail(e, "cudaHostAlloc");
      else if ((e = cudaHostGetDevicePointer(&src_dev_ptr, src, 0)) != cudaSuccess) fail(e, "cudaHostGetDevicePointer");
      else std::memset(src, 1, bytes);
    } else {
      int can = 0;
      cudaDeviceCanAccessPeer(&can, dst_dev, src_dev);
      if (!can) {
        set_error("device %d cannot access device %d", dst_dev, src_dev);
        return FERRY_E_INVAL;
      }
      e = cudaDeviceEnablePeerAccess(src_dev, 0);
      if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) fail(e, "cudaDeviceEnablePeerAccess");
      cudaGetLastError();
      if (!rc) {
        G gs(src_dev);
        if ((e = cudaMalloc(&src, bytes)) != cudaSuccess) fail(e, "cudaMalloc(src)");
        else if ((e = cudaMemset(src, 1, bytes)) != cudaSuccess) fail(e, "cudaMemset(src)");
        else cudaDeviceSynchronize();
        src_dev_ptr = src;
      }
    }
    if (!rc && (e = cudaMalloc(&dst, bytes)) != cudaSuccess) fail(e, "cudaMalloc(dst)");
    if (!rc) {
      cudaEventCreate(&e0);
      cudaEventCreate(&e1);
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dst_dev);
      const unsigned blocks = (unsigned)std::min<int64_t>((units + 7) / 8, (int64_t)sms * 16);
      pull_kernel<<<blocks, 256>>>((const uint8_t*)src_dev_ptr, (uint8_t*)dst, units);  // warm-up
      cudaEventRecord(e0);
      for (int i = 0; i < iters; ++i)
        pull_kernel<<<blocks, 256>>>((const uint8_t*)src_dev_ptr, (uint8_t*)dst, units);
      cudaEventRecord(e1);
      if ((e = cudaEventSynchronize(e1)) != cudaSuccess) fail(e, "probe kernel");
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      *gbs = (double)bytes * iters / (ms / 1e3) / 1e9;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(dst);
  }
  if (src) {
    if (src_dev < 0) {
      cudaFreeHost(src);
    } else {
      G gs(src_dev);
      cudaFree(src);
    }
  }
  return rc;
}

}  // extern "C"
