// deque.cu -- device-visible, lock-free, bounded work-stealing deque.
//
// Replaces the reference's host std::deque steal path (local_[v] under mtx_,
// src/runtime/wla_multigpu.cuh:1063-1506) and its device MPMC ring, whose
// waits spin without bound (src/queue/gpu_bounded_queue.cuh:70-149). Layout in
// the owner GPU's memory: a header {top, bottom, capacity} and a ring of
// 64-bit tasks. The owner pushes and pops at the bottom; thieves -- kernels on
// any GPU that maps this memory (NVLink peer access or CUDA IPC) -- take from
// the top with a system-scope CAS (Chase-Lev). No operation waits for another
// party: a CAS that keeps losing gives up after kCasTries and reports how many
// tasks it got, so a caller never hangs on a slow or dead peer.
#include "common.cuh"

namespace ferry {

struct DequeHdr {
  unsigned long long top;
  unsigned long long bottom;
  unsigned long long cap;
  unsigned long long pad;
};

namespace {

constexpr int kCasTries = 64;

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long cas_sys(unsigned long long* p, unsigned long long cmp,
                                                      unsigned long long val) {
  unsigned long long old;
  asm volatile("atom.acq_rel.sys.global.cas.b64 %0, [%1], %2, %3;"
               : "=l"(old)
               : "l"(p), "l"(cmp), "l"(val)
               : "memory");
  return old;
}
__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }

// ---- device operations (one thread) -------------------------------------
// push n tasks at the bottom; returns how many fitted
__device__ int dq_push(DequeHdr* h, unsigned long long* ring, const uint64_t* tasks, int n) {
  const unsigned long long b = ld_relaxed_sys(&h->bottom);
  const unsigned long long t = ld_acquire_sys(&h->top);
  const unsigned long long cap = h->cap;
  const unsigned long long room = cap - (b - t);
  const int m = (unsigned long long)n < room ? n : (int)room;
  for (int i = 0; i < m; ++i) st_relaxed_sys(&ring[(b + i) % cap], tasks[i]);
  st_release_sys(&h->bottom, b + m);  // publishes the tasks
  return m;
}

// owner pop of one task at the bottom (Chase-Lev); false when empty
__device__ bool dq_pop(DequeHdr* h, unsigned long long* ring, uint64_t* out) {
  const unsigned long long b0 = ld_relaxed_sys(&h->bottom);
  if (b0 == 0) return false;
  const unsigned long long b = b0 - 1;
  st_relaxed_sys(&h->bottom, b);
  fence_sc_sys();
  const unsigned long long t = ld_relaxed_sys(&h->top);
  if ((long long)(b - t) < 0) {  // empty
    st_relaxed_sys(&h->bottom, t);
    return false;
  }
  *out = ld_relaxed_sys(&ring[b % h->cap]);
  if (b != t) return true;
  // last task: race thieves for it
  const bool won = cas_sys(&h->top, t, t + 1) == t;
  st_relaxed_sys(&h->bottom, t + 1);
  return won;
}

// thief take of one task at the top; 1 taken, 0 empty, -1 lost kCasTries races
__device__ int dq_steal(DequeHdr* h, unsigned long long* ring, uint64_t* out) {
  for (int i = 0; i < kCasTries; ++i) {
    const unsigned long long t = ld_acquire_sys(&h->top);
    fence_sc_sys();
    const unsigned long long b = ld_acquire_sys(&h->bottom);
    if ((long long)(b - t) <= 0) return 0;
    const uint64_t v = ld_relaxed_sys(&ring[t % h->cap]);
    if (cas_sys(&h->top, t, t + 1) == t) {
      *out = v;
      return 1;
    }
  }
  return -1;
}

__global__ void push_kernel(DequeHdr* h, unsigned long long* ring, const uint64_t* tasks, int n,
                            int32_t* status) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int m = dq_push(h, ring, tasks, n);
    if (status) *status = m;
  }
}

__global__ void pop_kernel(DequeHdr* h, unsigned long long* ring, uint64_t* out, int max_n,
                           int32_t* count) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int c = 0;
    while (c < max_n && dq_pop(h, ring, &out[c])) ++c;
    *count = c;
  }
}

__global__ void steal_kernel(DequeHdr* h, unsigned long long* ring, uint64_t* out, int max_n,
                             int32_t* count) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int c = 0;
    while (c < max_n) {
      const int r = dq_steal(h, ring, &out[c]);
      if (r <= 0) break;
      ++c;
    }
    *count = c;
  }
}

// snapshot of up to max_n tasks at the top (what the next steals would take),
// without taking them; concurrent pops and steals may change them afterwards
__global__ void peek_kernel(DequeHdr* h, unsigned long long* ring, uint64_t* out, int max_n, int32_t* count) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const unsigned long long t = ld_acquire_sys(&h->top);
    const unsigned long long b = ld_acquire_sys(&h->bottom);
    long long n = (long long)(b - t);
    n = n < 0 ? 0 : (n > max_n ? max_n : n);
    const unsigned long long cap = h->cap;
    for (long long i = 0; i < n; ++i) out[i] = ld_relaxed_sys(&ring[(t + (unsigned long long)i) % cap]);
    *count = (int32_t)n;
  }
}

__global__ void size_kernel(const DequeHdr* h, int64_t* out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const unsigned long long t = ld_acquire_sys(&h->top);
    const unsigned long long b = ld_acquire_sys(&h->bottom);
    out[0] = (int64_t)(b - t) > 0 ? (int64_t)(b - t) : 0;
  }
}

// Exactly-once stress test (the device twin of the reference's bench_queue
// pc_kernel, src/benches/bench_queue.cu:26-59): block 0 is the owner -- it
// pushes tasks 0..n-1 in batches and pops from the bottom -- and every other
// block's thread 0 steals from the top until the owner reports it is done and
// the deque is empty. Every taken task bumps seen[task]; the host checks that
// every counter is exactly 1. Waits are bounded: a thief gives up after
// max_rounds polls and records kErrTimeout. Launched cooperatively so every
// block is resident.
__global__ void stress_kernel(DequeHdr* h, unsigned long long* ring, int n_tasks, int batch,
                              uint32_t* seen, unsigned long long* taken, int* owner_done,
                              long long max_rounds, uint32_t* err) {
  if (threadIdx.x != 0) return;
  if (blockIdx.x == 0) {
    uint64_t buf[32];
    int next = 0;
    long long rounds = 0;
    while (next < n_tasks && rounds++ < max_rounds) {
      const int m = min(batch, min(32, n_tasks - next));
      for (int i = 0; i < m; ++i) buf[i] = (uint64_t)(next + i);
      const int pushed = dq_push(h, ring, buf, m);
      next += pushed;
      // the owner also consumes some of its own work
      uint64_t v;
      if (dq_pop(h, ring, &v)) {
        atomicAdd(&seen[v], 1u);
        atomicAdd(taken, 1ull);
      }
    }
    if (next < n_tasks) record_error(err, kErrTimeout);
    uint64_t v;
    while (dq_pop(h, ring, &v)) {
      atomicAdd(&seen[v], 1u);
      atomicAdd(taken, 1ull);
    }
    __threadfence_system();
    atomicExch(owner_done, 1);
  } else {
    for (long long r = 0; r < max_rounds; ++r) {
      uint64_t v;
      const int got = dq_steal(h, ring, &v);
      if (got == 1) {
        atomicAdd(&seen[v], 1u);
        atomicAdd(taken, 1ull);
        continue;
      }
      if (atomicAdd(owner_done, 0) && got == 0) return;
      __nanosleep(64);
    }
    record_error(err, kErrTimeout);
  }
}

}  // namespace
}  // namespace ferry

struct ferry_deque {
  int device = -1;
  bool owned = true;  // false for an imported peer view
  bool ipc = false;   // the view maps the owner through CUDA IPC (closed on destroy)
  ferry::DequeHdr* hdr = nullptr;
  unsigned long long* ring = nullptr;
  uint64_t cap = 0;
};

using namespace ferry;

namespace {
struct DevGuard {
  int prev = -1;
  explicit DevGuard(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~DevGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

extern "C" {

int ferry_deque_create(int device, uint64_t capacity, ferry_deque** out) {
  if (!out || capacity < 1 || capacity > (1ull << 30))
    return set_error("deque_create: capacity must be in [1, 2^30]"), FERRY_E_INVAL;
  *out = nullptr;
  DevGuard g(device);
  auto* q = new ferry_deque;
  q->device = device;
  q->cap = capacity;
  // header and ring in one allocation, so one IPC handle exports both
  void* mem = nullptr;
  cudaError_t e = cudaMalloc(&mem, sizeof(DequeHdr) + capacity * 8);
  if (e != cudaSuccess) {
    delete q;
    return cuda_status(e, "cudaMalloc(deque)");
  }
  q->hdr = (DequeHdr*)mem;
  q->ring = (unsigned long long*)((char*)mem + sizeof(DequeHdr));
  DequeHdr h0{0, 0, capacity, 0};
  e = cudaMemcpy(q->hdr, &h0, sizeof h0, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(mem);
    delete q;
    return cuda_status(e, "cudaMemcpy(deque header)");
  }
  *out = q;
  return FERRY_OK;
}

int ferry_deque_destroy(ferry_deque* q) {
  if (!q) return FERRY_OK;
  DevGuard g(q->device);
  cudaDeviceSynchronize();
  if (q->owned)
    cudaFree(q->hdr);
  else if (q->ipc)
    cudaIpcCloseMemHandle(q->hdr);
  cudaGetLastError();  // teardown errors are not the caller's next launch's
  delete q;
  return FERRY_OK;
}

int ferry_deque_push(ferry_deque* q, void* stream, const uint64_t* d_tasks, int n,
                     int32_t* d_pushed) {
  if (!q || n < 0 || (n && !d_tasks)) return set_error("deque_push: bad arguments"), FERRY_E_INVAL;
  if (!q->owned) return set_error("deque_push: only the owner pushes"), FERRY_E_INVAL;
  if (n == 0) return FERRY_OK;
  push_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(q->hdr, q->ring, d_tasks, n, d_pushed);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_deque_pop(ferry_deque* q, void* stream, uint64_t* d_out, int max_n, int32_t* d_count) {
  if (!q || max_n < 0 || !d_out || !d_count) return set_error("deque_pop: bad arguments"), FERRY_E_INVAL;
  if (!q->owned) return set_error("deque_pop: only the owner pops"), FERRY_E_INVAL;
  pop_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(q->hdr, q->ring, d_out, max_n, d_count);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_deque_steal(ferry_deque* q, void* stream, uint64_t* d_out, int max_n, int32_t* d_count) {
  if (!q || max_n < 0 || !d_out || !d_count) return set_error("deque_steal: bad arguments"), FERRY_E_INVAL;
  steal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(q->hdr, q->ring, d_out, max_n, d_count);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_deque_peek(ferry_deque* q, void* stream, uint64_t* d_out, int max_n, int32_t* d_count) {
  if (!q || max_n < 0 || !d_out || !d_count) return set_error("deque_peek: bad arguments"), FERRY_E_INVAL;
  peek_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(q->hdr, q->ring, d_out, max_n, d_count);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_deque_size(ferry_deque* q, void* stream, int64_t* d_size) {
  if (!q || !d_size) return set_error("deque_size: bad arguments"), FERRY_E_INVAL;
  size_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(q->hdr, d_size);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int ferry_deque_export(ferry_deque* q, void* handle64) {
  if (!q || !handle64 || !q->owned) return set_error("deque_export: bad arguments"), FERRY_E_INVAL;
  DevGuard g(q->device);
  cudaIpcMemHandle_t h;
  FERRY_TRY(cudaIpcGetMemHandle(&h, q->hdr));
  std::memcpy(handle64, &h, sizeof h);
  return FERRY_OK;
}

int ferry_deque_import(int device, const void* handle64, uint64_t capacity, ferry_deque** out) {
  if (!handle64 || !out || capacity < 1) return set_error("deque_import: bad arguments"), FERRY_E_INVAL;
  *out = nullptr;
  DevGuard g(device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof h);
  void* p = nullptr;
  FERRY_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  auto* q = new ferry_deque;
  q->device = device;
  q->owned = false;
  q->ipc = true;
  q->hdr = (DequeHdr*)p;
  q->ring = (unsigned long long*)((char*)p + sizeof(DequeHdr));
  q->cap = capacity;
  *out = q;
  return FERRY_OK;
}

int ferry_deque_peer_view(int device, ferry_deque* owner, ferry_deque** out) {
  if (!owner || !out) return set_error("deque_peer_view: bad arguments"), FERRY_E_INVAL;
  *out = nullptr;
  if (device != owner->device) {
    DevGuard g(device);
    int can = 0;
    FERRY_TRY(cudaDeviceCanAccessPeer(&can, device, owner->device));
    if (!can) return set_error("device %d cannot access device %d", device, owner->device), FERRY_E_INVAL;
    cudaError_t e = cudaDeviceEnablePeerAccess(owner->device, 0);
    if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return cuda_status(e, "cudaDeviceEnablePeerAccess");
    cudaGetLastError();
  }
  auto* q = new ferry_deque;
  q->device = device;
  q->owned = false;
  q->hdr = owner->hdr;
  q->ring = owner->ring;
  q->cap = owner->cap;
  // a peer view never frees or closes the owner's memory
  q->owned = false;
  *out = q;
  return FERRY_OK;
}

int ferry_deque_stress(int device, uint64_t capacity, int n_tasks, int thieves, int batch,
                       uint64_t* taken_out, int32_t* dup_or_missing_out) {
  if (n_tasks < 1 || thieves < 0 || batch < 1 || !taken_out || !dup_or_missing_out)
    return set_error("deque_stress: bad arguments"), FERRY_E_INVAL;
  ferry_deque* q = nullptr;
  int rc = ferry_deque_create(device, capacity, &q);
  if (rc) return rc;
  DevGuard g(device);
  uint32_t* seen = nullptr;
  unsigned long long* taken = nullptr;
  int* done = nullptr;
  uint32_t* err = nullptr;
  auto cleanup = [&]() {
    cudaFree(seen);
    cudaFree(taken);
    cudaFree(done);
    cudaFree(err);
    ferry_deque_destroy(q);
  };
#define FERRY_ST(x)                         \
  do {                                      \
    cudaError_t e__ = (x);                  \
    if (e__ != cudaSuccess) {               \
      cleanup();                            \
      return cuda_status(e__, #x);          \
    }                                       \
  } while (0)
  FERRY_ST(cudaMalloc(&seen, (size_t)n_tasks * 4));
  FERRY_ST(cudaMalloc(&taken, 8));
  FERRY_ST(cudaMalloc(&done, 4));
  FERRY_ST(cudaMalloc(&err, 4));
  FERRY_ST(cudaMemset(seen, 0, (size_t)n_tasks * 4));
  FERRY_ST(cudaMemset(taken, 0, 8));
  FERRY_ST(cudaMemset(done, 0, 4));
  FERRY_ST(cudaMemset(err, 0, 4));
  int per_sm = 0, sms = 0;
  FERRY_ST(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stress_kernel, 32, 0));
  FERRY_ST(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  const int blocks = 1 + thieves;
  if (blocks > per_sm * sms) {
    cleanup();
    return set_error("deque_stress: %d blocks cannot all be resident", blocks), FERRY_E_INVAL;
  }
  DequeHdr* hdr = q->hdr;
  unsigned long long* ring = q->ring;
  long long max_rounds = 1ll << 24;
  void* args[] = {&hdr, &ring, &n_tasks, &batch, &seen, &taken, &done, &max_rounds, &err};
  FERRY_ST(cudaLaunchCooperativeKernel((void*)stress_kernel, blocks, 32, args, 0, 0));
  FERRY_ST(cudaDeviceSynchronize());
  unsigned long long tk = 0;
  uint32_t e = 0;
  FERRY_ST(cudaMemcpy(&tk, taken, 8, cudaMemcpyDeviceToHost));
  FERRY_ST(cudaMemcpy(&e, err, 4, cudaMemcpyDeviceToHost));
  uint32_t* hs = (uint32_t*)malloc((size_t)n_tasks * 4);
  FERRY_ST(cudaMemcpy(hs, seen, (size_t)n_tasks * 4, cudaMemcpyDeviceToHost));
  int bad = 0;
  for (int i = 0; i < n_tasks; ++i) bad += hs[i] != 1;
  free(hs);
  *taken_out = tk;
  *dup_or_missing_out = bad;
  cleanup();
#undef FERRY_ST
  if (e) return set_error("deque_stress: a bounded wait ran out"), FERRY_E_TIMEOUT;
  return FERRY_OK;
}

}  // extern "C"
