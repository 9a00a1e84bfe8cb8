// taskb.cu -- Workload B: the reference's synthetic task stream and its three
// executors, on B200.
//
// The reference's first workload (src/workloads/synthetic.cuh,
// src/workloads/baselines.cuh, src/runtime/redistribute.cuh): tasks arrive
// open-loop (steady / bursty / skewed / a recorded trace), each with a payload
// of 4, 16 or 64 KB that lives on a source GPU and an FMA work count; an
// executor moves the payloads to the compute GPU and runs the task kernel.
//   A  static: wait for the last arrival, move the whole pool, one kernel,
//      every task completes then (baselines.cuh:139-188)
//   B  dynamic, not batched: per segment of `stride` tasks, once its last
//      task arrived: move, sync, compute, sync (baselines.cuh:190-243)
//   C  batched pipeline: batch size from the adaptive policy (choose_batch,
//      baselines.cuh:127-137, over choose_mb, adaptive_batch.cuh:31-36) or the
//      fixed maximum; moves on a copy stream, the task kernel waits on the
//      move's event, up to `pending_ahead` batches in flight; with overlap
//      off each batch is moved, computed and synchronised in turn
//      (baselines.cuh:255-409)
// Transports:
//   FERRY_TASKB_P2P         the compute GPU pulls the payloads with a copy
//                           kernel: 16-byte loads from the source GPU's HBM
//                           over NVLink (peer access), or HBM to HBM when
//                           source and destination are one GPU
//   FERRY_TASKB_HOST_STAGED the reference's channel
//                           (src/comm/host_staged_channel.cpp:43-87): pieces
//                           of at most one slot copied device-to-host into a
//                           ring of pinned slots on the source GPU's stream,
//                           host-to-device on the destination's, a slot
//                           reused after its last host-to-device copy
// Completion times are host times (the open-loop replay runs on the host
// clock, as the reference's does): a batch completes when its event is seen
// done -- polled while the executor waits for arrivals or window room, so a
// pipelined batch is not charged the rest of the submission loop.
#include <algorithm>
#include <chrono>
#include <random>
#include <thread>
#include <vector>

#include "common.cuh"

namespace ferry {
namespace {

// The task kernel (baselines.cuh:40-48): element i of the launch iterates
// v = fma(v, 1.0000001, 1e-7) works[i] * inner_scale times. The constants and
// the element-to-work pairing are the reference's, so that outputs compare
// value for value.
__global__ void taskb_kernel(const float* __restrict__ in, float* __restrict__ out, uint64_t n,
                             const int32_t* __restrict__ works, int inner_scale) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int w = works[i] * inner_scale;
  float v = in[i];
  for (int k = 0; k < w; ++k) v = fmaf(v, 1.0000001f, 1e-7f);
  out[i] = v;
}

// Payload move over the device address space (a peer GPU's HBM over NVLink,
// or this GPU's): 16-byte loads and stores, grid-stride (payloads and their
// offsets are multiples of 16 bytes, checked at create).
__global__ void __launch_bounds__(256) taskb_copy_kernel(const uint8_t* __restrict__ src,
                                                         uint8_t* __restrict__ dst, uint64_t bytes) {
  const uint64_t n16 = bytes >> 4;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {  // four loads in flight per thread
    const uint4 a = s[i], b = s[i + stride], c = s[i + 2 * stride], e = s[i + 3 * stride];
    d[i] = a;
    d[i + stride] = b;
    d[i + 2 * stride] = c;
    d[i + 3 * stride] = e;
  }
  for (; i < n16; i += stride) d[i] = s[i];
}

using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

// The reference's channel restated for the host-staged transport.
struct Staged {
  int src = 0, dst = 0, nslots = 0;
  size_t slot_bytes = 0;
  std::vector<uint8_t*> slot;
  std::vector<cudaEvent_t> d2h, h2d;
  std::vector<bool> used;
  cudaStream_t out_st = nullptr, in_st = nullptr;
  int next = 0, last = -1;

  int open(int s, int d, int n, size_t bytes) {
    src = s, dst = d, nslots = n, slot_bytes = bytes;
    slot.assign(n, nullptr);
    d2h.assign(n, nullptr);
    h2d.assign(n, nullptr);
    used.assign(n, false);
    FERRY_TRY(cudaSetDevice(src));
    FERRY_TRY(cudaStreamCreateWithFlags(&out_st, cudaStreamNonBlocking));
    for (int i = 0; i < n; ++i) {
      FERRY_TRY(cudaHostAlloc((void**)&slot[i], bytes, cudaHostAllocPortable));
      FERRY_TRY(cudaEventCreateWithFlags(&d2h[i], cudaEventDisableTiming));
    }
    FERRY_TRY(cudaSetDevice(dst));
    FERRY_TRY(cudaStreamCreateWithFlags(&in_st, cudaStreamNonBlocking));
    for (int i = 0; i < n; ++i) FERRY_TRY(cudaEventCreateWithFlags(&h2d[i], cudaEventDisableTiming));
    return FERRY_OK;
  }
  void close() {
    if (in_st) cudaStreamSynchronize(in_st);
    for (int i = 0; i < nslots; ++i) {
      if (slot[i]) cudaFreeHost(slot[i]);
      if (d2h[i]) cudaEventDestroy(d2h[i]);
      if (h2d[i]) cudaEventDestroy(h2d[i]);
    }
    if (out_st) cudaStreamDestroy(out_st);
    if (in_st) cudaStreamDestroy(in_st);
    out_st = in_st = nullptr;
    nslots = 0;
  }
  // [s, s + bytes) on the source GPU -> [d, d + bytes) on the destination
  int submit(const uint8_t* s, uint64_t bytes, uint8_t* d) {
    for (uint64_t off = 0; off < bytes;) {
      const uint64_t nb = std::min<uint64_t>(slot_bytes, bytes - off);
      const int k = next;
      next = (next + 1) % nslots;
      if (used[k]) FERRY_TRY(cudaEventSynchronize(h2d[k]));  // the slot's last copy out is done
      FERRY_TRY(cudaSetDevice(src));
      FERRY_TRY(cudaMemcpyAsync(slot[k], s + off, nb, cudaMemcpyDeviceToHost, out_st));
      FERRY_TRY(cudaEventRecord(d2h[k], out_st));
      FERRY_TRY(cudaSetDevice(dst));
      FERRY_TRY(cudaStreamWaitEvent(in_st, d2h[k], 0));
      FERRY_TRY(cudaMemcpyAsync(d + off, slot[k], nb, cudaMemcpyHostToDevice, in_st));
      FERRY_TRY(cudaEventRecord(h2d[k], in_st));
      used[k] = true;
      last = k;
      off += nb;
    }
    return FERRY_OK;
  }
  int wait_last(cudaStream_t st) {  // st (destination GPU) waits for the newest piece
    if (last >= 0) FERRY_TRY(cudaStreamWaitEvent(st, h2d[last], 0));
    return FERRY_OK;
  }
};

}  // namespace
}  // namespace ferry

using namespace ferry;

struct ferry_taskb {
  int src = 0, dst = 0;
  uint64_t n = 0, payload = 0;
  std::vector<double> arrive_ms_tick;  // arrival in ticks (times tick_ms per run)
  uint8_t* d_payload = nullptr;        // source GPU: n * payload bytes
  float* d_in = nullptr;               // destination GPU: the moved payloads
  float* d_out = nullptr;              // destination GPU: task kernel outputs
  int32_t* d_work = nullptr;           // destination GPU
  int peer = 0;                        // peer access enabled src -> dst
};

namespace {

int taskb_move(ferry_taskb* T, int transport, Staged* ch, cudaStream_t xs, uint64_t off_b, uint64_t bytes) {
  const uint8_t* s = T->d_payload + off_b;
  uint8_t* d = reinterpret_cast<uint8_t*>(T->d_in) + off_b;
  if (transport == FERRY_TASKB_HOST_STAGED) return ch->submit(s, bytes, d);
  FERRY_TRY(cudaSetDevice(T->dst));
  const uint64_t blocks = std::min<uint64_t>(std::max<uint64_t>(1, (bytes / 16 + 1023) / 1024), 148 * 8);
  taskb_copy_kernel<<<(unsigned)blocks, 256, 0, xs>>>(s, d, bytes);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

int taskb_compute(ferry_taskb* T, cudaStream_t cs, uint64_t off, uint64_t cnt, int inner) {
  const uint64_t pf = T->payload / 4;  // floats per task
  FERRY_TRY(cudaSetDevice(T->dst));
  taskb_kernel<<<(unsigned)((cnt + 255) / 256), 256, 0, cs>>>(T->d_in + off * pf, T->d_out + off * pf, cnt,
                                                               T->d_work + off, inner);
  FERRY_TRY(cudaGetLastError());
  return FERRY_OK;
}

// batch of the C executor starting at task `off` (baselines.cuh:127-137, or
// the fixed maximum with the policy's adaptation off)
uint64_t c_batch(const ferry_taskb_params* p, uint64_t n, uint64_t off, uint64_t payload) {
  if (p->adaptive) {
    const double pending_mb = (double)(n - off) * (double)payload / (1 << 20);
    double g = pending_mb / p->target_batches;  // choose_mb, adaptive_batch.cuh:31-36
    g = std::max(g, p->min_mb);
    g = std::min(g, p->max_mb);
    const uint64_t by_bytes = std::max<uint64_t>((uint64_t)(g * (1 << 20)), 64 * payload);
    return std::min<uint64_t>(std::max<uint64_t>(by_bytes / payload, 64), n - off);
  }
  const uint64_t by_bytes = (uint64_t)(p->max_mb * (1 << 20));
  return std::min<uint64_t>(std::max<uint64_t>(by_bytes / payload, 64), n - off);
}

}  // namespace

extern "C" {

int ferry_taskb_generate(const ferry_taskb_spec* s, uint64_t seed, const double* trace_ticks,
                         ferry_taskb_task* out) {
  if (!s || !out || s->arrival < FERRY_TASKB_STEADY || s->arrival > FERRY_TASKB_TRACE || s->sparsity < 0 ||
      s->sparsity > 2 || (s->arrival == FERRY_TASKB_TRACE && !trace_ticks))
    return set_error("taskb_generate: bad arguments"), FERRY_E_INVAL;
  // The generator of synthetic.cuh:83-173, restated draw for draw (the same
  // engine, distributions and order of draws) so that a seed gives the
  // reference's task stream.
  std::mt19937_64 rng(seed);
  const uint64_t payload = s->sparsity == 0 ? (4u << 10) : s->sparsity == 2 ? (64u << 10) : (16u << 10);
  std::uniform_int_distribution<int> uni_work(100, 200);
  std::uniform_real_distribution<double> unit(0.0, 1.0);
  std::exponential_distribution<double> exp_gap(1.0);
  std::exponential_distribution<double> pareto_gap(1.16);
  const int hot_cards = s->dest_hot_cards > 0 ? std::min(s->dest_hot_cards, std::max(1, s->num_gpus))
                                              : std::max(1, s->num_gpus / 5);
  double t = 0.0;
  for (uint64_t i = 0; i < s->total; ++i) {
    ferry_taskb_task& k = out[i];
    k.payload = payload;
    if (s->imbalanced) {
      const double u = unit(rng);
      k.work = u < 0.8 ? uni_work(rng) : uni_work(rng) * 8;
    } else {
      k.work = uni_work(rng);
    }
    if (s->arrival == FERRY_TASKB_TRACE) {
      k.arrive_t = trace_ticks[i];
      continue;
    }
    if (s->arrival == FERRY_TASKB_STEADY) {
      t += 1.0;
    } else if (s->arrival == FERRY_TASKB_BURSTY) {
      if (i % 64 == 0) t += exp_gap(rng) * 16.0;  // a row of 64 tasks lands on one tick
    } else {
      t += pareto_gap(rng) * 2.0;
    }
    k.arrive_t = t;
  }
  uint64_t rr = 0;
  for (uint64_t i = 0; i < s->total; ++i) {
    if (s->imbalanced && s->num_gpus > 1 && s->dest_hot_frac > 0.0) {
      const double u = (double)(rng() % 1000) / 1000.0;
      out[i].dest = u < s->dest_hot_frac ? (int)(rng() % (uint64_t)hot_cards)
                                         : (int)(rng() % (uint64_t)s->num_gpus);
    } else {
      out[i].dest = (int)(rr++ % (uint64_t)std::max(1, s->num_gpus));
    }
  }
  return FERRY_OK;
}

int ferry_taskb_create(int src_dev, int dst_dev, const ferry_taskb_task* tasks, uint64_t n, ferry_taskb** out) {
  if (!tasks || !out || n == 0 || src_dev < 0 || dst_dev < 0)
    return set_error("taskb_create: bad arguments"), FERRY_E_INVAL;
  const uint64_t payload = tasks[0].payload;
  if (payload < 16 || payload % 16)
    return set_error("taskb_create: payloads of a multiple of 16 bytes"), FERRY_E_INVAL;
  for (uint64_t i = 0; i < n; ++i)
    if (tasks[i].payload != payload || (i && tasks[i].arrive_t < tasks[i - 1].arrive_t) || tasks[i].work < 0)
      return set_error("taskb_create: one payload size, ascending arrivals"), FERRY_E_INVAL;
  int ndev = 0;
  FERRY_TRY(cudaGetDeviceCount(&ndev));
  if (src_dev >= ndev || dst_dev >= ndev) return set_error("taskb_create: no such device"), FERRY_E_INVAL;
  DeviceGuard guard(dst_dev);
  auto* T = new ferry_taskb();
  T->src = src_dev, T->dst = dst_dev, T->n = n, T->payload = payload;
  T->arrive_ms_tick.resize(n);
  for (uint64_t i = 0; i < n; ++i) T->arrive_ms_tick[i] = tasks[i].arrive_t;
  const uint64_t pool = n * payload;
  auto fail = [&](int rc) {
    ferry_taskb_destroy(T);
    return rc;
  };
  // payload pool on the source GPU, filled as the reference fills it
  // (baselines.cuh:82-93: mt19937_64 seed 9, (rng() % 1000) / 8 as float)
  std::vector<float> h(pool / 4);
  std::mt19937_64 rng(9);
  for (float& v : h) v = (float)(rng() % 1000) / 8.0f;
  if (cudaSetDevice(src_dev) != cudaSuccess || cudaMalloc(&T->d_payload, pool) != cudaSuccess ||
      cudaMemcpy(T->d_payload, h.data(), pool, cudaMemcpyHostToDevice) != cudaSuccess)
    return cudaGetLastError(), set_error("taskb_create: payload pool"), fail(FERRY_E_OOM);
  std::vector<int32_t> w(n);
  for (uint64_t i = 0; i < n; ++i) w[i] = tasks[i].work;
  if (cudaSetDevice(dst_dev) != cudaSuccess || cudaMalloc(&T->d_in, pool) != cudaSuccess ||
      cudaMalloc(&T->d_out, pool) != cudaSuccess || cudaMalloc(&T->d_work, n * 4) != cudaSuccess ||
      cudaMemset(T->d_in, 0, pool) != cudaSuccess || cudaMemset(T->d_out, 0, pool) != cudaSuccess ||
      cudaMemcpy(T->d_work, w.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return cudaGetLastError(), set_error("taskb_create: destination buffers"), fail(FERRY_E_OOM);
  if (src_dev != dst_dev) {
    int can = 0;
    if (cudaDeviceCanAccessPeer(&can, dst_dev, src_dev) != cudaSuccess) can = 0;
    if (can) {
      const cudaError_t e = cudaDeviceEnablePeerAccess(src_dev, 0);
      if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return set_error("taskb_create: peer access"), fail(FERRY_E_CUDA);
      cudaGetLastError();
      T->peer = 1;
    }
  }
  *out = T;
  return FERRY_OK;
}

int ferry_taskb_run(ferry_taskb* T, const ferry_taskb_params* p, ferry_taskb_stats* st) {
  if (!T || !p || !st || p->mode < FERRY_TASKB_A || p->mode > FERRY_TASKB_C || p->inner_scale < 0 ||
      p->tick_ms < 0 || p->stride < 1 || p->pending_ahead < 1 || p->max_mb <= 0 || p->min_mb <= 0 ||
      p->target_batches <= 0 || (p->transport != FERRY_TASKB_P2P && p->transport != FERRY_TASKB_HOST_STAGED))
    return set_error("taskb_run: bad arguments"), FERRY_E_INVAL;
  if (p->transport == FERRY_TASKB_P2P && T->src != T->dst && !T->peer)
    return set_error("taskb_run: devices %d and %d have no peer access", T->src, T->dst), FERRY_E_STATE;
  DeviceGuard guard(T->dst);
  const uint64_t n = T->n, pb = T->payload;
  std::vector<double> arrive(n), done(n, 0.0);
  for (uint64_t i = 0; i < n; ++i) arrive[i] = T->arrive_ms_tick[i] * p->tick_ms;
  *st = ferry_taskb_stats{};
  st->arrival_span_ms = arrive[n - 1];

  Staged ch;
  int rc = FERRY_OK;
  cudaStream_t cs = nullptr, xs = nullptr;
  std::vector<cudaEvent_t> evs;
  auto new_event = [&](cudaEvent_t* e) -> int {
    FERRY_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    evs.push_back(*e);
    return FERRY_OK;
  };
  auto cleanup = [&]() {
    if (cs) cudaStreamSynchronize(cs);
    if (xs) cudaStreamSynchronize(xs);
    ch.close();
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
    if (cs) cudaStreamDestroy(cs);
    if (xs) cudaStreamDestroy(xs);
  };
#define TB_TRY(x)              \
  do {                         \
    if ((rc = (x))) {          \
      cleanup();               \
      return rc;               \
    }                          \
  } while (0)
#define TB_CUDA(x)                                                 \
  do {                                                             \
    const cudaError_t e__ = (x);                                   \
    if (e__ != cudaSuccess) TB_TRY(::ferry::cuda_status(e__, #x)); \
  } while (0)
  TB_CUDA(cudaSetDevice(T->dst));
  TB_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
  TB_CUDA(cudaStreamCreateWithFlags(&xs, cudaStreamNonBlocking));
  // slots: the reference's rings (A: 4 x 4 MiB; B: 2 x 1 MiB; C: pending + 2 slots of max_mb)
  if (p->transport == FERRY_TASKB_HOST_STAGED) {
    if (p->mode == FERRY_TASKB_A)
      TB_TRY(ch.open(T->src, T->dst, 4, 4u << 20));
    else if (p->mode == FERRY_TASKB_B)
      TB_TRY(ch.open(T->src, T->dst, 2, 1u << 20));
    else
      TB_TRY(ch.open(T->src, T->dst, (int)p->pending_ahead + 2, (size_t)(p->max_mb * (1 << 20))));
  }
  const auto t0 = Clock::now();
  auto wait_until = [&](double ms) {
    while (ms_since(t0) < ms) std::this_thread::sleep_for(std::chrono::microseconds(50));
  };
  auto move_and_wait = [&](cudaStream_t waiter, uint64_t off, uint64_t cnt) -> int {
    int r = taskb_move(T, p->transport, &ch, xs, off * pb, cnt * pb);
    if (r) return r;
    if (p->transport == FERRY_TASKB_HOST_STAGED) return ch.wait_last(waiter);
    cudaEvent_t e;
    if ((r = new_event(&e))) return r;
    FERRY_TRY(cudaEventRecord(e, xs));
    FERRY_TRY(cudaStreamWaitEvent(waiter, e, 0));
    return FERRY_OK;
  };
  if (p->mode == FERRY_TASKB_A) {
    wait_until(arrive[n - 1]);  // the global barrier: every task has arrived
    TB_TRY(move_and_wait(cs, 0, n));
    TB_TRY(taskb_compute(T, cs, 0, n, p->inner_scale));
    TB_CUDA(cudaStreamSynchronize(cs));
    const double now = ms_since(t0);
    std::fill(done.begin(), done.end(), now);
    st->migrations = 1;
    st->migrated_bytes = n * pb;
    st->backlog_max = (double)n;
  } else if (p->mode == FERRY_TASKB_B) {
    for (uint64_t i = 0; i < n;) {
      const uint64_t cnt = std::min<uint64_t>((uint64_t)p->stride, n - i);
      wait_until(arrive[i + cnt - 1]);
      TB_TRY(move_and_wait(cs, i, cnt));
      TB_TRY(taskb_compute(T, cs, i, cnt, p->inner_scale));
      TB_CUDA(cudaStreamSynchronize(cs));
      const double now = ms_since(t0);
      std::fill(done.begin() + i, done.begin() + i + cnt, now);
      st->migrations += 1;
      st->migrated_bytes += cnt * pb;
      i += cnt;
    }
  } else {
    struct Batch {
      uint64_t off, cnt;
      cudaEvent_t ev;
    };
    std::vector<Batch> open;  // in flight, oldest first
    auto harvest = [&](bool block_oldest) -> int {
      size_t k = 0;
      for (; k < open.size(); ++k) {
        if (k == 0 && block_oldest) {
          FERRY_TRY(cudaEventSynchronize(open[k].ev));
        } else {
          const cudaError_t q = cudaEventQuery(open[k].ev);
          if (q == cudaErrorNotReady) break;
          FERRY_TRY(q);
        }
        const double now = ms_since(t0);
        std::fill(done.begin() + open[k].off, done.begin() + open[k].off + open[k].cnt, now);
      }
      open.erase(open.begin(), open.begin() + k);
      return FERRY_OK;
    };
    for (uint64_t off = 0; off < n;) {
      const uint64_t cnt = c_batch(p, n, off, pb);
      while (ms_since(t0) < arrive[off + cnt - 1]) {  // the batch's last task has not arrived
        TB_TRY(harvest(false));
        std::this_thread::sleep_for(std::chrono::microseconds(50));
      }
      if (p->overlap) {
        TB_TRY(harvest(false));
        while (open.size() >= p->pending_ahead) TB_TRY(harvest(true));
        TB_TRY(move_and_wait(cs, off, cnt));
        TB_TRY(taskb_compute(T, cs, off, cnt, p->inner_scale));
        Batch b{off, cnt, nullptr};
        TB_TRY(new_event(&b.ev));
        TB_CUDA(cudaEventRecord(b.ev, cs));
        open.push_back(b);
      } else {
        TB_TRY(move_and_wait(cs, off, cnt));
        TB_CUDA(cudaStreamSynchronize(cs));  // the move is complete before the kernel starts
        TB_TRY(taskb_compute(T, cs, off, cnt, p->inner_scale));
        TB_CUDA(cudaStreamSynchronize(cs));
        const double now = ms_since(t0);
        std::fill(done.begin() + off, done.begin() + off + cnt, now);
      }
      st->migrations += 1;
      st->migrated_bytes += cnt * pb;
      off += cnt;
    }
    while (!open.empty()) TB_TRY(harvest(true));
    st->backlog_max = p->overlap ? (double)p->pending_ahead : 0.0;
  }
  st->makespan_ms = ms_since(t0);
  std::vector<double> lat(n);
  for (uint64_t i = 0; i < n; ++i) lat[i] = done[i] - arrive[i];
  std::sort(lat.begin(), lat.end());
  st->p50_ms = lat[n / 2];
  st->p99_ms = lat[(size_t)(0.99 * (double)(n - 1))];
  st->throughput = (double)n / (st->makespan_ms / 1000.0);
  cleanup();
#undef TB_CUDA
#undef TB_TRY
  return FERRY_OK;
}

int ferry_taskb_results(ferry_taskb* T, float* host_out, uint64_t n_floats) {
  if (!T || !host_out || n_floats > T->n * T->payload / 4) return set_error("taskb_results: bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(T->dst);
  FERRY_TRY(cudaDeviceSynchronize());
  FERRY_TRY(cudaMemcpy(host_out, T->d_out, n_floats * 4, cudaMemcpyDeviceToHost));
  return FERRY_OK;
}

int ferry_taskb_reset(ferry_taskb* T) {
  if (!T) return set_error("taskb_reset: bad arguments"), FERRY_E_INVAL;
  DeviceGuard guard(T->dst);
  FERRY_TRY(cudaMemset(T->d_in, 0, T->n * T->payload));
  FERRY_TRY(cudaMemset(T->d_out, 0, T->n * T->payload));
  FERRY_TRY(cudaDeviceSynchronize());
  return FERRY_OK;
}

int ferry_taskb_destroy(ferry_taskb* T) {
  if (!T) return FERRY_OK;
  DeviceGuard guard(T->dst);
  if (T->d_payload) {
    cudaSetDevice(T->src);
    cudaFree(T->d_payload);
  }
  cudaSetDevice(T->dst);
  cudaFree(T->d_in);
  cudaFree(T->d_out);
  cudaFree(T->d_work);
  delete T;
  return FERRY_OK;
}

}  // extern "C"
