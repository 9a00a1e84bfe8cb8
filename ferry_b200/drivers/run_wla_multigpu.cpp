// run_wla_multigpu -- the multi-GPU decode job on the C ABI, one host thread per
// GPU in one process.
//
// Counterpart of the reference's src/benches/run_wla_multigpu.cu:164-269 and
// the runtime it drives (WlaMultiGpuCtx, src/runtime/wla_multigpu.cuh:2291-2775):
// requests homed on GPUs round-robin or skewed, every GPU's exec thread ticks
// its executor (ferry_exec_tick: pop from its device deque, water-level steal
// from the peer deque with the largest excess, NVLink migration of stolen
// requests, fused decode step, push back), and at every epoch the threads
// share their ownership counts through host memory under a mutex -- the
// reference's own shared pending count (wla_multigpu.cuh:1518-1526) -- so the
// fair share and the termination test see the whole job. In one process the
// peers are linked directly (ferry_ctx_link, ferry_deque_peer_view); across
// processes the same executor runs with CUDA IPC handles and the NCCL
// ownership exchange (ferry_b200/cluster.py). Uses only include/ferry_cuda.h
// and the CUDA runtime.
//
//   run_wla_multigpu [--gpus 0,1] [--requests-per-gpu 16] [--steps 32]
//                    [--ctx 4096] [--heads 32] [--top-k 64] [--cache-frac 0.25]
//                    [--skew balanced|imbalanced] [--steal-batch 4]
//                    [--max-batch 16] [--kv-mode delta|full|drop] [--epoch 4]
//                    [--seed 42]
//
// --gpus may repeat a device ("0,0"): two executors then share one GPU.
// imbalanced: 80% of the requests on the first half of the GPUs (the
// reference's skew, wla_multigpu.cuh:483-492). Prints per GPU the tokens
// decoded, steals, stolen tasks and migrated bytes, then the job's decode
// tokens/s over the slowest GPU's device time and a check that every
// (request, step) was decoded exactly once in total.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "ferry_cuda.h"

namespace {

#define CK(x)                                                                            \
  do {                                                                                   \
    const int rc__ = (x);                                                                \
    if (rc__ != FERRY_OK) {                                                              \
      std::fprintf(stderr, "%s failed: status %d: %s\n", #x, rc__, ferry_last_error()); \
      std::exit(1);                                                                      \
    }                                                                                    \
  } while (0)
#define CU(x)                                                               \
  do {                                                                      \
    const cudaError_t e__ = (x);                                            \
    if (e__ != cudaSuccess) {                                               \
      std::fprintf(stderr, "%s failed: %s\n", #x, cudaGetErrorString(e__)); \
      std::exit(1);                                                         \
    }                                                                       \
  } while (0)

struct Args {
  std::vector<int> gpus{0, 1};
  int per_gpu = 16, steps = 32, ctx = 4096, heads = 32, top_k = 64, steal_batch = 4, max_batch = 16,
      epoch = 4;
  double cache_frac = 0.25;
  bool imbalanced = false;
  int mode = FERRY_MIGRATE_DELTA;
  uint64_t seed = 42;
};

Args parse(int argc, char** argv) {
  Args a;
  for (int i = 1; i < argc; ++i) {
    const std::string k = argv[i];
    auto val = [&]() -> std::string {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "%s needs a value\n", k.c_str());
        std::exit(2);
      }
      return argv[++i];
    };
    if (k == "--gpus") {
      a.gpus.clear();
      const std::string v = val();
      size_t p = 0;
      while (p <= v.size()) {
        const size_t q = v.find(',', p);
        a.gpus.push_back(std::atoi(v.substr(p, q == std::string::npos ? std::string::npos : q - p).c_str()));
        if (q == std::string::npos) break;
        p = q + 1;
      }
    } else if (k == "--requests-per-gpu") a.per_gpu = std::atoi(val().c_str());
    else if (k == "--steps") a.steps = std::atoi(val().c_str());
    else if (k == "--ctx") a.ctx = std::atoi(val().c_str());
    else if (k == "--heads") a.heads = std::atoi(val().c_str());
    else if (k == "--top-k") a.top_k = std::atoi(val().c_str());
    else if (k == "--cache-frac") a.cache_frac = std::atof(val().c_str());
    else if (k == "--steal-batch") a.steal_batch = std::atoi(val().c_str());
    else if (k == "--max-batch") a.max_batch = std::atoi(val().c_str());
    else if (k == "--epoch") a.epoch = std::atoi(val().c_str());
    else if (k == "--seed") a.seed = std::strtoull(val().c_str(), nullptr, 10);
    else if (k == "--skew") a.imbalanced = val() == "imbalanced";
    else if (k == "--kv-mode") {
      const std::string m = val();
      a.mode = m == "full" ? FERRY_MIGRATE_FULL : m == "drop" ? FERRY_MIGRATE_DROP : FERRY_MIGRATE_DELTA;
    } else {
      std::fprintf(stderr, "unknown option %s\n", k.c_str());
      std::exit(2);
    }
  }
  if (a.gpus.empty() || a.gpus.size() > FERRY_MAX_PEERS + 1) {
    std::fprintf(stderr, "--gpus: 1 to %d devices\n", FERRY_MAX_PEERS + 1);
    std::exit(2);
  }
  return a;
}

uint64_t splitmix(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

uint16_t hash_normal_f16(uint64_t seed, uint64_t idx) {
  const uint64_t a = splitmix(seed ^ splitmix(idx)), b = splitmix(a), c = splitmix(b);
  const uint64_t w[3] = {a, b, c};
  float s = 0.f;
  for (int i = 0; i < 12; ++i) s += (float)((w[i / 4] >> (16 * (i % 4))) & 0xFFFF) * (1.0f / 65536.0f);
  const __half h = __float2half_rn(s - 6.0f);
  uint16_t bits;
  std::memcpy(&bits, &h, 2);
  return bits;
}

// The threads' shared ownership state: the in-process form of the exchange.
// The last thread to arrive sums every thread's counts into the snapshot the
// others read after waking; the snapshot cannot change before they read it,
// since the next one needs every thread to arrive again.
struct Shared {
  std::mutex mu;
  std::condition_variable cv;
  int world = 0, arrived = 0;
  uint64_t generation = 0;
  std::vector<int64_t> admitted, finished;
  int64_t snap_adm = 0, snap_fin = 0;
  void barrier_exchange(int rank, int64_t adm, int64_t fin, int64_t* adm_all, int64_t* fin_all) {
    std::unique_lock<std::mutex> lk(mu);
    admitted[rank] = adm;
    finished[rank] = fin;
    const uint64_t gen = generation;
    if (++arrived == world) {
      int64_t a = 0, f = 0;
      for (int r = 0; r < world; ++r) {
        a += admitted[r];
        f += finished[r];
      }
      snap_adm = a;
      snap_fin = f;
      arrived = 0;
      ++generation;
      cv.notify_all();
    } else {
      cv.wait(lk, [&] { return generation != gen; });
    }
    *adm_all = snap_adm;
    *fin_all = snap_fin;
  }
};

struct Rank {
  int device = 0;
  ferry_ctx* ctx = nullptr;
  ferry_deque* deque = nullptr;
  ferry_exec* exec = nullptr;
  void* pool = nullptr;
  uint16_t* d_q = nullptr;
  cudaStream_t st = nullptr;
  std::vector<ferry_deque*> views;
  int64_t tokens = 0, steals = 0, stolen = 0, mig_bytes = 0;
  float device_ms = 0.f;
};

}  // namespace

int main(int argc, char** argv) {
  const Args a = parse(argc, argv);
  const int W = (int)a.gpus.size();
  const int total = a.per_gpu * W;
  const int N = a.ctx / 16;
  const int C = std::max(a.top_k, (int)std::lround(a.cache_frac * N));
  const int slots = std::min(total, 2 * a.per_gpu + a.max_batch);  // the busiest home + stolen work
  const size_t q_row = (size_t)a.heads * 128;
  ferry_cfg cfg{slots, 1, a.heads, a.heads, 128, 16, N, C, a.top_k, FERRY_KV_F16};

  // homes: round-robin, or 80% of the requests on the first half of the GPUs
  std::vector<int> home(total);
  {
    std::mt19937_64 rng(7);
    std::uniform_real_distribution<double> u(0.0, 1.0);
    const int half = std::max(1, W / 2);
    for (int r = 0; r < total; ++r)
      home[r] = !a.imbalanced ? r % W
                              : (u(rng) < 0.8 ? (int)(rng() % half) : half + (int)(rng() % std::max(1, W - half)));
    for (auto& h : home) h = std::min(h, W - 1);
  }

  // per GPU: ctx, pinned pool with the procedural KV of every request (homes
  // r * Hkv * N), device deque, resident query table, executor
  std::vector<Rank> R(W);
  std::vector<uint16_t> hq((size_t)total * a.steps * q_row);
  for (size_t i = 0; i < hq.size(); ++i) hq[i] = hash_normal_f16(a.seed ^ 0x51ull, i);
  const int64_t units = (int64_t)total * a.heads * N;
  for (int g = 0; g < W; ++g) {
    Rank& k = R[g];
    k.device = a.gpus[g];
    CU(cudaSetDevice(k.device));
    CU(cudaStreamCreate(&k.st));
    CK(ferry_ctx_create(k.device, &cfg, &k.ctx));
    CK(ferry_host_alloc((size_t)units * 8192, &k.pool));
    CK(ferry_kv_generate(k.st, a.seed, 0, units, k.pool, FERRY_KV_F16));
    CU(cudaStreamSynchronize(k.st));
    CK(ferry_kv_register(k.ctx, k.pool, (size_t)units * 8192));
    CK(ferry_page_summary_update(k.ctx, k.st, 0, units));
    CK(ferry_deque_create(k.device, (uint64_t)slots, &k.deque));
    CU(cudaMalloc(&k.d_q, hq.size() * 2));
    CU(cudaMemcpy(k.d_q, hq.data(), hq.size() * 2, cudaMemcpyHostToDevice));
    ferry_exec_cfg ec{g, W, a.max_batch, a.steal_batch, a.mode, a.steps, total, 0};
    CK(ferry_exec_create(k.ctx, k.deque, &ec, k.d_q, &k.exec));
    CU(cudaStreamSynchronize(k.st));
  }
  // peers in this process: direct links (peer access) and deque views
  for (int g = 0; g < W; ++g) {
    int slot = 0;
    for (int p = 0; p < W; ++p) {
      if (p == g) continue;
      CK(ferry_ctx_link(R[g].ctx, slot, R[p].ctx));
      ferry_deque* v = nullptr;
      CK(ferry_deque_peer_view(R[g].device, R[p].deque, &v));
      R[g].views.push_back(v);
      CK(ferry_exec_link_peer(R[g].exec, p, slot, v));
      ++slot;
    }
  }

  Shared sh;
  sh.world = W;
  sh.admitted.assign(W, 0);
  sh.finished.assign(W, 0);
  auto worker = [&](int g) {
    Rank& k = R[g];
    CU(cudaSetDevice(k.device));
    std::vector<int32_t> mine, pages;
    for (int r = 0; r < total; ++r)
      if (home[r] == g) mine.push_back(r);
    pages.assign(mine.size(), N);
    // every request arrives at tick 0 (one burst); admitted as slots free
    if (!mine.empty()) CK(ferry_exec_admit(k.exec, mine.data(), pages.data(), (int)mine.size()));
    int64_t admitted = (int64_t)mine.size(), finished = 0;
    cudaEvent_t e0, e1;
    CU(cudaEventCreate(&e0));
    CU(cudaEventCreate(&e1));
    CU(cudaEventRecord(e0, k.st));
    ferry_tick_stats ts{};
    for (int64_t t = 1; t < 1000000; ++t) {
      CK(ferry_exec_tick(k.exec, k.st, &ts));
      k.tokens += ts.decoded;
      finished += ts.finished;
      if (ts.stolen) {
        ++k.steals;
        k.stolen += ts.stolen;
        k.mig_bytes += ts.mig_bytes;
      }
      if (t % a.epoch == 0) {
        int64_t adm_all = 0, fin_all = 0;
        sh.barrier_exchange(g, admitted, finished, &adm_all, &fin_all);
        CK(ferry_exec_set_global(k.exec, adm_all - fin_all));
        if (fin_all >= total) break;
      }
    }
    CU(cudaEventRecord(e1, k.st));
    CU(cudaStreamSynchronize(k.st));
    CU(cudaEventElapsedTime(&k.device_ms, e0, e1));
    CK(ferry_ctx_check(k.ctx));
  };
  std::vector<std::thread> th;
  for (int g = 0; g < W; ++g) th.emplace_back(worker, g);
  for (auto& x : th) x.join();

  int64_t tokens = 0;
  float ms = 0.f;
  std::printf("[wla] gpus=%d requests=%d steps=%d sel=%d hot=%d skew=%s kv-mode=%s steal-batch=%d\n", W, total,
              a.steps, a.top_k, C, a.imbalanced ? "imbalanced" : "balanced",
              a.mode == FERRY_MIGRATE_FULL ? "full" : a.mode == FERRY_MIGRATE_DROP ? "drop" : "delta",
              a.steal_batch);
  for (int g = 0; g < W; ++g) {
    const Rank& k = R[g];
    const int homed = (int)std::count(home.begin(), home.end(), g);
    std::printf("  gpu%d dev=%d homed=%d tokens=%lld steals=%lld stolen=%lld migrated=%.2fMB device_ms=%.2f\n", g,
                k.device, homed, (long long)k.tokens, (long long)k.steals, (long long)k.stolen,
                k.mig_bytes / 1048576.0, k.device_ms);
    tokens += k.tokens;
    ms = std::max(ms, k.device_ms);
  }
  const bool exact = tokens == (int64_t)total * a.steps;
  std::printf("  tokens=%lld expected=%lld exactly_once=%s tokens/s=%.1f\n", (long long)tokens,
              (long long)total * a.steps, exact ? "yes" : "NO", tokens / (ms / 1e3));
  for (int g = 0; g < W; ++g) {
    Rank& k = R[g];
    CU(cudaSetDevice(k.device));
    for (auto* v : k.views) CK(ferry_deque_destroy(v));
    CK(ferry_exec_destroy(k.exec));
    CK(ferry_deque_destroy(k.deque));
    cudaFree(k.d_q);
    CK(ferry_ctx_destroy(k.ctx));
    CK(ferry_host_free(k.pool));
    cudaStreamDestroy(k.st);
  }
  return exact ? 0 : 3;
}
