// run_missstream -- the single-GPU miss-stream decode driver on the C ABI.
//
// Counterpart of the reference's src/benches/run_missstream.cu:33-67 (and the
// executor it drives, run_miss_workload mode C, src/workloads/kv_exec.cuh:
// 187-292): a job of requests arriving over decode ticks, each decoding
// `steps` tokens; every tick runs one fused ferry_decode_step over the active
// requests (select -> miss detect -> gather from pinned host memory ->
// attention) and is timed with CUDA events. Prints the reference's WlAStats
// line (makespan, steps/s, p50/p99 step, refill events and bytes) plus
// decode tokens/s. It uses nothing but include/ferry_cuda.h and the CUDA
// runtime -- the drop-in a reference build would link.
//
//   run_missstream [--requests 16] [--ctx 4096] [--layers 1] [--heads 32]
//                  [--kv-heads 32] [--top-k 64] [--cache-frac 0.25]
//                  [--steps 200] [--rate 50] [--tick-ms 20] [--seed 42]
//                  [--device 0] [--q-file F] [--join-file F] [--out-file F]
//                  [--select quest]
//
// --q-file: fp16 queries [requests][steps][layers][heads][128] (default: a
// counter hash of (seed, request, step, layer, head, dim), N(0,1) by an
// Irwin-Hall sum). --join-file: int64 join tick per request (default: Poisson
// arrivals at --rate on a --tick-ms tick, std::mt19937_64(seed)).
// --out-file: every tick's attention output appended in tick order, fp32
// [active][layers][heads][128].
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "ferry_cuda.h"

namespace {

#define CK(x)                                                                     \
  do {                                                                            \
    const int rc__ = (x);                                                         \
    if (rc__ != FERRY_OK) {                                                       \
      std::fprintf(stderr, "%s failed: status %d: %s\n", #x, rc__, ferry_last_error()); \
      std::exit(1);                                                               \
    }                                                                             \
  } while (0)
#define CU(x)                                                                   \
  do {                                                                          \
    const cudaError_t e__ = (x);                                                \
    if (e__ != cudaSuccess) {                                                   \
      std::fprintf(stderr, "%s failed: %s\n", #x, cudaGetErrorString(e__));     \
      std::exit(1);                                                             \
    }                                                                           \
  } while (0)

struct Args {
  int requests = 16, ctx = 4096, layers = 1, heads = 32, kv_heads = 32, top_k = 64, steps = 200;
  double cache_frac = 0.25, rate = 50.0, tick_ms = 20.0;
  uint64_t seed = 42;
  int device = 0;
  bool quest = false;
  std::string q_file, join_file, out_file;
};

Args parse(int argc, char** argv) {
  Args a;
  for (int i = 1; i < argc; ++i) {
    const std::string k = argv[i];
    auto val = [&]() -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "%s needs a value\n", k.c_str());
        std::exit(2);
      }
      return argv[++i];
    };
    if (k == "--requests") a.requests = std::atoi(val());
    else if (k == "--ctx") a.ctx = std::atoi(val());
    else if (k == "--layers") a.layers = std::atoi(val());
    else if (k == "--heads") a.heads = std::atoi(val());
    else if (k == "--kv-heads") a.kv_heads = std::atoi(val());
    else if (k == "--top-k") a.top_k = std::atoi(val());
    else if (k == "--steps") a.steps = std::atoi(val());
    else if (k == "--cache-frac") a.cache_frac = std::atof(val());
    else if (k == "--rate") a.rate = std::atof(val());
    else if (k == "--tick-ms") a.tick_ms = std::atof(val());
    else if (k == "--seed") a.seed = std::strtoull(val(), nullptr, 10);
    else if (k == "--device") a.device = std::atoi(val());
    else if (k == "--q-file") a.q_file = val();
    else if (k == "--join-file") a.join_file = val();
    else if (k == "--out-file") a.out_file = val();
    else if (k == "--select") a.quest = std::string(val()) == "quest";
    else {
      std::fprintf(stderr, "unknown option %s\n", k.c_str());
      std::exit(2);
    }
  }
  return a;
}

uint64_t splitmix(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// N(0,1) by the sum of twelve 16-bit uniforms (Irwin-Hall), as fp16
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

template <class T>
std::vector<T> read_file(const std::string& path, size_t count) {
  std::vector<T> v(count);
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f || std::fread(v.data(), sizeof(T), count, f) != count) {
    std::fprintf(stderr, "cannot read %zu items from %s\n", count, path.c_str());
    std::exit(1);
  }
  std::fclose(f);
  return v;
}

}  // namespace

int main(int argc, char** argv) {
  const Args a = parse(argc, argv);
  const int N = a.ctx / 16, LH = a.layers * a.kv_heads;
  const int C = std::max(a.top_k, (int)std::lround(a.cache_frac * N));
  const size_t q_row = (size_t)a.layers * a.heads * 128;  // fp16 elements per (request, step)
  ferry_cfg cfg{a.requests, a.layers, a.heads, a.kv_heads, 128, 16, N, C, a.top_k, FERRY_KV_F16};
  CU(cudaSetDevice(a.device));
  ferry_ctx* ctx = nullptr;
  CK(ferry_ctx_create(a.device, &cfg, &ctx));
  if (a.quest) CK(ferry_select_mode(ctx, FERRY_SELECT_QUEST));
  cudaStream_t st;
  CU(cudaStreamCreate(&st));

  // pinned host pool with the procedural KV; every unit's page summary on the device
  const int64_t units = (int64_t)a.requests * LH * N;
  void* pool = nullptr;
  CK(ferry_host_alloc((size_t)units * 8192, &pool));
  CK(ferry_kv_generate(st, a.seed, 0, units, pool, FERRY_KV_F16));
  CU(cudaStreamSynchronize(st));
  CK(ferry_kv_register(ctx, pool, (size_t)units * 8192));
  CK(ferry_page_summary_update(ctx, st, 0, units));

  // arrivals
  std::vector<int64_t> join(a.requests);
  if (!a.join_file.empty()) {
    join = read_file<int64_t>(a.join_file, a.requests);
  } else {
    std::mt19937_64 rng(a.seed);
    std::exponential_distribution<double> gap(a.rate / 1000.0);
    double t = 0.0;
    for (int r = 0; r < a.requests; ++r) {
      t += gap(rng);
      join[r] = (int64_t)std::ceil(t / a.tick_ms);
    }
  }
  const int64_t j0 = *std::min_element(join.begin(), join.end());
  for (auto& j : join) j -= j0;
  const int64_t ticks = *std::max_element(join.begin(), join.end()) + a.steps;

  // queries, resident on the device: [requests][steps][layers][heads][128]
  std::vector<uint16_t> hq;
  if (!a.q_file.empty()) {
    hq = read_file<uint16_t>(a.q_file, (size_t)a.requests * a.steps * q_row);
  } else {
    hq.resize((size_t)a.requests * a.steps * q_row);
    for (size_t i = 0; i < hq.size(); ++i) hq[i] = hash_normal_f16(a.seed ^ 0x51ull, i);
  }
  uint16_t *d_qtab = nullptr, *d_q = nullptr;
  int32_t *d_ids = nullptr, *d_new = nullptr, *d_pages = nullptr;
  float* d_out = nullptr;
  CU(cudaMalloc(&d_qtab, hq.size() * 2));
  CU(cudaMemcpy(d_qtab, hq.data(), hq.size() * 2, cudaMemcpyHostToDevice));
  CU(cudaMalloc(&d_q, (size_t)a.requests * q_row * 2));
  CU(cudaMalloc(&d_ids, a.requests * 4));
  CU(cudaMalloc(&d_new, a.requests * 4));
  CU(cudaMalloc(&d_pages, a.requests * 4));
  CU(cudaMalloc(&d_out, (size_t)a.requests * q_row * 4));
  {
    std::vector<int32_t> np(a.requests, N);
    CU(cudaMemcpy(d_pages, np.data(), a.requests * 4, cudaMemcpyHostToDevice));
  }
  FILE* fout = a.out_file.empty() ? nullptr : std::fopen(a.out_file.c_str(), "wb");
  std::vector<float> hout((size_t)a.requests * q_row);

  std::vector<cudaEvent_t> ev;
  std::vector<int> tick_tokens;
  int64_t tokens = 0;
  cudaEvent_t e_begin, e_end;
  CU(cudaEventCreate(&e_begin));
  CU(cudaEventCreate(&e_end));
  uint64_t stats0[FERRY_NUM_STATS];
  CK(ferry_stats_read(ctx, stats0, 1));
  CU(cudaEventRecord(e_begin, st));
  for (int64_t t = 0; t < ticks; ++t) {
    std::vector<int32_t> active, fresh;
    for (int r = 0; r < a.requests; ++r) {
      const int64_t s = t - join[r];
      if (s >= 0 && s < a.steps) {
        active.push_back(r);
        if (s == 0) fresh.push_back(r);
      }
    }
    if (active.empty()) continue;
    if (!fresh.empty()) {
      CU(cudaMemcpyAsync(d_new, fresh.data(), fresh.size() * 4, cudaMemcpyHostToDevice, st));
      CK(ferry_requests_begin(ctx, st, d_new, d_pages, nullptr, (int)fresh.size()));
    }
    // this tick's queries: one row per active request (request r at step t - join[r])
    for (size_t i = 0; i < active.size(); ++i) {
      const int r = active[i];
      const size_t row = (size_t)r * a.steps + (size_t)(t - join[r]);
      CU(cudaMemcpyAsync(d_q + i * q_row, d_qtab + row * q_row, q_row * 2, cudaMemcpyDeviceToDevice, st));
    }
    CU(cudaMemcpyAsync(d_ids, active.data(), active.size() * 4, cudaMemcpyHostToDevice, st));
    cudaEvent_t e0, e1;
    CU(cudaEventCreate(&e0));
    CU(cudaEventCreate(&e1));
    CU(cudaEventRecord(e0, st));
    CK(ferry_decode_step(ctx, st, d_q, d_ids, (int)active.size(), d_out));
    CU(cudaEventRecord(e1, st));
    ev.push_back(e0);
    ev.push_back(e1);
    tick_tokens.push_back((int)active.size());
    tokens += (int64_t)active.size();
    if (fout) {
      CU(cudaMemcpyAsync(hout.data(), d_out, active.size() * q_row * 4, cudaMemcpyDeviceToHost, st));
      CU(cudaStreamSynchronize(st));
      std::fwrite(hout.data(), 4, active.size() * q_row, fout);
    }
  }
  CU(cudaEventRecord(e_end, st));
  CU(cudaStreamSynchronize(st));
  CK(ferry_ctx_check(ctx));
  if (fout) std::fclose(fout);
  uint64_t stats[FERRY_NUM_STATS];
  CK(ferry_stats_read(ctx, stats, 0));

  std::vector<float> step_ms;
  double span = 0.0;
  for (size_t i = 0; i < ev.size(); i += 2) {
    float ms = 0.f;
    CU(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
    step_ms.push_back(ms);
    span += ms;
  }
  float wall = 0.f;
  CU(cudaEventElapsedTime(&wall, e_begin, e_end));
  std::vector<float> srt = step_ms;
  std::sort(srt.begin(), srt.end());
  const float p50 = srt.empty() ? 0.f : srt[srt.size() / 2];
  const float p99 = srt.empty() ? 0.f : srt[(size_t)(0.99 * (srt.size() - 1))];
  std::printf("[wlA] reqs=%d layers=%d steps=%d sel=%d hot=%d unit=8192B select=%s\n", a.requests, a.layers,
              a.steps, a.top_k, C, a.quest ? "quest" : "mean");
  std::printf("  %-10s makespan=%9.2fms steps/s=%8.1f p50=%7.3f p99=%8.3f refill=%8llu bytes=%9.2fMB\n",
              "ferry-b200", span, step_ms.size() / (span / 1e3), p50, p99, (unsigned long long)stats[0],
              stats[1] / 1048576.0);
  std::printf("  tokens=%lld ticks=%zu tokens/s(device, step sum)=%.1f tokens/s(stream wall)=%.1f\n",
              (long long)tokens, step_ms.size(), tokens / (span / 1e3), tokens / (wall / 1e3));
  for (auto e : ev) cudaEventDestroy(e);
  cudaFree(d_qtab);
  cudaFree(d_q);
  cudaFree(d_ids);
  cudaFree(d_new);
  cudaFree(d_pages);
  cudaFree(d_out);
  CK(ferry_ctx_destroy(ctx));
  CK(ferry_host_free(pool));
  cudaStreamDestroy(st);
  return 0;
}
