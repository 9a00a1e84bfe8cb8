// run_synthetic -- Workload B end to end on the C ABI.
//
// Counterpart of the reference's src/benches/run_synthetic.cu:24-123: one
// task stream (generate_tasks, src/workloads/synthetic.cuh:83-173) per
// scenario, run by baseline A, baseline B and executor C
// (src/workloads/baselines.cuh), each row the reference's ExecStats line;
// then C's speed-up over A and B and its transfers against B's. The payloads
// sit on --src and are computed on --dst; --transport p2p (default) moves them
// with a copy kernel on --dst reading --src's HBM (NVLink, or local), --transport
// host through the reference's pinned host ring. Uses nothing but
// include/ferry_cuda.h.
//
//   run_synthetic [--arrival steady|bursty|skewed] [--sparsity low|medium|high]
//                 [--skew balanced|imbalanced] [--tasks 65536] [--inner 1]
//                 [--tick 0.01] [--stride 64] [--pending 4] [--src 0] [--dst 0]
//                 [--transport p2p|host] [--seed 42] [--all]
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "ferry_cuda.h"

namespace {

#define CK(x)                                                                               \
  do {                                                                                      \
    const int rc__ = (x);                                                                   \
    if (rc__ != FERRY_OK) {                                                                 \
      std::fprintf(stderr, "%s failed: status %d: %s\n", #x, rc__, ferry_last_error());     \
      std::exit(1);                                                                         \
    }                                                                                       \
  } while (0)

int arrival_of(const std::string& s) {
  if (s == "steady") return FERRY_TASKB_STEADY;
  if (s == "bursty") return FERRY_TASKB_BURSTY;
  if (s == "skewed") return FERRY_TASKB_SKEWED;
  std::fprintf(stderr, "unknown arrival %s\n", s.c_str());
  std::exit(2);
}

int sparsity_of(const std::string& s) {
  if (s == "low") return 0;
  if (s == "medium") return 1;
  if (s == "high") return 2;
  std::fprintf(stderr, "unknown sparsity %s\n", s.c_str());
  std::exit(2);
}

void print_row(const char* name, const ferry_taskb_stats& st) {
  std::printf("  %-10s makespan=%9.2fms  tput=%9.0f t/s  p50=%9.2f  p99=%10.2f  migr=%7llu  bytes=%9.2fMB\n", name,
              st.makespan_ms, st.throughput, st.p50_ms, st.p99_ms, (unsigned long long)st.migrations,
              st.migrated_bytes / 1048576.0);
  std::fflush(stdout);
}

struct Opt {
  std::string arrival = "steady", sparsity = "medium", skew = "balanced", transport = "p2p";
  uint64_t tasks = 1 << 16, seed = 42;
  int inner = 1, stride = 64, src = 0, dst = 0;
  uint64_t pending = 4;
  double tick = 0.01;
};

void run_scenario(const Opt& o) {
  std::printf("[scenario] arrival=%s sparsity=%s skew=%s tasks=%llu tick=%.3fms transport=%s\n", o.arrival.c_str(),
              o.sparsity.c_str(), o.skew.c_str(), (unsigned long long)o.tasks, o.tick, o.transport.c_str());
  ferry_taskb_spec sp{};
  sp.arrival = arrival_of(o.arrival);
  sp.sparsity = sparsity_of(o.sparsity);
  sp.imbalanced = o.skew == "imbalanced";
  sp.num_gpus = 1;
  sp.total = o.tasks;
  sp.dest_hot_frac = 0.8;
  std::vector<ferry_taskb_task> tasks(o.tasks);
  CK(ferry_taskb_generate(&sp, o.seed, nullptr, tasks.data()));
  ferry_taskb* tb = nullptr;
  CK(ferry_taskb_create(o.src, o.dst, tasks.data(), o.tasks, &tb));
  ferry_taskb_params p{};
  p.transport = o.transport == "host" ? FERRY_TASKB_HOST_STAGED : FERRY_TASKB_P2P;
  p.inner_scale = o.inner;
  p.stride = o.stride;
  p.tick_ms = o.tick;
  p.pending_ahead = o.pending;
  p.adaptive = 1;
  p.overlap = 1;
  p.min_mb = 1.0;  // AdaptiveBatchPolicy, 8 target batches (run_synthetic.cu:99-102)
  p.max_mb = 4.0;
  p.target_batches = 8.0;
  ferry_taskb_stats a{}, b{}, c{};
  p.mode = FERRY_TASKB_A;
  CK(ferry_taskb_run(tb, &p, &a));
  print_row("baseline-A", a);
  p.mode = FERRY_TASKB_B;
  CK(ferry_taskb_run(tb, &p, &b));
  print_row("baseline-B", b);
  p.mode = FERRY_TASKB_C;
  CK(ferry_taskb_run(tb, &p, &c));
  print_row("ferry-C", c);
  std::printf("  => C vs A: %.2fx   C vs B: %.2fx   migrations C/B: %.4f\n\n", a.makespan_ms / c.makespan_ms,
              b.makespan_ms / c.makespan_ms, b.migrations ? (double)c.migrations / (double)b.migrations : 1.0);
  std::fflush(stdout);
  CK(ferry_taskb_destroy(tb));
}

}  // namespace

int main(int argc, char** argv) {
  Opt o;
  bool all = false;
  for (int i = 1; i < argc; ++i) {
    auto next = [&]() -> const char* {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "%s needs a value\n", argv[i]);
        std::exit(2);
      }
      return argv[++i];
    };
    const std::string a = argv[i];
    if (a == "--arrival") o.arrival = next();
    else if (a == "--sparsity") o.sparsity = next();
    else if (a == "--skew") o.skew = next();
    else if (a == "--tasks") o.tasks = std::strtoull(next(), nullptr, 10);
    else if (a == "--inner") o.inner = std::atoi(next());
    else if (a == "--tick") o.tick = std::atof(next());
    else if (a == "--stride") o.stride = std::atoi(next());
    else if (a == "--pending") o.pending = std::strtoull(next(), nullptr, 10);
    else if (a == "--src") o.src = std::atoi(next());
    else if (a == "--dst") o.dst = std::atoi(next());
    else if (a == "--transport") o.transport = next();
    else if (a == "--seed") o.seed = std::strtoull(next(), nullptr, 10);
    else if (a == "--all") all = true;
    else {
      std::fprintf(stderr, "unknown option %s\n", a.c_str());
      return 2;
    }
  }
  if (all) {
    for (const char* arr : {"steady", "bursty", "skewed"})
      for (const char* sk : {"balanced", "imbalanced"}) {
        Opt s = o;
        s.arrival = arr;
        s.skew = sk;
        run_scenario(s);
      }
  } else {
    run_scenario(o);
  }
  return 0;
}
