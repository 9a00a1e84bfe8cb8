// ref_driver.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Thin extern "C" shim over the reference's own host-only headers, compiled in
// place from the reference tree by oracle/Makefile (nothing is copied):
//   workloads/missstream.cuh     replay_miss_stream  (missstream.cuh:104-170)
//   workloads/miss_trace.cuh     load_miss_trace     (miss_trace.cuh:75-185)
//   runtime/adaptive_batch.cuh   choose_mb           (adaptive_batch.cuh:31-36)
//   workloads/synthetic.cuh      generate_tasks      (synthetic.cuh:83-173)
// The output (oracle/_ref/libferry_ref.so and oracle/_ref/ref_trace_check) is
// used only to validate the oracle restatement (ferry_oracle.cpp) and the GPU
// miss-detect kernel against the reference's exact LRU.

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "runtime/adaptive_batch.cuh"
#include "workloads/miss_trace.cuh"
#include "workloads/missstream.cuh"
#include "workloads/synthetic.cuh"

namespace {
ferry::MissSpec make_spec(int R, int L, int S, int sel, int hot, int kv, int d,
                          uint64_t seed) {
  ferry::MissSpec sp;
  sp.num_requests = R;
  sp.num_layers = L;
  sp.steps = S;
  sp.sel_blocks = sel;
  sp.hot_blocks = hot;
  sp.kv_heads = kv;
  sp.head_dim = d;
  sp.seed = seed;
  return sp;
}
void emit(const ferry::MissTrace& tr, int64_t* blocks, uint8_t* is_miss,
          uint64_t* totals) {
  for (size_t i = 0; i < tr.events.size(); ++i) {
    if (blocks) blocks[i] = (int64_t)tr.events[i].block_id;
    if (is_miss) is_miss[i] = tr.events[i].is_miss ? 1 : 0;
  }
  totals[0] = tr.total_selects;
  totals[1] = tr.total_misses;
  totals[2] = tr.miss_bytes;
}
}  // namespace

extern "C" {

int ref_replay_miss_stream(int R, int L, int S, int sel, int hot, int kv, int d,
                           uint64_t seed, int64_t* blocks, uint8_t* is_miss,
                           uint64_t* totals) {
  const ferry::MissTrace tr =
      ferry::replay_miss_stream(make_spec(R, L, S, sel, hot, kv, d, seed));
  emit(tr, blocks, is_miss, totals);
  return 0;
}

// Exits the process on any header/parameter mismatch, exactly like the
// reference (miss_trace.cuh:64-71); call only with files known to be valid.
int ref_load_miss_trace(const char* path, int R, int L, int S, int sel, int hot,
                        int kv, int d, int64_t* blocks, uint8_t* is_miss,
                        uint64_t* totals, int* slab_blocks) {
  ferry::MissSpec sp = make_spec(R, L, S, sel, hot, kv, d, 42);
  const ferry::MissTrace tr = ferry::load_miss_trace(path, sp, nullptr);
  emit(tr, blocks, is_miss, totals);
  *slab_blocks = sp.slab_blocks;
  return 0;
}

double ref_choose_mb(double pending_mb) {
  ferry::AdaptiveBatchPolicy pol;
  return pol.choose_mb(pending_mb);
}

// Workload B's task stream (arrival: steady | bursty | skewed; sparsity: low |
// medium | high; skew: balanced | imbalanced).
int ref_generate_tasks(const char* arrival, const char* sparsity, const char* skew, uint64_t total,
                       int num_gpus, double hot_frac, int hot_cards, uint64_t seed, double* arrive_t,
                       uint64_t* payload, int32_t* work, int32_t* dest) {
  ferry::ArrivalSpec sp;
  sp.arrival = arrival;
  sp.sparsity = sparsity;
  sp.load_skew = skew;
  sp.total = total;
  sp.num_gpus = num_gpus;
  sp.dest_hot_frac = hot_frac;
  sp.dest_hot_cards = hot_cards;
  const std::vector<ferry::Task> t = ferry::generate_tasks(sp, seed);
  for (size_t i = 0; i < t.size(); ++i) {
    arrive_t[i] = t[i].arrive_t;
    payload[i] = t[i].payload;
    work[i] = t[i].work;
    dest[i] = t[i].dest;
  }
  return 0;
}

}  // extern "C"

#ifdef FERRY_REF_MAIN
// ref_trace_check <path> R L S sel hot kv d : prints "selects misses bytes
// slab_blocks" or exits 1 with the reference's own diagnostic.
int main(int argc, char** argv) {
  if (argc != 9) {
    std::fprintf(stderr, "usage: %s path R L S sel hot kv d\n", argv[0]);
    return 2;
  }
  ferry::MissSpec sp =
      make_spec(std::atoi(argv[2]), std::atoi(argv[3]), std::atoi(argv[4]),
                std::atoi(argv[5]), std::atoi(argv[6]), std::atoi(argv[7]),
                std::atoi(argv[8]), 42);
  const ferry::MissTrace tr = ferry::load_miss_trace(argv[1], sp, nullptr);
  std::printf("%llu %llu %llu %d\n", (unsigned long long)tr.total_selects,
              (unsigned long long)tr.total_misses,
              (unsigned long long)tr.miss_bytes, sp.slab_blocks);
  return 0;
}
#endif
