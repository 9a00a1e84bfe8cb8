// executor.cu -- per-GPU decode executor with work stealing (host runtime).
//
// The B200 counterpart of the reference's exec thread + WlaMultiGpuCtx tick /
// steal protocol (src/runtime/wla_multigpu.cuh:829-864 tick_begin/tick_end,
// :1063-1506 steal_from, :1518-1526 fair_share, :2446-2704 exec loop). One
// executor drives one GPU (one process per GPU, or one thread per GPU).
//
// Work unit: a decode task (global request, local slot, step) in this GPU's
// device deque (deque.cu). A tick:
//   1. reclaim request slots whose requests a peer migrated away,
//   2. pop up to max_batch tasks from the bottom of the own deque,
//   3. water-level steal (the reference's rule): when this GPU holds fewer
//      tasks than its fair share ceil(pending / world), take from the peer
//      deque with the largest excess min(steal_batch, size - fair, size/2 + 1)
//      tasks from the top, then pull each stolen request's state over NVLink
//      (ferry_migrate_requests) into a free local slot,
//   4. gather the batch's queries from the resident query table and run the
//      fused decode step (select -> detect -> gather -> attention),
//   5. push (request, slot, step + 1) back, or free the slot when done.
// Everything on the data path runs on the GPU; the host only moves task ids.
#include <chrono>
#include <cstdio>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace ferry {
namespace {

// task = request:24 | slot:16 | step:24
__host__ __device__ inline uint64_t task_pack(uint64_t req, uint64_t slot, uint64_t step) {
  return (req << 40) | (slot << 24) | step;
}
__host__ __device__ inline int task_req(uint64_t t) { return (int)(t >> 40); }
__host__ __device__ inline int task_slot(uint64_t t) { return (int)((t >> 24) & 0xFFFF); }
__host__ __device__ inline int task_step(uint64_t t) { return (int)(t & 0xFFFFFF); }

// q of (request, step) from the resident table into the batch buffer
// (the table holds table_steps rows per request; later steps reuse them cyclically)
__global__ void gather_q_kernel(const uint16_t* __restrict__ table, const uint64_t* __restrict__ tasks,
                                int n, int steps, int table_steps, int64_t row_elems, int total_requests,
                                uint16_t* __restrict__ out, uint32_t* err) {
  const int i = blockIdx.y;
  if (i >= n) return;
  const uint64_t t = tasks[i];
  const int r = task_req(t), s = task_step(t);
  if (r >= total_requests || s >= steps) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(err, kErrRange);
    return;
  }
  const uint4* src =
      reinterpret_cast<const uint4*>(table + ((int64_t)r * table_steps + s % table_steps) * row_elems);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)i * row_elems);
  const int64_t n4 = row_elems / 8;
  for (int64_t j = blockIdx.x * blockDim.x + threadIdx.x; j < n4; j += (int64_t)gridDim.x * blockDim.x)
    dst[j] = src[j];
}

}  // namespace
}  // namespace ferry

struct ferry_exec {
  ferry_ctx* ctx = nullptr;
  ferry_deque* own = nullptr;
  ferry_exec_cfg cfg{};
  const uint16_t* q_table = nullptr;
  int64_t row_elems = 0;  // L * Hq * 128
  // peers
  std::vector<ferry_deque*> peer_deque;  // by rank (nullptr = none)
  std::vector<int> peer_slot;            // ctx peer slot by rank
  // slots
  std::vector<int> free_slots;
  std::vector<int> slot_req;  // global request in each slot (-1 free)
  std::vector<int> slot_step; // next decode step of the request in each slot
  int force_victim = -1, force_take = 0;  // a rebalance order for the next tick
  std::vector<std::pair<int, int>> pending_admit;  // (global request, n_pages)
  int64_t global_pending = 0;
  int64_t finished = 0;
  // device buffers
  uint64_t* d_tasks = nullptr;   // max_batch (popped + stolen)
  uint64_t* d_push = nullptr;    // max_batch
  uint64_t* d_admit = nullptr;   // R
  int32_t* d_cnt = nullptr;      // 4
  int64_t* d_sizes = nullptr;    // world
  int32_t* d_ids = nullptr;      // max_batch local slots
  int32_t* d_mig = nullptr;      // 2 * steal_batch (src, dst)
  int32_t* d_begin = nullptr;    // 2 * R (slots, n_pages)
  int64_t* d_base = nullptr;     // R
  uint16_t* d_q = nullptr;       // max_batch * row_elems
  float* d_out = nullptr;        // max_batch * row_elems
  // pinned host mirrors
  uint64_t* h_tasks = nullptr;
  uint64_t* h_push = nullptr;
  uint64_t* h_admit = nullptr;
  int32_t* h_cnt = nullptr;
  int64_t* h_sizes = nullptr;
  int32_t* h_ids = nullptr;
  int32_t* h_mig = nullptr;
  int32_t* h_begin = nullptr;
  int64_t* h_base = nullptr;
  std::vector<int32_t> slot_state;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev2 = nullptr, ev3 = nullptr;
  uint64_t mig_bytes_seen = 0;
  // steal policy (ferry_exec_policy)
  ferry_steal_policy pol{0, 2.0, 3.0, 700.0, 0.06};
  int64_t pending_fair = 0, pending_occ = 0, pending_vsize = 0;
  int pending_victim = -1, pending_forced = 0, pending_planned = 0;
  double step_ms_ema = 2.0;
  int last_n = 0;  // tasks decoded in the last tick (their outputs are in d_out)
  // decision log (ferry_exec_log): one record per steal, written at the tick's end
  FILE* log = nullptr;
  int64_t ticks = 0;
  std::vector<uint8_t> rec;        // the pending record of this tick
  std::vector<int32_t> h_res;      // resident units of the stolen requests' lanes
  int32_t* h_live = nullptr;  // steal_batch * lanes_per_req resident-page counts of candidates
};

using namespace ferry;

namespace {

struct Guard {
  int prev = -1;
  explicit Guard(int d) {
    cudaGetDevice(&prev);
    cudaSetDevice(d);
  }
  ~Guard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

void free_exec(ferry_exec* x) {
  cudaFree(x->d_tasks); cudaFree(x->d_push); cudaFree(x->d_admit); cudaFree(x->d_cnt);
  cudaFree(x->d_sizes); cudaFree(x->d_ids); cudaFree(x->d_mig); cudaFree(x->d_begin);
  cudaFree(x->d_base); cudaFree(x->d_q); cudaFree(x->d_out);
  cudaFreeHost(x->h_tasks); cudaFreeHost(x->h_push); cudaFreeHost(x->h_admit);
  cudaFreeHost(x->h_cnt); cudaFreeHost(x->h_sizes); cudaFreeHost(x->h_ids); cudaFreeHost(x->h_mig);
  cudaFreeHost(x->h_begin); cudaFreeHost(x->h_base); cudaFreeHost(x->h_live);
  for (cudaEvent_t e : {x->ev0, x->ev1, x->ev2, x->ev3})
    if (e) cudaEventDestroy(e);
  if (x->log) std::fclose(x->log);
  delete x;
}

int alloc_slot(ferry_exec* x, int g) {
  if (x->free_slots.empty()) return -1;
  const int s = x->free_slots.back();
  x->free_slots.pop_back();
  x->slot_req[s] = g;
  return s;
}

void release_slot(ferry_exec* x, int s) {
  x->slot_req[s] = -1;
  x->free_slots.push_back(s);
}

// admit as many pending requests as there are free slots: begin + push step 0
int admit_pending(ferry_exec* x, cudaStream_t st) {
  int n = 0;
  const int64_t LH = x->ctx->lanes_per_req, N = x->ctx->cfg.max_pages;
  while (!x->pending_admit.empty() && !x->free_slots.empty()) {
    const auto gp = x->pending_admit.front();
    x->pending_admit.erase(x->pending_admit.begin());
    const int s = alloc_slot(x, gp.first);
    x->slot_step[s] = 0;
    x->h_begin[n] = s;
    x->h_begin[x->ctx->cfg.num_requests + n] = gp.second;
    x->h_base[n] = (int64_t)gp.first * LH * N;  // the request's home in the (replicated) host pool
    x->h_admit[n] = task_pack((uint64_t)gp.first, (uint64_t)s, 0);
    ++n;
  }
  if (!n) return FERRY_OK;
  const size_t R = x->ctx->cfg.num_requests;
  FERRY_TRY(cudaMemcpyAsync(x->d_begin, x->h_begin, R * 2 * 4, cudaMemcpyHostToDevice, st));
  FERRY_TRY(cudaMemcpyAsync(x->d_base, x->h_base, (size_t)n * 8, cudaMemcpyHostToDevice, st));
  FERRY_TRY(cudaMemcpyAsync(x->d_admit, x->h_admit, (size_t)n * 8, cudaMemcpyHostToDevice, st));
  int rc = ferry_requests_begin(x->ctx, st, x->d_begin, x->d_begin + R, x->d_base, n);
  if (rc) return rc;
  return ferry_deque_push(x->own, st, x->d_admit, n, x->d_cnt + 3);
}

}  // namespace

// ---- decision log (ferry_exec_log): the B200 counterpart of the reference's
// FERRY_WLA_SNAPSHOT decision records (src/runtime/wla_multigpu.cuh:667-788)
// read by its offline counterfactual tool (src/tools/wla_counterfact.cpp).
// Little-endian binary: a 64-byte header
//   "FRYD" u32 version=1 | i32 rank, world, R, L, Hkv, N, C, k, unit_bytes,
//   steps_per_req, migrate_mode, steal_batch, max_batch, cost_filter
// then one record per steal:
//   i64 tick | i32 victim, forced | i64 fair, own_occupancy, victim_size |
//   i32 planned, got | f64 step_ms_ema | f32 mig_ms, pad | i64 mig_bytes |
//   got x { i32 request, step, victim_slot, thief_slot | i64 resident_units }
namespace {
template <class T>
void put(std::vector<uint8_t>& b, T v) {
  const size_t o = b.size();
  b.resize(o + sizeof(T));
  std::memcpy(b.data() + o, &v, sizeof(T));
}

void write_decision(ferry_exec* x, const ferry_tick_stats& ts, int n) {
  auto& b = x->rec;
  b.clear();
  const int got = ts.stolen, S = x->cfg.steal_batch, LH = x->ctx->lanes_per_req;
  put<int64_t>(b, x->ticks);
  put<int32_t>(b, x->pending_victim);
  put<int32_t>(b, x->pending_forced);
  put<int64_t>(b, x->pending_fair);
  put<int64_t>(b, x->pending_occ);
  put<int64_t>(b, x->pending_vsize);
  put<int32_t>(b, x->pending_planned);
  put<int32_t>(b, got);
  put<double>(b, x->step_ms_ema);
  put<float>(b, ts.mig_ms);
  put<float>(b, 0.f);
  put<int64_t>(b, ts.mig_bytes);
  // the stolen tasks are the last `got` of the tick's batch (h_tasks, repacked with the thief slot)
  for (int i = 0; i < got; ++i) {
    const uint64_t t = x->h_tasks[n - got + i];
    int64_t units = 0;
    for (int l = 0; l < LH; ++l) units += std::max(0, x->h_res[(size_t)i * LH + l]);
    put<int32_t>(b, task_req(t));
    put<int32_t>(b, task_step(t));
    put<int32_t>(b, x->h_mig[i]);
    put<int32_t>(b, x->h_mig[S + i]);
    put<int64_t>(b, units);
  }
  std::fwrite(b.data(), 1, b.size(), x->log);
}
}  // namespace

extern "C" {

int ferry_exec_create(ferry_ctx* ctx, ferry_deque* own, const ferry_exec_cfg* cfg,
                      const uint16_t* d_q_table, ferry_exec** out) {
  if (!ctx || !own || !cfg || !d_q_table || !out) return set_error("exec_create: bad arguments"), FERRY_E_INVAL;
  *out = nullptr;
  const int R = ctx->cfg.num_requests;
  if (cfg->world < 1 || cfg->rank < 0 || cfg->rank >= cfg->world || cfg->max_batch < 1 ||
      cfg->max_batch > R || cfg->steal_batch < 0 || cfg->steps_per_req < 1 ||
      cfg->total_requests < 1 || cfg->total_requests >= (1 << 24) || R > 65535 ||
      cfg->steps_per_req >= (1 << 24) || cfg->q_table_steps < 0 ||
      (cfg->migrate_mode != FERRY_MIGRATE_DELTA && cfg->migrate_mode != FERRY_MIGRATE_FULL &&
       cfg->migrate_mode != FERRY_MIGRATE_DROP))
    return set_error("exec_create: bad configuration"), FERRY_E_INVAL;
  Guard g(ctx->device);
  auto* x = new ferry_exec;
  x->ctx = ctx;
  x->own = own;
  x->cfg = *cfg;
  x->q_table = d_q_table;
  x->row_elems = (int64_t)ctx->cfg.num_layers * ctx->cfg.q_heads * kHeadDim;
  x->peer_deque.assign(cfg->world, nullptr);
  x->peer_slot.assign(cfg->world, -1);
  x->slot_req.assign(R, -1);
  x->slot_step.assign(R, 0);
  x->slot_state.assign(R, 0);
  for (int s = R - 1; s >= 0; --s) x->free_slots.push_back(s);
  const size_t B = cfg->max_batch, W = cfg->world, S = std::max(1, cfg->steal_batch);
#define FX(call)                      \
  do {                                \
    cudaError_t e__ = (call);         \
    if (e__ != cudaSuccess) {         \
      int rc__ = cuda_status(e__, #call); \
      free_exec(x);                   \
      return rc__;                    \
    }                                 \
  } while (0)
  FX(cudaMalloc(&x->d_tasks, B * 8));
  FX(cudaMalloc(&x->d_push, B * 8));
  FX(cudaMalloc(&x->d_admit, (size_t)R * 8));
  FX(cudaMalloc(&x->d_cnt, 16));
  FX(cudaMalloc(&x->d_sizes, W * 8));
  FX(cudaMalloc(&x->d_ids, B * 4));
  FX(cudaMalloc(&x->d_mig, 2 * S * 4));
  FX(cudaMalloc(&x->d_begin, (size_t)R * 2 * 4));
  FX(cudaMalloc(&x->d_base, (size_t)R * 8));
  FX(cudaMalloc(&x->d_q, B * x->row_elems * 2));
  FX(cudaMalloc(&x->d_out, B * x->row_elems * 4));
  FX(cudaMallocHost(&x->h_tasks, B * 8));
  FX(cudaMallocHost(&x->h_push, B * 8));
  FX(cudaMallocHost(&x->h_admit, (size_t)R * 8));
  FX(cudaMallocHost(&x->h_cnt, 16));
  FX(cudaMallocHost(&x->h_sizes, W * 8));
  FX(cudaMallocHost(&x->h_ids, B * 4));
  FX(cudaMallocHost(&x->h_mig, 2 * S * 4));
  FX(cudaMallocHost(&x->h_begin, (size_t)R * 2 * 4));
  FX(cudaMallocHost(&x->h_base, (size_t)R * 8));
  FX(cudaMallocHost(&x->h_live, (size_t)S * ctx->lanes_per_req * 4));
  FX(cudaEventCreate(&x->ev0));
  FX(cudaEventCreate(&x->ev1));
  FX(cudaEventCreate(&x->ev2));
  FX(cudaEventCreate(&x->ev3));
#undef FX
  *out = x;
  return FERRY_OK;
}

int ferry_exec_destroy(ferry_exec* x) {
  if (!x) return FERRY_OK;
  Guard g(x->ctx->device);
  cudaDeviceSynchronize();
  free_exec(x);
  return FERRY_OK;
}

int ferry_exec_link_peer(ferry_exec* x, int peer_rank, int ctx_peer_slot, ferry_deque* peer_deque) {
  if (!x || peer_rank < 0 || peer_rank >= x->cfg.world || peer_rank == x->cfg.rank ||
      ctx_peer_slot < 0 || ctx_peer_slot >= FERRY_MAX_PEERS || !peer_deque)
    return set_error("exec_link_peer: bad arguments"), FERRY_E_INVAL;
  if (!x->ctx->peers[ctx_peer_slot].cache) return set_error("exec_link_peer: ctx peer slot not linked"), FERRY_E_STATE;
  x->peer_deque[peer_rank] = peer_deque;
  x->peer_slot[peer_rank] = ctx_peer_slot;
  return FERRY_OK;
}

int ferry_exec_admit(ferry_exec* x, const int32_t* h_global_req, const int32_t* h_n_pages, int n) {
  if (!x || n < 0 || (n && (!h_global_req || !h_n_pages))) return set_error("exec_admit: bad arguments"), FERRY_E_INVAL;
  for (int i = 0; i < n; ++i) {
    if (h_global_req[i] < 0 || h_global_req[i] >= x->cfg.total_requests)
      return set_error("exec_admit: request %d out of range", h_global_req[i]), FERRY_E_INVAL;
    x->pending_admit.emplace_back(h_global_req[i], h_n_pages[i]);
  }
  return FERRY_OK;
}

int ferry_exec_set_global(ferry_exec* x, int64_t global_pending) {
  if (!x || global_pending < 0) return set_error("exec_set_global: bad arguments"), FERRY_E_INVAL;
  x->global_pending = global_pending;
  return FERRY_OK;
}

int ferry_exec_owned(ferry_exec* x, int32_t* h_out, int cap, int* n_out) {
  if (!x || !n_out || cap < 0 || (cap && !h_out)) return set_error("exec_owned: bad arguments"), FERRY_E_INVAL;
  int n = 0;
  for (int s = 0; s < (int)x->slot_req.size(); ++s)
    if (x->slot_req[s] >= 0) {
      if (n < cap) h_out[n] = x->slot_req[s];
      ++n;
    }
  *n_out = n;
  return FERRY_OK;
}

int ferry_exec_tick(ferry_exec* x, void* stream, ferry_tick_stats* out) {
  if (!x || !out) return set_error("exec_tick: bad arguments"), FERRY_E_INVAL;
  Guard g(x->ctx->device);
  cudaStream_t st = (cudaStream_t)stream;
  ferry_tick_stats ts{};
  int rc;
  // 1. reclaim slots whose requests a peer migrated away
  if (x->cfg.world > 1) {
    if ((rc = ferry_slot_states(x->ctx, x->slot_state.data(), 1))) return rc;
    for (int s = 0; s < (int)x->slot_state.size(); ++s)
      if (x->slot_state[s] == 2 && x->slot_req[s] >= 0) release_slot(x, s);
  }
  if ((rc = admit_pending(x, st))) return rc;
  FERRY_TRY(cudaEventRecord(x->ev0, st));
  // 2. pop own tasks
  const int B = x->cfg.max_batch;
  if ((rc = ferry_deque_pop(x->own, st, x->d_tasks, B, x->d_cnt))) return rc;
  if ((rc = ferry_deque_size(x->own, st, x->d_sizes + x->cfg.rank))) return rc;
  FERRY_TRY(cudaMemcpyAsync(x->h_cnt, x->d_cnt, 16, cudaMemcpyDeviceToHost, st));
  FERRY_TRY(cudaMemcpyAsync(x->h_tasks, x->d_tasks, (size_t)B * 8, cudaMemcpyDeviceToHost, st));
  FERRY_TRY(cudaStreamSynchronize(st));
  int n = x->h_cnt[0];
  // 3. steal: a rebalance order (ferry_exec_rebalance), else the water-level rule
  const bool forced = x->force_take > 0;
  if (x->cfg.world > 1 && x->cfg.steal_batch > 0 && n < B && !x->free_slots.empty()) {
    const int64_t fair = (x->global_pending + x->cfg.world - 1) / x->cfg.world;
    FERRY_TRY(cudaMemcpyAsync(x->h_sizes + x->cfg.rank, x->d_sizes + x->cfg.rank, 8,
                              cudaMemcpyDeviceToHost, st));
    for (int r = 0; r < x->cfg.world; ++r)
      if (x->peer_deque[r])
        if ((rc = ferry_deque_size(x->peer_deque[r], st, x->d_sizes + r))) return rc;
    FERRY_TRY(cudaMemcpyAsync(x->h_sizes, x->d_sizes, (size_t)x->cfg.world * 8, cudaMemcpyDeviceToHost, st));
    FERRY_TRY(cudaStreamSynchronize(st));
    const int64_t occ = n + x->h_sizes[x->cfg.rank];
    if (forced || occ < fair) {
      int victim = -1;
      int64_t best = 0;
      if (forced) {
        if (x->force_victim >= 0 && x->force_victim < x->cfg.world && x->peer_deque[x->force_victim])
          victim = x->force_victim;
      } else {
        for (int r = 0; r < x->cfg.world; ++r) {
          if (!x->peer_deque[r]) continue;
          const int64_t ex = x->h_sizes[r] - fair;
          if (ex > best) {
            best = ex;
            victim = r;
          }
        }
      }
      if (victim >= 0) {
        const int64_t cur = x->h_sizes[victim];
        int64_t take = forced ? std::min<int64_t>(std::min<int64_t>(x->force_take, x->cfg.steal_batch), cur)
                              : std::min<int64_t>(x->cfg.steal_batch, std::min<int64_t>(cur - fair, cur / 2 + 1));
        take = std::min<int64_t>(take, B - n);
        take = std::min<int64_t>(take, (int64_t)x->free_slots.size());
        x->pending_fair = fair;
        x->pending_occ = occ;
        x->pending_vsize = cur;
        x->pending_victim = victim;
        x->pending_forced = forced ? 1 : 0;
        x->pending_planned = (int)take;
        const ferry_peer& vp = x->ctx->peers[x->peer_slot[victim]];
        if (take > 0 && !forced && x->pol.cost_filter && vp.size) {
          // price the tasks the steal would take: remaining steps x step time
          // against moving their resident pages (policy E)
          if ((rc = ferry_deque_peek(x->peer_deque[victim], st, x->d_tasks + n, (int)take, x->d_cnt + 3))) return rc;
          FERRY_TRY(cudaMemcpyAsync(x->h_cnt, x->d_cnt, 16, cudaMemcpyDeviceToHost, st));
          FERRY_TRY(cudaMemcpyAsync(x->h_tasks + n, x->d_tasks + n, (size_t)take * 8, cudaMemcpyDeviceToHost, st));
          FERRY_TRY(cudaStreamSynchronize(st));
          const int seen = std::min<int>(x->h_cnt[3], (int)take);
          const int LH = x->ctx->lanes_per_req;
          for (int i = 0; i < seen; ++i) {
            const int vs = task_slot(x->h_tasks[n + i]);
            if (vs < 0 || vs >= x->ctx->cfg.num_requests) return set_error("exec: peeked task slot out of range"), FERRY_E_RANGE;
            FERRY_TRY(cudaMemcpyAsync(x->h_live + (size_t)i * LH, vp.size + (size_t)vs * LH, (size_t)LH * 4,
                                      cudaMemcpyDeviceToHost, st));
          }
          FERRY_TRY(cudaStreamSynchronize(st));
          int32_t remain[64];
          int64_t live[64];
          const int m = std::min(seen, 64);
          for (int i = 0; i < m; ++i) {
            remain[i] = x->cfg.steps_per_req - (int)task_step(x->h_tasks[n + i]);
            int64_t units = 0;
            for (int l = 0; l < LH; ++l) units += std::max(0, x->h_live[(size_t)i * LH + l]);
            live[i] = units * x->ctx->unit_bytes;
          }
          int acc = 0;
          if ((rc = ferry_steal_filter(&x->pol, m, remain, live, x->step_ms_ema, nullptr, nullptr, &acc))) return rc;
          take = std::min<int64_t>(take, acc);
        }
        if (take > 0) {
          if ((rc = ferry_deque_steal(x->peer_deque[victim], st, x->d_tasks + n, (int)take, x->d_cnt + 1))) return rc;
          FERRY_TRY(cudaMemcpyAsync(x->h_cnt, x->d_cnt, 16, cudaMemcpyDeviceToHost, st));
          FERRY_TRY(cudaMemcpyAsync(x->h_tasks + n, x->d_tasks + n, (size_t)take * 8, cudaMemcpyDeviceToHost, st));
          FERRY_TRY(cudaStreamSynchronize(st));
          const int got = x->h_cnt[1];
          const int S = x->cfg.steal_batch;
          for (int i = 0; i < got; ++i) {
            const uint64_t t = x->h_tasks[n + i];
            const int s = alloc_slot(x, task_req(t));
            x->slot_step[s] = (int)task_step(t);
            x->h_mig[i] = task_slot(t);
            x->h_mig[S + i] = s;
            x->h_tasks[n + i] = task_pack((uint64_t)task_req(t), (uint64_t)s, (uint64_t)task_step(t));
          }
          if (got && x->log) {  // resident pages of the stolen requests' lanes, before they move
            const int LH = x->ctx->lanes_per_req;
            for (int i = 0; i < got; ++i)
              FERRY_TRY(cudaMemcpyAsync(x->h_res.data() + (size_t)i * LH, vp.size + (size_t)x->h_mig[i] * LH,
                                        (size_t)LH * 4, cudaMemcpyDeviceToHost, st));
          }
          if (got) {
            FERRY_TRY(cudaMemcpyAsync(x->d_mig, x->h_mig, (size_t)2 * S * 4, cudaMemcpyHostToDevice, st));
            FERRY_TRY(cudaEventRecord(x->ev2, st));
            if ((rc = ferry_migrate_requests(x->ctx, st, x->peer_slot[victim], x->d_mig, x->d_mig + S, got,
                                             x->cfg.migrate_mode)))
              return rc;
            FERRY_TRY(cudaEventRecord(x->ev3, st));
            ts.mig_ms = -1.f;  // filled in after the tick's sync
            FERRY_TRY(cudaMemcpyAsync(x->d_tasks + n, x->h_tasks + n, (size_t)got * 8, cudaMemcpyHostToDevice, st));
            ts.stolen = got;
            ts.stolen_from = victim;
            n += got;
          }
        }
      }
    }
  }
  x->force_take = 0;  // an order lasts one tick
  // 4. decode the batch
  if (n > 0) {
    for (int i = 0; i < n; ++i) x->h_ids[i] = task_slot(x->h_tasks[i]);
    FERRY_TRY(cudaMemcpyAsync(x->d_ids, x->h_ids, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    dim3 grid((unsigned)std::min<int64_t>(64, (x->row_elems / 8 + 255) / 256), (unsigned)n);
    gather_q_kernel<<<grid, 256, 0, st>>>(x->q_table, x->d_tasks, n, x->cfg.steps_per_req,
                                          x->cfg.q_table_steps > 0 ? x->cfg.q_table_steps : x->cfg.steps_per_req,
                                          x->row_elems,
                                          x->cfg.total_requests, x->d_q, x->ctx->err);
    FERRY_TRY(cudaGetLastError());
    if ((rc = ferry_decode_step(x->ctx, st, x->d_q, x->d_ids, n, x->d_out))) return rc;
  }
  // 5. push the next steps back
  int np = 0;
  for (int i = 0; i < n; ++i) {
    const uint64_t t = x->h_tasks[i];
    if (task_step(t) + 1 < x->cfg.steps_per_req) {
      x->h_push[np++] = task_pack((uint64_t)task_req(t), (uint64_t)task_slot(t), (uint64_t)task_step(t) + 1);
      x->slot_step[task_slot(t)] = (int)task_step(t) + 1;
    } else {
      release_slot(x, task_slot(t));
      ++ts.finished;
    }
  }
  if (np) {
    FERRY_TRY(cudaMemcpyAsync(x->d_push, x->h_push, (size_t)np * 8, cudaMemcpyHostToDevice, st));
    if ((rc = ferry_deque_push(x->own, st, x->d_push, np, x->d_cnt + 2))) return rc;
  }
  FERRY_TRY(cudaEventRecord(x->ev1, st));
  FERRY_TRY(cudaStreamSynchronize(st));
  float ms = 0.f;
  FERRY_TRY(cudaEventElapsedTime(&ms, x->ev0, x->ev1));
  if (ts.mig_ms < 0.f) {
    FERRY_TRY(cudaEventElapsedTime(&ts.mig_ms, x->ev2, x->ev3));
    uint64_t st4[FERRY_NUM_STATS];
    if ((rc = ferry_stats_read(x->ctx, st4, 0))) return rc;
    // the counter may have been zeroed by ferry_stats_read(reset) since the last steal
    ts.mig_bytes = (int64_t)(st4[3] >= x->mig_bytes_seen ? st4[3] - x->mig_bytes_seen : st4[3]);
    x->mig_bytes_seen = st4[3];
  }
  x->finished += ts.finished;
  if (x->log && ts.stolen > 0) write_decision(x, ts, n);
  ++x->ticks;
  if (n > 0) x->step_ms_ema = 0.9 * x->step_ms_ema + 0.1 * ms;  // one step of every decoded request
  ts.decoded = n;
  x->last_n = n;
  ts.tick_ms = ms;
  ts.queued = np;
  *out = ts;
  return FERRY_OK;
}

int ferry_exec_log(ferry_exec* x, const char* path) {
  if (!x) return set_error("exec_log: NULL executor"), FERRY_E_INVAL;
  if (x->log) {
    std::fclose(x->log);
    x->log = nullptr;
  }
  if (!path) return FERRY_OK;
  FILE* f = std::fopen(path, "wb");
  if (!f) return set_error("exec_log: cannot open %s", path), FERRY_E_INVAL;
  const ferry_cfg& c = x->ctx->cfg;
  std::vector<uint8_t> h;
  const char magic[4] = {'F', 'R', 'Y', 'D'};
  h.insert(h.end(), magic, magic + 4);
  put<uint32_t>(h, 1u);
  for (int v : {x->cfg.rank, x->cfg.world, c.num_requests, c.num_layers, c.kv_heads, c.max_pages, c.cache_pages,
                c.top_k, x->ctx->unit_bytes, x->cfg.steps_per_req, x->cfg.migrate_mode, x->cfg.steal_batch,
                x->cfg.max_batch, x->pol.cost_filter})
    put<int32_t>(h, v);
  std::fwrite(h.data(), 1, h.size(), f);
  x->log = f;
  x->h_res.assign((size_t)std::max(1, x->cfg.steal_batch) * x->ctx->lanes_per_req, 0);
  return FERRY_OK;
}

int ferry_exec_output(ferry_exec* x, void* stream, float* host_out, int32_t* host_req, int cap_rows,
                      int* n_out) {
  if (!x || !n_out || cap_rows < 0 || (cap_rows && !host_out))
    return set_error("exec_output: bad arguments"), FERRY_E_INVAL;
  const int n = std::min(x->last_n, cap_rows);
  Guard g(x->ctx->device);
  if (n > 0)
    FERRY_TRY(cudaMemcpyAsync(host_out, x->d_out, (size_t)n * x->row_elems * 4, cudaMemcpyDeviceToHost,
                              (cudaStream_t)stream));
  if (host_req)
    for (int i = 0; i < n; ++i) host_req[i] = task_req(x->h_tasks[i]);
  *n_out = n;
  return FERRY_OK;
}

int ferry_steal_filter(const ferry_steal_policy* pol, int n, const int32_t* remain_steps,
                       const int64_t* live_bytes, double step_ms, double* value_ms, double* cost_ms,
                       int* n_accept) {
  if (!pol || !n_accept || n < 0 || (n && (!remain_steps || !live_bytes)) || !(pol->link_gbs > 0.0))
    return set_error("steal_filter: bad arguments"), FERRY_E_INVAL;
  const double ms_per_byte = 1e3 / (pol->link_gbs * 1e9);
  int ok = 0;
  bool open = true;
  for (int i = 0; i < n; ++i) {
    const double v = (double)remain_steps[i] * step_ms;
    const double c = pol->cost_scale * (double)live_bytes[i] * ms_per_byte + pol->fixed_ms;
    if (value_ms) value_ms[i] = v;
    if (cost_ms) cost_ms[i] = c;
    if (open && (!pol->cost_filter || v >= pol->margin * c))
      ++ok;
    else
      open = false;  // the accepted candidates are a prefix
  }
  *n_accept = ok;
  return FERRY_OK;
}

int ferry_exec_usage(ferry_exec* x, int64_t* remaining_steps, int32_t* requests) {
  if (!x || !remaining_steps || !requests) return set_error("exec_usage: bad arguments"), FERRY_E_INVAL;
  int64_t u = 0;
  int32_t n = 0;
  for (size_t s = 0; s < x->slot_req.size(); ++s)
    if (x->slot_req[s] >= 0) {
      u += std::max(0, x->cfg.steps_per_req - x->slot_step[s]);
      ++n;
    }
  *remaining_steps = u;
  *requests = n;
  return FERRY_OK;
}

int ferry_exec_rebalance(ferry_exec* x, int victim_rank, int k) {
  if (!x || victim_rank < 0 || victim_rank >= x->cfg.world || victim_rank == x->cfg.rank || k < 0)
    return set_error("exec_rebalance: bad arguments"), FERRY_E_INVAL;
  x->force_victim = victim_rank;
  x->force_take = k;
  return FERRY_OK;
}

int ferry_exec_policy(ferry_exec* x, const ferry_steal_policy* pol) {
  if (!x || !pol || !(pol->link_gbs > 0.0) || pol->margin < 0.0 || pol->cost_scale < 0.0 || pol->fixed_ms < 0.0)
    return set_error("exec_policy: bad arguments"), FERRY_E_INVAL;
  x->pol = *pol;
  return FERRY_OK;
}

}  // extern "C"
