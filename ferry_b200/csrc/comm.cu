// comm.cu -- the page-ownership exchange between ranks (NCCL all_gather).
//
// The reference keeps the cluster's request ownership in host memory shared
// by its per-GPU exec threads: the fair share reads the global pending count
// under the context mutex (src/runtime/wla_multigpu.cuh:1518-1526), refreshed
// at tick boundaries (:829-864), and the LLX rebalancer reads every GPU's load
// the same way (:2084-2112). With one process per GPU that state is exchanged
// instead: every rank contributes one fixed-size int32 row (finished,
// admitted, owned count, remaining decode steps, owned request ids) and an
// all_gather hands every rank all rows. It is the path's only collective; the
// data path (gathers, steals, migrations) never uses one.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy a PyTorch
// process has already loaded when there is one), so the library loads -- and
// every other entry point works -- where NCCL is absent; these calls then
// return FERRY_E_STATE.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "ferry_cuda.h"

namespace ferry {
namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_gather && api.comm_destroy && api.comm_abort;
  });
  return api;
}

int nccl_missing() {
  set_error("NCCL is not available (libnccl.so.2 could not be loaded)");
  return FERRY_E_STATE;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return FERRY_OK;
  set_error("%s failed: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
  return FERRY_E_CUDA;
}

// Runs f with `device` current and restores the caller's device.
template <class F>
int on_device(int device, F&& f) {
  int prev = 0;
  FERRY_TRY(cudaGetDevice(&prev));
  FERRY_TRY(cudaSetDevice(device));
  const int rc = f();
  cudaSetDevice(prev);
  return rc;
}

}  // namespace
}  // namespace ferry

struct ferry_comm {
  ncclComm_t comm;
  int device, world, rank;
};

extern "C" {

int ferry_comm_unique_id(void* id) {
  if (!id) return ferry::set_error("comm_unique_id: NULL id"), FERRY_E_INVAL;
  const auto& a = ferry::nccl();
  if (!a.ok) return ferry::nccl_missing();
  static_assert(sizeof(ncclUniqueId) == FERRY_COMM_ID_BYTES, "NCCL unique id size");
  ncclUniqueId u;
  const int rc = ferry::nccl_status(a.get_unique_id(&u), "ncclGetUniqueId");
  if (rc) return rc;
  std::memcpy(id, &u, sizeof(u));
  return FERRY_OK;
}

int ferry_comm_create(int device, int world, int rank, const void* id, ferry_comm** out) {
  if (out) *out = nullptr;
  if (!out || !id || world < 1 || rank < 0 || rank >= world)
    return ferry::set_error("comm_create: bad arguments (world %d, rank %d)", world, rank), FERRY_E_INVAL;
  const auto& a = ferry::nccl();
  if (!a.ok) return ferry::nccl_missing();
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  const int rc = ferry::on_device(device, [&] {
    return ferry::nccl_status(a.comm_init_rank(&c, world, u, rank), "ncclCommInitRank");
  });
  if (rc) return rc;
  *out = new ferry_comm{c, device, world, rank};
  return FERRY_OK;
}

int ferry_comm_destroy(ferry_comm* c) {
  if (!c) return FERRY_OK;
  int rc = FERRY_OK;
  const auto& a = ferry::nccl();
  if (a.ok && c->comm)
    rc = ferry::on_device(c->device, [&] { return ferry::nccl_status(a.comm_destroy(c->comm), "ncclCommDestroy"); });
  delete c;
  return rc;
}

int ferry_comm_abort(ferry_comm* c) {
  if (!c) return ferry::set_error("comm_abort: NULL comm"), FERRY_E_INVAL;
  if (!c->comm) return FERRY_OK;
  const auto& a = ferry::nccl();
  if (!a.ok) return ferry::nccl_missing();
  const int rc = ferry::on_device(c->device, [&] { return ferry::nccl_status(a.comm_abort(c->comm), "ncclCommAbort"); });
  c->comm = nullptr;  // destroy only frees the handle now
  return rc;
}

int ferry_exchange_ownership(ferry_comm* c, void* stream, const int32_t* d_row, int row_ints, int32_t* d_all) {
  if (!c || !d_row || !d_all || row_ints < 1)
    return ferry::set_error("exchange_ownership: bad arguments"), FERRY_E_INVAL;
  if (!c->comm) return ferry::set_error("exchange_ownership: communicator was aborted"), FERRY_E_STATE;
  const auto& a = ferry::nccl();
  if (!a.ok) return ferry::nccl_missing();
  return ferry::on_device(c->device, [&] {
    return ferry::nccl_status(a.all_gather(d_row, d_all, (size_t)row_ints, ncclInt32, c->comm,
                                           (cudaStream_t)stream),
                              "ncclAllGather");
  });
}

}  // extern "C"
