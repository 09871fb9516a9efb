// ec_comm.cu -- NCCL loaded at run time (dlopen), so the library links no
// NCCL and shares the one already in the process (PyTorch's) when there is
// one.  Used only by k-means, whose centroid update is the path's one real
// exchange step:
//
//  * exact mode (default): the per-cluster accumulators travel down a chain
//    of ranks in sample order (ncclSend / ncclRecv): rank r continues the
//    sums of ranks 0..r-1 with its own rows, so every float add happens in
//    the order of ann.lisp's serial loop; the last rank divides and
//    broadcasts the centroids (ncclBroadcast);
//  * all-reduce mode (EC_KMEANS_ALLREDUCE=1): one ncclAllReduce (f32 sum) of
//    the per-rank sums + counts, faster for many ranks but the cross-rank
//    float sums take a different order from the serial loop.
//
// Two ways to form the ranks: several local devices in one process
// (ncclCommInitAll, one host thread per device) and one process per GPU
// (ec_comm_get_id / ec_comm_init with ncclCommInitRank).  Every wait on a
// collective is a bounded host loop on the stream and ncclCommGetAsyncError.
// A rank that fails (error, timeout, or failure before its collective)
// raises a shared flag so the other local ranks stop waiting at once; the
// caller then aborts every communicator of the clique (comm_abort_all) and
// forgets them before any device memory is freed, so no handle is used or
// destroyed after its abort and no cudaFree waits behind a stuck collective.
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "ec_comm.h"
#include "ec_state.h"

namespace ec {

struct NcclApi {
  void* h = nullptr;
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRank) commInitRank = nullptr;
  decltype(&ncclCommInitAll) commInitAll = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
  decltype(&ncclBroadcast) broadcast = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclCommAbort) commAbort = nullptr;
  decltype(&ncclCommGetAsyncError) getAsyncError = nullptr;
  decltype(&ncclGetErrorString) errStr = nullptr;
};

static NcclApi g_nccl;
static std::vector<ncclComm_t> g_comms;  // one per local device, or one (process mode)
static bool g_process_mode = false;
static bool g_process_dead = false;      // process-mode communicator aborted
static std::atomic<bool> g_failed{false};

static std::atomic<int> g_arrived{0};

// test hooks: EC_FAKE_NCCL_FAIL=1 makes loading fail as if NCCL were absent;
// EC_FAKE_COMM_FAIL=<local index> makes that device's thread fail at the
// rendezvous before the first exchange (the failure-before-the-collective
// path, as after a failed allocation)
static int load_nccl() {
  if (g_nccl.h) return EC_OK;
  if (const char* f = getenv("EC_FAKE_NCCL_FAIL"))
    if (*f && *f != '0') return set_error(EC_ENCCL, "NCCL unavailable (EC_FAKE_NCCL_FAIL)");
  const char* names[] = {getenv("EC_NCCL_LIB"), "libnccl.so.2", "libnccl.so"};
  void* h = nullptr;
  for (const char* n : names) {
    if (!n || !*n) continue;
    h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (h) break;
  }
  if (!h) return set_error(EC_ENCCL, "cannot load NCCL (libnccl.so.2): %s", dlerror());
  NcclApi api;
#define EC_SYM(field, name)                                            \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));  \
  if (!api.field) {                                                    \
    dlclose(h);                                                        \
    return set_error(EC_ENCCL, "NCCL lacks %s", name);                 \
  }
  EC_SYM(getUniqueId, "ncclGetUniqueId");
  EC_SYM(commInitRank, "ncclCommInitRank");
  EC_SYM(commInitAll, "ncclCommInitAll");
  EC_SYM(allReduce, "ncclAllReduce");
  EC_SYM(broadcast, "ncclBroadcast");
  EC_SYM(send, "ncclSend");
  EC_SYM(recv, "ncclRecv");
  EC_SYM(commDestroy, "ncclCommDestroy");
  EC_SYM(commAbort, "ncclCommAbort");
  EC_SYM(getAsyncError, "ncclCommGetAsyncError");
  EC_SYM(errStr, "ncclGetErrorString");
#undef EC_SYM
  api.h = h;
  g_nccl = api;
  return EC_OK;
}

static int nccl_err(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return EC_OK;
  return set_error(EC_ENCCL, "%s: %s", what, g_nccl.errStr ? g_nccl.errStr(r) : "nccl error");
}

void comm_destroy() {
  for (ncclComm_t c : g_comms)
    if (c && g_nccl.commDestroy) g_nccl.commDestroy(c);
  g_comms.clear();
  g_process_mode = false;
  g_process_dead = false;
  g_failed = false;
  G().comm = nullptr;
  G().rank = 0;
  G().world = 1;
}

void comm_abort_all() {
  for (ncclComm_t c : g_comms)
    if (c && g_nccl.commAbort) g_nccl.commAbort(c);
  g_comms.clear();
  if (g_process_mode) g_process_dead = true;
  g_failed = false;
}

bool comm_process_mode() { return g_process_mode; }

void comm_begin() {
  g_failed = false;
  g_arrived = 0;
}

void comm_mark_failed() { g_failed = true; }

int comm_ensure_local() {
  if (g_process_mode) return EC_OK;
  const size_t nd = G().devs.size();
  if (nd <= 1 || g_comms.size() == nd) return EC_OK;
  int rc = load_nccl();
  if (rc) return rc;
  std::vector<int> ords;
  for (Device* d : G().devs) ords.push_back(d->ordinal);
  g_comms.assign(nd, nullptr);
  rc = nccl_err(g_nccl.commInitAll(g_comms.data(), static_cast<int>(nd), ords.data()),
                "ncclCommInitAll");
  if (rc) g_comms.clear();
  return rc;
}

int comm_check_ready() {
  if (!g_process_mode) return EC_OK;
  if (g_process_dead || g_comms.size() != 1)
    return set_error(EC_ESTATE, "the communicator was aborted after a failed collective; "
                                "call ec_comm_init again");
  return EC_OK;
}

static double comm_timeout() {
  const char* v = getenv("EC_COMM_TIMEOUT_S");
  const double t = v ? atof(v) : 120.0;
  return t > 0 ? t : 120.0;
}

// Wait for the collective on `st` with a bounded host loop.  On an
// asynchronous NCCL error, a timeout or another rank's failure it raises the
// shared flag and returns an error; the communicators are aborted by the
// caller once every local rank has returned (comm_abort_all).
static int wait_collective(ncclComm_t c, cudaStream_t st, const char* what) {
  const double timeout_s = comm_timeout();
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return EC_OK;
    if (q != cudaErrorNotReady) {
      g_failed = true;
      return check_cuda(q, what);
    }
    ncclResult_t ae = ncclSuccess;
    g_nccl.getAsyncError(c, &ae);
    if (ae != ncclSuccess && ae != ncclInProgress) {
      g_failed = true;
      return nccl_err(ae, what);
    }
    if (g_failed) return set_error(EC_ENCCL, "%s: another rank failed", what);
    const double el =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      g_failed = true;
      return set_error(EC_ENCCL, "%s timed out after %.0f s", what, el);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

static ncclComm_t comm_of(int local_index) {
  return g_process_mode ? g_comms[0] : g_comms[local_index];
}

int comm_rendezvous(int local_index, int nlocal) {
  const char* v = getenv("EC_FAKE_COMM_FAIL");
  if (v && *v && atoi(v) == local_index) {
    g_failed = true;
    return set_error(EC_ENCCL, "injected failure before the first exchange (EC_FAKE_COMM_FAIL)");
  }
  ++g_arrived;
  const double timeout_s = comm_timeout();
  const auto t0 = std::chrono::steady_clock::now();
  while (g_arrived.load() < nlocal) {
    if (g_failed) return set_error(EC_ENCCL, "another rank failed before the first exchange");
    const double el =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      g_failed = true;
      return set_error(EC_ENCCL, "ranks did not reach the first exchange within %.0f s", el);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  return g_failed ? set_error(EC_ENCCL, "another rank failed before the first exchange") : EC_OK;
}

int comm_allreduce_sum_f32(int local_index, float* buf, size_t count, cudaStream_t st) {
  ncclComm_t c = comm_of(local_index);
  int rc = nccl_err(g_nccl.allReduce(buf, buf, count, ncclFloat32, ncclSum, c, st),
                    "ncclAllReduce");
  if (rc) {
    g_failed = true;
    return rc;
  }
  return wait_collective(c, st, "all-reduce");
}

int comm_send_f32(int local_index, const float* buf, size_t count, int peer, cudaStream_t st) {
  ncclComm_t c = comm_of(local_index);
  int rc = nccl_err(g_nccl.send(buf, count, ncclFloat32, peer, c, st), "ncclSend");
  if (rc) {
    g_failed = true;
    return rc;
  }
  return wait_collective(c, st, "send");
}

int comm_recv_f32(int local_index, float* buf, size_t count, int peer, cudaStream_t st) {
  ncclComm_t c = comm_of(local_index);
  int rc = nccl_err(g_nccl.recv(buf, count, ncclFloat32, peer, c, st), "ncclRecv");
  if (rc) {
    g_failed = true;
    return rc;
  }
  return wait_collective(c, st, "receive");
}

int comm_bcast_f32(int local_index, float* buf, size_t count, int root, cudaStream_t st) {
  ncclComm_t c = comm_of(local_index);
  int rc = nccl_err(g_nccl.broadcast(buf, buf, count, ncclFloat32, root, c, st), "ncclBroadcast");
  if (rc) {
    g_failed = true;
    return rc;
  }
  return wait_collective(c, st, "broadcast");
}

int comm_world() { return g_process_mode ? G().world : static_cast<int>(G().devs.size()); }

int comm_rank(int local_index) { return g_process_mode ? G().rank : local_index; }

}  // namespace ec

using namespace ec;

extern "C" {

int ec_comm_id_size(void) { return static_cast<int>(sizeof(ncclUniqueId)); }

int ec_comm_get_id(void* id_out) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!id_out) return set_error(EC_EINVAL, "id_out is NULL");
  int rc = load_nccl();
  if (rc) return rc;
  ncclUniqueId id;
  rc = nccl_err(g_nccl.getUniqueId(&id), "ncclGetUniqueId");
  if (rc) return rc;
  std::memcpy(id_out, &id, sizeof(id));
  return EC_OK;
}

int ec_comm_init(int rank, int world, const void* id) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (G().devs.size() != 1)
    return set_error(EC_ESTATE, "process mode needs exactly one device per process");
  if (!id || world < 1 || rank < 0 || rank >= world) return set_error(EC_EINVAL, "bad rank/world");
  int rc = load_nccl();
  if (rc) return rc;
  comm_destroy();
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  rc = check_cuda(cudaSetDevice(G().devs[0]->ordinal), "cudaSetDevice");
  if (rc) return rc;
  ncclComm_t c = nullptr;
  rc = nccl_err(g_nccl.commInitRank(&c, world, uid, rank), "ncclCommInitRank");
  if (rc) return rc;
  g_comms.assign(1, c);
  g_process_mode = true;
  G().rank = rank;
  G().world = world;
  return EC_OK;
}

}  // extern "C"
