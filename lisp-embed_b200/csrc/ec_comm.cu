// ec_comm.cu -- NCCL loaded at run time (dlopen), so the library links no
// NCCL and shares the one already in the process (PyTorch's) when there is
// one.  Used only by k-means: one all-reduce (f32 sum) of the per-device
// centroid sums + counts per Lloyd iteration.
//
// Two modes: several local devices in one process (ncclCommInitAll, one host
// thread per device) and one process per GPU (ec_comm_get_id / ec_comm_init
// with ncclCommInitRank).  Collective failures are detected with a bounded
// host-side wait on ncclCommGetAsyncError and end in ncclCommAbort, never a
// hang.
#include <dlfcn.h>
#include <nccl.h>

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
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclCommAbort) commAbort = nullptr;
  decltype(&ncclCommGetAsyncError) getAsyncError = nullptr;
  decltype(&ncclGroupStart) groupStart = nullptr;
  decltype(&ncclGroupEnd) groupEnd = nullptr;
  decltype(&ncclGetErrorString) errStr = nullptr;
};

static NcclApi g_nccl;
static std::vector<ncclComm_t> g_comms;  // one per local device, or one (process mode)
static bool g_process_mode = false;

// test hook: EC_FAKE_NCCL_FAIL=1 makes loading fail as if NCCL were absent
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
#define EC_SYM(field, name)                                                  \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name));  \
  if (!g_nccl.field) {                                                       \
    dlclose(h);                                                              \
    return set_error(EC_ENCCL, "NCCL lacks %s", name);                       \
  }
  EC_SYM(getUniqueId, "ncclGetUniqueId");
  EC_SYM(commInitRank, "ncclCommInitRank");
  EC_SYM(commInitAll, "ncclCommInitAll");
  EC_SYM(allReduce, "ncclAllReduce");
  EC_SYM(commDestroy, "ncclCommDestroy");
  EC_SYM(commAbort, "ncclCommAbort");
  EC_SYM(getAsyncError, "ncclCommGetAsyncError");
  EC_SYM(groupStart, "ncclGroupStart");
  EC_SYM(groupEnd, "ncclGroupEnd");
  EC_SYM(errStr, "ncclGetErrorString");
#undef EC_SYM
  g_nccl.h = h;
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
  G().comm = nullptr;
  G().rank = 0;
  G().world = 1;
}

bool comm_process_mode() { return g_process_mode; }

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

// Wait for the collective on `st` with a bounded host loop; abort the
// communicator on an asynchronous NCCL error or timeout.
static int wait_collective(ncclComm_t c, cudaStream_t st, double timeout_s) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return EC_OK;
    if (q != cudaErrorNotReady) return check_cuda(q, "all-reduce");
    ncclResult_t ae = ncclSuccess;
    g_nccl.getAsyncError(c, &ae);
    if (ae != ncclSuccess && ae != ncclInProgress) {
      g_nccl.commAbort(c);
      return nccl_err(ae, "all-reduce (communicator aborted)");
    }
    const double el =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      g_nccl.commAbort(c);
      return set_error(EC_ENCCL, "all-reduce timed out after %.0f s (communicator aborted)", el);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

static double comm_timeout() {
  const char* v = getenv("EC_COMM_TIMEOUT_S");
  const double t = v ? atof(v) : 120.0;
  return t > 0 ? t : 120.0;
}

int comm_allreduce_sum_f32(int local_index, float* buf, size_t count, cudaStream_t st) {
  ncclComm_t c = g_process_mode ? g_comms[0] : g_comms[local_index];
  int rc = nccl_err(g_nccl.allReduce(buf, buf, count, ncclFloat32, ncclSum, c, st),
                    "ncclAllReduce");
  if (rc) return rc;
  return wait_collective(c, st, comm_timeout());
}

int comm_world() { return g_process_mode ? G().world : static_cast<int>(G().devs.size()); }

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
