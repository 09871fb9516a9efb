// ec_api.cu -- the C ABI of libembedcuda.so: context, errors, safetensors
// upload, model load and batched embedding across the library's devices.
#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include <unistd.h>

#include "ec_json.h"
#include "ec_state.h"

namespace ec {

Global& G() {
  static Global g;
  return g;
}

static thread_local std::string t_err;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

// every API entry starts here: forget this thread's message and any stale
// non-sticky CUDA error, so a failure is reported by the call that caused it
void clear_error() {
  t_err.clear();
  cudaGetLastError();
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return EC_OK;
  cudaGetLastError();
  if (e == cudaErrorMemoryAllocation)
    return set_error(EC_ENOMEM, "%s: %s", what, cudaGetErrorString(e));
  return set_error(EC_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

int sync_and_check(Device& d, const char* what) {
  // the status word travels with the stream's last copy: one wait
  int rc = d.status_host ? check_cuda(cudaMemcpyAsync(d.status_host, d.status, 4, cudaMemcpyDeviceToHost,
                                                      d.stream), "status read")
                         : EC_OK;
  if (rc) return rc;
  rc = check_cuda(cudaStreamSynchronize(d.stream), what);
  if (rc) return rc;
  unsigned st = 0;
  if (d.status_host) {
    st = *d.status_host;
  } else {
    rc = check_cuda(cudaMemcpy(&st, d.status, 4, cudaMemcpyDeviceToHost), "status read");
    if (rc) return rc;
  }
  if (st) {
    cudaMemsetAsync(d.status, 0, 4, d.stream);
    cudaStreamSynchronize(d.stream);
    return set_error(EC_ETIMEOUT, "%s: kernel wait timed out (device status %u)", what, st);
  }
  return EC_OK;
}

// Host threads that copy the pieces of one staging chunk in parallel: one
// pool for the process, created on first use and kept (its threads wait on a
// condition variable between jobs), so a multi-GB upload spawns no threads.
class CopyPool {
 public:
  explicit CopyPool(int workers) : n_(workers) {
    for (int i = 0; i < n_; ++i) std::thread([this, i] { loop(i + 1); }).detach();
  }
  // dst[0, len) = src[0, len), split over the workers and the calling thread
  void copy(char* dst, const char* src, size_t len) {
    const size_t per = (len + n_) / (n_ + 1);
    {
      std::lock_guard<std::mutex> lk(mu_);
      dst_ = dst;
      src_ = src;
      len_ = len;
      per_ = per;
      left_ = n_;
      ++gen_;
    }
    cv_.notify_all();
    std::memcpy(dst, src, std::min(len, per));
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [this] { return left_ == 0; });
  }

 private:
  void loop(int part) {
    uint64_t seen = 0;
    for (;;) {
      char* dst;
      const char* src;
      size_t a0, a1;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return gen_ != seen; });
        seen = gen_;
        a0 = std::min(len_, per_ * part);
        a1 = std::min(len_, per_ * (part + 1));
        dst = dst_;
        src = src_;
      }
      if (a1 > a0) std::memcpy(dst + a0, src + a0, a1 - a0);
      std::lock_guard<std::mutex> lk(mu_);
      if (--left_ == 0) done_.notify_one();
    }
  }
  const int n_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  char* dst_ = nullptr;
  const char* src_ = nullptr;
  size_t len_ = 0, per_ = 0;
  int left_ = 0;
  uint64_t gen_ = 0;
};

static CopyPool& copy_pool() {
  // never destroyed: its detached threads outlive static destruction.  A
  // forked child has none of its parent's threads, so it builds its own.
  static CopyPool* pool = nullptr;
  static pid_t owner = 0;
  if (!pool || owner != getpid()) {
    pool = new CopyPool(static_cast<int>(std::min(15u, std::max(1u, std::thread::hardware_concurrency()) - 1u)));
    owner = getpid();
  }
  return *pool;
}

// Host-to-device copy of a large pageable array: 64 MB pieces go through a
// ring of pinned staging buffers, each filled by the copy pool while earlier
// pieces are in flight to the device.  Concurrent calls (one thread per
// device) share the pool, one piece at a time.
int upload_h2d(Device& d, void* dst, const void* src, size_t bytes, const char* what) {
  constexpr size_t kChunk = size_t{64} << 20;
  constexpr int S = Device::kStages;
  if (bytes < 2 * kChunk) {
    int rc = check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, d.stream), what);
    if (rc) return rc;
    return check_cuda(cudaStreamSynchronize(d.stream), what);
  }
  for (int i = 0; i < S; ++i) {
    if (!d.stage[i] && cudaHostAlloc(&d.stage[i], kChunk, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      d.stage[i] = nullptr;
      // no pinned memory to spare: one pageable copy
      int rc = check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, d.stream), what);
      if (rc) return rc;
      return check_cuda(cudaStreamSynchronize(d.stream), what);
    }
    if (!d.stage_ev[i]) {
      int rc = check_cuda(cudaEventCreateWithFlags(&d.stage_ev[i], cudaEventDisableTiming), what);
      if (rc) return rc;
    }
  }
  static std::mutex pool_mu;  // one job at a time in the shared pool
  const char* s = static_cast<const char*>(src);
  char* t = static_cast<char*>(dst);
  bool used[S] = {};
  int b = 0;
  for (size_t off = 0; off < bytes; off += kChunk, b = (b + 1) % S) {
    const size_t len = std::min(kChunk, bytes - off);
    // the DMA that last read this buffer must be done
    if (used[b]) {
      int rc = check_cuda(cudaEventSynchronize(d.stage_ev[b]), what);
      if (rc) return rc;
    }
    char* buf = static_cast<char*>(d.stage[b]);
    {
      std::lock_guard<std::mutex> lk(pool_mu);
      copy_pool().copy(buf, s + off, len);
    }
    int rc = check_cuda(cudaMemcpyAsync(t + off, buf, len, cudaMemcpyHostToDevice, d.stream), what);
    if (!rc) rc = check_cuda(cudaEventRecord(d.stage_ev[b], d.stream), what);
    if (rc) return rc;
    used[b] = true;
  }
  return check_cuda(cudaStreamSynchronize(d.stream), what);
}

static thread_local bool t_pdl = true;
bool pdl_enabled() {
  static const bool on = getenv("EC_NO_PDL") == nullptr;
  return on && t_pdl;
}
void pdl_set_thread(bool on) { t_pdl = on; }

// Freed blocks are cached and handed to the next allocation of the same
// size: repeated builds and searches of one shape then make no cudaMalloc /
// cudaFree calls, whose cost varied from milliseconds to ~1 s for the same
// request (and every cudaFree waits for the whole device).
constexpr size_t kCacheMinBytes = 256;

static void cache_release(Device& d, size_t keep) {
  while (d.free_bytes > keep && !d.free_blocks.empty()) {
    cudaFree(d.free_blocks.front().first);
    d.free_bytes -= d.free_blocks.front().second;
    d.free_blocks.erase(d.free_blocks.begin());
  }
}

int dev_alloc(Device& d, void** p, size_t bytes, const char* what) {
  *p = nullptr;
  if (bytes == 0) bytes = 256;
  const size_t lim = G().max_bytes;
  if (lim && d.allocated + bytes > lim)
    return set_error(EC_ENOMEM, "%s: %zu bytes would exceed EC_MAX_BYTES=%zu (in use %zu)", what,
                     bytes, lim, d.allocated);
  if (bytes >= kCacheMinBytes) {
    for (size_t i = d.free_blocks.size(); i-- > 0;) {
      if (d.free_blocks[i].second != bytes) continue;
      *p = d.free_blocks[i].first;
      d.free_blocks.erase(d.free_blocks.begin() + static_cast<std::ptrdiff_t>(i));
      d.free_bytes -= bytes;
      d.allocated += bytes;
      return EC_OK;
    }
  }
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess && !d.free_blocks.empty()) {
    // the cached blocks go back to the driver and the request is retried
    cudaGetLastError();
    cache_release(d, 0);
    e = cudaMalloc(p, bytes);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    *p = nullptr;
    return set_error(EC_ENOMEM, "%s: cudaMalloc(%zu) failed: %s", what, bytes,
                     cudaGetErrorString(e));
  }
  d.allocated += bytes;
  return EC_OK;
}

void dev_free(Device& d, void* p, size_t bytes) {
  if (!p) return;
  if (bytes == 0) bytes = 256;
  d.allocated = d.allocated >= bytes ? d.allocated - bytes : 0;
  const size_t cap = G().cache_bytes;
  if (bytes >= kCacheMinBytes && bytes <= cap) {
    d.free_blocks.emplace_back(p, bytes);
    d.free_bytes += bytes;
    cache_release(d, cap);  // oldest blocks first
    return;
  }
  cudaFree(p);
}

static void free_uploads(Device& d) {
  for (auto& kv : d.uploads) cudaFree(kv.second.p);
  d.uploads.clear();
}

void free_index(Device& d) {
  for (void* p : d.index.owned) cudaFree(p);
  if (d.index.sws) cudaFree(d.index.sws);
  d.index = IndexW();
}

static void destroy_device(Device* d) {
  cudaSetDevice(d->ordinal);
  cudaStreamSynchronize(d->stream);
  free_model(*d);
  free_index(*d);
  free_uploads(*d);
  if (d->ws) cudaFree(d->ws);
  cache_release(*d, 0);
  if (d->pin) cudaFreeHost(d->pin);
  for (int i = 0; i < Device::kStages; ++i) {
    if (d->stage[i]) cudaFreeHost(d->stage[i]);
    if (d->stage_ev[i]) cudaEventDestroy(d->stage_ev[i]);
  }
  graphs_clear(*d);
  if (d->status) cudaFree(d->status);
  if (d->status_host) cudaFreeHost(d->status_host);
  if (d->res_host) cudaFreeHost(d->res_host);
  if (d->stream) cudaStreamDestroy(d->stream);
  for (cudaEvent_t e : d->evpool) cudaEventDestroy(e);
  delete d;
}

void comm_destroy();  // ec_comm.cu

static int ev_get(Device& d, size_t i) {
  while (d.evpool.size() <= i) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return -1;
    d.evpool.push_back(e);
  }
  return static_cast<int>(i);
}

int prof_begin(Device& d) {
  ++G().launches;
  if (!G().profile) return -1;
  const int i = ev_get(d, d.pend.size() * 2);
  if (i < 0) return -1;
  cudaEventRecord(d.evpool[i], d.stream);
  return i;
}

void prof_end(Device& d, int cls, double flops, double bytes, int e0) {
  if (!G().profile || e0 < 0) return;
  const int e1 = ev_get(d, e0 + 1);
  if (e1 < 0) return;
  cudaEventRecord(d.evpool[e1], d.stream);
  d.pend.push_back(PendingEv{cls, flops, bytes, e0, e1});
}

void trace_launch(Device& d, const char* what) {
  if (!G().sync_each) return;
  const auto t0 = std::chrono::steady_clock::now();
  auto ms = [&] {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  };
  cudaError_t e;
  while ((e = cudaStreamQuery(d.stream)) == cudaErrorNotReady) {
    if (ms() > 60000.0) {
      fprintf(stderr, "[ec] %s: still running after 60 s\n", what);
      return;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
  unsigned st = 0;
  if (e == cudaSuccess) cudaMemcpy(&st, d.status, 4, cudaMemcpyDeviceToHost);
  fprintf(stderr, "[ec] %s: %s, status %u, %.3f ms\n", what, cudaGetErrorString(e), st, ms());
}

void prof_collect(Device& d) {
  for (const PendingEv& p : d.pend) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, d.evpool[p.e0], d.evpool[p.e1]) == cudaSuccess) {
      ProfAcc& a = G().prof[p.cls];
      a.ms += ms;
      a.flops += p.flops;
      a.bytes += p.bytes;
      a.launches += 1;
    }
  }
  d.pend.clear();
}

static size_t env_size(const char* name, size_t def) {
  const char* v = getenv(name);
  if (!v || !*v) return def;
  char* end = nullptr;
  double x = strtod(v, &end);
  if (end && (*end == 'G' || *end == 'g')) x *= 1073741824.0;
  else if (end && (*end == 'M' || *end == 'm')) x *= 1048576.0;
  else if (end && (*end == 'K' || *end == 'k')) x *= 1024.0;
  return x > 0 ? static_cast<size_t>(x) : def;
}

}  // namespace ec

using namespace ec;

extern "C" {

const char* ec_last_error(void) { return t_err.c_str(); }

int ec_init(const int* devices, int ndev) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (G().inited) return set_error(EC_ESTATE, "ec_init called twice (call ec_shutdown first)");
  int count = 0;
  int rc = check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (rc) return rc;
  if (count <= 0) return set_error(EC_ECUDA, "no CUDA device");
  std::vector<int> list;
  if (devices && ndev > 0) {
    list.assign(devices, devices + ndev);
  } else if (const char* env = getenv("EC_DEVICES")) {
    std::string s(env);
    size_t p = 0;
    while (p < s.size()) {
      size_t q = s.find(',', p);
      if (q == std::string::npos) q = s.size();
      if (q > p) list.push_back(atoi(s.substr(p, q - p).c_str()));
      p = q + 1;
    }
  } else {
    for (int i = 0; i < count; ++i) list.push_back(i);
  }
  if (list.empty()) return set_error(EC_EINVAL, "empty device list");
  for (int o : list)
    if (o < 0 || o >= count) return set_error(EC_EINVAL, "device %d not visible (%d devices)", o, count);
  G().max_bytes = env_size("EC_MAX_BYTES", 0);
  {
    // EC_ALLOC_CACHE_MB: freed large blocks kept per device (0: none)
    const char* cm = getenv("EC_ALLOC_CACHE_MB");
    G().cache_bytes = (cm && *cm) ? static_cast<size_t>(strtoull(cm, nullptr, 10)) << 20 : size_t{24} << 30;
  }
  G().max_tokens = static_cast<int>(env_size("EC_MAX_TOKENS_PER_BATCH", 262144));
  G().sync_each = getenv("EC_SYNC_EACH_LAUNCH") != nullptr;
  if (G().max_tokens < 1024) G().max_tokens = 1024;
  if (!gemm_init_driver()) return set_error(EC_ECUDA, "cuTensorMapEncodeTiled unavailable");
  std::vector<Device*> made;
  for (int o : list) {
    Device* d = new Device();
    d->ordinal = o;
    made.push_back(d);
    rc = check_cuda(cudaSetDevice(o), "cudaSetDevice");
    int major = 0, minor = 0;
    if (!rc) rc = check_cuda(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, o), "attr");
    if (!rc) rc = check_cuda(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, o), "attr");
    if (!rc && major != 10)
      rc = set_error(EC_EUNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", o,
                     major, minor);
    if (!rc) rc = check_cuda(cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, o), "attr");
    if (!rc) rc = check_cuda(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "stream");
    if (!rc) rc = dev_alloc(*d, reinterpret_cast<void**>(&d->status), 256, "status word");
    if (!rc) rc = check_cuda(cudaMemset(d->status, 0, 256), "status clear");
    if (!rc && cudaHostAlloc(reinterpret_cast<void**>(&d->status_host), 64, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      d->status_host = nullptr;  // sync_and_check falls back to a plain copy
    }
    // place ec_flat_search_noalloc's static scratch array now, with the
    // library's other device memory, rather than at its first call
    void* scratch = nullptr;
    if (!rc) rc = noalloc_scratch_current(&scratch);
    if (rc) break;
  }
  if (rc) {
    for (Device* d : made) destroy_device(d);
    return rc;
  }
  G().devs = made;
  G().inited = true;
  return EC_OK;
}

int ec_device_count(void) {
  std::lock_guard<std::mutex> lk(G().mu);
  return G().inited ? static_cast<int>(G().devs.size()) : 0;
}

int ec_shutdown(void) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  comm_destroy();
  for (Device* d : G().devs) destroy_device(d);
  G().devs.clear();
  G().inited = false;
  return EC_OK;
}

int ec_upload_tensor(const char* name, int dtype, const int64_t* shape, int ndim, const void* data,
                     size_t nbytes) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!name || !data || ndim < 0 || ndim > 8 || (ndim && !shape))
    return set_error(EC_EINVAL, "bad tensor arguments");
  size_t numel = 1;
  std::vector<int64_t> sh(shape, shape + ndim);
  for (int64_t v : sh) {
    if (v < 0) return set_error(EC_EINVAL, "tensor %s: negative dimension", name);
    if (v && numel > SIZE_MAX / 4 / static_cast<size_t>(v))
      return set_error(EC_EINVAL, "tensor %s: shape too large", name);
    numel *= static_cast<size_t>(v);
  }
  size_t esz;
  switch (dtype) {
    case EC_F32: esz = 4; break;
    case EC_BF16: esz = 2; break;
    case EC_F16: esz = 2; break;
    default: return set_error(EC_EINVAL, "tensor %s has unsupported dtype %d", name, dtype);
  }
  if (numel * esz != nbytes)
    return set_error(EC_EINVAL, "tensor %s: %zu bytes for %zu elements of %zu bytes", name,
                     nbytes, numel, esz);
  for (Device* d : G().devs) {
    int rc = check_cuda(cudaSetDevice(d->ordinal), "cudaSetDevice");
    if (rc) return rc;
    auto it = d->uploads.find(name);
    if (it != d->uploads.end()) {
      dev_free(*d, it->second.p, it->second.numel * (it->second.dtype == kDtBf16 ? 2 : 4));
      d->uploads.erase(it);
    }
    Tensor t;
    t.shape = sh;
    t.numel = numel;
    t.dtype = dtype == EC_BF16 ? kDtBf16 : kDtF32;
    const size_t dev_bytes = numel * (t.dtype == kDtBf16 ? 2 : 4);
    rc = dev_alloc(*d, &t.p, dev_bytes, name);
    if (rc) return rc;
    // Copies are issued on the library's (non-blocking) stream and waited
    // for there: a plain cudaMemcpy from pageable memory may return before
    // its DMA lands, and the legacy stream it runs on does not order work
    // on a non-blocking stream.
    if (dtype == EC_F16) {
      // upload raw binary16, widen on the device (st.lisp:74-85)
      void* raw = nullptr;
      rc = dev_alloc(*d, &raw, nbytes, "f16 staging");
      if (!rc)
        rc = check_cuda(cudaMemcpyAsync(raw, data, nbytes, cudaMemcpyHostToDevice, d->stream), "upload");
      if (!rc) rc = check_cuda(launch_convert(kConvF16ToF32, raw, t.p, numel, d->stream), "f16 widen");
      if (!rc) rc = check_cuda(cudaStreamSynchronize(d->stream), "f16 widen");
      if (raw) dev_free(*d, raw, nbytes);
    } else {
      rc = check_cuda(cudaMemcpyAsync(t.p, data, nbytes, cudaMemcpyHostToDevice, d->stream), "upload");
      if (!rc) rc = check_cuda(cudaStreamSynchronize(d->stream), "upload");
    }
    if (rc) {
      dev_free(*d, t.p, dev_bytes);
      return rc;
    }
    d->uploads[name] = t;
  }
  return EC_OK;
}

int ec_load_model(const char* config_json, const char* pooling_json, int* family, int* dim) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!config_json) return set_error(EC_EINVAL, "config_json is NULL");
  JVal cfg, pool;
  std::string err;
  std::string cs(config_json);
  if (!JParser(cs).parse(cfg, err) || cfg.kind != JVal::Obj)
    return set_error(EC_EINVAL, "config.json: %s", err.empty() ? "not an object" : err.c_str());
  const JVal* pp = nullptr;
  std::string ps;
  if (pooling_json) {
    ps = pooling_json;
    if (!JParser(ps).parse(pool, err))
      return set_error(EC_EINVAL, "1_Pooling/config.json: %s", err.c_str());
    pp = &pool;
  }
  for (Device* d : G().devs) {
    int rc = check_cuda(cudaSetDevice(d->ordinal), "cudaSetDevice");
    if (!rc) rc = load_model_on(*d, cfg, pp);
    if (rc) return rc;
  }
  const ModelW& m = G().devs[0]->model;
  if (family) *family = m.family;
  if (dim) *dim = m.out_dim;
  return EC_OK;
}

int ec_dim(void) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited || !G().devs[0]->model.family) return set_error(EC_ESTATE, "no model loaded");
  return G().devs[0]->model.out_dim;
}

int ec_embed_batch(const int32_t* ids, const int64_t* offsets, int nseq, float* out,
                   int out_stride) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (nseq == 0) return EC_OK;
  if (nseq < 0 || !offsets || !out || (!ids && offsets[nseq] > 0))
    return set_error(EC_EINVAL, "bad batch arguments");
  const ModelW& m = G().devs[0]->model;
  if (!m.family) return set_error(EC_ESTATE, "no model loaded");
  if (out_stride < m.out_dim)
    return set_error(EC_EINVAL, "out_stride %d < dim %d", out_stride, m.out_dim);
  for (int s = 0; s < nseq; ++s)
    if (offsets[s + 1] < offsets[s]) return set_error(EC_EINVAL, "offsets not ascending at %d", s);
  const int nd = static_cast<int>(G().devs.size());
  // length-sorted greedy split over devices (embed.lisp / shard.lisp ranges
  // on one box): cost of a sequence ~ L * (1 + L / 4H)
  std::vector<int> order(nseq);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    return offsets[a + 1] - offsets[a] > offsets[b + 1] - offsets[b];
  });
  std::vector<std::vector<int>> part(nd);
  std::vector<double> load(nd, 0.0);
  for (int s : order) {
    const double L = static_cast<double>(offsets[s + 1] - offsets[s]);
    int best = 0;
    for (int k = 1; k < nd; ++k)
      if (load[k] < load[best]) best = k;
    part[best].push_back(s);
    load[best] += L * (1.0 + L / (4.0 * m.H));
  }
  for (auto& p : part) std::sort(p.begin(), p.end());
  if (nd == 1) return embed_on_device(*G().devs[0], ids, nullptr, part[0], offsets, out, out_stride, nullptr);
  std::vector<int> rcs(nd, EC_OK);
  std::vector<std::string> errs(nd);
  std::vector<std::thread> th;
  for (int k = 0; k < nd; ++k) {
    th.emplace_back([&, k] {
      if (part[k].empty()) return;
      rcs[k] = embed_on_device(*G().devs[k], ids, nullptr, part[k], offsets, out, out_stride, nullptr);
      if (rcs[k]) errs[k] = t_err;
    });
  }
  for (auto& t : th) t.join();
  for (int k = 0; k < nd; ++k)
    if (rcs[k]) return set_error(rcs[k], "device %d: %s", G().devs[k]->ordinal, errs[k].c_str());
  return EC_OK;
}

int ec_embed_batch_device(const int32_t* d_ids, const int64_t* offsets, int nseq, float* d_out,
                          int out_stride, void* stream) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (nseq == 0) return EC_OK;
  if (nseq < 0 || !offsets || !d_out || !d_ids) return set_error(EC_EINVAL, "bad batch arguments");
  const ModelW& m = G().devs[0]->model;
  if (!m.family) return set_error(EC_ESTATE, "no model loaded");
  if (out_stride < m.out_dim)
    return set_error(EC_EINVAL, "out_stride %d < dim %d", out_stride, m.out_dim);
  std::vector<int> all(nseq);
  std::iota(all.begin(), all.end(), 0);
  Device& d = *G().devs[0];
  cudaStream_t own = d.stream;
  if (stream) d.stream = static_cast<cudaStream_t>(stream);
  const int rc = embed_on_device(d, nullptr, d_ids, all, offsets, nullptr, out_stride, d_out);
  d.stream = own;
  return rc;
}

}  // extern "C"
