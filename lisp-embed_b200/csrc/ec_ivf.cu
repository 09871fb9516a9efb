// ec_ivf.cu -- C ABI of the IVF path: k-means (ann::kmeans), assignment
// (ann::assign-all), resident index, IVF and flat search (kb::top-k-ivf,
// kb::top-k-brute).  Rows are sharded over the library's devices (or over
// processes after ec_comm_init); only k-means exchanges data, with one NCCL
// all-reduce of the centroid sums + counts per Lloyd iteration.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "ec_comm.h"
#include "ec_gemm.cuh"
#include "ec_ivf.h"
#include "ec_state.h"

namespace ec {

#define EC_TRY(expr)              \
  do {                            \
    int rc_ = (expr);             \
    if (rc_ != EC_OK) return rc_; \
  } while (0)

// scoped device buffer
struct DBuf {
  Device* d = nullptr;
  void* p = nullptr;
  size_t n = 0;
  int alloc(Device& dev, size_t bytes, const char* what) {
    d = &dev;
    n = bytes;
    return dev_alloc(dev, &p, bytes, what);
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
  ~DBuf() {
    if (p) dev_free(*d, p, n);
  }
};

// run fn(k) on every device, one host thread each; first error wins
template <class F>
static int on_devices(int nd, F fn) {
  if (nd == 1) return fn(0);
  std::vector<int> rc(nd, EC_OK);
  std::vector<std::string> msg(nd);
  std::vector<std::thread> th;
  for (int k = 0; k < nd; ++k)
    th.emplace_back([&, k] {
      rc[k] = fn(k);
      if (rc[k]) msg[k] = ec_last_error();
    });
  for (auto& t : th) t.join();
  for (int k = 0; k < nd; ++k)
    if (rc[k]) return set_error(rc[k], "device %d: %s", G().devs[k]->ordinal, msg[k].c_str());
  return EC_OK;
}

static void split(int64_t n, int parts, int k, int64_t* b, int64_t* e) {
  const int64_t per = (n + parts - 1) / parts;
  *b = std::min<int64_t>(n, per * k);
  *e = std::min<int64_t>(n, per * (k + 1));
}

// ------------------------------------------------- tensor-core assignment --
// ann::nearest-centroid for n device-resident rows: bf16 tcgen05 scores with
// a rigorous error window, candidates re-scored exactly, the rest of the rows
// through the exact scan (ec_ivf_tc.cu).  Identical results to launch_assign.
struct TcAssign {
  DBuf xb, xnorm, cb, cmax, mloc, pk, fbr, fbn, tmp;
  int64_t n = 0;
  int d = 0, k = 0, parts = 0;
  float rel2 = 0.f;
  bool ready = false;
};

static bool tc_assign_eligible(int64_t n, int d, int k) {
  return getenv("EC_EXACT_ASSIGN") == nullptr && n > 0 && n < (int64_t{1} << 31) - 1 && d > 0 &&
         d % 64 == 0 && d <= 8192 && k > 0 && k % 128 == 0;
}

// buffers for n rows and the rows' bf16 copy; t.ready stays false (and no
// error is left set) when they do not fit, so the caller scans exactly
static int tc_assign_setup(Device& dv, TcAssign& t, const float* X, int64_t n, int d, int k,
                           cudaStream_t st) {
  t.ready = false;
  if (!tc_assign_eligible(n, d, k)) return EC_OK;
  const int bn = gemm_pick_bn(static_cast<int>(std::min<int64_t>(n, 1 << 30)), k, kEpiArgCand,
                              dv.num_sms);
  if (!bn) return EC_OK;
  t.n = n;
  t.d = d;
  t.k = k;
  t.parts = 2 * (k / bn);
  t.rel2 = 2.0f * argcand_rel(d);
  const size_t pn = static_cast<size_t>(t.parts) * n;
  const bool fit = !t.xb.alloc(dv, static_cast<size_t>(n) * d * 2, "assign rows bf16") &&
                   !t.xnorm.alloc(dv, static_cast<size_t>(n) * 4, "assign row norms") &&
                   !t.cb.alloc(dv, static_cast<size_t>(k) * d * 2, "assign centroids bf16") &&
                   !t.cmax.alloc(dv, 256, "assign centroid norm") &&
                   !t.mloc.alloc(dv, pn * 4, "assign part maxima") &&
                   !t.pk.alloc(dv, pn * 4, "assign candidates") &&
                   !t.fbr.alloc(dv, static_cast<size_t>(n) * 8, "assign exact rows") &&
                   !t.fbn.alloc(dv, 256, "assign exact count") &&
                   !t.tmp.alloc(dv, static_cast<size_t>(n) * 4, "assign exact results");
  if (!fit) {
    clear_error();  // not enough memory: the exact scan needs none of it
    return EC_OK;
  }
  EC_TRY(check_cuda(launch_round_rows(X, n, d, t.xb.as<__nv_bfloat16>(), t.xnorm.as<float>(),
                                      nullptr, st),
                    "round rows"));
  t.ready = true;
  return EC_OK;
}

static int tc_assign_run(Device& dv, TcAssign& t, const float* X, const float* C, int32_t* out,
                         cudaStream_t st) {
  const int64_t n = t.n;
  const int d = t.d, k = t.k;
  EC_TRY(check_cuda(cudaMemsetAsync(t.cmax.p, 0, 4, st), "centroid norm clear"));
  EC_TRY(check_cuda(launch_round_rows(C, k, d, t.cb.as<__nv_bfloat16>(), nullptr,
                                      t.cmax.as<unsigned>(), st),
                    "round centroids"));
  ArgCandEpi ac{t.xnorm.as<float>(), t.cmax.as<float>(), t.rel2, t.mloc.as<float>(),
                t.pk.as<uint32_t>()};
  GemmLaunch g;
  g.A = t.xb.as<__nv_bfloat16>();
  g.lda = d;
  g.W = t.cb.as<__nv_bfloat16>();
  g.ldw = d;
  g.M = static_cast<int>(n);
  g.N = k;
  g.K = d;
  g.bias = nullptr;
  g.resid = nullptr;
  g.ldr = 0;
  g.out = nullptr;
  g.ldo = 0;
  g.epi = kEpiArgCand;
  g.bn = 0;
  g.status = dv.status;
  g.ac = &ac;
  {
    // event-timed while profiling (class 0: tensor-core GEMMs)
    const int e0 = prof_begin(dv);
    const cudaError_t e = launch_gemm(g, st, dv.num_sms);
    prof_end(dv, 0, 2.0 * static_cast<double>(n) * k * d,
             2.0 * static_cast<double>(n) * d + 2.0 * k * d + 8.0 * t.parts * n, e0);
    EC_TRY(check_cuda(e, "assign scores"));
  }
  EC_TRY(check_cuda(cudaMemsetAsync(t.fbn.p, 0, 8, st), "exact count clear"));
  {
    const int e0 = prof_begin(dv);
    const cudaError_t e = launch_argcand_reduce(
        X, n, d, C, t.xnorm.as<float>(), t.cmax.as<float>(), t.rel2, t.parts, t.mloc.as<float>(),
        t.pk.as<uint32_t>(), out, t.fbr.as<int64_t>(),
        t.fbn.as<unsigned long long>(), st);
    prof_end(dv, 2, 0.0, 8.0 * t.parts * n + 4.0 * n * d, e0);
    EC_TRY(check_cuda(e, "assign candidates"));
  }
  unsigned long long nfb = 0;
  EC_TRY(check_cuda(cudaMemcpyAsync(&nfb, t.fbn.p, 8, cudaMemcpyDeviceToHost, st), "exact count"));
  EC_TRY(sync_and_check(dv, "assign scores"));
  {
    std::lock_guard<std::mutex> lk(G().stat_mu);
    prof_collect(dv);
  }
  if (nfb > static_cast<unsigned long long>(n)) return set_error(EC_ECUDA, "assign: bad exact count");
  if (nfb) {
    EC_TRY(check_cuda(launch_assign(X, t.fbr.as<int64_t>(), static_cast<int64_t>(nfb), C, k, d,
                                    t.tmp.as<int32_t>(), st),
                      "assign exact rows"));
    EC_TRY(check_cuda(launch_scatter_assign(t.fbr.as<int64_t>(), static_cast<int64_t>(nfb),
                                            t.tmp.as<int32_t>(), out, st),
                      "assign scatter"));
  }
  {
    std::lock_guard<std::mutex> lk(G().stat_mu);
    G().assign_tc_rows += n - static_cast<int64_t>(nfb);
    G().assign_exact_rows += static_cast<int64_t>(nfb);
  }
  return EC_OK;
}

// ------------------------------------------------------------------ kmeans --
// Device buffers of one rank's k-means; owned by ec_kmeans so that, after a
// failed exchange, the communicators are aborted before any of this memory
// is freed (cudaFree would wait behind a collective that never completes).
struct KmeansDev {
  DBuf bx, bc, ba, bh, bcnt, boffs, bl, bs, bprev;
  TcAssign tc;
};

enum KmeansExchange { kKmSingle = 0, kKmChain = 1, kKmAllReduce = 2 };

// One rank's Lloyd iterations over its contiguous shard sample[j0, j1).
// kKmChain: the per-cluster sums continue from the previous rank's (rank
// order = sample order), so every add follows ann.lisp:107-122's serial
// loop; the last rank divides and broadcasts the centroids.
// x_dev: the caller's n rows already on this device (the one-upload build);
// the training rows are then a slice of it or gathered from it on the device.
// On return *rows_dev is the device copy of the training rows.
static int kmeans_device(int li, const float* x, int64_t n, int d, const int64_t* sample,
                         int64_t j0, int64_t j1, int k, int iters, const float* cent0,
                         float* cent_out, KmeansExchange mode, KmeansDev& w,
                         const float* x_dev = nullptr, const float** rows_dev = nullptr) {
  Device& dv = *G().devs[li];
  EC_TRY(check_cuda(cudaSetDevice(dv.ordinal), "cudaSetDevice"));
  const int64_t ns = j1 - j0;
  const bool trace = getenv("EC_TRACE_IVF") != nullptr;
  auto t_start = std::chrono::steady_clock::now();
  auto phase = [&](const char* what) {
    if (!trace) return;
    cudaStreamSynchronize(dv.stream);
    const auto now = std::chrono::steady_clock::now();
    fprintf(stderr, "[ec kmeans dev %d] %s %.1f ms\n", dv.ordinal, what,
            std::chrono::duration<double, std::milli>(now - t_start).count());
    t_start = now;
  };
  // training rows of this shard, in sample order (ann.lisp:99-103); a
  // contiguous run of rows is uploaded from the caller's array directly
  bool run = ns > 0;
  for (int64_t j = 1; run && j < ns; ++j) run = sample[j0 + j] == sample[j0] + j;
  std::vector<float> xs;
  const float* src = run ? x + sample[j0] * d : nullptr;
  if (!run && !x_dev) {
    xs.resize(static_cast<size_t>(std::max<int64_t>(ns, 1)) * d);
    for (int64_t j = 0; j < ns; ++j)
      std::memcpy(&xs[static_cast<size_t>(j) * d], x + sample[j0 + j] * d, static_cast<size_t>(d) * 4);
    src = xs.data();
  }
  (void)n;
  phase("gather");
  const int64_t nt = sort_tiles(ns);
  const size_t nsum = static_cast<size_t>(k) * (d + 1);
  // X: the training rows on the device, in sample order
  const float* X = nullptr;
  if (x_dev && run) {
    X = x_dev + sample[j0] * d;
  } else {
    EC_TRY(w.bx.alloc(dv, static_cast<size_t>(std::max<int64_t>(ns, 1)) * d * 4, "kmeans rows"));
    X = w.bx.as<float>();
  }
  if (rows_dev) *rows_dev = X;
  EC_TRY(w.bc.alloc(dv, static_cast<size_t>(k) * d * 4, "centroids"));
  EC_TRY(w.ba.alloc(dv, static_cast<size_t>(std::max<int64_t>(ns, 1)) * 4, "assignments"));
  EC_TRY(w.bh.alloc(dv, static_cast<size_t>(std::max<int64_t>(nt, 1)) * k * 4, "sort scratch"));
  EC_TRY(w.bcnt.alloc(dv, static_cast<size_t>(k) * 4, "counts"));
  EC_TRY(w.boffs.alloc(dv, static_cast<size_t>(k + 1) * 8, "offsets"));
  EC_TRY(w.bl.alloc(dv, static_cast<size_t>(std::max<int64_t>(ns, 1)) * 4, "lists"));
  EC_TRY(w.bs.alloc(dv, nsum * 4, "sums"));
  if (mode == kKmChain) EC_TRY(w.bprev.alloc(dv, nsum * 4, "previous ranks' sums"));
  cudaStream_t st = dv.stream;
  if (x_dev) {
    if (ns > 0 && !run) {
      // the sample's rows gathered from the resident copy (indices checked
      // against n by the caller)
      DBuf bi;
      EC_TRY(bi.alloc(dv, static_cast<size_t>(ns) * 8, "sample indices"));
      EC_TRY(check_cuda(cudaMemcpyAsync(bi.p, sample + j0, static_cast<size_t>(ns) * 8,
                                        cudaMemcpyHostToDevice, st), "sample upload"));
      EC_TRY(check_cuda(launch_gather_rows(x_dev, bi.as<int64_t>(), ns, d, w.bx.as<float>(),
                                           dv.num_sms, st), "sample gather"));
      EC_TRY(check_cuda(cudaStreamSynchronize(st), "sample gather"));
    }
  } else if (ns > 0) {
    EC_TRY(upload_h2d(dv, w.bx.p, src, static_cast<size_t>(ns) * d * 4, "rows upload"));
  }
  EC_TRY(check_cuda(cudaMemcpyAsync(w.bc.p, cent0, static_cast<size_t>(k) * d * 4,
                                    cudaMemcpyHostToDevice, st), "centroid upload"));
  phase("alloc + upload");
  if (ns > 0) EC_TRY(tc_assign_setup(dv, w.tc, X, ns, d, k, st));
  phase("assign setup");
  const int rank = comm_rank(li), world = comm_world();
  if (mode != kKmSingle) EC_TRY(comm_rendezvous(li, static_cast<int>(G().devs.size())));
  for (int it = 0; it < iters; ++it) {
    if (ns > 0) {
      if (w.tc.ready) {
        EC_TRY(tc_assign_run(dv, w.tc, X, w.bc.as<float>(), w.ba.as<int32_t>(), st));
      } else {
        EC_TRY(check_cuda(launch_assign(X, nullptr, ns, w.bc.as<float>(), k, d,
                                        w.ba.as<int32_t>(), st), "assign"));
      }
    }
    EC_TRY(check_cuda(launch_lists(w.ba.as<int32_t>(), ns, k, w.bh.as<uint32_t>(), w.bcnt.as<uint32_t>(),
                                   w.boffs.as<int64_t>(), 0u, w.bl.as<uint32_t>(), st), "lists"));
    if (mode == kKmChain) {
      // sums of ranks 0..rank-1 arrive from rank-1; this shard's rows
      // continue them; the next rank continues from here
      if (rank > 0) EC_TRY(comm_recv_f32(li, w.bprev.as<float>(), nsum, rank - 1, st));
      EC_TRY(check_cuda(launch_segsum(X, w.bl.as<uint32_t>(), w.boffs.as<int64_t>(), k, d,
                                      rank > 0 ? w.bprev.as<float>() : nullptr, w.bs.as<float>(), st),
                        "sums"));
      if (rank + 1 < world) {
        EC_TRY(comm_send_f32(li, w.bs.as<float>(), nsum, rank + 1, st));
      } else {
        EC_TRY(check_cuda(launch_update(w.bs.as<float>(), k, d, w.bc.as<float>(), st), "update"));
      }
      EC_TRY(comm_bcast_f32(li, w.bc.as<float>(), static_cast<size_t>(k) * d, world - 1, st));
    } else {
      EC_TRY(check_cuda(launch_segsum(X, w.bl.as<uint32_t>(), w.boffs.as<int64_t>(), k, d,
                                      nullptr, w.bs.as<float>(), st),
                        "sums"));
      if (mode == kKmAllReduce) EC_TRY(comm_allreduce_sum_f32(li, w.bs.as<float>(), nsum, st));
      EC_TRY(check_cuda(launch_update(w.bs.as<float>(), k, d, w.bc.as<float>(), st), "update"));
    }
    if (it == 0 || it + 1 == iters) phase(it == 0 ? "iteration 1" : "remaining iterations");
  }
  if (cent_out)
    EC_TRY(check_cuda(cudaMemcpyAsync(cent_out, w.bc.p, static_cast<size_t>(k) * d * 4,
                                      cudaMemcpyDeviceToHost, st), "centroid download"));
  return sync_and_check(dv, "kmeans");
}

// ---------------------------------------------------------------- assign --
static int assign_resident(Device& dv, const float* X, int64_t m, int64_t r0, int d, const float* C,
                           int k, TcAssign* tc, int32_t* assign_out, uint32_t* counts_out,
                           int64_t* offs_out, uint32_t* lists_out);

static int assign_device(int li, const float* x, int64_t r0, int64_t r1, int d, const int64_t* rows,
                         const float* cent, int k, int32_t* assign_out, uint32_t* counts_out,
                         int64_t* offs_out, uint32_t* lists_out) {
  Device& dv = *G().devs[li];
  EC_TRY(check_cuda(cudaSetDevice(dv.ordinal), "cudaSetDevice"));
  const int64_t m = r1 - r0;
  if (m <= 0) {
    if (counts_out) std::fill(counts_out, counts_out + k, 0u);
    if (offs_out) std::fill(offs_out, offs_out + k + 1, 0);
    return EC_OK;
  }
  std::vector<float> xs;
  const float* src = x + r0 * d;
  if (rows) {
    xs.resize(static_cast<size_t>(m) * d);
    for (int64_t j = 0; j < m; ++j)
      std::memcpy(&xs[static_cast<size_t>(j) * d], x + rows[r0 + j] * d, static_cast<size_t>(d) * 4);
    src = xs.data();
  }
  DBuf bx, bc;
  EC_TRY(bx.alloc(dv, static_cast<size_t>(m) * d * 4, "rows"));
  EC_TRY(bc.alloc(dv, static_cast<size_t>(k) * d * 4, "centroids"));
  EC_TRY(upload_h2d(dv, bx.p, src, static_cast<size_t>(m) * d * 4, "rows upload"));
  EC_TRY(check_cuda(cudaMemcpyAsync(bc.p, cent, static_cast<size_t>(k) * d * 4, cudaMemcpyHostToDevice,
                                    dv.stream),
                    "centroid upload"));
  return assign_resident(dv, bx.as<float>(), m, r0, d, bc.as<float>(), k, nullptr, assign_out,
                         counts_out, offs_out, lists_out);
}

// ann::nearest-centroid of m rows already on the device (X; row j is the
// caller's row r0 + j) against centroids C on the device: assignments
// downloaded to assign_out + r0 and/or inverted lists (ann::assign-all,
// ids r0 + j) to counts_out / offs_out / lists_out.  tc: the tensor-core
// state of an earlier pass over the same X (k-means), reused when ready.
static int assign_resident(Device& dv, const float* X, int64_t m, int64_t r0, int d, const float* C,
                           int k, TcAssign* tc, int32_t* assign_out, uint32_t* counts_out,
                           int64_t* offs_out, uint32_t* lists_out) {
  cudaStream_t st = dv.stream;
  DBuf ba;
  EC_TRY(ba.alloc(dv, static_cast<size_t>(m) * 4, "assignments"));
  {
    TcAssign own;
    TcAssign* t = (tc && tc->ready && tc->n == m && tc->d == d && tc->k == k) ? tc : &own;
    if (t == &own) EC_TRY(tc_assign_setup(dv, own, X, m, d, k, st));
    if (t->ready) {
      EC_TRY(tc_assign_run(dv, *t, X, C, ba.as<int32_t>(), st));
    } else {
      EC_TRY(check_cuda(launch_assign(X, nullptr, m, C, k, d, ba.as<int32_t>(), st), "assign"));
    }
  }
  if (assign_out)
    EC_TRY(check_cuda(cudaMemcpyAsync(assign_out + r0, ba.p, static_cast<size_t>(m) * 4,
                                      cudaMemcpyDeviceToHost, st), "assign download"));
  if (lists_out) {
    DBuf bh, bcnt, boffs, bl;
    const int64_t nt = sort_tiles(m);
    EC_TRY(bh.alloc(dv, static_cast<size_t>(nt) * k * 4, "sort scratch"));
    EC_TRY(bcnt.alloc(dv, static_cast<size_t>(k) * 4, "counts"));
    EC_TRY(boffs.alloc(dv, static_cast<size_t>(k + 1) * 8, "offsets"));
    EC_TRY(bl.alloc(dv, static_cast<size_t>(m) * 4, "lists"));
    EC_TRY(check_cuda(launch_lists(ba.as<int32_t>(), m, k, bh.as<uint32_t>(), bcnt.as<uint32_t>(),
                                   boffs.as<int64_t>(), static_cast<uint32_t>(r0), bl.as<uint32_t>(), st),
                      "lists"));
    EC_TRY(check_cuda(cudaMemcpyAsync(counts_out, bcnt.p, static_cast<size_t>(k) * 4,
                                      cudaMemcpyDeviceToHost, st), "counts download"));
    EC_TRY(check_cuda(cudaMemcpyAsync(offs_out, boffs.p, static_cast<size_t>(k + 1) * 8,
                                      cudaMemcpyDeviceToHost, st), "offsets download"));
    EC_TRY(check_cuda(cudaMemcpyAsync(lists_out, bl.p, static_cast<size_t>(m) * 4,
                                      cudaMemcpyDeviceToHost, st), "lists download"));
    return sync_and_check(dv, "assign-all");
  }
  return sync_and_check(dv, "assign");
}

static int check_common(int64_t n, int d, int k) {
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (n < 0 || d <= 0 || d % 4 || d > 8192) return set_error(EC_EINVAL, "dim %d must be a positive multiple of 4 (<= 8192)", d);
  if (k <= 0 || k > 32768) return set_error(EC_EINVAL, "k %d outside 1..32768", k);
  if (n > 0xffffffffLL) return set_error(EC_EINVAL, "more than 2^32 rows");
  return EC_OK;
}

// --------------------------------------------------------------- search --
static int ensure_search_ws(Device& dv, size_t bytes, void** out) {
  IndexW& ix = dv.index;
  if (ix.sws && ix.sws_bytes >= bytes) {
    *out = ix.sws;
    return EC_OK;
  }
  if (ix.sws) {
    dev_free(dv, ix.sws, ix.sws_bytes);
    ix.sws = nullptr;
    ix.sws_bytes = 0;
  }
  EC_TRY(dev_alloc(dv, &ix.sws, bytes, "search workspace"));
  ix.sws_bytes = bytes;
  *out = ix.sws;
  return EC_OK;
}

static size_t a256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Rows the probes of one search batch cover (profiling only: reads the
// probes back, so the stream is idle when the timed scan starts).
static double probed_rows(Device& dv, const int32_t* dp, int64_t np) {
  const IndexW& ix = dv.index;
  std::vector<int32_t> h(static_cast<size_t>(np));
  if (np <= 0 || ix.h_offs.size() < static_cast<size_t>(ix.k) + 1) return 0;
  if (cudaMemcpyAsync(h.data(), dp, static_cast<size_t>(np) * 4, cudaMemcpyDeviceToHost, dv.stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(dv.stream) != cudaSuccess)
    return 0;
  double r = 0;
  for (const int32_t c : h)
    if (c >= 0 && c < ix.k) r += static_cast<double>(ix.h_offs[c + 1] - ix.h_offs[c]);
  return r;
}

// Tensor-core probe scores for a batch of at least 64 queries (d % 64 == 0,
// k % 128 == 0, nprobe <= 128); EC_EXACT_PROBE keeps the exact SIMT scores.
// Both give the same probes.
static bool probe_tc_ok(const IndexW& ix, int64_t nq, int nprobe) {
  static const bool off = getenv("EC_EXACT_PROBE") != nullptr;
  return !off && nq >= 64 && nq < (int64_t{1} << 31) && ix.d % 64 == 0 && ix.d <= 8192 && ix.k % 128 == 0 &&
         ix.k <= 8192 && nprobe <= 128;
}

// bf16 copy of the index centroids and their norm bound, made on first use
static int ensure_cent_bf16(Device& dv, cudaStream_t st) {
  IndexW& ix = dv.index;
  if (ix.cent_b) return EC_OK;
  void* cb = nullptr;
  void* cm = nullptr;
  EC_TRY(dev_alloc(dv, &cb, static_cast<size_t>(ix.k) * ix.d * 2, "probe centroids bf16"));
  ix.owned.push_back(cb);
  EC_TRY(dev_alloc(dv, &cm, 256, "probe centroid norm"));
  ix.owned.push_back(cm);
  EC_TRY(check_cuda(cudaMemsetAsync(cm, 0, 4, st), "centroid norm clear"));
  EC_TRY(check_cuda(launch_round_rows(ix.cent, ix.k, ix.d, static_cast<__nv_bfloat16*>(cb), nullptr,
                                      static_cast<unsigned*>(cm), st),
                    "round centroids"));
  ix.cent_b = cb;
  ix.cent_max = static_cast<float*>(cm);
  return EC_OK;
}

// Query-batched scan when each probed list gets 8 queries on average (IVF)
// or there are 8 queries (flat); EC_SCAN_PER_QUERY keeps one CTA per
// (query, list / chunk).  Search workspaces are 256-byte aligned, so Q is.
static bool scan_batched_ok(const IndexW& ix, int64_t nq, int nprobe, int topk, bool ivf) {
  static const bool off = getenv("EC_SCAN_PER_QUERY") != nullptr;
  if (off || !batched_scan_supported(ix.x, ix.x, ix.d, topk)) return false;
  return ivf ? nq * nprobe >= 8 * static_cast<int64_t>(ix.k) : nq >= 8;
}

static int search_device(int li, const float* q, int64_t q0, int64_t q1, int nprobe, int topk, bool ivf,
                         int64_t* ids, float* scores) {
  Device& dv = *G().devs[li];
  IndexW& ix = dv.index;
  EC_TRY(check_cuda(cudaSetDevice(dv.ordinal), "cudaSetDevice"));
  const int d = ix.d;
  cudaStream_t st = dv.stream;
  const int64_t QB = 16384;
  // EC_TRACE_SEARCH: per-phase device time of each batch on stderr
  static const bool trace = getenv("EC_TRACE_SEARCH") != nullptr;
  struct Events {
    cudaEvent_t e[7] = {};
    ~Events() {
      for (auto x : e)
        if (x) cudaEventDestroy(x);
    }
  } tevs;
  cudaEvent_t* tev = tevs.e;
  if (trace)
    for (int i = 0; i < 7; ++i) cudaEventCreate(&tev[i]);
  auto mark = [&](int i) {
    if (trace) cudaEventRecord(tev[i], st);
  };
  for (int64_t a = q0; a < q1; a += QB) {
    const int64_t nq = std::min(QB, q1 - a);
    const int nchunks = ivf ? 0 : static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(1, (ix.n + 8191) / 8192)));
    // query-batched scans once a batch gives each list several queries
    // (flat: once there are several queries); one CTA per (query, list)
    // otherwise, each list split over up to 8 CTAs while the batch leaves
    // the SMs idle (a single query probes only nprobe lists)
    const bool batched = scan_batched_ok(ix, nq, nprobe, topk, ivf);
    int parts = 1;
    if (ivf && !batched) {
      const int64_t ctas = nq * nprobe;
      while (parts < 8 && ctas * parts < 4 * dv.num_sms &&
             static_cast<int64_t>(nprobe) * parts * 2 * topk * 8 <= 150 * 1024)
        parts *= 2;
    }
    const int ngroups = ivf ? nprobe * parts : nchunks;
    const size_t s_q = a256(static_cast<size_t>(nq) * d * 4);
    const size_t s_s = ivf ? a256(static_cast<size_t>(nq) * ix.k * 4) : 0;
    const size_t s_p = ivf ? a256(static_cast<size_t>(nq) * nprobe * 4) : 0;
    const size_t s_c = a256(static_cast<size_t>(nq) * ngroups * topk * 8);
    const size_t s_i = a256(static_cast<size_t>(nq) * topk * 8);
    const size_t s_f = a256(static_cast<size_t>(nq) * topk * 4);
    const size_t s_b = batched && ivf ? a256(batched_list_scan_ws(ix.k, nq * nprobe)) : 0;
    const bool tcp = ivf && probe_tc_ok(ix, nq, nprobe);
    const size_t s_qb = tcp ? a256(static_cast<size_t>(nq) * d * 2) : 0;
    const size_t s_qn = tcp ? a256(static_cast<size_t>(nq) * 4) : 0;
    if (tcp) EC_TRY(ensure_cent_bf16(dv, st));
    void* ws;
    EC_TRY(ensure_search_ws(dv, s_q + s_s + s_p + s_c + s_i + s_f + s_b + s_qb + s_qn, &ws));
    char* w = static_cast<char*>(ws);
    float* dq = reinterpret_cast<float*>(w);
    float* dS = reinterpret_cast<float*>(w + s_q);
    int32_t* dp = reinterpret_cast<int32_t*>(w + s_q + s_s);
    unsigned long long* dc = reinterpret_cast<unsigned long long*>(w + s_q + s_s + s_p);
    int64_t* di = reinterpret_cast<int64_t*>(w + s_q + s_s + s_p + s_c);
    float* df = reinterpret_cast<float*>(w + s_q + s_s + s_p + s_c + s_i);
    mark(0);
    EC_TRY(check_cuda(cudaMemcpyAsync(dq, q + a * d, static_cast<size_t>(nq) * d * 4,
                                      cudaMemcpyHostToDevice, st), "query upload"));
    mark(1);
    if (ivf && tcp) {
      // bf16 queries (and norm bounds) x bf16 centroids on the tensor cores,
      // then the window re-check against the exact scores
      char* wq = w + s_q + s_s + s_p + s_c + s_i + s_f + s_b;
      __nv_bfloat16* dqb = reinterpret_cast<__nv_bfloat16*>(wq);
      float* dqn = reinterpret_cast<float*>(wq + s_qb);
      EC_TRY(check_cuda(launch_round_rows(dq, nq, d, dqb, dqn, nullptr, st), "round queries"));
      GemmLaunch g;
      g.A = dqb;
      g.lda = d;
      g.W = static_cast<const __nv_bfloat16*>(ix.cent_b);
      g.ldw = d;
      g.M = static_cast<int>(nq);
      g.N = ix.k;
      g.K = d;
      g.bias = nullptr;
      g.resid = nullptr;
      g.ldr = 0;
      g.out = dS;
      g.ldo = ix.k;
      g.epi = kEpiF32;
      g.bn = 0;
      g.status = dv.status;
      EC_TRY(check_cuda(launch_gemm(g, st, dv.num_sms), "probe scores"));
      mark(2);
      EC_TRY(check_cuda(launch_probe_select_tc(dS, dq, ix.cent, dqn, ix.cent_max, 2.0f * argcand_rel(d), nq,
                                               ix.k, d, nprobe, dp, st),
                        "probe select"));
      mark(3);
    } else if (ivf) {
      EC_TRY(check_cuda(launch_scores(dq, nq, ix.cent, ix.k, d, dS, st, dv.status), "probe scores"));
      mark(2);
      EC_TRY(check_cuda(launch_probe_select(dS, nq, ix.k, nprobe, dp, st), "probe select"));
      mark(3);
    }
    if (ivf) {
      // event-timed while profiling (class 3: scans; algorithmic work = the
      // probed lists' rows, d multiply-adds and d * 4 bytes each)
      double rows = 0;
      if (G().profile) rows = probed_rows(dv, dp, nq * nprobe);
      const int e0 = prof_begin(dv);
      const cudaError_t e =
          batched ? launch_list_scan_batched(ix.x, d, ix.lists, ix.offs, ix.k, dp, nprobe, dq, nq, topk,
                                             w + s_q + s_s + s_p + s_c + s_i + s_f, dc, st)
                  : launch_list_scan(ix.x, d, ix.lists, ix.offs, dp, nprobe, dq, nq, topk, parts, dc, st,
                                     dv.status);
      prof_end(dv, 3, 2.0 * rows * d, 4.0 * rows * d, e0);
      EC_TRY(check_cuda(e, "list scan"));
    } else {
      mark(2);
      mark(3);
      const int e0 = prof_begin(dv);
      const cudaError_t e = batched ? launch_flat_scan_batched(ix.x, ix.n, d, nchunks, dq, nq, topk, dc, st)
                                    : launch_flat_scan(ix.x, ix.n, d, nchunks, dq, nq, topk, dc, st);
      prof_end(dv, 3, 2.0 * static_cast<double>(nq) * ix.n * d, 4.0 * static_cast<double>(nq) * ix.n * d, e0);
      EC_TRY(check_cuda(e, "flat scan"));
    }
    mark(4);
    EC_TRY(check_cuda(launch_merge(dc, nq, ngroups, topk, di, df, st), "merge"));
    mark(5);
    // small results (one query, say) land in pinned memory with one copy
    // (ids and scores are adjacent in the workspace); larger ones go
    // straight to the caller's arrays
    const size_t res_bytes = s_i + static_cast<size_t>(nq) * topk * 4;
    if (res_bytes <= Device::kResHostBytes && !dv.res_host &&
        cudaHostAlloc(&dv.res_host, Device::kResHostBytes, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      dv.res_host = nullptr;
    }
    const bool pinned = res_bytes <= Device::kResHostBytes && dv.res_host;
    if (pinned) {
      EC_TRY(check_cuda(cudaMemcpyAsync(dv.res_host, di, res_bytes, cudaMemcpyDeviceToHost, st),
                        "results download"));
    } else {
      EC_TRY(check_cuda(cudaMemcpyAsync(ids + a * topk, di, static_cast<size_t>(nq) * topk * 8,
                                        cudaMemcpyDeviceToHost, st), "ids download"));
      EC_TRY(check_cuda(cudaMemcpyAsync(scores + a * topk, df, static_cast<size_t>(nq) * topk * 4,
                                        cudaMemcpyDeviceToHost, st), "scores download"));
    }
    mark(6);
    EC_TRY(sync_and_check(dv, "search"));
    if (pinned) {
      const char* rh = static_cast<const char*>(dv.res_host);
      std::memcpy(ids + a * topk, rh, static_cast<size_t>(nq) * topk * 8);
      std::memcpy(scores + a * topk, rh + s_i, static_cast<size_t>(nq) * topk * 4);
    }
    if (trace) {
      float ms[6] = {};
      for (int i = 0; i < 6; ++i)
        cudaEventElapsedTime(&ms[i], tev[i], tev[i + 1]);
      fprintf(stderr,
              "[ec search dev %d] nq %lld: upload %.3f scores %.3f select %.3f scan %.3f merge %.3f "
              "download %.3f ms\n",
              dv.ordinal, static_cast<long long>(nq), ms[0], ms[1], ms[2], ms[3], ms[4], ms[5]);
    }
    if (G().profile) {
      std::lock_guard<std::mutex> lk(G().stat_mu);
      prof_collect(dv);
    }
  }
  return EC_OK;
}

}  // namespace ec

using namespace ec;

// ec_kmeans without the lock.  x_dev: the caller's rows already on the one
// device (then the training rows are a slice of it or gathered from it);
// post(li, w, X) runs on each device after its iterations, with the k-means
// buffers still alive (X = the device's training rows, w.bc = the final
// centroids).
template <class Post>
static int kmeans_impl(const float* x, int64_t n, int d, const int64_t* sample, int64_t nsample, int k,
                       int iters, const float* init, float* centroids, const float* x_dev, Post post) {
  if (!x || !sample || !centroids || iters < 0 || nsample < 0)
    return set_error(EC_EINVAL, "bad kmeans arguments");
  for (int64_t j = 0; j < nsample; ++j)
    if (sample[j] < 0 || sample[j] >= n) return set_error(EC_EINVAL, "sample[%lld] out of range", (long long)j);
  std::vector<float> c0(static_cast<size_t>(k) * d);
  if (init) {
    std::memcpy(c0.data(), init, c0.size() * 4);
  } else {
    // init: copy k sample rows (ann.lisp:83-86)
    if (nsample < k) return set_error(EC_EINVAL, "sample of %lld rows < k %d", (long long)nsample, k);
    for (int c = 0; c < k; ++c)
      std::memcpy(&c0[static_cast<size_t>(c) * d], x + sample[c] * d, static_cast<size_t>(d) * 4);
  }
  const bool proc = comm_process_mode();
  const int nd = static_cast<int>(G().devs.size());
  if (proc) EC_TRY(comm_check_ready());
  if (!proc && nd > 1) EC_TRY(comm_ensure_local());
  const bool multi = proc ? G().world > 1 : nd > 1;
  const char* ar = getenv("EC_KMEANS_ALLREDUCE");
  const KmeansExchange mode = !multi ? kKmSingle : (ar && *ar && *ar != '0') ? kKmAllReduce : kKmChain;
  std::vector<KmeansDev> work(nd);
  comm_begin();
  const int rc = on_devices(nd, [&](int li) {
    int64_t j0, j1;
    split(nsample, nd, li, &j0, &j1);
    const float* X = nullptr;
    int r = kmeans_device(li, x, n, d, sample, j0, j1, k, iters, c0.data(),
                          li == 0 ? centroids : nullptr, mode, work[li], x_dev, &X);
    if (!r) r = post(li, work[li], X);
    if (r && multi) comm_mark_failed();  // the other ranks stop waiting on this one
    return r;
  });
  if (rc && multi) {
    // abort the whole clique before `work` frees device memory
    const std::string msg = ec_last_error();
    comm_abort_all();
    return set_error(rc, "%s", msg.c_str());
  }
  return rc;
}

extern "C" {

int ec_kmeans(const float* x, int64_t n, int d, const int64_t* sample, int64_t nsample, int k,
              int iters, const float* init, float* centroids) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  EC_TRY(check_common(n, d, k));
  return kmeans_impl(x, n, d, sample, nsample, k, iters, init, centroids, nullptr,
                     [](int, KmeansDev&, const float*) { return EC_OK; });
}

int ec_assign(const float* x, int64_t n, int d, const int64_t* rows, int64_t nrows,
              const float* centroids, int k, int32_t* assign) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  EC_TRY(check_common(n, d, k));
  if (!x || !centroids || !assign) return set_error(EC_EINVAL, "bad assign arguments");
  const int64_t m = rows ? nrows : n;
  if (rows)
    for (int64_t j = 0; j < nrows; ++j)
      if (rows[j] < 0 || rows[j] >= n) return set_error(EC_EINVAL, "rows[%lld] out of range", (long long)j);
  const int nd = static_cast<int>(G().devs.size());
  return on_devices(nd, [&](int li) {
    int64_t r0, r1;
    split(m, nd, li, &r0, &r1);
    return assign_device(li, x, r0, r1, d, rows, centroids, k, assign, nullptr, nullptr, nullptr);
  });
}

// ec_assign_all without the lock
static int assign_all_impl(const float* x, int64_t n, int d, const float* centroids, int k,
                           uint32_t* counts, uint32_t* lists) {
  if (!x || !centroids || !counts || !lists) return set_error(EC_EINVAL, "bad assign-all arguments");
  const int nd = static_cast<int>(G().devs.size());
  if (nd == 1) {
    std::vector<int64_t> offs(k + 1);
    return assign_device(0, x, 0, n, d, nullptr, centroids, k, nullptr, counts, offs.data(), lists);
  }
  std::vector<std::vector<uint32_t>> cnt(nd, std::vector<uint32_t>(k)), lst(nd);
  std::vector<std::vector<int64_t>> offs(nd, std::vector<int64_t>(k + 1));
  for (int li = 0; li < nd; ++li) {
    int64_t r0, r1;
    split(n, nd, li, &r0, &r1);
    lst[li].resize(static_cast<size_t>(std::max<int64_t>(r1 - r0, 1)));
  }
  EC_TRY(on_devices(nd, [&](int li) {
    int64_t r0, r1;
    split(n, nd, li, &r0, &r1);
    return assign_device(li, x, r0, r1, d, nullptr, centroids, k, nullptr, cnt[li].data(), offs[li].data(),
                         lst[li].data());
  }));
  // concatenate the per-device runs of each list in device order: shards are
  // ascending row ranges, so ids stay ascending within a list (ann.lisp:153-157)
  int64_t pos = 0;
  for (int c = 0; c < k; ++c) {
    uint32_t tot = 0;
    for (int li = 0; li < nd; ++li) {
      const int64_t b = offs[li][c], e = offs[li][c + 1];
      std::memcpy(lists + pos, lst[li].data() + b, static_cast<size_t>(e - b) * 4);
      pos += e - b;
      tot += cnt[li][c];
    }
    counts[c] = tot;
  }
  return EC_OK;
}

int ec_assign_all(const float* x, int64_t n, int d, const float* centroids, int k, uint32_t* counts,
                  uint32_t* lists) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  EC_TRY(check_common(n, d, k));
  return assign_all_impl(x, n, d, centroids, k, counts, lists);
}

int ec_ann_build(const float* x, int64_t n, int d, const int64_t* sample, int64_t nsample, int k,
                 int iters, const float* init, float* centroids, uint32_t* counts, uint32_t* lists) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  EC_TRY(check_common(n, d, k));
  if (!x || !centroids || !counts || !lists) return set_error(EC_EINVAL, "bad ann build arguments");
  const int nd = static_cast<int>(G().devs.size());
  if (nd > 1) {
    // several devices in this process: the two passes, each split over them
    EC_TRY(kmeans_impl(x, n, d, sample, nsample, k, iters, init, centroids, nullptr,
                       [](int, KmeansDev&, const float*) { return EC_OK; }));
    return assign_all_impl(x, n, d, centroids, k, counts, lists);
  }
  // one device: the rows go up once; k-means trains on them (a slice, or
  // the sample gathered on the device) and the final assignment reads the
  // same copy, with the k-means pass's bf16 rows when it covered them all
  Device& dv = *G().devs[0];
  EC_TRY(check_cuda(cudaSetDevice(dv.ordinal), "cudaSetDevice"));
  const bool trace = getenv("EC_TRACE_IVF") != nullptr;
  auto t_last = std::chrono::steady_clock::now();
  auto phase = [&](const char* what) {
    if (!trace) return;
    const auto now = std::chrono::steady_clock::now();
    fprintf(stderr, "[ec ann build dev %d] %s %.1f ms\n", dv.ordinal, what,
            std::chrono::duration<double, std::milli>(now - t_last).count());
    t_last = now;
  };
  DBuf bx;
  EC_TRY(bx.alloc(dv, static_cast<size_t>(std::max<int64_t>(n, 1)) * d * 4, "rows"));
  phase("alloc");
  if (n > 0) EC_TRY(upload_h2d(dv, bx.p, x, static_cast<size_t>(n) * d * 4, "rows upload"));
  phase("rows upload");
  std::vector<int64_t> offs(static_cast<size_t>(k) + 1);
  return kmeans_impl(x, n, d, sample, nsample, k, iters, init, centroids, bx.as<float>(),
                     [&](int, KmeansDev& w, const float* X) {
                       phase("k-means");
                       if (n == 0) {
                         std::fill(counts, counts + k, 0u);
                         return static_cast<int>(EC_OK);
                       }
                       TcAssign* tc = X == bx.as<float>() ? &w.tc : nullptr;
                       const int r = assign_resident(dv, bx.as<float>(), n, 0, d, w.bc.as<float>(), k,
                                                     tc, nullptr, counts, offs.data(), lists);
                       phase("assign-all");
                       return r;
                     });
}

int ec_index_load(const float* x, int64_t n, int d, const float* centroids, int k,
                  const uint32_t* counts, const uint32_t* lists) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!x || n <= 0 || d <= 0 || d % 4 || d > 8192) return set_error(EC_EINVAL, "bad index arguments");
  // the scans keep row ids in the low 32 bits of each candidate key
  if (n > 0xffffffffLL) return set_error(EC_EINVAL, "more than 2^32 rows");
  if (k < 0 || (k > 0 && (!centroids || !counts || !lists)) || k > 8192)
    return set_error(EC_EINVAL, "bad ivf arguments (k <= 8192)");
  std::vector<int64_t> offs(k + 1, 0);
  for (int c = 0; c < k; ++c) offs[c + 1] = offs[c] + counts[c];
  if (k > 0 && offs[k] != n) return set_error(EC_EINVAL, "counts sum to %lld, not n", (long long)offs[k]);
  if (k > 0)
    for (int64_t i = 0; i < n; ++i)
      if (lists[i] >= n) return set_error(EC_EINVAL, "list entry %lld out of range", (long long)i);
  for (Device* dv : G().devs) {
    EC_TRY(check_cuda(cudaSetDevice(dv->ordinal), "cudaSetDevice"));
    if (dv->index.sws) dev_free(*dv, dv->index.sws, dv->index.sws_bytes);
    for (void* p : dv->index.owned) cudaFree(p);
    dv->index = IndexW();
    IndexW& ix = dv->index;
    auto take = [&](void** p, size_t bytes, const char* what) -> int {
      int rc = dev_alloc(*dv, p, bytes, what);
      if (!rc) ix.owned.push_back(*p);
      return rc;
    };
    EC_TRY(take(reinterpret_cast<void**>(&ix.x), static_cast<size_t>(n) * d * 4, "index vectors"));
    EC_TRY(upload_h2d(*dv, ix.x, x, static_cast<size_t>(n) * d * 4, "vectors upload"));
    if (k > 0) {
      EC_TRY(take(reinterpret_cast<void**>(&ix.cent), static_cast<size_t>(k) * d * 4, "centroids"));
      EC_TRY(take(reinterpret_cast<void**>(&ix.lists), static_cast<size_t>(n) * 4, "lists"));
      EC_TRY(take(reinterpret_cast<void**>(&ix.offs), static_cast<size_t>(k + 1) * 8, "offsets"));
      // on the device's stream (searches run there), waited for before the
      // host offsets go away
      EC_TRY(check_cuda(cudaMemcpyAsync(ix.cent, centroids, static_cast<size_t>(k) * d * 4,
                                        cudaMemcpyHostToDevice, dv->stream),
                        "centroids upload"));
      EC_TRY(check_cuda(cudaMemcpyAsync(ix.lists, lists, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice,
                                        dv->stream),
                        "lists upload"));
      EC_TRY(check_cuda(cudaMemcpyAsync(ix.offs, offs.data(), static_cast<size_t>(k + 1) * 8,
                                        cudaMemcpyHostToDevice, dv->stream),
                        "offsets upload"));
      EC_TRY(check_cuda(cudaStreamSynchronize(dv->stream), "index upload"));
    }
    ix.n = n;
    ix.d = d;
    ix.k = k;
    ix.h_offs = offs;
  }
  return EC_OK;
}

int ec_ivf_search(const float* q, int nq, int nprobe, int topk, int64_t* ids, float* scores) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  const IndexW& ix = G().devs[0]->index;
  if (!ix.x || ix.k <= 0) return set_error(EC_ESTATE, "no IVF index loaded");
  if (nq == 0) return EC_OK;
  if (!q || nq < 0 || !ids || !scores || topk < 1 || topk > 64 || nprobe < 1)
    return set_error(EC_EINVAL, "bad search arguments (1 <= topk <= 64, nprobe >= 1)");
  nprobe = std::min(nprobe, ix.k);  // (min *ann-nprobe* *ann-k*) kb.lisp:350
  if (static_cast<size_t>(nprobe) * topk * 8 + 256 > 200 * 1024)
    return set_error(EC_EINVAL, "nprobe * topk too large");
  const int nd = static_cast<int>(G().devs.size());
  return on_devices(nd, [&](int li) {
    int64_t a, b;
    split(nq, nd, li, &a, &b);
    return a < b ? search_device(li, q, a, b, nprobe, topk, true, ids, scores) : EC_OK;
  });
}

int ec_flat_search(const float* q, int nq, int topk, int64_t* ids, float* scores) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  const IndexW& ix = G().devs[0]->index;
  if (!ix.x) return set_error(EC_ESTATE, "no index loaded");
  if (nq == 0) return EC_OK;
  if (!q || nq < 0 || !ids || !scores || topk < 1 || topk > 64)
    return set_error(EC_EINVAL, "bad search arguments (1 <= topk <= 64)");
  const int nd = static_cast<int>(G().devs.size());
  return on_devices(nd, [&](int li) {
    int64_t a, b;
    split(nq, nd, li, &a, &b);
    return a < b ? search_device(li, q, a, b, 0, topk, false, ids, scores) : EC_OK;
  });
}

}  // extern "C"
