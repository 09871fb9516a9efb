// ec_debug.cu -- kernel-level test hooks (include/embedcuda_debug.h).
#include <algorithm>
#include <numeric>
#include <vector>

#include "../../include/embedcuda_debug.h"
#include "ec_ptx.cuh"
#include "ec_state.h"

using namespace ec;

namespace {

// Waits on a barrier that never completes; the bounded wait gives up after
// limit_ns and the kernel reports kDevTimeoutOther.
__global__ void wait_timeout_kernel(unsigned* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = globaltimer_ns();
    bool done = false;
    while (!done) {
      done = mbar_try_wait(&bar, 0);
      if (!done && globaltimer_ns() - t0 > limit_ns) break;
    }
    if (!done) report(status, kDevTimeoutOther);
  }
  __syncthreads();
}

}  // namespace

extern "C" {

int ecdbg_gemm(const void* A, const void* W, int M, int N, int K, const float* bias,
               const float* resid, void* out, int epi, int bn) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  Device& d = *G().devs[0];
  int rc = check_cuda(cudaSetDevice(d.ordinal), "cudaSetDevice");
  if (rc) return rc;
  GemmLaunch g;
  g.A = static_cast<const bf16*>(A);
  g.lda = K;
  g.W = static_cast<const bf16*>(W);
  g.ldw = K;
  g.M = M;
  g.N = N;
  g.K = K;
  g.bias = bias;
  g.resid = resid;
  g.ldr = N;
  g.out = out;
  g.ldo = (epi == 3 || epi == 6) ? N / 2 : N;
  g.epi = epi;
  g.bn = bn;
  g.status = d.status;
  rc = check_cuda(launch_gemm(g, d.stream, d.num_sms), "gemm");
  if (rc) return rc;
  return sync_and_check(d, "gemm");
}

int ecdbg_mlp(const void* A, const void* W1, const void* W2, const float* b1, const float* b2,
              const float* resid, const float* ln_g, const float* ln_b, float* out32, void* outb,
              int M, int H, int F) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!mlp_supported(H, F)) return set_error(EC_EUNSUPPORTED, "fused mlp H %d F %d", H, F);
  Device& d = *G().devs[0];
  int rc = check_cuda(cudaSetDevice(d.ordinal), "cudaSetDevice");
  if (rc) return rc;
  MlpLaunch l{static_cast<const bf16*>(A), static_cast<const bf16*>(W1), static_cast<const bf16*>(W2),
              b1, b2, resid, ln_g, ln_b, out32, static_cast<bf16*>(outb), M, H, F, d.status};
  rc = check_cuda(launch_mlp(l, d.stream, d.num_sms), "fused mlp");
  if (rc) return rc;
  return sync_and_check(d, "fused mlp");
}

int ecdbg_gemm_ln(const void* A, const void* W, int M, int N, int K, const float* bias,
                  const float* resid, const float* ln_g, const float* ln_b, float* out32,
                  void* outb) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!gemm_ln_supported(N)) return set_error(EC_EUNSUPPORTED, "gemm+layernorm N %d", N);
  if (!A || !W || !resid || !ln_g || !ln_b || !out32 || !outb || M <= 0 || K <= 0 || K % 64)
    return set_error(EC_EINVAL, "bad gemm+layernorm arguments");
  Device& d = *G().devs[0];
  int rc = check_cuda(cudaSetDevice(d.ordinal), "cudaSetDevice");
  if (rc) return rc;
  GemmLnLaunch g{static_cast<const bf16*>(A), K, static_cast<const bf16*>(W), M, N, K, bias, resid,
                 ln_g, ln_b, out32, static_cast<bf16*>(outb), d.status};
  rc = check_cuda(launch_gemm_ln(g, d.stream, d.num_sms), "gemm+layernorm");
  if (rc) return rc;
  return sync_and_check(d, "gemm+layernorm");
}

int ecdbg_gemm_norm(const void* A, const void* W, int M, int N, int K, const float* resid,
                    const float* g1, const float* g2, float* out32, void* outb, int mode, float eps,
                    float scale, int has_scale) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!gemm_rms_supported(N)) return set_error(EC_EUNSUPPORTED, "gemm+rmsnorm N %d", N);
  if (!A || !W || !g1 || mode < 1 || mode > 3 || M <= 0 || K <= 0 || K % 64)
    return set_error(EC_EINVAL, "bad gemm+rmsnorm arguments");
  Device& d = *G().devs[0];
  int rc = check_cuda(cudaSetDevice(d.ordinal), "cudaSetDevice");
  if (rc) return rc;
  GemmLnLaunch g{static_cast<const bf16*>(A), K, static_cast<const bf16*>(W), M, N, K, nullptr,
                 resid, g1, g2, out32, static_cast<bf16*>(outb), d.status};
  g.mode = mode;
  g.eps = eps;
  g.scale = scale;
  g.has_scale = has_scale;
  rc = check_cuda(launch_gemm_ln(g, d.stream, d.num_sms), "gemm+rmsnorm");
  if (rc) return rc;
  return sync_and_check(d, "gemm+rmsnorm");
}

int ecdbg_attention(const void* qkv, int ld, int q_off, int k_off, int v_off, void* out,
                    const int32_t* cu_dev, const int32_t* lens_host, int nseq, int heads,
                    int kv_heads, int head_dim, int causal) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!qkv || !out || !cu_dev || !lens_host || nseq <= 0 || heads <= 0 || kv_heads <= 0 ||
      heads % kv_heads || (head_dim != 32 && head_dim != 64 && head_dim != 128) ||
      q_off + heads * head_dim > ld || k_off + kv_heads * head_dim > ld || v_off + kv_heads * head_dim > ld)
    return set_error(EC_EINVAL, "bad attention arguments (heads %% kv_heads == 0, offsets inside ld)");
  for (int s = 0; s < nseq; ++s)
    if (lens_host[s] <= 0) return set_error(EC_EINVAL, "sequence %d is empty", s);
  Device& d = *G().devs[0];
  int rc = check_cuda(cudaSetDevice(d.ordinal), "cudaSetDevice");
  if (rc) return rc;
  std::vector<int2> blk;
  std::vector<int> order(nseq);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lens_host[a] > lens_host[b]; });
  for (int s : order)
    for (int q0 = 0; q0 < lens_host[s]; q0 += 64) blk.push_back(make_int2(s, q0));
  const size_t n64 = blk.size();
  std::vector<int> starts(nseq + 1, 0);
  for (int s = 0; s < nseq; ++s) starts[s + 1] = starts[s] + lens_host[s];
  const int T = starts[nseq];
  std::vector<int4> blk128;
  std::vector<int2> seqs;
  int n_long = 0, nblk128_long = 0, max_short = 0;
  for (int s : order) {
    for (int q0 = 0; q0 < lens_host[s]; q0 += 128)
      blk128.push_back(make_int4(starts[s], lens_host[s], q0, 0));
    seqs.push_back(make_int2(starts[s], lens_host[s]));
    if (lens_host[s] > kAttnShortCap) {
      ++n_long;
      nblk128_long = static_cast<int>(blk128.size());
    } else {
      max_short = std::max(max_short, lens_host[s]);
    }
  }
  const size_t b64 = (n64 * 8 + 15) & ~static_cast<size_t>(15);
  const size_t b128 = blk128.size() * 16;
  const size_t tbytes = b64 + b128 + seqs.size() * 8 + 16;
  void* dblk = nullptr;
  rc = dev_alloc(d, &dblk, tbytes, "blocks");
  if (rc) return rc;
  rc = check_cuda(cudaMemcpyAsync(dblk, blk.data(), n64 * 8, cudaMemcpyHostToDevice, d.stream), "blocks");
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(static_cast<char*>(dblk) + b64, blk128.data(), b128,
                                    cudaMemcpyHostToDevice, d.stream),
                    "blocks");
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(static_cast<char*>(dblk) + b64 + b128, seqs.data(), seqs.size() * 8,
                                    cudaMemcpyHostToDevice, d.stream),
                    "sequences");
  AttnLaunch a;
  a.qkv = static_cast<const bf16*>(qkv);
  a.ld = ld;
  a.q_off = q_off;
  a.k_off = k_off;
  a.v_off = v_off;
  a.out = static_cast<bf16*>(out);
  a.ldo = heads * head_dim;
  a.cu = cu_dev;
  a.blocks = static_cast<const int2*>(dblk);
  a.nblocks = static_cast<int>(n64);
  a.blocks128 = reinterpret_cast<const int4*>(static_cast<char*>(dblk) + b64);
  a.nblocks128 = static_cast<int>(blk128.size());
  a.rows = T;
  a.status = d.status;
  a.num_sms = d.num_sms;
  a.seqs = reinterpret_cast<const int2*>(static_cast<char*>(dblk) + b64 + b128);
  a.nseq = nseq;
  a.n_long = n_long;
  a.nblocks128_long = nblk128_long;
  a.max_short_len = max_short;
  {
    std::vector<int> sl;
    for (int s : order) sl.push_back(lens_host[s]);
    attn_short_buckets(sl.data(), n_long, nseq, &a);
  }
  a.heads = heads;
  a.kv_group = heads / kv_heads;
  a.head_dim = head_dim;
  a.causal = causal;
  a.relbias = nullptr;
  a.rel_max = 0;
  if (!rc) rc = check_cuda(launch_attention(a, d.stream), "attention");
  if (!rc) rc = sync_and_check(d, "attention");
  dev_free(d, dblk, tbytes);
  return rc;
}

int ecdbg_profile(int enable) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (enable) {
    for (auto& a : G().prof) a = ProfAcc();
    G().launches = 0;
    for (Device* d : G().devs) d->pend.clear();
  }
  G().profile = enable != 0;
  return EC_OK;
}

int ecdbg_profile_read(const char* cls, double* ms, double* flops, double* bytes,
                       long long* launches) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!cls) return set_error(EC_EINVAL, "class is NULL");
  const std::string c(cls);
  const int i = c == "gemm" ? 0 : c == "attention" ? 1 : c == "rows" ? 2 : c == "scan" ? 3 : -1;
  if (i < 0) return set_error(EC_EINVAL, "unknown class %s", cls);
  const ProfAcc& a = G().prof[i];
  if (ms) *ms = a.ms;
  if (flops) *flops = a.flops;
  if (bytes) *bytes = a.bytes;
  if (launches) *launches = a.launches;
  return EC_OK;
}

int ecdbg_wait_timeout(int limit_ms) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (limit_ms < 1 || limit_ms > 1000) return set_error(EC_EINVAL, "limit_ms outside 1..1000");
  Device& d = *G().devs[0];
  int rc = check_cuda(cudaSetDevice(d.ordinal), "cudaSetDevice");
  if (rc) return rc;
  wait_timeout_kernel<<<1, 32, 0, d.stream>>>(d.status, 1000000ull * limit_ms);
  rc = check_cuda(cudaGetLastError(), "wait kernel");
  if (rc) return rc;
  return sync_and_check(d, "bounded wait");
}

long long ecdbg_launches(void) {
  std::lock_guard<std::mutex> lk(G().mu);
  return G().launches;
}

int ecdbg_kernel_arch(int* binary_version, int* ptx_version) {
  clear_error();
  cudaFuncAttributes a{};
  int rc = check_cuda(cudaFuncGetAttributes(&a, wait_timeout_kernel), "cudaFuncGetAttributes");
  if (rc) return rc;
  if (binary_version) *binary_version = a.binaryVersion;
  if (ptx_version) *ptx_version = a.ptxVersion;
  return EC_OK;
}

int ecdbg_tensor_read(const char* name, void* host, size_t nbytes, int* dtype) {
  std::lock_guard<std::mutex> lk(G().mu);
  clear_error();
  if (!G().inited) return set_error(EC_ESTATE, "ec_init first");
  if (!name || !host) return set_error(EC_EINVAL, "name and host must not be NULL");
  Device& d = *G().devs[0];
  auto it = d.uploads.find(name);
  if (it == d.uploads.end()) return set_error(EC_EINVAL, "no uploaded tensor '%s'", name);
  const Tensor& t = it->second;
  const size_t bytes = t.numel * (t.dtype == kDtBf16 ? 2 : 4);
  if (nbytes != bytes) return set_error(EC_EINVAL, "tensor '%s' holds %zu bytes, not %zu", name, bytes, nbytes);
  if (dtype) *dtype = t.dtype == kDtBf16 ? EC_BF16 : EC_F32;
  int rc = check_cuda(cudaSetDevice(d.ordinal), "cudaSetDevice");
  if (rc) return rc;
  return check_cuda(cudaMemcpy(host, t.p, bytes, cudaMemcpyDeviceToHost), "tensor download");
}

int ecdbg_assign_rows(long long* tc_rows, long long* exact_rows, int reset) {
  std::lock_guard<std::mutex> lk(G().stat_mu);
  if (tc_rows) *tc_rows = G().assign_tc_rows;
  if (exact_rows) *exact_rows = G().assign_exact_rows;
  if (reset) G().assign_tc_rows = G().assign_exact_rows = 0;
  return EC_OK;
}

}  // extern "C"
