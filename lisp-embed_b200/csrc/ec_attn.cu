// ec_attn.cu -- instantiations and host launcher of the varlen attention.
#include <cstdlib>
#include <mutex>
#include <string>

#include <cudaTypedefs.h>

#include "ec_attn.cuh"
#include "ec_attn_short.cuh"
#include "ec_attn_tc.cuh"
#include "ec_fa.cuh"
#include "ec_kernels.h"

namespace ec {

template <int HD, int MODE>
static cudaError_t run_attn(const AttnLaunch& l, cudaStream_t st) {
  static std::mutex mu;
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<HD, MODE>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(AttnSmem<HD>::BYTES));
      if (e != cudaSuccess) return e;
      set[dev] = true;
    }
  }
  AttnArgs a;
  a.qkv = l.qkv;
  a.ld = l.ld;
  a.q_off = l.q_off;
  a.k_off = l.k_off;
  a.v_off = l.v_off;
  a.out = l.out;
  a.ldo = l.ldo;
  a.cu = l.cu;
  a.blocks = l.blocks;
  a.heads = l.heads;
  a.kv_group = l.kv_group;
  a.scale_log2 = 1.4426950408889634f * (l.scale > 0.f ? l.scale : 1.f / sqrtf(static_cast<float>(HD)));
  a.causal = l.causal;
  a.relbias = l.relbias;
  a.rel_max = l.rel_max;
  // heads per CTA: enough CTAs to fill the GPU several times over, else walk
  // several heads per CTA to amortise the tile loads
  int hpc = l.heads % 4 == 0 ? 4 : (l.heads % 2 == 0 ? 2 : 1);
  if (const char* e = getenv("EC_ATTN_HEADS_PER_CTA")) hpc = atoi(e);
  if (hpc < 1 || l.heads % hpc) hpc = 1;
  a.heads_per_cta = hpc;
  dim3 grid(l.nblocks, l.heads / hpc);
  attn_fwd_kernel<HD, MODE><<<grid, kAttnThreads, AttnSmem<HD>::BYTES, st>>>(a);
  return cudaGetLastError();
}

PFN_cuTensorMapEncodeTiled_v12000 gemm_encode_fn();  // ec_gemm.cu

template <int HD, int MODE>
static cudaError_t run_fa(const AttnLaunch& l, cudaStream_t st) {
  using Cfg = FaCfg<HD, MODE>;
  static std::mutex mu;
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(fa_fwd_kernel<HD, MODE>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(Cfg::SMEM_BYTES));
      if (e != cudaSuccess) return e;
      set[dev] = true;
    }
  }
  auto enc = gemm_encode_fn();
  if (!enc) return cudaErrorInvalidValue;
  // the packed Q/K/V rows: total tokens = cu[nseq] is not known on the host
  // here, so the map spans the rows the blocks can reach (the last block's
  // start + 128 is clipped by zero fill past `rows`)
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(l.ld), static_cast<cuuint64_t>(l.rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(l.ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(Cfg::BOX_C), 128};
  cuuint32_t es[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(l.qkv), dims,
          strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
          Cfg::SW64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  FaArgs a;
  a.cu = l.cu;
  a.qinfo = l.blocks128;
  a.nqb = l.nblocks128;
  a.heads = l.heads;
  a.kv_group = l.kv_group;
  a.q_off = l.q_off;
  a.k_off = l.k_off;
  a.v_off = l.v_off;
  a.out = l.out;
  a.ldo = l.ldo;
  a.scale_log2 = 1.4426950408889634f * (l.scale > 0.f ? l.scale : 1.f / sqrtf(static_cast<float>(HD)));
  a.relbias = l.relbias;
  a.rel_max = l.rel_max;
  a.status = l.status;
  const int items = l.nblocks128 * l.heads;
  const int grid = items < l.num_sms ? items : l.num_sms;
  fa_fwd_kernel<HD, MODE><<<grid, kFaThreads, Cfg::SMEM_BYTES, st>>>(tm, a);
  return cudaGetLastError();
}

template <int HD>
static cudaError_t run_fa_mode(const AttnLaunch& l, cudaStream_t st) {
  if (l.causal) return run_fa<HD, 2>(l, st);
  if (l.relbias) {
    // the relative-bias table does not fit beside double-buffered K/V and P
    // at head dim 128; that combination uses the mma.sync kernel
    if constexpr (HD == 128) return run_attn<HD, 1>(l, st);
    else return run_fa<HD, 1>(l, st);
  }
  return run_fa<HD, 0>(l, st);
}

template <int HD>
static cudaError_t run_mode(const AttnLaunch& l, cudaStream_t st) {
  if (l.causal) return run_attn<HD, 2>(l, st);
  if (l.relbias) return run_attn<HD, 1>(l, st);
  return run_attn<HD, 0>(l, st);
}

// sequences [n_long, nseq) of head dim 32 without bias or mask on the
// tcgen05 short-sequence kernel (ec_attn_tc.cuh): persistent, two CTAs per SM
static cudaError_t run_short_tc(const AttnLaunch& l, cudaStream_t st) {
  using Cfg = TcsCfg;
  static std::mutex mu;
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(attn_tc_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(Cfg::SMEM_BYTES));
      if (e != cudaSuccess) return e;
      set[dev] = true;
    }
  }
  if (l.max_short_len <= 0 || l.max_short_len > kAttnShortCap) return cudaErrorInvalidValue;
  auto enc = gemm_encode_fn();
  if (!enc) return cudaErrorInvalidValue;
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(l.ld), static_cast<cuuint64_t>(l.rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(l.ld) * 2};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t es[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<__nv_bfloat16*>(l.qkv), dims, strides,
          box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  TcShortArgs a;
  a.seqs = l.seqs;
  a.first = l.n_long;
  a.nseq = l.nseq - l.n_long;
  a.n_two = l.n_gt128;
  a.heads = l.heads;
  a.kv_group = l.kv_group;
  a.q_off = l.q_off;
  a.k_off = l.k_off;
  a.v_off = l.v_off;
  a.out = l.out;
  a.ldo = l.ldo;
  a.scale_log2 = 1.4426950408889634f * (l.scale > 0.f ? l.scale : 1.f / sqrtf(32.f));
  a.status = l.status;
  const int units = (a.n_two * 2 + (a.nseq - a.n_two)) * a.heads;
  const int grid = units < l.num_sms ? units : l.num_sms;
  if (grid <= 0) return cudaSuccess;
  attn_tc_short_kernel<<<grid, kTcsThreads, Cfg::SMEM_BYTES, st>>>(tm, a);
  return cudaGetLastError();
}

void attn_short_buckets(const int* lens_sorted, int n_long, int nseq, AttnLaunch* a) {
  static const int cap[4] = {kAttnShortCap, 192, 128, 64};
  a->nbuckets = 0;
  a->n_gt128 = 0;
  int prev = -1;
  for (int k = n_long; k < nseq; ++k) {
    if (lens_sorted[k] > 128) ++a->n_gt128;
    int b = 0;
    while (b < 3 && lens_sorted[k] <= cap[b + 1]) ++b;
    if (b != prev) {
      a->bucket_first[a->nbuckets] = k;
      a->bucket_max[a->nbuckets] = lens_sorted[k];
      ++a->nbuckets;
      prev = b;
    }
  }
  a->bucket_first[a->nbuckets] = nseq;
}

// sequences [n_long, nseq) of the launch, one CTA per (sequence, head);
// F16P: the kernel with fp16 probabilities (attn_short_h_kernel, key blocks
// of BK, PV2 accumulator sets); bucketed: one launch per length bucket, each
// sized for its longest sequence (less shared memory per CTA)
template <int HD, int MODE, int BK, int MINB, bool F16P, bool PV2 = false>
static cudaError_t run_short(const AttnLaunch& l, cudaStream_t st, bool bucketed = false) {
  using S = ShortAttnSmem<HD, MODE>;
  static_assert(kShortAttnMaxLen == kAttnShortCap, "short-kernel capacity");
  static std::mutex mu;
  static bool set[64] = {};
  const void* fn = F16P ? reinterpret_cast<const void*>(attn_short_h_kernel<HD, MODE, MINB, BK, PV2>)
                        : reinterpret_cast<const void*>(attn_short_kernel<HD, MODE, BK, MINB>);
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(S::MAX_BYTES));
      if (e != cudaSuccess) return e;
      set[dev] = true;
    }
  }
  if (l.max_short_len <= 0 || l.max_short_len > kShortAttnMaxLen) return cudaErrorInvalidValue;
  ShortAttnArgs a;
  a.qkv = l.qkv;
  a.ld = l.ld;
  a.q_off = l.q_off;
  a.k_off = l.k_off;
  a.v_off = l.v_off;
  a.out = l.out;
  a.ldo = l.ldo;
  a.seqs = l.seqs;
  a.first = l.n_long;
  a.heads = l.heads;
  a.kv_group = l.kv_group;
  a.scale_log2 = 1.4426950408889634f * (l.scale > 0.f ? l.scale : 1.f / sqrtf(static_cast<float>(HD)));
  a.relbias = l.relbias;
  a.rel_max = l.rel_max;
  const int nb = bucketed && l.nbuckets > 0 ? l.nbuckets : 1;
  for (int b = 0; b < nb; ++b) {
    const int first = nb > 1 ? l.bucket_first[b] : l.n_long;
    const int last = nb > 1 ? l.bucket_first[b + 1] : l.nseq;
    const int maxlen = nb > 1 ? l.bucket_max[b] : l.max_short_len;
    if (last <= first) continue;
    a.first = first;
    a.kcap = (maxlen + 15) & ~15;
    dim3 grid(last - first, l.heads);
    cudaError_t e;
    if (F16P) {
      e = launch_pdl(attn_short_h_kernel<HD, MODE, MINB, BK, PV2>, grid, dim3(kShortAttnThreads),
                     S::bytes(a.kcap), st, a);
    } else {
      attn_short_kernel<HD, MODE, BK, MINB><<<grid, kShortAttnThreads, S::bytes(a.kcap), st>>>(a);
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

template <int HD, int MODE>
static cudaError_t run_short_h(const AttnLaunch& l, cudaStream_t st) {
  // EC_SHORT_ATTN_CFG=<key block>,<two accumulator sets>,<CTAs per SM>[,b]
  // picks a measured variant of the fp16-probability kernel for head dim
  // 32 (default 64,0,5); a trailing ",b" launches per length bucket
  constexpr int MINB = HD == 32 ? 5 : 1;
  const char* cfg = getenv("EC_SHORT_ATTN_CFG");
  const std::string c = cfg ? cfg : "";
  const bool bk = c.find(",b") != std::string::npos;
  if constexpr (HD == 32) {
    if (c.rfind("32,0,6", 0) == 0) return run_short<HD, MODE, 32, 6, true, false>(l, st, bk);
    if (c.rfind("64,1,4", 0) == 0) return run_short<HD, MODE, 64, 4, true, true>(l, st, bk);
    if (c.rfind("32,1,5", 0) == 0) return run_short<HD, MODE, 32, 5, true, true>(l, st, bk);
  }
  return run_short<HD, MODE, 64, MINB, true, false>(l, st, bk);
}

template <int HD>
static cudaError_t run_short_mode(const AttnLaunch& l, cudaStream_t st) {
  // head dim 32 fits five CTAs per SM (94 registers, 40 KB of K/V); the
  // register budget for that measured fastest among 64/128-key blocks and
  // 4..6 CTAs per SM on MiniLM batches.  EC_SHORT_ATTN_BF16 keeps the fp32
  // exponentials with bf16 probabilities.
  constexpr int MINB = HD == 32 ? 5 : 1;
  const bool bf16p = getenv("EC_SHORT_ATTN_BF16") != nullptr;
  if (bf16p) {
    if (l.causal) return run_short<HD, 2, 64, MINB, false>(l, st);
    if (l.relbias) return run_short<HD, 1, 64, MINB, false>(l, st);
    return run_short<HD, 0, 64, MINB, false>(l, st);
  }
  if (l.causal) return run_short_h<HD, 2>(l, st);
  if (l.relbias) return run_short_h<HD, 1>(l, st);
  // head dim 32, no bias or mask: the tcgen05 kernel when EC_SHORT_ATTN_TC
  if (HD == 32 && getenv("EC_SHORT_ATTN_TC") != nullptr) return run_short_tc(l, st);
  return run_short_h<HD, 0>(l, st);
}

// Sequences longer than kAttnShortCap go to the tcgen05 kernel (their
// 128-row blocks are the prefix of the table), the rest to the short kernel.
template <int HD>
static cudaError_t run_split(const AttnLaunch& l, cudaStream_t st) {
  if (l.n_long > 0) {
    AttnLaunch lg = l;
    lg.nblocks128 = l.nblocks128_long;
    const cudaError_t e = run_fa_mode<HD>(lg, st);
    if (e != cudaSuccess) return e;
  }
  return l.nseq > l.n_long ? run_short_mode<HD>(l, st) : cudaSuccess;
}

cudaError_t launch_attention(const AttnLaunch& l, cudaStream_t st) {
  if (l.nblocks <= 0) return cudaSuccess;
  if (l.causal && l.relbias) return cudaErrorInvalidValue;
  if (getenv("EC_LEGACY_ATTN") != nullptr || !l.blocks128 || l.rows <= 0) {
    switch (l.head_dim) {
      case 32: return run_mode<32>(l, st);
      case 64: return run_mode<64>(l, st);
      case 128: return run_mode<128>(l, st);
      default: return cudaErrorInvalidValue;
    }
  }
  // head dims 32 / 64: sequences up to 256 tokens on the shared-memory
  // kernel (measured faster than tcgen05 tiles of 128 padded rows for
  // MiniLM / BERT-base / MPNet batches) unless EC_NO_SHORT_ATTN
  const bool split = l.seqs && getenv("EC_NO_SHORT_ATTN") == nullptr;
  switch (l.head_dim) {
    case 32: return split ? run_split<32>(l, st) : run_fa_mode<32>(l, st);
    case 64: return split ? run_split<64>(l, st) : run_fa_mode<64>(l, st);
    case 128: return run_fa_mode<128>(l, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ec
