// ec_attn.cu -- instantiations and host launcher of the varlen attention.
#include <cstdlib>
#include <mutex>

#include <cudaTypedefs.h>

#include "ec_attn.cuh"
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
  a.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
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
  a.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
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

cudaError_t launch_attention(const AttnLaunch& l, cudaStream_t st) {
  if (l.nblocks <= 0) return cudaSuccess;
  if (l.causal && l.relbias) return cudaErrorInvalidValue;
  const bool legacy = getenv("EC_LEGACY_ATTN") != nullptr || !l.blocks128 || l.rows <= 0;
  switch (l.head_dim) {
    // head dim 32: the mma.sync kernel unless EC_TC_ATTN32 asks for tcgen05
    case 32: return (legacy || !getenv("EC_TC_ATTN32")) ? run_mode<32>(l, st) : run_fa_mode<32>(l, st);
    case 64: return legacy ? run_mode<64>(l, st) : run_fa_mode<64>(l, st);
    case 128: return legacy ? run_mode<128>(l, st) : run_fa_mode<128>(l, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ec
