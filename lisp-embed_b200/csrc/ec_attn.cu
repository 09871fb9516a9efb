// ec_attn.cu -- instantiations and host launcher of the varlen attention.
#include <cstdlib>
#include <mutex>

#include "ec_attn.cuh"
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

template <int HD>
static cudaError_t run_mode(const AttnLaunch& l, cudaStream_t st) {
  if (l.causal) return run_attn<HD, 2>(l, st);
  if (l.relbias) return run_attn<HD, 1>(l, st);
  return run_attn<HD, 0>(l, st);
}

cudaError_t launch_attention(const AttnLaunch& l, cudaStream_t st) {
  if (l.nblocks <= 0) return cudaSuccess;
  if (l.causal && l.relbias) return cudaErrorInvalidValue;
  switch (l.head_dim) {
    case 32: return run_mode<32>(l, st);
    case 64: return run_mode<64>(l, st);
    case 128: return run_mode<128>(l, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ec
