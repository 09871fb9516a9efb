// ec_mlp.cu -- host launcher of the fused feed-forward block (ec_mlp.cuh).
#include <cudaTypedefs.h>

#include <mutex>

#include "ec_kernels.h"
#include "ec_mlp.cuh"

namespace ec {

PFN_cuTensorMapEncodeTiled_v12000 gemm_encode_fn();  // ec_gemm.cu

static bool enc(CUtensorMap* m, CUtensorMapDataType dt, const void* p, uint64_t rows,
                uint64_t cols, uint64_t ld_bytes, uint32_t box_c, uint32_t box_r,
                CUtensorMapSwizzle sw) {
  auto fn = gemm_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_c, box_r};
  cuuint32_t es[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(p), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int H>
static cudaError_t run(const MlpLaunch& l, cudaStream_t st, int num_sms) {
  using Cfg = MlpCfg<H>;
  // clusters of two CTAs (one CTA per SM): as many as fit at once
  static std::mutex mu;
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kMlpThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!max_clusters[dev]) {
      cudaError_t e = cudaFuncSetAttribute(mlp_fused_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(Cfg::SMEM_BYTES));
      if (e != cudaSuccess) return e;
      int n = 0;
      cfg.gridDim = dim3((num_sms / 2) * 2, 1, 1);
      e = cudaOccupancyMaxActiveClusters(&n, mlp_fused_kernel<H>, &cfg);
      if (e != cudaSuccess) return e;
      if (n <= 0) return cudaErrorInvalidConfiguration;
      max_clusters[dev] = n;
    }
  }
  CUtensorMap tx, tw1, tw2, to32, tob;
  const auto BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  // X: 128-row boxes of 64 columns; W1: this CTA's 32 rows of a 64-row
  // slice; W2: this CTA's half of a column part of H
  float* o32 = l.out32 ? l.out32 : reinterpret_cast<float*>(l.outb);  // unused map when absent
  if (!enc(&tx, BF, l.A, l.M, H, H * 2ull, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !enc(&tw1, BF, l.W1, l.F, H, H * 2ull, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !enc(&tw2, BF, l.W2, H, l.F, l.F * 2ull, 64, Cfg::NPW / 2, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !enc(&to32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, o32, l.M, l.out32 ? H : H / 2, l.out32 ? H * 4ull : H * 2ull,
           32, 32, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !enc(&tob, BF, l.outb, l.M, H, H * 2ull, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  MlpArgs a;
  a.M = l.M;
  a.F = l.F;
  a.b1 = l.b1;
  a.b2 = l.b2;
  a.resid = l.resid;
  a.resid_b = l.A;
  a.ln_g = l.ln_g;
  a.ln_b = l.ln_b;
  a.out32 = l.out32 != nullptr;
  a.num_tiles = (l.M + 255) / 256;
  a.status = l.status;
  const int clusters = a.num_tiles < max_clusters[dev] ? a.num_tiles : max_clusters[dev];
  cfg.gridDim = dim3(clusters * 2, 1, 1);
  return cudaLaunchKernelEx(&cfg, mlp_fused_kernel<H>, tx, tw1, tw2, to32, tob, a);
}

bool mlp_supported(int H, int F) { return (H == 384 || H == 256 || H == 128) && F % 128 == 0; }

cudaError_t launch_mlp(const MlpLaunch& l, cudaStream_t st, int num_sms) {
  if (l.M <= 0 || l.F % 128 || !l.A || !l.outb) return cudaErrorInvalidValue;
  switch (l.H) {
    case 384: return run<384>(l, st, num_sms);
    case 256: return run<256>(l, st, num_sms);
    case 128: return run<128>(l, st, num_sms);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ec
