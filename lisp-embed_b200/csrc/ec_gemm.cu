// ec_gemm.cu -- instantiations and host launcher of the tcgen05 GEMM.
#include <cudaTypedefs.h>

#include <mutex>

#include "ec_gemm.cuh"
#include "ec_kernels.h"

namespace ec {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 gemm_encode_fn() { return g_encode; }

bool gemm_init_driver() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

// 2D bf16 tensor map over rows x cols (cols contiguous), box = box_rows x 64
// columns (128 bytes), 128-byte swizzle.  Rows past `rows` read as zero.
static bool encode_2d_bf16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols,
                           uint64_t ld_elems, uint32_t box_rows) {
  if (!g_encode) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output map of the epilogue's bulk stores: 32 x 32 boxes, fp32 rows of
// 128 B with 128-byte swizzle or bf16 rows of 64 B with 64-byte swizzle (the
// layouts stage_off writes); rows past `rows` are not written.
static bool encode_2d_out(CUtensorMap* map, void* ptr, bool f32, uint64_t rows, uint64_t cols,
                          uint64_t ld_elems) {
  if (!g_encode) return false;
  const uint64_t es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * es};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int EPI>
static cudaError_t run(const GemmLaunch& g, cudaStream_t st, int num_sms) {
  using Cfg = GemmCfg<BN, EPI>;
  // the shared-memory opt-in is a per-device function attribute
  static std::mutex attr_mu;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(attr_mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gemm_tn_bf16_kernel<BN, EPI>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(Cfg::SMEM_BYTES));
      if (e != cudaSuccess) return e;
      attr_set[dev] = true;
    }
  }
  CUtensorMap ta, tb, tc;
  if (!encode_2d_bf16(&ta, g.A, g.M, g.K, g.lda, kGemmBM)) return cudaErrorInvalidValue;
  if (!encode_2d_bf16(&tb, g.W, g.N, g.K, g.ldw, BN)) return cudaErrorInvalidValue;
  const uint64_t out_cols = EPI == kEpiBf16Swiglu ? g.N / 2 : g.N;
  if (!encode_2d_out(&tc, g.out, Cfg::OUT_F32, g.M, out_cols, g.ldo)) return cudaErrorInvalidValue;
  GemmArgs a;
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.bias = g.bias;
  a.resid = g.resid;
  a.ldr = g.ldr;
  a.out = g.out;
  a.ldo = g.ldo;
  a.n_tiles_n = g.N / BN;
  a.num_tiles = ((g.M + kGemmBM - 1) / kGemmBM) * a.n_tiles_n;
  a.status = g.status;
  const int grid = a.num_tiles < num_sms ? a.num_tiles : num_sms;
  gemm_tn_bf16_kernel<BN, EPI><<<grid, kGemmThreads, Cfg::SMEM_BYTES, st>>>(ta, tb, tc, a);
  return cudaGetLastError();
}

template <int BN>
static cudaError_t dispatch_epi(const GemmLaunch& g, cudaStream_t st, int num_sms) {
  switch (g.epi) {
    case kEpiBf16: return run<BN, kEpiBf16>(g, st, num_sms);
    case kEpiBf16Gelu: return run<BN, kEpiBf16Gelu>(g, st, num_sms);
    case kEpiF32Resid: return run<BN, kEpiF32Resid>(g, st, num_sms);
    case kEpiF32: return run<BN, kEpiF32>(g, st, num_sms);
    case kEpiBf16Swiglu:
      if constexpr (BN == 128 || BN == 256) return run<BN, kEpiBf16Swiglu>(g, st, num_sms);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

int gemm_pick_bn(int M, int N, int epi, int num_sms) {
  if (epi == kEpiBf16Swiglu) return N % 256 == 0 ? 256 : (N % 128 == 0 ? 128 : 0);
  const int mt = (M + kGemmBM - 1) / kGemmBM;
  int best = 0;
  double best_cost = 1e300;
  const int cands[3] = {256, 192, 128};
  for (int bn : cands) {
    if (N % bn) continue;
    const long tiles = static_cast<long>(mt) * (N / bn);
    const long waves = (tiles + num_sms - 1) / num_sms;
    // time ~ waves * per-tile cost; per-tile cost ~ bn plus a fixed overhead
    // for the A tile (shared-memory bandwidth favours wide tiles)
    const double cost = static_cast<double>(waves) * (bn + 96);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = bn;
    }
  }
  if (!best && N % 64 == 0) best = 64;
  return best;
}

cudaError_t launch_gemm(const GemmLaunch& g, cudaStream_t st, int num_sms) {
  if (g.K % kGemmBK || g.M <= 0) return cudaErrorInvalidValue;
  const int bn = g.bn ? g.bn : gemm_pick_bn(g.M, g.N, g.epi, num_sms);
  if (!bn || g.N % bn) return cudaErrorInvalidValue;
  switch (bn) {
    case 256: return dispatch_epi<256>(g, st, num_sms);
    case 192: return dispatch_epi<192>(g, st, num_sms);
    case 128: return dispatch_epi<128>(g, st, num_sms);
    case 64: return dispatch_epi<64>(g, st, num_sms);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ec
