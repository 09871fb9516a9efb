// ec_gemm.cu -- instantiations and host launcher of the tcgen05 GEMM.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "ec_gemm.cuh"
#include "ec_gemm_ln.cuh"
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

template <int BN, int EPI, int CG = 1, bool WR = false>
static cudaError_t run(const GemmLaunch& g, cudaStream_t st, int num_sms) {
  using Cfg = GemmCfg<BN, EPI, CG, WR>;
  if (WR && g.K > kGemmWrMaxK) return cudaErrorInvalidValue;
  // the shared-memory opt-in is a per-device function attribute; pairs also
  // need the number of clusters that fit at once
  static std::mutex attr_mu;
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    std::lock_guard<std::mutex> lk(attr_mu);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!max_clusters[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gemm_tn_bf16_kernel<BN, EPI, CG, WR>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(Cfg::SMEM_BYTES));
      if (e != cudaSuccess) return e;
      int n = num_sms;
      if constexpr (CG == 2) {
        cfg.gridDim = dim3((num_sms / 2) * 2, 1, 1);
        e = cudaOccupancyMaxActiveClusters(&n, gemm_tn_bf16_kernel<BN, EPI, CG, WR>, &cfg);
        if (e != cudaSuccess) return e;
        if (n <= 0) return cudaErrorInvalidConfiguration;
      }
      max_clusters[dev] = n;
    }
  }
  CUtensorMap ta, tb, tc;
  if (!encode_2d_bf16(&ta, g.A, g.M, g.K, g.lda, kGemmBM)) return cudaErrorInvalidValue;
  if (!encode_2d_bf16(&tb, g.W, g.N, g.K, g.ldw, BN / CG)) return cudaErrorInvalidValue;
  const uint64_t out_cols = (EPI == kEpiBf16Swiglu || EPI == kEpiBf16GeluTanhGate) ? g.N / 2 : g.N;
  if constexpr (EPI == kEpiArgCand) {
    // no dense output: the map is never used (any valid encoding will do)
    if (!g.ac || !encode_2d_out(&tc, g.ac->mloc, true, 32, 32, 32)) return cudaErrorInvalidValue;
  } else if (!encode_2d_out(&tc, g.out, Cfg::OUT_F32, g.M, out_cols, g.ldo)) {
    return cudaErrorInvalidValue;
  }
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
  a.num_tiles = ((g.M + kGemmBM * CG - 1) / (kGemmBM * CG)) * a.n_tiles_n;
  a.status = g.status;
  a.qk = QkRopeEpi{};
  a.ac = ArgCandEpi{};
  if constexpr (EPI == kEpiArgCand) a.ac = *g.ac;
  if constexpr (EPI == kEpiF32Resid || EPI == kEpiBf16GeluTanhMul) {
    // the epilogue reads 16-byte pieces of the residual / multiplier rows
    if (!g.resid || g.ldr % 4 || reinterpret_cast<uintptr_t>(g.resid) % 16)
      return cudaErrorInvalidValue;
  }
  if constexpr (EPI == kEpiBf16QkRope) {
    if (!g.qk) return cudaErrorInvalidValue;
    a.qk = *g.qk;
  }
  if constexpr (WR) {
    // every unit (CTA, or pair) keeps one W tile resident: all units run,
    // in groups of n_tiles_n that share row blocks
    const int units = CG == 2 ? max_clusters[dev] : num_sms;
    if (units < a.n_tiles_n) return cudaErrorInvalidConfiguration;
    if constexpr (CG == 1) {
      gemm_tn_bf16_kernel<BN, EPI, CG, WR><<<units, kGemmThreads, Cfg::SMEM_BYTES, st>>>(ta, tb, tc, a);
      return cudaGetLastError();
    } else {
      cfg.gridDim = dim3(units * 2, 1, 1);
      return cudaLaunchKernelEx(&cfg, gemm_tn_bf16_kernel<BN, EPI, CG, WR>, ta, tb, tc, a);
    }
  }
  if constexpr (CG == 1) {
    const int grid = a.num_tiles < num_sms ? a.num_tiles : num_sms;
    gemm_tn_bf16_kernel<BN, EPI, CG, WR><<<grid, kGemmThreads, Cfg::SMEM_BYTES, st>>>(ta, tb, tc, a);
    return cudaGetLastError();
  } else {
    const int clusters = a.num_tiles < max_clusters[dev] ? a.num_tiles : max_clusters[dev];
    cfg.gridDim = dim3(clusters * 2, 1, 1);
    return cudaLaunchKernelEx(&cfg, gemm_tn_bf16_kernel<BN, EPI, CG, WR>, ta, tb, tc, a);
  }
}

template <int BN>
static cudaError_t dispatch_epi(const GemmLaunch& g, cudaStream_t st, int num_sms) {
  switch (g.epi) {
    case kEpiBf16: return run<BN, kEpiBf16>(g, st, num_sms);
    case kEpiBf16Gelu: return run<BN, kEpiBf16Gelu>(g, st, num_sms);
    case kEpiF32Resid: return run<BN, kEpiF32Resid>(g, st, num_sms);
    case kEpiF32: return run<BN, kEpiF32>(g, st, num_sms);
    case kEpiBf16QkRope:
      if constexpr (BN == 256) return run<BN, kEpiBf16QkRope>(g, st, num_sms);
      return cudaErrorInvalidValue;
    case kEpiBf16GeluTanhGate:
      if constexpr (BN == 128 || BN == 256) return run<BN, kEpiBf16GeluTanhGate>(g, st, num_sms);
      return cudaErrorInvalidValue;
    case kEpiBf16GeluTanhMul:
      if constexpr (BN == 128 || BN == 256) return run<BN, kEpiBf16GeluTanhMul>(g, st, num_sms);
      return cudaErrorInvalidValue;
    case kEpiArgCand:
      if constexpr (BN == 128 || BN == 256) return run<BN, kEpiArgCand>(g, st, num_sms);
      return cudaErrorInvalidValue;
    case kEpiBf16Swiglu:
      if constexpr (BN == 128 || BN == 256) return run<BN, kEpiBf16Swiglu>(g, st, num_sms);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

int gemm_pick_bn(int M, int N, int epi, int num_sms) {
  if (epi == kEpiBf16Swiglu || epi == kEpiBf16GeluTanhGate || epi == kEpiBf16GeluTanhMul ||
      epi == kEpiArgCand)
    return N % 256 == 0 ? 256 : (N % 128 == 0 ? 128 : 0);
  if (epi == kEpiBf16QkRope) return N % 256 == 0 ? 256 : 0;
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
  // CTA pairs (256 x 256 tiles, each CTA loads half of the W tile) where the
  // mainloop dominates: K >= 768 and epilogues lighter than GELU (measured:
  // 8-12% faster there, neutral or slower at K = 384 or with GELU).
  // EC_GEMM_PAIR forces pairs for every eligible shape, EC_NO_GEMM_PAIR none.
  // EC_GEMM_WR: K <= 384 with the plain / GELU epilogues (QKV, FFN-up of
  // the small encoders) on weight-resident CTA pairs (each pair keeps one W
  // tile in shared memory and streams only A).  Opt-in: on the MiniLM
  // forward it measured 4% slower than the streaming schedule.
  if (!g.bn && g.K <= kGemmWrMaxK && (g.epi == kEpiBf16 || g.epi == kEpiBf16Gelu) &&
      getenv("EC_GEMM_WR") != nullptr && getenv("EC_NO_GEMM_WR") == nullptr) {
    cudaError_t e = cudaErrorInvalidConfiguration;
    if (g.N % 256 == 0)
      e = g.epi == kEpiBf16 ? run<256, kEpiBf16, 2, true>(g, st, num_sms)
                            : run<256, kEpiBf16Gelu, 2, true>(g, st, num_sms);
    else if (g.N % 192 == 0)
      e = g.epi == kEpiBf16 ? run<192, kEpiBf16, 2, true>(g, st, num_sms)
                            : run<192, kEpiBf16Gelu, 2, true>(g, st, num_sms);
    if (e != cudaErrorInvalidConfiguration) return e;
    cudaGetLastError();  // fewer units than W tiles: the streaming schedule below
  }
  const bool force_pair = getenv("EC_GEMM_PAIR") != nullptr;
  if (!g.bn && g.N % 256 == 0 && getenv("EC_NO_GEMM_PAIR") == nullptr &&
      (force_pair || (g.K >= 768 && g.epi != kEpiBf16Gelu))) {
    switch (g.epi) {
      case kEpiBf16: return run<256, kEpiBf16, 2>(g, st, num_sms);
      case kEpiBf16Gelu: return run<256, kEpiBf16Gelu, 2>(g, st, num_sms);
      case kEpiF32Resid: return run<256, kEpiF32Resid, 2>(g, st, num_sms);
      case kEpiF32: return run<256, kEpiF32, 2>(g, st, num_sms);
      case kEpiBf16Swiglu: return run<256, kEpiBf16Swiglu, 2>(g, st, num_sms);
      case kEpiBf16GeluTanhGate: return run<256, kEpiBf16GeluTanhGate, 2>(g, st, num_sms);
      case kEpiBf16QkRope: return run<256, kEpiBf16QkRope, 2>(g, st, num_sms);
      default: break;
    }
  }
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

// ---------------------------------------------------------------------------
// GEMM + residual + LayerNorm on clusters of C CTAs (one column slice each)
template <int BN, int C, bool RB, int NM = kNormLayer>
static cudaError_t run_ln(const GemmLnLaunch& g, cudaStream_t st, int num_sms) {
  using Cfg = GemmLnCfg<BN, C, RB, NM>;
  static std::mutex mu;
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!max_clusters[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gemm_ln_kernel<BN, C, RB, NM>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(Cfg::SMEM_BYTES));
      if (e != cudaSuccess) return e;
      // clusters that fit at once (GPC boundaries leave some SMs idle)
      cfg.gridDim = dim3((num_sms / C) * C, 1, 1);
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, gemm_ln_kernel<BN, C, RB, NM>, &cfg);
      if (e != cudaSuccess) return e;
      if (n <= 0) return cudaErrorInvalidConfiguration;
      max_clusters[dev] = n;
    }
  }
  CUtensorMap ta, tb, t32, tbf, tr;
  if (!encode_2d_bf16(&ta, g.A, g.M, g.K, g.lda, kGemmBM)) return cudaErrorInvalidValue;
  if (!encode_2d_bf16(&tb, g.W, g.N, g.K, g.K, BN)) return cudaErrorInvalidValue;
  // a map that is never used (no such output / residual) borrows a valid one
  if (g.outb && !encode_2d_out(&tbf, g.outb, false, g.M, g.N, g.N)) return cudaErrorInvalidValue;
  if (g.out32 && !encode_2d_out(&t32, g.out32, true, g.M, g.N, g.N)) return cudaErrorInvalidValue;
  if (!g.outb) tbf = t32;
  if (!g.out32) t32 = tbf;
  // the residual is read with the matching output's box and swizzle (rows
  // past M read as zero)
  if (RB) {
    if (!encode_2d_out(&tr, const_cast<__nv_bfloat16*>(g.resid_b), false, g.M, g.N, g.N))
      return cudaErrorInvalidValue;
  } else if (g.resid) {
    if (!encode_2d_out(&tr, const_cast<float*>(g.resid), true, g.M, g.N, g.N))
      return cudaErrorInvalidValue;
  } else {
    tr = t32;
  }
  GemmLnArgs a;
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.bias = g.bias;
  a.out32 = g.out32 ? 1 : 0;
  a.outb = g.outb ? 1 : 0;
  a.eps = g.eps;
  a.scale = g.scale;
  a.has_scale = g.has_scale;
  a.ln_g = g.ln_g;
  a.ln_b = g.ln_b;
  a.m_tiles = (g.M + kGemmBM - 1) / kGemmBM;
  a.status = g.status;
  const int clusters = a.m_tiles < max_clusters[dev] ? a.m_tiles : max_clusters[dev];
  cfg.gridDim = dim3(clusters * C, 1, 1);
  return cudaLaunchKernelEx(&cfg, gemm_ln_kernel<BN, C, RB, NM>, ta, tb, t32, tbf, tr, a);
}

bool gemm_ln_supported(int N) { return N == 384 || N == 768 || N == 1024; }
bool gemm_rms_supported(int N) { return N == 512 || N == 768 || N == 1024; }

template <int NM>
static cudaError_t launch_rms(const GemmLnLaunch& g, cudaStream_t st, int num_sms) {
  switch (g.N) {
    case 512: return run_ln<256, 2, false, NM>(g, st, num_sms);
    case 768: return run_ln<192, 4, false, NM>(g, st, num_sms);
    case 1024: return run_ln<256, 4, false, NM>(g, st, num_sms);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm_ln(const GemmLnLaunch& g, cudaStream_t st, int num_sms) {
  if (g.K % kGemmBK || g.M <= 0 || !g.ln_g) return cudaErrorInvalidValue;
  if (g.mode != kNormLayer) {
    if (g.resid_b || !(g.out32 || g.outb)) return cudaErrorInvalidValue;
    switch (g.mode) {
      case kNormResRms:
        if (!g.resid || !g.out32 || !g.outb) return cudaErrorInvalidValue;
        return launch_rms<kNormResRms>(g, st, num_sms);
      case kNormPostAdd:
        if (!g.resid || !g.out32) return cudaErrorInvalidValue;
        return launch_rms<kNormPostAdd>(g, st, num_sms);
      case kNormScaled:
        if (g.resid || !g.out32) return cudaErrorInvalidValue;
        return launch_rms<kNormScaled>(g, st, num_sms);
      default: return cudaErrorInvalidValue;
    }
  }
  if (!(g.resid || g.resid_b) || !g.ln_b || !g.outb) return cudaErrorInvalidValue;
  const bool rb = g.resid_b != nullptr;
  switch (g.N) {
    case 384: return rb ? run_ln<192, 2, true>(g, st, num_sms) : run_ln<192, 2, false>(g, st, num_sms);
    case 768: return rb ? run_ln<192, 4, true>(g, st, num_sms) : run_ln<192, 4, false>(g, st, num_sms);
    case 1024: return rb ? run_ln<256, 4, true>(g, st, num_sms) : run_ln<256, 4, false>(g, st, num_sms);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ec
