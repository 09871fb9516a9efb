// ec_skinny.cu -- GEMMs of a few rows (a single query or a handful of short
// sequences): out[m, n] = epilogue(A[m, :] . W[n, :] + bias[n]) for M <=
// kSkinnyRows.  The tcgen05 GEMMs tile M by 128, so with ten rows they run
// on N / BN CTAs (two for the LayerNorm clusters) and each of those streams
// a whole W tile alone.  Here one warp owns one output column: its lanes
// stream that column's weight row in 16-byte pieces (coalesced), multiply
// them with the M input rows held in shared memory, accumulate in fp32 and
// reduce across the warp; N / 8 CTAs of eight warps spread the weights over
// the whole GPU.  Epilogues: bias -> bf16, bias + GELU (bert::gelu's
// A&S 7.1.26 erf) -> bf16, (acc + bias) + residual -> fp32 (the pre-norm
// row of bert.lisp:250-256 and :265-270, normalised by the LayerNorm row
// kernel).
#include <cuda_bf16.h>

#include "ec_gemm.cuh"
#include "ec_kernels.h"

namespace ec {

namespace {

__device__ __forceinline__ void bf8_to_f32(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
  }
}

// weight pieces (16 bytes) each lane loads ahead: K <= 32 * 8 * kSkChunks
// (1536) is covered by the prefetch
constexpr int kSkChunks = 6;

template <int EPI>
__global__ void __launch_bounds__(256) skinny_gemm_kernel(const SkinnyLaunch a) {
  extern __shared__ __align__(16) uint8_t sk_smem[];
  uint4* sA = reinterpret_cast<uint4*>(sk_smem);  // [M][K / 8]
  const int M = a.M, k8 = a.K / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const bool col = n < a.N;
  // this lane's first kSkChunks weight pieces, requested before the rows of
  // A (the previous kernel's output) are waited for and staged
  const uint4* wr = reinterpret_cast<const uint4*>(a.W + static_cast<size_t>(col ? n : 0) * a.K);
  uint4 wv[kSkChunks];
#pragma unroll
  for (int j = 0; j < kSkChunks; ++j) {
    const int c = lane + 32 * j;
    wv[j] = (col && c < k8) ? __ldg(wr + c) : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < M * k8; i += blockDim.x) {
    const int m = i / k8, c = i - m * k8;
    sA[i] = *reinterpret_cast<const uint4*>(a.A + static_cast<size_t>(m) * a.lda + c * 8);
  }
  __syncthreads();
  if (!col) return;
  float acc[kSkinnyRows];
#pragma unroll
  for (int m = 0; m < kSkinnyRows; ++m) acc[m] = 0.f;
  // the same order as one loop over c = lane, lane + 32, ...: the prefetched
  // pieces first, then the rest of the row
  auto piece = [&](const uint4 wq, int c) {
    float w[8];
    bf8_to_f32(wq, w);
#pragma unroll
    for (int m = 0; m < kSkinnyRows; ++m) {
      if (m < M) {
        float x[8];
        bf8_to_f32(sA[m * k8 + c], x);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[m] = fmaf(x[e], w[e], acc[m]);
      }
    }
  };
#pragma unroll
  for (int j = 0; j < kSkChunks; ++j)
    if (lane + 32 * j < k8) piece(wv[j], lane + 32 * j);
  for (int c = lane + 32 * kSkChunks; c < k8; c += 32) piece(wr[c], c);
  // every lane gets every row's total; lane m keeps row m
  float mine = 0.f;
#pragma unroll
  for (int m = 0; m < kSkinnyRows; ++m) {
    if (m < M) {
      float v = acc[m];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == m) mine = v;
    }
  }
  if (lane >= M) return;
  const float x = mine + (a.bias ? a.bias[n] : 0.f);
  if constexpr (EPI == kSkF32Resid) {
    const size_t r = static_cast<size_t>(lane) * a.ldr + n;
    const float res = a.resid ? a.resid[r] : __bfloat162float(a.resid_b[r]);
    static_cast<float*>(a.out)[static_cast<size_t>(lane) * a.ldo + n] = x + res;
  } else {
    const float y = EPI == kSkGelu ? gelu_as(x) : x;
    static_cast<__nv_bfloat16*>(a.out)[static_cast<size_t>(lane) * a.ldo + n] = __float2bfloat16_rn(y);
  }
}

template <int EPI>
cudaError_t run_skinny(const SkinnyLaunch& s, size_t smem, cudaStream_t st) {
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(skinny_gemm_kernel<EPI>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(skinny_gemm_kernel<EPI>, dim3(static_cast<unsigned>((s.N + 7) / 8)), dim3(256), smem, st,
                    s);
}

}  // namespace

cudaError_t launch_skinny_gemm(const SkinnyLaunch& s, cudaStream_t st) {
  if (s.M <= 0 || s.M > kSkinnyRows || s.N <= 0 || s.K <= 0 || s.K % 8 || s.lda % 8 || !s.A || !s.W ||
      !s.out)
    return cudaErrorInvalidValue;
  if (s.epi == kSkF32Resid && !s.resid && !s.resid_b) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(s.M) * s.K * 2;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  switch (s.epi) {
    case kSkBf16: return run_skinny<kSkBf16>(s, smem, st);
    case kSkGelu: return run_skinny<kSkGelu>(s, smem, st);
    case kSkF32Resid: return run_skinny<kSkF32Resid>(s, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ec
