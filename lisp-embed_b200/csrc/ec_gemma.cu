// ec_gemma.cu -- row kernels of the EmbeddingGemma / Gemma-3n text forward
// (gemma.lisp): scaled embedding gather, per-head q/k/v RMSNorm + RoPE,
// post-norm residual adds, per-layer-embedding (PLE) preparation and gating,
// and the final mean pool + 512 -> 768 projection + L2.  One warp per row
// (token or token-head) unless stated; norms accumulate the sum of squares in
// double as gemma::rmsnorm does (gemma.lisp:62-83).
#include <cuda_bf16.h>

#include "ec_kernels.h"

namespace ec {

namespace {

__device__ __forceinline__ double warp_sum_dd(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// inv = 1 / sqrt(ss / n + eps) in double, rounded to single (gemma.lisp:70)
__device__ __forceinline__ float rms_inv(double ss, int n, double eps) {
  return static_cast<float>(1.0 / sqrt(ss / static_cast<double>(n) + eps));
}

// gemma::gelu-tanh (gemma.lisp:85-89) in single precision
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float c = 0.7978845608028654f * (x + ((0.044715f * x) * x) * x);
  return (0.5f * x) * (1.0f + tanhf(c));
}

__device__ __forceinline__ float ld_elem(const void* base, int dtype, size_t i) {
  if (dtype == kDtBf16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
  return static_cast<const float*>(base)[i];
}

// h = sqrt(hidden) * embed[id] (gemma.lisp:326-330); also the bf16 copy that
// feeds every layer's per-layer-embedding projection (gemma.lisp:331-333)
__global__ void gemma_embed_kernel(GemmaEmbedArgs a) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const size_t src = static_cast<size_t>(a.ids[t]) * a.H;
  for (int i = lane; i < a.H; i += 32) {
    const float v = a.scale * ld_elem(a.table, a.dtype, src + i);
    a.h32[static_cast<size_t>(t) * a.H + i] = v;
    a.h0b[static_cast<size_t>(t) * a.H + i] = __float2bfloat16_rn(v);
  }
}

// One warp per (token, head): q heads get RMSNorm(q_norm) + RoPE, k heads
// RMSNorm(k_norm) + RoPE, v heads the unscaled RMSNorm (gemma.lisp:236-247),
// in place on the packed bf16 QKV rows.  Head dim <= 256.
__global__ void head_norm_rope_kernel(HeadNormRopeArgs a) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nh = a.q_heads + 2 * a.kv_heads;
  if (w >= a.T * nh) return;
  const int t = w / nh, hh = w % nh;
  const int hd = a.hd, half = hd / 2;
  const int kind = hh < a.q_heads ? 0 : (hh < a.q_heads + a.kv_heads ? 1 : 2);
  __nv_bfloat16* row = a.qkv + static_cast<size_t>(t) * a.ld + static_cast<size_t>(hh) * hd;
  // lane holds pairs (i, i + half) for i = lane + 32 j < half
  float lo[4], hi[4];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j;
    lo[j] = hi[j] = 0.f;
    if (i < half) {
      lo[j] = __bfloat162float(row[i]);
      hi[j] = __bfloat162float(row[i + half]);
      ss += static_cast<double>(lo[j] * lo[j]) + static_cast<double>(hi[j] * hi[j]);
    }
  }
  ss = warp_sum_dd(ss);
  const float inv = rms_inv(ss, hd, a.eps);
  const float* g = kind == 0 ? a.q_norm : (kind == 1 ? a.k_norm : nullptr);
  const int p = a.pos[t];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j;
    if (i >= half) continue;
    float x = lo[j] * inv, y = hi[j] * inv;
    if (g) {
      x = x * g[i];
      y = y * g[i + half];
    }
    if (kind < 2) {
      // rotate-half RoPE at the token's position (gemma.lisp:105-119)
      const float c = a.cos_t[static_cast<size_t>(p) * half + i];
      const float s = a.sin_t[static_cast<size_t>(p) * half + i];
      const float nx = x * c - y * s, ny = x * s + y * c;
      x = nx;
      y = ny;
    }
    row[i] = __float2bfloat16_rn(x);
    row[i + half] = __float2bfloat16_rn(y);
  }
}

// h = (h + RMSNorm(x, g1)) [* scalar]; then hb = bf16(RMSNorm(h, g2)) or
// bf16(h) when g2 is null (gemma.lisp:268-302)
__global__ void norm_add_kernel(NormAddArgs a) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const float* x = a.x + static_cast<size_t>(t) * a.H;
  float* h = a.h32 + static_cast<size_t>(t) * a.H;
  double ss = 0.0;
  for (int i = lane; i < a.H; i += 32) ss += static_cast<double>(x[i] * x[i]);
  const float inv = rms_inv(warp_sum_dd(ss), a.H, a.eps);
  double ss2 = 0.0;
  for (int i = lane; i < a.H; i += 32) {
    float v = h[i] + (x[i] * inv) * a.g1[i];
    if (a.scale_h) v = v * a.scalar;
    h[i] = v;
    ss2 += static_cast<double>(v * v);
  }
  if (!a.outb) return;
  if (!a.g2) {
    for (int i = lane; i < a.H; i += 32)
      a.outb[static_cast<size_t>(t) * a.H + i] = __float2bfloat16_rn(h[i]);
    return;
  }
  const float inv2 = rms_inv(warp_sum_dd(ss2), a.H, a.eps);
  for (int i = lane; i < a.H; i += 32)
    a.outb[static_cast<size_t>(t) * a.H + i] = __float2bfloat16_rn((h[i] * inv2) * a.g2[i]);
}

// this layer's per-layer embedding: x = x * (1 / sqrt(hidden)), then
// RMSNorm(per_layer_projection_norm) over the P values (gemma.lisp:334-343)
__global__ void ple_prep_kernel(PlePrepArgs a) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  float* x = a.x + static_cast<size_t>(t) * a.P;
  double ss = 0.0;
  for (int i = lane; i < a.P; i += 32) {
    const float v = x[i] * a.inv_sqrt_h;
    x[i] = v;
    ss += static_cast<double>(v * v);
  }
  const float inv = rms_inv(warp_sum_dd(ss), a.P, a.eps);
  for (int i = lane; i < a.P; i += 32) x[i] = (x[i] * inv) * a.g[i];
}

// gelu-tanh(gate(h)) * per-layer embedding, to bf16 for the PLE projection
// (gemma.lisp:290-293)
__global__ void ple_gate_kernel(PleGateArgs a) {
  const size_t n = static_cast<size_t>(a.T) * a.P;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    a.outb[i] = __float2bfloat16_rn(gelu_tanh_f(a.gate[i]) * a.ple[i]);
}

// One CTA per sequence: mean over tokens in order (gemma.lisp:366-370),
// projection by embedding_projection with sequential dot products
// (:371), L2 normalisation (:372-376).
__global__ void gemma_pool_kernel(GemmaPoolArgs a) {
  extern __shared__ float gp_smem[];
  float* pooled = gp_smem;            // [H]
  float* proj = gp_smem + a.H;        // [out_dim]
  const int s = blockIdx.x;
  const int base = a.cu[s], L = a.cu[s + 1] - base;
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < L; ++t) acc = acc + a.h[static_cast<size_t>(base + t) * a.H + i];
    pooled[i] = acc / static_cast<float>(L);
  }
  __syncthreads();
  for (int o = threadIdx.x; o < a.out_dim; o += blockDim.x) {
    const float* w = a.w_out + static_cast<size_t>(o) * a.H;
    float acc = 0.f;
    for (int i = 0; i < a.H; ++i) acc = acc + pooled[i] * w[i];
    proj[o] = acc;
  }
  __syncthreads();
  __shared__ float norm;
  if (threadIdx.x == 0) {
    float n2 = 0.f;
    for (int o = 0; o < a.out_dim; ++o) n2 = n2 + proj[o] * proj[o];
    norm = static_cast<float>(sqrt(static_cast<double>(n2)));
  }
  __syncthreads();
  for (int o = threadIdx.x; o < a.out_dim; o += blockDim.x)
    a.out[static_cast<size_t>(s) * a.out_stride + o] = proj[o] / norm;
}

int warps_grid(size_t rows) { return static_cast<int>((rows + 7) / 8); }

}  // namespace

cudaError_t launch_gemma_embed(const GemmaEmbedArgs& a, cudaStream_t st) {
  gemma_embed_kernel<<<warps_grid(a.T), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_head_norm_rope(const HeadNormRopeArgs& a, cudaStream_t st) {
  if (a.hd > 256 || a.hd % 2) return cudaErrorInvalidValue;
  const size_t rows = static_cast<size_t>(a.T) * (a.q_heads + 2 * a.kv_heads);
  head_norm_rope_kernel<<<warps_grid(rows), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_norm_add(const NormAddArgs& a, cudaStream_t st) {
  norm_add_kernel<<<warps_grid(a.T), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ple_prep(const PlePrepArgs& a, cudaStream_t st) {
  ple_prep_kernel<<<warps_grid(a.T), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_ple_gate(const PleGateArgs& a, cudaStream_t st) {
  const size_t n = static_cast<size_t>(a.T) * a.P;
  size_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  ple_gate_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_gemma_pool(const GemmaPoolArgs& a, int nseq, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(a.H + a.out_dim) * 4;
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  gemma_pool_kernel<<<nseq, 256, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace ec
