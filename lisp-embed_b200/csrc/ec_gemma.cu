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

__device__ __forceinline__ double sq4(float4 v) {
  return static_cast<double>(v.x * v.x) + static_cast<double>(v.y * v.y) +
         static_cast<double>(v.z * v.z) + static_cast<double>(v.w * v.w);
}

__device__ __forceinline__ uint2 bf16x4(float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

// h = sqrt(hidden) * embed[id] (gemma.lisp:326-330); also the bf16 copy that
// feeds every layer's per-layer-embedding projection (gemma.lisp:331-333).
// One warp per token, four columns per lane step (H % 128 == 0).
__global__ void gemma_embed_kernel(GemmaEmbedArgs a) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const size_t src = static_cast<size_t>(a.ids[t]) * a.H;
  float4* h4 = reinterpret_cast<float4*>(a.h32 + static_cast<size_t>(t) * a.H);
  uint2* hb4 = reinterpret_cast<uint2*>(a.h0b + static_cast<size_t>(t) * a.H);
  for (int i = lane; i < a.H / 4; i += 32) {
    float4 v;
    if (a.dtype == kDtBf16) {
      const uint2 r = reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.table) + src)[i];
      v = make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u),
                      __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xffff0000u));
    } else {
      v = reinterpret_cast<const float4*>(static_cast<const float*>(a.table) + src)[i];
    }
    v = make_float4(a.scale * v.x, a.scale * v.y, a.scale * v.z, a.scale * v.w);
    h4[i] = v;
    hb4[i] = bf16x4(v.x, v.y, v.z, v.w);
  }
}

// One warp per (token, head): q heads get RMSNorm(q_norm) + RoPE, k heads
// RMSNorm(k_norm) + RoPE, v heads the unscaled RMSNorm (gemma.lisp:236-247),
// in place on the packed bf16 QKV rows.  Lane l holds the element pairs
// (i, i + hd/2) for i in [l * E, l * E + E), E = hd / 64 (head dim 64..256).
template <int E>
__global__ void head_norm_rope_kernel(HeadNormRopeArgs a) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nh = a.q_heads + 2 * a.kv_heads;
  if (w >= a.T * nh) return;
  const int t = w / nh, hh = w % nh;
  constexpr int HD = 64 * E, HALF = 32 * E;
  const int kind = hh < a.q_heads ? 0 : (hh < a.q_heads + a.kv_heads ? 1 : 2);
  __nv_bfloat16* row = a.qkv + static_cast<size_t>(t) * a.ld + static_cast<size_t>(hh) * HD;
  float lo[E], hi[E];
  double ss = 0.0;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    lo[e] = __bfloat162float(row[lane * E + e]);
    hi[e] = __bfloat162float(row[HALF + lane * E + e]);
    ss += static_cast<double>(lo[e] * lo[e]) + static_cast<double>(hi[e] * hi[e]);
  }
  ss = warp_sum_dd(ss);
  const float inv = rms_inv(ss, HD, a.eps);
  const float* g = kind == 0 ? a.q_norm : (kind == 1 ? a.k_norm : nullptr);
  const int p = a.pos[t];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    float x = lo[e] * inv, y = hi[e] * inv;
    if (g) {
      x = x * g[i];
      y = y * g[i + HALF];
    }
    if (kind < 2) {
      // rotate-half RoPE at the token's position (gemma.lisp:105-119)
      const float c = a.cos_t[static_cast<size_t>(p) * HALF + i];
      const float s = a.sin_t[static_cast<size_t>(p) * HALF + i];
      const float nx = x * c - y * s, ny = x * s + y * c;
      x = nx;
      y = ny;
    }
    lo[e] = x;
    hi[e] = y;
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    row[lane * E + e] = __float2bfloat16_rn(lo[e]);
    row[HALF + lane * E + e] = __float2bfloat16_rn(hi[e]);
  }
}

// h = (h + RMSNorm(x, g1)) [* scalar]; then hb = bf16(RMSNorm(h, g2)) or
// bf16(h) when g2 is null (gemma.lisp:268-302).  One warp per token, four
// columns per lane step; the second and third passes re-read this warp's
// own rows, which are still in L1 / L2.
__global__ void norm_add_kernel(NormAddArgs a) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const int n4 = a.H / 4;
  const float4* x = reinterpret_cast<const float4*>(a.x + static_cast<size_t>(t) * a.H);
  float4* h = reinterpret_cast<float4*>(a.h32 + static_cast<size_t>(t) * a.H);
  const float4* g1 = reinterpret_cast<const float4*>(a.g1);
  double ss = 0.0;
#pragma unroll 4
  for (int i = lane; i < n4; i += 32) ss += sq4(x[i]);
  const float inv = rms_inv(warp_sum_dd(ss), a.H, a.eps);
  double ss2 = 0.0;
#pragma unroll 4
  for (int i = lane; i < n4; i += 32) {
    const float4 xv = x[i], gv = g1[i];
    float4 v = h[i];
    v.x = v.x + (xv.x * inv) * gv.x;
    v.y = v.y + (xv.y * inv) * gv.y;
    v.z = v.z + (xv.z * inv) * gv.z;
    v.w = v.w + (xv.w * inv) * gv.w;
    if (a.scale_h) v = make_float4(v.x * a.scalar, v.y * a.scalar, v.z * a.scalar, v.w * a.scalar);
    h[i] = v;
    ss2 += sq4(v);
  }
  if (!a.outb) return;
  uint2* ob = reinterpret_cast<uint2*>(a.outb + static_cast<size_t>(t) * a.H);
  if (!a.g2) {
#pragma unroll 4
    for (int i = lane; i < n4; i += 32) {
      const float4 v = h[i];
      ob[i] = bf16x4(v.x, v.y, v.z, v.w);
    }
    return;
  }
  const float inv2 = rms_inv(warp_sum_dd(ss2), a.H, a.eps);
  const float4* g2 = reinterpret_cast<const float4*>(a.g2);
#pragma unroll 4
  for (int i = lane; i < n4; i += 32) {
    const float4 v = h[i], gv = g2[i];
    ob[i] = bf16x4((v.x * inv2) * gv.x, (v.y * inv2) * gv.y, (v.z * inv2) * gv.z,
                   (v.w * inv2) * gv.w);
  }
}

// this layer's per-layer embedding: x = x * (1 / sqrt(hidden)), then
// RMSNorm(per_layer_projection_norm) over the P values (gemma.lisp:334-343)
__global__ void ple_prep_kernel(PlePrepArgs a) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= a.T) return;
  const int n4 = a.P / 4;
  float4* x = reinterpret_cast<float4*>(a.x + static_cast<size_t>(t) * a.P);
  const float4* g = reinterpret_cast<const float4*>(a.g);
  const float s = a.inv_sqrt_h;
  double ss = 0.0;
#pragma unroll 4
  for (int i = lane; i < n4; i += 32) {
    float4 v = x[i];
    v = make_float4(v.x * s, v.y * s, v.z * s, v.w * s);
    ss += sq4(v);
  }
  const float inv = rms_inv(warp_sum_dd(ss), a.P, a.eps);
#pragma unroll 4
  for (int i = lane; i < n4; i += 32) {
    float4 v = x[i];
    const float4 gv = g[i];
    v = make_float4(((v.x * s) * inv) * gv.x, ((v.y * s) * inv) * gv.y, ((v.z * s) * inv) * gv.z,
                    ((v.w * s) * inv) * gv.w);
    x[i] = v;
  }
}

// gelu-tanh(gate(h)) * per-layer embedding, to bf16 for the PLE projection
// (gemma.lisp:290-293); four elements per thread step
__global__ void ple_gate_kernel(PleGateArgs a) {
  const size_t n4 = static_cast<size_t>(a.T) * a.P / 4;
  const float4* g4 = reinterpret_cast<const float4*>(a.gate);
  const float4* p4 = reinterpret_cast<const float4*>(a.ple);
  uint2* o4 = reinterpret_cast<uint2*>(a.outb);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float4 g = g4[i], p = p4[i];
    o4[i] = bf16x4(gelu_tanh_f(g.x) * p.x, gelu_tanh_f(g.y) * p.y, gelu_tanh_f(g.z) * p.z,
                   gelu_tanh_f(g.w) * p.w);
  }
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
  const size_t rows = static_cast<size_t>(a.T) * (a.q_heads + 2 * a.kv_heads);
  switch (a.hd) {
    case 64: head_norm_rope_kernel<1><<<warps_grid(rows), 256, 0, st>>>(a); break;
    case 128: head_norm_rope_kernel<2><<<warps_grid(rows), 256, 0, st>>>(a); break;
    case 256: head_norm_rope_kernel<4><<<warps_grid(rows), 256, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
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
  if (a.P % 4) return cudaErrorInvalidValue;
  const size_t n = static_cast<size_t>(a.T) * a.P / 4;
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
