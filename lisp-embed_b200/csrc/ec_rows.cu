// ec_rows.cu -- row-wise HBM-bound kernels of the encoder forward:
// embedding gather + LayerNorm, LayerNorm, RMSNorm, Qwen3 q/k RMSNorm + RoPE,
// pooling + L2, and the dtype conversions of weight upload.  One warp per
// row, 16-byte vector loads, warp-shuffle reductions.
#include "ec_kernels.h"
#include "ec_ln.cuh"
#include "ec_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <float.h>

namespace ec {

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 ld_row4(const void* base, int dtype, size_t idx4) {
  if (dtype == kDtBf16) {
    const uint2 u = reinterpret_cast<const uint2*>(base)[idx4];
    __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    return make_float4(__bfloat162float(a.x), __bfloat162float(a.y), __bfloat162float(b.x),
                       __bfloat162float(b.y));
  }
  return reinterpret_cast<const float4*>(base)[idx4];
}

// Embedding gather (word + position [+ token type 0]) then LayerNorm:
// bert.lisp:290-298 (type row 0), bert.lisp:473-479 (MPNet, no type).
template <int NV>
__global__ void embed_ln_kernel(EmbedLnArgs a) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.T) return;
  const int id = a.ids[warp];
  const int pos = a.pos[warp] + a.pos_offset;
  const int H4 = a.H / 4;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c4 = i * 32 + lane;
    const float4 w = ld_row4(a.word, a.word_dtype, static_cast<size_t>(id) * H4 + c4);
    const float4 p = ld_row4(a.posemb, a.pos_dtype, static_cast<size_t>(pos) * H4 + c4);
    float4 s = make_float4(w.x + p.x, w.y + p.y, w.z + p.z, w.w + p.w);
    if (a.type0) {
      const float4 t = ld_row4(a.type0, a.type_dtype, c4);
      s = make_float4(s.x + t.x, s.y + t.y, s.z + t.z, s.w + t.w);
    }
    v[i] = s;
  }
  ln_finish<NV>(v, a.H, a.g, a.b, a.out32 ? a.out32 + static_cast<size_t>(warp) * a.H : nullptr,
                a.outb + static_cast<size_t>(warp) * a.H, lane);
}

// Plain LayerNorm of an fp32 row (residual already added by the GEMM).
template <int NV>
__global__ void ln_kernel(LnArgs a) {
  pdl_trigger();
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.T) return;
  const float4* x = reinterpret_cast<const float4*>(a.x + static_cast<size_t>(warp) * a.H);
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = x[i * 32 + lane];
  ln_finish<NV>(v, a.H, a.g, a.b, a.out32 ? a.out32 + static_cast<size_t>(warp) * a.H : nullptr,
                a.outb + static_cast<size_t>(warp) * a.H, lane);
}

// llama::rmsnorm (llama.lisp:106-117): sum of squares accumulated in double,
// inv = 1 / sqrt(ss / n + eps) in double, y = (x * inv) * g.
template <int NV>
__global__ void rmsnorm_kernel(RmsArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= a.T) return;
  const size_t row = a.rows ? static_cast<size_t>(a.rows[warp]) : static_cast<size_t>(warp);
  const float4* x = reinterpret_cast<const float4*>(a.x + row * a.H);
  float4 v[NV];
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = x[i * 32 + lane];
    ss += static_cast<double>(v[i].x * v[i].x) + static_cast<double>(v[i].y * v[i].y) +
          static_cast<double>(v[i].z * v[i].z) + static_cast<double>(v[i].w * v[i].w);
  }
  ss = warp_sum_d(ss);
  const float inv = static_cast<float>(1.0 / sqrt(ss / a.H + a.eps));
  const float4* g4 = reinterpret_cast<const float4*>(a.g);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c4 = i * 32 + lane;
    const float4 g = __ldg(g4 + c4);
    const float4 y = make_float4((v[i].x * inv) * g.x, (v[i].y * inv) * g.y,
                                 (v[i].z * inv) * g.z, (v[i].w * inv) * g.w);
    if (a.outb) {
      uint2 p;
      p.x = pack_bf16(y.x, y.y);
      p.y = pack_bf16(y.z, y.w);
      reinterpret_cast<uint2*>(a.outb + static_cast<size_t>(warp) * a.H)[c4] = p;
    }
    if (a.out32) reinterpret_cast<float4*>(a.out32 + static_cast<size_t>(warp) * a.H)[c4] = y;
  }
}

// Per-head q/k RMSNorm then rotate-half RoPE, in place on the packed bf16
// QKV rows (llama.lisp:244-253, 137-151).  One warp per (token, head); lane
// l holds elements 2l, 2l+1 and hd/2 + 2l, hd/2 + 2l + 1 (hd = 128).
__global__ void qk_norm_rope_kernel(QkRopeArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nh = a.q_heads + a.k_heads;
  if (warp >= a.T * nh) return;
  const int t = warp / nh, hh = warp % nh;
  const bool isq = hh < a.q_heads;
  const int col = isq ? a.q_off + hh * 128 : a.k_off + (hh - a.q_heads) * 128;
  const float* w = isq ? a.q_norm : a.k_norm;
  __nv_bfloat16* row = a.qkv + static_cast<size_t>(t) * a.ld + col;
  __nv_bfloat162 lo = reinterpret_cast<__nv_bfloat162*>(row)[lane];
  __nv_bfloat162 hi = reinterpret_cast<__nv_bfloat162*>(row + 64)[lane];
  float x0 = __bfloat162float(lo.x), x1 = __bfloat162float(lo.y);
  float y0 = __bfloat162float(hi.x), y1 = __bfloat162float(hi.y);
  if (w) {
    double ss = static_cast<double>(x0 * x0) + static_cast<double>(x1 * x1) +
                static_cast<double>(y0 * y0) + static_cast<double>(y1 * y1);
    ss = warp_sum_d(ss);
    const float inv = static_cast<float>(1.0 / sqrt(ss / 128.0 + a.eps));
    const int i0 = 2 * lane;
    x0 = (x0 * inv) * w[i0];
    x1 = (x1 * inv) * w[i0 + 1];
    y0 = (y0 * inv) * w[64 + i0];
    y1 = (y1 * inv) * w[64 + i0 + 1];
  }
  const int pos = a.pos[t];
  const float* cs = a.cos_t + static_cast<size_t>(pos) * 64;
  const float* sn = a.sin_t + static_cast<size_t>(pos) * 64;
  const int i0 = 2 * lane;
  const float c0 = cs[i0], c1 = cs[i0 + 1], s0 = sn[i0], s1 = sn[i0 + 1];
  const float nx0 = x0 * c0 - y0 * s0, ny0 = x0 * s0 + y0 * c0;
  const float nx1 = x1 * c1 - y1 * s1, ny1 = x1 * s1 + y1 * c1;
  reinterpret_cast<__nv_bfloat162*>(row)[lane] = __floats2bfloat162_rn(nx0, nx1);
  reinterpret_cast<__nv_bfloat162*>(row + 64)[lane] = __floats2bfloat162_rn(ny0, ny1);
}

// Pooling + L2 (bert.lisp:302-319, llama.lisp:327-343).  One block per
// sequence, threads over hidden dims, tokens summed in order as the Lisp does.
// mode 0 = first token (:cls), 1 = mean, 2 = last token (:last).
// With final_norm (llama), each pooled token is RMS-normalised first
// (llama.lisp:325-326).
__global__ void pool_l2_kernel(PoolArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  __shared__ double redd[32];
  const int s = blockIdx.x;
  const int base = a.cu[s], L = a.cu[s + 1] - base;
  const int H = a.H;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // H <= 4 * blockDim
  const int t_first = a.mode == 2 ? L - 1 : 0;
  const int t_last = a.mode == 1 ? L : t_first + 1;
  if (!a.final_norm) {
    // sums in token order per dimension (bert.lisp:307-310); eight tokens'
    // loads are issued ahead of their adds to hide memory latency
    int j = 0;
    for (int i = threadIdx.x; i < H; i += blockDim.x, ++j) {
      const float* x = a.h + static_cast<size_t>(base) * H + i;
      float s0 = 0.f;
      int t = t_first;
      for (; t + 8 <= t_last; t += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = x[static_cast<size_t>(t + u) * H];
#pragma unroll
        for (int u = 0; u < 8; ++u) s0 = s0 + v[u];
      }
      for (; t < t_last; ++t) s0 = s0 + x[static_cast<size_t>(t) * H];
      acc[j] = s0;
    }
  } else {
    for (int t = t_first; t < t_last; ++t) {
      const float* x = a.h + static_cast<size_t>(base + t) * H;
      double ss = 0.0;
      for (int i = threadIdx.x; i < H; i += blockDim.x) ss += static_cast<double>(x[i] * x[i]);
      ss = warp_sum_d(ss);
      if ((threadIdx.x & 31) == 0) redd[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        double v = threadIdx.x < (blockDim.x >> 5) ? redd[threadIdx.x] : 0.0;
        v = warp_sum_d(v);
        if (threadIdx.x == 0) redd[0] = v;
      }
      __syncthreads();
      const float inv = static_cast<float>(1.0 / sqrt(redd[0] / H + a.eps));
      __syncthreads();
      int j = 0;
      for (int i = threadIdx.x; i < H; i += blockDim.x, ++j)
        acc[j] = acc[j] + (x[i] * inv) * a.norm_w[i];
    }
  }
  float sq = 0.f;
  int j = 0;
  for (int i = threadIdx.x; i < H; i += blockDim.x, ++j) {
    if (a.mode == 1) acc[j] = acc[j] / static_cast<float>(L);
    sq += acc[j] * acc[j];
  }
  sq = warp_sum(sq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float norm = sqrtf(red[0]);
  j = 0;
  for (int i = threadIdx.x; i < H; i += blockDim.x, ++j)
    a.out[static_cast<size_t>(s) * a.out_stride + i] = acc[j] / norm;
}

// h[t] = table[ids[t]] widened to fp32 (llama.lisp:316-320)
__global__ void gather_rows_kernel(const void* table, int dtype, const int* ids, float* out,
                                   int T, int H) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const size_t H4 = H / 4;
  const size_t src = static_cast<size_t>(ids[warp]) * H4;
  float4* dst = reinterpret_cast<float4*>(out + static_cast<size_t>(warp) * H);
  for (int c = lane; c < H / 4; c += 32) dst[c] = ld_row4(table, dtype, src + c);
}

// position of every packed token within its sequence
__global__ void positions_kernel(const int* cu, int nseq, int* pos) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.x;
  if (s >= nseq) return;
  const int b = cu[s], e = cu[s + 1];
  for (int t = b + threadIdx.x; t < e; t += blockDim.x) pos[t] = t - b;
}

// st::half-to-float (st.lisp:22-30), exponent 31 -> +-most-positive-single.
__global__ void f16_to_f32_kernel(const uint16_t* src, float* dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint16_t h = src[i];
    const int e = (h >> 10) & 31;
    const float sign = (h & 0x8000) ? -1.f : 1.f;
    float v;
    if (e == 31) v = sign * FLT_MAX;
    else v = __half2float(__ushort_as_half(h));
    dst[i] = v;
  }
}

__global__ void bf16_to_f32_kernel(const uint16_t* src, float* dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = __uint_as_float(static_cast<uint32_t>(src[i]) << 16);
}

__global__ void f32_to_bf16_kernel(const float* src, __nv_bfloat16* dst, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

// ------------------------------------------------------------- launchers --
static inline int grid_for(size_t n, int per_block) {
  size_t g = (n + per_block - 1) / per_block;
  return static_cast<int>(g > 0x7fffffff ? 0x7fffffff : g);
}

cudaError_t launch_embed_ln(const EmbedLnArgs& a, cudaStream_t st) {
  const int nv = a.H / 128;
  const int blocks = grid_for(static_cast<size_t>(a.T), 8);
  switch (nv) {
    case 3: return launch_pdl(embed_ln_kernel<3>, dim3(blocks), dim3(256), 0, st, a);
    case 6: return launch_pdl(embed_ln_kernel<6>, dim3(blocks), dim3(256), 0, st, a);
    case 8: return launch_pdl(embed_ln_kernel<8>, dim3(blocks), dim3(256), 0, st, a);
    case 4: return launch_pdl(embed_ln_kernel<4>, dim3(blocks), dim3(256), 0, st, a);
    case 2: return launch_pdl(embed_ln_kernel<2>, dim3(blocks), dim3(256), 0, st, a);
    case 1: return launch_pdl(embed_ln_kernel<1>, dim3(blocks), dim3(256), 0, st, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_ln(const LnArgs& a, cudaStream_t st) {
  const int nv = a.H / 128;
  const int blocks = grid_for(static_cast<size_t>(a.T), 8);
  switch (nv) {
    case 3: return launch_pdl(ln_kernel<3>, dim3(blocks), dim3(256), 0, st, a);
    case 6: return launch_pdl(ln_kernel<6>, dim3(blocks), dim3(256), 0, st, a);
    case 8: return launch_pdl(ln_kernel<8>, dim3(blocks), dim3(256), 0, st, a);
    case 4: return launch_pdl(ln_kernel<4>, dim3(blocks), dim3(256), 0, st, a);
    case 2: return launch_pdl(ln_kernel<2>, dim3(blocks), dim3(256), 0, st, a);
    case 1: return launch_pdl(ln_kernel<1>, dim3(blocks), dim3(256), 0, st, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rmsnorm(const RmsArgs& a, cudaStream_t st) {
  const int nv = a.H / 128;
  const int blocks = grid_for(static_cast<size_t>(a.T), 8);
  switch (nv) {
    case 8: rmsnorm_kernel<8><<<blocks, 256, 0, st>>>(a); break;
    case 6: rmsnorm_kernel<6><<<blocks, 256, 0, st>>>(a); break;
    case 3: rmsnorm_kernel<3><<<blocks, 256, 0, st>>>(a); break;
    case 4: rmsnorm_kernel<4><<<blocks, 256, 0, st>>>(a); break;
    case 2: rmsnorm_kernel<2><<<blocks, 256, 0, st>>>(a); break;
    case 1: rmsnorm_kernel<1><<<blocks, 256, 0, st>>>(a); break;
    case 16: rmsnorm_kernel<16><<<blocks, 256, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(const QkRopeArgs& a, cudaStream_t st) {
  const size_t warps = static_cast<size_t>(a.T) * (a.q_heads + a.k_heads);
  qk_norm_rope_kernel<<<grid_for(warps, 8), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_pool_l2(const PoolArgs& a, int nseq, cudaStream_t st) {
  const int threads = a.H <= 512 ? 128 : 256;
  if (a.H > 4 * threads) return cudaErrorInvalidValue;
  return launch_pdl(pool_l2_kernel, dim3(nseq), dim3(threads), 0, st, a);
}

cudaError_t launch_gather_rows(const void* table, int dtype, const int* ids, float* out, int T,
                               int H, cudaStream_t st) {
  gather_rows_kernel<<<grid_for(static_cast<size_t>(T), 8), 256, 0, st>>>(table, dtype, ids, out,
                                                                          T, H);
  return cudaGetLastError();
}

cudaError_t launch_positions(const int* cu, int nseq, int* pos, cudaStream_t st) {
  return launch_pdl(positions_kernel, dim3(nseq), dim3(128), 0, st, cu, nseq, pos);
}

cudaError_t launch_convert(int kind, const void* src, void* dst, size_t n, cudaStream_t st) {
  const int g = grid_for(n, 256 * 4);
  const int grid = g < 4096 ? (g > 0 ? g : 1) : 4096;
  switch (kind) {
    case kConvF16ToF32:
      f16_to_f32_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(src),
                                              static_cast<float*>(dst), n);
      break;
    case kConvBf16ToF32:
      bf16_to_f32_kernel<<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(src),
                                               static_cast<float*>(dst), n);
      break;
    case kConvF32ToBf16:
      f32_to_bf16_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(src),
                                               static_cast<__nv_bfloat16*>(dst), n);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace ec
