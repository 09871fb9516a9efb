// ec_ln.cuh -- the LayerNorm row arithmetic of the row kernels
// (ec_rows.cu), kept apart so that any kernel finishing rows gives the
// same bits: one warp per row, NV float4 per lane.
#pragma once

#include <cuda_bf16.h>

#include "ec_ptx.cuh"

namespace ec {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// LayerNorm of bert::layernorm (bert.lisp:155-174): two-pass mean/variance,
// std = sqrt(var) + 1e-12, y = ((x - mean) / std) * g + b.
template <int NV>
__device__ __forceinline__ void ln_finish(float4 (&v)[NV], int H, const float* g,
                                          const float* b, float* out32, __nv_bfloat16* outb,
                                          int lane) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) / static_cast<float>(H);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + bb * bb) + (c * c + d * d);
  }
  const float var = warp_sum(q) / static_cast<float>(H);
  const float stdv = sqrtf(var) + 1e-12f;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c4 = i * 32 + lane;
    const float4 gg = __ldg(g4 + c4), bb = __ldg(b4 + c4);
    float4 y;
    y.x = ((v[i].x - mean) / stdv) * gg.x + bb.x;
    y.y = ((v[i].y - mean) / stdv) * gg.y + bb.y;
    y.z = ((v[i].z - mean) / stdv) * gg.z + bb.z;
    y.w = ((v[i].w - mean) / stdv) * gg.w + bb.w;
    if (out32) reinterpret_cast<float4*>(out32)[c4] = y;
    if (outb) {
      uint2 p;
      p.x = pack_bf16(y.x, y.y);
      p.y = pack_bf16(y.z, y.w);
      reinterpret_cast<uint2*>(outb)[c4] = p;
    }
  }
}

}  // namespace ec
