// ec_ivf_tc.cu -- k-means assignment (ann::nearest-centroid for every row,
// ann.lisp:69-77 / 90-105) on the tensor cores, with results identical to
// the exact scan.
//
// 1. rows and centroids are rounded to bf16 once (centroids per iteration),
//    with upper bounds of their Euclidean norms;
// 2. a tcgen05 GEMM computes the approximate scores S~ = bf16(x) . bf16(c)^T
//    and its epilogue (kEpiArgCand) keeps, per row and column part, the
//    largest S~ and the columns of the largest two;
// 3. per row, the exact argmax must lie within w_r of max S~: rounding each
//    factor to bf16 moves a product by at most (2^-7 + 2^-16)|x_k c_k|, the
//    fp32 sums add at most 3 * d * 2^-24 sum |x_k c_k| (the tensor-core sum,
//    even truncating, and the reference's sequential sum), and
//    sum |x_k c_k| <= |x| |c|, so |S~ - S| <= rel |x| max|c| = w_r / 2 with
//    rel = 1.01 (2^-7 + 2^-16 + 3 d 2^-24) (argcand_rel).  Every column
//    within the window is re-scored with the reference's own arithmetic
//    (sequential single-float __fmul_rn / __fadd_rn over k) and the highest
//    score with the lowest index wins, as in the exact scan;
// 4. rows whose window holds more than two columns of one part, or whose
//    norms are not finite, go through the exact scan.
#include <cfloat>
#include <cstdint>

#include <cuda_bf16.h>

#include "ec_ivf.h"

namespace ec {

namespace {

__device__ __forceinline__ uint2 to_bf16x4(float4 v) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

// one warp per row: bf16 copy and an upper bound of the norm (the fp32 sum
// of squares is within d * 2^-24 of the true one: `slack` covers that and
// the square root); the largest norm goes to *nmax (non-negative floats
// order like their bit patterns)
__global__ void round_rows_kernel(const float* X, int64_t n, int d, float slack,
                                  __nv_bfloat16* Xb, float* norms, unsigned* nmax) {
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const float4* x4 = reinterpret_cast<const float4*>(X + r * d);
  uint2* o4 = reinterpret_cast<uint2*>(Xb + r * d);
  float ss = 0.f;
  for (int i = lane; i < d / 4; i += 32) {
    const float4 v = x4[i];
    ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
    o4[i] = to_bf16x4(v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) {
    float nv = sqrtf(ss) * slack;
    if (!(nv < INFINITY)) nv = INFINITY;  // NaN / overflow: no finite bound
    if (norms) norms[r] = nv;
    if (nmax) atomicMax(nmax, __float_as_uint(nv));
  }
}

// One thread per row: the exact argmax over the window's columns.  A row
// whose window holds a single column is decided without reading it (that
// column is the exact argmax: every column tied with or above it would lie
// in the window too).  Rows with two to kMaxCand candidates pass through
// shared memory in 32-column slices (coalesced loads of those rows only,
// padded rows: thread t reads bank (t + k) % 32), each thread keeping up to
// kMaxCand running sequential sums -- the same single-float order as the
// reference's %dot; a block with no such row reads no rows at all.  Rows
// with more candidates take the exact scan.
constexpr int kRedRows = 128;
constexpr int kMaxCand = 8;

__global__ void __launch_bounds__(kRedRows)
    argcand_reduce_kernel(const float* X, int64_t n, int d, const float* C, const float* xnorm,
                          const float* cmax, float rel2, int parts, const float* mloc,
                          const uint32_t* pk, int32_t* out, int64_t* fb_rows,
                          unsigned long long* fb_count) {
  // rows padded to 36 floats: 16-byte aligned, and the eight threads of a
  // 128-bit shared-memory phase land on distinct banks
  __shared__ __align__(16) float xs[kRedRows][36];
  __shared__ int need[kRedRows];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRedRows;
  const int64_t r = r0 + threadIdx.x;
  const bool live = r < n;
  int cand[kMaxCand];
  int nc = 0;
  bool exact = false;
  bool rescore = false;
  if (live) {
    const float w = rel2 * *cmax * xnorm[r];
    // the part maxima, four independent chains (several loads in flight)
    float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
    int t = 0;
#pragma unroll 2
    for (; t + 4 <= parts; t += 4) {
      m0 = fmaxf(m0, mloc[static_cast<size_t>(t) * n + r]);
      m1 = fmaxf(m1, mloc[static_cast<size_t>(t + 1) * n + r]);
      m2 = fmaxf(m2, mloc[static_cast<size_t>(t + 2) * n + r]);
      m3 = fmaxf(m3, mloc[static_cast<size_t>(t + 3) * n + r]);
    }
    for (; t < parts; ++t) m0 = fmaxf(m0, mloc[static_cast<size_t>(t) * n + r]);
    const float m = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
    exact = !(w >= 0.f && w < INFINITY) || !(m > -INFINITY && m < INFINITY);
    const float lo = m - w;
    for (int t = 0; !exact && t < parts; ++t) {
      const size_t o = static_cast<size_t>(t) * n + r;
      if (!(mloc[o] >= lo)) continue;
      const uint32_t p = pk[o];
      const uint32_t mt = p >> 30;
      const int need_c = (mt & 1u) ? 2 : 1;
      if ((mt & 2u) || nc + need_c > kMaxCand) {
        exact = true;
        break;
      }
#pragma unroll
      for (int q = 0; q < kMaxCand; ++q)
        if (q == nc) cand[q] = static_cast<int>(p & 0x7fffu);
      ++nc;
      if (mt & 1u) {
#pragma unroll
        for (int q = 0; q < kMaxCand; ++q)
          if (q == nc) cand[q] = static_cast<int>((p >> 15) & 0x7fffu);
        ++nc;
      }
    }
    if (exact) {
      nc = 0;
      fb_rows[atomicAdd(fb_count, 1ull)] = r;
    } else if (nc == 1 && lo > -FLT_MAX) {
      // the exact score is at least m - w / 2 > -FLT_MAX: the Lisp's strict
      // comparison against most-negative-single-float picks this column
      out[r] = cand[0];
      nc = 0;
    } else {
      rescore = nc > 0;
    }
  }
  need[threadIdx.x] = rescore ? 1 : 0;
  if (!__syncthreads_or(rescore)) return;
  float acc[kMaxCand];
#pragma unroll
  for (int q = 0; q < kMaxCand; ++q) acc[q] = 0.f;
  for (int k0 = 0; k0 < d; k0 += 32) {
    __syncthreads();
    for (int i = threadIdx.x; i < kRedRows * 8; i += kRedRows) {
      const int rr = i >> 3, c4 = i & 7;
      if (need[rr])
        *reinterpret_cast<float4*>(&xs[rr][c4 * 4]) =
            *reinterpret_cast<const float4*>(X + (r0 + rr) * d + k0 + c4 * 4);
    }
    __syncthreads();
    // d % 32 == 0 on this path: whole 32-column slices
#pragma unroll 1
    for (int q = 0; q < kMaxCand; ++q) {
      if (q >= nc) break;
      int cq = cand[0];
#pragma unroll
      for (int u = 1; u < kMaxCand; ++u)
        if (u == q) cq = cand[u];
      const float4* c4 = reinterpret_cast<const float4*>(C + static_cast<int64_t>(cq) * d + k0);
      float s = 0.f;
#pragma unroll
      for (int u = 0; u < kMaxCand; ++u)
        if (u == q) s = acc[u];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 cv = __ldg(c4 + i);
        const float4 xv = *reinterpret_cast<const float4*>(&xs[threadIdx.x][4 * i]);
        s = __fadd_rn(s, __fmul_rn(xv.x, cv.x));
        s = __fadd_rn(s, __fmul_rn(xv.y, cv.y));
        s = __fadd_rn(s, __fmul_rn(xv.z, cv.z));
        s = __fadd_rn(s, __fmul_rn(xv.w, cv.w));
      }
#pragma unroll
      for (int u = 0; u < kMaxCand; ++u)
        if (u == q) acc[u] = s;
    }
  }
  if (!rescore) return;
  float best = -FLT_MAX;
  int bidx = 0x7fffffff;
#pragma unroll
  for (int q = 0; q < kMaxCand; ++q) {
    if (q >= nc) break;
    const float sq = acc[q];
    const int c = cand[q];
    if (sq > best || (sq == best && c < bidx)) {
      best = sq;
      bidx = c;
    }
  }
  // no score above most-negative-single-float: the Lisp keeps centroid 0
  out[r] = (bidx == 0x7fffffff || !(best > -FLT_MAX)) ? 0 : bidx;
}

__global__ void scatter_assign_kernel(const int64_t* fb_rows, int64_t nfb, const int32_t* vals,
                                      int32_t* out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < nfb) out[fb_rows[i]] = vals[i];
}

// out[j] = X[rows[j]] for j < m, one warp per row in 16-byte pieces; grid
// stride over the rows
__global__ void gather_rows_kernel(const float* __restrict__ X, const int64_t* __restrict__ rows,
                                   int64_t m, int d4, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); j < m;
       j += warps) {
    const float4* src = reinterpret_cast<const float4*>(X) + rows[j] * d4;
    float4* dst = reinterpret_cast<float4*>(out) + j * d4;
    for (int c = lane; c < d4; c += 32) dst[c] = __ldcs(src + c);
  }
}

}  // namespace

float argcand_rel(int d) {
  return 1.01f * (0x1p-7f + 0x1p-16f + 3.0f * static_cast<float>(d) * 0x1p-24f);
}

cudaError_t launch_round_rows(const float* X, int64_t n, int d, __nv_bfloat16* Xb, float* norms,
                              unsigned* nmax, cudaStream_t st) {
  if (d % 4 || n <= 0) return cudaErrorInvalidValue;
  const float slack = 1.0f + 2.0f * static_cast<float>(d + 4) * 0x1p-24f;
  const int64_t blocks = (n + 7) / 8;
  round_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(X, n, d, slack, Xb, norms, nmax);
  return cudaGetLastError();
}

cudaError_t launch_argcand_reduce(const float* X, int64_t n, int d,
                                  const float* C, const float* xnorm, const float* cmax, float rel2,
                                  int parts, const float* mloc, const uint32_t* pk, int32_t* out,
                                  int64_t* fb_rows, unsigned long long* fb_count, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (d % 32) return cudaErrorInvalidValue;
  const int64_t blocks = (n + kRedRows - 1) / kRedRows;
  argcand_reduce_kernel<<<static_cast<unsigned>(blocks), kRedRows, 0, st>>>(
      X, n, d, C, xnorm, cmax, rel2, parts, mloc, pk, out, fb_rows, fb_count);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float* X, const int64_t* rows, int64_t m, int d, float* out,
                               int num_sms, cudaStream_t st) {
  if (m <= 0) return cudaSuccess;
  if (d % 4) return cudaErrorInvalidValue;
  const int64_t want = (m + 7) / 8;  // eight warps per CTA, one row each
  const int64_t cap = static_cast<int64_t>(num_sms > 0 ? num_sms : 148) * 8;
  gather_rows_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, st>>>(X, rows, m, d / 4,
                                                                                      out);
  return cudaGetLastError();
}

cudaError_t launch_scatter_assign(const int64_t* fb_rows, int64_t nfb, const int32_t* vals,
                                  int32_t* out, cudaStream_t st) {
  if (nfb <= 0) return cudaSuccess;
  scatter_assign_kernel<<<static_cast<unsigned>((nfb + 255) / 256), 256, 0, st>>>(fb_rows, nfb,
                                                                                 vals, out);
  return cudaGetLastError();
}

}  // namespace ec
