// ec_ivf_kernels.cu -- IVF kernels: k-means assignment, stable inverted-list
// build, per-cluster sums, IVF probe and list scan, flat scan.
//
// Scores are computed with the reference's exact arithmetic: a sequential
// single-float sum over k of separately rounded products (ann.lisp:25-35,
// kb.lisp:153-162), written with __fmul_rn / __fadd_rn so the compiler
// cannot contract them into FMAs.  Every score is therefore bit-identical to
// the Lisp's, and argmax / top-k decisions (ties included) match exactly.
// The score kernel is a register-tiled SIMT GEMM: a 128 x 128 output tile
// per CTA, an 8 x 8 micro-tile per thread, k staged through shared memory
// in chunks of 32 -- each thread still walks k in order for each of its
// outputs.
#include <cfloat>
#include <cstdint>

#include "ec_ivf.h"
#include "ec_ptx.cuh"

namespace ec {

constexpr int SB = 128;   // rows / centroids per tile
constexpr int SK = 32;    // k chunk
constexpr int SPAD = 4;

// ordered key: ascending key == descending score, then ascending tiebreak
__device__ __forceinline__ unsigned long long desc_key(float s, uint32_t tie) {
  s = s + 0.0f;  // -0.0 -> +0.0 (they compare equal in the reference)
  uint32_t u = __float_as_uint(s);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // ascending float order
  return (static_cast<unsigned long long>(~u) << 32) | tie;
}
__device__ __forceinline__ float key_score(unsigned long long k) {
  uint32_t u = ~static_cast<uint32_t>(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(u);
}

// Load a SB x SK chunk (rows r0.., cols k0..) of a row-major [n, d] matrix
// transposed into smem T[SK][SB + SPAD]; rows past n read as 0.
__device__ __forceinline__ void load_chunk_t(float (*T)[SB + SPAD], const float* X, const int64_t* rows,
                                             int64_t r0, int64_t n, int d, int k0) {
  // 128 rows x 32 cols = 1024 float4; 256 threads x 4
  for (int i = threadIdx.x; i < SB * (SK / 4); i += blockDim.x) {
    const int r = i / (SK / 4), c4 = i % (SK / 4);
    const int64_t gr = r0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (gr < n && k0 + c4 * 4 < d) {
      const int64_t src = rows ? rows[gr] : gr;
      v = *reinterpret_cast<const float4*>(X + src * d + k0 + c4 * 4);
    }
    T[c4 * 4 + 0][r] = v.x;
    T[c4 * 4 + 1][r] = v.y;
    T[c4 * 4 + 2][r] = v.z;
    T[c4 * 4 + 3][r] = v.w;
  }
}

// acc[i][j] = sum_k A[row i][k] * B[col j][k], k ascending, no FMA.
// Thread (ty, tx) of a 16 x 16 grid owns rows ty + 16 i and cols tx + 16 j.
__device__ __forceinline__ void exact_tile(float (&acc)[8][8], float (*As)[SB + SPAD],
                                           float (*Bs)[SB + SPAD], const float* X,
                                           const int64_t* xrows, int64_t r0, int64_t n,
                                           const float* C, int64_t c0, int64_t kc, int d) {
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < d; k0 += SK) {
    __syncthreads();
    load_chunk_t(As, X, xrows, r0, n, d, k0);
    load_chunk_t(Bs, C, nullptr, c0, kc, d, k0);
    __syncthreads();
    const int kend = d - k0 < SK ? d - k0 : SK;
    for (int k = 0; k < kend; ++k) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = Bs[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
    }
  }
}

// ann::nearest-centroid for every row: strict > over ascending centroid
// index, i.e. the highest score with the lowest index among equals.
__global__ void __launch_bounds__(256) assign_kernel(const float* X, const int64_t* xrows, int64_t n,
                                                     const float* C, int k, int d, int32_t* out) {
  __shared__ float As[SK][SB + SPAD];
  __shared__ float Bs[SK][SB + SPAD];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * SB;
  float best[8];
  int bidx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    best[i] = -FLT_MAX;
    bidx[i] = 0x7fffffff;
  }
  for (int c0 = 0; c0 < k; c0 += SB) {
    float acc[8][8];
    exact_tile(acc, As, Bs, X, xrows, r0, n, C, c0, k, d);
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + tx + 16 * j;
        if (c < k) {
          const float s = acc[i][j];
          if (s > best[i] || (s == best[i] && c < bidx[i])) {
            best[i] = s;
            bidx[i] = c;
          }
        }
      }
  }
  // combine the 16 threads (tx) of each row: lanes differ in bits 0..3
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float s = best[i];
    int c = bidx[i];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const int c2 = __shfl_xor_sync(0xffffffffu, c, o);
      if (s2 > s || (s2 == s && c2 < c)) {
        s = s2;
        c = c2;
      }
    }
    const int64_t row = r0 + ty + 16 * i;
    // no score above most-negative-single-float: the Lisp keeps best = 0
    if (tx == 0 && row < n) out[row] = (c == 0x7fffffff || !(s > -FLT_MAX)) ? 0 : c;
  }
}

// full score matrix S[q, c] (IVF probe, kb.lisp:351-352)
__global__ void __launch_bounds__(256) scores_kernel(const float* Q, int64_t nq, const float* C, int k,
                                                     int d, float* S) {
  __shared__ float As[SK][SB + SPAD];
  __shared__ float Bs[SK][SB + SPAD];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * SB;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * SB;
  float acc[8][8];
  exact_tile(acc, As, Bs, Q, nullptr, r0, nq, C, c0, k, d);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t r = r0 + ty + 16 * i;
    if (r >= nq) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t c = c0 + tx + 16 * j;
      if (c < k) S[r * k + c] = acc[i][j];
    }
  }
}

// S[q, c] for a few queries (nq <= kSmallQ): one thread per centroid, the
// sequential single-float sum of exact_tile (bit-identical scores); the
// centroid row is read once for all the queries, several loads in flight.
// (The 128 x 128 tiles of scores_kernel would be almost all padding.)
constexpr int kSmallQ = 8;
__global__ void __launch_bounds__(128) scores_small_kernel(const float* Q, int nq, const float* C, int k,
                                                           int d, float* S) {
  extern __shared__ float qs[];  // [nq][d]
  for (int i = threadIdx.x; i < nq * d; i += blockDim.x) qs[i] = Q[i];
  __syncthreads();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= k) return;
  float acc[kSmallQ];
#pragma unroll
  for (int j = 0; j < kSmallQ; ++j) acc[j] = 0.f;
  const float4* cr = reinterpret_cast<const float4*>(C + static_cast<int64_t>(c) * d);
#pragma unroll 8
  for (int c4 = 0; c4 < d / 4; ++c4) {
    const float4 v = cr[c4];
#pragma unroll
    for (int j = 0; j < kSmallQ; ++j) {
      if (j < nq) {
        const float* qj = qs + j * d + 4 * c4;
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qj[0], v.x));
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qj[1], v.y));
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qj[2], v.z));
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qj[3], v.w));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kSmallQ; ++j)
    if (j < nq) S[static_cast<int64_t>(j) * k + c] = acc[j];
}

// The same scores with the centroid rows staged whole in shared memory: one
// warp per 32 centroids copies its 32 rows and the queries with one untiled
// bulk copy per row (lane r copies row r), all completing on one mbarrier,
// waits once, and each lane then runs its centroid's sequential sum from
// shared memory (rows padded to an odd number of 16-byte pieces: the eight
// lanes of a 128-bit phase hit distinct banks).  One memory latency per warp
// and a few copy instructions; bit-identical to scores_small_kernel.  The
// wait is bounded: on a timeout the status word is set and the copies in
// flight are waited for (bounded again) before the CTA exits.
constexpr int kScoreRows = 32;

__global__ void __launch_bounds__(32) scores_rows_kernel(const float* Q, int nq, const float* C, int k,
                                                         int d, float* S, unsigned* status) {
  extern __shared__ __align__(16) float srow[];
  __shared__ uint64_t bar;
  const int ld = 4 * ((d >> 2) | 1);     // odd count of 16-byte pieces per row
  float* cs = srow;                     // [kScoreRows][ld]
  float* qs = srow + kScoreRows * ld;   // [nq][d]
  const int lane = threadIdx.x;
  const int c0 = blockIdx.x * kScoreRows;
  const int rows = min(kScoreRows, k - c0);
  const uint32_t row_bytes = static_cast<uint32_t>(d) * 4u;
  if (lane == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(&bar, row_bytes * static_cast<uint32_t>(rows + nq));
  }
  __syncwarp();
  if (lane < rows) bulk_load(cs + lane * ld, C + static_cast<int64_t>(c0 + lane) * d, row_bytes, &bar);
  for (int j = lane; j < nq; j += 32) bulk_load(qs + j * d, Q + static_cast<int64_t>(j) * d, row_bytes, &bar);
  if (!mbar_wait(&bar, 0, nullptr)) {
    report(status, kDevTimeoutOther);
    mbar_wait(&bar, 0, nullptr);
    return;
  }
  if (lane >= rows) return;
  float acc[kSmallQ];
#pragma unroll
  for (int j = 0; j < kSmallQ; ++j) acc[j] = 0.f;
  const float4* cr = reinterpret_cast<const float4*>(cs + lane * ld);
  const int d4 = d >> 2;
#pragma unroll 4
  for (int c4 = 0; c4 < d4; ++c4) {
    const float4 v = cr[c4];
#pragma unroll
    for (int j = 0; j < kSmallQ; ++j) {
      if (j < nq) {
        const float4 qv = reinterpret_cast<const float4*>(qs + j * d)[c4];
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.x, v.x));
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.y, v.y));
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.z, v.z));
        acc[j] = __fadd_rn(acc[j], __fmul_rn(qv.w, v.w));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kSmallQ; ++j)
    if (j < nq) S[static_cast<int64_t>(j) * k + c0 + lane] = acc[j];
}

// ---------------------------------------------------- stable counting sort --
constexpr int kSortTile = 4096;

__global__ void hist_kernel(const int32_t* a, int64_t n, int k, uint32_t* tile_hist) {
  extern __shared__ uint32_t h[];
  for (int c = threadIdx.x; c < k; c += blockDim.x) h[c] = 0;
  __syncthreads();
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kSortTile;
  for (int64_t i = t0 + threadIdx.x; i < t0 + kSortTile && i < n; i += blockDim.x)
    atomicAdd(&h[a[i]], 1u);
  __syncthreads();
  for (int c = threadIdx.x; c < k; c += blockDim.x)
    tile_hist[static_cast<int64_t>(blockIdx.x) * k + c] = h[c];
}

// single-block exclusive scan of counts -> offs[0..k], k <= 32 * 1024
__global__ void scan_kernel(const uint32_t* counts, int k, int64_t* offs) {
  __shared__ int64_t part[1024];
  const int per = (k + blockDim.x - 1) / blockDim.x;
  const int b = threadIdx.x * per;
  int64_t s = 0;
  for (int i = 0; i < per && b + i < k; ++i) s += counts[b + i];
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int t = 0; t < static_cast<int>(blockDim.x); ++t) {
      const int64_t v = part[t];
      part[t] = acc;
      acc += v;
    }
    offs[k] = acc;
  }
  __syncthreads();
  int64_t acc = part[threadIdx.x];
  for (int i = 0; i < per && b + i < k; ++i) {
    offs[b + i] = acc;
    acc += counts[b + i];
  }
}

// one warp per tile, rows in ascending order: lists[pos] = base + row (for
// k too large for scatter_cta_kernel's per-warp histograms)
__global__ void scatter_kernel(const int32_t* a, int64_t n, int k, const uint32_t* tile_off,
                               uint32_t base, uint32_t* lists) {
  extern __shared__ uint32_t cur[];
  for (int c = threadIdx.x; c < k; c += blockDim.x)
    cur[c] = tile_off[static_cast<int64_t>(blockIdx.x) * k + c];
  __syncwarp();
  const int lane = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kSortTile;
  for (int64_t i0 = t0; i0 < t0 + kSortTile && i0 < n; i0 += 32) {
    const int64_t i = i0 + lane;
    const bool valid = i < n && i < t0 + kSortTile;
    const int c = valid ? a[i] : -1 - lane;  // invalid lanes never match
    const unsigned peers = __match_any_sync(0xffffffffu, c);
    if (valid) {
      const unsigned lower = peers & ((1u << lane) - 1u);
      const uint32_t pos = cur[c] + __popc(lower);
      lists[pos] = base + static_cast<uint32_t>(i);
      __syncwarp(peers);
      if (lower == 0) cur[c] += __popc(peers);
    }
    __syncwarp();
  }
}

// Column sums and tile offsets of tile_hist with the tiles of each column
// split over the eight warps of a block (32 columns per block, lane =
// column): coalesced rows of tile_hist, eight segments in flight per column.
constexpr int kSegWarps = 8;

// counts[c] = sum over tiles
__global__ void __launch_bounds__(256) colsum_seg_kernel(const uint32_t* tile_hist, int ntiles, int k,
                                                         uint32_t* counts) {
  __shared__ uint32_t part[kSegWarps][32];
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int per = (ntiles + kSegWarps - 1) / kSegWarps;
  const int t0 = min(ntiles, seg * per), t1 = min(ntiles, t0 + per);
  uint32_t s = 0;
  if (c < k)
    for (int t = t0; t < t1; ++t) s += tile_hist[static_cast<int64_t>(t) * k + c];
  part[seg][lane] = s;
  __syncthreads();
  if (seg == 0 && c < k) {
    uint32_t tot = 0;
#pragma unroll
    for (int w = 0; w < kSegWarps; ++w) tot += part[w][lane];
    counts[c] = tot;
  }
}

// tile_hist[t][c] <- start of tile t's run inside list c
__global__ void __launch_bounds__(256) tile_offsets_seg_kernel(uint32_t* tile_hist, int ntiles, int k,
                                                               const int64_t* offs) {
  __shared__ uint32_t part[kSegWarps][32];
  const int lane = threadIdx.x & 31, seg = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int per = (ntiles + kSegWarps - 1) / kSegWarps;
  const int t0 = min(ntiles, seg * per), t1 = min(ntiles, t0 + per);
  uint32_t s = 0;
  if (c < k)
    for (int t = t0; t < t1; ++t) s += tile_hist[static_cast<int64_t>(t) * k + c];
  part[seg][lane] = s;
  __syncthreads();
  if (c >= k) return;
  uint32_t run = static_cast<uint32_t>(offs[c]);
  for (int w = 0; w < seg; ++w) run += part[w][lane];
  for (int t = t0; t < t1; ++t) {
    const uint32_t v = tile_hist[static_cast<int64_t>(t) * k + c];
    tile_hist[static_cast<int64_t>(t) * k + c] = run;
    run += v;
  }
}

// lists[pos] = base + row with one block of eight warps per tile: warp w
// owns rows [w * 512, w * 512 + 512) of the tile, so its run inside each
// list starts after the tile's earlier warps' rows (per-warp histograms in
// shared memory, prefixed in warp order); each warp then scatters its rows
// in ascending order (match_any groups equal lists within a step).
constexpr int kScatWarps = 8;
constexpr int kScatRows = kSortTile / kScatWarps;

__global__ void __launch_bounds__(256) scatter_cta_kernel(const int32_t* a, int64_t n, int k,
                                                          const uint32_t* tile_off, uint32_t base,
                                                          uint32_t* lists) {
  extern __shared__ uint32_t wh[];  // [kScatWarps][k]
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kScatWarps * k; i += blockDim.x) wh[i] = 0;
  __syncthreads();
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kSortTile + static_cast<int64_t>(w) * kScatRows;
  const int64_t t1 = min(n, t0 + kScatRows);
  uint32_t* mine = wh + static_cast<size_t>(w) * k;
  for (int64_t i = t0 + lane; i < t1; i += 32) atomicAdd(&mine[a[i]], 1u);
  __syncthreads();
  for (int c = threadIdx.x; c < k; c += blockDim.x) {
    uint32_t run = tile_off[static_cast<int64_t>(blockIdx.x) * k + c];
#pragma unroll
    for (int v = 0; v < kScatWarps; ++v) {
      const uint32_t cnt = wh[static_cast<size_t>(v) * k + c];
      wh[static_cast<size_t>(v) * k + c] = run;
      run += cnt;
    }
  }
  __syncthreads();
  for (int64_t i0 = t0; i0 < t1; i0 += 32) {
    const int64_t i = i0 + lane;
    const bool valid = i < t1;
    const int c = valid ? a[i] : -1 - lane;  // invalid lanes never match
    const unsigned peers = __match_any_sync(0xffffffffu, c);
    if (valid) {
      const unsigned lower = peers & ((1u << lane) - 1u);
      const uint32_t pos = mine[c] + __popc(lower);
      lists[pos] = base + static_cast<uint32_t>(i);
      __syncwarp(peers);
      if (lower == 0) mine[c] += __popc(peers);
    }
    __syncwarp();
  }
}

// sums[c] = x[rows of list c] summed in list order (ann.lisp:109-115) as
// float4 columns; out[c * (d + 1) + d] = count.
__global__ void segsum_kernel(const float* X, const uint32_t* lists, const int64_t* offs, int k,
                              int d, const float* init, float* out) {
  const int c = blockIdx.x;
  if (c >= k) return;
  const int64_t b = offs[c], e = offs[c + 1];
  const float* in = init ? init + static_cast<int64_t>(c) * (d + 1) : nullptr;
  for (int c4 = threadIdx.x; c4 < d / 4; c4 += blockDim.x) {
    // continue the accumulators of the rows before this shard (exact
    // multi-rank update) or start from zero
    float4 s = in ? make_float4(in[c4 * 4], in[c4 * 4 + 1], in[c4 * 4 + 2], in[c4 * 4 + 3])
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t j = b; j < e; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(X + static_cast<int64_t>(lists[j]) * d + c4 * 4);
      s.x = __fadd_rn(s.x, v.x);
      s.y = __fadd_rn(s.y, v.y);
      s.z = __fadd_rn(s.z, v.z);
      s.w = __fadd_rn(s.w, v.w);
    }
    float* o = out + static_cast<int64_t>(c) * (d + 1) + c4 * 4;
    o[0] = s.x;
    o[1] = s.y;
    o[2] = s.z;
    o[3] = s.w;
  }
  // the count continues in float: exact while a cluster holds fewer than
  // 2^24 rows of the sample
  if (threadIdx.x == 0)
    out[static_cast<int64_t>(c) * (d + 1) + d] = (in ? in[d] : 0.f) + static_cast<float>(e - b);
}

// centroid = sum / count for non-empty clusters (ann.lisp:116-122)
__global__ void update_kernel(const float* sums, int k, int d, float* cent) {
  const int c = blockIdx.x;
  if (c >= k) return;
  const float cnt = sums[static_cast<int64_t>(c) * (d + 1) + d];
  if (!(cnt > 0.f)) return;
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    cent[static_cast<int64_t>(c) * d + i] = __fdiv_rn(sums[static_cast<int64_t>(c) * (d + 1) + i], cnt);
}

// --------------------------------------------------------------- search --
__device__ __forceinline__ unsigned long long warp_min_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w < v ? w : v;
  }
  return v;
}

// block-wide min of one key per thread (blockDim multiple of 32, <= 1024)
__device__ unsigned long long block_min_u64(unsigned long long v, unsigned long long* red) {
  v = warp_min_u64(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : ~0ull;
    v = warp_min_u64(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// top nprobe centroids of each query: score desc, index asc (stable sort of
// kb.lisp:353).  One block per query, bitonic sort of k <= 8192 keys.
// The nprobe best centroids of query q in (score desc, index asc) order --
// the first nprobe of kb.lisp:352's sort -- without sorting all k: a radix
// select finds the nprobe-th smallest key (8 bits per pass over the 32-bit
// score key, then over the index among equal scores), the keys at or below
// it are gathered and only those are sorted.  One block of 256 threads per
// query, k <= 8192 (32 keys per thread in registers).
constexpr int kSelThreads = 256;
constexpr int kSelPer = 32;

__device__ __forceinline__ uint32_t score_key32(float s) {
  return static_cast<uint32_t>(desc_key(s, 0u) >> 32);
}

// bin of the 256-bin histogram where the running count reaches `need`;
// warp 0 only; writes (bin, count before it, count in it)
__device__ __forceinline__ void sel_find(const uint32_t* hist, uint32_t need, uint32_t* out) {
  const int lane = threadIdx.x & 31;
  uint32_t c[8], sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c[j] = hist[8 * lane + j];
    sum += c[j];
  }
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  const uint32_t excl = incl - sum;
  if (excl < need && need <= incl) {
    uint32_t run = excl;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (run + c[j] >= need) {
        out[0] = 8 * lane + j;
        out[1] = run;
        out[2] = c[j];
        break;
      }
      run += c[j];
    }
  }
}

struct SelSmem {
  uint32_t* hist;  // [256]
  uint32_t* found; // [3]
  int* nsel;
};

// One 8-bit radix pass over the fields f(m) (m < nv) with (f & mask) ==
// prefix, one warp atomic per distinct bin; returns (bin, count below it).
template <class F>
__device__ __forceinline__ uint2 sel_pass(F field, int nv, uint32_t mask, uint32_t prefix, int shift,
                                          uint32_t need, const SelSmem& sm, uint32_t* in_bin = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31;
  sm.hist[tid] = 0;
  __syncthreads();
#pragma unroll
  for (int m = 0; m < kSelPer; ++m) {
    const uint32_t f = field(m);
    const bool on = m < nv && (f & mask) == prefix;
    const uint32_t bin = on ? (f >> shift) & 255u : 256u;
    const unsigned grp = __match_any_sync(0xffffffffu, bin);
    if (on && lane == __ffs(grp) - 1) atomicAdd(&sm.hist[bin], static_cast<uint32_t>(__popc(grp)));
  }
  __syncthreads();
  if (tid < 32) sel_find(sm.hist, need, sm.found);
  __syncthreads();
  const uint2 r = make_uint2(sm.found[0], sm.found[1]);
  if (in_bin) *in_bin = sm.found[2];
  __syncthreads();  // found[] is rewritten by the next pass
  return r;
}

// The 32-bit key v of the need-th smallest of key[m] (m < nv); *left = how
// many keys equal to v are among the need smallest, *equal = how many keys
// equal v in all.
__device__ __forceinline__ uint32_t sel_kth(const uint32_t (&key)[kSelPer], int nv, uint32_t need,
                                            const SelSmem& sm, uint32_t* left, uint32_t* equal) {
  uint32_t prefix = 0, mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    const uint2 r = sel_pass([&](int m) { return key[m]; }, nv, mask, prefix, shift, need, sm, equal);
    prefix |= r.x << shift;
    mask |= 0xffu << shift;
    need -= r.y;
  }
  *left = need;
  return prefix;
}

// Ascending bitonic sort of sel[0, P) (P a power of two), whole block.
__device__ __forceinline__ void sel_sort(unsigned long long* sel, int P) {
  const int tid = threadIdx.x;
  for (int size = 2; size <= P; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += kSelThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const unsigned long long a = sel[i], b = sel[j];
          if ((a > b) == up) {
            sel[i] = b;
            sel[j] = a;
          }
        }
      }
      __syncthreads();
    }
}

// Writes the indices of the nprobe smallest (key[m], index tid + 256 m) to
// out[0, nprobe) in order; sel needs pow2(nprobe) slots.
__device__ void select_emit(const uint32_t (&key)[kSelPer], int nv, int nprobe, const SelSmem& sm,
                            unsigned long long* sel, int32_t* out) {
  const int tid = threadIdx.x;
  uint32_t need, equal;
  const uint32_t v = sel_kth(key, nv, static_cast<uint32_t>(nprobe), sm, &need, &equal);
  // among the keys equal to v, the `need` lowest indices: index <= ip (all
  // of them, without the index passes, when every key equal to v is kept)
  uint32_t ip = 0, imask = 0;
  if (need == equal) ip = 0xffffffffu;
  for (int shift = 8; need != equal && shift >= 0; shift -= 8) {
    const uint2 r = sel_pass(
        [&](int m) { return key[m] == v ? static_cast<uint32_t>(tid + kSelThreads * m) : 0xffffffffu; }, nv,
        imask | 0xffff0000u, ip, shift, need, sm);
    ip |= r.x << shift;
    imask |= 0xffu << shift;
    need -= r.y;
  }
  int P = 1;
  while (P < nprobe) P <<= 1;
  if (tid == 0) *sm.nsel = 0;
  for (int i = tid; i < P; i += kSelThreads) sel[i] = ~0ull;
  __syncthreads();
#pragma unroll
  for (int m = 0; m < kSelPer; ++m) {
    const uint32_t idx = static_cast<uint32_t>(tid + kSelThreads * m);
    if (m < nv && (key[m] < v || (key[m] == v && idx <= ip)))
      sel[atomicAdd(sm.nsel, 1)] = (static_cast<unsigned long long>(key[m]) << 32) | idx;
  }
  __syncthreads();
  sel_sort(sel, P);
  for (int i = tid; i < nprobe; i += kSelThreads) out[i] = static_cast<int32_t>(sel[i] & 0xffffffffu);
}

__global__ void __launch_bounds__(kSelThreads) probe_select_kernel(const float* S, int k, int nprobe,
                                                                   int32_t* probes) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t found[3];
  __shared__ int nsel;
  extern __shared__ unsigned long long sel[];  // [P2], P2 = pow2 >= nprobe
  const int64_t q = blockIdx.x;
  const float* sq = S + q * k;
  const int tid = threadIdx.x;
  const int nv = tid < k ? (k - tid + kSelThreads - 1) / kSelThreads : 0;  // keys of this thread
  uint32_t key[kSelPer];
#pragma unroll
  for (int m = 0; m < kSelPer; ++m) key[m] = m < nv ? score_key32(sq[tid + kSelThreads * m]) : 0u;
  select_emit(key, nv, nprobe, SelSmem{hist, found, &nsel}, sel, probes + q * nprobe);
}

// ---- probe selection from tensor-core scores --------------------------------
// S holds bf16-operand tcgen05 scores (fp32 accumulation) of query q against
// every centroid; |S - exact| <= w / 2 with w = rel2 |q| max|c| (the bound of
// the k-means assignment window, qnorm and cmax upper bounds of the norms).
// With t the approximate nprobe-th largest score, every centroid of the exact
// first nprobe has S >= t - w, and every centroid below t - w has an exact
// score below the exact nprobe-th.  So the candidates S >= t - w are
// re-scored with the reference's sequential single-float dot, sorted by
// (exact score desc, index asc), and the first nprobe are exactly
// kb.lisp:352's.  A query with more than kTcCand candidates, or a window that
// is not a finite number, scores every centroid exactly instead.
constexpr int kTcCand = 256;

__device__ __forceinline__ float key32_score(uint32_t v) {
  return key_score(static_cast<unsigned long long>(v) << 32);
}

__device__ __forceinline__ float exact_dot(const float* qs, const float* c, int d) {
  const float4* c4 = reinterpret_cast<const float4*>(c);
  float acc = 0.f;
  for (int j = 0; j < d; j += 4) {
    const float4 x = __ldg(c4 + (j >> 2));
    acc = __fadd_rn(acc, __fmul_rn(qs[j], x.x));
    acc = __fadd_rn(acc, __fmul_rn(qs[j + 1], x.y));
    acc = __fadd_rn(acc, __fmul_rn(qs[j + 2], x.z));
    acc = __fadd_rn(acc, __fmul_rn(qs[j + 3], x.w));
  }
  return acc;
}

__global__ void __launch_bounds__(kSelThreads) probe_select_tc_kernel(
    const float* S, const float* Q, const float* C, const float* qnorm, const float* cmax, float rel2, int k,
    int d, int nprobe, int32_t* probes) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t found[3];
  __shared__ int nsel, ncand;
  extern __shared__ __align__(16) unsigned char tc_sm[];
  unsigned long long* sel = reinterpret_cast<unsigned long long*>(tc_sm);  // [max(kTcCand, pow2(nprobe))]
  int P2 = 1;
  while (P2 < nprobe) P2 <<= 1;
  const int nsel_slots = P2 > kTcCand ? P2 : kTcCand;
  int* cand = reinterpret_cast<int*>(sel + nsel_slots);  // [kTcCand]
  float* qs = reinterpret_cast<float*>(cand + kTcCand);  // [d]
  const SelSmem sm{hist, found, &nsel};
  const int64_t q = blockIdx.x;
  const float* sq = S + q * k;
  const int tid = threadIdx.x;
  for (int j = tid; j < d; j += kSelThreads) qs[j] = Q[q * d + j];
  const int nv = tid < k ? (k - tid + kSelThreads - 1) / kSelThreads : 0;
  uint32_t key[kSelPer];
#pragma unroll
  for (int m = 0; m < kSelPer; ++m) key[m] = m < nv ? score_key32(sq[tid + kSelThreads * m]) : 0u;
  uint32_t left, equal;
  const float t = key32_score(sel_kth(key, nv, static_cast<uint32_t>(nprobe), sm, &left, &equal));
  const float w = __fmul_ru(__fmul_ru(rel2, qnorm[q]), *cmax);
  const float lo = __fsub_rd(t, w);
  bool ok = w >= 0.f && w < INFINITY && lo > -INFINITY && lo < INFINITY;  // block-uniform
  if (tid == 0) ncand = 0;
  __syncthreads();
  if (ok) {
#pragma unroll
    for (int m = 0; m < kSelPer; ++m)
      if (m < nv && key32_score(key[m]) >= lo) {
        const int p = atomicAdd(&ncand, 1);
        if (p < kTcCand) cand[p] = tid + kSelThreads * m;
      }
  }
  __syncthreads();
  const int n = ncand;
  ok = ok && n <= kTcCand && n >= nprobe;
  if (ok) {
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = tid; i < P; i += kSelThreads) {
      unsigned long long v = ~0ull;
      if (i < n) {
        const int c = cand[i];
        v = (static_cast<unsigned long long>(score_key32(exact_dot(qs, C + static_cast<int64_t>(c) * d, d)))
             << 32) |
            static_cast<uint32_t>(c);
      }
      sel[i] = v;
    }
    __syncthreads();
    sel_sort(sel, P);
    for (int i = tid; i < nprobe; i += kSelThreads)
      probes[q * nprobe + i] = static_cast<int32_t>(sel[i] & 0xffffffffu);
  } else {
#pragma unroll
    for (int m = 0; m < kSelPer; ++m)
      if (m < nv)
        key[m] = score_key32(exact_dot(qs, C + static_cast<int64_t>(tid + kSelThreads * m) * d, d));
    select_emit(key, nv, nprobe, sm, sel, probes + q * nprobe);
  }
}

// Exact scores of `cnt` rows against one query, top `topk` by (score desc,
// position asc), merged into a running list in smem.  rows_of(pos) maps a
// position to a row id.  Shared by the list scan and the flat scan.
template <bool kIndirect>
__device__ void scan_rows(const float* X, int d, const uint32_t* lists, int64_t start, int64_t cnt,
                          const float* qs, int topk, unsigned long long* best,
                          unsigned long long* tile, unsigned long long* red) {
  constexpr int TILE = 2048;
  for (int64_t t0 = 0; t0 < cnt; t0 += TILE) {
    const int m = static_cast<int>(cnt - t0 < TILE ? cnt - t0 : TILE);
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      const int64_t p = t0 + i;
      const int64_t row = kIndirect ? static_cast<int64_t>(lists[start + p]) : start + p;
      const float4* xr = reinterpret_cast<const float4*>(X + row * d);
      float s = 0.f;
      // the row in register chunks of 8 x 16 bytes, all loads of a chunk in
      // flight before its adds (which stay one sequential chain)
      const int d4 = d / 4;
      for (int c0 = 0; c0 < d4; c0 += 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = c0 + u < d4 ? xr[c0 + u] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (c0 + u < d4) {
            const float* qq = qs + 4 * (c0 + u);
            s = __fadd_rn(s, __fmul_rn(v[u].x, qq[0]));
            s = __fadd_rn(s, __fmul_rn(v[u].y, qq[1]));
            s = __fadd_rn(s, __fmul_rn(v[u].z, qq[2]));
            s = __fadd_rn(s, __fmul_rn(v[u].w, qq[3]));
          }
        }
      }
      tile[i] = desc_key(s, static_cast<uint32_t>(p));
    }
    // append the running best as candidates (their positions are smaller)
    for (int i = threadIdx.x; i < topk; i += blockDim.x) tile[m + i] = best[i];
    __syncthreads();
    const int tot = m + topk;
    for (int r = 0; r < topk; ++r) {
      unsigned long long mine = ~0ull;
      int at = -1;
      for (int i = threadIdx.x; i < tot; i += blockDim.x)
        if (tile[i] < mine) {
          mine = tile[i];
          at = i;
        }
      const unsigned long long w = block_min_u64(mine, red);
      if (w == mine && at >= 0 && w != ~0ull) tile[at] = ~0ull;  // keys are unique
      if (threadIdx.x == 0) best[r] = w;
      __syncthreads();
    }
  }
}

// scan_rows with the rows staged in shared memory: per pass of up to kStageRows
// rows, thread i copies row i with one untiled bulk copy (all on one
// mbarrier), the block waits once (bounded), then thread i runs row i's
// sequential sum from shared memory -- one memory latency per pass instead
// of one per 128 bytes of every row.  Rows padded to an odd number of
// 16-byte pieces.  Same keys, same top-k as scan_rows.
constexpr int kStageRows = 64;

template <bool kIndirect>
__device__ void scan_rows_staged(const float* X, int d, const uint32_t* lists, int64_t start, int64_t cnt,
                                 const float* qs, int topk, unsigned long long* best,
                                 unsigned long long* tile, unsigned long long* red, float* stage,
                                 uint64_t* bar, unsigned* status) {
  const int ld = 4 * ((d >> 2) | 1);
  const uint32_t row_bytes = static_cast<uint32_t>(d) * 4u;
  uint32_t phase = 0;
  for (int64_t t0 = 0; t0 < cnt; t0 += kStageRows) {
    const int m = static_cast<int>(cnt - t0 < kStageRows ? cnt - t0 : kStageRows);
    if (threadIdx.x == 0) mbar_arrive_expect_tx(bar, row_bytes * static_cast<uint32_t>(m));
    // the previous pass's reads of the staging rows are done (the barrier
    // ending its top-k round) before the copies overwrite them
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x < m) {
      const int64_t p = t0 + threadIdx.x;
      const int64_t row = kIndirect ? static_cast<int64_t>(lists[start + p]) : start + p;
      bulk_load(stage + threadIdx.x * ld, X + row * d, row_bytes, bar);
    }
    if (!__syncthreads_and(mbar_wait(bar, phase, nullptr))) {
      if (threadIdx.x == 0) report(status, kDevTimeoutOther);
      mbar_wait(bar, phase, nullptr);  // the copies in flight land first
      return;
    }
    phase ^= 1u;
    if (threadIdx.x < m) {
      const float4* xr = reinterpret_cast<const float4*>(stage + threadIdx.x * ld);
      float s = 0.f;
      const int d4 = d / 4;
#pragma unroll 4
      for (int c4 = 0; c4 < d4; ++c4) {
        const float4 v = xr[c4];
        const float* qq = qs + 4 * c4;
        s = __fadd_rn(s, __fmul_rn(v.x, qq[0]));
        s = __fadd_rn(s, __fmul_rn(v.y, qq[1]));
        s = __fadd_rn(s, __fmul_rn(v.z, qq[2]));
        s = __fadd_rn(s, __fmul_rn(v.w, qq[3]));
      }
      tile[threadIdx.x] = desc_key(s, static_cast<uint32_t>(t0 + threadIdx.x));
    }
    // append the running best as candidates (their positions are smaller)
    for (int i = threadIdx.x; i < topk; i += blockDim.x) tile[m + i] = best[i];
    __syncthreads();
    const int tot = m + topk;
    for (int r = 0; r < topk; ++r) {
      unsigned long long mine = ~0ull;
      int at = -1;
      for (int i = threadIdx.x; i < tot; i += blockDim.x)
        if (tile[i] < mine) {
          mine = tile[i];
          at = i;
        }
      const unsigned long long w = block_min_u64(mine, red);
      if (w == mine && at >= 0 && w != ~0ull) tile[at] = ~0ull;  // keys are unique
      if (threadIdx.x == 0) best[r] = w;
      __syncthreads();
    }
  }
}

// list_scan_kernel with the staged row loads (d % 4 == 0, 16-byte aligned X)
__global__ void list_scan_staged_kernel(const float* X, int d, const uint32_t* lists, const int64_t* offs,
                                        const int32_t* probes, int nprobe, const float* Q, int topk,
                                        unsigned long long* cand, unsigned* status) {
  extern __shared__ __align__(16) unsigned long long sm[];
  unsigned long long* best = sm;              // [64]
  unsigned long long* red = best + 64;        // [32]
  unsigned long long* tile = red + 32;        // [kStageRows + 64]
  uint64_t* bar = reinterpret_cast<uint64_t*>(tile + kStageRows + 64);  // [2] (16-byte slot)
  float* qs = reinterpret_cast<float*>(bar + 2);
  float* stage = qs + ((d + 3) & ~3);         // 16-byte aligned
  const int p = blockIdx.x;
  const int64_t q = blockIdx.y;
  for (int i = threadIdx.x; i < d; i += blockDim.x) qs[i] = Q[q * d + i];
  for (int i = threadIdx.x; i < topk; i += blockDim.x) best[i] = ~0ull;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int c = probes[q * nprobe + p];
  const int parts = static_cast<int>(gridDim.z), z = static_cast<int>(blockIdx.z);
  const int64_t len = offs[c + 1] - offs[c];
  const int64_t per = (len + parts - 1) / parts;
  const int64_t pb = per * z < len ? per * z : len;
  const int64_t cnt = len - pb < per ? len - pb : per;
  scan_rows_staged<true>(X, d, lists, offs[c] + pb, cnt, qs, topk, best, tile, red, stage, bar, status);
  for (int i = threadIdx.x; i < topk; i += blockDim.x) {
    const unsigned long long kk = best[i];
    cand[((q * nprobe + p) * parts + z) * topk + i] =
        kk == ~0ull ? ~0ull
                    : (kk & 0xffffffff00000000ull) |
                          lists[offs[c] + pb + static_cast<int64_t>(kk & 0xffffffffu)];
  }
}

// grid (nprobe, nq): top-k of list probes[q][p] for query q.
// cand[(q * nprobe + p) * topk + r] = key with tiebreak = position in list.
// grid (nprobe, nq, parts): part z of the z-th probed list of query q; its
// candidates are group p * parts + z, so the merge's (group, rank) order is
// (probe rank, list position) as with one part per list
__global__ void list_scan_kernel(const float* X, int d, const uint32_t* lists, const int64_t* offs,
                                 const int32_t* probes, int nprobe, const float* Q, int topk,
                                 unsigned long long* cand) {
  extern __shared__ unsigned long long sm[];
  unsigned long long* best = sm;              // [topk]
  unsigned long long* red = best + 64;        // [32]
  unsigned long long* tile = red + 32;        // [2048 + topk]
  float* qs = reinterpret_cast<float*>(tile + 2048 + 64);
  const int p = blockIdx.x;
  const int64_t q = blockIdx.y;
  for (int i = threadIdx.x; i < d; i += blockDim.x) qs[i] = Q[q * d + i];
  for (int i = threadIdx.x; i < topk; i += blockDim.x) best[i] = ~0ull;
  __syncthreads();
  const int c = probes[q * nprobe + p];
  const int parts = static_cast<int>(gridDim.z), z = static_cast<int>(blockIdx.z);
  const int64_t len = offs[c + 1] - offs[c];
  const int64_t per = (len + parts - 1) / parts;
  const int64_t pb = per * z < len ? per * z : len;
  const int64_t cnt = len - pb < per ? len - pb : per;
  scan_rows<true>(X, d, lists, offs[c] + pb, cnt, qs, topk, best, tile, red);
  for (int i = threadIdx.x; i < topk; i += blockDim.x) {
    const unsigned long long kk = best[i];
    // replace the position by the row id (kept for the merge)
    cand[((q * nprobe + p) * parts + z) * topk + i] =
        kk == ~0ull ? ~0ull
                    : (kk & 0xffffffff00000000ull) |
                          lists[offs[c] + pb + static_cast<int64_t>(kk & 0xffffffffu)];
  }
}

// grid (nchunks, nq): top-k of rows [chunk * rows_per, ...) for query q
__global__ void flat_scan_kernel(const float* X, int64_t n, int d, int64_t rows_per, const float* Q,
                                 int topk, unsigned long long* cand) {
  extern __shared__ unsigned long long sm[];
  unsigned long long* best = sm;
  unsigned long long* red = best + 64;
  unsigned long long* tile = red + 32;
  float* qs = reinterpret_cast<float*>(tile + 2048 + 64);
  const int64_t ch = blockIdx.x;
  const int64_t q = blockIdx.y;
  for (int i = threadIdx.x; i < d; i += blockDim.x) qs[i] = Q[q * d + i];
  for (int i = threadIdx.x; i < topk; i += blockDim.x) best[i] = ~0ull;
  __syncthreads();
  const int64_t s = ch * rows_per;
  const int64_t cnt = s >= n ? 0 : (n - s < rows_per ? n - s : rows_per);
  scan_rows<false>(X, d, nullptr, s, cnt, qs, topk, best, tile, red);
  for (int i = threadIdx.x; i < topk; i += blockDim.x) {
    const unsigned long long kk = best[i];
    cand[(q * gridDim.x + ch) * topk + i] =
        kk == ~0ull ? ~0ull : (kk & 0xffffffff00000000ull) | static_cast<uint32_t>(s + (kk & 0xffffffffu));
  }
}

// Final top-k per query over ngroups x topk candidates.  Order: score desc,
// then group (probe rank / chunk) asc, then the candidate's rank inside its
// group -- the stable merge of kb.lisp:363 and :199.
__global__ void merge_kernel(const unsigned long long* cand, int ngroups, int topk, int64_t* ids,
                             float* scores) {
  extern __shared__ unsigned long long mk[];
  unsigned long long* keys = mk + 32;
  const int64_t q = blockIdx.x;
  const int tot = ngroups * topk;
  const int nw = blockDim.x >> 5;
  // the candidates' row ids, so the final picks read no global memory
  uint32_t* rid = reinterpret_cast<uint32_t*>(keys + tot + nw * topk);
#pragma unroll 4
  for (int i = threadIdx.x; i < tot; i += blockDim.x) {
    const unsigned long long c = cand[q * tot + i];
    // re-key: score bits high, then flat index (group * topk + rank) low
    keys[i] = c == ~0ull ? ~0ull : ((c & 0xffffffff00000000ull) | static_cast<uint32_t>(i));
    rid[i] = static_cast<uint32_t>(c & 0xffffffffu);
  }
  __syncthreads();
  // each warp takes the topk smallest keys of its slice (no block barrier
  // per round), then warp 0 takes the topk smallest of the warps' lists;
  // keys are unique, so the result is the same as one pass over all keys
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int per = (tot + nw - 1) / nw;
  const int b = min(tot, wid * per), e = min(tot, b + per);
  unsigned long long* wtop = keys + tot;  // [nw][topk]
  for (int r = 0; r < topk; ++r) {
    unsigned long long mine = ~0ull;
    int at = -1;
    for (int i = b + lane; i < e; i += 32)
      if (keys[i] < mine) {
        mine = keys[i];
        at = i;
      }
    const unsigned long long w = warp_min_u64(mine);
    if (w == mine && at >= 0 && w != ~0ull) keys[at] = ~0ull;
    if (lane == 0) wtop[wid * topk + r] = w;
    __syncwarp();
  }
  __syncthreads();
  if (wid != 0) return;
  const int tw = nw * topk;
  for (int r = 0; r < topk; ++r) {
    unsigned long long mine = ~0ull;
    int at = -1;
    for (int i = lane; i < tw; i += 32)
      if (wtop[i] < mine) {
        mine = wtop[i];
        at = i;
      }
    const unsigned long long w = warp_min_u64(mine);
    if (w == mine && at >= 0 && w != ~0ull) wtop[at] = ~0ull;
    if (lane == 0) {
      if (w == ~0ull) {
        ids[q * topk + r] = -1;
        scores[q * topk + r] = -FLT_MAX;
      } else {
        // the key keeps the candidate's score bits above its flat index
        ids[q * topk + r] = static_cast<int64_t>(rid[static_cast<int>(w & 0xffffffffu)]);
        scores[q * topk + r] = key_score(w);
      }
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------- launchers --
cudaError_t launch_assign(const float* X, const int64_t* rows, int64_t n, const float* C, int k, int d,
                          int32_t* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t grid = (n + SB - 1) / SB;
  assign_kernel<<<static_cast<unsigned>(grid), 256, 0, st>>>(X, rows, n, C, k, d, out);
  return cudaGetLastError();
}

cudaError_t launch_scores(const float* Q, int64_t nq, const float* C, int k, int d, float* S,
                          cudaStream_t st, unsigned* status) {
  if (nq <= 0) return cudaSuccess;
  if (nq <= kSmallQ && d % 4 == 0 && ((reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(Q)) & 15) == 0) {
    const size_t sm = (static_cast<size_t>(kScoreRows) * 4 * ((d / 4) | 1) + static_cast<size_t>(nq) * d) * 4;
    constexpr size_t kMaxSm = 160 * 1024;
    if (sm <= kMaxSm) {
      // (set on every call: the attribute belongs to the current device)
      if (cudaFuncSetAttribute(scores_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kMaxSm)) == cudaSuccess) {
        scores_rows_kernel<<<static_cast<unsigned>((k + kScoreRows - 1) / kScoreRows), 32, sm, st>>>(
            Q, static_cast<int>(nq), C, k, d, S, status);
        return cudaGetLastError();
      }
      cudaGetLastError();
    }
  }
  if (nq <= kSmallQ && d % 4 == 0 && static_cast<size_t>(nq) * d * sizeof(float) <= 48 * 1024 &&
      (reinterpret_cast<uintptr_t>(C) & 15) == 0) {
    scores_small_kernel<<<static_cast<unsigned>((k + 127) / 128), 128,
                          static_cast<size_t>(nq) * d * sizeof(float), st>>>(Q, static_cast<int>(nq), C, k, d, S);
    return cudaGetLastError();
  }
  dim3 grid(static_cast<unsigned>((nq + SB - 1) / SB), static_cast<unsigned>((k + SB - 1) / SB));
  scores_kernel<<<grid, 256, 0, st>>>(Q, nq, C, k, d, S);
  return cudaGetLastError();
}

int64_t sort_tiles(int64_t n) { return (n + kSortTile - 1) / kSortTile; }

cudaError_t launch_lists(const int32_t* a, int64_t n, int k, uint32_t* tile_hist, uint32_t* counts,
                         int64_t* offs, uint32_t base, uint32_t* lists, cudaStream_t st) {
  const int64_t nt = sort_tiles(n);
  const size_t hsm = static_cast<size_t>(k) * 4;
  if (hsm > 200 * 1024) return cudaErrorInvalidValue;
  if (hsm > 48 * 1024) {
    cudaFuncSetAttribute(hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(hsm));
    cudaFuncSetAttribute(scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(hsm));
  }
  if (nt > 0) hist_kernel<<<static_cast<unsigned>(nt), 256, hsm, st>>>(a, n, k, tile_hist);
  colsum_seg_kernel<<<(k + 31) / 32, 256, 0, st>>>(tile_hist, static_cast<int>(nt), k, counts);
  scan_kernel<<<1, 1024, 0, st>>>(counts, k, offs);
  tile_offsets_seg_kernel<<<(k + 31) / 32, 256, 0, st>>>(tile_hist, static_cast<int>(nt), k, offs);
  // eight warps per tile while their histograms fit in shared memory
  const size_t wsm = static_cast<size_t>(kScatWarps) * k * 4;
  if (nt > 0 && wsm <= 200 * 1024) {
    if (wsm > 48 * 1024)
      cudaFuncSetAttribute(scatter_cta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(wsm));
    scatter_cta_kernel<<<static_cast<unsigned>(nt), 256, wsm, st>>>(a, n, k, tile_hist, base, lists);
  } else if (nt > 0) {
    scatter_kernel<<<static_cast<unsigned>(nt), 32, hsm, st>>>(a, n, k, tile_hist, base, lists);
  }
  return cudaGetLastError();
}

cudaError_t launch_segsum(const float* X, const uint32_t* lists, const int64_t* offs, int k, int d,
                          const float* init, float* out, cudaStream_t st) {
  int th = d / 4;
  th = th < 32 ? 32 : (th > 256 ? 256 : ((th + 31) / 32) * 32);
  segsum_kernel<<<k, th, 0, st>>>(X, lists, offs, k, d, init, out);
  return cudaGetLastError();
}

cudaError_t launch_update(const float* sums, int k, int d, float* cent, cudaStream_t st) {
  update_kernel<<<k, 128, 0, st>>>(sums, k, d, cent);
  return cudaGetLastError();
}

cudaError_t launch_probe_select(const float* S, int64_t nq, int k, int nprobe, int32_t* probes,
                                cudaStream_t st) {
  if (k > kSelThreads * kSelPer || nprobe < 1 || nprobe > k) return cudaErrorInvalidValue;
  int P = 1;
  while (P < nprobe) P <<= 1;
  const size_t sm = static_cast<size_t>(P) * 8;
  cudaFuncSetAttribute(probe_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  probe_select_kernel<<<static_cast<unsigned>(nq), kSelThreads, sm, st>>>(S, k, nprobe, probes);
  return cudaGetLastError();
}

cudaError_t launch_probe_select_tc(const float* S, const float* Q, const float* C, const float* qnorm,
                                   const float* cmax, float rel2, int64_t nq, int k, int d, int nprobe,
                                   int32_t* probes, cudaStream_t st) {
  if (k > kSelThreads * kSelPer || nprobe < 1 || nprobe > k || d % 4) return cudaErrorInvalidValue;
  int P = 1;
  while (P < nprobe) P <<= 1;
  const size_t sm = static_cast<size_t>(P > kTcCand ? P : kTcCand) * 8 + kTcCand * 4 + static_cast<size_t>(d) * 4;
  if (sm > 200 * 1024) return cudaErrorInvalidValue;
  cudaFuncSetAttribute(probe_select_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  probe_select_tc_kernel<<<static_cast<unsigned>(nq), kSelThreads, sm, st>>>(S, Q, C, qnorm, cmax, rel2, k, d,
                                                                            nprobe, probes);
  return cudaGetLastError();
}

static size_t scan_smem(int d) { return (64 + 32 + 2048 + 64) * 8 + static_cast<size_t>(d) * 4; }

cudaError_t launch_list_scan(const float* X, int d, const uint32_t* lists, const int64_t* offs,
                             const int32_t* probes, int nprobe, const float* Q, int64_t nq, int topk,
                             int parts, unsigned long long* cand, cudaStream_t st, unsigned* status) {
  if (parts < 1) return cudaErrorInvalidValue;
  if (d % 4 == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0 && topk <= 64) {
    const size_t sm = (64 + 32 + kStageRows + 64 + 2) * 8 + static_cast<size_t>((d + 3) & ~3) * 4 +
                      static_cast<size_t>(kStageRows) * 4 * ((d / 4) | 1) * 4;
    if (sm <= 160 * 1024 &&
        cudaFuncSetAttribute(list_scan_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sm)) == cudaSuccess) {
      dim3 grid(nprobe, static_cast<unsigned>(nq), static_cast<unsigned>(parts));
      list_scan_staged_kernel<<<grid, 256, sm, st>>>(X, d, lists, offs, probes, nprobe, Q, topk, cand, status);
      return cudaGetLastError();
    }
    cudaGetLastError();
  }
  const size_t sm = scan_smem(d);
  cudaFuncSetAttribute(list_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  dim3 grid(nprobe, static_cast<unsigned>(nq), static_cast<unsigned>(parts));
  list_scan_kernel<<<grid, 256, sm, st>>>(X, d, lists, offs, probes, nprobe, Q, topk, cand);
  return cudaGetLastError();
}

cudaError_t launch_flat_scan(const float* X, int64_t n, int d, int nchunks, const float* Q, int64_t nq,
                             int topk, unsigned long long* cand, cudaStream_t st) {
  const size_t sm = scan_smem(d);
  cudaFuncSetAttribute(flat_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  const int64_t rows_per = (n + nchunks - 1) / nchunks;
  dim3 grid(nchunks, static_cast<unsigned>(nq));
  flat_scan_kernel<<<grid, 256, sm, st>>>(X, n, d, rows_per, Q, topk, cand);
  return cudaGetLastError();
}

cudaError_t launch_merge(const unsigned long long* cand, int64_t nq, int ngroups, int topk, int64_t* ids,
                         float* scores, cudaStream_t st) {
  // keys, the eight warps' lists, then the row ids
  const size_t sm = (32 + static_cast<size_t>(ngroups) * topk + 8 * static_cast<size_t>(topk)) * 8 +
                    static_cast<size_t>(ngroups) * topk * 4;
  if (sm > 200 * 1024) return cudaErrorInvalidValue;
  cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  merge_kernel<<<static_cast<unsigned>(nq), 256, sm, st>>>(cand, ngroups, topk, ids, scores);
  return cudaGetLastError();
}

}  // namespace ec
