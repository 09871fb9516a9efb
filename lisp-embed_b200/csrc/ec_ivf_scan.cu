// ec_ivf_scan.cu -- query-batched exact scans for IVF and flat search.
//
// kb::top-k-ivf (kb.lisp:348-364) scores every row of each probed list
// against the query with the sequential single-float dot of kb.lisp:153-162
// and keeps the list's top k by strict `>` (earlier position wins a tie);
// kb::top-k-brute (kb.lisp:164-200) does the same over contiguous ranges.
// Scanning one (query, list) pair per CTA re-reads each list once per query
// that probes it, and every row is one dependent 384-step chain.  Here a
// batch of queries is regrouped by list first (counting sort of the
// (query, probe) pairs), so that one CTA scores one list against up to 32 of
// the queries that probe it: each thread owns 4 queries x 4 rows of a 128-row
// tile, and the rows stream through shared memory in 16-column chunks with
// cp.async.  Every score is still the same sequential chain of
// separately rounded products and sums (__fmul_rn / __fadd_rn, in column
// order), so scores are bit-identical to the reference's; the per-pair
// top-k keeps the (score desc, position asc) order with a threshold filter
// and a rank merge.  Output is the per-(query, group) candidate layout that
// the merge kernel in ec_ivf_kernels.cu reads.
#include <algorithm>
#include <cstdint>

#include "ec_ivf.h"

namespace ec {

namespace {

constexpr int kTsLanes = 32;   // queries per CTA
// each thread: 4 queries x RW rows.  lane = rg * 8 + qg: query group qg
// (queries 4 qg .. 4 qg + 3), row group rg (rows RW rg .. RW rg + RW - 1 of
// the warp's 4 RW); a warp covers all 32 queries, the CTA WARPS x 4 x RW =
// 128 rows.  Each 16-byte shared-memory load feeds 4 RW (query operand) or
// 16 (row operand) multiply-adds per lane: (4 + RW) x 16 bytes of register
// writeback per 16 RW multiply-adds.
constexpr int kTsQW = 4;
constexpr int kTsWarps = 8, kTsRW = 4;  // the configuration launched
constexpr int kTsRows = 128;            // rows per tile
constexpr int kTsChunk = 16;                   // columns per pipeline stage
constexpr int kTsStages = 3;
constexpr int kTsHalf = kTsRows / 2;           // candidates per query per round

__device__ __forceinline__ unsigned long long ts_key(float s, uint32_t tie) {
  s = s + 0.0f;  // -0.0 -> +0.0 (they compare equal in the reference)
  uint32_t u = __float_as_uint(s);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(~u) << 32) | tie;
}

__device__ __forceinline__ void ts_cp16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void ts_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void ts_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// acc = acc + x * q, column by column (the reference's rounding order)
__device__ __forceinline__ float ts_dot4(float acc, const float4& x, const float4& q) {
  acc = __fadd_rn(acc, __fmul_rn(x.x, q.x));
  acc = __fadd_rn(acc, __fmul_rn(x.y, q.y));
  acc = __fadd_rn(acc, __fmul_rn(x.z, q.z));
  acc = __fadd_rn(acc, __fmul_rn(x.w, q.w));
  return acc;
}

struct TileScanArgs {
  const float* X;
  int d;
  // IVF: rows of list c are lists[offs[c] .. offs[c + 1]); pairs grouped by
  // list: pairs[pair_off[c] .. pair_off[c + 1]) = q * ngroups + probe rank,
  // work items of list c: item_off[c] .. item_off[c + 1]
  const uint32_t* lists;
  const int64_t* offs;
  const int32_t* pair_off;
  const int32_t* item_off;
  const int32_t* pairs;
  int k;
  // flat: rows [g * rows_per, min(n, (g + 1) * rows_per)) for group g
  int64_t n;
  int64_t rows_per;
  int nqc;  // flat: 32-query chunks
  int ngroups;
  const float* Q;
  int64_t nq;
  int topk;
  unsigned long long* cand;  // [(q * ngroups + g) * topk + r]
};

size_t ts_smem(int d, int topk) {
  return static_cast<size_t>(d) * kTsLanes * 4 +                    // queries
         static_cast<size_t>(kTsStages) * kTsRows * kTsChunk * 4 +  // row stages
         static_cast<size_t>(kTsLanes) * topk * 8 +                 // running top-k
         static_cast<size_t>(kTsLanes) * kTsHalf * 8 +              // candidates
         static_cast<size_t>(kTsLanes) * (8 + 4 + 4 + 4);            // thr, cnt, nb, slot
}

template <bool kIvf, int WARPS, int RW>
__global__ void __launch_bounds__(WARPS * 32, 2) tile_scan_kernel(const TileScanArgs a) {
  static_assert(WARPS * 4 * RW == kTsRows && RW % 2 == 0, "tile shape");
  constexpr int kThreads = WARPS * 32;
  constexpr int kNp = kTsRows * (kTsChunk / 4) / kThreads;  // 16-byte pieces per thread per stage
  constexpr int kRowStep = kThreads / (kTsChunk / 4);
  extern __shared__ __align__(16) uint8_t ts_sm[];
  const int d = a.d, topk = a.topk;
  const int d4 = d >> 2;
  // queries as float4 column quads: qs4[c4 * 32 + i * 8 + qg] = columns
  // 4 c4 .. 4 c4 + 3 of query 4 qg + i (the 8 query groups of one load sit
  // in 8 consecutive 16-byte slots: conflict-free)
  float4* qs4 = reinterpret_cast<float4*>(ts_sm);
  float* rs = reinterpret_cast<float*>(qs4 + static_cast<size_t>(d4) * kTsLanes);  // [stages][128][16]
  unsigned long long* best = reinterpret_cast<unsigned long long*>(rs + kTsStages * kTsRows * kTsChunk);
  unsigned long long* cbuf = best + kTsLanes * topk;
  unsigned long long* thr = cbuf + kTsLanes * kTsHalf;
  int* cnt = reinterpret_cast<int*>(thr + kTsLanes);
  int* nb = cnt + kTsLanes;
  int* slot = nb + kTsLanes;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qg = lane & 7, rg = lane >> 3;

  // ---- work item -> (row source, queries)
  int64_t row0 = 0, nrows = 0;
  int npairs = 0;
  const uint32_t* lrows = nullptr;
  int pair_base = 0;
  int g_flat = 0, qc = 0;
  if constexpr (kIvf) {
    const int b = blockIdx.x;
    if (b >= a.item_off[a.k]) return;
    int lo = 0, hi = a.k;  // largest c with item_off[c] <= b
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (a.item_off[mid] <= b) lo = mid;
      else hi = mid;
    }
    // item_off[lo] <= b < item_off[lo + 1]: list lo (empty lists own no items)
    const int c = lo;
    const int j = b - a.item_off[c];
    pair_base = a.pair_off[c] + j * kTsLanes;
    npairs = min(kTsLanes, a.pair_off[c + 1] - pair_base);
    row0 = a.offs[c];
    nrows = a.offs[c + 1] - row0;
    lrows = a.lists + row0;
  } else {
    const int64_t b = blockIdx.x;
    g_flat = static_cast<int>(b / a.nqc);
    qc = static_cast<int>(b % a.nqc);
    row0 = static_cast<int64_t>(g_flat) * a.rows_per;
    nrows = row0 >= a.n ? 0 : (a.n - row0 < a.rows_per ? a.n - row0 : a.rows_per);
    npairs = static_cast<int>(min(static_cast<int64_t>(kTsLanes), a.nq - static_cast<int64_t>(qc) * kTsLanes));
  }

  if (tid < kTsLanes) {
    int s = -1;
    if (tid < npairs) {
      if constexpr (kIvf) s = a.pairs[pair_base + tid];
      else s = (qc * kTsLanes + tid) * a.ngroups + g_flat;
    }
    slot[tid] = s;
    cnt[tid] = 0;
    nb[tid] = 0;
    thr[tid] = ~0ull;
  }
  __syncthreads();
  for (int i = tid; i < kTsLanes * d4; i += kThreads) {
    const int q = i / d4, c4 = i - q * d4;
    const int s = slot[q];
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s >= 0) v = reinterpret_cast<const float4*>(a.Q + (s / a.ngroups) * static_cast<int64_t>(d))[c4];
    qs4[c4 * kTsLanes + (q & 3) * 8 + (q >> 2)] = v;
  }
  // (the first __syncthreads of the pipeline below publishes qs4)

  const int nchunks = (d + kTsChunk - 1) / kTsChunk;
  const int ntiles = static_cast<int>((nrows + kTsRows - 1) / kTsRows);

  // Issue side of the pipeline: stage = (tile ti, column chunk ci) into
  // buffer bi.  Each thread copies kNp 16-byte pieces per stage: rows
  // tid / 4 + kRowStep h of the tile, piece tid % 4.  The row ids of the
  // next tile are fetched one tile ahead (nx), so no cp.async waits on an
  // id load.
  const int piece = tid & 3;
  const int pr = tid >> 2;
  int ti = 0, ci = 0, bi = 0;
  int64_t cur[kNp], nx[kNp];  // row ids (-1: past the rows)
  auto row_of = [&](int t, int r) -> int64_t {
    const int64_t pos = static_cast<int64_t>(t) * kTsRows + r;
    if (pos >= nrows) return -1;
    return kIvf ? static_cast<int64_t>(lrows[pos]) : row0 + pos;
  };
#pragma unroll
  for (int h = 0; h < kNp; ++h) nx[h] = ntiles > 0 ? row_of(0, pr + kRowStep * h) : -1;
  auto issue = [&]() {
    if (ti < ntiles) {
      if (ci == 0) {
#pragma unroll
        for (int h = 0; h < kNp; ++h) {
          cur[h] = nx[h];
          if (ti + 1 < ntiles) nx[h] = row_of(ti + 1, pr + kRowStep * h);
        }
      }
      const int c = ci * kTsChunk + piece * 4;
      const bool cok = c < d;
      float* dst = rs + bi * (kTsRows * kTsChunk) + piece * 4;
#pragma unroll
      for (int h = 0; h < kNp; ++h)
        ts_cp16(dst + (pr + kRowStep * h) * kTsChunk, a.X + (cur[h] >= 0 && cok ? cur[h] * d + c : 0),
                cur[h] >= 0 && cok);
      if (++ci == nchunks) {
        ci = 0;
        ++ti;
      }
      bi = bi + 1 == kTsStages ? 0 : bi + 1;
    }
    ts_commit();
  };

#pragma unroll
  for (int s = 0; s < kTsStages - 1; ++s) issue();

  float acc[RW][kTsQW];
#pragma unroll
  for (int j = 0; j < RW; ++j)
#pragma unroll
    for (int i = 0; i < kTsQW; ++i) acc[j][i] = 0.f;

  const int myrow = warp * 4 * RW + rg * RW;  // first of this thread's RW tile rows
  int bc = 0;
  for (int t = 0; t < ntiles; ++t) {
    for (int kc = 0; kc < nchunks; ++kc) {
      ts_wait<kTsStages - 2>();
      __syncthreads();
      issue();
      const float4* rb = reinterpret_cast<const float4*>(rs + bc * (kTsRows * kTsChunk)) + myrow * (kTsChunk / 4);
      const float4* qb = qs4 + static_cast<size_t>(kc * (kTsChunk / 4)) * kTsLanes + qg;
      bc = bc + 1 == kTsStages ? 0 : bc + 1;
      const int nq4 = min(kTsChunk, d - kc * kTsChunk) >> 2;
      if (nq4 == kTsChunk / 4) {
#pragma unroll
        for (int c4 = 0; c4 < kTsChunk / 4; ++c4) {
          float4 qv[kTsQW], xv[RW];
#pragma unroll
          for (int i = 0; i < kTsQW; ++i) qv[i] = qb[c4 * kTsLanes + i * 8];
#pragma unroll
          for (int j = 0; j < RW; ++j) xv[j] = rb[j * (kTsChunk / 4) + c4];
#pragma unroll
          for (int j = 0; j < RW; ++j)
#pragma unroll
            for (int i = 0; i < kTsQW; ++i) acc[j][i] = ts_dot4(acc[j][i], xv[j], qv[i]);
        }
      } else {
        for (int c4 = 0; c4 < nq4; ++c4) {
          float4 qv[kTsQW], xv[RW];
#pragma unroll
          for (int i = 0; i < kTsQW; ++i) qv[i] = qb[c4 * kTsLanes + i * 8];
#pragma unroll
          for (int j = 0; j < RW; ++j) xv[j] = rb[j * (kTsChunk / 4) + c4];
#pragma unroll
          for (int j = 0; j < RW; ++j)
#pragma unroll
            for (int i = 0; i < kTsQW; ++i) acc[j][i] = ts_dot4(acc[j][i], xv[j], qv[i]);
        }
      }
    }

    // ---- tile t complete: two rounds (the first then the second half of
    // each thread's rows, 64 rows per query per round) of candidates better
    // than the query's k-th best, each followed by a rank merge
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int i = 0; i < kTsQW; ++i) {
        const int q = qg * 4 + i;
        if (q < npairs) {
          const unsigned long long th = thr[q];
#pragma unroll
          for (int jj = 0; jj < RW / 2; ++jj) {
            const int j = (RW / 2) * h + jj;
            const int64_t pos = static_cast<int64_t>(t) * kTsRows + myrow + j;
            if (pos < nrows) {
              const unsigned long long key = ts_key(acc[j][i], static_cast<uint32_t>(pos));
              if (key < th) cbuf[q * kTsHalf + atomicAdd(&cnt[q], 1)] = key;
            }
          }
        }
      }
      __syncthreads();
      // warp w merges queries w, w + WARPS, ...
      for (int j = warp; j < npairs; j += WARPS) {
        const int nc = cnt[j];
        if (nc == 0) continue;
        const int n0 = nb[j];
        const int tot = n0 + nc;  // <= topk + 64 <= 128
        const unsigned long long* bj = best + j * topk;
        const unsigned long long* cj = cbuf + j * kTsHalf;
        unsigned long long v[4];
        int rk[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = lane + 32 * u;
          v[u] = e < tot ? (e < n0 ? bj[e] : cj[e - n0]) : ~0ull;
          rk[u] = 0;
        }
        // rank = number of smaller keys (keys are distinct)
        if (tot <= 32) {
          for (int e = 0; e < tot; ++e) rk[0] += (e < n0 ? bj[e] : cj[e - n0]) < v[0];
        } else if (tot <= 64) {
          for (int e = 0; e < tot; ++e) {
            const unsigned long long x = e < n0 ? bj[e] : cj[e - n0];
            rk[0] += x < v[0];
            rk[1] += x < v[1];
          }
        } else {
          for (int e = 0; e < tot; ++e) {
            const unsigned long long x = e < n0 ? bj[e] : cj[e - n0];
#pragma unroll
            for (int u = 0; u < 4; ++u) rk[u] += x < v[u];
          }
        }
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (lane + 32 * u < tot && rk[u] < topk) best[j * topk + rk[u]] = v[u];
        __syncwarp();
        if (lane == 0) {
          const int m = tot < topk ? tot : topk;
          nb[j] = m;
          thr[j] = m == topk ? best[j * topk + topk - 1] : ~0ull;
          cnt[j] = 0;
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < RW; ++j)
#pragma unroll
      for (int i = 0; i < kTsQW; ++i) acc[j][i] = 0.f;
  }
  ts_wait<0>();

  // ---- output: positions -> row ids, empty slots ~0
  for (int j = warp; j < npairs; j += WARPS) {
    const int s = slot[j];
    const int m = nb[j];
    for (int r = lane; r < topk; r += 32) {
      unsigned long long o = ~0ull;
      if (r < m) {
        const unsigned long long kk = best[j * topk + r];
        const uint32_t pos = static_cast<uint32_t>(kk & 0xffffffffu);
        const uint32_t row = kIvf ? lrows[pos] : static_cast<uint32_t>(row0 + pos);
        o = (kk & 0xffffffff00000000ull) | row;
      }
      a.cand[static_cast<int64_t>(s) * topk + r] = o;
    }
  }
}

// ---- grouping of (query, probe) pairs by list
__global__ void pair_count_kernel(const int32_t* probes, int64_t npairs, int32_t* cnt) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < npairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    atomicAdd(&cnt[probes[i]], 1);
}

// pair_off = exclusive scan of cnt, item_off = exclusive scan of
// ceil(cnt / 32); both [k + 1].  One block; fill[] zeroed for the scatter.
__global__ void pair_scan_kernel(const int32_t* cnt, int k, int32_t* pair_off, int32_t* item_off,
                                 int32_t* fill) {
  __shared__ int32_t wp[32], wi[32];
  const int tid = threadIdx.x, nt = blockDim.x;
  const int per = (k + nt - 1) / nt;
  const int b = tid * per, e = min(k, b + per);
  int sp = 0, si = 0;
  for (int c = b; c < e; ++c) {
    sp += cnt[c];
    si += (cnt[c] + kTsLanes - 1) / kTsLanes;
  }
  // inclusive scan of (sp, si) over threads
  int ip = sp, ii = si;
  const int lane = tid & 31, w = tid >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int xp = __shfl_up_sync(0xffffffffu, ip, o), xi = __shfl_up_sync(0xffffffffu, ii, o);
    if (lane >= o) {
      ip += xp;
      ii += xi;
    }
  }
  if (lane == 31) {
    wp[w] = ip;
    wi[w] = ii;
  }
  __syncthreads();
  if (w == 0) {
    int vp = lane < (nt + 31) / 32 ? wp[lane] : 0, vi = lane < (nt + 31) / 32 ? wi[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int xp = __shfl_up_sync(0xffffffffu, vp, o), xi = __shfl_up_sync(0xffffffffu, vi, o);
      if (lane >= o) {
        vp += xp;
        vi += xi;
      }
    }
    wp[lane] = vp;
    wi[lane] = vi;
  }
  __syncthreads();
  int rp = ip - sp + (w > 0 ? wp[w - 1] : 0);
  int ri = ii - si + (w > 0 ? wi[w - 1] : 0);
  for (int c = b; c < e; ++c) {
    pair_off[c] = rp;
    item_off[c] = ri;
    fill[c] = 0;
    rp += cnt[c];
    ri += (cnt[c] + kTsLanes - 1) / kTsLanes;
  }
  if (tid == nt - 1) {
    pair_off[k] = rp;
    item_off[k] = ri;
  }
}

__global__ void pair_scatter_kernel(const int32_t* probes, int64_t npairs, const int32_t* pair_off,
                                    int32_t* fill, int32_t* pairs) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < npairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = probes[i];
    pairs[pair_off[c] + atomicAdd(&fill[c], 1)] = static_cast<int32_t>(i);
  }
}

template <bool kIvf>
cudaError_t set_smem(size_t sm) {
  static int done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (done[dev] >= static_cast<int>(sm)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(tile_scan_kernel<kIvf, kTsWarps, kTsRW>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sm));
  if (e == cudaSuccess) done[dev] = static_cast<int>(sm);
  return e;
}

}  // namespace

bool batched_scan_supported(const float* X, const float* Q, int d, int topk) {
  return d > 0 && d % 4 == 0 && topk >= 1 && topk <= 64 &&
         reinterpret_cast<uintptr_t>(X) % 16 == 0 && reinterpret_cast<uintptr_t>(Q) % 16 == 0 &&
         ts_smem(d, topk) + 16 <= 227 * 1024;
}

size_t batched_list_scan_ws(int k, int64_t npairs) {
  // cnt, fill [k]; pair_off, item_off [k + 1]; pairs [npairs]
  return (static_cast<size_t>(2 * k) + 2 * static_cast<size_t>(k + 1) + static_cast<size_t>(npairs)) * 4;
}

cudaError_t launch_list_scan_batched(const float* X, int d, const uint32_t* lists, const int64_t* offs,
                                     int k, const int32_t* probes, int nprobe, const float* Q, int64_t nq,
                                     int topk, void* ws, unsigned long long* cand, cudaStream_t st) {
  const int64_t np = nq * nprobe;
  if (np > INT32_MAX / 2) return cudaErrorInvalidValue;
  int32_t* cnt = static_cast<int32_t*>(ws);
  int32_t* fill = cnt + k;
  int32_t* pair_off = fill + k;
  int32_t* item_off = pair_off + (k + 1);
  int32_t* pairs = item_off + (k + 1);
  cudaError_t e = cudaMemsetAsync(cnt, 0, static_cast<size_t>(k) * 4, st);
  if (e != cudaSuccess) return e;
  const int gb = static_cast<int>(std::min<int64_t>(4096, (np + 255) / 256));
  if (np > 0) pair_count_kernel<<<gb, 256, 0, st>>>(probes, np, cnt);
  pair_scan_kernel<<<1, 1024, 0, st>>>(cnt, k, pair_off, item_off, fill);
  if (np > 0) pair_scatter_kernel<<<gb, 256, 0, st>>>(probes, np, pair_off, fill, pairs);
  const size_t sm = ts_smem(d, topk) + 16;
  if ((e = set_smem<true>(sm)) != cudaSuccess) return e;
  TileScanArgs a{};
  a.X = X;
  a.d = d;
  a.lists = lists;
  a.offs = offs;
  a.pair_off = pair_off;
  a.item_off = item_off;
  a.pairs = pairs;
  a.k = k;
  a.ngroups = nprobe;
  a.Q = Q;
  a.nq = nq;
  a.topk = topk;
  a.cand = cand;
  // items <= sum over lists of (pairs / 32 + 1) for the non-empty lists;
  // blocks past item_off[k] return at once
  const int64_t grid = std::min<int64_t>(k, np) + (np + kTsLanes - 1) / kTsLanes;
  if (grid <= 0) return cudaGetLastError();
  if (grid > INT32_MAX) return cudaErrorInvalidValue;
  tile_scan_kernel<true, kTsWarps, kTsRW><<<static_cast<unsigned>(grid), kTsWarps * 32, sm, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_flat_scan_batched(const float* X, int64_t n, int d, int nchunks, const float* Q,
                                     int64_t nq, int topk, unsigned long long* cand, cudaStream_t st) {
  const size_t sm = ts_smem(d, topk) + 16;
  cudaError_t e = set_smem<false>(sm);
  if (e != cudaSuccess) return e;
  TileScanArgs a{};
  a.X = X;
  a.d = d;
  a.n = n;
  a.rows_per = (n + nchunks - 1) / nchunks;
  a.nqc = static_cast<int>((nq + kTsLanes - 1) / kTsLanes);
  a.ngroups = nchunks;
  a.Q = Q;
  a.nq = nq;
  a.topk = topk;
  a.cand = cand;
  const int64_t grid = static_cast<int64_t>(nchunks) * a.nqc;
  if (grid <= 0) return cudaGetLastError();
  if (grid > INT32_MAX) return cudaErrorInvalidValue;
  tile_scan_kernel<false, kTsWarps, kTsRW><<<static_cast<unsigned>(grid), kTsWarps * 32, sm, st>>>(a);
  return cudaGetLastError();
}

}  // namespace ec
