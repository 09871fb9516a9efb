// ec_attn_short.cuh -- attention for sequences of at most kShortAttnMaxLen
// tokens, the common case of sentence embedding (MiniLM / BERT batches of
// 16..256 tokens).
//
// Same arithmetic as ec_attn.cuh (softmax(Q K^T * scale + bias) V per
// sequence and head: bert::encoder-layer bert.lisp:226-248, the MPNet bias of
// bert::mpnet-layer :408-423, causal llama::layer-forward llama.lisp:255-271),
// organised for short sequences: one CTA per (sequence, head) copies the
// head's whole K and V into shared memory once, then each warp walks 16-row
// query tiles on its own -- no block-wide barrier inside the loop, no 64-row
// query padding, and K/V leave HBM once per (sequence, head).  Math is
// mma.sync.m16n8k16 bf16 -> fp32 with the online softmax in registers over
// 64-key blocks.
#pragma once

#include "ec_attn.cuh"
#include "ec_kernels.h"

namespace ec {

constexpr int kShortAttnMaxLen = 256;  // keys resident in shared memory
constexpr int kShortAttnThreads = 128;

struct ShortAttnArgs {
  const __nv_bfloat16* qkv;  // packed rows, row stride ld elements
  int ld;
  int q_off, k_off, v_off;
  __nv_bfloat16* out;        // [T, heads * HD], row stride ldo
  int ldo;
  const int2* seqs;          // (first token, length) per sequence, longest first
  int first;                 // index of the first sequence this launch handles
  int heads, kv_group;
  float scale_log2;          // log2(e) / sqrt(head_dim)
  const float* relbias;      // MODE 1: [heads][2 * rel_max - 1] (* log2 e)
  int rel_max;
  int kcap;                  // K/V rows reserved in shared memory: the longest
                             // sequence of the launch rounded up to 16
};

template <int HD, int MODE>
struct ShortAttnSmem {
  static constexpr int LDS = HD + 8;  // padded rows: conflict-free ldmatrix
  static size_t bytes(int kcap) {
    return static_cast<size_t>(2) * kcap * LDS * 2 + (MODE == 1 ? static_cast<size_t>(2) * kcap * 4 : 0);
  }
  static constexpr size_t MAX_BYTES =
      static_cast<size_t>(2) * kShortAttnMaxLen * LDS * 2 + (MODE == 1 ? 2 * kShortAttnMaxLen * 4 : 0);
};

// BK: keys per online-softmax block (64 or 128); MINB: CTAs per SM the
// register budget is sized for
template <int HD, int MODE, int BK, int MINB>
__global__ void __launch_bounds__(kShortAttnThreads, MINB)
    attn_short_kernel(const ShortAttnArgs a) {
  constexpr int NT = BK / 8;     // 8-key n-tiles per block
  constexpr bool kBias = MODE == 1;
  constexpr bool kCausal = MODE == 2;
  constexpr int LDS = ShortAttnSmem<HD, MODE>::LDS;
  constexpr int NT_D = HD / 8;   // n-tiles of the output
  constexpr int KS_D = HD / 16;  // k-steps over the head dim
  constexpr int CH = HD / 8;     // 16-byte chunks per row
  extern __shared__ __align__(16) uint8_t short_smem[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(short_smem);
  __nv_bfloat16* sV = sK + a.kcap * LDS;
  float* sBias = reinterpret_cast<float*>(sV + a.kcap * LDS);

  const int2 sq = a.seqs[a.first + blockIdx.x];
  const int base = sq.x, L = sq.y;
  const int h = blockIdx.y;
  const int kvh = h / a.kv_group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Lr = (L + 15) & ~15;  // keys rounded up to whole 16-key MMA steps

  // K and V of this head: rows [0, L) copied, rows [L, Lr) zeroed so that the
  // masked tail of the last step multiplies zeros, never stale values
  for (int i = threadIdx.x; i < Lr * CH; i += kShortAttnThreads) {
    const int r = i / CH, c = i % CH;
    const bool live = r < L;
    const size_t g = static_cast<size_t>(base + (live ? r : 0)) * a.ld;
    cp_async16(sK + r * LDS + c * 8, a.qkv + g + a.k_off + kvh * HD + c * 8, live);
    cp_async16(sV + r * LDS + c * 8, a.qkv + g + a.v_off + kvh * HD + c * 8, live);
  }
  cp_async_commit();
  if (kBias) {
    // sBias[i - j + L - 1] for query i, key j < L
    const int nb = 2 * a.rel_max - 1;
    const float* src = a.relbias + static_cast<size_t>(h) * nb;
    for (int i = threadIdx.x; i < 2 * L - 1; i += kShortAttnThreads) {
      const int dlt = i - (L - 1);
      sBias[i] = (dlt > -a.rel_max && dlt < a.rel_max) ? src[dlt + a.rel_max - 1] : 0.f;
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  const float sc = kBias ? 1.0f : a.scale_log2;
  for (int tile = warp; tile * 16 < L; tile += kShortAttnThreads / 32) {
    const int q0 = tile * 16;
    const int row_a = q0 + (lane >> 2), row_b = row_a + 8;
    // Q fragments straight from global memory (rows past L read as zero)
    uint32_t qf[KS_D][4];
    {
      const __nv_bfloat16* qa = a.qkv + static_cast<size_t>(base + row_a) * a.ld + a.q_off + h * HD;
      const __nv_bfloat16* qb = qa + static_cast<size_t>(8) * a.ld;
#pragma unroll
      for (int ks = 0; ks < KS_D; ++ks) {
        const int c = ks * 16 + (lane & 3) * 2;
        qf[ks][0] = row_a < L ? *reinterpret_cast<const uint32_t*>(qa + c) : 0u;
        qf[ks][1] = row_b < L ? *reinterpret_cast<const uint32_t*>(qb + c) : 0u;
        qf[ks][2] = row_a < L ? *reinterpret_cast<const uint32_t*>(qa + c + 8) : 0u;
        qf[ks][3] = row_b < L ? *reinterpret_cast<const uint32_t*>(qb + c + 8) : 0u;
      }
    }
    float o[NT_D][4];
#pragma unroll
    for (int n = 0; n < NT_D; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    const int kv_end = kCausal ? min(L, q0 + 16) : L;
    for (int k0 = 0; k0 < kv_end; k0 += BK) {
      const int nt_live = min(NT, (kv_end - k0 + 7) >> 3);  // live 8-key n-tiles
      const bool need_mask = (k0 + BK > L) || (kCausal && k0 + BK - 1 > q0);
      float s[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS_D; ++ks) {
#pragma unroll
        for (int n = 0; n < NT; n += 2) {
          if (n < nt_live) {
            uint32_t b[4];
            const int mi = lane >> 3;
            const int key = k0 + n * 8 + (mi >> 1) * 8 + (lane & 7);
            ldsm_x4(b, sK + key * LDS + ks * 16 + (mi & 1) * 8);
            mma_bf16_16816(s[n], qf[ks], b[0], b[1]);
            mma_bf16_16816(s[n + 1], qf[ks], b[2], b[3]);
          }
        }
      }
      if (kBias) {
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = k0 + n * 8 + (lane & 3) * 2 + (e & 1);
            const int qr = (e < 2) ? row_a : row_b;
            const int bi = qr - key + (L - 1);
            s[n][e] = fmaf(s[n][e], a.scale_log2, sBias[bi < 0 ? 0 : (bi > 2 * L - 2 ? 2 * L - 2 : bi)]);
          }
      }
      if (need_mask) {
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = k0 + n * 8 + (lane & 3) * 2 + (e & 1);
            const int qr = (e < 2) ? row_a : row_b;
            if (key >= L || (kCausal && key > qr)) s[n][e] = -INFINITY;
          }
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        mx[0] = fmaxf(mx[0], fmaxf(s[n][0], s[n][1]));
        mx[1] = fmaxf(mx[1], fmaxf(s[n][2], s[n][3]));
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      }
      // key 0 is visible to every row (0 < L, 0 <= row), so after the first
      // block every running max is finite: no -inf - -inf below
      float corr[2], rs[2] = {0.f, 0.f}, nm[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float mnew = fmaxf(m_r[r], mx[r] * sc);
        corr[r] = fast_exp2(m_r[r] - mnew);
        m_r[r] = mnew;
        nm[r] = -mnew;
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        if (n < nt_live) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p = fast_exp2(fmaf(s[n][e], sc, nm[e >> 1]));
            s[n][e] = p;
            rs[e >> 1] += p;
          }
        } else {
          s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
        l_r[r] = l_r[r] * corr[r] + rs[r];
      }
#pragma unroll
      for (int n = 0; n < NT_D; ++n) {
        o[n][0] *= corr[0];
        o[n][1] *= corr[0];
        o[n][2] *= corr[1];
        o[n][3] *= corr[1];
      }
      // O += P V over the live 16-key steps (rows past L of V are zero)
#pragma unroll
      for (int t = 0; t < NT / 2; ++t) {
        if (2 * t < nt_live) {
          uint32_t pa[4];
          pa[0] = pack2_bf16(s[2 * t][0], s[2 * t][1]);
          pa[1] = pack2_bf16(s[2 * t][2], s[2 * t][3]);
          pa[2] = pack2_bf16(s[2 * t + 1][0], s[2 * t + 1][1]);
          pa[3] = pack2_bf16(s[2 * t + 1][2], s[2 * t + 1][3]);
#pragma unroll
          for (int n = 0; n < NT_D; n += 2) {
            uint32_t b[4];
            const int mi = lane >> 3;
            const int key = k0 + t * 16 + (mi & 1) * 8 + (lane & 7);
            const int d = (n + (mi >> 1)) * 8;
            ldsm_x4_t(b, sV + key * LDS + d);
            mma_bf16_16816(o[n], pa, b[0], b[1]);
            mma_bf16_16816(o[n + 1], pa, b[2], b[3]);
          }
        }
      }
    }
    const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
    const float inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
    __nv_bfloat16* out_h = a.out + h * HD;
#pragma unroll
    for (int n = 0; n < NT_D; ++n) {
      const int d = n * 8 + (lane & 3) * 2;
      if (row_a < L)
        *reinterpret_cast<uint32_t*>(out_h + static_cast<size_t>(base + row_a) * a.ldo + d) =
            pack2_bf16(o[n][0] * inv0, o[n][1] * inv0);
      if (row_b < L)
        *reinterpret_cast<uint32_t*>(out_h + static_cast<size_t>(base + row_b) * a.ldo + d) =
            pack2_bf16(o[n][2] * inv1, o[n][3] * inv1);
    }
  }
}

// ---------------------------------------------------------------------------
// The same attention with the probabilities in fp16: each pair of scores
// becomes x = s * scale - max (packed fp32 fma), one cvt to f16x2 and ONE
// ex2.approx.f16x2 for both exponentials (half the MUFU instructions of the
// fp32 path), and the f16x2 result is already the A fragment of the P.V MMA
// (f16 x f16 -> fp32).  V is converted to f16 once in shared memory (exact
// for |v| in [2^-14, 65504]; post-LayerNorm encoders keep V far inside that).
// The row sums come from the tensor core: one more MMA per 16 keys against a
// constant all-ones B fragment, accumulated and rescaled like the output.
// Q fragments of the warp's next tile are fetched while the current tile
// runs.  Relative error of p: f16 rounding of x (|x| * 2^-11 * ln 2) plus
// ex2.approx.f16's own, the same order as the bf16 rounding of P in the fp32
// path.
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
  uint32_t r;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
// (lo, hi) -> f16x2 with lo in the low half (the lower column of an MMA pair)
__device__ __forceinline__ uint32_t cvt_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// bf16x2 -> f16x2 (through fp32; exact inside the f16 normal range)
__device__ __forceinline__ uint32_t bf2_to_h2(uint32_t v) {
  const float lo = __uint_as_float(v << 16), hi = __uint_as_float(v & 0xffff0000u);
  return cvt_h2(lo, hi);
}

// BK: keys per online-softmax block (32 or 64); PV2: two independent P.V
// accumulator sets (even / odd 16-key steps), summed at the end, so that
// consecutive MMAs of the accumulation do not wait on each other
template <int HD, int MODE, int MINB, int BK = 64, bool PV2 = false>
__global__ void __launch_bounds__(kShortAttnThreads, MINB)
    attn_short_h_kernel(const ShortAttnArgs a) {
  static_assert(BK == 32 || BK == 64, "key block");
  pdl_trigger();
  pdl_wait();
  constexpr int NT = BK / 8;
  constexpr int NS = PV2 ? 2 : 1;
  constexpr bool kBias = MODE == 1;
  constexpr bool kCausal = MODE == 2;
  constexpr int LDS = ShortAttnSmem<HD, MODE>::LDS;
  constexpr int NT_D = HD / 8;
  constexpr int KS_D = HD / 16;
  constexpr int CH = HD / 8;
  constexpr int NW = kShortAttnThreads / 32;
  constexpr uint32_t kOnes = 0x3C003C00u;  // f16x2 (1, 1)
  extern __shared__ __align__(16) uint8_t short_smem[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(short_smem);
  __nv_bfloat16* sV = sK + a.kcap * LDS;  // f16 after the conversion below
  float* sBias = reinterpret_cast<float*>(sV + a.kcap * LDS);

  const int2 sq = a.seqs[a.first + blockIdx.x];
  const int base = sq.x, L = sq.y;
  const int h = blockIdx.y;
  const int kvh = h / a.kv_group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Lr = (L + 15) & ~15;

  for (int i = threadIdx.x; i < Lr * CH; i += kShortAttnThreads) {
    const int r = i / CH, c = i % CH;
    const bool live = r < L;
    const size_t g = static_cast<size_t>(base + (live ? r : 0)) * a.ld;
    cp_async16(sK + r * LDS + c * 8, a.qkv + g + a.k_off + kvh * HD + c * 8, live);
    cp_async16(sV + r * LDS + c * 8, a.qkv + g + a.v_off + kvh * HD + c * 8, live);
  }
  cp_async_commit();
  if (kBias) {
    const int nb = 2 * a.rel_max - 1;
    const float* src = a.relbias + static_cast<size_t>(h) * nb;
    for (int i = threadIdx.x; i < 2 * L - 1; i += kShortAttnThreads) {
      const int dlt = i - (L - 1);
      sBias[i] = (dlt > -a.rel_max && dlt < a.rel_max) ? src[dlt + a.rel_max - 1] : 0.f;
    }
  }
  cp_async_wait<0>();
  // each thread converts the V chunks it copied (zero rows stay zero)
  for (int i = threadIdx.x; i < Lr * CH; i += kShortAttnThreads) {
    const int r = i / CH, c = i % CH;
    uint4* p = reinterpret_cast<uint4*>(sV + r * LDS + c * 8);
    uint4 v = *p;
    v.x = bf2_to_h2(v.x);
    v.y = bf2_to_h2(v.y);
    v.z = bf2_to_h2(v.z);
    v.w = bf2_to_h2(v.w);
    *p = v;
  }
  __syncthreads();

  const float sc = kBias ? 1.0f : a.scale_log2;
  const int ntiles = (L + 15) >> 4;
  // Q fragments of a tile straight from global memory (rows past L are zero)
  auto load_q = [&](int tile, uint32_t (&qf)[KS_D][4]) {
    const int ra = tile * 16 + (lane >> 2), rb = ra + 8;
    const __nv_bfloat16* qa = a.qkv + static_cast<size_t>(base + (ra < L ? ra : 0)) * a.ld + a.q_off + h * HD;
    const __nv_bfloat16* qb = a.qkv + static_cast<size_t>(base + (rb < L ? rb : 0)) * a.ld + a.q_off + h * HD;
#pragma unroll
    for (int ks = 0; ks < KS_D; ++ks) {
      const int c = ks * 16 + (lane & 3) * 2;
      qf[ks][0] = ra < L ? *reinterpret_cast<const uint32_t*>(qa + c) : 0u;
      qf[ks][1] = rb < L ? *reinterpret_cast<const uint32_t*>(qb + c) : 0u;
      qf[ks][2] = ra < L ? *reinterpret_cast<const uint32_t*>(qa + c + 8) : 0u;
      qf[ks][3] = rb < L ? *reinterpret_cast<const uint32_t*>(qb + c + 8) : 0u;
    }
  };
  uint32_t qn[KS_D][4];
  if (warp < ntiles) load_q(warp, qn);
  for (int tile = warp; tile < ntiles; tile += NW) {
    uint32_t qf[KS_D][4];
#pragma unroll
    for (int ks = 0; ks < KS_D; ++ks)
#pragma unroll
      for (int j = 0; j < 4; ++j) qf[ks][j] = qn[ks][j];
    if (tile + NW < ntiles) load_q(tile + NW, qn);
    const int q0 = tile * 16;
    const int row_a = q0 + (lane >> 2), row_b = row_a + 8;
    float o[NS][NT_D][4], osum[NS][4];
#pragma unroll
    for (int v = 0; v < NS; ++v) {
      osum[v][0] = osum[v][1] = osum[v][2] = osum[v][3] = 0.f;
#pragma unroll
      for (int n = 0; n < NT_D; ++n) o[v][n][0] = o[v][n][1] = o[v][n][2] = o[v][n][3] = 0.f;
    }
    float m_r[2] = {-INFINITY, -INFINITY};
    const int kv_end = kCausal ? min(L, q0 + 16) : L;
    for (int k0 = 0; k0 < kv_end; k0 += BK) {
      const int nt_live = min(NT, (kv_end - k0 + 7) >> 3);
      const bool need_mask = (k0 + BK > L) || (kCausal && k0 + BK - 1 > q0);
      float s[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS_D; ++ks) {
#pragma unroll
        for (int n = 0; n < NT; n += 2) {
          if (n < nt_live) {
            uint32_t b[4];
            const int mi = lane >> 3;
            const int key = k0 + n * 8 + (mi >> 1) * 8 + (lane & 7);
            ldsm_x4(b, sK + key * LDS + ks * 16 + (mi & 1) * 8);
            mma_bf16_16816(s[n], qf[ks], b[0], b[1]);
            mma_bf16_16816(s[n + 1], qf[ks], b[2], b[3]);
          }
        }
      }
      if (kBias) {
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = k0 + n * 8 + (lane & 3) * 2 + (e & 1);
            const int qr = (e < 2) ? row_a : row_b;
            const int bi = qr - key + (L - 1);
            s[n][e] = fmaf(s[n][e], a.scale_log2, sBias[bi < 0 ? 0 : (bi > 2 * L - 2 ? 2 * L - 2 : bi)]);
          }
      }
      // keys past the sequence (and, causal, after the row) -> -inf: their
      // p is exactly 0, which also covers n-tiles that were not computed
      if (need_mask) {
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = k0 + n * 8 + (lane & 3) * 2 + (e & 1);
            const int qr = (e < 2) ? row_a : row_b;
            if (key >= L || (kCausal && key > qr)) s[n][e] = -INFINITY;
          }
      }
      // row maxima by a pairwise tree (depth log2 NT + 1, not a chain of NT)
      float mt[2][NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        mt[0][n] = fmaxf(s[n][0], s[n][1]);
        mt[1][n] = fmaxf(s[n][2], s[n][3]);
      }
#pragma unroll
      for (int w = NT / 2; w >= 1; w /= 2)
#pragma unroll
        for (int n = 0; n < w; ++n) {
          mt[0][n] = fmaxf(mt[0][n], mt[0][n + w]);
          mt[1][n] = fmaxf(mt[1][n], mt[1][n + w]);
        }
      float mx[2] = {mt[0][0], mt[1][0]};
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      }
      // key 0 is visible to every row, so after the first block every
      // running max is finite
      float corr[2];
      float2 nm[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float mnew = fmaxf(m_r[r], mx[r] * sc);
        corr[r] = fast_exp2(m_r[r] - mnew);
        m_r[r] = mnew;
        nm[r] = make_float2(-mnew, -mnew);
      }
      const float2 sc2 = make_float2(sc, sc);
      // p = 2^(s * sc - m) two at a time, already packed as MMA A halves
      uint32_t ph[NT][2];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const float2 xa = __ffma2_rn(make_float2(s[n][0], s[n][1]), sc2, nm[0]);
        const float2 xb = __ffma2_rn(make_float2(s[n][2], s[n][3]), sc2, nm[1]);
        ph[n][0] = ex2_h2(cvt_h2(xa.x, xa.y));
        ph[n][1] = ex2_h2(cvt_h2(xb.x, xb.y));
      }
      const float2 c0 = make_float2(corr[0], corr[0]), c1 = make_float2(corr[1], corr[1]);
#pragma unroll
      for (int v = 0; v < NS; ++v) {
#pragma unroll
        for (int n = 0; n < NT_D; ++n) {
          const float2 u = __fmul2_rn(make_float2(o[v][n][0], o[v][n][1]), c0);
          const float2 w = __fmul2_rn(make_float2(o[v][n][2], o[v][n][3]), c1);
          o[v][n][0] = u.x;
          o[v][n][1] = u.y;
          o[v][n][2] = w.x;
          o[v][n][3] = w.y;
        }
        const float2 u = __fmul2_rn(make_float2(osum[v][0], osum[v][1]), c0);
        const float2 w = __fmul2_rn(make_float2(osum[v][2], osum[v][3]), c1);
        osum[v][0] = u.x;
        osum[v][1] = u.y;
        osum[v][2] = w.x;
        osum[v][3] = w.y;
      }
      // O += P V and the row sums += P . 1 over the live 16-key steps
#pragma unroll
      for (int t = 0; t < NT / 2; ++t) {
        if (2 * t < nt_live) {
          const int v = PV2 ? (t & 1) : 0;
          const uint32_t pa[4] = {ph[2 * t][0], ph[2 * t][1], ph[2 * t + 1][0], ph[2 * t + 1][1]};
          mma_f16_16816(osum[v], pa, kOnes, kOnes);
#pragma unroll
          for (int n = 0; n < NT_D; n += 2) {
            uint32_t b[4];
            const int mi = lane >> 3;
            const int key = k0 + t * 16 + (mi & 1) * 8 + (lane & 7);
            const int d = (n + (mi >> 1)) * 8;
            ldsm_x4_t(b, sV + key * LDS + d);
            mma_f16_16816(o[v][n], pa, b[0], b[1]);
            mma_f16_16816(o[v][n + 1], pa, b[2], b[3]);
          }
        }
      }
    }
    if constexpr (PV2) {
#pragma unroll
      for (int n = 0; n < NT_D; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[0][n][e] += o[1][n][e];
#pragma unroll
      for (int e = 0; e < 4; ++e) osum[0][e] += osum[1][e];
    }
    const float inv0 = osum[0][0] > 0.f ? 1.f / osum[0][0] : 0.f;
    const float inv1 = osum[0][2] > 0.f ? 1.f / osum[0][2] : 0.f;
    __nv_bfloat16* out_h = a.out + h * HD;
#pragma unroll
    for (int n = 0; n < NT_D; ++n) {
      const int d = n * 8 + (lane & 3) * 2;
      if (row_a < L)
        *reinterpret_cast<uint32_t*>(out_h + static_cast<size_t>(base + row_a) * a.ldo + d) =
            pack2_bf16(o[0][n][0] * inv0, o[0][n][1] * inv0);
      if (row_b < L)
        *reinterpret_cast<uint32_t*>(out_h + static_cast<size_t>(base + row_b) * a.ldo + d) =
            pack2_bf16(o[0][n][2] * inv1, o[0][n][3] * inv1);
    }
  }
}

}  // namespace ec
