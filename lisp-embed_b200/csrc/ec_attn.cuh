// ec_attn.cuh -- varlen fused attention over packed tokens.
//
// softmax(Q K^T * scale + bias) V per (sequence, head), the triple loop of
// bert::encoder-layer (bert.lisp:226-248), bert::mpnet-layer (:408-423, with
// the relative-position bias) and llama::layer-forward (llama.lisp:255-271,
// causal grouped-query attention).  Sequences are packed back to back (no
// padding); one CTA handles 64 query rows of one sequence for every head and
// streams the sequence's keys in blocks of 64 with an online softmax, so the
// L x L score matrix never leaves registers.  Tensor-core math is
// mma.sync.m16n8k16 bf16 -> fp32.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace ec {

struct AttnArgs {
  const __nv_bfloat16* qkv;  // packed rows, row stride ld elements
  int ld;
  int q_off, k_off, v_off;   // column offsets of Q, K, V head 0
  __nv_bfloat16* out;        // [T, heads * HD], row stride ldo
  int ldo;
  const int* cu;             // [nseq + 1] token offsets
  const int2* blocks;        // (sequence, first query row) per CTA row of the grid
  int heads;
  int kv_group;              // heads per kv head
  float scale_log2;          // log2(e) / sqrt(head_dim)
  int causal;
  const float* relbias;      // [heads][2 * rel_max - 1] (already * log2 e) or nullptr
  int rel_max;               // bias index = (i - j) + rel_max - 1
  int heads_per_cta;         // heads walked by one CTA (grid.y = heads / heads_per_cta)
};

constexpr int kAttnBQ = 64;
constexpr int kAttnBK = 64;
constexpr int kAttnThreads = 128;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float fast_exp2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ uint32_t pack2_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int HD>
struct AttnSmem {
  static constexpr int LDS = HD + 8;  // padded row (elements) -> conflict-free ldmatrix
  static constexpr int TILE = kAttnBK * LDS;
  // Q, K, V double-buffered + relative-bias row
  static constexpr size_t BYTES = static_cast<size_t>(6 * TILE) * 2 + 2048 * 4;
};

// Load a 64-row tile (rows r0.. of the sequence starting at token `base`,
// `n` valid rows) of HD columns starting at column `col` into smem.
template <int HD>
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src_base,
                                          int ld, int base, int r0, int n, int col) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  constexpr int LDS = AttnSmem<HD>::LDS;
  for (int i = threadIdx.x; i < kAttnBK * CH; i += kAttnThreads) {
    const int r = i / CH, c = i % CH;
    const bool ok = (r0 + r) < n;
    const __nv_bfloat16* g =
        src_base + static_cast<size_t>(base + (ok ? r0 + r : 0)) * ld + col + c * 8;
    cp_async16(dst + r * LDS + c * 8, g, ok);
  }
}

// One CTA per (sequence, 64-query block, group of heads_per_cta heads).  The
// work is the flattened sequence of (head, key block) items; the Q/K/V tiles
// of item i+1 are fetched with cp.async while item i computes, across head
// boundaries.
// MODE 0: bidirectional with padding (BERT); 1: + relative bias (MPNet);
// 2: causal (Llama / Qwen3).
template <int HD, int MODE>
__global__ void __launch_bounds__(kAttnThreads)
    attn_fwd_kernel(const AttnArgs a) {
  constexpr bool kBias = MODE == 1;
  constexpr bool kCausal = MODE == 2;
  constexpr int LDS = AttnSmem<HD>::LDS;
  constexpr int TILE = AttnSmem<HD>::TILE;
  constexpr int NT_D = HD / 8;    // n-tiles of the output
  constexpr int KS_D = HD / 16;   // k-steps over head dim
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(attn_smem);  // 2 buffers
  __nv_bfloat16* sK = sQ + 2 * TILE;                                   // 2 buffers
  __nv_bfloat16* sV = sK + 2 * TILE;                                   // 2 buffers
  float* sBias = reinterpret_cast<float*>(sV + 2 * TILE);

  const int2 blk = a.blocks[blockIdx.x];
  const int seq = blk.x, q0 = blk.y;
  const int base = a.cu[seq];
  const int L = a.cu[seq + 1] - base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int kv_end = L;
  if (kCausal) kv_end = min(L, q0 + kAttnBQ);
  const int nkb = (kv_end + kAttnBK - 1) / kAttnBK;
  const int h0 = blockIdx.y * a.heads_per_cta;
  const int total = a.heads_per_cta * nkb;

  auto issue = [&](int it) {
    const int h = h0 + it / nkb, kb = it % nkb;
    const int kvh = h / a.kv_group;
    if (kb == 0) load_tile<HD>(sQ + (h & 1) * TILE, a.qkv, a.ld, base, q0, L, a.q_off + h * HD);
    load_tile<HD>(sK + (it & 1) * TILE, a.qkv, a.ld, base, kb * kAttnBK, L, a.k_off + kvh * HD);
    load_tile<HD>(sV + (it & 1) * TILE, a.qkv, a.ld, base, kb * kAttnBK, L, a.v_off + kvh * HD);
    cp_async_commit();
  };

  float o[NT_D][4];
  float m_r[2], l_r[2];
  uint32_t qf[KS_D][4];
  const int row_a = q0 + warp * 16 + (lane >> 2);  // query row (within seq) of c0/c1
  const int row_b = row_a + 8;

  issue(0);
  for (int it = 0; it < total; ++it) {
    const int h = h0 + it / nkb, kb = it % nkb;
    if (it + 1 < total) {
      issue(it + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
      if (kBias) {
        // bias for i - j over this sequence: |i - j| < L
        const int nb = 2 * a.rel_max - 1;
        const float* src = a.relbias + static_cast<size_t>(h) * nb;
        for (int i = threadIdx.x; i < 2 * L - 1 && i < 2048; i += kAttnThreads)
          sBias[i] = src[i - (L - 1) + a.rel_max - 1];
        __syncthreads();
      }
      const __nv_bfloat16* cQ = sQ + (h & 1) * TILE;
#pragma unroll
      for (int ks = 0; ks < KS_D; ++ks)
        ldsm_x4(qf[ks], cQ + (warp * 16 + (lane & 15)) * LDS + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int n = 0; n < NT_D; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      m_r[0] = m_r[1] = -INFINITY;
      l_r[0] = l_r[1] = 0.f;
    }
    const __nv_bfloat16* cK = sK + (it & 1) * TILE;
    const __nv_bfloat16* cV = sV + (it & 1) * TILE;
    const int k0 = kb * kAttnBK;
    // warps whose 16 query rows all lie past the sequence skip the math
    const bool warp_live = q0 + warp * 16 < L;
    // keys k0 + 8n .. for n < nt_live exist in this sequence
    const int nt_live = min(8, (L - k0 + 7) >> 3);
    // only the last block (or one touching the causal diagonal) needs masks
    const bool need_mask = (k0 + kAttnBK > L) || (kCausal && k0 + kAttnBK - 1 > q0 + warp * 16);
    if (warp_live) {
      // S = Q K^T : 16 x 64 per warp (raw dot products)
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS_D; ++ks) {
#pragma unroll
        for (int n = 0; n < 8; n += 2) {
          if (n < nt_live) {
            uint32_t b[4];
            const int mi = lane >> 3;  // matrix index
            const int key = n * 8 + (mi >> 1) * 8 + (lane & 7);
            ldsm_x4(b, cK + key * LDS + ks * 16 + (mi & 1) * 8);
            mma_bf16_16816(s[n], qf[ks], b[0], b[1]);
            mma_bf16_16816(s[n + 1], qf[ks], b[2], b[3]);
          }
        }
      }
      // logits in log2 units are s * scale_log2 (+ bias); without a bias the
      // scale is applied inside the exp (scale > 0 keeps the max)
      if (kBias) {
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = k0 + n * 8 + (lane & 3) * 2 + (e & 1);
            const int qr = (e < 2) ? row_a : row_b;
            const int bi = qr - key + (L - 1);
            s[n][e] = fmaf(s[n][e], a.scale_log2, sBias[bi < 0 ? 0 : (bi > 2046 ? 2046 : bi)]);
          }
      }
      if (need_mask) {
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = k0 + n * 8 + (lane & 3) * 2 + (e & 1);
            const int qr = (e < 2) ? row_a : row_b;
            const bool masked = key >= L || (kCausal && key > qr);
            s[n][e] = masked ? -INFINITY : s[n][e];
          }
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        mx[0] = fmaxf(mx[0], fmaxf(s[n][0], s[n][1]));
        mx[1] = fmaxf(mx[1], fmaxf(s[n][2], s[n][3]));
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      }
      // Key 0 is visible to every query row (0 < L and 0 <= row), so after the
      // first key block every running max is finite and the updates below
      // never see -inf - -inf.  Running maxima are kept in log2 units.
      const float sc = kBias ? 1.0f : a.scale_log2;
      float corr[2], rs[2] = {0.f, 0.f}, nm[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float mnew = fmaxf(m_r[r], mx[r] * sc);
        corr[r] = fast_exp2(m_r[r] - mnew);
        m_r[r] = mnew;
        nm[r] = -mnew;
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        if (n < nt_live) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int r = e >> 1;
            const float p = fast_exp2(fmaf(s[n][e], sc, nm[r]));
            s[n][e] = p;
            rs[r] += p;
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
      // O += P V over the live 16-key steps
#pragma unroll
      for (int t = 0; t < 4; ++t) {
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
            const int key = t * 16 + (mi & 1) * 8 + (lane & 7);
            const int d = (n + (mi >> 1)) * 8;
            ldsm_x4_t(b, cV + key * LDS + d);
            mma_bf16_16816(o[n], pa, b[0], b[1]);
            mma_bf16_16816(o[n + 1], pa, b[2], b[3]);
          }
        }
      }
    }
    if (kb == nkb - 1 && warp_live) {
      // normalise and store this head's rows
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
    __syncthreads();  // buffers of item `it` are refilled by issue(it + 2)
  }
}

}  // namespace ec
