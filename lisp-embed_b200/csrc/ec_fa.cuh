// ec_fa.cuh -- varlen attention on the 5th-generation tensor cores.
//
// softmax(Q K^T * scale (+ bias)) V for one (128-query block, head) work item
// at a time, the triple loop of bert::encoder-layer (bert.lisp:226-248),
// bert::mpnet-layer (:408-423) and llama::layer-forward (llama.lisp:255-271):
//
//   per 128-key block j:
//     S_j = Q K_j^T          tcgen05.mma (A = Q, B = K, both K-major in smem)
//                            -> TMEM, double-buffered (columns 0 / 128)
//     softmax warps          one thread per query row reads its 128 scores
//                            from TMEM twice (max, then exp), keeps the
//                            running max / sum, writes P_j (bf16) to a
//                            128B-swizzled K-major shared-memory tile
//     O += P_j V_j           tcgen05.mma (A = P, B = V read MN-major straight
//                            from the row-major V tile) -> TMEM columns 256..
//   O is rescaled in TMEM only when the running max grows by more than 8
//   (log2 units); the final O / l is written as bf16.
//
// Persistent CTAs walk the work items (long sequences first); warp 0 issues
// TMA loads (Q once per item, K/V per block, 2 stages, next item prefetched),
// warp 1 issues the MMAs (S_{j+1} before PV_j), warps 2..5 run the softmax.
// All waits are bounded.
#pragma once

#include "ec_ptx.cuh"

namespace ec {

struct FaArgs {
  const int* cu;        // [nseq + 1]
  const int2* qblocks;  // (sequence, first query row), 128-row blocks, long first
  int nqb;
  int heads, kv_group;
  int q_off, k_off, v_off;
  __nv_bfloat16* out;   // [T, heads * HD]
  int ldo;
  float scale_log2;     // log2(e) / sqrt(HD)
  const float* relbias; // MODE 1: [heads][2 * rel_max - 1] (* log2 e)
  int rel_max;
  unsigned* status;
};

constexpr int kFaThreads = 192;  // producer, MMA, 4 softmax warps

template <int HD>
struct FaCfg {
  static_assert(HD == 64 || HD == 128, "head dim");
  static constexpr int AT = HD / 64;                      // 128-byte atoms per row
  static constexpr uint32_t TILE = AT * 16384;            // 128 rows x HD bf16
  static constexpr uint32_t P_BYTES = 2 * 16384;          // 128 x 128 bf16, 2 K-atoms
  static constexpr uint32_t BIAS_BYTES = 8192;
  static constexpr size_t SMEM_BYTES = 1024 + TILE /*Q*/ + 4 * TILE /*K,V x2*/ + P_BYTES +
                                       BIAS_BYTES + 512;
  static constexpr uint32_t O_COL = 256;
};

// MN-major operand, 128-byte swizzle: 64 elements contiguous along MN, rows
// along K 128 B apart, 8-row K groups 1024 B apart (SBO), 64-element MN
// blocks `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t desc_sw128_mnmajor(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

__device__ __forceinline__ float fa_exp2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// MODE 0: bidirectional with padding; 1: + relative bias; 2: causal.
template <int HD, int MODE>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQKV, const FaArgs a) {
  using Cfg = FaCfg<HD>;
  constexpr int AT = Cfg::AT;
  constexpr bool kBias = MODE == 1;
  constexpr bool kCausal = MODE == 2;
  constexpr uint32_t IDESC_S = make_idesc(1, 128, 128);
  constexpr uint32_t IDESC_PV = make_idesc(1, 128, HD) | (1u << 16);  // B MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::TILE;            // 2 stages
  uint8_t* sV = sK + 2 * Cfg::TILE;        // 2 stages
  uint8_t* sP = sV + 2 * Cfg::TILE;
  float* sBias = reinterpret_cast<float*>(sP + Cfg::P_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sBias) + Cfg::BIAS_BYTES);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;
  uint64_t* kv_full = q_empty + 1;   // [2]
  uint64_t* kv_empty = kv_full + 2;  // [2]
  uint64_t* s_full = kv_empty + 2;   // [2]
  uint64_t* s_empty = s_full + 2;    // [2]
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 1;
  uint64_t* o_full = p_empty + 1;
  uint64_t* o_empty = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nitems = a.nqb * a.heads;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 4);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmQKV);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // item -> (sequence base, length, first query row, head, key blocks)
  auto item_info = [&](int t, int& base, int& L, int& q0, int& h, int& nkb) {
    const int2 qb = a.qblocks[t / a.heads];
    h = t % a.heads;
    base = a.cu[qb.x];
    L = a.cu[qb.x + 1] - base;
    q0 = qb.y;
    const int kv_end = kCausal ? min(L, q0 + 128) : L;
    nkb = (kv_end + 127) >> 7;
  };

  if (warp == 0) {
    // --------------------------------------------------------------- producer
    if (elect_one()) {
      int st = 0;
      uint32_t kv_ph = 0, q_ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < nitems; t += gridDim.x) {
        int base, L, q0, h, nkb;
        item_info(t, base, L, q0, h, nkb);
        const int kvh = h / a.kv_group;
        if (!mbar_wait(q_empty, q_ph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        q_ph ^= 1;
        mbar_arrive_expect_tx(q_full, Cfg::TILE);
        for (int at = 0; at < AT; ++at)
          tma_load_2d(sQ + at * 16384, &tmQKV, q_full, a.q_off + h * HD + at * 64, base + q0);
        for (int j = 0; j < nkb; ++j) {
          if (!mbar_wait(&kv_empty[st], kv_ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * Cfg::TILE);
          for (int at = 0; at < AT; ++at) {
            tma_load_2d(sK + st * Cfg::TILE + at * 16384, &tmQKV, &kv_full[st],
                        a.k_off + kvh * HD + at * 64, base + j * 128);
            tma_load_2d(sV + st * Cfg::TILE + at * 16384, &tmQKV, &kv_full[st],
                        a.v_off + kvh * HD + at * 64, base + j * 128);
          }
          if (++st == 2) {
            st = 0;
            kv_ph ^= 1;
          }
        }
      }
      if (!ok) {
        report(a.status, kDevTimeoutProducer);
        *abort_flag = 1;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      int st = 0;
      uint32_t kv_ph = 0, q_ph = 0, p_ph = 0, oe_ph = 0;
      uint32_t se_ph[2] = {0, 0};
      int sbuf = 0;
      bool ok = true;
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      auto mma_s = [&](int& used_st) -> bool {
        if (!mbar_wait(&kv_full[st], kv_ph, abort_flag)) return false;
        if (!mbar_wait(&s_empty[sbuf], se_ph[sbuf] ^ 1, abort_flag)) return false;
        se_ph[sbuf] ^= 1;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * Cfg::TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16(tmem_base + sbuf * 128, desc_sw128_kmajor(q_addr + off),
                   desc_sw128_kmajor(k_addr + off), IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sbuf]);
        sbuf ^= 1;
        used_st = st;
        if (++st == 2) {
          st = 0;
          kv_ph ^= 1;
        }
        return true;
      };
      auto mma_pv = [&](int j, int used_st) -> bool {
        if (j == 0) {
          if (!mbar_wait(o_empty, oe_ph ^ 1, abort_flag)) return false;
          oe_ph ^= 1;
        }
        if (!mbar_wait(p_full, p_ph, abort_flag)) return false;
        p_ph ^= 1;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + used_st * Cfg::TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem_base + Cfg::O_COL,
                   desc_sw128_kmajor(p_addr + (kk >> 2) * 16384 + (kk & 3) * 32),
                   desc_sw128_mnmajor(v_addr + kk * 2048, 16384), IDESC_PV,
                   (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kv_empty[used_st]);
        umma_commit(p_empty);
        umma_commit(o_full);
        return true;
      };
      for (int t = blockIdx.x; ok && t < nitems; t += gridDim.x) {
        int base, L, q0, h, nkb;
        item_info(t, base, L, q0, h, nkb);
        if (!mbar_wait(q_full, q_ph, abort_flag)) {
          ok = false;
          break;
        }
        q_ph ^= 1;
        tc_fence_after();
        int prev_st = 0, cur_st = 0;
        if (!mma_s(cur_st)) {
          ok = false;
          break;
        }
        for (int j = 1; ok && j < nkb; ++j) {
          prev_st = cur_st;
          if (!mma_s(cur_st) || !mma_pv(j - 1, prev_st)) ok = false;
        }
        if (!ok) break;
        umma_commit(q_empty);  // every S of this item has read Q
        if (!mma_pv(nkb - 1, cur_st)) ok = false;
      }
      if (!ok) {
        report(a.status, kDevTimeoutMma);
        *abort_flag = 1;
      }
    }
  } else {
    // --------------------------------------------------------------- softmax
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row in the block == TMEM lane
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    int sbuf = 0;
    uint32_t sf_ph[2] = {0, 0};
    uint32_t pe_ph = 0;
    long long pv_done = 0;  // PVs of earlier items (global PV index base)
    bool ok = true;
    uint8_t* p_row0 = sP + r * 128;          // K-atom 0 (keys 0..63)
    uint8_t* p_row1 = sP + 16384 + r * 128;  // K-atom 1 (keys 64..127)
    for (int t = blockIdx.x; ok && t < nitems; t += gridDim.x) {
      int base, L, q0, h, nkb;
      item_info(t, base, L, q0, h, nkb);
      const int q = q0 + r;  // query position in the sequence
      if (kBias) {
        named_bar(1, 128);  // previous item's readers are done
        const int nb = 2 * a.rel_max - 1;
        const float* src = a.relbias + static_cast<size_t>(h) * nb;
        for (int i = threadIdx.x - 64; i < 2 * L - 1 && i < 2048; i += 128)
          sBias[i] = src[i - (L - 1) + a.rel_max - 1];
        named_bar(1, 128);
      }
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < nkb; ++j) {
        if (!mbar_wait(&s_full[sbuf], sf_ph[sbuf], abort_flag)) {
          ok = false;
          break;
        }
        sf_ph[sbuf] ^= 1;
        tc_fence_after();
        const uint32_t s_addr = t_lane + sbuf * 128;
        const int k0 = j * 128;
        const bool need_mask = (k0 + 128 > L) || (kCausal && k0 + 127 > q0);
        // pass 1: row max of the logits (log2 units)
        float mx = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(s_addr + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float x = __uint_as_float(v[i]) * a.scale_log2;
            const int key = k0 + c * 32 + i;
            if (kBias) {
              const int bi = q - key + (L - 1);
              x += sBias[bi < 0 ? 0 : (bi > 2046 ? 2046 : bi)];
            }
            if (need_mask && (key >= L || (kCausal && key > q))) x = -INFINITY;
            mx = fmaxf(mx, x);
          }
        }
        // lazy rescale: keep the stale max unless the new one is 2^8 larger
        if (mx > m_run + 8.0f) {
          const float corr = fa_exp2(m_run - mx);
          if (j > 0) {
            // O holds PV of blocks < j: wait for PV(j-1), then scale it
            const long long g = pv_done + j - 1;
            if (!mbar_wait(o_full, static_cast<uint32_t>(g & 1), abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
              uint32_t v[32];
              tmem_ld_32x32b_x32(t_lane + Cfg::O_COL + c * 32, v);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
              tmem_st_32x32b_x32(t_lane + Cfg::O_COL + c * 32, v);
            }
            tmem_wait_st();
          }
          l_run *= corr;
          m_run = mx;
        }
        // pass 2: P = exp2(logit - m_run) to shared memory, row sum
        if (!mbar_wait(p_empty, pe_ph ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        pe_ph ^= 1;
        float sum = 0.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(s_addr + c * 32, v);
          tmem_wait_ld();
          float p[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float x = __uint_as_float(v[i]) * a.scale_log2;
            const int key = k0 + c * 32 + i;
            if (kBias) {
              const int bi = q - key + (L - 1);
              x += sBias[bi < 0 ? 0 : (bi > 2046 ? 2046 : bi)];
            }
            float e = fa_exp2(x - m_run);
            if (need_mask && (key >= L || (kCausal && key > q))) e = 0.f;
            p[i] = e;
            sum += e;
          }
          uint8_t* prow = (c < 2) ? p_row0 : p_row1;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c16 = (c & 1) * 4 + u;  // 16-byte chunk within the 128-byte row
            *reinterpret_cast<uint4*>(prow + ((c16 ^ (r & 7)) << 4)) =
                make_uint4(pack_bf16(p[8 * u], p[8 * u + 1]), pack_bf16(p[8 * u + 2], p[8 * u + 3]),
                           pack_bf16(p[8 * u + 4], p[8 * u + 5]),
                           pack_bf16(p[8 * u + 6], p[8 * u + 7]));
          }
        }
        l_run += sum;
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s_empty[sbuf]);
          mbar_arrive(p_full);
        }
        sbuf ^= 1;
      }
      if (!ok) break;
      // final: O / l for rows inside the sequence
      const long long g = pv_done + nkb - 1;
      if (!mbar_wait(o_full, static_cast<uint32_t>(g & 1), abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = a.out + static_cast<size_t>(base + q) * a.ldo + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_lane + Cfg::O_COL + c * 32, v);
        tmem_wait_ld();
        if (q < L) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            dst[u] = make_uint4(pack_bf16(__uint_as_float(v[8 * u]) * inv, __uint_as_float(v[8 * u + 1]) * inv),
                                pack_bf16(__uint_as_float(v[8 * u + 2]) * inv, __uint_as_float(v[8 * u + 3]) * inv),
                                pack_bf16(__uint_as_float(v[8 * u + 4]) * inv, __uint_as_float(v[8 * u + 5]) * inv),
                                pack_bf16(__uint_as_float(v[8 * u + 6]) * inv, __uint_as_float(v[8 * u + 7]) * inv));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
      pv_done += nkb;
    }
    if (!ok) {
      report(a.status, kDevTimeoutEpilogue);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace ec
