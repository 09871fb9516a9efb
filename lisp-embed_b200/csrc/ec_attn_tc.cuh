// ec_attn_tc.cuh -- short-sequence attention on the 5th-generation tensor
// cores, for head dim 32 (the MiniLM / all-MiniLM-L6 shape): the
// bidirectional padded softmax(Q K^T / sqrt(hd)) V of bert::encoder-layer
// (bert.lisp:226-248) for sequences of at most 256 tokens.
//
// One work item is one (sequence, head); persistent CTAs of four warps walk
// the items (longest sequences first), two CTAs per SM.  Per item:
//
//   TMA        Q, K, V rows of the head (128-row boxes, 64-byte swizzle)
//   per 128-query tile:
//     S = Q K^T       one tcgen05.mma group over all keys (N = L rounded up
//                     to 16, at most 256) -> TMEM columns [0, N)
//     softmax         thread r owns query row r (TMEM lane r): pass 1 reads
//                     its scores from TMEM for the row max, pass 2 reads them
//                     again, writes p = 2^((s - max) * log2e / sqrt(hd)) as
//                     bf16 into a 128-byte-swizzled K-major P tile in shared
//                     memory (keys past the sequence -> 0) and sums p in fp32
//     O = P V         tcgen05.mma, V read MN-major from its row-major tile
//                     -> TMEM columns [0, 32) (S is consumed by then)
//     O / sum         bf16 rows to global memory
//
// The whole row of scores is in TMEM at once, so the softmax needs no
// running max or rescaling; the tensor core does all the multiply-adds and
// the four warps do only the exponentials (the kernel's bound).  Every wait
// is bounded (mbarriers with the kernel abort flag, a bounded CTA
// rendezvous in place of __syncthreads inside the item loop).
#pragma once

#include "ec_fa.cuh"

namespace ec {

struct TcShortArgs {
  const int2* seqs;  // (first token, length) per sequence, longest first
  int first;         // first sequence of this launch in seqs
  int nseq;          // sequences of this launch (all <= 256 tokens)
  int heads, kv_group;
  int q_off, k_off, v_off;
  __nv_bfloat16* out;  // [T, heads * 32]
  int ldo;
  float scale_log2;  // log2(e) / sqrt(32)
  unsigned* status;
};

constexpr int kTcsThreads = 128;

struct TcsCfg {
  static constexpr int HD = 32;
  static constexpr uint32_t BOX = 8192;          // 128 rows x 64 B (one TMA box, one SW64 atom)
  static constexpr uint32_t Q_BYTES = 2 * BOX;   // up to 256 query rows
  static constexpr uint32_t K_BYTES = 2 * BOX;   // up to 256 keys
  static constexpr uint32_t V_BYTES = 2 * BOX;
  static constexpr uint32_t P_ATOM = 16384;      // 128 rows x 64 keys bf16 (128-byte rows)
  static constexpr uint32_t P_BYTES = 4 * P_ATOM;  // 256 keys
  static constexpr uint32_t GROUP = 512;         // 8 rows of 64 B
  static constexpr size_t SMEM_BYTES = P_BYTES + Q_BYTES + K_BYTES + V_BYTES + 256;
  static constexpr uint32_t TMEM_COLS = 256;
};

__global__ void __launch_bounds__(kTcsThreads, 2)
    attn_tc_short_kernel(const __grid_constant__ CUtensorMap tm, const TcShortArgs a) {
  using Cfg = TcsCfg;
  constexpr int HD = Cfg::HD;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) report(a.status, kDevBadArg);
    return;
  }
  uint8_t* sP = smem_raw;
  uint8_t* sQ = sP + Cfg::P_BYTES;
  uint8_t* sK = sQ + Cfg::Q_BYTES;
  uint8_t* sV = sK + Cfg::K_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + Cfg::V_BYTES);
  uint64_t* ld_full = bars;      // Q, K, V of the item have landed
  uint64_t* s_full = bars + 1;   // S of the tile is in TMEM
  uint64_t* o_full = bars + 2;   // O of the tile is in TMEM
  uint64_t* cbar = bars + 3;     // CTA rendezvous (128 threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(ld_full, 1);
    mbar_init(s_full, 1);
    mbar_init(o_full, 1);
    mbar_init(cbar, kTcsThreads);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int r = warp * 32 + lane;  // query row within a tile == TMEM lane
  const float sc = a.scale_log2;
  constexpr uint32_t IDESC_PV = make_idesc(1, 128, HD) | (1u << 16);  // B MN-major

  uint32_t ld_ph = 0, s_ph = 0, o_ph = 0, c_ph = 0;
  bool ok = true;
  const int nitems = a.nseq * a.heads;
  for (int t = blockIdx.x; ok && t < nitems; t += gridDim.x) {
    const int2 sq = a.seqs[a.first + t / a.heads];
    const int h = t % a.heads;
    const int base = sq.x, L = sq.y;
    const int kvh = h / a.kv_group;
    const int nqt = (L + 127) >> 7;  // 128-row tiles of queries (and boxes of K, V)
    const int Lr = (L + 15) & ~15;   // keys rounded up to whole 16-key MMA steps
    if (threadIdx.x == 0) {
      // rows past the sequence come from the next one (finite, masked below)
      // or are zero-filled past the last token
      mbar_arrive_expect_tx(ld_full, 3 * nqt * Cfg::BOX);
      for (int b = 0; b < nqt; ++b) {
        tma_load_2d(sQ + b * Cfg::BOX, &tm, ld_full, a.q_off + h * HD, base + b * 128);
        tma_load_2d(sK + b * Cfg::BOX, &tm, ld_full, a.k_off + kvh * HD, base + b * 128);
        tma_load_2d(sV + b * Cfg::BOX, &tm, ld_full, a.v_off + kvh * HD, base + b * 128);
      }
    }
    if (!mbar_wait_warp(ld_full, ld_ph, abort_flag)) {
      ok = false;
      break;
    }
    ld_ph ^= 1;
    for (int qt = 0; qt < nqt; ++qt) {
      if (threadIdx.x == 0) {
        tc_fence_after();
        const uint32_t idesc_s = make_idesc(1, 128, Lr);
        const uint32_t q_addr = smem_u32(sQ + qt * Cfg::BOX), k_addr = smem_u32(sK);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem, desc_kmajor<true>(q_addr + kk * 32), desc_kmajor<true>(k_addr + kk * 32),
                   idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
      }
      if (!mbar_wait_warp(s_full, s_ph, abort_flag)) {
        ok = false;
        break;
      }
      s_ph ^= 1;
      tc_fence_after();
      const int q = qt * 128 + r;  // query position in the sequence
      // a warp whose 32 rows all lie past the sequence skips the softmax
      // (its P rows only feed O rows that are never stored)
      const bool warp_live = qt * 128 + warp * 32 < L;
      float sum = 0.f;
      if (warp_live) {
        // pass 1: row max over the keys of the sequence
        const int nch = (L + 31) >> 5;
        float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_lane + c * 32, v);
          tmem_wait_ld();
          if (c * 32 + 32 <= L) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              m0 = fmaxf(m0, __uint_as_float(v[i]));
              m1 = fmaxf(m1, __uint_as_float(v[i + 1]));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i < L) m0 = fmaxf(m0, __uint_as_float(v[i]));
          }
        }
        const float nm = -fmaxf(m0, m1) * sc;
        // pass 2: p for the keys of every 16-key step the P.V MMA reads
        const int nch2 = (Lr + 31) >> 5;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 1
        for (int c = 0; c < nch2; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_lane + c * 32, v);
          tmem_wait_ld();
          float p[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float e = fa_exp2(fmaf(__uint_as_float(v[i]), sc, nm));
            p[i] = c * 32 + i < L ? e : 0.f;
          }
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            s0 += p[i];
            s1 += p[i + 1];
            s2 += p[i + 2];
            s3 += p[i + 3];
          }
          // keys 32c.. are 16-byte chunks (c & 1) * 4 .. + 3 of K-atom c / 2
          uint8_t* prow = sP + (c >> 1) * Cfg::P_ATOM + r * 128;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c16 = (c & 1) * 4 + u;
            *reinterpret_cast<uint4*>(prow + ((c16 ^ (r & 7)) << 4)) =
                make_uint4(pack_bf16(p[8 * u], p[8 * u + 1]), pack_bf16(p[8 * u + 2], p[8 * u + 3]),
                           pack_bf16(p[8 * u + 4], p[8 * u + 5]), pack_bf16(p[8 * u + 6], p[8 * u + 7]));
          }
        }
        sum = (s0 + s1) + (s2 + s3);
      }
      // P complete and every TMEM read of S done before O overwrites it
      fence_proxy_async_smem();
      tc_fence_before();
      if (!mbar_sync(cbar, c_ph, abort_flag)) {
        ok = false;
        break;
      }
      if (threadIdx.x == 0) {
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP), v_addr = smem_u32(sV);
        for (int kk = 0; kk < Lr / 16; ++kk)
          umma_f16(tmem, desc_sw128_kmajor(p_addr + (kk >> 2) * Cfg::P_ATOM + (kk & 3) * 32),
                   desc_mnmajor<true>(v_addr + kk * 2 * Cfg::GROUP, Cfg::BOX), IDESC_PV,
                   kk > 0 ? 1u : 0u);
        umma_commit(o_full);
      }
      if (!mbar_wait_warp(o_full, o_ph, abort_flag)) {
        ok = false;
        break;
      }
      o_ph ^= 1;
      tc_fence_after();
      if (warp_live) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_lane, v);
        tmem_wait_ld();
        if (q < L) {
          const float inv = sum > 0.f ? 1.f / sum : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(base + q) * a.ldo + h * HD);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            dst[u] = make_uint4(
                pack_bf16(__uint_as_float(v[8 * u]) * inv, __uint_as_float(v[8 * u + 1]) * inv),
                pack_bf16(__uint_as_float(v[8 * u + 2]) * inv, __uint_as_float(v[8 * u + 3]) * inv),
                pack_bf16(__uint_as_float(v[8 * u + 4]) * inv, __uint_as_float(v[8 * u + 5]) * inv),
                pack_bf16(__uint_as_float(v[8 * u + 6]) * inv, __uint_as_float(v[8 * u + 7]) * inv));
        }
      }
      // every O read done before the next tile's S (or the next item's
      // loads) overwrite TMEM and shared memory
      tc_fence_before();
      if (!mbar_sync(cbar, c_ph, abort_flag)) {
        ok = false;
        break;
      }
    }
  }
  if (!ok) {
    report(a.status, kDevTimeoutOther);
    *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // let copies and MMAs already in flight land before the CTA exits
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace ec
