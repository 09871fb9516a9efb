// ec_attn_tc.cuh -- short-sequence attention on the 5th-generation tensor
// cores, for head dim 32 (the MiniLM / all-MiniLM-L6 shape): the
// bidirectional padded softmax(Q K^T / sqrt(hd)) V of bert::encoder-layer
// (bert.lisp:226-248) for sequences of at most 256 tokens.
//
// A work unit is one (sequence, head, 128-query tile): one unit for
// sequences of at most 128 tokens, two for longer ones.  One persistent CTA
// per SM, warp-specialised, units pipelined:
//
//   warp 0       TMA producer: Q box of the unit's tile, K and V boxes of
//                all its keys (128-row boxes, 64-byte swizzle) into a
//                three-stage ring
//   warp 1       TMEM allocator + MMA issuer (one lane):
//                  S = Q K^T   one tcgen05.mma group over all keys (N = L
//                              rounded up to 16) into the unit's TMEM buffer
//                  O = P [V|1] tcgen05.mma with P read from TMEM (f16) and
//                              B = V (converted to f16 in place) next to a
//                              block of f16 ones: columns 32.. of O hold the
//                              row sums of P, accumulated in fp32
//                S of unit j+1 is issued before O of unit j, so the tensor
//                core computes ahead of the softmax
//   warps 2-5,   two softmax groups; group g takes the units j = g mod 2 and
//   warps 6-9    owns TMEM buffer g (columns 256 g .. 256 g + 255).  Thread
//                r of a group owns query row r (TMEM lane r): pass 1 reads
//                its scores for the row max, pass 2 reads them again and
//                writes p = 2^((s - max) log2(e) / sqrt(hd)) as f16 pairs
//                (cvt.rn.f16x2.f32 + ex2.approx.f16x2) over the columns of S
//                already consumed; the group converts the unit's V tile to
//                f16, then reads O and the row sum from TMEM and stores
//                O / sum as bf16 rows
//
// The whole row of scores is in TMEM at once, so the softmax needs no running
// max or rescaling, and each group's softmax overlaps the other group's MMAs
// and the producer's loads.  Every wait is bounded (mbarriers with the kernel
// abort flag); on a timeout the CTA records a status, lets copies and MMAs in
// flight land and frees its TMEM.
#pragma once

#include "ec_attn_short.cuh"
#include "ec_fa.cuh"

namespace ec {

struct TcShortArgs {
  const int2* seqs;  // (first token, length) per sequence, longest first
  int first;         // first sequence of this launch in seqs
  int nseq;          // sequences of this launch (all <= 256 tokens)
  int n_two;         // sequences [first, first + n_two) have more than 128 tokens
  int heads, kv_group;
  int q_off, k_off, v_off;
  __nv_bfloat16* out;  // [T, heads * 32]
  int ldo;
  float scale_log2;  // log2(e) / sqrt(32)
  unsigned* status;
};

constexpr int kTcsThreads = 320;  // producer, MMA, two softmax groups of four warps

struct TcsCfg {
  static constexpr int HD = 32;
  static constexpr int STAGES = 3;
  static constexpr uint32_t BOX = 8192;  // 128 rows x 64 B (one TMA box, one SW64 tile)
  static constexpr uint32_t Q_OFF = 0;
  static constexpr uint32_t K_OFF = BOX;      // two boxes: up to 256 keys
  static constexpr uint32_t V_OFF = 3 * BOX;  // two boxes
  static constexpr uint32_t STAGE_BYTES = 5 * BOX;
  static constexpr uint32_t ONES_OFF = STAGES * STAGE_BYTES;  // 256 rows x 64 B of f16 ones
  static constexpr uint32_t BAR_OFF = ONES_OFF + 2 * BOX;
  static constexpr size_t SMEM_BYTES = BAR_OFF + 256;
  static constexpr uint32_t GROUP = 512;  // 8 rows of 64 B (one 16-key MMA step = 2 groups)
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t BUF_COLS = 256;  // per softmax group: S, then P (f16) + O
  static constexpr uint32_t O_COL = 128;     // O (32 columns), then the row sums (32 more)
};

// unit u -> (sequence index, head, query tile); the two-tile sequences come
// first, their two tiles adjacent
__device__ __forceinline__ void tcs_unit(const TcShortArgs& a, int u, int& seq, int& h, int& qt) {
  const int n2 = a.n_two * a.heads * 2;
  int item;
  if (u < n2) {
    item = u >> 1;
    qt = u & 1;
  } else {
    item = a.n_two * a.heads + (u - n2);
    qt = 0;
  }
  seq = a.first + item / a.heads;
  h = item % a.heads;
}

__global__ void __launch_bounds__(kTcsThreads, 1)
    attn_tc_short_kernel(const __grid_constant__ CUtensorMap tm, const TcShortArgs a) {
  using Cfg = TcsCfg;
  constexpr int HD = Cfg::HD;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) report(a.status, kDevBadArg);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + Cfg::BAR_OFF);
  uint64_t* full = bars;           // [3] Q, K, V of the stage have landed
  uint64_t* empty = bars + 3;      // [3] the stage's last MMA has completed
  uint64_t* s_full = bars + 6;     // [2] S of the group's unit is in TMEM
  uint64_t* p_full = bars + 8;     // [2] P in TMEM, V converted (4 warp arrivals)
  uint64_t* o_full = bars + 10;    // [2] O of the group's unit is in TMEM
  uint64_t* buf_free = bars + 12;  // [2] the group has read O (4 warp arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nunits = (a.n_two * 2 + (a.nseq - a.n_two)) * a.heads;

  // the ones block: f16 1.0 everywhere (so its swizzle does not matter)
  {
    uint4* ones = reinterpret_cast<uint4*>(smem_raw + Cfg::ONES_OFF);
    for (int i = threadIdx.x; i < static_cast<int>(2 * Cfg::BOX / 16); i += kTcsThreads)
      ones[i] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 4);
      mbar_init(&o_full[g], 1);
      mbar_init(&buf_free[g], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int j = 0;
      for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++j) {
        const int s = j % Cfg::STAGES;
        const uint32_t ph = static_cast<uint32_t>(j / Cfg::STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        int seq, h, qt;
        tcs_unit(a, u, seq, h, qt);
        const int2 sq = a.seqs[seq];
        const int kvh = h / a.kv_group;
        const int nkb = (sq.y + 127) >> 7;
        uint8_t* st = smem_raw + s * Cfg::STAGE_BYTES;
        // rows past the sequence come from the next one (finite, masked) or
        // are zero-filled past the last token
        mbar_arrive_expect_tx(&full[s], (1 + 2 * nkb) * Cfg::BOX);
        tma_load_2d(st + Cfg::Q_OFF, &tm, &full[s], a.q_off + h * HD, sq.x + qt * 128);
        for (int b = 0; b < nkb; ++b) {
          tma_load_2d(st + Cfg::K_OFF + b * Cfg::BOX, &tm, &full[s], a.k_off + kvh * HD, sq.x + b * 128);
          tma_load_2d(st + Cfg::V_OFF + b * Cfg::BOX, &tm, &full[s], a.v_off + kvh * HD, sq.x + b * 128);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t ones_addr = smem_u32(smem_raw + Cfg::ONES_OFF);
      // P (f16, from TMEM) x [V | ones] (f16, MN-major): N = 64
      constexpr uint32_t IDESC_PV = make_idesc(0, 128, 64) | (1u << 16);
      auto lr_of = [&](int u) {
        int seq, h, qt;
        tcs_unit(a, u, seq, h, qt);
        return (a.seqs[seq].y + 15) & ~15;
      };
      auto issue_s = [&](int j, int u) {
        const int g = j & 1, s = j % Cfg::STAGES;
        tc_fence_after();
        const uint32_t idesc_s = make_idesc(1, 128, lr_of(u));
        const uint32_t st = smem_u32(smem_raw + s * Cfg::STAGE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16(tmem + g * Cfg::BUF_COLS, desc_kmajor<true>(st + Cfg::Q_OFF + kk * 32),
                   desc_kmajor<true>(st + Cfg::K_OFF + kk * 32), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[g]);
      };
      auto issue_pv = [&](int j, int u) {
        const int g = j & 1, s = j % Cfg::STAGES;
        tc_fence_after();
        const int nk = lr_of(u) / 16;
        const uint32_t v_addr = smem_u32(smem_raw + s * Cfg::STAGE_BYTES + Cfg::V_OFF);
        const uint32_t lbo = ones_addr - v_addr;  // the ones block is the second MN block
        const uint32_t buf = tmem + g * Cfg::BUF_COLS;
        for (int kk = 0; kk < nk; ++kk)
          umma_f16_ts(buf + Cfg::O_COL, buf + kk * 8,
                      desc_mnmajor<true>(v_addr + kk * 2 * Cfg::GROUP, lbo), IDESC_PV, kk > 0 ? 1u : 0u);
        umma_commit(&o_full[g]);
        umma_commit(&empty[s]);
      };
      // Issue in readiness order, so that the two groups' units do not wait
      // on each other: S of local unit js once its stage has landed and its
      // group's buffer is free (O of unit js - 2 read), P.V of unit jp once
      // its group's P is complete.  Each barrier can be at most one phase
      // ahead of the parity tested (the next phase needs this MMA), so the
      // parity tests are exact.
      int nloc = 0;
      for (int u = blockIdx.x; u < nunits; u += gridDim.x) ++nloc;
      int js = 0, jp = 0;
      uint64_t t_last = globaltimer_ns();
      while (jp < nloc) {
        bool moved = false;
        if (js < nloc &&
            mbar_test_wait(&full[js % Cfg::STAGES], static_cast<uint32_t>(js / Cfg::STAGES) & 1u) &&
            mbar_test_wait(&buf_free[js & 1], (static_cast<uint32_t>(js >> 1) & 1u) ^ 1u)) {
          issue_s(js, blockIdx.x + js * gridDim.x);
          ++js;
          moved = true;
        }
        if (jp < js && mbar_test_wait(&p_full[jp & 1], static_cast<uint32_t>(jp >> 1) & 1u)) {
          issue_pv(jp, blockIdx.x + jp * gridDim.x);
          ++jp;
          moved = true;
        }
        if (moved) {
          t_last = globaltimer_ns();
        } else if (*abort_flag || globaltimer_ns() - t_last > EC_WAIT_NS) {
          ok = false;
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int g = (warp - 2) >> 2;               // group
    const int quad = warp & 3;                   // TMEM lane quadrant of this warp
    const int r = quad * 32 + lane;              // query row within the tile
    const int gt = threadIdx.x - 64 - g * 128;  // thread within the group
    const uint32_t t_buf = tmem + (static_cast<uint32_t>(quad * 32) << 16) + g * Cfg::BUF_COLS;
    const float sc = a.scale_log2;
    int i = 0;
    for (int u = blockIdx.x + g * gridDim.x; u < nunits; u += 2 * gridDim.x, ++i) {
      const int j = 2 * i + g;
      const int s = j % Cfg::STAGES;
      const uint32_t ph = static_cast<uint32_t>(i) & 1u;
      int seq, h, qt;
      tcs_unit(a, u, seq, h, qt);
      const int2 sq = a.seqs[seq];
      const int L = sq.y;
      const int Lr = (L + 15) & ~15;
      if (!mbar_wait_warp(&s_full[g], ph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // V of the keys the P.V MMA reads, bf16 -> f16 in place.  The stage has
      // landed (S was computed from it); waiting on its barrier as well makes
      // the copy's writes visible to these threads.  The stage cannot be
      // refilled before this group's P of this unit is complete.
      if (!mbar_wait_warp(&full[s], static_cast<uint32_t>(j / Cfg::STAGES) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      {
        uint4* v = reinterpret_cast<uint4*>(smem_raw + s * Cfg::STAGE_BYTES + Cfg::V_OFF);
        for (int c = gt; c < Lr * 4; c += 128) {
          uint4 x = v[c];
          x.x = bf2_to_h2(x.x);
          x.y = bf2_to_h2(x.y);
          x.z = bf2_to_h2(x.z);
          x.w = bf2_to_h2(x.w);
          v[c] = x;
        }
      }
      // a warp whose 32 rows all lie past the sequence skips the softmax
      // (its P rows only feed O rows that are never stored)
      const bool warp_live = qt * 128 + quad * 32 < L;
      if (warp_live) {
        // pass 1: row max over the keys of the sequence, two 32-key chunks
        // per TMEM wait
        const int nch = (L + 31) >> 5;
        float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < nch; c += 2) {
          uint32_t v[2][32];
          tmem_ld_32x32b_x32(t_buf + c * 32, v[0]);
          if (c + 1 < nch) tmem_ld_32x32b_x32(t_buf + (c + 1) * 32, v[1]);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int k0 = (c + q) * 32;
            if (k0 + 32 <= L) {
#pragma unroll
              for (int k = 0; k < 32; k += 2) {
                m0 = fmaxf(m0, __uint_as_float(v[q][k]));
                m1 = fmaxf(m1, __uint_as_float(v[q][k + 1]));
              }
            } else if (k0 < L) {
#pragma unroll
              for (int k = 0; k < 32; ++k)
                if (k0 + k < L) m0 = fmaxf(m0, __uint_as_float(v[q][k]));
            }
          }
        }
        const float nm = -fmaxf(m0, m1) * sc;
        // pass 2: f16 p over the keys of every 16-key step the P.V MMA
        // reads; chunk c of S (columns 32c..) becomes P columns 16c.., which
        // S no longer needs
        const int nch2 = (Lr + 31) >> 5;
#pragma unroll 1
        for (int c = 0; c < nch2; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_buf + c * 32, v);
          tmem_wait_ld();
          uint32_t p[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[2 * k]), __uint_as_float(v[2 * k + 1])),
                                        make_float2(sc, sc), make_float2(nm, nm));
            p[k] = ex2_h2(cvt_h2(x.x, x.y));
          }
          if (c * 32 + 32 > L) {
            // keys past the sequence: p = 0 (low half = the even key)
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int key = c * 32 + 2 * k;
              if (key >= L)
                p[k] = 0u;
              else if (key + 1 >= L)
                p[k] &= 0xFFFFu;
            }
          }
          tmem_st_32x32b_x16(t_buf + c * 16, p);
        }
        tmem_wait_st();
      }
      // P and the converted V are complete: hand them to the MMA warp
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
      if (!mbar_wait_warp(&o_full[g], ph, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t o[32];
      float sum = 1.f;
      if (warp_live) {
        tmem_ld_32x32b_x32(t_buf + Cfg::O_COL, o);
        const uint32_t sm = tmem_ld_32x32b_x1(t_buf + Cfg::O_COL + 32);
        tmem_wait_ld();
        sum = __uint_as_float(sm);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&buf_free[g]);
      const int q = qt * 128 + r;
      if (warp_live && q < L) {
        const float inv = sum > 0.f ? 1.f / sum : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(a.out + static_cast<size_t>(sq.x + q) * a.ldo + h * HD);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          dst[k] = make_uint4(
              pack_bf16(__uint_as_float(o[8 * k]) * inv, __uint_as_float(o[8 * k + 1]) * inv),
              pack_bf16(__uint_as_float(o[8 * k + 2]) * inv, __uint_as_float(o[8 * k + 3]) * inv),
              pack_bf16(__uint_as_float(o[8 * k + 4]) * inv, __uint_as_float(o[8 * k + 5]) * inv),
              pack_bf16(__uint_as_float(o[8 * k + 6]) * inv, __uint_as_float(o[8 * k + 7]) * inv));
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
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

}  // namespace ec
