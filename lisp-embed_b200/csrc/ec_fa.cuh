// ec_fa.cuh -- varlen attention on the 5th-generation tensor cores.
//
// softmax(Q K^T * scale (+ bias)) V for one (128-query block, head) work item
// at a time, the triple loop of bert::encoder-layer (bert.lisp:226-248),
// bert::mpnet-layer (:408-423) and llama::layer-forward (llama.lisp:255-271):
//
//   per 128-key block j:
//     S_j = Q K_j^T          tcgen05.mma (A = Q, B = K, both K-major in smem)
//                            -> TMEM, double-buffered (columns 0 / 128)
//     softmax warps          two threads per query row read its 128 scores
//                            from TMEM twice (max, then exp), keep the
//                            running max / sum, writes P_j (bf16) to a
//                            128B-swizzled K-major shared-memory tile
//     O += P_j V_j           tcgen05.mma (A = P, B = V read MN-major straight
//                            from the row-major V tile) -> TMEM columns 256..
//   O is rescaled in TMEM only when the running max grows by more than 8
//   (log2 units); the final O / l is written as bf16.
//
// Persistent CTAs walk the work items (long sequences first); warp 0 issues
// TMA loads (Q once per item, K/V per block, 2 stages, next item prefetched),
// warp 1 issues the MMAs (S_{j+1} before PV_j), warps 2..9 run the softmax,
// two per query row (one per 64-key half of each block).
// All waits are bounded.
#pragma once

#include "ec_ptx.cuh"

namespace ec {

struct FaArgs {
  const int* cu;        // [nseq + 1]
  const int4* qinfo;    // per 128-row query block: (first token, length, first row, 0), long first
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

// warps 0..7 softmax (two warpgroups), 8 TMA producer, 9 MMA issuer; with
// ten warps a thread gets at most 168 registers (three warps share one SM
// sub-partition's 16K registers), which the softmax code fits without spills
constexpr int kFaThreads = 320;

template <int HD, int MODE>
struct FaCfg {
  static_assert(HD == 32 || HD == 64 || HD == 128, "head dim");
  // Q / K / V rows of HD bf16: 64-byte rows with 64-byte swizzle for HD 32,
  // else 128-byte atoms with 128-byte swizzle (two atoms side by side for 128)
  static constexpr bool SW64 = HD == 32;
  static constexpr int AT = HD == 128 ? 2 : 1;             // atoms along the head dim
  static constexpr uint32_t ATOM = SW64 ? 8192 : 16384;    // 128 rows of one atom
  static constexpr uint32_t TILE = AT * ATOM;              // 128 rows x HD bf16
  static constexpr uint32_t GROUP = SW64 ? 512 : 1024;     // 8-row group stride
  static constexpr int BOX_C = SW64 ? 32 : 64;             // TMA box columns
  static constexpr uint32_t P_BYTES = 2 * 2 * 16384;       // 2 buffers of 128 x 128 bf16
  static constexpr uint32_t BIAS_BYTES = MODE == 1 ? 8192 : 0;  // bias of i - j + 127 + L
  static constexpr uint32_t XCH_BYTES = 2 * 8 * 32 * 4;    // partner row max / sum slots
  // no alignment slack: the kernel checks that dynamic shared memory starts
  // on a 1024-byte boundary (it does when the kernel has no static smem)
  static constexpr size_t SMEM_BYTES = TILE /*Q*/ + 4 * TILE /*K,V x2*/ + P_BYTES +
                                       BIAS_BYTES + XCH_BYTES + 512;
  static_assert(SMEM_BYTES <= 232448, "shared memory");
  static constexpr uint32_t O_COL = 256;
};

// K-major operand tile: rows of 64 B (64-byte swizzle, 512 B groups) or
// 128 B (128-byte swizzle, 1024 B groups)
template <bool SW64>
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t smem_addr) {
  if constexpr (!SW64) return desc_sw128_kmajor(smem_addr);
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;  // SWIZZLE_64B
  return d;
}

// MN-major operand (V read from its row-major tile): 64 (128-byte swizzle) or
// 32 (64-byte swizzle) elements contiguous along MN, K rows one row apart,
// 8-row K groups one group apart (SBO), MN blocks `lbo` bytes apart (LBO).
template <bool SW64>
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((SW64 ? 512u : 1024u) >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(SW64 ? 4u : 2u) << 61;
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
  using Cfg = FaCfg<HD, MODE>;
  constexpr int AT = Cfg::AT;
  constexpr bool kBias = MODE == 1;
  constexpr bool kCausal = MODE == 2;
  constexpr uint32_t IDESC_S = make_idesc(1, 128, 128);
  constexpr uint32_t IDESC_PV = make_idesc(1, 128, HD) | (1u << 16);  // B MN-major

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // swizzled tiles need 1024-byte alignment
    if (threadIdx.x == 0) report(a.status, kDevBadArg);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::TILE;            // 2 stages
  uint8_t* sV = sK + 2 * Cfg::TILE;        // 2 stages
  uint8_t* sP = sV + 2 * Cfg::TILE;
  float* sBias = reinterpret_cast<float*>(sP + Cfg::P_BYTES);
  float* sX = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sBias) + Cfg::BIAS_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sX) + Cfg::XCH_BYTES);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;
  uint64_t* kv_full = q_empty + 1;   // [2]
  uint64_t* kv_empty = kv_full + 2;  // [2]
  uint64_t* s_full = kv_empty + 2;   // [2]
  uint64_t* s_empty = s_full + 2;    // [2]
  uint64_t* p_full = s_empty + 2;    // [2]
  uint64_t* p_empty = p_full + 2;    // [2]
  uint64_t* o_full = p_empty + 2;    // [2]: PV of even / odd global block index
  uint64_t* o_empty = o_full + 2;
  uint64_t* xbar = o_empty + 1;  // [4 quads][2 slots] partner rendezvous, 64 threads
  uint64_t* bbar = xbar + 8;     // bias table rendezvous, 256 threads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bbar + 1);
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
      mbar_init(&s_empty[i], 8);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 8);
      mbar_init(&p_empty[i], 1);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(o_empty, 8);
    for (int i = 0; i < 8; ++i) mbar_init(&xbar[i], 64);
    mbar_init(bbar, 256);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8 && lane == 0) tma_prefetch_desc(&tmQKV);
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // item -> (sequence base, length, first query row, head, key blocks)
  auto item_info = [&](int t, int& base, int& L, int& q0, int& h, int& nkb) {
    const int4 qb = a.qinfo[t / a.heads];
    h = t % a.heads;
    base = qb.x;
    L = qb.y;
    q0 = qb.z;
    const int kv_end = kCausal ? min(L, q0 + 128) : L;
    nkb = (kv_end + 127) >> 7;
  };

  if (warp == 8) {
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
          tma_load_2d(sQ + at * Cfg::ATOM, &tmQKV, q_full, a.q_off + h * HD + at * 64, base + q0);
        for (int j = 0; j < nkb; ++j) {
          if (!mbar_wait(&kv_empty[st], kv_ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * Cfg::TILE);
          for (int at = 0; at < AT; ++at) {
            tma_load_2d(sK + st * Cfg::TILE + at * Cfg::ATOM, &tmQKV, &kv_full[st],
                        a.k_off + kvh * HD + at * 64, base + j * 128);
            tma_load_2d(sV + st * Cfg::TILE + at * Cfg::ATOM, &tmQKV, &kv_full[st],
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
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      int st = 0;
      uint32_t kv_ph = 0, q_ph = 0, oe_ph = 0;
      // phase parities of the two-entry barrier pairs, one bit per entry
      // (bit arrays, not indexed arrays, so they stay in registers)
      uint32_t se_bits = 0, pf_bits = 0;
      int sbuf = 0;
      long long pv_count = 0;  // global PV index: P buffer and o_full barrier parity
      bool ok = true;
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      auto mma_s = [&](int& used_st) -> bool {
        if (!mbar_wait(&kv_full[st], kv_ph, abort_flag)) return false;
        if (!mbar_wait(&s_empty[sbuf], ((se_bits >> sbuf) & 1u) ^ 1u, abort_flag)) return false;
        se_bits ^= 1u << sbuf;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * Cfg::TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * Cfg::ATOM + (kk & 3) * 32;
          umma_f16(tmem_base + sbuf * 128, desc_kmajor<Cfg::SW64>(q_addr + off),
                   desc_kmajor<Cfg::SW64>(k_addr + off), IDESC_S, kk > 0 ? 1u : 0u);
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
        const int pb = static_cast<int>(pv_count & 1);
        if (!mbar_wait(&p_full[pb], (pf_bits >> pb) & 1u, abort_flag)) return false;
        pf_bits ^= 1u << pb;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + used_st * Cfg::TILE);
        const uint32_t pa = p_addr + pb * 32768;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem_base + Cfg::O_COL,
                   desc_sw128_kmajor(pa + (kk >> 2) * 16384 + (kk & 3) * 32),
                   desc_mnmajor<Cfg::SW64>(v_addr + kk * 2 * Cfg::GROUP, Cfg::ATOM), IDESC_PV,
                   (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kv_empty[used_st]);
        umma_commit(&p_empty[pb]);
        umma_commit(&o_full[pb]);
        ++pv_count;
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
  } else if (warp < 8) {
    // --------------------------------------------------------------- softmax
    // warps 0..7: TMEM lane quadrant warp % 4 (query rows), key half
    // warp / 4: keys [64 * half, 64 * half + 64) of every block, which is
    // exactly one K-atom of P; partners exchange row max / sum in smem.
    const int sw = warp;
    const int quad = warp & 3;
    const int half = sw >> 2;
    const int r = quad * 32 + lane;  // query row in the block == TMEM lane
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr int OH = HD / 2;       // O columns handled by this warp
    int sbuf = 0;
    uint32_t sf_bits = 0, pe_bits = 0;  // phase parity per buffer, one bit each
    long long pv_done = 0;  // PVs of earlier items (global PV index base)
    bool ok = true;
    uint8_t* p_row = sP + half * 16384 + r * 128;  // this warp's K-atom of P buffer 0
    // wait for PV with global index g: o_full[g & 1] completes once per PV of
    // that parity, so its phase parity is (g >> 1) & 1.  Every PV up to g - 2
    // is already known complete (the P-buffer waits), so the parity test is
    // never two phases behind.
    auto wait_pv = [&](long long g) -> bool {
      return mbar_wait_warp(&o_full[g & 1], static_cast<uint32_t>((g >> 1) & 1), abort_flag);
    };
    float* xch = sX;                               // [2 slots][8 warps][32]
    int xslot = 0;
    uint32_t xbits = 0, bph = 0;
    // partner's value for this row; false if the rendezvous gave up
    auto exchange = [&](float v, float& other) -> bool {
      xch[(xslot * 8 + sw) * 32 + lane] = v;
      mbar_arrive(&xbar[quad * 2 + xslot]);
      const bool fine = mbar_wait_warp(&xbar[quad * 2 + xslot], (xbits >> xslot) & 1u, abort_flag);
      xbits ^= 1u << xslot;
      other = xch[(xslot * 8 + (sw ^ 4)) * 32 + lane];
      xslot ^= 1;
      return fine;
    };
    for (int t = blockIdx.x; ok && t < nitems; t += gridDim.x) {
      int base, L, q0, h, nkb;
      item_info(t, base, L, q0, h, nkb);
      const int q = q0 + r;  // query position in the sequence
      if (kBias) {
        if (!mbar_sync(bbar, bph, abort_flag)) {  // previous item's readers are done
          ok = false;
          break;
        }
        // sBias[i - j + 127 + L] for every (query i, key j) a block can pair:
        // i <= L + 126, j <= L + 126, so the index stays in [1, 2L + 253]
        const int nb = 2 * a.rel_max - 1;
        const float* src = a.relbias + static_cast<size_t>(h) * nb;
        for (int i = threadIdx.x; i < 2048; i += 256) {
          const int dlt = i - 127 - L;  // i - j
          sBias[i] = (dlt > -(a.rel_max) && dlt < a.rel_max) ? src[dlt + a.rel_max - 1] : 0.f;
        }
        if (!mbar_sync(bbar, bph, abort_flag)) {
          ok = false;
          break;
        }
      }
      const bool warp_live = q0 + quad * 32 < L;  // both partners agree
      float m_run = -INFINITY, l_part = 0.f;
      for (int j = 0; j < nkb; ++j) {
        if (!mbar_wait_warp(&s_full[sbuf], (sf_bits >> sbuf) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        sf_bits ^= 1u << sbuf;
        tc_fence_after();
        const int kh0 = j * 128 + half * 64;  // first key of this warp's half
        const uint32_t s_addr = t_lane + sbuf * 128 + half * 64;
        const bool need_mask = (kh0 + 64 > L) || (kCausal && kh0 + 63 > q0);
        const int live_chunks = max(0, min(2, (L - kh0 + 31) >> 5));
        if (warp_live) {
          float mx = -INFINITY;
#pragma unroll 1
          for (int c = 0; c < live_chunks; ++c) {
            uint32_t v[1][32];
            tmem_ld_32x32b_x32(s_addr + c * 32, v[0]);
            tmem_wait_ld();
            if (!need_mask && !kBias) {
#pragma unroll
              for (int i = 0; i < 32; i += 2)
                mx = fmaxf(mx, fmaxf(__uint_as_float(v[0][i]), __uint_as_float(v[0][i + 1])));
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                float x = __uint_as_float(v[0][i]);
                const int key = kh0 + c * 32 + i;
                if (kBias) x = fmaf(x, a.scale_log2, sBias[q - key + 127 + L]);
                if (need_mask && (key >= L || (kCausal && key > q))) x = -INFINITY;
                mx = fmaxf(mx, x);
              }
            }
          }
          if (!kBias) mx *= a.scale_log2;
          float mo;
          if (!exchange(mx, mo)) {
            ok = false;
            break;
          }
          mx = fmaxf(mx, mo);
          // lazy rescale: keep the stale max unless the new one is 2^8 larger.
          // The decision is per row (lane) but the TMEM loads / stores below
          // are warp-collective (.sync.aligned), so the whole warp rescales
          // when any row needs it, each row by its own factor (1 where its
          // max did not grow).  The partner warp sees the same row maxima
          // and takes the same branch.
          if (__any_sync(0xffffffffu, mx > m_run + 8.0f)) {
            const float m_new = fmaxf(m_run, mx);
            const float corr = m_new == -INFINITY ? 1.f : fa_exp2(m_run - m_new);
            mx = m_new;
            if (j > 0) {
              // O holds PV of blocks < j: wait for PV(j-1), then scale our half
              if (!wait_pv(pv_done + j - 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t o_addr = t_lane + Cfg::O_COL + half * OH;
              if constexpr (OH >= 32) {
#pragma unroll 1
                for (int c = 0; c < OH / 32; ++c) {
                  uint32_t v[32];
                  tmem_ld_32x32b_x32(o_addr + c * 32, v);
                  tmem_wait_ld();
#pragma unroll
                  for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
                  tmem_st_32x32b_x32(o_addr + c * 32, v);
                }
              } else {
                uint32_t v[16];
                tmem_ld_32x32b_x16(o_addr, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * corr);
                tmem_st_32x32b_x16(o_addr, v);
              }
              tmem_wait_st();
            }
            l_part *= corr;
            m_run = mx;
          }
        }
        // pass 2: P = exp2(logit - m_run) into this warp's K-atom of P buffer
        // pb (the PV two blocks back has released it), row sum
        const int pb = static_cast<int>((pv_done + j) & 1);
        if (!mbar_wait_warp(&p_empty[pb], ((pe_bits >> pb) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        pe_bits ^= 1u << pb;
        uint8_t* prow = p_row + pb * 32768;
        if (warp_live) {
          float sum = 0.f;
          const float nm = -m_run;
          uint32_t v[2][32];
#pragma unroll
          for (int c = 0; c < 2; ++c)
            if (c < live_chunks) tmem_ld_32x32b_x32(s_addr + c * 32, v[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float p[32];
            if (c < live_chunks) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const int key = kh0 + c * 32 + i;
                const float x = __uint_as_float(v[c][i]);
                float e = kBias ? fa_exp2(fmaf(x, a.scale_log2, sBias[q - key + 127 + L]) + nm)
                                : fa_exp2(fmaf(x, a.scale_log2, nm));
                if (need_mask && (key >= L || (kCausal && key > q))) e = 0.f;
                p[i] = e;
                sum += e;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) p[i] = 0.f;  // keys past the sequence
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int c16 = c * 4 + u;  // 16-byte chunk within the 128-byte row
              *reinterpret_cast<uint4*>(prow + ((c16 ^ (r & 7)) << 4)) =
                  make_uint4(pack_bf16(p[8 * u], p[8 * u + 1]), pack_bf16(p[8 * u + 2], p[8 * u + 3]),
                             pack_bf16(p[8 * u + 4], p[8 * u + 5]),
                             pack_bf16(p[8 * u + 6], p[8 * u + 7]));
            }
          }
          l_part += sum;
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s_empty[sbuf]);
          mbar_arrive(&p_full[pb]);
        }
        sbuf ^= 1;
      }
      if (!ok) break;
      // final: O / l for rows inside the sequence, this warp's column half
      float l_other;
      if (!exchange(l_part, l_other)) {
        ok = false;
        break;
      }
      const float l_run = l_part + l_other;
      if (!wait_pv(pv_done + nkb - 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = a.out + static_cast<size_t>(base + q) * a.ldo + h * HD + half * OH;
      const uint32_t o_addr = t_lane + Cfg::O_COL + half * OH;
      if constexpr (OH >= 32) {
#pragma unroll 1
        for (int c = 0; c < OH / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(o_addr + c * 32, v);
          tmem_wait_ld();
          if (q < L) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int u = 0; u < 4; ++u)
              dst[u] = make_uint4(
                  pack_bf16(__uint_as_float(v[8 * u]) * inv, __uint_as_float(v[8 * u + 1]) * inv),
                  pack_bf16(__uint_as_float(v[8 * u + 2]) * inv, __uint_as_float(v[8 * u + 3]) * inv),
                  pack_bf16(__uint_as_float(v[8 * u + 4]) * inv, __uint_as_float(v[8 * u + 5]) * inv),
                  pack_bf16(__uint_as_float(v[8 * u + 6]) * inv, __uint_as_float(v[8 * u + 7]) * inv));
          }
        }
      } else {
        uint32_t v[16];
        tmem_ld_32x32b_x16(o_addr, v);
        tmem_wait_ld();
        if (q < L) {
          uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
          for (int u = 0; u < 2; ++u)
            dst[u] = make_uint4(
                pack_bf16(__uint_as_float(v[8 * u]) * inv, __uint_as_float(v[8 * u + 1]) * inv),
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
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace ec
