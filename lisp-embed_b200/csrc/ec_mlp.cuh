// ec_mlp.cuh -- fused feed-forward block for hidden sizes up to 384:
//
//   out = LayerNorm( W2 . gelu(W1 . x + b1) + b2 + resid )
//
// the FFN half of bert::encoder-layer (bert.lisp:259-271) and of
// bert::mpnet-layer (:435-452), on CTA pairs: the two CTAs of a cluster
// share a 256-row tile (CTA r owns rows 128 r ..) and every MMA is a
// tcgen05.mma.cta_group::2 of M = 256, so each CTA streams only half of each
// weight block.  Per tile:
//
//   X (the tile's input rows) stays in shared memory for all slices
//   Y = X . I (the bf16 residual, by an identity MMA; or 0 with an fp32
//   residual, added in the epilogue)
//   for each 64-wide slice f of the intermediate (F / 64 slices):
//     U_f = X . W1[f]^T           M 256, N 64  -> TMEM [H + 64 (f & 1), +64)
//     P_f = gelu(U_f + b1[f])     epilogue warps, bf16 -> shared memory ring of 4
//     Y  += P_f . W2[:, f]^T      M 256, N = H in parts of <= 256 -> TMEM [0, H)
//   then bias (+ fp32 residual) + LayerNorm over each CTA's full rows in TMEM,
//   and TMA bulk stores of the bf16 row (and the fp32 row when asked).
// MMA1 runs two slices ahead of MMA2 (U is double-buffered), so the tensor
// core has MMA1(f+1), MMA1(f+2) to do while GELU(f) is computed.
//
// The intermediate activation never leaves the SM.  The residual is either
// the fp32 stream or, when none is given, the bf16 input X itself (the
// previous LayerNorm's bf16 output, the residual the unfused path uses); it
// is read from global memory (L2) because X is released to the next tile's
// loads once the last MMA1 of a tile is issued.
//
// Warp roles per CTA: warp 0 TMA producer (X once per tile, then the CTA's
// halves of the W1 / W2 blocks through a ring), warp 1 TMEM allocator and,
// in the even CTA, the MMA issuer, warps 2..9 epilogue (two warps per TMEM
// lane quadrant, one per column half).  The odd CTA's loads and epilogue arrivals land on the even
// CTA's barriers; MMA completions are multicast to both.  All waits are
// bounded.
#pragma once

#include "ec_gemm.cuh"

namespace ec {

struct MlpArgs {
  int M, F;
  const float* b1;                 // [F]
  const float* b2;                 // [H]
  const float* resid;              // [M, H] fp32, or nullptr: the bf16 input rows
  const __nv_bfloat16* resid_b;    // [M, H] the bf16 input (when resid is nullptr)
  const float* ln_g;               // [H]
  const float* ln_b;               // [H]
  int out32;                       // 1: also store the fp32 row
  int num_tiles;                   // 256-row tiles
  unsigned* status;
};

constexpr int kMlpThreads = 320;
constexpr uint32_t kMlpAtom = 16384;  // 128 rows x 64 bf16 (128-byte rows, SW128)

template <int H>
struct MlpCfg {
  static_assert(H == 128 || H == 256 || H == 384, "hidden");
  static constexpr int FS = 64;                     // intermediate columns per slice
  static constexpr int KA = H / 64;                 // 64-wide k-blocks of X / W1
  static constexpr int NPART = H == 384 ? 2 : 1;    // MMA2 column parts
  static constexpr int NPW = H / NPART;             // columns per MMA2 part (<= 256)
  static constexpr uint32_t W1_BOX = 32 * 128;      // this CTA's 32 rows x 64 k of W1
  static constexpr uint32_t STAGE = (NPW / 2) * 128;  // this CTA's rows x 64 k of W2
  static constexpr int W1_PER = static_cast<int>(STAGE / W1_BOX);  // W1 boxes per stage
  static constexpr int W1_ST = KA / W1_PER;         // W1 stages per slice
  static_assert(W1_ST * W1_PER == KA, "W1 stages");
  static constexpr int PB = 4;                      // P ring (one 128 x 64 atom each)
  static constexpr uint32_t X_BYTES = KA * kMlpAtom;
  static constexpr uint32_t P_BYTES = PB * kMlpAtom;
  // this CTA's 32 rows of a 64 x 64 identity (the B operand of Y = X . I,
  // which puts the bf16 residual into the accumulator)
  static constexpr uint32_t I_BYTES = 32 * 128;
  static constexpr int MAX_STAGES =
      static_cast<int>((232448 - 1024 - 2048 - X_BYTES - P_BYTES - I_BYTES) / STAGE);
  static constexpr int STAGES = MAX_STAGES > 8 ? 8 : MAX_STAGES;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t U_COL = H;              // U buffers at [H, H + 64), [H + 64, H + 128)
  static constexpr size_t SMEM_BYTES = 1024 + X_BYTES + P_BYTES + I_BYTES + STAGES * STAGE + 2048;
  static_assert(STAGES >= 3, "stages");
  static_assert(H + 2 * FS <= 512, "TMEM");
};

template <int H>
__global__ void __launch_bounds__(kMlpThreads, 1)
    mlp_fused_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmO32,
                     const __grid_constant__ CUtensorMap tmOb, const MlpArgs args) {
  using Cfg = MlpCfg<H>;
  constexpr int S = Cfg::STAGES;
  constexpr int KA = Cfg::KA;
  constexpr int NPART = Cfg::NPART;
  constexpr int NPW = Cfg::NPW;
  constexpr int W1_PER = Cfg::W1_PER;
  constexpr int W1_ST = Cfg::W1_ST;
  constexpr int PB = Cfg::PB;
  constexpr uint32_t IDESC1 = make_idesc(1, 256, Cfg::FS);
  constexpr uint32_t IDESC2 = make_idesc(1, 256, NPW);
  constexpr uint32_t IDESC_I = make_idesc(1, 256, 64);
  const bool resid_mma = args.resid == nullptr;  // residual = the input rows X

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smX = smem;                          // KA atoms of 128 x 64
  uint8_t* smP = smX + Cfg::X_BYTES;            // PB atoms
  uint8_t* smI = smP + Cfg::P_BYTES;            // identity rows (4 KB)
  uint8_t* smW = smI + Cfg::I_BYTES;            // S stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smW + S * Cfg::STAGE);
  uint64_t* w_full = bars;           // [S] (even CTA: both CTAs' halves)
  uint64_t* w_empty = w_full + S;    // [S] (multicast commit)
  uint64_t* x_full = w_empty + S;    // (even CTA)
  uint64_t* x_empty = x_full + 1;    // (multicast commit)
  uint64_t* u_full = x_empty + 1;    // [2] (multicast commit)
  uint64_t* u_empty = u_full + 2;    // [2] (even CTA: 16 warp arrivals)
  uint64_t* p_full = u_empty + 2;    // [PB] (even CTA: 16 warp arrivals)
  uint64_t* p_empty = p_full + PB;   // [PB] (multicast commit)
  uint64_t* y_full = p_empty + PB;   // (multicast commit)
  uint64_t* y_empty = y_full + 1;    // (even CTA: 16 warp arrivals)
  uint64_t* xbar = y_empty + 1;      // [4 quads] partner rendezvous, 64 threads
  float* xsum = reinterpret_cast<float*>(xbar + 4);  // [8 warps][32] partial row sums
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xsum + 8 * 32);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cl = static_cast<int>(blockIdx.x) / 2;
  const int ncl = static_cast<int>(gridDim.x) / 2;
  const int NF = args.F / Cfg::FS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&u_full[b], 1);
      mbar_init(&u_empty[b], 16);
    }
    for (int b = 0; b < PB; ++b) {
      mbar_init(&p_full[b], 16);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(y_full, 1);
    mbar_init(y_empty, 16);
    for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW1);
    tma_prefetch_desc(&tmW2);
    tma_prefetch_desc(&tmO32);
    tma_prefetch_desc(&tmOb);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  {
    // identity rows: CTA r holds B rows n = 32 r + i (i < 32), whose single
    // 1.0 sits at k = n (K-major, 128-byte rows, SW128)
    uint4* iz = reinterpret_cast<uint4*>(smI);
    for (int i = threadIdx.x; i < static_cast<int>(Cfg::I_BYTES / 16); i += kMlpThreads)
      iz[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    if (threadIdx.x < 32) {
      const int i = threadIdx.x, k = static_cast<int>(rank) * 32 + i;
      *reinterpret_cast<__nv_bfloat16*>(smI + i * 128 + (((k >> 3) ^ (i & 7)) << 4) + (k & 7) * 2) =
          __float2bfloat16(1.0f);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  cluster_sync_all();  // the partner's barriers exist
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto fail = [&](unsigned code) {
    report(args.status, code);
    *abort_flag = 1;
  };
  // arrive on barrier `b` of the even CTA (remotely from the odd one)
  auto arrive_even = [&](uint64_t* b) {
    if (rank == 0) mbar_arrive(b);
    else mbar_arrive_remote(cluster_map(smem_u32(b), 0));
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0, x_phase = 0;
      bool ok = true;
      // one stage: both CTAs' halves land on the even CTA's barrier
      auto open_stage = [&]() -> bool {
        if (!mbar_wait(&w_empty[stage], phase ^ 1, abort_flag)) return false;
        if (rank == 0) mbar_arrive_expect_tx(&w_full[stage], 2 * Cfg::STAGE);
        return true;
      };
      auto next_stage = [&]() {
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      };
      // W1 of slice f: W1_ST stages of W1_PER k-blocks (this CTA's 32 rows)
      auto load_w1 = [&](int f) -> bool {
        for (int si = 0; si < W1_ST; ++si) {
          if (!open_stage()) return false;
          const uint32_t fb = cluster_map(smem_u32(&w_full[stage]), 0);
          for (int bx = 0; bx < W1_PER; ++bx)
            tma_load_2d_pair(smW + stage * Cfg::STAGE + bx * Cfg::W1_BOX, &tmW1, fb,
                             (si * W1_PER + bx) * 64, f * Cfg::FS + static_cast<int>(rank) * 32);
          next_stage();
        }
        return true;
      };
      // W2 of slice f: one stage per column part (this CTA's NPW / 2 rows)
      auto load_w2 = [&](int f) -> bool {
        for (int j = 0; j < NPART; ++j) {
          if (!open_stage()) return false;
          tma_load_2d_pair(smW + stage * Cfg::STAGE, &tmW2, cluster_map(smem_u32(&w_full[stage]), 0),
                           f * Cfg::FS, j * NPW + static_cast<int>(rank) * (NPW / 2));
          next_stage();
        }
        return true;
      };
      for (int tile = cl; ok && tile < args.num_tiles; tile += ncl) {
        if (!mbar_wait(x_empty, x_phase ^ 1, abort_flag)) {
          fail(kDevTimeoutProducer);
          break;
        }
        x_phase ^= 1;
        if (rank == 0) mbar_arrive_expect_tx(x_full, 2 * Cfg::X_BYTES);
        const uint32_t xb = cluster_map(smem_u32(x_full), 0);
        for (int kb = 0; kb < KA; ++kb)
          tma_load_2d_pair(smX + kb * kMlpAtom, &tmX, xb, kb * 64, tile * 256 + static_cast<int>(rank) * 128);
        // the MMA order: W1(0), W1(1), then for each f: W1(f + 2), W2(f)
        ok = load_w1(0) && (NF < 2 || load_w1(1));
        for (int f = 0; ok && f < NF; ++f) {
          if (f + 2 < NF) ok = load_w1(f + 2);
          if (ok) ok = load_w2(f);
        }
        if (!ok) fail(kDevTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer (even CTA)
    if (rank == 0 && elect_one()) {
      int stage = 0;
      uint32_t phase = 0, x_phase = 0, y_phase = 0;
      uint32_t ue_bits = 0, pf_bits = 0;  // phase parity per buffer
      bool ok = true;
      const uint32_t x_base = smem_u32(smX), p_base = smem_u32(smP);
      auto next_w = [&]() -> int {
        if (!mbar_wait(&w_full[stage], phase, abort_flag)) return -1;
        tc_fence_after();
        return stage;
      };
      auto release_w = [&]() {
        umma_commit_pair(&w_empty[stage], 0x3);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      };
      // X is handed back once the last MMA1 and the residual MMA have read it
      bool x_mma1_done = false, x_id_done = false;
      auto release_x = [&]() {
        if (x_mma1_done && x_id_done) umma_commit_pair(x_empty, 0x3);
      };
      // MMA1(f): U[f & 1] = X . W1[f]^T, once GELU(f - 2) has read that buffer
      auto mma1 = [&](int f) -> bool {
        const int b = f & 1;
        // GELU's arrivals are cluster-scope releases
        if (!mbar_wait_cluster(&u_empty[b], ((ue_bits >> b) & 1u) ^ 1u, abort_flag)) return false;
        ue_bits ^= 1u << b;
        tc_fence_after();
        for (int si = 0; si < W1_ST; ++si) {
          const int st = next_w();
          if (st < 0) return false;
          const uint32_t wa = smem_u32(smW + st * Cfg::STAGE);
          for (int bx = 0; bx < W1_PER; ++bx) {
            const int kb = si * W1_PER + bx;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16_pair(tmem_base + Cfg::U_COL + b * Cfg::FS,
                            desc_sw128_kmajor(x_base + kb * kMlpAtom + k * 32),
                            desc_sw128_kmajor(wa + bx * Cfg::W1_BOX + k * 32), IDESC1,
                            (kb > 0 || k > 0) ? 1u : 0u);
          }
          release_w();
        }
        umma_commit_pair(&u_full[b], 0x3);
        if (f == NF - 1) {
          x_mma1_done = true;
          release_x();
        }
        return true;
      };
      // MMA2(f): Y += P[f % PB] . W2[:, f]^T
      auto mma2 = [&](int f) -> bool {
        if (f == 0) {
          if (!mbar_wait_cluster(y_empty, y_phase ^ 1, abort_flag)) return false;
          y_phase ^= 1;
          if (resid_mma) {
            // Y = X . I block by block: the bf16 residual, exact in fp32
            tc_fence_after();
            const uint32_t ia = smem_u32(smI);
            for (int j = 0; j < KA; ++j)
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f16_pair(tmem_base + j * 64, desc_sw128_kmajor(x_base + j * kMlpAtom + k * 32),
                              desc_sw128_kmajor(ia + k * 32), IDESC_I, k > 0 ? 1u : 0u);
          }
          x_id_done = true;
          release_x();
        }
        const int q = f % PB;
        if (!mbar_wait_cluster(&p_full[q], (pf_bits >> q) & 1u, abort_flag)) return false;
        pf_bits ^= 1u << q;
        tc_fence_after();
        const uint32_t pa = p_base + q * kMlpAtom;
        for (int j = 0; j < NPART; ++j) {
          const int st = next_w();
          if (st < 0) return false;
          const uint32_t wa = smem_u32(smW + st * Cfg::STAGE);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_pair(tmem_base + j * NPW, desc_sw128_kmajor(pa + k * 32), desc_sw128_kmajor(wa + k * 32),
                          IDESC2, (resid_mma || f > 0 || k > 0) ? 1u : 0u);
          release_w();
        }
        umma_commit_pair(&p_empty[q], 0x3);
        return true;
      };
      for (int tile = cl; ok && tile < args.num_tiles; tile += ncl) {
        if (!mbar_wait(x_full, x_phase, abort_flag)) {
          fail(kDevTimeoutMma);
          break;
        }
        x_phase ^= 1;
        tc_fence_after();
        x_mma1_done = false;
        x_id_done = false;
        ok = mma1(0) && (NF < 2 || mma1(1));
        for (int f = 0; ok && f < NF; ++f) {
          if (f + 2 < NF && !mma1(f + 2)) ok = false;
          if (ok && !mma2(f)) ok = false;
        }
        if (!ok) {
          fail(kDevTimeoutMma);
          break;
        }
        umma_commit_pair(y_full, 0x3);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int half = ew >> 2;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    // this warp's rows of P atoms 2 half and 2 half + 1 (4 KB each): TMA-store
    // staging during the LayerNorm phase (the ring is idle once y_full has
    // arrived)
    uint8_t* p_mine0 = smP + (2 * half) * kMlpAtom + quad * 4096;
    uint8_t* p_mine1 = smP + (2 * half + 1) * kMlpAtom + quad * 4096;
    uint32_t y_phase = 0, x_phase = 0;
    uint32_t uf_bits = 0, pe_bits = 0;  // phase parity per buffer
    bool ok = true;
    for (int tile = cl; ok && tile < args.num_tiles; tile += ncl) {
      const int row0 = tile * 256 + static_cast<int>(rank) * 128 + quad * 32;
      for (int f = 0; f < NF; ++f) {
        const int b = f & 1, q = f % PB;
        if (!mbar_wait_warp(&u_full[b], (uf_bits >> b) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        uf_bits ^= 1u << b;
        tc_fence_after();
        // this warp's 32 rows x 32 columns (column half) of the slice
        uint32_t ua[32];
        tmem_ld_32x32b_x32(t_lane + Cfg::U_COL + b * Cfg::FS + half * 32, ua);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_even(&u_empty[b]);
        if (!mbar_wait_warp(&p_empty[q], ((pe_bits >> q) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        pe_bits ^= 1u << q;
        const float* b1 = args.b1 + f * Cfg::FS + half * 32;
        uint8_t* prow = smP + q * kMlpAtom + row_in_tile * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 8 columns per 16-byte chunk
          const float4 bb0 = __ldg(reinterpret_cast<const float4*>(b1 + c * 8));
          const float4 bb1 = __ldg(reinterpret_cast<const float4*>(b1 + c * 8 + 4));
          const float2 bv[4] = {make_float2(bb0.x, bb0.y), make_float2(bb0.z, bb0.w),
                                make_float2(bb1.x, bb1.y), make_float2(bb1.z, bb1.w)};
          float2 x[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            x[e] = gelu_as2(__fadd2_rn(make_float2(__uint_as_float(ua[c * 8 + 2 * e]),
                                                   __uint_as_float(ua[c * 8 + 2 * e + 1])),
                                       bv[e]));
          // K-major SW128 atom: row r, 16-byte chunk cc at (cc ^ (r & 7))
          const int cc = half * 4 + c;
          *reinterpret_cast<uint4*>(prow + ((cc ^ (row_in_tile & 7)) << 4)) =
              make_uint4(pack_bf16(x[0].x, x[0].y), pack_bf16(x[1].x, x[1].y), pack_bf16(x[2].x, x[2].y),
                         pack_bf16(x[3].x, x[3].y));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) arrive_even(&p_full[q]);
      }
      if (!ok) break;
      // ------------------------------------------- bias + residual + LayerNorm
      if (!mbar_wait_warp(y_full, y_phase, abort_flag)) {
        ok = false;
        break;
      }
      y_phase ^= 1;
      tc_fence_after();
      constexpr int HC = H / 2 / 32;  // 32-column chunks of this warp's half
      const int c0 = half * (H / 2);
      const int grow = row0 + lane;   // this thread's row
      const bool live = grow < args.M;
      // pass A: x = acc + b2 (+ the fp32 residual; the bf16 residual is in
      // the accumulator already), back to TMEM; this thread's mean and sum of
      // squared deviations over its H / 2 columns, chunk by chunk merged with
      // the pairwise formula of Chan, Golub and LeVeque
      float wmean = 0.f, wm2 = 0.f;
      for (int c = 0; c < HC; ++c) {
        const int col0 = c0 + c * 32;
        uint32_t yv[32];
        tmem_ld_32x32b_x32(t_lane + col0, yv);
        float rs[32];
        if (!resid_mma) {
          const float4* rp = reinterpret_cast<const float4*>(args.resid + static_cast<size_t>(grow) * H + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 q = live ? rp[j] : make_float4(0.f, 0.f, 0.f, 0.f);
            rs[4 * j] = q.x;
            rs[4 * j + 1] = q.y;
            rs[4 * j + 2] = q.z;
            rs[4 * j + 3] = q.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) rs[j] = 0.f;
        }
        tmem_wait_ld();
        float cs = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 b = __ldg(reinterpret_cast<const float4*>(args.b2 + col0 + 4 * j));
          // (dense + bias) + residual, bert.lisp:265-270
          const float v0 = (__uint_as_float(yv[4 * j]) + b.x) + rs[4 * j];
          const float v1 = (__uint_as_float(yv[4 * j + 1]) + b.y) + rs[4 * j + 1];
          const float v2 = (__uint_as_float(yv[4 * j + 2]) + b.z) + rs[4 * j + 2];
          const float v3 = (__uint_as_float(yv[4 * j + 3]) + b.w) + rs[4 * j + 3];
          yv[4 * j] = __float_as_uint(v0);
          yv[4 * j + 1] = __float_as_uint(v1);
          yv[4 * j + 2] = __float_as_uint(v2);
          yv[4 * j + 3] = __float_as_uint(v3);
          cs += (v0 + v1) + (v2 + v3);
        }
        tmem_st_32x32b_x32(t_lane + col0, yv);
        const float cm = cs * (1.f / 32.f);
        float cq = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float d = __uint_as_float(yv[j]) - cm;
          cq += d * d;
        }
        // merge (32 c, wmean, wm2) with (32, cm, cq)
        const float n0 = 32.f * c, n1 = n0 + 32.f;
        const float dl = cm - wmean;
        wmean += dl * (32.f / n1);
        wm2 += cq + dl * dl * (n0 * 32.f / n1);
      }
      tmem_wait_st();
      // merge with the partner warp (the other half of the same rows)
      xsum[ew * 32 + lane] = wmean;
      if (!mbar_sync(&xbar[quad], x_phase, abort_flag)) {
        ok = false;
        break;
      }
      const float pmean = xsum[(ew ^ 4) * 32 + lane];
      if (!mbar_sync(&xbar[quad], x_phase, abort_flag)) {  // both have read the means
        ok = false;
        break;
      }
      xsum[ew * 32 + lane] = wm2;
      if (!mbar_sync(&xbar[quad], x_phase, abort_flag)) {
        ok = false;
        break;
      }
      const float pm2 = xsum[(ew ^ 4) * 32 + lane];
      const float mean = 0.5f * (wmean + pmean);
      const float dd = wmean - pmean;
      const float var = (wm2 + pm2 + dd * dd * (0.25f * static_cast<float>(H))) / static_cast<float>(H);
      const float stdv = sqrtf(var) + 1e-12f;  // bert.lisp:169
      const float inv = 1.0f / stdv;            // as the unfused LayerNorm epilogue
      // rows of this warp that exist (a tile's last rows may lie past M)
      const bool any_live = row0 < args.M;
      const bool two_bufs = !args.out32;  // bf16 rows only: alternate staging
      int sb = 0;
      for (int c = 0; c < HC; ++c) {
        const int col0 = c0 + c * 32;
        uint32_t yv[32];
        tmem_ld_32x32b_x32(t_lane + col0, yv);
        tmem_wait_ld();
        float o[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 g = __ldg(reinterpret_cast<const float4*>(args.ln_g + col0 + 4 * j));
          const float4 b = __ldg(reinterpret_cast<const float4*>(args.ln_b + col0 + 4 * j));
          o[4 * j] = ((__uint_as_float(yv[4 * j]) - mean) * inv) * g.x + b.x;
          o[4 * j + 1] = ((__uint_as_float(yv[4 * j + 1]) - mean) * inv) * g.y + b.y;
          o[4 * j + 2] = ((__uint_as_float(yv[4 * j + 2]) - mean) * inv) * g.z + b.z;
          o[4 * j + 3] = ((__uint_as_float(yv[4 * j + 3]) - mean) * inv) * g.w + b.w;
        }
        uint8_t* st32 = p_mine0;              // fp32 staging (4 KB)
        uint8_t* stb = sb ? p_mine0 : p_mine1;  // bf16 staging (2 KB)
        if (lane == 0) {
          if (two_bufs)
            tma_store_wait_read<1>();
          else
            tma_store_wait_read<0>();
        }
        __syncwarp();
        if (args.out32) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(st32 + stage_off<true>(lane, j)) =
                make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(stb + stage_off<false>(lane, j)) =
              make_uint4(pack_bf16(o[8 * j], o[8 * j + 1]), pack_bf16(o[8 * j + 2], o[8 * j + 3]),
                         pack_bf16(o[8 * j + 4], o[8 * j + 5]), pack_bf16(o[8 * j + 6], o[8 * j + 7]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && any_live) {
          if (args.out32) tma_store_2d(&tmO32, st32, col0, row0);
          tma_store_2d(&tmOb, stb, col0, row0);
        }
        if (lane == 0) tma_store_commit();
        if (two_bufs) sb ^= 1;
      }
      // staging lives in this warp's P regions: drain before GELU reuses them
      if (lane == 0) tma_store_wait_read<0>();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_even(y_empty);
    }
    if (!ok) fail(kDevTimeoutEpilogue);
    if (lane == 0) tma_store_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync_all();  // neither CTA leaves while the pair MMAs run
  if (*abort_flag) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace ec
