// ec_mlp.cuh -- fused feed-forward block for hidden sizes up to 384:
//
//   out = LayerNorm( W2 . gelu(W1 . x + b1) + b2 + resid )
//
// the FFN half of bert::encoder-layer (bert.lisp:259-271) and of
// bert::mpnet-layer (:435-452) for one 128-token tile per CTA step:
//
//   for each 128-wide slice f of the intermediate (F / 128 slices):
//     U   = A . W1[f]^T             tcgen05.mma -> TMEM columns [H, H+128)
//     P_f = gelu(U + b1[f])         epilogue warps, bf16 -> shared memory
//     Y  += P_f . W2[:, f]^T        tcgen05.mma -> TMEM columns [0, H)
//   then bias + residual + LayerNorm over the full row held in TMEM, and TMA
//   bulk stores of the fp32 residual stream and its bf16 copy.
//
// The intermediate activation never leaves the SM.  Warp roles: warp 0 TMA
// producer (A tile once per row tile, then W1 / W2 slices through a 16 KB
// ring), warp 1 UMMA issuer (MMA1 of slice f+1 is issued before MMA2 of slice
// f, so GELU(f) overlaps tensor work), warps 2..9 epilogue (two warps per
// TMEM lane quadrant, one per column half).  All waits are bounded.
#pragma once

#include "ec_gemm.cuh"

namespace ec {

struct MlpArgs {
  int M, F;
  const float* b1;     // [F]
  const float* b2;     // [H]
  const float* resid;  // [M, H] fp32 (may alias the fp32 output)
  const float* ln_g;   // [H]
  const float* ln_b;   // [H]
  int num_tiles;
  unsigned* status;
};

constexpr int kMlpThreads = 320;
constexpr int kMlpStage = 16384;  // one 128 x 64 bf16 operand block

template <int H>
struct MlpCfg {
  static_assert(H % 128 == 0 && H <= 384, "hidden");
  static constexpr int KA = H / 64;                 // k-blocks of A / W1
  static constexpr uint32_t A_BYTES = KA * kMlpStage;
  static constexpr int PBUF = 2;                    // P buffers (GELU(f+1) overlaps MMA2(f))
  static constexpr uint32_t P_BYTES = PBUF * 2 * kMlpStage;  // buffers x 2 k-atoms
  // 1024 B alignment slack in front, 2048 B of barriers / row sums behind
  static constexpr int STAGES = (232448 - 1024 - 2048 - A_BYTES - P_BYTES) / kMlpStage;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t U_COL = H;              // U at columns [H, H + 128)
  static constexpr size_t SMEM_BYTES = 1024 + A_BYTES + P_BYTES + STAGES * kMlpStage + 2048;
  static_assert(STAGES >= 2, "stages");
  static_assert(H + 128 <= 512, "TMEM");
};

template <int H>
__global__ void __launch_bounds__(kMlpThreads, 1)
    mlp_fused_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmO32,
                     const __grid_constant__ CUtensorMap tmOb, const MlpArgs args) {
  using Cfg = MlpCfg<H>;
  constexpr int S = Cfg::STAGES;
  constexpr int KA = Cfg::KA;
  constexpr int NSUB = H / 128;  // 128-wide column blocks of Y
  constexpr uint32_t IDESC = make_idesc(1, 128, 128);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smA = smem;                         // KA atoms of 128 x 64
  uint8_t* smP = smA + Cfg::A_BYTES;           // 2 buffers x 2 atoms
  uint8_t* smB = smP + Cfg::P_BYTES;           // S stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smB + S * kMlpStage);
  uint64_t* b_full = bars;
  uint64_t* b_empty = b_full + S;
  uint64_t* a_full = b_empty + S;
  uint64_t* a_empty = a_full + 1;
  uint64_t* u_full = a_empty + 1;
  uint64_t* u_empty = u_full + 1;
  uint64_t* p_full = u_empty + 1;   // [2]
  uint64_t* p_empty = p_full + 2;   // [2]
  uint64_t* y_full = p_empty + 2;
  uint64_t* y_empty = y_full + 1;
  uint64_t* xbar = y_empty + 1;  // [4 quads] partner rendezvous, 64 threads
  float* xsum = reinterpret_cast<float*>(xbar + 4);  // [8 warps][32] partial row sums
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xsum + 8 * 32);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NF = args.F / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    mbar_init(u_full, 1);
    mbar_init(u_empty, 8);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&p_full[b], 8);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(y_full, 1);
    mbar_init(y_empty, 8);
    for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW1);
    tma_prefetch_desc(&tmW2);
    tma_prefetch_desc(&tmO32);
    tma_prefetch_desc(&tmOb);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto fail = [&](unsigned code) {
    report(args.status, code);
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      const uint64_t pol_w = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, a_phase = 0;
      bool ok = true;
      auto load_b = [&](const CUtensorMap* map, int x, int y) -> bool {
        if (!mbar_wait(&b_empty[stage], phase ^ 1, abort_flag)) return false;
        mbar_arrive_expect_tx(&b_full[stage], kMlpStage);
        tma_load_2d_hint(smB + stage * kMlpStage, map, &b_full[stage], x, y, pol_w);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
        return true;
      };
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
        if (!mbar_wait(a_empty, a_phase ^ 1, abort_flag)) {
          fail(kDevTimeoutProducer);
          break;
        }
        a_phase ^= 1;
        mbar_arrive_expect_tx(a_full, Cfg::A_BYTES);
        for (int kb = 0; kb < KA; ++kb)
          tma_load_2d(smA + kb * kMlpStage, &tmA, a_full, kb * 64, tile * 128);
        // B order: W1[0], then for f >= 1: W1[f], W2[f-1]; finally W2[NF-1]
        for (int f = 0; ok && f <= NF; ++f) {
          if (f < NF)
            for (int kb = 0; ok && kb < KA; ++kb) ok = load_b(&tmW1, kb * 64, f * 128);
          if (f >= 1)
            for (int k2 = 0; ok && k2 < 2; ++k2)
              for (int ns = 0; ok && ns < NSUB; ++ns)
                ok = load_b(&tmW2, (f - 1) * 128 + k2 * 64, ns * 128);
        }
        if (!ok) fail(kDevTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0, a_phase = 0, u_phase = 0, y_phase = 0;
      uint32_t p_phase[2] = {0, 0};
      bool ok = true;
      const uint32_t a_base = smem_u32(smA), p_base = smem_u32(smP);
      auto next_b = [&]() -> int {
        if (!mbar_wait(&b_full[stage], phase, abort_flag)) return -1;
        tc_fence_after();
        return stage;
      };
      auto release_b = [&]() {
        umma_commit(&b_empty[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      };
      auto mma2 = [&](int g) -> bool {
        if (g == 0) {
          if (!mbar_wait(y_empty, y_phase ^ 1, abort_flag)) return false;
          y_phase ^= 1;
          tc_fence_after();
        }
        const int pb = g % Cfg::PBUF;
        if (!mbar_wait(&p_full[pb], p_phase[pb], abort_flag)) return false;
        p_phase[pb] ^= 1;
        tc_fence_after();
        for (int k2 = 0; k2 < 2; ++k2)
          for (int ns = 0; ns < NSUB; ++ns) {
            const int st = next_b();
            if (st < 0) return false;
            const uint32_t pa = p_base + pb * 2 * kMlpStage + k2 * kMlpStage;
            const uint32_t ba = smem_u32(smB + st * kMlpStage);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(tmem_base + ns * 128, desc_sw128_kmajor(pa + k * 32),
                       desc_sw128_kmajor(ba + k * 32), IDESC,
                       (g > 0 || k2 > 0 || k > 0) ? 1u : 0u);
            release_b();
          }
        umma_commit(&p_empty[pb]);
        return true;
      };
      for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
        if (!mbar_wait(a_full, a_phase, abort_flag)) {
          fail(kDevTimeoutMma);
          break;
        }
        a_phase ^= 1;
        tc_fence_after();
        for (int f = 0; ok && f < NF; ++f) {
          // MMA1(f): U = A . W1[f]^T
          if (!mbar_wait(u_empty, u_phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kb = 0; kb < KA; ++kb) {
            const int st = next_b();
            if (st < 0) {
              ok = false;
              break;
            }
            const uint32_t ba = smem_u32(smB + st * kMlpStage);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(tmem_base + Cfg::U_COL, desc_sw128_kmajor(a_base + kb * kMlpStage + k * 32),
                       desc_sw128_kmajor(ba + k * 32), IDESC, (kb > 0 || k > 0) ? 1u : 0u);
            release_b();
          }
          if (!ok) break;
          umma_commit(u_full);
          u_phase ^= 1;
          if (f == NF - 1) umma_commit(a_empty);
          // MMA2(f-1): Y += P[f-1] . W2[:, f-1]^T
          if (f >= 1 && !mma2(f - 1)) ok = false;
        }
        if (ok && !mma2(NF - 1)) ok = false;
        if (!ok) {
          fail(kDevTimeoutMma);
          break;
        }
        umma_commit(y_full);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int half = ew >> 2;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    // this warp's private 4 KB regions of the two P buffers: its rows of its
    // column half; reused as TMA-store staging during the LayerNorm phase
    // this warp's private 4 KB regions of the two P buffers: its rows of its
    // column half; reused as TMA-store staging during the LayerNorm phase
    // (both buffers are idle once y_full has arrived)
    uint8_t* p_mine0 = smP + half * kMlpStage + quad * 4096;
    uint8_t* p_mine1 = p_mine0 + 2 * kMlpStage;
    uint32_t u_phase = 0, y_phase = 0, x_phase = 0;
    uint32_t pe_phase[2] = {0, 0};
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < args.num_tiles; tile += gridDim.x) {
      const int row0 = tile * 128 + quad * 32;
      for (int f = 0; f < NF; ++f) {
        if (!mbar_wait_warp(u_full, u_phase, abort_flag)) {
          ok = false;
          break;
        }
        u_phase ^= 1;
        tc_fence_after();
        uint32_t ua[32], ub[32];
        tmem_ld_32x32b_x32(t_lane + Cfg::U_COL + half * 64, ua);
        tmem_ld_32x32b_x32(t_lane + Cfg::U_COL + half * 64 + 32, ub);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(u_empty);
        const int pb = f % Cfg::PBUF;
        if (!mbar_wait_warp(&p_empty[pb], pe_phase[pb] ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        pe_phase[pb] ^= 1;
        const float* b1 = args.b1 + f * 128 + half * 64;
        uint8_t* pdst = pb ? p_mine1 : p_mine0;
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 8 columns per 16-byte chunk
          float x[8];
          const float4 bb0 = __ldg(reinterpret_cast<const float4*>(b1 + c * 8));
          const float4 bb1 = __ldg(reinterpret_cast<const float4*>(b1 + c * 8 + 4));
          const float bv[8] = {bb0.x, bb0.y, bb0.z, bb0.w, bb1.x, bb1.y, bb1.z, bb1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int j = c * 8 + e;
            const float u = __uint_as_float(j < 32 ? ua[j] : ub[j - 32]);
            x[e] = gelu_as(u + bv[e]);
          }
          // K-major SW128 atom: row r, 16-byte chunk c at (c ^ (r & 7))
          *reinterpret_cast<uint4*>(pdst + lane * 128 + ((c ^ (row_in_tile & 7)) << 4)) =
              make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]),
                         pack_bf16(x[6], x[7]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[pb]);
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
      uint8_t* st32 = p_mine0;        // fp32 staging (4 KB)
      uint8_t* stb = p_mine1;         // bf16 staging (2 KB)
      float part = 0.f;
      for (int c = 0; c < HC; ++c) {
        const int col0 = c0 + c * 32;
        float4 res[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = row0 + 4 * k + (lane >> 3);
          res[k] = r < args.M ? *reinterpret_cast<const float4*>(
                                    args.resid + static_cast<size_t>(r) * H + col0 + (lane & 7) * 4)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        uint32_t yv[32];
        tmem_ld_32x32b_x32(t_lane + col0, yv);
        if (lane == 0) tma_store_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(st32 + stage_off<true>(4 * k + (lane >> 3), lane & 7)) = res[k];
        __syncwarp();
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 q = *reinterpret_cast<const float4*>(st32 + stage_off<true>(lane, j));
          const float4 b = __ldg(reinterpret_cast<const float4*>(args.b2 + col0 + 4 * j));
          // (dense + bias) + residual, bert.lisp:265-270
          float v0 = (__uint_as_float(yv[4 * j]) + b.x) + q.x;
          float v1 = (__uint_as_float(yv[4 * j + 1]) + b.y) + q.y;
          float v2 = (__uint_as_float(yv[4 * j + 2]) + b.z) + q.z;
          float v3 = (__uint_as_float(yv[4 * j + 3]) + b.w) + q.w;
          yv[4 * j] = __float_as_uint(v0);
          yv[4 * j + 1] = __float_as_uint(v1);
          yv[4 * j + 2] = __float_as_uint(v2);
          yv[4 * j + 3] = __float_as_uint(v3);
          part += (v0 + v1) + (v2 + v3);
        }
        __syncwarp();
        tmem_st_32x32b_x32(t_lane + col0, yv);
      }
      tmem_wait_st();
      // mean over the full row: partner warp (other half) holds the rest
      xsum[ew * 32 + lane] = part;
      if (!mbar_sync(&xbar[ew & 3], x_phase, abort_flag)) {
        ok = false;
        break;
      }
      const float mean = (part + xsum[(ew ^ 4) * 32 + lane]) / static_cast<float>(H);
      float q2 = 0.f;
      for (int c = 0; c < HC; ++c) {
        uint32_t yv[32];
        tmem_ld_32x32b_x32(t_lane + c0 + c * 32, yv);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float d = __uint_as_float(yv[j]) - mean;
          q2 += d * d;
        }
      }
      // both partners have read the mean slots before they are rewritten
      if (!mbar_sync(&xbar[ew & 3], x_phase, abort_flag)) {
        ok = false;
        break;
      }
      xsum[ew * 32 + lane] = q2;
      if (!mbar_sync(&xbar[ew & 3], x_phase, abort_flag)) {
        ok = false;
        break;
      }
      const float var = (q2 + xsum[(ew ^ 4) * 32 + lane]) / static_cast<float>(H);
      const float stdv = sqrtf(var) + 1e-12f;  // bert.lisp:169
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
          o[4 * j] = ((__uint_as_float(yv[4 * j]) - mean) / stdv) * g.x + b.x;
          o[4 * j + 1] = ((__uint_as_float(yv[4 * j + 1]) - mean) / stdv) * g.y + b.y;
          o[4 * j + 2] = ((__uint_as_float(yv[4 * j + 2]) - mean) / stdv) * g.z + b.z;
          o[4 * j + 3] = ((__uint_as_float(yv[4 * j + 3]) - mean) / stdv) * g.w + b.w;
        }
        if (lane == 0) tma_store_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(st32 + stage_off<true>(lane, j)) =
              make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(stb + stage_off<false>(lane, j)) =
              make_uint4(pack_bf16(o[8 * j], o[8 * j + 1]), pack_bf16(o[8 * j + 2], o[8 * j + 3]),
                         pack_bf16(o[8 * j + 4], o[8 * j + 5]), pack_bf16(o[8 * j + 6], o[8 * j + 7]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmO32, st32, col0, row0);
          tma_store_2d(&tmOb, stb, col0, row0);
          tma_store_commit();
        }
      }
      // staging lives in this warp's P regions: drain before GELU reuses them
      if (lane == 0) tma_store_wait_read<0>();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(y_empty);
    }
    if (!ok) fail(kDevTimeoutEpilogue);
    if (lane == 0) tma_store_wait_all();
    __syncwarp();
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
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace ec
