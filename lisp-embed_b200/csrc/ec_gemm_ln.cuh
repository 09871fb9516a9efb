// ec_gemm_ln.cuh -- tcgen05 GEMM with the residual add and LayerNorm fused
// into the epilogue: the two "add & norm" steps of bert::encoder-layer
// (attention output, bert.lisp:250-256; feed-forward output, :266-270) and of
// bert::mpnet-layer.
//
//   x = A . W^T + bias + resid        (fp32, one full row of N = hidden)
//   y = (x - mean(x)) / (sqrt(var(x)) + 1e-12) * g + b
//   outb = bf16(y) (next GEMM's input), out32 = y (fp32, optional)
//
// The residual is either the fp32 stream or (RB) the previous LayerNorm's
// bf16 output -- the same rounded row the next GEMM already reads.
//
// A LayerNorm needs whole rows, wider than one CTA's accumulator, so a
// thread-block cluster of C CTAs shares each 128-row tile: CTA r computes
// columns [r * BN, (r + 1) * BN).  Each epilogue warp covers a quarter of the
// rows and half of the CTA's columns, computes the sum and the sum of squared
// deviations from its own partial mean, and the parts are merged with the
// pairwise formula of Chan, Golub and LeVeque (M2 = sum M2_i + n_i (mean_i -
// mean)^2) after ONE exchange through distributed shared memory -- the same
// mean and variance as the reference's two passes, up to rounding.  The rest
// follows ec_gemm.cuh: warp 0 TMA producer, warp 1 UMMA issuer with
// double-buffered TMEM accumulators, warps 2..9 epilogue.  The residual
// arrives by TMA in the swizzled layout the epilogue reads (two chunks in
// flight per warp); x = acc + bias + resid is written back to TMEM (pass A),
// the deviations are summed (pass B), then rows are normalised, staged and
// bulk-stored with TMA (pass C).  The pre-norm row never touches HBM.
#pragma once

#include "ec_gemm.cuh"

namespace ec {

struct GemmLnArgs {
  int M, N, K;
  const float* bias;   // [N] or nullptr
  const float* ln_g;   // [N] (RMS modes: the first gain)
  const float* ln_b;   // [N] (kNormPostAdd: the second gain, or nullptr)
  int m_tiles;
  int out32;           // 1: also store the fp32 row
  int outb;            // 1: store the bf16 row
  float eps;           // RMS modes
  float scale;         // kNormPostAdd: layer scalar (when has_scale); kNormScaled: input scale
  int has_scale;
  unsigned* status;
};

// epilogue of gemm_ln_kernel (x = the accumulator row of N = hidden columns)
enum GemmNorm : int {
  kNormLayer = 0,    // LayerNorm(x + bias + resid) -> out32 / outb (bert.lisp)
  kNormResRms = 1,   // h = x + resid -> out32, outb = RMSNorm(h) * g (llama.lisp
                     // residual add + the next pre-norm)
  kNormPostAdd = 2,  // h = (resid + RMSNorm(x) * g) [* scale] -> out32, outb =
                     // RMSNorm(h) * g2 or h (gemma::layer-forward post-norms)
  kNormScaled = 3,   // out32 = RMSNorm(x * scale) * g (gemma per-layer input)
};

// RB: the residual arrives as bf16 (the previous LayerNorm's bf16 output,
// which is also the next GEMM's input) instead of fp32
template <int BN, int C, bool RB = false, int NM = kNormLayer>
struct GemmLnCfg {
  static constexpr int NCH = BN / 32;                      // 32-column chunks per CTA
  static constexpr uint32_t A_BYTES = kGemmBM * kGemmBK * 2;
  static constexpr uint32_t B_BYTES = BN * kGemmBK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  // per epilogue warp: two fp32 32 x 32 buffers (residual in by TMA, then
  // fp32 out) and one bf16 32 x 32 staging chunk
  static constexpr uint32_t BUF_BYTES = 4096;
  static constexpr uint32_t RES_BYTES = RB ? 2048 : 4096;  // one residual chunk
  static constexpr uint32_t WARP_BYTES = 2 * BUF_BYTES + 2048;
  static constexpr uint32_t EPI_BYTES = kGemmEpiWarps * WARP_BYTES;
  // exchange slots: float2 (sum, M2) [2 tile parities][C ranks][2 halves][128 rows]
  static constexpr uint32_t XS_BYTES = 2 * C * 2 * 128 * 8;
  static constexpr uint32_t XS_TX = C * kGemmEpiWarps * 32 * 8;  // bytes landing per tile
  // bias, LayerNorm gain and shift of this CTA's column slice
  static constexpr uint32_t VEC_BYTES = 3 * BN * 4;
  static constexpr int MAX_STAGES =
      (232448 - 1024 - 512 - static_cast<int>(EPI_BYTES + XS_BYTES + VEC_BYTES)) /
      static_cast<int>(STAGE_BYTES);
  static constexpr int STAGES = MAX_STAGES > 6 ? 6 : MAX_STAGES;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
  static constexpr size_t SMEM_BYTES =
      1024 + STAGES * STAGE_BYTES + EPI_BYTES + XS_BYTES + VEC_BYTES + 512;
  static_assert(STAGES >= 2, "shared memory budget");
  static_assert(NCH % 2 == 0, "both epilogue halves take whole chunks");
};

template <int BN, int C, bool RB, int NM>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO32,
                   const __grid_constant__ CUtensorMap tmOb,
                   const __grid_constant__ CUtensorMap tmR, const GemmLnArgs args) {
  using Cfg = GemmLnCfg<BN, C, RB, NM>;
  constexpr int STAGES = Cfg::STAGES;
  static_assert(NM == kNormLayer || !RB, "RMS modes take an fp32 residual");
  constexpr int NCH = Cfg::NCH;
  constexpr uint32_t IDESC = make_idesc(1, kGemmBM, BN);
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* smE = smB + STAGES * Cfg::B_BYTES;  // epilogue buffers, WARP_BYTES per warp
  float2* xs = reinterpret_cast<float2*>(smE + Cfg::EPI_BYTES);
  float* sVec = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + Cfg::XS_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sVec) + Cfg::VEC_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* xbar = tempty + 2;  // [2 tile parities]: local expect_tx + C * 256 remote stores
  uint64_t* rbar = xbar + 2;    // [8 epilogue warps][2 buffers] residual loads
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2 * kGemmEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_rank());  // = column slice
  const int cluster = blockIdx.x / C;
  const int nclusters = gridDim.x / C;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kGemmEpiWarps);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&xbar[i], 1);
    for (int i = 0; i < 2 * kGemmEpiWarps; ++i) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmO32);
    tma_prefetch_desc(&tmOb);
    tma_prefetch_desc(&tmR);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= 2) {
    // bias (0 when absent), gain and shift of columns [rank * BN, +BN)
    const int rk = static_cast<int>(cluster_rank());
    for (int i = threadIdx.x - 64; i < BN; i += kGemmThreads - 64) {
      sVec[i] = args.bias ? args.bias[rk * BN + i] : 0.f;
      sVec[BN + i] = args.ln_g[rk * BN + i];
      sVec[2 * BN + i] = args.ln_b ? args.ln_b[rk * BN + i] : 0.f;
    }
  }
  tc_fence_before();
  cluster_sync_all();  // every CTA's barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int k_blocks = args.K / kGemmBK;

  if (warp == 0) {
    if (elect_one()) {
      const uint64_t pol_w = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int mb = cluster; ok && mb < args.m_tiles; mb += nclusters) {
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            report(args.status, kDevTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_2d(smA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * kGemmBK, mb * kGemmBM);
          tma_load_2d_hint(smB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * kGemmBK, rank * BN,
                           pol_w);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int mb = cluster; ok && mb < args.m_tiles; mb += nclusters) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          report(args.status, kDevTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            report(args.status, kDevTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(smB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k)
            umma_f16(d_tmem, desc_sw128_kmajor(a_addr + k * 32), desc_sw128_kmajor(b_addr + k * 32),
                     IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // epilogue warps 2..9: lane quadrant warp % 4 (rows), chunk parity half
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int half = ew >> 2;
    const int row = quad * 32 + lane;  // row in the tile == TMEM lane
    constexpr int NLOC = NCH / 2;      // chunks of this warp: c = half + 2 * ci
    constexpr float kLocCols = static_cast<float>(NLOC * 32);
    uint8_t* bufs = smE + ew * Cfg::WARP_BYTES;
    uint8_t* stb = bufs + 2 * Cfg::BUF_BYTES;  // bf16 staging
    uint64_t* rb = rbar + ew * 2;
    uint32_t rbits = 0;  // phase parity of rb[0], rb[1]
    const float inv_n = 1.0f / static_cast<float>(args.N);
    // xs[par][r][hf][row]
    auto slot = [&](int par, int r, int hf) -> int { return ((par * C + r) * 2 + hf) * 128 + row; };
    auto load_res = [&](int b, int c, int row0) {
      mbar_arrive_expect_tx(&rb[b], Cfg::RES_BYTES);
      tma_load_2d(bufs + b * Cfg::BUF_BYTES, &tmR, &rb[b], rank * BN + c * 32, row0);
    };
    int acc = 0;
    uint32_t acc_phase = 0;
    int tcount = 0;
    bool ok = true;
    for (int mb = cluster; mb < args.m_tiles; mb += nclusters, ++tcount) {
      const int par = tcount & 1;
      const int row0 = mb * kGemmBM + quad * 32;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      // residual chunks by TMA into the two buffers, once the previous
      // tile's bulk stores have finished reading them
      // kNormPostAdd with a second gain exchanges twice per tile, through
      // fixed slots 0 / 1 (a partner can only overwrite slot e after every
      // CTA has passed the other exchange); one exchange alternates slots
      // with the tile parity
      const bool two_ex = NM == kNormPostAdd && args.ln_b != nullptr;
      if (lane == 0) {
        tma_store_wait_read<0>();
        if constexpr (NM != kNormScaled) {
          load_res(0, half, row0);
          if (NLOC > 1) load_res(1, half + 2, row0);
        }
        // this tile's exchange: C * 256 partners' 8-byte stores land here
        if (ew == 0) {
          if (two_ex) {
            mbar_arrive_expect_tx(&xbar[0], Cfg::XS_TX);
            mbar_arrive_expect_tx(&xbar[1], Cfg::XS_TX);
          } else {
            mbar_arrive_expect_tx(&xbar[par], Cfg::XS_TX);
          }
        }
      }
      __syncwarp();
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if constexpr (NM != kNormLayer) {
        // ---------------------------------------------- RMS epilogues --
        // this lane's fp32 residual row of chunk ci (buffer ci & 1), then
        // the next load into the same buffer once every lane has read it
        auto take_res = [&](int ci, float (&rr)[32]) -> bool {
          const int b = ci & 1;
          if (!mbar_wait_warp(&rb[b], (rbits >> b) & 1u, abort_flag)) return false;
          rbits ^= 1u << b;
          const uint8_t* buf = bufs + b * Cfg::BUF_BYTES;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 q = *reinterpret_cast<const float4*>(buf + stage_off<true>(lane, j));
            rr[4 * j] = q.x;
            rr[4 * j + 1] = q.y;
            rr[4 * j + 2] = q.z;
            rr[4 * j + 3] = q.w;
          }
          __syncwarp();
          if (lane == 0 && ci + 2 < NLOC) load_res(b, half + 2 * (ci + 2), row0);
          return true;
        };
        // one exchange of this warp's partial sum of squares; total over the row
        auto exchange = [&](int sl, uint32_t parity, float val, float& total) -> bool {
          const uint32_t dst = smem_u32(xs + slot(sl, rank, half));
          const uint32_t bar = smem_u32(&xbar[sl]);
#pragma unroll
          for (int r = 0; r < C; ++r)
            st_async_cluster_v2(cluster_map(dst, r), val, 0.f, cluster_map(bar, r));
          if (!mbar_wait_cluster_warp(&xbar[sl], parity, abort_flag)) return false;
          float t = 0.f;
#pragma unroll
          for (int r = 0; r < C; ++r) t += xs[slot(sl, r, 0)].x + xs[slot(sl, r, 1)].x;
          total = t;
          return true;
        };
        const int sl0 = two_ex ? 0 : par;
        const uint32_t ph0 = two_ex ? static_cast<uint32_t>(tcount & 1)
                                    : static_cast<uint32_t>((tcount >> 1) & 1);
        // ---- pass A: x (+ resid / * scale) -> TMEM where it changes; sum x^2
        float ss = 0.f;
#pragma unroll 1
        for (int ci = 0; ci < NLOC; ++ci) {
          const int cl = (half + 2 * ci) * 32;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + cl, v);
          float rr[32];
          if constexpr (NM == kNormResRms) {
            if (!take_res(ci, rr)) {
              ok = false;
              break;
            }
          }
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = __uint_as_float(v[j]);
            if constexpr (NM == kNormResRms) x = x + rr[j];
            if constexpr (NM == kNormScaled) x = x * args.scale;
            ss += x * x;
            v[j] = __float_as_uint(x);
          }
          if constexpr (NM != kNormPostAdd) tmem_st_32x32b_x32(t_row + cl, v);
        }
        if (!ok) break;
        if constexpr (NM != kNormPostAdd) tmem_wait_st();
        float tot = 0.f;
        if (!exchange(sl0, ph0, ss, tot)) {
          ok = false;
          break;
        }
        const float inv1 = 1.0f / sqrtf(tot * inv_n + args.eps);
        float inv2 = 1.f;
        if constexpr (NM == kNormPostAdd) {
          // ---- pass B: h = resid + RMSNorm(x) * g1 [* scale] -> TMEM; sum h^2
          float ss2 = 0.f;
#pragma unroll 1
          for (int ci = 0; ci < NLOC; ++ci) {
            const int cl = (half + 2 * ci) * 32;
            uint32_t v[32];
            tmem_ld_32x32b_x32(t_row + cl, v);
            float rr[32];
            if (!take_res(ci, rr)) {
              ok = false;
              break;
            }
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float hv = rr[j] + (__uint_as_float(v[j]) * inv1) * sVec[BN + cl + j];
              if (args.has_scale) hv = hv * args.scale;
              ss2 += hv * hv;
              v[j] = __float_as_uint(hv);
            }
            tmem_st_32x32b_x32(t_row + cl, v);
          }
          if (!ok) break;
          tmem_wait_st();
          if (two_ex) {
            float tot2 = 0.f;
            if (!exchange(1, static_cast<uint32_t>(tcount & 1), ss2, tot2)) {
              ok = false;
              break;
            }
            inv2 = 1.0f / sqrtf(tot2 * inv_n + args.eps);
          }
        }
        // ---- pass C: stage and bulk-store the fp32 and / or bf16 rows
#pragma unroll 1
        for (int ci = 0; ci < NLOC; ++ci) {
          const int cl = (half + 2 * ci) * 32;
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + cl, v);
          uint8_t* st32 = bufs + (ci & 1) * Cfg::BUF_BYTES;
          if (lane == 0) tma_store_wait_read<0>();
          __syncwarp();
          tmem_wait_ld();
          if (ci + 1 == NLOC) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float o32[8], ob[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int k = 8 * j + e;
              const float x = __uint_as_float(v[k]);
              if constexpr (NM == kNormResRms) {
                o32[e] = x;
                ob[e] = (x * inv1) * sVec[BN + cl + k];
              } else if constexpr (NM == kNormPostAdd) {
                o32[e] = x;
                ob[e] = two_ex ? (x * inv2) * sVec[2 * BN + cl + k] : x;
              } else {
                o32[e] = (x * inv1) * sVec[BN + cl + k];
                ob[e] = o32[e];
              }
            }
            if (args.out32) {
              *reinterpret_cast<float4*>(st32 + stage_off<true>(lane, 2 * j)) =
                  make_float4(o32[0], o32[1], o32[2], o32[3]);
              *reinterpret_cast<float4*>(st32 + stage_off<true>(lane, 2 * j + 1)) =
                  make_float4(o32[4], o32[5], o32[6], o32[7]);
            }
            if (args.outb)
              *reinterpret_cast<uint4*>(stb + stage_off<false>(lane, j)) =
                  make_uint4(pack_bf16(ob[0], ob[1]), pack_bf16(ob[2], ob[3]),
                             pack_bf16(ob[4], ob[5]), pack_bf16(ob[6], ob[7]));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (args.out32) tma_store_2d(&tmO32, st32, rank * BN + cl, row0);
            if (args.outb) tma_store_2d(&tmOb, stb, rank * BN + cl, row0);
            tma_store_commit();
          }
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
        continue;
      }
      // ---- pass A: x = acc + bias + resid, back into TMEM; partial sum;
      // chunk ci's residual is in buffer ci & 1
      float s_loc = 0.f;
#pragma unroll 1
      for (int ci = 0; ci < NLOC; ++ci) {
        const int b = ci & 1;
        const int cl = (half + 2 * ci) * 32;  // column within the slice
        const uint8_t* buf = bufs + b * Cfg::BUF_BYTES;
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + cl, v);
        if (!mbar_wait_warp(&rb[b], (rbits >> b) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        rbits ^= 1u << b;
        tmem_wait_ld();
        float rr[32];  // this lane's row of the residual chunk
        if constexpr (RB) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 u = *reinterpret_cast<const uint4*>(buf + stage_off<false>(lane, j));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              rr[8 * j + 2 * e] = __uint_as_float(w[e] << 16);
              rr[8 * j + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 q = *reinterpret_cast<const float4*>(buf + stage_off<true>(lane, j));
            rr[4 * j] = q.x;
            rr[4 * j + 1] = q.y;
            rr[4 * j + 2] = q.z;
            rr[4 * j + 3] = q.w;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 q = make_float4(rr[4 * j], rr[4 * j + 1], rr[4 * j + 2], rr[4 * j + 3]);
          const float4 bb = *reinterpret_cast<const float4*>(sVec + cl + 4 * j);
          const float x0 = (__uint_as_float(v[4 * j]) + bb.x) + q.x;
          const float x1 = (__uint_as_float(v[4 * j + 1]) + bb.y) + q.y;
          const float x2 = (__uint_as_float(v[4 * j + 2]) + bb.z) + q.z;
          const float x3 = (__uint_as_float(v[4 * j + 3]) + bb.w) + q.w;
          s_loc += (x0 + x1) + (x2 + x3);
          v[4 * j] = __float_as_uint(x0);
          v[4 * j + 1] = __float_as_uint(x1);
          v[4 * j + 2] = __float_as_uint(x2);
          v[4 * j + 3] = __float_as_uint(x3);
        }
        tmem_st_32x32b_x32(t_row + cl, v);
        __syncwarp();  // every lane has read the buffer
        if (lane == 0 && ci + 2 < NLOC) load_res(b, half + 2 * (ci + 2), row0);
      }
      if (!ok) break;
      tmem_wait_st();
      // ---- pass B: squared deviations from this warp's partial mean
      const float m_loc = s_loc / kLocCols;
      float m2_loc = 0.f;
#pragma unroll 1
      for (int ci = 0; ci < NLOC; ++ci) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + (half + 2 * ci) * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float d0 = __uint_as_float(v[j]) - m_loc, d1 = __uint_as_float(v[j + 1]) - m_loc;
          m2_loc += d0 * d0 + d1 * d1;
        }
      }
      // ---- one exchange of (sum, M2): an 8-byte asynchronous store into
      // every CTA of the cluster, counted by that CTA's transaction barrier
      {
        const uint32_t dst = smem_u32(xs + slot(par, rank, half));
        const uint32_t bar = smem_u32(&xbar[par]);
#pragma unroll
        for (int r = 0; r < C; ++r)
          st_async_cluster_v2(cluster_map(dst, r), s_loc, m2_loc, cluster_map(bar, r));
      }
      if (!mbar_wait_cluster_warp(&xbar[par], static_cast<uint32_t>((tcount >> 1) & 1), abort_flag)) {
        ok = false;
        break;
      }
      // merge in a fixed order, identical on every CTA of the cluster
      float sum = 0.f;
#pragma unroll
      for (int r = 0; r < C; ++r) sum += xs[slot(par, r, 0)].x + xs[slot(par, r, 1)].x;
      const float mean = sum * inv_n;
      float m2 = 0.f;
#pragma unroll
      for (int r = 0; r < C; ++r)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const float2 p = xs[slot(par, r, hf)];
          const float dm = p.x / kLocCols - mean;
          m2 += p.y + kLocCols * dm * dm;
        }
      const float stdv = sqrtf(m2 * inv_n) + 1e-12f;
      const float inv = 1.0f / stdv;
      // ---- pass C: normalise, stage, bulk-store fp32 and bf16 rows
#pragma unroll 1
      for (int ci = 0; ci < NLOC; ++ci) {
        const int cl = (half + 2 * ci) * 32;  // column within the slice
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_row + cl, v);
        uint8_t* st32 = bufs + (ci & 1) * Cfg::BUF_BYTES;
        // fp32 buffer and the bf16 chunk are free once earlier stores read them
        if (lane == 0) tma_store_wait_read<0>();
        __syncwarp();
        tmem_wait_ld();
        if (ci + 1 == NLOC) {
          // last TMEM read of the tile: the accumulator goes back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            y[e] = ((__uint_as_float(v[8 * j + e]) - mean) * inv) * sVec[BN + cl + 8 * j + e] +
                   sVec[2 * BN + cl + 8 * j + e];
          if (args.out32) {
            *reinterpret_cast<float4*>(st32 + stage_off<true>(lane, 2 * j)) =
                make_float4(y[0], y[1], y[2], y[3]);
            *reinterpret_cast<float4*>(st32 + stage_off<true>(lane, 2 * j + 1)) =
                make_float4(y[4], y[5], y[6], y[7]);
          }
          *reinterpret_cast<uint4*>(stb + stage_off<false>(lane, j)) =
              make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]),
                         pack_bf16(y[6], y[7]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (args.out32) tma_store_2d(&tmO32, st32, rank * BN + cl, row0);
          tma_store_2d(&tmOb, stb, rank * BN + cl, row0);
          tma_store_commit();
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (!ok) {
      report(args.status, kDevTimeoutEpilogue);
      *abort_flag = 1;
    }
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
  cluster_sync_all();  // no partner still writes into this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace ec
