// ec_gemm.cuh -- persistent tcgen05 GEMM for sm_100a.
//
//   C[M, N] = A[M, K] . W[N, K]^T  (+ fused epilogue)
//
// A (activations, bf16, row-major, K contiguous) and W (weights, bf16,
// PyTorch Linear layout [out, in]) are both K-major.  This is the product
// `linear` computes one token at a time in the reference (bert.lisp:145-153,
// llama.lisp:97-104); here one launch covers every token of the batch.
//
// Structure (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      : TMA producer (one elected lane) -- A tile 128x64 and W tile
//                 BNx64 per stage, 128-byte swizzle, STAGES-deep ring.
//   warp 1      : TMEM allocator + UMMA issuer (one elected lane):
//                 tcgen05.mma.cta_group::1.kind::f16, M=128, N=BN, K=16,
//                 fp32 accumulators in TMEM, double-buffered (2 x BN columns)
//                 so the epilogue of tile i overlaps the MMAs of tile i+1.
//   warps 2..9  : epilogue; warp w owns TMEM lanes 32*(w%4).. (= tile rows),
//                 two warps per lane quadrant take alternate 32-column chunks
//                 (tcgen05.ld), apply the epilogue in fp32, stage the 32x32
//                 chunk in swizzled shared memory (double-buffered) and write
//                 it with a TMA bulk tensor store; rows past M are clipped by
//                 the tensor map.  The fp32 residual of a chunk is read with
//                 coalesced 16-byte loads issued before the TMEM read and
//                 transposed to row-per-lane through the same staging buffer.
// All waits are bounded (ec_ptx.cuh); a timeout records a status code,
// raises the CTA abort flag and every role unwinds, then TMEM is freed.
#pragma once

#include "ec_ptx.cuh"

namespace ec {

enum GemmEpi : int {
  kEpiBf16 = 0,        // out bf16 = acc + bias
  kEpiBf16Gelu = 1,    // out bf16 = gelu(acc + bias)           (bert.lisp:263-264)
  kEpiF32Resid = 2,    // out f32  = (acc + bias) + resid       (bert.lisp:250-256)
  kEpiBf16Swiglu = 3,  // out bf16 = silu(gate) * up, N/2 wide  (llama.lisp:284-290)
  kEpiF32 = 4,         // out f32  = acc + bias
  kEpiBf16QkRope = 5,  // out bf16 = acc, with per-head RMSNorm + RoPE on the
                       // q/k heads (llama.lisp:244-253, 137-151), head dim 128
  kEpiBf16GeluTanhGate = 6,  // out bf16 = gelu_tanh(gate) * up, N/2 wide
                             // (gemma.lisp:277-283), SwiGLU's tile layout
  kEpiBf16GeluTanhMul = 7,   // out bf16 = gelu_tanh(acc) * resid, resid fp32
                             // [M, ldr] (the PLE gate, gemma.lisp:290-293)
  kEpiArgCand = 8,           // no dense output: per row and column part the
                             // best approximate score and the candidates for
                             // the exact argmax (ArgCandEpi)
};

// k-means assignment prefilter (kEpiArgCand).  For row r and column part t
// (= 2 * column tile + epilogue half) of the approximate scores S~ = bf16(x)
// . bf16(c)^T: mloc[t][r] = the largest S~; the part's window is the columns
// with S~ >= mloc - w_r; col1/col2 = its first two columns in column order
// (with one, col1 is the argmax), meta bit 0 = it holds at least two, bit 1
// = at least three (then two columns do not cover the part and the row
// needs the exact scan); the three are packed in pk[t][r].  w_r = wscale *
// xnorm[r] is twice the bound on |S~ - S| for that row, so the exact argmax -- and every column exactly tied
// with it -- has S~ >= max S~ - w_r.  Arrays are [parts][M].  (w_r =
// rel2 * cmax * xnorm[r]; wscale below is rel2 * cmax.)
struct ArgCandEpi {
  const float* xnorm;   // [M] upper bounds of the row norms
  const float* cmax;    // [1] upper bound of the largest centroid norm
  float rel2;           // 2 * relative bound: w_r = rel2 * cmax * xnorm[r]
  float* mloc;
  uint32_t* pk;         // col1 | col2 << 15 | meta << 30 (k <= 32768)
};

// per-head q/k RMSNorm + rotate-half RoPE applied in the QKV epilogue
struct QkRopeEpi {
  const float* q_norm;  // [128] or nullptr (no q/k norm)
  const float* k_norm;
  int q_heads, k_heads; // heads [0, q_heads) use q_norm, the next k_heads k_norm
  double eps;
  const int* pos;       // [M] position of each row
  const float* cos_t;   // [max_pos, 64]
  const float* sin_t;
  int v_heads = 0;      // v heads after the k heads get the unweighted
  int v_norm = 0;       // RMSNorm (gemma.lisp:244) when v_norm, no RoPE
};

struct GemmArgs {
  int M, N, K;
  const float* bias;   // [N] or nullptr
  const float* resid;  // [M, ldr] fp32 (kEpiF32Resid, kEpiBf16GeluTanhMul); may alias out
  int ldr;
  void* out;           // bf16 or fp32, row stride ldo elements
  int ldo;
  int n_tiles_n;       // N / BN
  int num_tiles;       // ceil(M / 128) * n_tiles_n
  unsigned* status;    // device status word
  QkRopeEpi qk;        // kEpiBf16QkRope only
  ArgCandEpi ac;       // kEpiArgCand only
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 320;  // 2 control warps + 8 epilogue warps
constexpr int kGemmEpiWarps = 8;
// threads of a GEMM CTA with EW epilogue warps
constexpr int gemm_threads(int ew) { return (2 + ew) * 32; }

// CG: CTAs per MMA (1, or 2 = a cluster pair issuing cta_group::2 MMAs of
// M = 256: each CTA loads only half of the W tile, so the operand traffic per
// output drops by a third -- the mainloop is bound by L2 -> SM bandwidth).
// WR: weight-resident mode for K <= kGemmWrMaxK -- each CTA keeps its rows
// of one W tile (all K) in shared memory for the whole launch and streams A
// only (see the tile schedule in gemm_tn_bf16_kernel).
constexpr int kGemmWrMaxK = 384;

template <int BN, int EPI, int CG = 1, bool WR = false>
struct GemmCfg {
  static constexpr bool OUT_F32 = EPI == kEpiF32Resid || EPI == kEpiF32 || EPI == kEpiArgCand;
  // one 32 x 32 output chunk: fp32 rows of 128 B (128B swizzle) or bf16
  // rows of 64 B (64B swizzle); two per epilogue warp
  // (kEpiBf16GeluTanhMul stages its fp32 multiplier chunk in the same slot)
  static constexpr uint32_t CHUNK_BYTES = (OUT_F32 || EPI == kEpiBf16GeluTanhMul) ? 4096 : 2048;
  // (kEpiArgCand stores nothing through shared memory)
  static constexpr uint32_t EPI_BYTES = EPI == kEpiArgCand ? 0 : kGemmEpiWarps * 2 * CHUNK_BYTES;
  static constexpr uint32_t A_BYTES = kGemmBM * kGemmBK * 2;
  static constexpr uint32_t B_BYTES = (BN / CG) * kGemmBK * 2;  // this CTA's rows of W
  // WR: the resident W rows (kGemmWrMaxK / kGemmBK k-blocks), stages of A only
  static constexpr uint32_t W_BYTES = WR ? (kGemmWrMaxK / kGemmBK) * B_BYTES : 0;
  static constexpr uint32_t STAGE_BYTES = WR ? A_BYTES : A_BYTES + B_BYTES;
  static constexpr int MAX_STAGES = (232448 - 1024 - 512 - static_cast<int>(EPI_BYTES) -
                                     static_cast<int>(W_BYTES)) /
                                    static_cast<int>(STAGE_BYTES);
  static constexpr int STAGES = MAX_STAGES > 6 ? 6 : MAX_STAGES;
  static constexpr uint32_t TMEM_COLS =
      2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512));
  static constexpr size_t SMEM_BYTES = 1024 + W_BYTES + STAGES * STAGE_BYTES + EPI_BYTES + 512;
  static_assert(STAGES >= 2, "shared memory budget");
};

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// max(a, b, c) in one instruction (sm_100); a NaN operand is ignored, as by fmaxf
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// all ones when a >= b, else 0 (false for NaN)
__device__ __forceinline__ uint32_t ge_mask(float a, float b) {
  uint32_t r;
  asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(r) : "f"(a), "f"(b));
  return r;
}

// GELU with the erf of Abramowitz-Stegun 7.1.26 (|error| <= 1.5e-7), the
// form bert::gelu uses (bert.lisp:176-192).  Branch-free: one approximate
// reciprocal and one exp2 per element (relative error ~1e-6, far below the
// bf16 rounding of the result).
__device__ __forceinline__ float gelu_as(float x) {
  const float z = x * 0.70710678118654752f;
  const float az = fabsf(z);
  const float t = rcp_approx(fmaf(0.3275911f, az, 1.0f));
  const float poly =
      t * (0.254829592f +
           t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
  const float e = fmaf(-poly, ex2_approx(-1.4426950408889634f * az * az), 1.0f);
  const float se = copysignf(e, z);
  const float hx = 0.5f * x;
  return fmaf(hx, se, hx);
}

// gelu_as on two values with the packed fp32 pipe (fma/mul .f32x2 issue two
// lanes' worth of arithmetic per instruction); same formula, same constants.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 gelu_as2(float2 x) {
  const float2 z = __fmul2_rn(x, f2(0.70710678118654752f));
  const float2 az = make_float2(fabsf(z.x), fabsf(z.y));
  const float2 den = __ffma2_rn(f2(0.3275911f), az, f2(1.0f));
  const float2 t = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  // -poly(t), Horner with negated coefficients, so that 1 - poly * e is one fma
  float2 p = __ffma2_rn(t, f2(-1.061405429f), f2(1.453152027f));
  p = __ffma2_rn(t, p, f2(-1.421413741f));
  p = __ffma2_rn(t, p, f2(0.284496736f));
  p = __ffma2_rn(t, p, f2(-0.254829592f));
  p = __fmul2_rn(t, p);
  const float2 q = __fmul2_rn(__fmul2_rn(az, az), f2(-1.4426950408889634f));
  const float2 e = make_float2(ex2_approx(q.x), ex2_approx(q.y));
  const float2 r = __ffma2_rn(p, e, f2(1.0f));
  const float2 se = make_float2(copysignf(r.x, z.x), copysignf(r.y, z.y));
  const float2 hx = __fmul2_rn(x, f2(0.5f));
  return __ffma2_rn(hx, se, hx);
}

// gelu_pytorch_tanh (gemma::gelu-tanh, gemma.lisp:85-89) in single precision
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float c = 0.7978845608028654f * (x + ((0.044715f * x) * x) * x);
  return (0.5f * x) * (1.0f + tanhf(c));
}

// x * sigmoid(x) (llama::silu, llama.lisp:119-122)
__device__ __forceinline__ float silu_f(float x) {
  return x * rcp_approx(1.0f + ex2_approx(-1.4426950408889634f * x));
}

// Byte offset of 16-byte column chunk c of row r in a swizzled staging chunk:
// fp32 rows are 128 B (chunk c ^ (r & 7)), bf16 rows 64 B (c ^ ((r >> 1) & 3)),
// the layouts TMA's 128B / 64B swizzle modes read.
template <bool F32>
__device__ __forceinline__ uint32_t stage_off(int r, int c) {
  if constexpr (F32) return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
  return static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

template <int BN, int EPI, int CG = 1, bool WR = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tn_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using Cfg = GemmCfg<BN, EPI, CG, WR>;
  constexpr int EW = kGemmEpiWarps;
  static_assert(CG == 1 || CG == 2, "CTA group");
  constexpr int STAGES = Cfg::STAGES;
  constexpr bool F32 = Cfg::OUT_F32;
  constexpr uint32_t IDESC = make_idesc(1, kGemmBM * CG, BN);
  constexpr int TM = kGemmBM * CG;  // rows per tile
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(EPI != kEpiBf16Swiglu || BN % 64 == 0, "swiglu BN");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* smA = smem;
  // WR: smB is the resident W (k-block kb at kb * B_BYTES); else B stages
  uint8_t* smB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* smE = smB + (WR ? Cfg::W_BYTES : STAGES * Cfg::B_BYTES);  // epilogue staging, 2 chunks per warp
  uint64_t* full = reinterpret_cast<uint64_t*>(smE + Cfg::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* w_full = tempty + 2;  // WR: the resident W has landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(w_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // pair: CTA `rank` owns rows rank * 128.. of each 256-row tile; the even
  // CTA issues the MMAs; both walk the same tiles
  const uint32_t rank = CG == 2 ? cluster_rank() : 0u;
  const int unit = CG == 2 ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
  const int units = CG == 2 ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);
  // Tile schedule.  Default: tiles unit, unit + units, ... of the row-block
  // major order (tile = mb * n_tiles_n + nb).  WR: units form groups of
  // n_tiles_n; unit u keeps W tile nb = u % n_tiles_n resident and takes the
  // row blocks of its group's contiguous share (the launcher guarantees
  // units >= n_tiles_n), so the units of a group read the same A tiles at
  // about the same time (L2 hits) and W crosses to the SM once.  For WR a
  // "tile" below is the row block mb itself.
  int tile0, tstep, tend, wr_nb = 0;
  if constexpr (WR) {
    const int groups = units / args.n_tiles_n;
    const int g = unit / args.n_tiles_n;
    const int m_tiles = args.num_tiles / args.n_tiles_n;
    const int per = (m_tiles + groups - 1) / groups;
    wr_nb = unit % args.n_tiles_n;
    tile0 = g < groups ? g * per : m_tiles;
    tend = g < groups ? min(m_tiles, tile0 + per) : m_tiles;
    tstep = 1;
  } else {
    tile0 = unit;
    tstep = units;
    tend = args.num_tiles;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EW * CG);  // the even CTA's counts both epilogues
    }
    mbar_init(w_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync_all();  // the partner's barriers exist
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int k_blocks = args.K / kGemmBK;
  // hand accumulator buffer b back to the MMA issuer (the even CTA's barrier)
  auto release_acc = [&](int b) {
    if constexpr (CG == 2) mbar_arrive_remote(cluster_map(smem_u32(&tempty[b]), 0));
    else mbar_arrive(&tempty[b]);
  };

  if (warp == 0) {
    if (elect_one()) {
      const uint64_t pol_w = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      if constexpr (WR) {
        // the resident W rows of this unit's tile, once for the launch
        if (tile0 < tend) {
          if constexpr (CG == 2) {
            if (rank == 0) mbar_arrive_expect_tx(w_full, 2 * k_blocks * Cfg::B_BYTES);
            const uint32_t fb = cluster_map(smem_u32(w_full), 0);
            for (int kb = 0; kb < k_blocks; ++kb)
              tma_load_2d_pair(smB + kb * Cfg::B_BYTES, &tmB, fb, kb * kGemmBK,
                               wr_nb * BN + static_cast<int>(rank) * (BN / 2));
          } else {
            mbar_arrive_expect_tx(w_full, k_blocks * Cfg::B_BYTES);
            for (int kb = 0; kb < k_blocks; ++kb)
              tma_load_2d_hint(smB + kb * Cfg::B_BYTES, &tmB, w_full, kb * kGemmBK, wr_nb * BN, pol_w);
          }
        }
      }
      for (int tile = tile0; ok && tile < tend; tile += tstep) {
        const int mb = WR ? tile : tile / args.n_tiles_n, nb = WR ? wr_nb : tile % args.n_tiles_n;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            report(args.status, kDevTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          if constexpr (CG == 2) {
            // both CTAs' bytes land on the even CTA's barrier, which expects them
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
            const uint32_t fb = cluster_map(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(smA + stage * Cfg::A_BYTES, &tmA, fb, kb * kGemmBK,
                             mb * TM + static_cast<int>(rank) * kGemmBM);
            if constexpr (!WR)
              tma_load_2d_pair(smB + stage * Cfg::B_BYTES, &tmB, fb, kb * kGemmBK,
                               nb * BN + static_cast<int>(rank) * (BN / 2));
          } else {
            mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
            tma_load_2d(smA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * kGemmBK,
                        mb * kGemmBM);
            if constexpr (!WR)
              tma_load_2d_hint(smB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * kGemmBK,
                               nb * BN, pol_w);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      if constexpr (WR) {
        if (tile0 < tend && !mbar_wait(w_full, 0, abort_flag)) {
          report(args.status, kDevTimeoutMma);
          *abort_flag = 1;
          ok = false;
        }
      }
      for (int tile = tile0; ok && tile < tend; tile += tstep) {
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
          const uint32_t b_addr = smem_u32(smB + (WR ? kb : stage) * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            if constexpr (CG == 2)
              umma_f16_pair(d_tmem, desc_sw128_kmajor(a_addr + k * 32),
                            desc_sw128_kmajor(b_addr + k * 32), IDESC, (kb > 0 || k > 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, desc_sw128_kmajor(a_addr + k * 32),
                       desc_sw128_kmajor(b_addr + k * 32), IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          if constexpr (CG == 2) umma_commit_pair(&empty[stage], 0x3);
          else umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (CG == 2) umma_commit_pair(&tfull[acc], 0x3);
        else umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // epilogue warps 2..EW+1: lane quadrant warp % 4, column part (warp - 2) / 4;
    // part p takes chunks p, p + PARTS, ...
    constexpr int PARTS = EW / 4;
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int half = ew >> 2;  // the column part
    uint8_t* stage_base = smE + ew * 2 * Cfg::CHUNK_BYTES;
    constexpr int NCH = (EPI == kEpiBf16Swiglu || EPI == kEpiBf16GeluTanhGate) ? BN / 64 : BN / 32;  // output chunks per tile
    static_assert(NCH >= PARTS, "every epilogue warp needs a chunk per tile");
    int acc = 0;
    uint32_t acc_phase = 0;
    int sbuf = 0;
    if constexpr (EPI == kEpiArgCand) {
      // All NCH / PARTS chunks of this thread's row part are read from TMEM
      // at once (one wait; the accumulator goes back straight away).  Pass 1:
      // the part's largest approximate score m (three-input max).  Pass 2:
      // one bit per column with S~ >= m - w (a set + a lop3 per score), the
      // first two such columns and their count.  The window holds the
      // part's argmax, so count 1 means col1 is the argmax; count 2 means
      // col1 / col2 are the two columns that need the exact re-score; count
      // >= 3 sends the row to the exact scan.
      constexpr int NCP = NCH / PARTS;
      static_assert(NCH % PARTS == 0 && NCP <= 4, "ArgCand chunks per part");
      const float wscale = args.ac.rel2 * *args.ac.cmax;
      for (int tile = tile0; tile < tend; tile += tstep) {
        const int mb = WR ? tile : tile / args.n_tiles_n, nb = WR ? wr_nb : tile % args.n_tiles_n;
        const int grow = mb * TM + static_cast<int>(rank) * kGemmBM + quad * 32 + lane;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                               static_cast<uint32_t>(acc * BN);
        const float w = grow < args.M ? wscale * args.ac.xnorm[grow] : 0.f;
        if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag)) {
          report(args.status, kDevTimeoutEpilogue);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint32_t r[NCP][32];
#pragma unroll
        for (int j = 0; j < NCP; ++j) tmem_ld_32x32b_x32(t_row + (half + j * PARTS) * 32, r[j]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(acc);
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < NCP; ++j) {
          float cm[11];
#pragma unroll
          for (int q = 0; q < 10; ++q)
            cm[q] = fmax3(__uint_as_float(r[j][3 * q]), __uint_as_float(r[j][3 * q + 1]),
                          __uint_as_float(r[j][3 * q + 2]));
          cm[10] = fmaxf(__uint_as_float(r[j][30]), __uint_as_float(r[j][31]));
          const float a = fmax3(cm[0], cm[1], cm[2]), b = fmax3(cm[3], cm[4], cm[5]),
                      c = fmax3(cm[6], cm[7], cm[8]);
          m = fmax3(m, fmax3(a, b, c), fmaxf(cm[9], cm[10]));
        }
        const float lo = m - w;
        int cnt = 0, c1 = 0, c2 = 0;
#pragma unroll
        for (int j = 0; j < NCP; ++j) {
          uint32_t bits = 0;
#pragma unroll
          for (int e = 0; e < 32; ++e) bits |= ge_mask(__uint_as_float(r[j][e]), lo) & (1u << e);
          const int col0 = nb * BN + (half + j * PARTS) * 32;
          const int f1 = __ffs(bits) - 1;                // -1 when empty
          const int f2 = __ffs(bits & (bits - 1u)) - 1;  // the second set bit
          c2 = cnt == 1 && f1 >= 0 ? col0 + f1 : (cnt == 0 && f2 >= 0 ? col0 + f2 : c2);
          c1 = cnt == 0 && f1 >= 0 ? col0 + f1 : c1;
          cnt += __popc(bits);
        }
        if (grow < args.M) {
          const size_t o = static_cast<size_t>(nb * PARTS + half) * args.M + grow;
          // a row whose window is not a finite number takes the exact scan
          const bool bad = !(w >= 0.f && w < INFINITY) || !(m > -INFINITY && m < INFINITY);
          args.ac.mloc[o] = bad ? INFINITY : m;
          const uint32_t meta = (cnt >= 2 ? 1u : 0u) | ((cnt >= 3 || bad) ? 2u : 0u);
          args.ac.pk[o] = static_cast<uint32_t>(c1) | (static_cast<uint32_t>(c2) << 15) | (meta << 30);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
    // bias / GELU / fp32 epilogues: two chunks per step (two TMEM loads, one
    // wait, 64 independent element chains), accumulator handed back as soon
    // as the last TMEM read lands
    constexpr bool kPaired =
        EPI == kEpiBf16 || EPI == kEpiBf16Gelu || EPI == kEpiF32 || EPI == kEpiBf16QkRope;
    for (int tile = tile0; kPaired && tile < tend; tile += tstep) {
      const int mb = WR ? tile : tile / args.n_tiles_n, nb = WR ? wr_nb : tile % args.n_tiles_n;
      const int row0 = mb * TM + static_cast<int>(rank) * kGemmBM + quad * 32;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      bool fine = true;
      if constexpr (EPI == kEpiBf16QkRope) {
        static_assert(BN == 256 && EW == 8, "two 128-wide heads per tile, one per warp half");
        const int qk_heads = args.qk.q_heads + args.qk.k_heads;
        if (nb * 2 < qk_heads + (args.qk.v_norm ? args.qk.v_heads : 0)) {
          // this warp half owns head gh = 2 nb + half (chunks 4 half .. 4 half + 3);
          // pass 1: the head's sum of squares (in double, as llama::rmsnorm),
          // pass 2: scale by the norm weight, rotate pairs (i, i + 64), store.
          // A v head in such a tile gets the unweighted norm (v_norm) or
          // nothing, and no rotation.
          const int gh = nb * 2 + half;
          const bool is_v = gh >= qk_heads;
          const float* wn = gh < args.qk.q_heads ? args.qk.q_norm : (is_v ? nullptr : args.qk.k_norm);
          const bool do_norm = is_v ? args.qk.v_norm != 0 : wn != nullptr;
          if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag)) {
            report(args.status, kDevTimeoutEpilogue);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t t_head = t_row + half * 128;
          float inv = 1.f;
          if (do_norm) {
            double ss = 0.0;
#pragma unroll 1
            for (int c = 0; c < 4; c += 2) {
              uint32_t r[2][32];
              tmem_ld_32x32b_x32(t_head + c * 32, r[0]);
              tmem_ld_32x32b_x32(t_head + (c + 1) * 32, r[1]);
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  const float x = __uint_as_float(r[h][j]);
                  ss += static_cast<double>(x * x);
                }
            }
            inv = static_cast<float>(1.0 / sqrt(ss / 128.0 + args.qk.eps));
          }
          const int grow = mb * TM + static_cast<int>(rank) * kGemmBM + quad * 32 + lane;
          const int p = grow < args.M ? args.qk.pos[grow] : 0;
          const float* cs = args.qk.cos_t + static_cast<size_t>(p) * 64;
          const float* sn = args.qk.sin_t + static_cast<size_t>(p) * 64;
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            // chunk c (columns 32c.. of the head) and its rotation partner c + 2
            uint32_t r[2][32];
            tmem_ld_32x32b_x32(t_head + c * 32, r[0]);
            tmem_ld_32x32b_x32(t_head + (c + 2) * 32, r[1]);
            tmem_wait_ld();
            if (c == 1) {
              // the head is in registers: hand the accumulator back
              tc_fence_before();
              __syncwarp();
              if (lane == 0) release_acc(acc);
            }
            float lo[32], hi[32];
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 c4 = *reinterpret_cast<const float4*>(cs + c * 32 + j);
              const float4 s4 = *reinterpret_cast<const float4*>(sn + c * 32 + j);
              float4 wl = make_float4(1.f, 1.f, 1.f, 1.f), wh = wl;
              if (wn) {
                wl = __ldg(reinterpret_cast<const float4*>(wn + c * 32 + j));
                wh = __ldg(reinterpret_cast<const float4*>(wn + 64 + c * 32 + j));
              }
              const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ssn[4] = {s4.x, s4.y, s4.z, s4.w};
              const float gl[4] = {wl.x, wl.y, wl.z, wl.w}, gh4[4] = {wh.x, wh.y, wh.z, wh.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float x = __uint_as_float(r[0][j + e]), y = __uint_as_float(r[1][j + e]);
                if (wn) {
                  x = (x * inv) * gl[e];
                  y = (y * inv) * gh4[e];
                } else if (do_norm) {
                  x = x * inv;
                  y = y * inv;
                }
                if (is_v) {
                  lo[j + e] = x;
                  hi[j + e] = y;
                } else {
                  lo[j + e] = x * cc[e] - y * ssn[e];
                  hi[j + e] = x * ssn[e] + y * cc[e];
                }
              }
            }
            auto emit = [&](const float (&v)[32], int col0) {
              uint8_t* st = stage_base + sbuf * Cfg::CHUNK_BYTES;
              if (lane == 0) tma_store_wait_read<1>();
              __syncwarp();
#pragma unroll
              for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4*>(st + stage_off<false>(lane, j)) =
                    make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                               pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmC, st, col0, row0);
                tma_store_commit();
              }
              sbuf ^= 1;
            };
            emit(lo, nb * BN + half * 128 + c * 32);
            emit(hi, nb * BN + half * 128 + (c + 2) * 32);
          }
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1;
          continue;
        }
      }
      // eight warps: chunk pairs (c, c + 2); more warps: one chunk per step
      constexpr bool PAIR = EW == 8;
      constexpr int STEP = PAIR ? 4 : PARTS;
#pragma unroll 1
      for (int c0 = half; c0 < NCH; c0 += STEP) {
        const bool two = PAIR && c0 + 2 < NCH;
        if (c0 == half) {
          if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag)) {
            fine = false;
            break;
          }
          tc_fence_after();
        }
        uint32_t r[PAIR ? 2 : 1][32];
        tmem_ld_32x32b_x32(t_row + c0 * 32, r[0]);
        if constexpr (PAIR)
          if (two) tmem_ld_32x32b_x32(t_row + (c0 + 2) * 32, r[PAIR ? 1 : 0]);
        tmem_wait_ld();
        if (c0 + STEP >= NCH) {
          // every TMEM column of this warp is in registers: release the buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(acc);
        }
#pragma unroll
        for (int h = 0; h < (PAIR ? 2 : 1); ++h) {
          if (h == 1 && !two) break;
          const int col0 = nb * BN + (c0 + 2 * h) * 32;
          float4 bq[8];  // this chunk's bias (L1-resident after the first tile)
          const float4* b4 = reinterpret_cast<const float4*>(args.bias + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) bq[j] = args.bias ? __ldg(b4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
          uint8_t* st = stage_base + sbuf * Cfg::CHUNK_BYTES;
          if (lane == 0) tma_store_wait_read<1>();
          __syncwarp();
          if constexpr (F32) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<float4*>(st + stage_off<true>(lane, j)) = make_float4(
                  __uint_as_float(r[h][4 * j]) + bq[j].x, __uint_as_float(r[h][4 * j + 1]) + bq[j].y,
                  __uint_as_float(r[h][4 * j + 2]) + bq[j].z, __uint_as_float(r[h][4 * j + 3]) + bq[j].w);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float2 x[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float4 b = bq[2 * j + (e >> 1)];
                x[e] = __fadd2_rn(make_float2(__uint_as_float(r[h][8 * j + 2 * e]),
                                              __uint_as_float(r[h][8 * j + 2 * e + 1])),
                                  (e & 1) ? make_float2(b.z, b.w) : make_float2(b.x, b.y));
                if constexpr (EPI == kEpiBf16Gelu) x[e] = gelu_as2(x[e]);
              }
              *reinterpret_cast<uint4*>(st + stage_off<false>(lane, j)) =
                  make_uint4(pack_bf16(x[0].x, x[0].y), pack_bf16(x[1].x, x[1].y),
                             pack_bf16(x[2].x, x[2].y), pack_bf16(x[3].x, x[3].y));
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, st, col0, row0);
            tma_store_commit();
          }
          sbuf ^= 1;
        }
      }
      if (!fine) {
        report(args.status, kDevTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    for (int tile = tile0; !kPaired && EPI != kEpiArgCand && tile < tend; tile += tstep) {
      const int mb = WR ? tile : tile / args.n_tiles_n, nb = WR ? wr_nb : tile % args.n_tiles_n;
      const int row0 = mb * TM + static_cast<int>(rank) * kGemmBM + quad * 32;  // first row of this warp's 32
#pragma unroll 1
      for (int c = half; c < NCH; c += PARTS) {
        const int col0 = ((EPI == kEpiBf16Swiglu || EPI == kEpiBf16GeluTanhGate) ? nb * (BN / 2) : nb * BN) + c * 32;
        // residual rows row0 + 4k + lane/8, columns col0 + (lane%8)*4 .. +3:
        // coalesced 128-byte rows, issued before the TMEM wait
        float4 res[8];
        if constexpr (EPI == kEpiF32Resid || EPI == kEpiBf16GeluTanhMul) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int r = row0 + 4 * k + (lane >> 3);
            res[k] = r < args.M
                         ? *reinterpret_cast<const float4*>(
                               args.resid + static_cast<size_t>(r) * args.ldr + col0 + (lane & 7) * 4)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
        if (c == half) {
          if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag)) {
            report(args.status, kDevTimeoutEpilogue);
            *abort_flag = 1;
            tile = args.num_tiles;  // leave both loops
            break;
          }
          tc_fence_after();
        }
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                               static_cast<uint32_t>(acc * BN);
        float v[32];
        if constexpr ((EPI == kEpiBf16Swiglu || EPI == kEpiBf16GeluTanhGate)) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_row + c * 32, g);
          tmem_ld_32x32b_x32(t_row + BN / 2 + c * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if constexpr (EPI == kEpiBf16GeluTanhGate)
              v[j] = gelu_tanh_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
            else
              v[j] = silu_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
          }
        } else {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (args.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(args.bias + col0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 b = __ldg(b4 + j);
              v[4 * j] += b.x;
              v[4 * j + 1] += b.y;
              v[4 * j + 2] += b.z;
              v[4 * j + 3] += b.w;
            }
          }
        }
        // staging buffer sbuf: the bulk store issued from it two chunks ago
        // must have finished reading it
        uint8_t* st = stage_base + sbuf * Cfg::CHUNK_BYTES;
        if (lane == 0) tma_store_wait_read<1>();
        __syncwarp();
        if constexpr (EPI == kEpiF32Resid || EPI == kEpiBf16GeluTanhMul) {
          // transpose the residual to row-per-lane through the staging chunk
#pragma unroll
          for (int k = 0; k < 8; ++k)
            *reinterpret_cast<float4*>(st + stage_off<true>(4 * k + (lane >> 3), lane & 7)) = res[k];
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 q = *reinterpret_cast<const float4*>(st + stage_off<true>(lane, j));
            if constexpr (EPI == kEpiF32Resid) {
              v[4 * j] += q.x;
              v[4 * j + 1] += q.y;
              v[4 * j + 2] += q.z;
              v[4 * j + 3] += q.w;
            } else {
              v[4 * j] = gelu_tanh_f(v[4 * j]) * q.x;
              v[4 * j + 1] = gelu_tanh_f(v[4 * j + 1]) * q.y;
              v[4 * j + 2] = gelu_tanh_f(v[4 * j + 2]) * q.z;
              v[4 * j + 3] = gelu_tanh_f(v[4 * j + 3]) * q.w;
            }
          }
          // the bf16 rows below overlap other lanes' fp32 rows of this chunk
          if constexpr (EPI == kEpiBf16GeluTanhMul) __syncwarp();
        }
        if constexpr (F32) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(st + stage_off<true>(lane, j)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float x[8];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              float2 xx = make_float2(v[8 * j + e], v[8 * j + e + 1]);
              if constexpr (EPI == kEpiBf16Gelu) xx = gelu_as2(xx);
              x[e] = xx.x;
              x[e + 1] = xx.y;
            }
            *reinterpret_cast<uint4*>(st + stage_off<false>(lane, j)) =
                make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]),
                           pack_bf16(x[6], x[7]));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, st, col0, row0);
          tma_store_commit();
        }
        sbuf ^= 1;
        if (c + PARTS >= NCH) {
          // last chunk of this warp in the tile: hand the accumulator back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(acc);
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) tma_store_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag) {
    // let copies and MMAs already in flight land before the CTA exits
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 2000000ull) {
    }
  }
  if constexpr (CG == 2) cluster_sync_all();  // neither CTA leaves while the pair MMAs run
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2) tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace ec
