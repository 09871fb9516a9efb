// ec_kernels.h -- host-side launchers of the sm_100a kernels and their
// argument blocks.  Each .cu file instantiates its kernels and exposes only
// these plain functions, so the host code (ec_api.cu) never sees a template.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ec {

// Programmatic dependent launch for the chains of small row / skinny /
// attention kernels: a kernel launched by launch_pdl may be scheduled while
// its predecessor in the stream drains, so it calls pdl_wait() before it
// reads or writes anything that kernel touches (the wait returns once the
// predecessor grid has completed and its writes are visible; without the
// launch attribute it returns at once), and pdl_trigger() early so that its
// own successor can be scheduled.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif
bool pdl_enabled();            // EC_NO_PDL turns it off; per thread, see pdl_set_thread
void pdl_set_thread(bool on);  // this thread's launches (a graph capture turns it off)

template <class... P, class... A>
cudaError_t launch_pdl(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<A&&>(args)...);
}

enum DtKind : int { kDtF32 = 0, kDtBf16 = 1 };
enum ConvKind : int { kConvF16ToF32 = 0, kConvBf16ToF32 = 1, kConvF32ToBf16 = 2 };

struct EmbedLnArgs {
  const int* ids;
  const int* pos;       // position of each token inside its sequence
  int pos_offset;       // 2 for roberta and mpnet, else 0
  const void* word;     // [vocab, H]
  int word_dtype;
  const void* posemb;   // [max_pos, H]
  int pos_dtype;
  const void* type0;    // row 0 of token_type_embeddings or nullptr
  int type_dtype;
  const float* g;
  const float* b;
  float* out32;         // [T, H]
  __nv_bfloat16* outb;  // [T, H]
  int T, H;
};

struct LnArgs {
  const float* x;       // [T, H]
  const float* g;
  const float* b;
  float* out32;         // may alias x
  __nv_bfloat16* outb;
  int T, H;
};

struct RmsArgs {
  const float* x;       // [*, H]
  const int* rows;      // optional row gather (nullptr = identity)
  const float* g;
  double eps;
  __nv_bfloat16* outb;  // [T, H] or nullptr
  float* out32;         // [T, H] or nullptr
  int T, H;
};

struct QkRopeArgs {
  __nv_bfloat16* qkv;
  int ld;
  int q_off, k_off;
  int q_heads, k_heads;  // head_dim is 128
  const float* q_norm;   // [128] or nullptr
  const float* k_norm;
  double eps;
  const int* pos;
  const float* cos_t;    // [max_pos, 64]
  const float* sin_t;
  int T;
};

struct PoolArgs {
  const float* h;       // [T, H] fp32
  const int* cu;        // [nseq + 1]
  int mode;             // 0 first, 1 mean, 2 last
  int final_norm;       // llama final RMSNorm on pooled tokens
  const float* norm_w;
  double eps;
  float* out;
  int out_stride;
  int H;
};

// ---- EmbeddingGemma rows (ec_gemma.cu) ---------------------------------------
struct GemmaEmbedArgs {
  const int* ids;
  const void* table;
  int dtype;
  float scale;          // sqrt(hidden) as a single-float
  float* h32;           // [T, H]
  __nv_bfloat16* h0b;   // [T, H] bf16 copy
  int T, H;
};
struct HeadNormRopeArgs {
  __nv_bfloat16* qkv;   // [T, ld] packed q | k | v heads
  int ld;
  int q_heads, kv_heads, hd;
  const float* q_norm;
  const float* k_norm;
  double eps;
  const int* pos;
  const float* cos_t;   // [max_pos, hd / 2]
  const float* sin_t;
  int T;
};
struct NormAddArgs {
  const float* x;       // [T, H] sub-block output
  const float* g1;      // its RMSNorm weight
  float* h32;           // residual stream, updated in place
  int scale_h;          // multiply h by `scalar` after the add
  float scalar;
  const float* g2;      // RMSNorm weight for hb, or nullptr (hb = bf16(h))
  __nv_bfloat16* outb;  // [T, H] or nullptr
  double eps;
  int T, H;
};
struct PlePrepArgs {
  float* x;             // [T, P], in place
  float inv_sqrt_h;
  const float* g;
  double eps;
  int T, P;
};
struct PleGateArgs {
  const float* gate;    // [T, P]
  const float* ple;     // [T, P]
  __nv_bfloat16* outb;  // [T, P]
  int T, P;
};
struct GemmaPoolArgs {
  const float* h;       // [T, H] after the final RMSNorm
  const int* cu;        // [nseq + 1]
  const float* w_out;   // [out_dim, H]
  float* out;
  int out_stride;
  int H, out_dim;
};
cudaError_t launch_gemma_embed(const GemmaEmbedArgs& a, cudaStream_t st);
cudaError_t launch_head_norm_rope(const HeadNormRopeArgs& a, cudaStream_t st);
cudaError_t launch_norm_add(const NormAddArgs& a, cudaStream_t st);
cudaError_t launch_ple_prep(const PlePrepArgs& a, cudaStream_t st);
cudaError_t launch_ple_gate(const PleGateArgs& a, cudaStream_t st);
cudaError_t launch_gemma_pool(const GemmaPoolArgs& a, int nseq, cudaStream_t st);

cudaError_t launch_embed_ln(const EmbedLnArgs& a, cudaStream_t st);
cudaError_t launch_ln(const LnArgs& a, cudaStream_t st);
cudaError_t launch_rmsnorm(const RmsArgs& a, cudaStream_t st);
cudaError_t launch_qk_norm_rope(const QkRopeArgs& a, cudaStream_t st);
cudaError_t launch_pool_l2(const PoolArgs& a, int nseq, cudaStream_t st);
cudaError_t launch_gather_rows(const void* table, int dtype, const int* ids, float* out, int T,
                               int H, cudaStream_t st);
cudaError_t launch_positions(const int* cu, int nseq, int* pos, cudaStream_t st);
cudaError_t launch_convert(int kind, const void* src, void* dst, size_t n, cudaStream_t st);

// ---- GEMM (ec_gemm.cu) -------------------------------------------------------
// C[M, N] = A[M, K] . W[N, K]^T with epilogue `epi` (GemmEpi in ec_gemm.cuh:
// 0 bf16, 1 bf16+gelu, 2 f32+resid, 3 bf16 swiglu, 4 f32, 5 bf16 with head
// norms + RoPE, 6 bf16 gelu-tanh gate, 7 bf16 gelu-tanh * multiplier).  A and W bf16,
// K-major; K % 64 == 0; N % bn == 0.  `bn` 0 = pick automatically.
struct QkRopeEpi;   // ec_gemm.cuh
struct ArgCandEpi;  // ec_gemm.cuh
struct GemmLaunch {
  const __nv_bfloat16* A;
  int lda;              // elements
  const __nv_bfloat16* W;
  int ldw;
  int M, N, K;
  const float* bias;
  const float* resid;
  int ldr;
  void* out;
  int ldo;
  int epi;
  int bn;
  unsigned* status;
  const QkRopeEpi* qk = nullptr;  // kEpiBf16QkRope (5)
  const ArgCandEpi* ac = nullptr; // kEpiArgCand (8)
};
int gemm_pick_bn(int M, int N, int epi, int num_sms);
cudaError_t launch_gemm(const GemmLaunch& g, cudaStream_t st, int num_sms);
// encode function for TMA descriptors (driver entry point), set once
bool gemm_init_driver();

// ---- GEMM + bias + residual + LayerNorm (ec_gemm_ln.cuh) ---------------------
// out32 = LN(A . W^T + bias + resid) * g + b (fp32, may alias resid) and
// outb = bf16(out32); whole rows of N in {384, 768, 1024} per CTA cluster.
struct GemmLnLaunch {
  const __nv_bfloat16* A;
  int lda;
  const __nv_bfloat16* W;  // [N, K]
  int M, N, K;
  const float* bias;
  const float* resid;      // [M, N] fp32 residual, or
  const float* ln_g;
  const float* ln_b;
  float* out32;            // [M, N] or nullptr (no fp32 output)
  __nv_bfloat16* outb;     // [M, N]
  unsigned* status;
  const __nv_bfloat16* resid_b = nullptr;  // [M, N] bf16 residual (replaces resid)
  // epilogue (GemmNorm in ec_gemm_ln.cuh): 0 LayerNorm (ln_g, ln_b); RMS
  // modes with eps: 1 out32 = x + resid, outb = RMSNorm(out32) * ln_g;
  // 2 out32 = (resid + RMSNorm(x) * ln_g) [* scale when has_scale], outb =
  // RMSNorm(out32) * ln_b (ln_b nullptr: bf16(out32)); 3 out32 =
  // RMSNorm(x * scale) * ln_g (outb may be nullptr)
  int mode = 0;
  float eps = 0.f;
  float scale = 1.f;
  int has_scale = 0;
};
bool gemm_ln_supported(int N);
bool gemm_rms_supported(int N);
cudaError_t launch_gemm_ln(const GemmLnLaunch& g, cudaStream_t st, int num_sms);

// ---- fused feed-forward block (ec_mlp.cu) -------------------------------------
// out = LayerNorm(W2 . gelu(W1 . A + b1) + b2 + resid) for H in {128, 256, 384},
// F % 128 == 0; writes the fp32 row (out32, may alias resid) and its bf16
// copy (outb, may alias A).
struct MlpLaunch {
  const __nv_bfloat16* A;   // [M, H]
  const __nv_bfloat16* W1;  // [F, H]
  const __nv_bfloat16* W2;  // [H, F]
  const float* b1;
  const float* b2;
  const float* resid;       // [M, H] fp32, or nullptr: the residual is A itself
  const float* ln_g;
  const float* ln_b;
  float* out32;             // [M, H] or nullptr (no fp32 row)
  __nv_bfloat16* outb;      // [M, H] (may alias A)
  int M, H, F;
  unsigned* status;
};
bool mlp_supported(int H, int F);

// GEMMs of at most kSkinnyRows rows (ec_skinny.cu): out[m, n] =
// epilogue(A[m, :] . W[n, :] + bias[n]), one warp per output column
constexpr int kSkinnyRows = 16;
enum SkinnyEpi : int {
  kSkBf16 = 0,      // bf16 out = acc + bias
  kSkGelu = 1,      // bf16 out = gelu(acc + bias)
  kSkF32Resid = 2,  // fp32 out = (acc + bias) + resid (resid fp32, else resid_b bf16)
};
struct SkinnyLaunch {
  const __nv_bfloat16* A;  // [M, lda]
  int lda;
  const __nv_bfloat16* W;  // [N, K]
  int M, N, K;
  const float* bias;              // [N] or nullptr
  const float* resid;             // [M, ldr] or nullptr
  const __nv_bfloat16* resid_b;   // [M, ldr] when resid is nullptr
  int ldr;
  void* out;                      // [M, ldo]
  int ldo;
  int epi;
};
cudaError_t launch_skinny_gemm(const SkinnyLaunch& s, cudaStream_t st);
cudaError_t launch_mlp(const MlpLaunch& l, cudaStream_t st, int num_sms);

// ---- attention (ec_attn.cu) --------------------------------------------------
struct AttnLaunch {
  const __nv_bfloat16* qkv;
  int ld;
  int q_off, k_off, v_off;
  __nv_bfloat16* out;
  int ldo;
  const int* cu;
  const int2* blocks;
  int nblocks;
  int heads, kv_group, head_dim;
  int causal;
  const float* relbias;  // [heads][2 * rel_max - 1], pre-scaled by log2(e)
  int rel_max;
  const int4* blocks128; // (first token, length, first query row, 0) per 128-row block, long first
  int nblocks128;
  int rows;              // packed token rows in qkv (T)
  unsigned* status;
  int num_sms;
  // per sequence (first token, length), longest first; sequences [0, n_long)
  // are longer than the short-sequence kernel's key capacity and own the
  // first nblocks128_long entries of blocks128
  const int2* seqs;
  int nseq;
  int n_long;
  int nblocks128_long;
  int max_short_len;     // longest sequence in [n_long, nseq)
  // [n_long, nseq) cut where the length falls to 192 / 128 / 64 or below:
  // bucket b is [bucket_first[b], bucket_first[b + 1]) with its longest
  // sequence bucket_max[b] (nbuckets 0: one launch over the whole range)
  int nbuckets = 0;
  int bucket_first[5] = {0, 0, 0, 0, 0};
  int bucket_max[4] = {0, 0, 0, 0};
  int n_gt128 = 0;       // sequences of [n_long, nseq) longer than 128 tokens
  float scale = 0.f;     // logit scale; 0 = 1 / sqrt(head_dim) (Gemma uses 1.0)
};
// key capacity of the short-sequence attention kernel (ec_attn_short.cuh)
constexpr int kAttnShortCap = 256;
// fill AttnLaunch's length buckets from the sequence lengths in launch
// order (descending), sequences [n_long, nseq)
void attn_short_buckets(const int* lens_sorted, int n_long, int nseq, AttnLaunch* a);
// tcgen05 kernel (ec_fa.cuh) for head_dim 32 / 64 / 128; the mma.sync kernel
// (ec_attn.cuh) when EC_LEGACY_ATTN is set
cudaError_t launch_attention(const AttnLaunch& a, cudaStream_t st);

}  // namespace ec
