/* embedcuda_debug.h -- kernel-level test hooks of libembedcuda.so.
 *
 * Not part of the reference-facing interface (no reference counterpart):
 * they let the test suite check a single kernel against a PyTorch fp32
 * reference.  All pointers are device pointers on the library's device 0.
 */
#ifndef EMBEDCUDA_DEBUG_H
#define EMBEDCUDA_DEBUG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out = epilogue(A[M, K] . W[N, K]^T), A and W bf16 row-major.
 * epi: 0 bf16 (+bias), 1 bf16 gelu(+bias), 2 f32 (+bias) + resid,
 *      3 bf16 swiglu over 2 x (bn/2)-column gate/up blocks, 4 f32 (+bias).
 * bn: tile width (64, 128, 192, 256) or 0 for automatic. */
int ecdbg_gemm(const void *A, const void *W, int M, int N, int K, const float *bias,
               const float *resid, void *out, int epi, int bn);

/* Fused feed-forward block: out = LayerNorm(W2 . gelu(W1 . A + b1) + b2 +
 * resid), A bf16 [M, H], W1 bf16 [F, H], W2 bf16 [H, F], vectors fp32;
 * writes out32 fp32 [M, H] and outb bf16 [M, H].  H in {128, 256, 384}. */
int ecdbg_mlp(const void *A, const void *W1, const void *W2, const float *b1, const float *b2,
              const float *resid, const float *ln_g, const float *ln_b, float *out32,
              void *outb, int M, int H, int F);

/* GEMM + bias + residual + LayerNorm: out32 = LN(A . W^T + bias + resid) * g
 * + b (fp32 [M, N], may alias resid) and outb = bf16 of it; A bf16 [M, K],
 * W bf16 [N, K]; N in {384, 768, 1024} (one row per CTA cluster). */
int ecdbg_gemm_ln(const void *A, const void *W, int M, int N, int K, const float *bias,
                  const float *resid, const float *ln_g, const float *ln_b, float *out32,
                  void *outb);
/* The same cluster GEMM with an RMSNorm epilogue (x = A . W^T, fp32 rows):
 * mode 1: out32 = x + resid, outb = RMSNorm(out32) * g1;
 * mode 2: out32 = (resid + RMSNorm(x) * g1) [* scale when has_scale],
 *         outb = RMSNorm(out32) * g2, or bf16(out32) when g2 is NULL;
 * mode 3: out32 = RMSNorm(x * scale) * g1 (outb may be NULL).
 * RMSNorm(v) = v / sqrt(mean(v^2) + eps).  N in {512, 768, 1024}. */
int ecdbg_gemm_norm(const void *A, const void *W, int M, int N, int K, const float *resid,
                    const float *g1, const float *g2, float *out32, void *outb, int mode,
                    float eps, float scale, int has_scale);

/* Varlen attention over packed bf16 rows qkv[T, ld]; cu[nseq + 1] (device,
 * int32) token offsets; lens on the host.  out[T, heads * head_dim] bf16. */
int ecdbg_attention(const void *qkv, int ld, int q_off, int k_off, int v_off, void *out,
                    const int32_t *cu_dev, const int32_t *lens_host, int nseq, int heads,
                    int kv_heads, int head_dim, int causal);

/* Per-kernel-class device timing of the embedding forward, for the
 * benchmark's roofline figures.  ecdbg_profile(1) clears the counters and
 * brackets every later launch with CUDA events on its stream; (0) stops.
 * ecdbg_profile_read fills the summed event time (ms), algorithmic FLOPs and
 * bytes and the launch count of class `cls` ("gemm", "attention", "rows"). */
int ecdbg_profile(int enable);
int ecdbg_profile_read(const char *cls, double *ms, double *flops, double *bytes,
                       long long *launches);
/* Kernel launches issued by the library since the last ecdbg_profile(1). */
long long ecdbg_launches(void);
/* Rows assigned by the tensor-core path of ec_kmeans / ec_assign /
 * ec_assign_all (scores re-checked exactly) and rows that took the exact
 * single-float scan, since the last reset; reset != 0 clears them. */
int ecdbg_assign_rows(long long *tc_rows, long long *exact_rows, int reset);

/* binaryVersion / ptxVersion (major * 10 + minor) of the library's device
 * code as the CUDA runtime loaded it on the current device: 100 for sm_100. */
int ecdbg_kernel_arch(int *binary_version, int *ptx_version);

/* Copy the device copy of an uploaded tensor (device 0) to host memory, as
 * stored after ec_upload_tensor: F32 and F16 uploads as f32 (F16 widened on
 * the device), BF16 as bf16.  nbytes must equal the stored size; *dtype
 * receives EC_F32 or EC_BF16. */
int ecdbg_tensor_read(const char *name, void *host, size_t nbytes, int *dtype);

/* Failure-path check of the bounded waits: launches one CTA that waits on an
 * mbarrier no thread arrives on, with a limit of `limit_ms` milliseconds.
 * The wait gives up, the kernel records a status and exits, and the call
 * returns EC_ETIMEOUT with the context still usable. */
int ecdbg_wait_timeout(int limit_ms);

#ifdef __cplusplus
}
#endif
#endif
