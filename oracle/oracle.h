/* oracle.h -- CPU restatement of lisp-embed's embedding and IVF arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: tests/, the smoke
 * entry point and bench.py's CPU-baseline leg load it to compute expected
 * values.  The product path (libembedcuda.so) never links or calls it.
 *
 * Parity status: UNPINNED by the reference.  The reference (pure SBCL Lisp)
 * ships no tests, fixtures or golden vectors for this path and SBCL is not
 * available to run it, so this file restates the Lisp function by function,
 * in the same loop and accumulation order, single-float except where the Lisp
 * uses double.  It is cross-checked against HF transformers on CPU
 * (tests/test_oracle.py) as a secondary check.
 *
 * Float semantics follow SBCL on x86-64:
 *   - single-float + - * / are IEEE binary32 ops, never contracted to FMA
 *     (build with -ffp-contract=off, no -ffast-math);
 *   - (exp x), (log x), (sqrt x) on a single-float are computed in double and
 *     rounded to single (SBCL's irrational.lisp dispatch), so we use
 *     (float)exp((double)x) and friends;
 *   - (* a b c) associates left: (a*b)*c.
 */
#ifndef EC_ORACLE_H
#define EC_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- BERT / RoBERTa / MPNet (bert.lisp) ---------------------------------- */
typedef struct {
  /* BERT names (bert.lisp:96-127); MPNet maps attn.o -> ao_*, attention
   * LayerNorm -> ao_g/ao_b2 (bert.lisp:356-387). */
  const float *q_w, *q_b, *k_w, *k_b, *v_w, *v_b;
  const float *ao_w, *ao_b, *ao_g, *ao_b2;
  const float *ff_w, *ff_b, *o_w, *o_b, *o_g, *o_b2;
} or_bert_layer;

typedef struct {
  int hidden, layers, heads, head_dim, inter;
  int pooling;     /* 0 = :cls, 1 = :mean */
  int mpnet;       /* 1 = embed-mpnet / mpnet-layer path */
  int pos_offset;  /* 2 for roberta, 0 for bert (bert.lisp:294) */
  int causal;      /* bert::*causal* */
  const float *w_word, *w_pos, *w_type; /* w_type: row 0 used; NULL -> zeros */
  const float *emb_g, *emb_b;
  const float *rel_bias;                /* MPNet [32 * heads] */
  const or_bert_layer *L;
} or_bert;

int or_bert_embed(const or_bert *m, const int32_t *ids, int seq, float *out);
int or_mpnet_bucket(int i, int j);

/* ---- Llama / Qwen3 (llama.lisp) ------------------------------------------ */
typedef struct {
  const float *in_ln, *post_ln, *q_w, *k_w, *v_w, *o_w;
  const float *q_norm, *k_norm; /* NULL when absent (get-tensor-opt) */
  const float *gate, *up, *down;
} or_llama_layer;

typedef struct {
  int hidden, layers, heads, kv_heads, head_dim, inter;
  int pooling;     /* 0 = :last, 1 = :mean */
  int max_pos;     /* llama::*max-pos* (1024) */
  double rope_theta, eps;
  const float *w_embed, *w_norm;
  const or_llama_layer *L;
} or_llama;

int or_llama_embed(const or_llama *m, const int32_t *ids, int seq, float *out);

/* ---- EmbeddingGemma / Gemma-3n text (gemma.lisp) ------------------------- */
typedef struct {
  int head_dim, kv_heads;
  double rope_theta;   /* 1e6 for full_attention layers, 1e4 otherwise */
  const float *in_ln, *post_ln, *pre_ff_ln, *post_ff_ln;
  const float *q_w, *k_w, *v_w, *o_w, *q_norm, *k_norm;
  const float *gate, *up, *down;
  const float *ple_gate, *ple_proj, *ple_norm;
  float scalar;
} or_gemma_layer;

typedef struct {
  int hidden, layers, heads, inter, ple_dim, out_dim;
  int max_pos;         /* gemma::*max-pos* (2048) */
  double eps;
  const float *w_embed, *w_ple_proj, *w_ple_norm, *w_norm, *w_out;
  const or_gemma_layer *L;
} or_gemma;

int or_gemma_embed(const or_gemma *m, const int32_t *ids, int seq, float *out);

/* Threads one sequence's forward may split its token and head loops over
 * (default 1, the reference's one thread per sequence).  Results do not
 * depend on it: each token row or head is computed by the same code. */
void or_set_seq_threads(int n);

/* Batch driver mirroring embed.lisp:88-105: batches of `threads` sequences,
 * one thread per sequence, joined in input order.  kind 0 = bert, 1 = llama,
 * 2 = gemma. */
int or_embed_batch(int kind, const void *model, const int32_t *ids,
                   const int64_t *offsets, int nseq, int dim, float *out,
                   int threads);

/* ---- safetensors widening (st.lisp) -------------------------------------- */
void or_bf16_to_f32(const uint16_t *src, float *dst, int64_t n);
void or_f16_to_f32(const uint16_t *src, float *dst, int64_t n);

/* ---- IVF (ann.lisp, kb.lisp) --------------------------------------------- */
float or_dot(const float *a, const float *b, int n);
int32_t or_nearest_centroid(const float *x, const float *cent, int k, int dim);
void or_assign(const float *vecs, const int64_t *rows, int64_t nrows,
               const float *cent, int k, int dim, int32_t *assign, int threads);
/* the same results one row and one centroid at a time, as ann.lisp's loop
 * runs (or_assign interleaves sixteen %dot chains for speed) */
void or_assign_scalar(const float *vecs, const int64_t *rows, int64_t nrows,
                      const float *cent, int k, int dim, int32_t *assign, int threads);
/* one Lloyd update given assignments (ann.lisp:107-122); cent in/out */
void or_kmeans_update(const float *vecs, const int64_t *sample, int64_t ns,
                      const int32_t *assign, int k, int dim, float *cent);
/* full kmeans (ann.lisp:79-125) */
void or_kmeans(const float *vecs, const int64_t *sample, int64_t ns, int k,
               int dim, int iters, float *cent, int threads);
/* assign-all (ann.lisp:127-158) */
void or_assign_all(const float *vecs, int64_t n, const float *cent, int k,
                   int dim, uint32_t *counts, uint32_t *lists, int threads);
/* kb::top-k-ivf (kb.lisp:348-364); returns number of results (<= topk) */
int or_top_k_ivf(const float *vecs, int dim, const float *cent, int k,
                 const uint32_t *counts, const uint32_t *lists, int nprobe,
                 const float *q, int topk, int64_t *ids, float *scores);
/* kb::top-k-brute (kb.lisp:186-200) */
int or_top_k_brute(const float *vecs, int64_t n, int dim, const float *q,
                   int topk, int threads, int64_t *ids, float *scores);

#ifdef __cplusplus
}
#endif
#endif
