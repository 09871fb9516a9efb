/* oracle.c -- CPU restatement of lisp-embed's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product).  Parity is
 * UNPINNED by the reference: it has no tests or golden vectors and SBCL is
 * not available; every function below restates the cited Lisp in the same
 * operation order.  See oracle.h for the float-semantics rules.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* SBCL computes exp/log/sqrt of a single-float in double and rounds. */
static inline float sexp(float x) { return (float)exp((double)x); }
static inline float slog(float x) { return (float)log((double)x); }
static inline float ssqrt(float x) { return (float)sqrt((double)x); }

/* ---- intra-sequence parallel loops --------------------------------------
 * or_set_seq_threads(n) lets one sequence's forward split its loops over
 * tokens and over heads between n threads.  Every value is still computed
 * by the same sequential code (each token row or head is one task), so the
 * results do not depend on n; 1, the default, keeps the reference's one
 * thread per sequence. */
static int g_seq_threads = 1;
void or_set_seq_threads(int n) { g_seq_threads = n < 1 ? 1 : n; }

typedef void (*par_body)(void *ctx, int i);
typedef struct {
  par_body fn;
  void *ctx;
  int n;
  int next;
  pthread_mutex_t mu;
} par_job;

static void *par_worker(void *arg) {
  par_job *j = (par_job *)arg;
  for (;;) {
    pthread_mutex_lock(&j->mu);
    const int i = j->next++;
    pthread_mutex_unlock(&j->mu);
    if (i >= j->n) return NULL;
    j->fn(j->ctx, i);
  }
}

/* fn(ctx, i) for i in [0, n): on the calling thread alone, or on up to
 * g_seq_threads threads taking indices in turn */
static void par_for(int n, par_body fn, void *ctx) {
  int nt = g_seq_threads < n ? g_seq_threads : n;
  if (nt <= 1) {
    for (int i = 0; i < n; ++i) fn(ctx, i);
    return;
  }
  par_job j = {fn, ctx, n, 0, PTHREAD_MUTEX_INITIALIZER};
  pthread_t tid[256];
  if (nt > 256) nt = 256;
  int started = 0;
  for (int t = 1; t < nt; ++t)
    if (pthread_create(&tid[started], NULL, par_worker, &j) == 0) ++started;
  par_worker(&j);
  for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
}

/* %dot (bert.lisp:133-143, llama.lisp:86-95, ann.lisp:25-35, kb.lisp:153-162):
 * sequential single-float sum of products. */
float or_dot(const float *a, const float *b, int n) {
  float s = 0.0f;
  for (int k = 0; k < n; ++k) s = s + a[k] * b[k];
  return s;
}

/* bert::linear (bert.lisp:145-153): y[o] = b[o] + dot(x, W[o,:]). */
static void linear_b(const float *x, const float *w, const float *b, float *y,
                     int in_dim, int out_dim) {
  for (int o = 0; o < out_dim; ++o)
    y[o] = b[o] + or_dot(x, w + (size_t)o * in_dim, in_dim);
}

/* llama::linear (llama.lisp:97-104): no bias. */
static void linear_nb(const float *x, const float *w, float *y, int in_dim,
                      int out_dim) {
  for (int o = 0; o < out_dim; ++o)
    y[o] = or_dot(x, w + (size_t)o * in_dim, in_dim);
}

/* bert::layernorm (bert.lisp:155-174): std = sqrt(var) + 1e-12. */
static void layernorm(float *x, int n, const float *g, const float *b) {
  float mean = 0.0f, var = 0.0f;
  for (int i = 0; i < n; ++i) mean = mean + x[i];
  mean = mean / (float)n;
  for (int i = 0; i < n; ++i) {
    float d = x[i] - mean;
    var = var + d * d;
  }
  var = var / (float)n;
  float std = ssqrt(var) + 1e-12f;
  for (int i = 0; i < n; ++i) x[i] = ((x[i] - mean) / std) * g[i] + b[i];
}

/* bert::erf-approx (bert.lisp:176-188), Abramowitz-Stegun 7.1.26. */
static float erf_approx(float x) {
  float ax = fabsf(x);
  float t1 = 1.0f / (1.0f + 0.3275911f * ax);
  float poly =
      t1 * (0.254829592f +
            t1 * (-0.284496736f +
                  t1 * (1.421413741f + t1 * (-1.453152027f + t1 * 1.061405429f))));
  float erf_pos = 1.0f - poly * sexp(-(ax * ax));
  float sign = (x < 0.0f) ? -1.0f : 1.0f;
  return sign * erf_pos;
}

/* bert::gelu (bert.lisp:190-192). */
static float gelu(float x) {
  return (0.5f * x) * (1.0f + erf_approx(x / ssqrt(2.0f)));
}

/* bert::softmax / llama::softmax (bert.lisp:194-210, llama.lisp:153-168). */
static void softmax(float *a, int n) {
  float maxv = -FLT_MAX;
  for (int i = 0; i < n; ++i) maxv = (a[i] > maxv) ? a[i] : maxv;
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    float e = sexp(a[i] - maxv);
    a[i] = e;
    sum = sum + e;
  }
  for (int i = 0; i < n; ++i) a[i] = a[i] / sum;
}

/* bert::mpnet-bucket (bert.lisp:324-331). */
int or_mpnet_bucket(int i, int j) {
  int n = i - j;
  int an = n < 0 ? -n : n;
  int ret = n < 0 ? 16 : 0;
  if (an < 8) return ret + an;
  float v = 8.0f + 8.0f * (slog((float)an / 8.0f) / slog(16.0f));
  int f = (int)floorf(v);
  return ret + (f < 15 ? f : 15);
}

/* Shared state of one BERT / MPNet forward, for the parallel loop bodies. */
typedef struct {
  const or_bert *m;
  const or_bert_layer *lw;
  int seq;
  float *h, *tmp, *ctx, *qb, *kb, *vb, *normed, *scores, *ff;
} bert_state;

/* Shared attention body for bert::encoder-layer (bert.lisp:226-248) and
 * bert::mpnet-layer (bert.lisp:408-423): one head per task, each with its
 * own seq x seq score block. */
static void bert_attention_head(void *arg, int hh) {
  const bert_state *S = (const bert_state *)arg;
  const or_bert *m = S->m;
  const int H = m->hidden, hd = m->head_dim, seq = S->seq;
  const float *q = S->qb, *k = S->kb, *v = S->vb;
  float *ctx = S->ctx, *scores = S->scores + (size_t)hh * seq * seq;
  const float sqrt_hd = ssqrt((float)hd);
  for (int t1 = 0; t1 < seq; ++t1) {
    for (int t2 = 0; t2 < seq; ++t2) {
      float s;
      if (m->mpnet) {
        s = or_dot(q + (size_t)t1 * H + hh * hd, k + (size_t)t2 * H + hh * hd, hd) / sqrt_hd +
            m->rel_bias[or_mpnet_bucket(t1, t2) * m->heads + hh];
      } else if (m->causal && t2 > t1) {
        s = -1e9f;
      } else {
        s = or_dot(q + (size_t)t1 * H + hh * hd, k + (size_t)t2 * H + hh * hd, hd) / sqrt_hd;
      }
      scores[(size_t)t1 * seq + t2] = s;
    }
    if (m->mpnet) softmax(scores + (size_t)t1 * seq, seq);
  }
  if (!m->mpnet)
    for (int t1 = 0; t1 < seq; ++t1) softmax(scores + (size_t)t1 * seq, seq);
  for (int t1 = 0; t1 < seq; ++t1)
    for (int i = 0; i < hd; ++i) {
      float acc = 0.0f;
      for (int t2 = 0; t2 < seq; ++t2)
        acc = acc + scores[(size_t)t1 * seq + t2] * v[(size_t)t2 * H + hh * hd + i];
      ctx[(size_t)t1 * H + hh * hd + i] = acc;
    }
}

/* q, k, v projections of token t (bert.lisp:220-225) */
static void bert_qkv_tok(void *arg, int t) {
  const bert_state *S = (const bert_state *)arg;
  const int H = S->m->hidden;
  const or_bert_layer *lw = S->lw;
  linear_b(S->h + (size_t)t * H, lw->q_w, lw->q_b, S->qb + (size_t)t * H, H, H);
  linear_b(S->h + (size_t)t * H, lw->k_w, lw->k_b, S->kb + (size_t)t * H, H, H);
  linear_b(S->h + (size_t)t * H, lw->v_w, lw->v_b, S->vb + (size_t)t * H, H, H);
}

/* encoder-layer (bert.lisp:250-258): output projection + residual + LN */
static void bert_ao_tok(void *arg, int t) {
  const bert_state *S = (const bert_state *)arg;
  const int H = S->m->hidden;
  const or_bert_layer *lw = S->lw;
  float *tr = S->tmp + (size_t)t * H;
  linear_b(S->ctx + (size_t)t * H, lw->ao_w, lw->ao_b, tr, H, H);
  for (int i = 0; i < H; ++i) tr[i] = tr[i] + S->h[(size_t)t * H + i];
  layernorm(tr, H, lw->ao_g, lw->ao_b2);
}

/* encoder-layer (bert.lisp:259-271): GELU FFN + residual + LN into h */
static void bert_ffn_tok(void *arg, int t) {
  const bert_state *S = (const bert_state *)arg;
  const int H = S->m->hidden, F = S->m->inter;
  const or_bert_layer *lw = S->lw;
  float *f = S->ff + (size_t)t * F; /* a fresh per-token array in the Lisp */
  float *hr = S->h + (size_t)t * H;
  linear_b(S->tmp + (size_t)t * H, lw->ff_w, lw->ff_b, f, H, F);
  for (int i = 0; i < F; ++i) f[i] = gelu(f[i]);
  linear_b(f, lw->o_w, lw->o_b, hr, F, H);
  for (int i = 0; i < H; ++i) hr[i] = hr[i] + S->tmp[(size_t)t * H + i];
  layernorm(hr, H, lw->o_g, lw->o_b2);
}

/* mpnet-layer (bert.lisp:424-437): output projection, residual + LN, FFN in */
static void mpnet_ao_ff1_tok(void *arg, int t) {
  const bert_state *S = (const bert_state *)arg;
  const int H = S->m->hidden, F = S->m->inter;
  const or_bert_layer *lw = S->lw;
  linear_b(S->ctx + (size_t)t * H, lw->ao_w, lw->ao_b, S->tmp + (size_t)t * H, H, H);
  float *nr = S->normed + (size_t)t * H;
  for (int i = 0; i < H; ++i) nr[i] = S->tmp[(size_t)t * H + i] + S->h[(size_t)t * H + i];
  layernorm(nr, H, lw->ao_g, lw->ao_b2);
  float *f = S->ff + (size_t)t * F;
  linear_b(nr, lw->ff_w, lw->ff_b, f, H, F);
  for (int i = 0; i < F; ++i) f[i] = gelu(f[i]);
}

/* mpnet-layer (bert.lisp:438-452): FFN out, residual + LN into h */
static void mpnet_ff2_tok(void *arg, int t) {
  const bert_state *S = (const bert_state *)arg;
  const int H = S->m->hidden, F = S->m->inter;
  const or_bert_layer *lw = S->lw;
  float *tr = S->tmp + (size_t)t * H;
  linear_b(S->ff + (size_t)t * F, lw->o_w, lw->o_b, tr, F, H);
  for (int i = 0; i < H; ++i) tr[i] = tr[i] + S->normed[(size_t)t * H + i];
  layernorm(tr, H, lw->o_g, lw->o_b2);
  memcpy(S->h + (size_t)t * H, tr, H * sizeof(float));
}

/* bert::embed-bert (bert.lisp:275-320) and bert::embed-mpnet (:455-499). */
int or_bert_embed(const or_bert *m, const int32_t *ids, int seq, float *out) {
  const int H = m->hidden, F = m->inter;
  size_t sh = (size_t)seq * H;
  float *h = malloc(sh * sizeof(float));
  float *tmp = malloc(sh * sizeof(float));
  float *ctx = malloc(sh * sizeof(float));
  float *qb = malloc(sh * sizeof(float));
  float *kb = malloc(sh * sizeof(float));
  float *vb = malloc(sh * sizeof(float));
  float *normed = malloc(sh * sizeof(float));
  float *scores = malloc((size_t)m->heads * seq * seq * sizeof(float));
  float *ff = malloc((size_t)seq * F * sizeof(float));
  if (!h || !tmp || !ctx || !qb || !kb || !vb || !normed || !scores || !ff) {
    free(h); free(tmp); free(ctx); free(qb); free(kb); free(vb);
    free(normed); free(scores); free(ff);
    return -1;
  }
  /* embeddings (bert.lisp:290-298; mpnet :473-479) */
  for (int t = 0; t < seq; ++t) {
    const float *wr = m->w_word + (size_t)ids[t] * H;
    /* position ids: t (+2 for roberta, bert.lisp:294); MPNet t+2 (:477) */
    const float *pr = m->w_pos + (size_t)(t + (m->mpnet ? 2 : m->pos_offset)) * H;
    for (int i = 0; i < H; ++i) {
      if (m->mpnet) {
        h[(size_t)t * H + i] = wr[i] + pr[i];
      } else {
        float ty = m->w_type ? m->w_type[i] : 0.0f;
        h[(size_t)t * H + i] = (wr[i] + pr[i]) + ty;
      }
    }
  }
  for (int t = 0; t < seq; ++t) layernorm(h + (size_t)t * H, H, m->emb_g, m->emb_b);

  bert_state S = {m, NULL, seq, h, tmp, ctx, qb, kb, vb, normed, scores, ff};
  for (int li = 0; li < m->layers; ++li) {
    S.lw = &m->L[li];
    par_for(seq, bert_qkv_tok, &S);
    par_for(m->heads, bert_attention_head, &S);
    if (!m->mpnet) {
      par_for(seq, bert_ao_tok, &S);
      par_for(seq, bert_ffn_tok, &S);
    } else {
      par_for(seq, mpnet_ao_ff1_tok, &S);
      par_for(seq, mpnet_ff2_tok, &S);
    }
  }
  /* pooling + L2 (bert.lisp:302-319) */
  for (int i = 0; i < H; ++i) out[i] = 0.0f;
  if (m->pooling == 1) {
    for (int t = 0; t < seq; ++t)
      for (int i = 0; i < H; ++i) out[i] = out[i] + h[(size_t)t * H + i];
    for (int i = 0; i < H; ++i) out[i] = out[i] / (float)seq;
  } else {
    for (int i = 0; i < H; ++i) out[i] = h[i];
  }
  float norm = 0.0f;
  for (int i = 0; i < H; ++i) norm = norm + out[i] * out[i];
  norm = ssqrt(norm);
  for (int i = 0; i < H; ++i) out[i] = out[i] / norm;
  free(h); free(tmp); free(ctx); free(qb); free(kb); free(vb);
  free(normed); free(scores); free(ff);
  return 0;
}

/* ---- llama.lisp ----------------------------------------------------------- */

/* llama::rmsnorm (llama.lisp:106-117): sum of squares in double. */
static void rmsnorm(float *x, int n, const float *g, double eps) {
  double ss = 0.0;
  for (int i = 0; i < n; ++i) ss += (double)(x[i] * x[i]);
  float inv = (float)(1.0 / sqrt(ss / (double)n + eps));
  for (int i = 0; i < n; ++i) x[i] = (x[i] * inv) * g[i];
}

/* llama::silu (llama.lisp:119-122): in double. */
static float silu(float x) {
  double xd = (double)x;
  return (float)(xd / (1.0 + exp(-xd)));
}

/* llama::rope (llama.lisp:137-151): rotate-half pairing (i, i+hd/2). */
static void rope(float *x, int pos, int heads, int hd, const float *cs,
                 const float *sn) {
  int half = hd / 2;
  for (int h = 0; h < heads; ++h) {
    float *base = x + (size_t)h * hd;
    for (int i = 0; i < half; ++i) {
      float c = cs[(size_t)pos * half + i], s = sn[(size_t)pos * half + i];
      float a = base[i], b = base[i + half];
      base[i] = a * c - b * s;
      base[i + half] = a * s + b * c;
    }
  }
}

/* Shared state of one Llama / Qwen3 forward, for the parallel loop bodies. */
typedef struct {
  const or_llama *m;
  const or_llama_layer *lw;
  int seq, tw;
  const float *cs, *sn;
  float *h, *normed, *qb, *kb, *vb, *ctx, *scores, *tmp, *o;
} llama_state;

/* input RMSNorm, q/k/v projections, q/k RMSNorm and RoPE of token t
 * (llama.lisp:296-312) */
static void llama_qkv_tok(void *arg, int t) {
  const llama_state *S = (const llama_state *)arg;
  const or_llama *m = S->m;
  const or_llama_layer *lw = S->lw;
  const int H = m->hidden, hd = m->head_dim, heads = m->heads, kv = m->kv_heads;
  const int qd = heads * hd, kvd = kv * hd;
  float *nr = S->normed + (size_t)t * H;
  memcpy(nr, S->h + (size_t)t * H, H * sizeof(float));
  rmsnorm(nr, H, lw->in_ln, m->eps);
  linear_nb(nr, lw->q_w, S->qb + (size_t)t * qd, H, qd);
  linear_nb(nr, lw->k_w, S->kb + (size_t)t * kvd, H, kvd);
  linear_nb(nr, lw->v_w, S->vb + (size_t)t * kvd, H, kvd);
  if (lw->q_norm)
    for (int hh = 0; hh < heads; ++hh) rmsnorm(S->qb + (size_t)t * qd + hh * hd, hd, lw->q_norm, m->eps);
  if (lw->k_norm)
    for (int hh = 0; hh < kv; ++hh) rmsnorm(S->kb + (size_t)t * kvd + hh * hd, hd, lw->k_norm, m->eps);
  rope(S->qb + (size_t)t * qd, t, heads, hd, S->cs, S->sn);
  rope(S->kb + (size_t)t * kvd, t, kv, hd, S->cs, S->sn);
}

/* causal GQA attention of one query head (llama.lisp:313-324) */
static void llama_attention_head(void *arg, int hh) {
  const llama_state *S = (const llama_state *)arg;
  const or_llama *m = S->m;
  const int hd = m->head_dim, heads = m->heads, kv = m->kv_heads, seq = S->seq;
  const int qd = heads * hd, kvd = kv * hd, kvh = hh / (heads / kv);
  const float sqrt_hd = ssqrt((float)hd);
  float *scores = S->scores + (size_t)hh * seq;
  for (int t1 = 0; t1 < seq; ++t1) {
    for (int t2 = 0; t2 <= t1; ++t2)
      scores[t2] = or_dot(S->qb + (size_t)t1 * qd + hh * hd, S->kb + (size_t)t2 * kvd + kvh * hd, hd) /
                   sqrt_hd;
    softmax(scores, t1 + 1);
    for (int i = 0; i < hd; ++i) {
      float acc = 0.0f;
      for (int t2 = 0; t2 <= t1; ++t2) acc = acc + scores[t2] * S->vb[(size_t)t2 * kvd + kvh * hd + i];
      S->ctx[(size_t)t1 * qd + hh * hd + i] = acc;
    }
  }
}

/* output projection + residual, post-attention RMSNorm, SwiGLU FFN +
 * residual of token t (llama.lisp:325-343) */
static void llama_out_ffn_tok(void *arg, int t) {
  const llama_state *S = (const llama_state *)arg;
  const or_llama *m = S->m;
  const or_llama_layer *lw = S->lw;
  const int H = m->hidden, F = m->inter, qd = m->heads * m->head_dim;
  float *hr = S->h + (size_t)t * H;
  float *trow = S->tmp + (size_t)t * S->tw, *orow = S->o + (size_t)t * F;
  linear_nb(S->ctx + (size_t)t * qd, lw->o_w, trow, qd, H);
  for (int i = 0; i < H; ++i) hr[i] = hr[i] + trow[i];
  float *nr = S->normed + (size_t)t * H;
  memcpy(nr, hr, H * sizeof(float));
  rmsnorm(nr, H, lw->post_ln, m->eps);
  linear_nb(nr, lw->gate, orow, H, F);
  linear_nb(nr, lw->up, trow, H, F);
  for (int i = 0; i < F; ++i) orow[i] = silu(orow[i]) * trow[i];
  linear_nb(orow, lw->down, trow, F, H); /* the up row is consumed: reuse it */
  for (int i = 0; i < H; ++i) hr[i] = hr[i] + trow[i];
}

/* llama::embed / layer-forward (llama.lisp:224-344). */
int or_llama_embed(const or_llama *m, const int32_t *ids, int seq, float *out) {
  const int H = m->hidden, heads = m->heads, kv = m->kv_heads, hd = m->head_dim;
  const int F = m->inter, kvd = kv * hd, qd = heads * hd;
  const int half = hd / 2;
  if (seq > m->max_pos) return -2;
  /* init-rope (llama.lisp:124-135) */
  float *cs = malloc((size_t)m->max_pos * half * sizeof(float));
  float *sn = malloc((size_t)m->max_pos * half * sizeof(float));
  float *h = malloc((size_t)seq * H * sizeof(float));
  float *normed = malloc((size_t)seq * H * sizeof(float));
  float *qb = malloc((size_t)seq * qd * sizeof(float));
  float *kb = malloc((size_t)seq * kvd * sizeof(float));
  float *vb = malloc((size_t)seq * kvd * sizeof(float));
  float *ctx = malloc((size_t)seq * qd * sizeof(float));
  float *scores = malloc((size_t)heads * seq * sizeof(float));
  int tw = H > F ? H : F;
  float *tmp = malloc((size_t)seq * tw * sizeof(float));
  float *o = malloc((size_t)seq * F * sizeof(float));
  if (!cs || !sn || !h || !normed || !qb || !kb || !vb || !ctx || !scores || !tmp || !o) {
    free(cs); free(sn); free(h); free(normed); free(qb); free(kb); free(vb);
    free(ctx); free(scores); free(tmp); free(o);
    return -1;
  }
  for (int p = 0; p < m->max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      double freq = 1.0 / pow(m->rope_theta, (2.0 * i) / (double)hd);
      double ang = p * freq;
      cs[(size_t)p * half + i] = (float)cos(ang);
      sn[(size_t)p * half + i] = (float)sin(ang);
    }
  for (int t = 0; t < seq; ++t)
    memcpy(h + (size_t)t * H, m->w_embed + (size_t)ids[t] * H, H * sizeof(float));
  llama_state S = {m, NULL, seq, tw, cs, sn, h, normed, qb, kb, vb, ctx, scores, tmp, o};
  for (int li = 0; li < m->layers; ++li) {
    S.lw = &m->L[li];
    par_for(seq, llama_qkv_tok, &S);
    par_for(heads, llama_attention_head, &S);
    par_for(seq, llama_out_ffn_tok, &S);
  }
  for (int t = 0; t < seq; ++t) rmsnorm(h + (size_t)t * H, H, m->w_norm, m->eps);
  for (int i = 0; i < H; ++i) out[i] = 0.0f;
  if (m->pooling == 1) {
    for (int t = 0; t < seq; ++t)
      for (int i = 0; i < H; ++i) out[i] = out[i] + h[(size_t)t * H + i];
    for (int i = 0; i < H; ++i) out[i] = out[i] / (float)seq;
  } else {
    for (int i = 0; i < H; ++i) out[i] = h[(size_t)(seq - 1) * H + i];
  }
  float norm = 0.0f;
  for (int i = 0; i < H; ++i) norm = norm + out[i] * out[i];
  norm = ssqrt(norm);
  for (int i = 0; i < H; ++i) out[i] = out[i] / norm;
  free(cs); free(sn); free(h); free(normed); free(qb); free(kb); free(vb);
  free(ctx); free(scores); free(tmp); free(o);
  return 0;
}

/* ---- gemma.lisp ------------------------------------------------------------ */

/* gemma::rmsnorm-noscale (gemma.lisp:74-83): the v-norm, no learned scale. */
static void rmsnorm_noscale(float *x, int n, double eps) {
  double ss = 0.0;
  for (int i = 0; i < n; ++i) ss += (double)(x[i] * x[i]);
  float inv = (float)(1.0 / sqrt(ss / (double)n + eps));
  for (int i = 0; i < n; ++i) x[i] = x[i] * inv;
}

/* gemma::gelu-tanh (gemma.lisp:85-89): gelu_pytorch_tanh evaluated in double. */
static float gelu_tanh(float x) {
  double xd = (double)x;
  double c = 0.7978845608028654 * (xd + ((0.044715 * xd) * xd) * xd);
  return (float)((0.5 * xd) * (1.0 + tanh(c)));
}

/* gemma::embed + layer-forward (gemma.lisp:216-376). */
int or_gemma_embed(const or_gemma *m, const int32_t *ids, int seq, float *out) {
  const int H = m->hidden, heads = m->heads, F = m->inter, P = m->ple_dim, NL = m->layers;
  if (seq > m->max_pos) return -2;
  int maxq = 0, maxkv = 0, maxhalf = 0;
  for (int li = 0; li < NL; ++li) {
    const int hd = m->L[li].head_dim;
    if (heads * hd > maxq) maxq = heads * hd;
    if (m->L[li].kv_heads * hd > maxkv) maxkv = m->L[li].kv_heads * hd;
    if (hd / 2 > maxhalf) maxhalf = hd / 2;
  }
  int tw = H > F ? H : F;
  if (P > tw) tw = P;
  int ow = F > P ? F : P;
  float *h = malloc((size_t)seq * H * sizeof(float));
  float *ple = malloc((size_t)seq * NL * P * sizeof(float));
  float *qb = malloc((size_t)seq * maxq * sizeof(float));
  float *kb = malloc((size_t)seq * maxkv * sizeof(float));
  float *vb = malloc((size_t)seq * maxkv * sizeof(float));
  float *ctx = malloc((size_t)seq * maxq * sizeof(float));
  float *scores = malloc((size_t)seq * sizeof(float));
  float *tmp = malloc((size_t)seq * tw * sizeof(float));
  float *o = malloc((size_t)seq * ow * sizeof(float));
  float *normed = malloc((size_t)seq * H * sizeof(float));
  float *cs = malloc((size_t)m->max_pos * maxhalf * sizeof(float));
  float *sn = malloc((size_t)m->max_pos * maxhalf * sizeof(float));
  float *pooled = malloc((size_t)H * sizeof(float));
  int rc = 0;
  if (!h || !ple || !qb || !kb || !vb || !ctx || !scores || !tmp || !o || !normed || !cs || !sn ||
      !pooled) {
    rc = -1;
    goto done;
  }
  /* token embeddings scaled by sqrt(hidden) (gemma.lisp:326-330) */
  const float scale = ssqrt((float)H);
  for (int t = 0; t < seq; ++t)
    for (int i = 0; i < H; ++i) h[(size_t)t * H + i] = scale * m->w_embed[(size_t)ids[t] * H + i];
  /* per-layer embeddings: projection, * 1/sqrt(hidden), RMSNorm per layer
   * slice (gemma.lisp:331-343) */
  for (int t = 0; t < seq; ++t)
    linear_nb(h + (size_t)t * H, m->w_ple_proj, ple + (size_t)t * NL * P, H, NL * P);
  {
    const float inv = 1.0f / ssqrt((float)H);
    for (size_t i = 0; i < (size_t)seq * NL * P; ++i) ple[i] = ple[i] * inv;
    for (int t = 0; t < seq; ++t)
      for (int li = 0; li < NL; ++li)
        rmsnorm(ple + (size_t)t * NL * P + (size_t)li * P, P, m->w_ple_norm, m->eps);
  }
  for (int li = 0; li < NL; ++li) {
    const or_gemma_layer *lw = &m->L[li];
    const int hd = lw->head_dim, kv = lw->kv_heads, half = hd / 2;
    const int qd = heads * hd, kvd = kv * hd, group = heads / kv;
    /* gemma::init-rope (gemma.lisp:91-103) with this layer's theta */
    for (int p = 0; p < m->max_pos; ++p)
      for (int i = 0; i < half; ++i) {
        double freq = 1.0 / pow(lw->rope_theta, (2.0 * i) / (double)hd);
        double ang = p * freq;
        cs[(size_t)p * half + i] = (float)cos(ang);
        sn[(size_t)p * half + i] = (float)sin(ang);
      }
    /* attention sub-block (gemma.lisp:228-274) */
    for (int t = 0; t < seq; ++t) {
      memcpy(normed + (size_t)t * H, h + (size_t)t * H, H * sizeof(float));
      rmsnorm(normed + (size_t)t * H, H, lw->in_ln, m->eps);
    }
    for (int t = 0; t < seq; ++t) {
      linear_nb(normed + (size_t)t * H, lw->q_w, qb + (size_t)t * qd, H, qd);
      linear_nb(normed + (size_t)t * H, lw->k_w, kb + (size_t)t * kvd, H, kvd);
      linear_nb(normed + (size_t)t * H, lw->v_w, vb + (size_t)t * kvd, H, kvd);
    }
    for (int t = 0; t < seq; ++t) {
      for (int hh = 0; hh < heads; ++hh) rmsnorm(qb + (size_t)t * qd + hh * hd, hd, lw->q_norm, m->eps);
      for (int hh = 0; hh < kv; ++hh) {
        rmsnorm(kb + (size_t)t * kvd + hh * hd, hd, lw->k_norm, m->eps);
        rmsnorm_noscale(vb + (size_t)t * kvd + hh * hd, hd, m->eps);
      }
      rope(qb + (size_t)t * qd, t, heads, hd, cs, sn);
      rope(kb + (size_t)t * kvd, t, kv, hd, cs, sn);
    }
    /* bidirectional attention, scale 1.0 (gemma.lisp:250-265) */
    for (int hh = 0; hh < heads; ++hh) {
      int kvh = hh / group;
      for (int t1 = 0; t1 < seq; ++t1) {
        for (int t2 = 0; t2 < seq; ++t2)
          scores[t2] = or_dot(qb + (size_t)t1 * qd + hh * hd, kb + (size_t)t2 * kvd + kvh * hd, hd);
        softmax(scores, seq);
        for (int i = 0; i < hd; ++i) {
          float acc = 0.0f;
          for (int t2 = 0; t2 < seq; ++t2)
            acc = acc + scores[t2] * vb[(size_t)t2 * kvd + kvh * hd + i];
          ctx[(size_t)t1 * qd + hh * hd + i] = acc;
        }
      }
    }
    for (int t = 0; t < seq; ++t) {
      float *tr = tmp + (size_t)t * H;
      linear_nb(ctx + (size_t)t * qd, lw->o_w, tr, qd, H);
      rmsnorm(tr, H, lw->post_ln, m->eps);
      for (int i = 0; i < H; ++i) h[(size_t)t * H + i] = h[(size_t)t * H + i] + tr[i];
    }
    /* FFN sub-block: GELU-tanh gated MLP between pre/post norms (:275-287) */
    for (int t = 0; t < seq; ++t) {
      memcpy(normed + (size_t)t * H, h + (size_t)t * H, H * sizeof(float));
      rmsnorm(normed + (size_t)t * H, H, lw->pre_ff_ln, m->eps);
    }
    for (int t = 0; t < seq; ++t) {
      float *orow = o + (size_t)t * ow, *trow = tmp + (size_t)t * tw;
      linear_nb(normed + (size_t)t * H, lw->gate, orow, H, F);
      linear_nb(normed + (size_t)t * H, lw->up, trow, H, F);
      for (int i = 0; i < F; ++i) orow[i] = gelu_tanh(orow[i]) * trow[i];
      linear_nb(orow, lw->down, trow, F, H);
      rmsnorm(trow, H, lw->post_ff_ln, m->eps);
      for (int i = 0; i < H; ++i) h[(size_t)t * H + i] = h[(size_t)t * H + i] + trow[i];
    }
    /* PLE sub-block: gate(h) -> GELU-tanh * ple -> proj -> norm -> residual
     * (:288-298) */
    for (int t = 0; t < seq; ++t) {
      float *orow = o + (size_t)t * ow, *trow = tmp + (size_t)t * tw;
      const float *prow = ple + (size_t)t * NL * P + (size_t)li * P;
      linear_nb(h + (size_t)t * H, lw->ple_gate, orow, H, P);
      for (int i = 0; i < P; ++i) orow[i] = gelu_tanh(orow[i]) * prow[i];
      linear_nb(orow, lw->ple_proj, trow, P, H);
      rmsnorm(trow, H, lw->ple_norm, m->eps);
      for (int i = 0; i < H; ++i) h[(size_t)t * H + i] = h[(size_t)t * H + i] + trow[i];
    }
    /* layer scalar (:300-302) */
    for (size_t i = 0; i < (size_t)seq * H; ++i) h[i] = h[i] * lw->scalar;
  }
  /* final norm, mean pool, projection, L2 (:359-376) */
  for (int t = 0; t < seq; ++t) rmsnorm(h + (size_t)t * H, H, m->w_norm, m->eps);
  for (int i = 0; i < H; ++i) pooled[i] = 0.0f;
  for (int t = 0; t < seq; ++t)
    for (int i = 0; i < H; ++i) pooled[i] = pooled[i] + h[(size_t)t * H + i];
  for (int i = 0; i < H; ++i) pooled[i] = pooled[i] / (float)seq;
  linear_nb(pooled, m->w_out, out, H, m->out_dim);
  {
    float norm = 0.0f;
    for (int i = 0; i < m->out_dim; ++i) norm = norm + out[i] * out[i];
    norm = ssqrt(norm);
    for (int i = 0; i < m->out_dim; ++i) out[i] = out[i] / norm;
  }
done:
  free(h); free(ple); free(qb); free(kb); free(vb); free(ctx); free(scores); free(tmp);
  free(o); free(normed); free(cs); free(sn); free(pooled);
  return rc;
}

/* ---- embed.lisp batch driver ---------------------------------------------- */
typedef struct {
  int kind;
  const void *model;
  const int32_t *ids;
  int seq;
  float *out;
  int rc;
} embed_job;

static void *embed_thread(void *arg) {
  embed_job *j = (embed_job *)arg;
  j->rc = j->kind == 0   ? or_bert_embed((const or_bert *)j->model, j->ids, j->seq, j->out)
          : j->kind == 1 ? or_llama_embed((const or_llama *)j->model, j->ids, j->seq, j->out)
                         : or_gemma_embed((const or_gemma *)j->model, j->ids, j->seq, j->out);
  return NULL;
}

int or_embed_batch(int kind, const void *model, const int32_t *ids,
                   const int64_t *offsets, int nseq, int dim, float *out,
                   int threads) {
  if (threads < 1) threads = 1;
  embed_job *jobs = calloc((size_t)threads, sizeof(embed_job));
  pthread_t *tid = calloc((size_t)threads, sizeof(pthread_t));
  int rc = 0;
  /* embed.lisp:88-105: take `threads` chunks, one thread each, join in order */
  for (int base = 0; base < nseq && rc == 0; base += threads) {
    int cnt = nseq - base < threads ? nseq - base : threads;
    for (int j = 0; j < cnt; ++j) {
      int s = base + j;
      jobs[j].kind = kind;
      jobs[j].model = model;
      jobs[j].ids = ids + offsets[s];
      jobs[j].seq = (int)(offsets[s + 1] - offsets[s]);
      jobs[j].out = out + (size_t)s * dim;
      pthread_create(&tid[j], NULL, embed_thread, &jobs[j]);
    }
    for (int j = 0; j < cnt; ++j) {
      pthread_join(tid[j], NULL);
      if (jobs[j].rc) rc = jobs[j].rc;
    }
  }
  free(jobs);
  free(tid);
  return rc;
}

/* ---- st.lisp widening ------------------------------------------------------ */
void or_bf16_to_f32(const uint16_t *src, float *dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t b = (uint32_t)src[i] << 16;
    memcpy(&dst[i], &b, 4);
  }
}

/* st::half-to-float (st.lisp:22-30): exponent 31 -> +-most-positive-single. */
void or_f16_to_f32(const uint16_t *src, float *dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint16_t hbits = src[i];
    float sign = (hbits & 0x8000) ? -1.0f : 1.0f;
    int e = (hbits >> 10) & 31, mant = hbits & 1023;
    float v;
    if (e == 0) v = (sign * ldexpf(1.0f, -14)) * ((float)mant / 1024.0f);
    else if (e == 31) v = sign * FLT_MAX;
    else v = (sign * ldexpf(1.0f, e - 15)) * (1.0f + (float)mant / 1024.0f);
    dst[i] = v;
  }
}

/* ---- ann.lisp -------------------------------------------------------------- */

/* ann::nearest-centroid (ann.lisp:69-77): strict > so ties keep the lowest c. */
int32_t or_nearest_centroid(const float *x, const float *cent, int k, int dim) {
  int32_t best = 0;
  float best_score = -FLT_MAX;
  for (int c = 0; c < k; ++c) {
    float s = or_dot(x, cent + (size_t)c * dim, dim);
    if (s > best_score) {
      best_score = s;
      best = c;
    }
  }
  return best;
}

typedef struct {
  const float *vecs, *cent;
  const int64_t *rows;
  int64_t s, e;
  int k, dim;
  int32_t *assign;
} assign_job;

/* Four rows at a time against four centroids at a time: sixteen independent
 * %dot chains, each still the sequential single-float sum of or_dot, and the
 * strict-> argmax visits the centroids of every row in index order, so the
 * result equals or_nearest_centroid row by row (only faster). */
static void nearest4(const float *const xr[4], int nr, const float *cent, int k, int dim,
                     int32_t out[4]) {
  float best_s[4] = {-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX};
  int32_t best[4] = {0, 0, 0, 0};
  int c = 0;
  for (; c + 4 <= k; c += 4) {
    const float *c0 = cent + (size_t)c * dim, *c1 = c0 + dim, *c2 = c1 + dim, *c3 = c2 + dim;
    for (int r = 0; r < nr; ++r) {
      const float *x = xr[r];
      float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
      for (int i = 0; i < dim; ++i) {
        const float xi = x[i];
        s0 = s0 + xi * c0[i];
        s1 = s1 + xi * c1[i];
        s2 = s2 + xi * c2[i];
        s3 = s3 + xi * c3[i];
      }
      const float sc[4] = {s0, s1, s2, s3};
      for (int j = 0; j < 4; ++j)
        if (sc[j] > best_s[r]) {
          best_s[r] = sc[j];
          best[r] = c + j;
        }
    }
  }
  for (; c < k; ++c)
    for (int r = 0; r < nr; ++r) {
      const float sc = or_dot(xr[r], cent + (size_t)c * dim, dim);
      if (sc > best_s[r]) {
        best_s[r] = sc;
        best[r] = c;
      }
    }
  for (int r = 0; r < nr; ++r) out[r] = best[r];
}

static void *assign_thread(void *arg) {
  assign_job *j = (assign_job *)arg;
  for (int64_t i = j->s; i < j->e; i += 4) {
    const int nr = j->e - i < 4 ? (int)(j->e - i) : 4;
    const float *xr[4];
    for (int r = 0; r < nr; ++r) {
      const int64_t row = j->rows ? j->rows[i + r] : i + r;
      xr[r] = j->vecs + (size_t)row * j->dim;
    }
    int32_t out[4];
    nearest4(xr, nr, j->cent, j->k, j->dim, out);
    for (int r = 0; r < nr; ++r) j->assign[i + r] = out[r];
  }
  return NULL;
}

/* the reference's own loop shape: or_nearest_centroid per row, one
 * centroid at a time (ann.lisp:69-77), for the timed CPU baseline */
static void *assign_thread_scalar(void *arg) {
  assign_job *j = (assign_job *)arg;
  for (int64_t i = j->s; i < j->e; ++i) {
    const int64_t row = j->rows ? j->rows[i] : i;
    j->assign[i] = or_nearest_centroid(j->vecs + (size_t)row * j->dim, j->cent, j->k, j->dim);
  }
  return NULL;
}

static void assign_ranges(const float *vecs, const int64_t *rows, int64_t nrows,
                          const float *cent, int k, int dim, int32_t *assign, int threads,
                          void *(*body)(void *)) {
  if (threads < 1) threads = 1;
  int64_t per = (nrows + threads - 1) / threads;
  pthread_t *tid = calloc((size_t)threads, sizeof(pthread_t));
  assign_job *jobs = calloc((size_t)threads, sizeof(assign_job));
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    int64_t s = (int64_t)t * per, e = s + per < nrows ? s + per : nrows;
    if (s >= e) continue;
    jobs[started] = (assign_job){vecs, cent, rows, s, e, k, dim, assign};
    pthread_create(&tid[started], NULL, body, &jobs[started]);
    ++started;
  }
  for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
  free(tid);
  free(jobs);
}

/* ann.lisp:90-105's parallel assign, one row and one centroid at a time */
void or_assign_scalar(const float *vecs, const int64_t *rows, int64_t nrows,
                      const float *cent, int k, int dim, int32_t *assign, int threads) {
  assign_ranges(vecs, rows, nrows, cent, k, dim, assign, threads, assign_thread_scalar);
}

/* parallel assign over contiguous ranges (ann.lisp:90-105 / :131-144) */
void or_assign(const float *vecs, const int64_t *rows, int64_t nrows,
               const float *cent, int k, int dim, int32_t *assign, int threads) {
  assign_ranges(vecs, rows, nrows, cent, k, dim, assign, threads, assign_thread);
}

/* Lloyd update (ann.lisp:107-122): serial sums in sample order; an empty
 * cluster keeps its centroid. */
void or_kmeans_update(const float *vecs, const int64_t *sample, int64_t ns,
                      const int32_t *assign, int k, int dim, float *cent) {
  float *sums = calloc((size_t)k * dim, sizeof(float));
  int64_t *counts = calloc((size_t)k, sizeof(int64_t));
  for (int64_t j = 0; j < ns; ++j) {
    int64_t row = sample[j];
    int c = assign[j];
    counts[c] += 1;
    for (int d = 0; d < dim; ++d)
      sums[(size_t)c * dim + d] = sums[(size_t)c * dim + d] + vecs[(size_t)row * dim + d];
  }
  for (int c = 0; c < k; ++c)
    if (counts[c] > 0)
      for (int d = 0; d < dim; ++d)
        cent[(size_t)c * dim + d] = sums[(size_t)c * dim + d] / (float)counts[c];
  free(sums);
  free(counts);
}

/* ann::kmeans (ann.lisp:79-125): init from sample[0..k). */
void or_kmeans(const float *vecs, const int64_t *sample, int64_t ns, int k,
               int dim, int iters, float *cent, int threads) {
  for (int c = 0; c < k; ++c)
    memcpy(cent + (size_t)c * dim, vecs + (size_t)sample[c] * dim, dim * sizeof(float));
  int32_t *assign = malloc((size_t)ns * sizeof(int32_t));
  for (int it = 0; it < iters; ++it) {
    or_assign(vecs, sample, ns, cent, k, dim, assign, threads);
    or_kmeans_update(vecs, sample, ns, assign, k, dim, cent);
  }
  free(assign);
}

/* ann::assign-all (ann.lisp:127-158): counting sort, ascending ids per list. */
void or_assign_all(const float *vecs, int64_t n, const float *cent, int k,
                   int dim, uint32_t *counts, uint32_t *lists, int threads) {
  int32_t *assign = malloc((size_t)n * sizeof(int32_t));
  or_assign(vecs, NULL, n, cent, k, dim, assign, threads);
  for (int c = 0; c < k; ++c) counts[c] = 0;
  for (int64_t i = 0; i < n; ++i) counts[assign[i]] += 1;
  int64_t *cursor = malloc((size_t)k * sizeof(int64_t));
  int64_t acc = 0;
  for (int c = 0; c < k; ++c) {
    cursor[c] = acc;
    acc += counts[c];
  }
  for (int64_t i = 0; i < n; ++i) lists[cursor[assign[i]]++] = (uint32_t)i;
  free(cursor);
  free(assign);
}

/* ---- kb.lisp --------------------------------------------------------------- */

/* insertion top-k with strict > (kb.lisp:164-184, :316-334) */
static void topk_insert(float *sc, int64_t *ix, int k, float s, int64_t id) {
  if (!(s > sc[k - 1])) return;
  int pos = k - 1;
  while (pos > 0 && s > sc[pos - 1]) {
    sc[pos] = sc[pos - 1];
    ix[pos] = ix[pos - 1];
    --pos;
  }
  sc[pos] = s;
  ix[pos] = id;
}

typedef struct { int64_t id; float s; int64_t ord; } cand;

/* SBCL's list `sort` is a stable merge sort: order by score desc, then by
 * position in the appended list. */
static int cand_cmp(const void *a, const void *b) {
  const cand *x = a, *y = b;
  if (x->s > y->s) return -1;
  if (x->s < y->s) return 1;
  return (x->ord > y->ord) - (x->ord < y->ord);
}

int or_top_k_ivf(const float *vecs, int dim, const float *cent, int k,
                 const uint32_t *counts, const uint32_t *lists, int nprobe,
                 const float *q, int topk, int64_t *ids, float *scores) {
  if (nprobe > k) nprobe = k;
  /* centroid scores: dot-arrays(centroids, q) (kb.lisp:351-352) */
  cand *cs = malloc((size_t)k * sizeof(cand));
  int64_t *offs = malloc((size_t)k * sizeof(int64_t));
  int64_t acc = 0;
  for (int c = 0; c < k; ++c) {
    offs[c] = acc;
    acc += counts[c];
    cs[c].id = c;
    cs[c].s = or_dot(cent + (size_t)c * dim, q, dim);
    cs[c].ord = c;
  }
  qsort(cs, (size_t)k, sizeof(cand), cand_cmp);
  cand *all = malloc((size_t)nprobe * topk * sizeof(cand));
  float *sc = malloc((size_t)topk * sizeof(float));
  int64_t *ix = malloc((size_t)topk * sizeof(int64_t));
  int64_t na = 0;
  for (int p = 0; p < nprobe; ++p) {
    int c = (int)cs[p].id;
    for (int j = 0; j < topk; ++j) { sc[j] = -FLT_MAX; ix[j] = -1; }
    for (int64_t j = offs[c]; j < offs[c] + counts[c]; ++j) {
      uint32_t row = lists[j];
      /* kb::%dot(base, q): vectors[base+j] * q[j] */
      topk_insert(sc, ix, topk, or_dot(vecs + (size_t)row * dim, q, dim), row);
    }
    for (int j = 0; j < topk; ++j)
      if (ix[j] >= 0) { all[na].id = ix[j]; all[na].s = sc[j]; all[na].ord = na; ++na; }
  }
  qsort(all, (size_t)na, sizeof(cand), cand_cmp);
  int r = (int)(na < topk ? na : topk);
  for (int j = 0; j < r; ++j) { ids[j] = all[j].id; scores[j] = all[j].s; }
  for (int j = r; j < topk; ++j) { ids[j] = -1; scores[j] = -FLT_MAX; }
  free(cs); free(offs); free(all); free(sc); free(ix);
  return r;
}

typedef struct {
  const float *vecs, *q;
  int64_t s, e;
  int dim, k;
  float *sc;
  int64_t *ix;
} brute_job;

static void *brute_thread(void *arg) {
  brute_job *j = arg;
  for (int t = 0; t < j->k; ++t) { j->sc[t] = -FLT_MAX; j->ix[t] = -1; }
  for (int64_t i = j->s; i < j->e; ++i)
    topk_insert(j->sc, j->ix, j->k, or_dot(j->vecs + (size_t)i * j->dim, j->q, j->dim), i);
  return NULL;
}

int or_top_k_brute(const float *vecs, int64_t n, int dim, const float *q,
                   int topk, int threads, int64_t *ids, float *scores) {
  if (threads < 1) threads = 1;
  int64_t per = (n + threads - 1) / threads;
  brute_job *jobs = calloc((size_t)threads, sizeof(brute_job));
  pthread_t *tid = calloc((size_t)threads, sizeof(pthread_t));
  float *sc = malloc((size_t)threads * topk * sizeof(float));
  int64_t *ix = malloc((size_t)threads * topk * sizeof(int64_t));
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    int64_t s = (int64_t)t * per, e = s + per < n ? s + per : n;
    if (s >= e) continue;
    jobs[started] = (brute_job){vecs, q, s, e, dim, topk, sc + (size_t)started * topk,
                                ix + (size_t)started * topk};
    pthread_create(&tid[started], NULL, brute_thread, &jobs[started]);
    ++started;
  }
  for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
  cand *all = malloc((size_t)started * topk * sizeof(cand) + 1);
  int64_t na = 0;
  for (int t = 0; t < started; ++t)
    for (int j = 0; j < topk; ++j)
      if (jobs[t].ix[j] >= 0) {
        all[na].id = jobs[t].ix[j]; all[na].s = jobs[t].sc[j]; all[na].ord = na; ++na;
      }
  qsort(all, (size_t)na, sizeof(cand), cand_cmp);
  int r = (int)(na < topk ? na : topk);
  for (int j = 0; j < r; ++j) { ids[j] = all[j].id; scores[j] = all[j].s; }
  for (int j = r; j < topk; ++j) { ids[j] = -1; scores[j] = -FLT_MAX; }
  free(jobs); free(tid); free(sc); free(ix); free(all);
  return r;
}
