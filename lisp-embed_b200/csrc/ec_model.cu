// ec_model.cu -- model assembly from uploaded safetensors and the batched
// encoder forward on one device.
//
// Assembly replaces the per-tensor st:get-tensor calls of bert:load-model
// (bert.lisp:83-127), bert::load-mpnet-weights (bert.lisp:343-389) and
// llama:load-model (llama.lisp:189-218): Q/K/V weights are fused into one
// [3H, H] (or [(heads + 2 kv) * hd, H]) bf16 matrix, gate/up into one
// block-interleaved [2F, H] matrix, vectors stay fp32.
//
// The forward replaces embed-bert / embed-mpnet / llama:embed for a whole
// batch of packed sequences: every linear of every token of every sequence of
// a layer is one tcgen05 GEMM launch.
#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <chrono>
#include <climits>
#include <cstring>
#include <numeric>

#include "ec_gemm.cuh"
#include "ec_json.h"
#include "ec_state.h"

namespace ec {

// ----------------------------------------------------------------- helpers --
static const Tensor* find_t(Device& d, const std::string& name) {
  auto it = d.uploads.find(name);
  return it == d.uploads.end() ? nullptr : &it->second;
}

static int need_t(Device& d, const std::string& name, const Tensor** out,
                  std::initializer_list<int64_t> shape) {
  const Tensor* t = find_t(d, name);
  if (!t) return set_error(EC_EINVAL, "missing tensor %s", name.c_str());
  if (shape.size()) {
    std::vector<int64_t> want(shape);
    if (t->shape != want) {
      std::string got, exp;
      for (auto v : t->shape) got += std::to_string(v) + ",";
      for (auto v : want) exp += std::to_string(v) + ",";
      return set_error(EC_EINVAL, "tensor %s has shape [%s], expected [%s]", name.c_str(),
                       got.c_str(), exp.c_str());
    }
  }
  *out = t;
  return EC_OK;
}

static int model_alloc(Device& d, void** p, size_t bytes, const char* what) {
  int rc = dev_alloc(d, p, bytes, what);
  if (rc == EC_OK) d.model.owned.push_back(*p);
  return rc;
}

// fp32 copy of a vector tensor (LayerNorm / RMSNorm weights, biases)
static int as_f32(Device& d, const Tensor* t, float** out) {
  if (t->dtype == kDtF32) {
    *out = static_cast<float*>(t->p);
    return EC_OK;
  }
  void* p;
  int rc = model_alloc(d, &p, t->numel * 4, "f32 vector");
  if (rc) return rc;
  rc = check_cuda(launch_convert(kConvBf16ToF32, t->p, p, t->numel, d.stream), "convert");
  *out = static_cast<float*>(p);
  return rc;
}

// copy `rows` rows of a [*, cols] tensor starting at row r0 into dst (bf16)
static int rows_to_bf16(Device& d, const Tensor* t, int64_t r0, int64_t rows, int64_t cols,
                        bf16* dst) {
  const size_t n = static_cast<size_t>(rows * cols);
  if (t->dtype == kDtBf16) {
    return check_cuda(cudaMemcpyAsync(dst, static_cast<const bf16*>(t->p) + r0 * cols,
                                      n * 2, cudaMemcpyDeviceToDevice, d.stream),
                      "weight copy");
  }
  return check_cuda(launch_convert(kConvF32ToBf16, static_cast<const float*>(t->p) + r0 * cols,
                                   dst, n, d.stream),
                    "weight convert");
}

// vertical concatenation of [rows_i, cols] matrices into one bf16 matrix
static int concat_bf16(Device& d, const std::vector<const Tensor*>& parts, int64_t cols,
                       bf16** out) {
  int64_t rows = 0;
  for (auto* t : parts) rows += t->shape[0];
  void* p;
  int rc = model_alloc(d, &p, static_cast<size_t>(rows * cols) * 2, "bf16 weight");
  if (rc) return rc;
  int64_t r = 0;
  for (auto* t : parts) {
    rc = rows_to_bf16(d, t, 0, t->shape[0], cols, static_cast<bf16*>(p) + r * cols);
    if (rc) return rc;
    r += t->shape[0];
  }
  *out = static_cast<bf16*>(p);
  return EC_OK;
}

static int concat_f32(Device& d, const std::vector<const Tensor*>& parts, float** out) {
  size_t n = 0;
  for (auto* t : parts) n += t->numel;
  void* p;
  int rc = model_alloc(d, &p, n * 4, "f32 vector");
  if (rc) return rc;
  size_t o = 0;
  for (auto* t : parts) {
    if (t->dtype == kDtF32)
      rc = check_cuda(cudaMemcpyAsync(static_cast<float*>(p) + o, t->p, t->numel * 4,
                                      cudaMemcpyDeviceToDevice, d.stream),
                      "vector copy");
    else
      rc = check_cuda(
          launch_convert(kConvBf16ToF32, t->p, static_cast<float*>(p) + o, t->numel, d.stream),
          "vector convert");
    if (rc) return rc;
    o += t->numel;
  }
  *out = static_cast<float*>(p);
  return EC_OK;
}

void graphs_clear(Device& d) {
  for (auto& g : d.graphs) cudaGraphExecDestroy(g.exec);
  d.graphs.clear();
}

void free_model(Device& d) {
  graphs_clear(d);
  for (void* p : d.model.owned) cudaFree(p);
  d.model = ModelW();
}

// bert::mpnet-bucket (bert.lisp:324-331); single-float log computed in double
// and rounded, as SBCL does for (log single-float).
static int mpnet_bucket(int i, int j) {
  const int n = i - j;
  const int an = n < 0 ? -n : n;
  const int ret = n < 0 ? 16 : 0;
  if (an < 8) return ret + an;
  const float a = static_cast<float>(std::log(static_cast<double>(static_cast<float>(an) / 8.0f)));
  const float b = static_cast<float>(std::log(16.0));
  const float v = 8.0f + 8.0f * (a / b);
  const int f = static_cast<int>(std::floor(v));
  return ret + (f < 15 ? f : 15);
}

// ------------------------------------------------------------ load model --
static int cfg_int(const JVal& c, const char* k, int* out, bool required = true, int def = 0) {
  const JVal* v = c.get(k);
  if (!v || !v->is_num()) {
    if (required) return set_error(EC_EINVAL, "config.json lacks %s", k);
    *out = def;
    return EC_OK;
  }
  *out = static_cast<int>(v->num());
  return EC_OK;
}

static int load_bert(Device& d, const JVal& cfg, const std::string& mt, int pooling) {
  ModelW& m = d.model;
  int rc;
  if ((rc = cfg_int(cfg, "hidden_size", &m.H)) || (rc = cfg_int(cfg, "num_hidden_layers", &m.layers)) ||
      (rc = cfg_int(cfg, "num_attention_heads", &m.heads)) ||
      (rc = cfg_int(cfg, "intermediate_size", &m.F)))
    return rc;
  if (m.heads <= 0 || m.H % m.heads) return set_error(EC_EINVAL, "hidden %% heads != 0");
  m.hd = m.H / m.heads;  // bert.lisp:75
  m.kv_heads = m.heads;
  m.pooling = pooling;
  const bool mpnet = mt == "mpnet";
  m.family = mpnet ? EC_FAMILY_MPNET : EC_FAMILY_BERT;
  m.pos_offset = (mpnet || mt == "roberta") ? 2 : 0;  // bert.lisp:294, :477
  if (m.hd != 32 && m.hd != 64 && m.hd != 128)
    return set_error(EC_EUNSUPPORTED, "head dim %d (supported: 32, 64, 128)", m.hd);
  if (m.H % 128 || m.H > 1024 || m.F % 64)
    return set_error(EC_EUNSUPPORTED, "hidden %d / ffn %d outside this build", m.H, m.F);
  const int H = m.H, F = m.F;
  const Tensor *w = nullptr, *p = nullptr, *ty = nullptr, *g = nullptr, *b = nullptr;
  if ((rc = need_t(d, "embeddings.word_embeddings.weight", &w, {})) ||
      (rc = need_t(d, "embeddings.position_embeddings.weight", &p, {})) ||
      (rc = need_t(d, "embeddings.LayerNorm.weight", &g, {H})) ||
      (rc = need_t(d, "embeddings.LayerNorm.bias", &b, {H})))
    return rc;
  if (w->shape.size() != 2 || w->shape[1] != H || p->shape.size() != 2 || p->shape[1] != H)
    return set_error(EC_EINVAL, "embedding tables must be [*, %d]", H);
  m.word = w->p;
  m.word_dt = w->dtype;
  m.vocab = static_cast<int>(w->shape[0]);
  m.pos = p->p;
  m.pos_dt = p->dtype;
  m.max_pos = static_cast<int>(p->shape[0]);
  if (!mpnet) {
    ty = find_t(d, "embeddings.token_type_embeddings.weight");  // bert.lisp:87-89
    if (ty) {
      m.type0 = ty->p;
      m.type_dt = ty->dtype;
    }
  }
  if ((rc = as_f32(d, g, &m.emb_g)) || (rc = as_f32(d, b, &m.emb_b))) return rc;
  if (mpnet) {
    const Tensor* rb = nullptr;
    rc = need_t(d, "encoder.relative_attention_bias.weight", &rb, {32, m.heads});
    if (rc) return rc;
    // table over i - j in [-(rel_max-1), rel_max-1], pre-multiplied by log2(e)
    m.rel_max = 1024;
    const int nb = 2 * m.rel_max - 1;
    std::vector<float> rbh(rb->numel);
    if (rb->dtype == kDtF32) {
      if ((rc = check_cuda(cudaMemcpy(rbh.data(), rb->p, rb->numel * 4, cudaMemcpyDeviceToHost),
                           "rel bias read")))
        return rc;
    } else {
      std::vector<uint16_t> raw(rb->numel);
      if ((rc = check_cuda(cudaMemcpy(raw.data(), rb->p, rb->numel * 2, cudaMemcpyDeviceToHost),
                           "rel bias read")))
        return rc;
      for (size_t i = 0; i < raw.size(); ++i) {
        uint32_t u = static_cast<uint32_t>(raw[i]) << 16;
        std::memcpy(&rbh[i], &u, 4);
      }
    }
    std::vector<float> tab(static_cast<size_t>(m.heads) * nb);
    for (int dlt = -(m.rel_max - 1); dlt <= m.rel_max - 1; ++dlt) {
      const int bk = mpnet_bucket(dlt, 0);
      for (int h = 0; h < m.heads; ++h)
        tab[static_cast<size_t>(h) * nb + dlt + m.rel_max - 1] =
            rbh[static_cast<size_t>(bk) * m.heads + h] * 1.4426950408889634f;
    }
    void* dp;
    if ((rc = model_alloc(d, &dp, tab.size() * 4, "rel bias table"))) return rc;
    if ((rc = check_cuda(cudaMemcpyAsync(dp, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice,
                                         d.stream),
                         "rel bias upload")))
      return rc;
    m.relbias = static_cast<float*>(dp);
    // the table must outlive the async copy of `tab`
    if ((rc = check_cuda(cudaStreamSynchronize(d.stream), "rel bias sync"))) return rc;
  }
  m.bl.resize(m.layers);
  for (int li = 0; li < m.layers; ++li) {
    const std::string pf = "encoder.layer." + std::to_string(li) + ".";
    BertLayerW& L = m.bl[li];
    const Tensor *qw, *qb, *kw, *kb, *vw, *vb, *ow, *ob, *l1g, *l1b, *fw, *fb, *dw, *db, *l2g,
        *l2b;
    const std::string a = mpnet ? "attention.attn." : "attention.self.";
    const std::string qn = mpnet ? "q" : "query", kn = mpnet ? "k" : "key",
                      vn = mpnet ? "v" : "value";
    const std::string on = mpnet ? "attention.attn.o." : "attention.output.dense.";
    const std::string l1 = mpnet ? "attention.LayerNorm." : "attention.output.LayerNorm.";
    if ((rc = need_t(d, pf + a + qn + ".weight", &qw, {H, H})) ||
        (rc = need_t(d, pf + a + qn + ".bias", &qb, {H})) ||
        (rc = need_t(d, pf + a + kn + ".weight", &kw, {H, H})) ||
        (rc = need_t(d, pf + a + kn + ".bias", &kb, {H})) ||
        (rc = need_t(d, pf + a + vn + ".weight", &vw, {H, H})) ||
        (rc = need_t(d, pf + a + vn + ".bias", &vb, {H})) ||
        (rc = need_t(d, pf + on + "weight", &ow, {H, H})) ||
        (rc = need_t(d, pf + on + "bias", &ob, {H})) ||
        (rc = need_t(d, pf + l1 + "weight", &l1g, {H})) ||
        (rc = need_t(d, pf + l1 + "bias", &l1b, {H})) ||
        (rc = need_t(d, pf + "intermediate.dense.weight", &fw, {F, H})) ||
        (rc = need_t(d, pf + "intermediate.dense.bias", &fb, {F})) ||
        (rc = need_t(d, pf + "output.dense.weight", &dw, {H, F})) ||
        (rc = need_t(d, pf + "output.dense.bias", &db, {H})) ||
        (rc = need_t(d, pf + "output.LayerNorm.weight", &l2g, {H})) ||
        (rc = need_t(d, pf + "output.LayerNorm.bias", &l2b, {H})))
      return rc;
    if ((rc = concat_bf16(d, {qw, kw, vw}, H, &L.wqkv)) ||
        (rc = concat_f32(d, {qb, kb, vb}, &L.bqkv)) || (rc = concat_bf16(d, {ow}, H, &L.wo)) ||
        (rc = as_f32(d, ob, &L.bo)) || (rc = as_f32(d, l1g, &L.ln1g)) ||
        (rc = as_f32(d, l1b, &L.ln1b)) || (rc = concat_bf16(d, {fw}, H, &L.wff)) ||
        (rc = as_f32(d, fb, &L.bff)) || (rc = concat_bf16(d, {dw}, F, &L.wout)) ||
        (rc = as_f32(d, db, &L.bout)) || (rc = as_f32(d, l2g, &L.ln2g)) ||
        (rc = as_f32(d, l2b, &L.ln2b)))
      return rc;
  }
  return EC_OK;
}

static int load_llama(Device& d, const JVal& cfg) {
  ModelW& m = d.model;
  int rc;
  if ((rc = cfg_int(cfg, "hidden_size", &m.H)) || (rc = cfg_int(cfg, "num_hidden_layers", &m.layers)) ||
      (rc = cfg_int(cfg, "num_attention_heads", &m.heads)) ||
      (rc = cfg_int(cfg, "intermediate_size", &m.F)))
    return rc;
  if ((rc = cfg_int(cfg, "num_key_value_heads", &m.kv_heads, false, m.heads))) return rc;
  if ((rc = cfg_int(cfg, "head_dim", &m.hd, false, m.heads ? m.H / m.heads : 0))) return rc;
  const JVal* th = cfg.get("rope_theta");
  m.theta = (th && th->is_num()) ? th->num() : 10000.0;   // llama.lisp:184
  const JVal* ep = cfg.get("rms_norm_eps");
  m.eps = (ep && ep->is_num()) ? ep->num() : 1e-6;        // llama.lisp:185
  m.family = EC_FAMILY_LLAMA;
  m.pooling = 2;      // llama::*pooling* :last (llama.lisp:19)
  m.max_pos = 1024;   // llama::*max-pos* (llama.lisp:21)
  if (m.hd != 128) return set_error(EC_EUNSUPPORTED, "llama head_dim %d (supported: 128)", m.hd);
  if (m.kv_heads <= 0 || m.heads % m.kv_heads)
    return set_error(EC_EINVAL, "heads %d not a multiple of kv heads %d", m.heads, m.kv_heads);
  if (m.H % 128 || m.H > 2048 || m.F % 128)
    return set_error(EC_EUNSUPPORTED, "hidden %d / ffn %d outside this build", m.H, m.F);
  const int H = m.H, F = m.F, qd = m.heads * m.hd, kvd = m.kv_heads * m.hd;
  const Tensor *emb, *nw;
  if ((rc = need_t(d, "embed_tokens.weight", &emb, {})) || (rc = need_t(d, "norm.weight", &nw, {H})))
    return rc;
  if (emb->shape.size() != 2 || emb->shape[1] != H)
    return set_error(EC_EINVAL, "embed_tokens must be [*, %d]", H);
  m.word = emb->p;
  m.word_dt = emb->dtype;
  m.vocab = static_cast<int>(emb->shape[0]);
  if ((rc = as_f32(d, nw, &m.final_norm))) return rc;
  // init-rope (llama.lisp:124-135): double table rounded to single
  const int half = m.hd / 2;
  std::vector<float> cs(static_cast<size_t>(m.max_pos) * half), sn(cs.size());
  for (int p = 0; p < m.max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      const double freq = 1.0 / std::pow(m.theta, (2.0 * i) / m.hd);
      const double ang = p * freq;
      cs[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(ang));
      sn[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(ang));
    }
  void *dc, *ds;
  if ((rc = model_alloc(d, &dc, cs.size() * 4, "rope cos")) ||
      (rc = model_alloc(d, &ds, sn.size() * 4, "rope sin")))
    return rc;
  // on the library's stream, waited for before the host tables go away
  if ((rc = check_cuda(cudaMemcpyAsync(dc, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, d.stream),
                       "rope")) ||
      (rc = check_cuda(cudaMemcpyAsync(ds, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, d.stream),
                       "rope")) ||
      (rc = check_cuda(cudaStreamSynchronize(d.stream), "rope")))
    return rc;
  m.cos_t = static_cast<float*>(dc);
  m.sin_t = static_cast<float*>(ds);
  m.ll.resize(m.layers);
  for (int li = 0; li < m.layers; ++li) {
    const std::string pf = "layers." + std::to_string(li) + ".";
    LlamaLayerW& L = m.ll[li];
    const Tensor *in, *post, *qw, *kw, *vw, *ow, *gw, *uw, *dw;
    if ((rc = need_t(d, pf + "input_layernorm.weight", &in, {H})) ||
        (rc = need_t(d, pf + "post_attention_layernorm.weight", &post, {H})) ||
        (rc = need_t(d, pf + "self_attn.q_proj.weight", &qw, {qd, H})) ||
        (rc = need_t(d, pf + "self_attn.k_proj.weight", &kw, {kvd, H})) ||
        (rc = need_t(d, pf + "self_attn.v_proj.weight", &vw, {kvd, H})) ||
        (rc = need_t(d, pf + "self_attn.o_proj.weight", &ow, {H, qd})) ||
        (rc = need_t(d, pf + "mlp.gate_proj.weight", &gw, {F, H})) ||
        (rc = need_t(d, pf + "mlp.up_proj.weight", &uw, {F, H})) ||
        (rc = need_t(d, pf + "mlp.down_proj.weight", &dw, {H, F})))
      return rc;
    const Tensor* qn = find_t(d, pf + "self_attn.q_norm.weight");  // get-tensor-opt
    const Tensor* kn = find_t(d, pf + "self_attn.k_norm.weight");
    if ((rc = as_f32(d, in, &L.in_ln)) || (rc = as_f32(d, post, &L.post_ln)) ||
        (rc = concat_bf16(d, {qw, kw, vw}, H, &L.wqkv)) || (rc = concat_bf16(d, {ow}, qd, &L.wo)) ||
        (rc = concat_bf16(d, {dw}, F, &L.wdown)))
      return rc;
    if (qn && (rc = as_f32(d, qn, &L.q_norm))) return rc;
    if (kn && (rc = as_f32(d, kn, &L.k_norm))) return rc;
    // gate/up interleaved in blocks of 128 rows: [g0 u0 g1 u1 ...], the
    // layout the SwiGLU epilogue of a 256-wide tile expects
    void* p;
    if ((rc = model_alloc(d, &p, static_cast<size_t>(2) * F * H * 2, "gate/up"))) return rc;
    bf16* gu = static_cast<bf16*>(p);
    for (int b = 0; b < F / 128; ++b) {
      if ((rc = rows_to_bf16(d, gw, b * 128, 128, H, gu + static_cast<size_t>(2 * b) * 128 * H)) ||
          (rc = rows_to_bf16(d, uw, b * 128, 128, H,
                             gu + static_cast<size_t>(2 * b + 1) * 128 * H)))
        return rc;
    }
    L.wgu = gu;
  }
  return EC_OK;
}

// RoPE table of gemma::init-rope / llama::init-rope: double, rounded to single
static int rope_table(Device& d, double theta, int hd, int max_pos, float** cos_t, float** sin_t) {
  const int half = hd / 2;
  std::vector<float> cs(static_cast<size_t>(max_pos) * half), sn(cs.size());
  for (int p = 0; p < max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      const double freq = 1.0 / std::pow(theta, (2.0 * i) / hd);
      const double ang = p * freq;
      cs[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(ang));
      sn[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(ang));
    }
  void *dc, *ds;
  int rc;
  if ((rc = model_alloc(d, &dc, cs.size() * 4, "rope cos")) ||
      (rc = model_alloc(d, &ds, sn.size() * 4, "rope sin")))
    return rc;
  // on the library's stream, waited for before the host tables go away
  if ((rc = check_cuda(cudaMemcpyAsync(dc, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, d.stream),
                       "rope")) ||
      (rc = check_cuda(cudaMemcpyAsync(ds, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, d.stream),
                       "rope")) ||
      (rc = check_cuda(cudaStreamSynchronize(d.stream), "rope")))
    return rc;
  *cos_t = static_cast<float*>(dc);
  *sin_t = static_cast<float*>(ds);
  return EC_OK;
}

// gemma:load-model (gemma.lisp:140-212): text_config fields, weights under
// language_model., per-layer head dim from q_norm and kv heads from k_proj;
// RoPE theta 1e6 on full_attention layers, 1e4 otherwise (:173-175).
static int load_gemma(Device& d, const JVal& tc) {
  ModelW& m = d.model;
  int rc;
  if ((rc = cfg_int(tc, "hidden_size", &m.H)) || (rc = cfg_int(tc, "num_hidden_layers", &m.layers)) ||
      (rc = cfg_int(tc, "num_attention_heads", &m.heads)) ||
      (rc = cfg_int(tc, "intermediate_size", &m.F)))
    return rc;
  if ((rc = cfg_int(tc, "hidden_size_per_layer_input", &m.ple_dim, false, m.H)) ||
      (rc = cfg_int(tc, "embedding_dim", &m.out_dim, false, 768)))
    return rc;
  const JVal* ep = tc.get("rms_norm_eps");
  m.eps = (ep && ep->is_num()) ? ep->num() : 1e-6;
  m.family = EC_FAMILY_GEMMA;
  m.pooling = 1;      // gemma::*pooling* :mean
  m.max_pos = 2048;   // gemma::*max-pos*
  const int H = m.H, F = m.F, P = m.ple_dim, NL = m.layers;
  const std::string pre = "language_model.";
  const Tensor *emb = nullptr, *pp = nullptr, *ppn = nullptr, *nw = nullptr, *wo = nullptr;
  if ((rc = need_t(d, pre + "embed_tokens.weight", &emb, {})) ||
      (rc = need_t(d, pre + "ple.per_layer_model_projection.weight", &pp,
                   {static_cast<int64_t>(NL) * P, H})) ||
      (rc = need_t(d, pre + "ple.per_layer_projection_norm.weight", &ppn, {P})) ||
      (rc = need_t(d, pre + "norm.weight", &nw, {H})) ||
      (rc = need_t(d, pre + "embedding_projection.weight", &wo, {m.out_dim, H})))
    return rc;
  if (emb->shape.size() != 2 || emb->shape[1] != H)
    return set_error(EC_EINVAL, "embed_tokens must be [*, %d]", H);
  // head dim / kv heads of layer 0; every layer must agree (one workspace)
  const Tensor *qn0 = nullptr, *k0 = nullptr;
  if ((rc = need_t(d, pre + "layers.0.self_attn.q_norm.weight", &qn0, {})) ||
      (rc = need_t(d, pre + "layers.0.self_attn.k_proj.weight", &k0, {})))
    return rc;
  m.hd = static_cast<int>(qn0->numel);
  m.kv_heads = m.hd ? static_cast<int>(k0->shape[0] / m.hd) : 0;
  if (m.hd != 64 && m.hd != 128)
    return set_error(EC_EUNSUPPORTED, "gemma head_dim %d (this build: 64, 128)", m.hd);
  if (m.kv_heads <= 0 || m.heads % m.kv_heads)
    return set_error(EC_EINVAL, "heads %d not a multiple of kv heads %d", m.heads, m.kv_heads);
  if (H % 128 || P % 128 || F % 128 || ((m.heads + 2 * m.kv_heads) * m.hd) % 64 || H > 2048 ||
      H + m.out_dim > 12288)
    return set_error(EC_EUNSUPPORTED, "gemma widths H %d P %d F %d outside this build", H, P, F);
  m.word = emb->p;
  m.word_dt = emb->dtype;
  m.vocab = static_cast<int>(emb->shape[0]);
  if ((rc = as_f32(d, nw, &m.final_norm)) || (rc = as_f32(d, ppn, &m.ple_norm)) ||
      (rc = as_f32(d, wo, &m.w_out)))
    return rc;
  if ((rc = rope_table(d, 10000.0, m.hd, m.max_pos, &m.cos_t, &m.sin_t)) ||
      (rc = rope_table(d, 1e6, m.hd, m.max_pos, &m.cos2_t, &m.sin2_t)))
    return rc;
  const JVal* types = tc.get("layer_types");
  const int qd = m.heads * m.hd, kvd = m.kv_heads * m.hd;
  m.gl.resize(NL);
  for (int li = 0; li < NL; ++li) {
    const std::string pf = pre + "layers." + std::to_string(li) + ".";
    GemmaLayerW& L = m.gl[li];
    const Tensor *in, *post, *pre_ff, *post_ff, *qw, *kw, *vw, *ow, *qn, *kn, *gw, *uw, *dw, *pg, *pj,
        *pn, *sc;
    if ((rc = need_t(d, pf + "input_layernorm.weight", &in, {H})) ||
        (rc = need_t(d, pf + "post_attention_layernorm.weight", &post, {H})) ||
        (rc = need_t(d, pf + "pre_feedforward_layernorm.weight", &pre_ff, {H})) ||
        (rc = need_t(d, pf + "post_feedforward_layernorm.weight", &post_ff, {H})) ||
        (rc = need_t(d, pf + "self_attn.q_proj.weight", &qw, {qd, H})) ||
        (rc = need_t(d, pf + "self_attn.k_proj.weight", &kw, {kvd, H})) ||
        (rc = need_t(d, pf + "self_attn.v_proj.weight", &vw, {kvd, H})) ||
        (rc = need_t(d, pf + "self_attn.o_proj.weight", &ow, {H, qd})) ||
        (rc = need_t(d, pf + "self_attn.q_norm.weight", &qn, {m.hd})) ||
        (rc = need_t(d, pf + "self_attn.k_norm.weight", &kn, {m.hd})) ||
        (rc = need_t(d, pf + "mlp.gate_proj.weight", &gw, {F, H})) ||
        (rc = need_t(d, pf + "mlp.up_proj.weight", &uw, {F, H})) ||
        (rc = need_t(d, pf + "mlp.down_proj.weight", &dw, {H, F})) ||
        (rc = need_t(d, pf + "ple_block.per_layer_input_gate.weight", &pg, {P, H})) ||
        (rc = need_t(d, pf + "ple_block.per_layer_projection.weight", &pj, {H, P})) ||
        (rc = need_t(d, pf + "ple_block.post_per_layer_input_norm.weight", &pn, {H})) ||
        (rc = need_t(d, pf + "layer_scalar", &sc, {})))
      return rc;
    if (sc->numel < 1) return set_error(EC_EINVAL, "%slayer_scalar is empty", pf.c_str());
    if ((rc = as_f32(d, in, &L.in_ln)) || (rc = as_f32(d, post, &L.post_ln)) ||
        (rc = as_f32(d, pre_ff, &L.pre_ff_ln)) || (rc = as_f32(d, post_ff, &L.post_ff_ln)) ||
        (rc = as_f32(d, qn, &L.q_norm)) || (rc = as_f32(d, kn, &L.k_norm)) ||
        (rc = as_f32(d, pn, &L.ple_norm)) ||
        (rc = concat_bf16(d, {qw, kw, vw}, H, &L.wqkv)) || (rc = concat_bf16(d, {ow}, qd, &L.wo)) ||
        (rc = concat_bf16(d, {dw}, F, &L.wdown)) || (rc = concat_bf16(d, {pg}, H, &L.wple_gate)) ||
        (rc = concat_bf16(d, {pj}, P, &L.wple_proj)))
      return rc;
    // this layer's P rows of the per-layer-embedding projection
    void* p;
    if ((rc = model_alloc(d, &p, static_cast<size_t>(P) * H * 2, "ple rows"))) return rc;
    if ((rc = rows_to_bf16(d, pp, static_cast<int64_t>(li) * P, P, H, static_cast<bf16*>(p))))
      return rc;
    L.wpp = static_cast<bf16*>(p);
    // gate/up interleaved by 128 rows for the gated epilogue
    if ((rc = model_alloc(d, &p, static_cast<size_t>(2) * F * H * 2, "gate/up"))) return rc;
    bf16* gu = static_cast<bf16*>(p);
    for (int b = 0; b < F / 128; ++b) {
      if ((rc = rows_to_bf16(d, gw, b * 128, 128, H, gu + static_cast<size_t>(2 * b) * 128 * H)) ||
          (rc = rows_to_bf16(d, uw, b * 128, 128, H, gu + static_cast<size_t>(2 * b + 1) * 128 * H)))
        return rc;
    }
    L.wgu = gu;
    // the layer scalar, read back once (a [1] tensor of the upload dtype)
    float* scd;
    if ((rc = as_f32(d, sc, &scd))) return rc;
    if ((rc = check_cuda(cudaMemcpy(&L.scalar, scd, 4, cudaMemcpyDeviceToHost), "layer scalar")))
      return rc;
    const JVal* ty = (types && types->kind == JVal::Arr && li < static_cast<int>(types->a.size()))
                         ? &types->a[li]
                         : nullptr;
    L.rope = (ty && ty->kind == JVal::Str && ty->s == "full_attention") ? 1 : 0;
  }
  return EC_OK;
}

int load_model_on(Device& d, const JVal& cfg, const JVal* pool) {
  free_model(d);
  // the workspace is laid out for a model; a new model starts from scratch
  if (d.ws) {
    cudaStreamSynchronize(d.stream);
    dev_free(d, d.ws, d.ws_bytes);
    d.ws = nullptr;
  }
  d.ws_bytes = 0;
  d.ws_tokens = 0;
  d.ws_seqs = 0;
  const JVal* tc = cfg.get("text_config");
  std::string mt;
  if (tc && tc->kind == JVal::Obj && tc->get("model_type") && tc->get("model_type")->kind == JVal::Str)
    mt = tc->get("model_type")->s;  // model.lisp:20-26
  else if (cfg.get("model_type") && cfg.get("model_type")->kind == JVal::Str)
    mt = cfg.get("model_type")->s;
  if (mt.empty()) return set_error(EC_EINVAL, "no config.json model_type");
  int rc;
  if (mt == "bert" || mt == "roberta" || mt == "distilbert" || mt == "mpnet") {
    int pooling = 0;  // :cls unless pooling_mode_mean_tokens (bert.lisp:76-78)
    if (pool && pool->get("pooling_mode_mean_tokens") &&
        pool->get("pooling_mode_mean_tokens")->truthy())
      pooling = 1;
    rc = load_bert(d, cfg, mt, pooling);
  } else if (mt == "llama" || mt == "qwen2" || mt == "qwen3" || mt == "mistral" || mt == "gemma" ||
             mt == "gemma2") {
    rc = load_llama(d, cfg);
  } else if (mt == "embedding_gemma2" || mt == "embedding_gemma2_text") {
    rc = load_gemma(d, tc && tc->kind == JVal::Obj ? *tc : cfg);  // model.lisp:41-43
  } else {
    rc = set_error(EC_EUNSUPPORTED, "unsupported model_type %s", mt.c_str());
  }
  if (rc == EC_OK && d.model.out_dim == 0) d.model.out_dim = d.model.H;
  if (rc == EC_OK) rc = sync_and_check(d, "model assembly");
  if (rc != EC_OK) free_model(d);
  return rc;
}

// --------------------------------------------------------------- forward --
struct WsLayout {
  size_t ids, pos, cu, blocks, blocks128, seqs, h32, tmp, hb, qkv, ctx, ff, out, total;
  size_t h0b = 0, ple = 0, pg = 0, pgb = 0;  // Gemma per-layer-embedding buffers
};

static size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

static WsLayout layout_for(const ModelW& m, size_t T, size_t nseq) {
  WsLayout L;
  const size_t nqkv = static_cast<size_t>(m.heads + 2 * m.kv_heads) * m.hd;
  const size_t nctx = static_cast<size_t>(m.heads) * m.hd;
  const size_t nblk = T / 64 + nseq + 1;
  size_t o = 0;
  L.ids = o; o += al256(T * 4);
  L.pos = o; o += al256(T * 4);
  L.cu = o; o += al256((nseq + 1) * 4);
  L.blocks = o; o += al256(nblk * 8);
  L.blocks128 = o; o += al256((T / 128 + nseq + 1) * 16);
  L.seqs = o; o += al256(nseq * 8);
  L.h32 = o; o += al256(T * m.H * 4);
  L.tmp = o; o += al256(T * m.H * 4);
  L.hb = o; o += al256(T * m.H * 2);
  L.qkv = o; o += al256(T * nqkv * 2);
  L.ctx = o; o += al256(T * nctx * 2);
  L.ff = o; o += al256(T * m.F * 2);
  L.out = o; o += al256(nseq * std::max(m.H, m.out_dim) * 4);
  if (m.family == EC_FAMILY_GEMMA) {
    const size_t P = m.ple_dim;
    L.h0b = o; o += al256(T * m.H * 2);
    L.ple = o; o += al256(T * P * 4);
    L.pg = o; o += al256(T * P * 4);
    L.pgb = o; o += al256(T * P * 2);
  }
  L.total = o;
  return L;
}

// CUDA graphs of whole forwards: batches up to this many tokens, this many
// distinct length sets per device
constexpr int64_t kGraphMaxTokens = 8192;
constexpr size_t kGraphCache = 64;

static int ensure_ws(Device& d, int T, int nseq) {
  // the layout depends on the model (hidden, qkv, ffn widths), so size by
  // bytes, not only by token / sequence counts
  const int t2 = std::max(T, d.ws_tokens), s2 = std::max(nseq, d.ws_seqs);
  const WsLayout L = layout_for(d.model, t2, s2);
  const size_t pin = static_cast<size_t>(t2) * 4 + (static_cast<size_t>(s2) + 1) * 4 +
                     (static_cast<size_t>(t2) / 64 + s2 + 1) * 8 +
                     (static_cast<size_t>(t2) / 128 + s2 + 1) * 16 + static_cast<size_t>(s2) * 8 + 768 +
                     static_cast<size_t>(s2) * std::max(d.model.H, d.model.out_dim) * 4 + 1024;
  if (!d.ws || L.total > d.ws_bytes || t2 != d.ws_tokens || s2 != d.ws_seqs || pin > d.pin_bytes)
    graphs_clear(d);  // the layout or the buffers change
  if (!d.ws || L.total > d.ws_bytes) {
    if (d.ws) {
      cudaStreamSynchronize(d.stream);
      dev_free(d, d.ws, d.ws_bytes);
      d.ws = nullptr;
      d.ws_bytes = 0;
    }
    int rc = dev_alloc(d, &d.ws, L.total, "forward workspace");
    if (rc) return rc;
    d.ws_bytes = L.total;
  }
  d.ws_tokens = t2;
  d.ws_seqs = s2;
  if (pin > d.pin_bytes) {
    if (d.pin) {
      cudaStreamSynchronize(d.stream);
      cudaFreeHost(d.pin);
    }
    d.pin = nullptr;
    d.pin_bytes = 0;
    if (cudaHostAlloc(&d.pin, pin, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      return set_error(EC_ENOMEM, "pinned staging of %zu bytes failed", pin);
    }
    d.pin_bytes = pin;
  }
  return EC_OK;
}

#define EC_TRY(expr)              \
  do {                            \
    int rc_ = (expr);             \
    if (rc_ != EC_OK) return rc_; \
  } while (0)

// Run the forward for sequences seqs[s0..s1) (indices into offsets) that are
// packed in `ids_dev` (already on the device) and write pooled rows to out.
// counts of the uploaded attention tables of one chunk
struct AttnTables {
  int nblk = 0, nblk128 = 0;     // 64-row and 128-row query blocks
  int n_long = 0;                // sequences longer than kAttnShortCap (first in order)
  int nblk128_long = 0;          // their 128-row blocks (a prefix of blocks128)
  int max_short = 0;             // longest sequence of the rest
  std::vector<int> sorted_lens;  // lengths in launch order (descending)
};

static int forward_packed(Device& d, const WsLayout& L, int T, int nseq, const AttnTables& tb,
                          double attn_pairs, float* out, int out_stride) {
  const int nblk = tb.nblk, nblk128 = tb.nblk128;
  ModelW& m = d.model;
  char* ws = static_cast<char*>(d.ws);
  int* ids = reinterpret_cast<int*>(ws + L.ids);
  int* pos = reinterpret_cast<int*>(ws + L.pos);
  int* cu = reinterpret_cast<int*>(ws + L.cu);
  int2* blocks = reinterpret_cast<int2*>(ws + L.blocks);
  float* h32 = reinterpret_cast<float*>(ws + L.h32);
  float* tmp = reinterpret_cast<float*>(ws + L.tmp);
  bf16* hb = reinterpret_cast<bf16*>(ws + L.hb);
  bf16* qkv = reinterpret_cast<bf16*>(ws + L.qkv);
  bf16* ctx = reinterpret_cast<bf16*>(ws + L.ctx);
  bf16* ff = reinterpret_cast<bf16*>(ws + L.ff);
  cudaStream_t st = d.stream;
  const int H = m.H, F = m.F;
  const int nqkv = (m.heads + 2 * m.kv_heads) * m.hd, nctx = m.heads * m.hd;

  // every launch is bracketed by prof_begin / prof_end (events only while
  // profiling): class 0 gemm, 1 attention, 2 row kernels
  auto rows = [&](cudaError_t e, const char* what, double bytes, int e0) -> int {
    prof_end(d, 2, 0.0, bytes, e0);
    trace_launch(d, what);
    return check_cuda(e, what);
  };
  const double TH = static_cast<double>(T) * H;
  {
    const int e0 = prof_begin(d);
    EC_TRY(rows(launch_positions(cu, nseq, pos, st), "positions", T * 4.0, e0));
  }

  auto gemm = [&](const bf16* A, int lda, const bf16* W, int N, int K, const float* bias,
                  const float* resid, void* o, int ldo, int epi,
                  const QkRopeEpi* qk = nullptr, int ldr = 0) -> int {
    GemmLaunch g;
    g.qk = qk;
    g.A = A;
    g.lda = lda;
    g.W = W;
    g.ldw = K;
    g.M = T;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.resid = resid;
    g.ldr = ldr ? ldr : H;
    g.out = o;
    g.ldo = ldo;
    g.epi = epi;
    g.bn = 0;
    g.status = d.status;
    const double out_b = epi == kEpiF32Resid || epi == kEpiF32 ? 4.0 * T * N
                         : epi == kEpiBf16Swiglu || epi == kEpiBf16GeluTanhGate ? 1.0 * T * N
                                                                                : 2.0 * T * N;
    const double bytes = 2.0 * T * K + 2.0 * N * K + out_b + (resid ? 4.0 * T * N : 0.0);
    const int e0 = prof_begin(d);
    const cudaError_t e = launch_gemm(g, st, d.num_sms);
    prof_end(d, 0, 2.0 * T * N * K, bytes, e0);
    trace_launch(d, "gemm");
    return check_cuda(e, "gemm");
  };
  // h32 = LayerNorm(A . W^T + bias + h32), hb = bf16(h32) in one kernel
  // (EC_NO_GEMM_LN keeps the GEMM + separate LayerNorm pair)
  const bool fuse_ln = gemm_ln_supported(H) && getenv("EC_NO_GEMM_LN") == nullptr;
  // post-LayerNorm models with the fused kernel carry the residual between
  // sublayers as the LayerNorm's bf16 output (the row the next GEMM reads
  // anyway); only the last LayerNorm also writes fp32 rows, for pooling.
  // EC_F32_RESIDUAL keeps the fp32 stream everywhere.
  const bool bf16_resid = fuse_ln && getenv("EC_F32_RESIDUAL") == nullptr;
  auto gemm_ln = [&](const bf16* A, int K, const bf16* W, const float* bias, const float* lg,
                     const float* lb, bool out32 = true) -> int {
    GemmLnLaunch g{A, K, W, T, H, K, bias, h32, lg, lb, h32, hb, d.status};
    if (bf16_resid) {
      g.resid = nullptr;
      g.resid_b = hb;
      if (!out32) g.out32 = nullptr;
    }
    const double bytes = 2.0 * T * K + 2.0 * H * K + (bf16_resid ? 2.0 : 4.0) * T * H +
                         (g.out32 ? 6.0 : 2.0) * T * H;
    const int e0 = prof_begin(d);
    const cudaError_t e = launch_gemm_ln(g, st, d.num_sms);
    prof_end(d, 0, 2.0 * T * H * K, bytes, e0);
    trace_launch(d, "gemm+layernorm");
    return check_cuda(e, "gemm+layernorm");
  };
  // out32 / outb = an RMSNorm-family epilogue of A . W^T on N = H columns
  // (GemmNorm modes 1-3, see GemmLnLaunch)
  auto gemm_norm = [&](const bf16* A, int K, const bf16* W, int mode, const float* resid,
                       const float* g1, const float* g2, float* o32, bf16* ob, float scale,
                       int has_scale, int N) -> int {
    GemmLnLaunch g{A, K, W, T, N, K, nullptr, resid, g1, g2, o32, ob, d.status};
    g.mode = mode;
    g.eps = static_cast<float>(m.eps);
    g.scale = scale;
    g.has_scale = has_scale;
    const double bytes = 2.0 * T * K + 2.0 * N * K + (resid ? 4.0 * T * N : 0.0) +
                         (o32 ? 4.0 * T * N : 0.0) + (ob ? 2.0 * T * N : 0.0);
    const int e0 = prof_begin(d);
    const cudaError_t e = launch_gemm_ln(g, st, d.num_sms);
    prof_end(d, 0, 2.0 * T * N * K, bytes, e0);
    trace_launch(d, "gemm+rmsnorm");
    return check_cuda(e, "gemm+rmsnorm");
  };
  AttnLaunch at;
  at.qkv = qkv;
  at.ld = nqkv;
  at.q_off = 0;
  at.k_off = m.heads * m.hd;
  at.v_off = (m.heads + m.kv_heads) * m.hd;
  at.out = ctx;
  at.ldo = nctx;
  at.cu = cu;
  at.blocks = blocks;
  at.nblocks = nblk;
  at.heads = m.heads;
  at.kv_group = m.heads / m.kv_heads;
  at.head_dim = m.hd;
  at.causal = m.family == EC_FAMILY_LLAMA ? 1 : 0;
  at.relbias = m.relbias;
  at.rel_max = m.rel_max;
  at.blocks128 = reinterpret_cast<const int4*>(ws + L.blocks128);
  at.nblocks128 = nblk128;
  at.seqs = reinterpret_cast<const int2*>(ws + L.seqs);
  at.nseq = nseq;
  at.n_long = tb.n_long;
  at.nblocks128_long = tb.nblk128_long;
  at.max_short_len = tb.max_short;
  if (!tb.sorted_lens.empty()) attn_short_buckets(tb.sorted_lens.data(), tb.n_long, nseq, &at);
  at.rows = T;
  at.status = d.status;
  at.num_sms = d.num_sms;
  auto attention = [&]() -> int {
    const int e0 = prof_begin(d);
    const cudaError_t e = launch_attention(at, st);
    prof_end(d, 1, attn_pairs * 4.0 * m.heads * m.hd, 2.0 * T * (nqkv + nctx), e0);
    trace_launch(d, "attention");
    return check_cuda(e, "attention");
  };

  if (m.family == EC_FAMILY_BERT || m.family == EC_FAMILY_MPNET) {
    EmbedLnArgs e;
    e.ids = ids;
    e.pos = pos;
    e.pos_offset = m.pos_offset;
    e.word = m.word;
    e.word_dtype = m.word_dt;
    e.posemb = m.pos;
    e.pos_dtype = m.pos_dt;
    e.type0 = m.family == EC_FAMILY_BERT ? m.type0 : nullptr;
    e.type_dtype = m.type_dt;
    e.g = m.emb_g;
    e.b = m.emb_b;
    e.out32 = bf16_resid && m.layers > 0 ? nullptr : h32;
    e.outb = hb;
    e.T = T;
    e.H = H;
    {
      const int e0 = prof_begin(d);
      EC_TRY(rows(launch_embed_ln(e, st), "embed", TH * (8.0 + 6.0), e0));
    }
    // a few rows (a query, a handful of short texts): the skinny GEMMs,
    // weights spread over the whole GPU, and the LayerNorm row kernel
    // (EC_NO_SKINNY: the tcgen05 GEMMs at every size)
    const bool skinny = T <= kSkinnyRows && getenv("EC_NO_SKINNY") == nullptr;
    auto sk = [&](const bf16* A, int lda, const bf16* W, int N, int K, const float* bias, int epi, void* o,
                  int ldo) -> int {
      SkinnyLaunch s{A, lda, W, T, N, K, bias, bf16_resid ? nullptr : h32, hb, H, o, ldo, epi};
      const int e0 = prof_begin(d);
      const cudaError_t e = launch_skinny_gemm(s, st);
      prof_end(d, 0, 2.0 * T * N * K, 2.0 * T * K + 2.0 * N * K + (epi == kSkF32Resid ? 8.0 : 2.0) * T * N, e0);
      trace_launch(d, "skinny gemm");
      return check_cuda(e, "skinny gemm");
    };
    auto ln_rows = [&](const float* g, const float* b) -> int {
      LnArgs l{tmp, g, b, h32, hb, T, H};
      const int e0 = prof_begin(d);
      return rows(launch_ln(l, st), "layernorm", TH * 10.0, e0);
    };
    for (int li = 0; li < m.layers; ++li) {
      const BertLayerW& w = m.bl[li];
      if (skinny) {
        EC_TRY(sk(hb, H, w.wqkv, nqkv, H, w.bqkv, kSkBf16, qkv, nqkv));
        EC_TRY(attention());
        EC_TRY(sk(ctx, nctx, w.wo, H, nctx, w.bo, kSkF32Resid, tmp, H));
        EC_TRY(ln_rows(w.ln1g, w.ln1b));
        EC_TRY(sk(hb, H, w.wff, F, H, w.bff, kSkGelu, ff, F));
        EC_TRY(sk(ff, F, w.wout, H, F, w.bout, kSkF32Resid, tmp, H));
        EC_TRY(ln_rows(w.ln2g, w.ln2b));
        continue;
      }
      EC_TRY(gemm(hb, H, w.wqkv, nqkv, H, w.bqkv, nullptr, qkv, nqkv, kEpiBf16));
      EC_TRY(attention());
      if (fuse_ln) {
        EC_TRY(gemm_ln(ctx, nctx, w.wo, w.bo, w.ln1g, w.ln1b, false));
      } else {
        EC_TRY(gemm(ctx, nctx, w.wo, H, nctx, w.bo, h32, tmp, H, kEpiF32Resid));
        LnArgs l1{tmp, w.ln1g, w.ln1b, h32, hb, T, H};
        const int e0 = prof_begin(d);
        EC_TRY(rows(launch_ln(l1, st), "layernorm", TH * 10.0, e0));
      }
      // the fused block: opt-in (EC_FUSED_MLP) until it beats the unfused pair
      if (mlp_supported(H, F) && fuse_ln && getenv("EC_FUSED_MLP")) {
        // up + GELU + down + bias + residual + LayerNorm in one kernel; the
        // residual is the bf16 input rows (or the fp32 stream), the fp32 row
        // is stored where the unfused path stores it
        const bool want32 = !bf16_resid || li + 1 == m.layers;
        MlpLaunch ml{hb, w.wff, w.wout, w.bff, w.bout, bf16_resid ? nullptr : h32, w.ln2g, w.ln2b,
                     want32 ? h32 : nullptr, hb, T, H, F, d.status};
        const int e0 = prof_begin(d);
        const cudaError_t e = launch_mlp(ml, st, d.num_sms);
        prof_end(d, 0, 4.0 * T * H * F,
                 2.0 * T * H + 4.0 * H * F + (bf16_resid ? 2.0 : 4.0) * T * H + (want32 ? 6.0 : 2.0) * T * H,
                 e0);
        EC_TRY(check_cuda(e, "fused mlp"));
      } else {
        EC_TRY(gemm(hb, H, w.wff, F, H, w.bff, nullptr, ff, F, kEpiBf16Gelu));
        if (fuse_ln) {
          EC_TRY(gemm_ln(ff, F, w.wout, w.bout, w.ln2g, w.ln2b, li + 1 == m.layers));
        } else {
          EC_TRY(gemm(ff, F, w.wout, H, F, w.bout, h32, tmp, H, kEpiF32Resid));
          LnArgs l2{tmp, w.ln2g, w.ln2b, h32, hb, T, H};
          const int e0 = prof_begin(d);
          EC_TRY(rows(launch_ln(l2, st), "layernorm", TH * 10.0, e0));
        }
      }
    }
    PoolArgs pa;
    pa.h = h32;
    pa.cu = cu;
    pa.mode = m.pooling;
    pa.final_norm = 0;
    pa.norm_w = nullptr;
    pa.eps = 0.0;
    pa.out = out;
    pa.out_stride = out_stride;
    pa.H = H;
    {
      const int e0 = prof_begin(d);
      EC_TRY(rows(launch_pool_l2(pa, nseq, st), "pool",
                  (m.pooling == 1 ? TH : static_cast<double>(nseq) * H) * 4.0, e0));
    }
    return EC_OK;
  }
  if (m.family == EC_FAMILY_GEMMA) {
    // gemma::embed / layer-forward (gemma.lisp:216-376)
    const int P = m.ple_dim;
    bf16* h0b = reinterpret_cast<bf16*>(ws + L.h0b);
    float* ple = reinterpret_cast<float*>(ws + L.ple);
    float* pg = reinterpret_cast<float*>(ws + L.pg);
    bf16* pgb = reinterpret_cast<bf16*>(ws + L.pgb);
    at.scale = 1.0f;  // bidirectional attention with scale 1.0 (gemma.lisp:250-265)
    at.causal = 0;
    // the start event is recorded before the launch (the launcher is
    // called inside)
    auto row = [&](auto&& launch, const char* what, double bytes) -> int {
      const int e0 = prof_begin(d);
      const cudaError_t e = launch();
      return rows(e, what, bytes, e0);
    };
    {
      GemmaEmbedArgs ea{ids, m.word, m.word_dt, sqrtf(static_cast<float>(H)), h32, h0b, T, H};
      EC_TRY(row([&] { return launch_gemma_embed(ea, st); }, "gemma embed", TH * 10.0));
    }
    const float inv_sqrt_h = 1.0f / sqrtf(static_cast<float>(H));
    const bool fuse_qkv_norm = m.hd == 128 && nqkv % 256 == 0 && getenv("EC_NO_FUSED_ROPE") == nullptr;
    // the post-norm residual adds and the per-layer-input norm in the
    // epilogues of the GEMMs that produce them (clusters over the full row);
    // EC_NO_GEMM_RMS keeps fp32 GEMM outputs + the row kernels
    const bool fuse_rms = gemm_rms_supported(H) && gemm_rms_supported(P) &&
                          getenv("EC_NO_GEMM_RMS") == nullptr;
    for (int li = 0; li < m.layers; ++li) {
      const GemmaLayerW& w = m.gl[li];
      // attention sub-block; the input RMSNorm of layers after the first
      // came out of the previous layer's last residual add
      if (li == 0) {
        RmsArgs r1{h32, nullptr, w.in_ln, m.eps, hb, nullptr, T, H};
        EC_TRY(row([&] { return launch_rmsnorm(r1, st); }, "rmsnorm", TH * 6.0));
      }
      const float* cos_l = w.rope ? m.cos2_t : m.cos_t;
      const float* sin_l = w.rope ? m.sin2_t : m.sin_t;
      if (fuse_qkv_norm) {
        // q/k RMSNorm + RoPE and the v RMSNorm in the QKV GEMM's epilogue
        QkRopeEpi qe{w.q_norm, w.k_norm, m.heads, m.kv_heads, m.eps, pos, cos_l, sin_l};
        qe.v_heads = m.kv_heads;
        qe.v_norm = 1;
        EC_TRY(gemm(hb, H, w.wqkv, nqkv, H, nullptr, nullptr, qkv, nqkv, kEpiBf16QkRope, &qe));
      } else {
        EC_TRY(gemm(hb, H, w.wqkv, nqkv, H, nullptr, nullptr, qkv, nqkv, kEpiBf16));
        HeadNormRopeArgs hr{qkv, nqkv, m.heads, m.kv_heads, m.hd, w.q_norm, w.k_norm, m.eps, pos,
                            cos_l, sin_l, T};
        EC_TRY(row([&] { return launch_head_norm_rope(hr, st); }, "head norm rope",
                   4.0 * T * nqkv));
      }
      EC_TRY(attention());
      if (fuse_rms) {
        // h = h + RMSNorm(o) * g, hb = RMSNorm(h) * g' in the O GEMM
        EC_TRY(gemm_norm(ctx, nctx, w.wo, 2, h32, w.post_ln, w.pre_ff_ln, h32, hb, 1.f, 0, H));
      } else {
        EC_TRY(gemm(ctx, nctx, w.wo, H, nctx, nullptr, nullptr, tmp, H, kEpiF32));
        NormAddArgs na1{tmp, w.post_ln, h32, 0, 1.f, w.pre_ff_ln, hb, m.eps, T, H};
        EC_TRY(row([&] { return launch_norm_add(na1, st); }, "norm add", TH * 14.0));
      }
      // gated GELU-tanh MLP
      EC_TRY(gemm(hb, H, w.wgu, 2 * F, H, nullptr, nullptr, ff, F, kEpiBf16GeluTanhGate));
      if (fuse_rms) {
        // h = h + RMSNorm(down) * g, hb = bf16(h) (the PLE gate's input)
        EC_TRY(gemm_norm(ff, F, w.wdown, 2, h32, w.post_ff_ln, nullptr, h32, hb, 1.f, 0, H));
      } else {
        EC_TRY(gemm(ff, F, w.wdown, H, F, nullptr, nullptr, tmp, H, kEpiF32));
        NormAddArgs na2{tmp, w.post_ff_ln, h32, 0, 1.f, nullptr, hb, m.eps, T, H};
        EC_TRY(row([&] { return launch_norm_add(na2, st); }, "norm add", TH * 14.0));
      }
      // per-layer embedding of this layer from the scaled token embedding
      if (fuse_rms) {
        EC_TRY(gemm_norm(h0b, H, w.wpp, 3, nullptr, m.ple_norm, nullptr, ple, nullptr, inv_sqrt_h,
                         0, P));
      } else {
        EC_TRY(gemm(h0b, H, w.wpp, P, H, nullptr, nullptr, ple, P, kEpiF32));
        PlePrepArgs pa{ple, inv_sqrt_h, m.ple_norm, m.eps, T, P};
        EC_TRY(row([&] { return launch_ple_prep(pa, st); }, "ple prep", 8.0 * T * P));
      }
      // PLE block: gate(h) -> GELU-tanh * ple -> projection -> norm -> residual
      // gelu-tanh(gate(h)) * ple straight out of the gate GEMM's epilogue
      // (EC_NO_FUSED_PLE_GATE: fp32 gate, then the row kernel)
      if (getenv("EC_NO_FUSED_PLE_GATE") == nullptr) {
        EC_TRY(gemm(hb, H, w.wple_gate, P, H, nullptr, ple, pgb, P, kEpiBf16GeluTanhMul, nullptr,
                    P));
      } else {
        EC_TRY(gemm(hb, H, w.wple_gate, P, H, nullptr, nullptr, pg, P, kEpiF32));
        PleGateArgs pga{pg, ple, pgb, T, P};
        EC_TRY(row([&] { return launch_ple_gate(pga, st); }, "ple gate", 10.0 * T * P));
      }
      // h = (h + RMSNorm(ple)) * layer_scalar, and hb = the next layer's
      // input RMSNorm of it
      const bool more = li + 1 < m.layers;
      if (fuse_rms) {
        EC_TRY(gemm_norm(pgb, P, w.wple_proj, 2, h32, w.ple_norm,
                         more ? m.gl[li + 1].in_ln : nullptr, h32, more ? hb : nullptr, w.scalar,
                         1, H));
      } else {
        EC_TRY(gemm(pgb, P, w.wple_proj, H, P, nullptr, nullptr, tmp, H, kEpiF32));
        NormAddArgs na3{tmp, w.ple_norm, h32, 1, w.scalar, more ? m.gl[li + 1].in_ln : nullptr,
                        more ? hb : nullptr, m.eps, T, H};
        EC_TRY(row([&] { return launch_norm_add(na3, st); }, "norm add scale",
                   TH * (more ? 14.0 : 12.0)));
      }
    }
    // final RMSNorm per token, then mean pool + projection + L2
    RmsArgs rf{h32, nullptr, m.final_norm, m.eps, nullptr, h32, T, H};
    EC_TRY(row([&] { return launch_rmsnorm(rf, st); }, "final rmsnorm", TH * 8.0));
    GemmaPoolArgs gp{h32, cu, m.w_out, out, out_stride, H, m.out_dim};
    EC_TRY(row([&] { return launch_gemma_pool(gp, nseq, st); }, "pool project", TH * 4.0));
    return EC_OK;
  }
  // llama family: h = embed_tokens[ids] (llama.lisp:316-320)
  {
    const int e0 = prof_begin(d);
    EC_TRY(rows(launch_gather_rows(m.word, m.word_dt, ids, h32, T, H, st), "gather",
                TH * (m.word_dt == kDtBf16 ? 6.0 : 8.0), e0));
  }
  // q/k norm + RoPE fused into the QKV GEMM (head dim 128, heads in 256-wide
  // tiles); EC_NO_FUSED_ROPE keeps the separate row kernel
  const bool fuse_rope = m.hd == 128 && nqkv % 256 == 0 && getenv("EC_NO_FUSED_ROPE") == nullptr;
  // EC_GEMM_RES_RMS (opt-in): the residual adds and the next pre-norm in the
  // O / down GEMMs' cluster epilogue (h32 += x, hb = RMSNorm(h32) * g;
  // GemmNorm mode 1); the first layer's input norm stays a row kernel, the
  // last layer's down GEMM only adds (the final norm is the pooled token's).
  // Measured 9% slower on the Qwen3-0.6B batch than the CTA-pair GEMMs plus
  // the RMSNorm row kernel, which stay the default.
  const bool fuse_res_rms = fuse_rope && gemm_rms_supported(H) && getenv("EC_GEMM_RES_RMS") != nullptr;
  for (int li = 0; li < m.layers; ++li) {
    const LlamaLayerW& w = m.ll[li];
    if (li == 0 || !fuse_res_rms) {
      RmsArgs r1{h32, nullptr, w.in_ln, m.eps, hb, nullptr, T, H};
      const int e0 = prof_begin(d);
      EC_TRY(rows(launch_rmsnorm(r1, st), "rmsnorm", TH * 6.0, e0));
    }
    if (fuse_rope) {
      // QKV projection with the per-head q/k RMSNorm and RoPE in its epilogue
      const QkRopeEpi qe{w.q_norm, w.k_norm, m.heads, m.kv_heads, m.eps, pos, m.cos_t, m.sin_t};
      EC_TRY(gemm(hb, H, w.wqkv, nqkv, H, nullptr, nullptr, qkv, nqkv, kEpiBf16QkRope, &qe));
      EC_TRY(attention());
      if (fuse_res_rms) {
        EC_TRY(gemm_norm(ctx, nctx, w.wo, 1, h32, w.post_ln, nullptr, h32, hb, 1.f, 0, H));
      } else {
        EC_TRY(gemm(ctx, nctx, w.wo, H, nctx, nullptr, h32, h32, H, kEpiF32Resid));
        RmsArgs r2f{h32, nullptr, w.post_ln, m.eps, hb, nullptr, T, H};
        const int e0 = prof_begin(d);
        EC_TRY(rows(launch_rmsnorm(r2f, st), "rmsnorm", TH * 6.0, e0));
      }
      EC_TRY(gemm(hb, H, w.wgu, 2 * F, H, nullptr, nullptr, ff, F, kEpiBf16Swiglu));
      if (fuse_res_rms && li + 1 < m.layers)
        EC_TRY(gemm_norm(ff, F, w.wdown, 1, h32, m.ll[li + 1].in_ln, nullptr, h32, hb, 1.f, 0, H));
      else
        EC_TRY(gemm(ff, F, w.wdown, H, F, nullptr, h32, h32, H, kEpiF32Resid));
      continue;
    }
    EC_TRY(gemm(hb, H, w.wqkv, nqkv, H, nullptr, nullptr, qkv, nqkv, kEpiBf16));
    QkRopeArgs q;
    q.qkv = qkv;
    q.ld = nqkv;
    q.q_off = 0;
    q.k_off = m.heads * m.hd;
    q.q_heads = m.heads;
    q.k_heads = m.kv_heads;
    q.q_norm = w.q_norm;
    q.k_norm = w.k_norm;
    q.eps = m.eps;
    q.pos = pos;
    q.cos_t = m.cos_t;
    q.sin_t = m.sin_t;
    q.T = T;
    {
      const int e0 = prof_begin(d);
      EC_TRY(rows(launch_qk_norm_rope(q, st), "qk norm rope",
                  4.0 * T * (m.heads + m.kv_heads) * m.hd, e0));
    }
    EC_TRY(attention());
    EC_TRY(gemm(ctx, nctx, w.wo, H, nctx, nullptr, h32, h32, H, kEpiF32Resid));
    RmsArgs r2{h32, nullptr, w.post_ln, m.eps, hb, nullptr, T, H};
    {
      const int e0 = prof_begin(d);
      EC_TRY(rows(launch_rmsnorm(r2, st), "rmsnorm", TH * 6.0, e0));
    }
    EC_TRY(gemm(hb, H, w.wgu, 2 * F, H, nullptr, nullptr, ff, F, kEpiBf16Swiglu));
    EC_TRY(gemm(ff, F, w.wdown, H, F, nullptr, h32, h32, H, kEpiF32Resid));
  }
  PoolArgs pa;
  pa.h = h32;
  pa.cu = cu;
  pa.mode = m.pooling;
  pa.final_norm = 1;
  pa.norm_w = m.final_norm;
  pa.eps = m.eps;
  pa.out = out;
  pa.out_stride = out_stride;
  pa.H = H;
  {
    const int e0 = prof_begin(d);
    EC_TRY(rows(launch_pool_l2(pa, nseq, st), "pool", static_cast<double>(nseq) * H * 4.0, e0));
  }
  return EC_OK;
}

// Build the per-chunk host tables (cu offsets, attention blocks sorted by
// descending length) into pinned staging (fill_tables), and enqueue their
// upload (copy_tables).  The staging layout depends only on the lengths.
static void fill_tables(Device& d, const std::vector<int>& lens, AttnTables* tb) {
  const int nseq = static_cast<int>(lens.size());
  char* pin = static_cast<char*>(d.pin);
  int* hcu = reinterpret_cast<int*>(pin);
  int2* hblk = reinterpret_cast<int2*>(pin + al256((nseq + 1) * 4));
  hcu[0] = 0;
  for (int i = 0; i < nseq; ++i) hcu[i + 1] = hcu[i] + lens[i];
  std::vector<int> order(nseq);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lens[a] > lens[b]; });
  int nb = 0;
  for (int s : order)
    for (int q0 = 0; q0 < lens[s]; q0 += 64) hblk[nb++] = make_int2(s, q0);
  int4* hblk128 = reinterpret_cast<int4*>(reinterpret_cast<char*>(hblk) + al256(static_cast<size_t>(nb) * 8));
  int nb128 = 0;
  for (int s : order) {
    for (int q0 = 0; q0 < lens[s]; q0 += 128) hblk128[nb128++] = make_int4(hcu[s], lens[s], q0, 0);
    if (lens[s] > kAttnShortCap) {
      ++tb->n_long;
      tb->nblk128_long = nb128;
    } else {
      tb->max_short = std::max(tb->max_short, lens[s]);
    }
  }
  int2* hseq = reinterpret_cast<int2*>(reinterpret_cast<char*>(hblk128) + al256(static_cast<size_t>(nb128) * 16));
  for (int k = 0; k < nseq; ++k) hseq[k] = make_int2(hcu[order[k]], lens[order[k]]);
  tb->sorted_lens.resize(nseq);
  for (int k = 0; k < nseq; ++k) tb->sorted_lens[k] = lens[order[k]];
  tb->nblk = nb;
  tb->nblk128 = nb128;
}

static int copy_tables(Device& d, const WsLayout& L, int nseq, const AttnTables& tb) {
  char* pin = static_cast<char*>(d.pin);
  const int nb = tb.nblk, nb128 = tb.nblk128;
  const char* hcu = pin;
  const char* hblk = pin + al256((nseq + 1) * 4);
  const char* hblk128 = hblk + al256(static_cast<size_t>(nb) * 8);
  const char* hseq = hblk128 + al256(static_cast<size_t>(nb128) * 16);
  char* ws = static_cast<char*>(d.ws);
  EC_TRY(check_cuda(cudaMemcpyAsync(ws + L.seqs, hseq, static_cast<size_t>(nseq) * 8,
                                    cudaMemcpyHostToDevice, d.stream),
                    "sequence upload"));
  EC_TRY(check_cuda(cudaMemcpyAsync(ws + L.blocks128, hblk128, static_cast<size_t>(nb128) * 16,
                                    cudaMemcpyHostToDevice, d.stream),
                    "block upload"));
  EC_TRY(check_cuda(cudaMemcpyAsync(ws + L.cu, hcu, (nseq + 1) * 4, cudaMemcpyHostToDevice, d.stream),
                    "cu upload"));
  EC_TRY(check_cuda(cudaMemcpyAsync(ws + L.blocks, hblk, static_cast<size_t>(nb) * 8,
                                    cudaMemcpyHostToDevice, d.stream),
                    "block upload"));
  return EC_OK;
}


int embed_on_device(Device& d, const int32_t* ids_host, const int32_t* ids_dev,
                    const std::vector<int>& seqs, const int64_t* offsets, float* out_host,
                    int out_stride, float* out_dev) {
  ModelW& m = d.model;
  if (!m.family) return set_error(EC_ESTATE, "no model loaded");
  EC_TRY(check_cuda(cudaSetDevice(d.ordinal), "set device"));
  // EC_TRACE_EMBED: host time of each phase of the call on stderr
  static const bool trace = getenv("EC_TRACE_EMBED") != nullptr;
  auto t_last = std::chrono::steady_clock::now();
  auto tmark = [&](const char* what) {
    if (!trace) return;
    const auto now = std::chrono::steady_clock::now();
    fprintf(stderr, "[ec embed dev %d] %s %.3f ms\n", d.ordinal, what,
            std::chrono::duration<double, std::milli>(now - t_last).count());
    t_last = now;
  };
  // validate lengths and ids (host ids only; device ids are trusted)
  const int maxlen = m.family == EC_FAMILY_LLAMA ? m.max_pos : m.max_pos - m.pos_offset;
  for (int s : seqs) {
    const int64_t L = offsets[s + 1] - offsets[s];
    if (offsets[s] < 0)  // before the start of the ids (host or device)
      return set_error(EC_EINVAL, "sequence %d starts at offset %lld", s, static_cast<long long>(offsets[s]));
    if (L <= 0) return set_error(EC_EINVAL, "sequence %d is empty", s);
    if (L > maxlen)
      return set_error(EC_EINVAL, "sequence %d has %lld tokens, above the %d positions of the model",
                       s, static_cast<long long>(L), maxlen);
    if (m.family == EC_FAMILY_MPNET && L > 512)
      return set_error(EC_EUNSUPPORTED, "MPNet sequence %d longer than 512 tokens", s);
    if (ids_host) {
      // min / max over the sequence's ids (a vectorisable pass); the slow
      // search for the message only when one is out of range
      int32_t lo = INT32_MAX, hi = INT32_MIN;
      for (int64_t t = offsets[s]; t < offsets[s + 1]; ++t) {
        lo = std::min(lo, ids_host[t]);
        hi = std::max(hi, ids_host[t]);
      }
      if (lo < 0 || hi >= m.vocab)
        for (int64_t t = offsets[s]; t < offsets[s + 1]; ++t)
          if (ids_host[t] < 0 || ids_host[t] >= m.vocab)
            return set_error(EC_EINVAL, "token id %d of sequence %d outside vocab %d", ids_host[t],
                             s, m.vocab);
    }
  }
  tmark("validate");
  size_t i = 0;
  while (i < seqs.size()) {
    // chunk: as many sequences as fit the token budget (at least one)
    size_t j = i;
    int64_t T = 0;
    while (j < seqs.size()) {
      const int64_t L = offsets[seqs[j] + 1] - offsets[seqs[j]];
      if (j > i && T + L > G().max_tokens) break;
      T += L;
      ++j;
    }
    if (ids_dev) {
      // device ids must be one contiguous range of consecutive sequences
      for (size_t k = i + 1; k < j; ++k)
        if (seqs[k] != seqs[k - 1] + 1) return set_error(EC_EINVAL, "non-contiguous device chunk");
    }
    const int nseq = static_cast<int>(j - i);
    EC_TRY(ensure_ws(d, static_cast<int>(T), nseq));
    WsLayout L = layout_for(m, d.ws_tokens, d.ws_seqs);
    std::vector<int> lens(nseq);
    for (int k = 0; k < nseq; ++k)
      lens[k] = static_cast<int>(offsets[seqs[i + k] + 1] - offsets[seqs[i + k]]);
    AttnTables tb;
    char* ws = static_cast<char*>(d.ws);
    // pinned layout: tables at the front, ids at the back, outputs below them
    int* hid = reinterpret_cast<int*>(static_cast<char*>(d.pin) + d.pin_bytes -
                                      al256(static_cast<size_t>(T) * 4) - 256);
    const size_t obytes = static_cast<size_t>(nseq) * m.out_dim * 4;
    float* hout = reinterpret_cast<float*>(static_cast<char*>(d.pin) + d.pin_bytes -
                                           al256(static_cast<size_t>(T) * 4) - 256 - al256(obytes));
    // consecutive sequences: their ids and output rows are contiguous in
    // the caller's arrays, which the copies then use directly
    bool contig = true;
    for (int k = 1; k < nseq && contig; ++k) contig = seqs[i + k] == seqs[i + k - 1] + 1;
    const bool graph = ids_host && !out_dev && j - i == seqs.size() && T <= kGraphMaxTokens &&
                       !G().profile && !G().sync_each && getenv("EC_NO_GRAPH") == nullptr;
    const bool direct = contig && !graph;
    const bool direct_out = direct && !out_dev && out_stride == m.out_dim;
    if (ids_host && !direct) {
      int64_t o = 0;
      for (int k = 0; k < nseq; ++k) {
        const int s = seqs[i + k];
        std::memcpy(hid + o, ids_host + offsets[s], static_cast<size_t>(lens[k]) * 4);
        o += lens[k];
      }
    }
    float* dout = out_dev ? out_dev + static_cast<size_t>(seqs[i]) * out_stride
                          : reinterpret_cast<float*>(ws + L.out);
    const int ostride = out_dev ? out_stride : m.out_dim;
    double pairs = 0.0;  // (query, key) pairs that attention scores
    for (int k = 0; k < nseq; ++k)
      pairs += m.family == EC_FAMILY_LLAMA ? 0.5 * lens[k] * (lens[k] + 1.0)
                                           : static_cast<double>(lens[k]) * lens[k];
    // the stream work of this chunk: tables and ids up, forward, rows down
    auto enqueue = [&]() -> int {
      EC_TRY(copy_tables(d, L, nseq, tb));
      if (ids_dev) {
        EC_TRY(check_cuda(cudaMemcpyAsync(ws + L.ids, ids_dev + offsets[seqs[i]],
                                          static_cast<size_t>(T) * 4, cudaMemcpyDeviceToDevice,
                                          d.stream),
                          "ids copy"));
      } else {
        EC_TRY(check_cuda(cudaMemcpyAsync(ws + L.ids, direct ? ids_host + offsets[seqs[i]] : hid,
                                          static_cast<size_t>(T) * 4, cudaMemcpyHostToDevice, d.stream),
                          "ids upload"));
      }
      EC_TRY(forward_packed(d, L, static_cast<int>(T), nseq, tb, pairs, dout, ostride));
      if (!out_dev)
        EC_TRY(check_cuda(cudaMemcpyAsync(direct_out ? out_host + static_cast<size_t>(seqs[i]) * out_stride : hout,
                                          dout, obytes, cudaMemcpyDeviceToHost, d.stream),
                          "output download"));
      return EC_OK;
    };
    fill_tables(d, lens, &tb);
    tmark("staging (ids, tables)");
    // Small host batches (query serving) replay a CUDA graph of the whole
    // chunk, captured at the first batch with these lengths on this
    // workspace: one launch in place of ~30, the host writes only the pinned
    // tables and ids.  Not while profiling or checking every launch.
    Device::FwdGraph* g = nullptr;
    if (graph) {
      for (auto& e : d.graphs)
        if (e.lens == lens && e.ws == d.ws && e.ws_tokens == d.ws_tokens && e.ws_seqs == d.ws_seqs &&
            e.pin == d.pin && e.pin_bytes == d.pin_bytes) {
          g = &e;
          break;
        }
      if (!g) {
        cudaGraph_t cg = nullptr;
        EC_TRY(check_cuda(cudaStreamBeginCapture(d.stream, cudaStreamCaptureModeRelaxed), "graph capture"));
        // the captured forward is launched plainly: programmatic edges made
        // the replayed 10-token query slower (0.367 -> 0.383 ms p50)
        pdl_set_thread(false);
        const int rc = enqueue();
        pdl_set_thread(true);
        const cudaError_t ce = cudaStreamEndCapture(d.stream, &cg);
        if (rc) {
          if (cg) cudaGraphDestroy(cg);
          return rc;
        }
        EC_TRY(check_cuda(ce, "graph capture"));
        cudaGraphExec_t ex = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&ex, cg, 0);
        cudaGraphDestroy(cg);
        EC_TRY(check_cuda(ie, "graph instantiate"));
        if (d.graphs.size() >= kGraphCache) {
          // drop the least recently used
          size_t lru = 0;
          for (size_t e = 1; e < d.graphs.size(); ++e)
            if (d.graphs[e].used < d.graphs[lru].used) lru = e;
          cudaGraphExecDestroy(d.graphs[lru].exec);
          d.graphs.erase(d.graphs.begin() + static_cast<std::ptrdiff_t>(lru));
        }
        d.graphs.push_back({lens, d.ws, d.ws_tokens, d.ws_seqs, d.pin, d.pin_bytes, ex, 0});
        g = &d.graphs.back();
      }
      g->used = ++d.graph_clock;
      EC_TRY(check_cuda(cudaGraphLaunch(g->exec, d.stream), "graph launch"));
    } else {
      EC_TRY(enqueue());
    }
    tmark(g ? "graph launch" : "enqueue");
    EC_TRY(sync_and_check(d, "forward"));
    tmark("device (wait)");
    prof_collect(d);
    if (!out_dev && !direct_out)
      for (int k = 0; k < nseq; ++k)
        std::memcpy(out_host + static_cast<size_t>(seqs[i + k]) * out_stride,
                    hout + static_cast<size_t>(k) * m.out_dim, static_cast<size_t>(m.out_dim) * 4);
    tmark("copy out");
    i = j;
  }
  return EC_OK;
}

}  // namespace ec
