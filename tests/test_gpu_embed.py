"""End-to-end parity of the encoder forwards against the CPU oracle
(restatement of bert.lisp / llama.lisp / gemma.lisp) on the same seeded
weights and ids.

Tolerances (per-vector cosine against the oracle):
  * F32 models (MiniLM, MPNet, and F16 weights, which st.lisp widens to
    F32): >= 0.9999;
  * BF16 models (BERT-base, Qwen3) and EmbeddingGemma: >= 0.999.
Full-depth cases run every layer of the BASELINE shapes (12-layer BERT-base
and MPNet, 28-layer Qwen3 with its full 151,669-row vocabulary) on a few
sequences up to the longest length each workload draws.
"""
import os

import numpy as np
import pytest

from embedcuda import model, synth
from oracle import oracle

pytestmark = pytest.mark.gpu

COS_F32 = 0.9999
COS_BF16 = 0.999


def _cos(a, b):
    return np.sum(a * b, axis=1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


def _tol(shape):
    return COS_BF16 if shape.dtype == "BF16" or shape.model_type == "embedding_gemma2" else COS_F32


def _check(shape, seed, lengths, synth_root, ec, workload, d=None):
    d = d or synth.build_model_dir(shape, seed, synth_root)
    fam = model.load_model(d)
    ids, offs = synth.make_short_inputs(workload, lengths, seed, shape.vocab)
    got = model.embed_batch(ids, offs)
    # one host thread per sequence, each splitting its token / head loops
    # over its share of the cores (same values as one thread)
    per = max(1, (os.cpu_count() or 1) // len(lengths))
    ref = oracle.OracleModel(d).embed_batch(ids, offs, threads=len(lengths), seq_threads=per)
    cos = _cos(got, ref)
    assert np.all(np.isfinite(got))
    assert np.allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    assert cos.min() >= _tol(shape), (fam, cos)
    return fam, cos


# default: the residual between sublayers is the LayerNorm's bf16 output;
# EC_F32_RESIDUAL keeps an fp32 residual stream; EC_SHORT_ATTN_TC runs the
# attention of these short sequences on the tcgen05 short-sequence kernel;
# EC_FUSED_MLP runs each feed-forward block as one kernel (bf16 and fp32
# residual)
@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4])
def test_minilm_full_depth(synth_root, ec, monkeypatch, variant):
    if variant in (1, 4):
        monkeypatch.setenv("EC_F32_RESIDUAL", "1")
    if variant == 2:
        monkeypatch.setenv("EC_SHORT_ATTN_TC", "1")
    if variant in (3, 4):
        monkeypatch.setenv("EC_FUSED_MLP", "1")
    fam, cos = _check(synth.MINILM, 0, [1, 2, 16, 63, 64, 65, 130, 256], synth_root, ec, "minilm")
    assert fam == "bert"


@pytest.mark.parametrize("f32_resid", [0, 1])
def test_bert_base_bf16(synth_root, ec, monkeypatch, f32_resid):
    if f32_resid:
        monkeypatch.setenv("EC_F32_RESIDUAL", "1")
    s = synth.with_layers(synth.BERT_BASE, 2)
    fam, _ = _check(s, 1, [3, 32, 100, 129, 512], synth_root, ec, "bert")
    assert fam == "bert"


def test_mpnet(synth_root, ec):
    s = synth.with_layers(synth.MPNET_BASE, 2)
    fam, _ = _check(s, 2, [2, 9, 64, 140, 384], synth_root, ec, "mpnet")
    assert fam == "mpnet"


def test_qwen3(synth_root, ec):
    s = synth.with_layers(synth.QWEN3_06B, 2, vocab=4096)
    fam, _ = _check(s, 3, [1, 2, 40, 129, 300], synth_root, ec, "qwen3")
    assert fam == "llama"


# ---- full depth: every layer of the BASELINE shapes --------------------------

def test_bert_base_full_depth(synth_root, ec):
    """12 layers, BF16 weights, CLS pooling; lengths up to 512."""
    fam, cos = _check(synth.BERT_BASE, 1, [32, 200, 512], synth_root, ec, "bert")
    assert fam == "bert"


def test_mpnet_full_depth(synth_root, ec):
    """12 layers, F32 weights, relative-position buckets; lengths up to 384."""
    fam, cos = _check(synth.MPNET_BASE, 2, [64, 230, 384], synth_root, ec, "mpnet")
    assert fam == "mpnet"


def test_qwen3_full_depth_full_vocab(synth_root, ec):
    """28 layers, 151,669-row vocabulary, GQA 16:8, causal, last-token
    pooling; the longest sequence is 512 body tokens + EOS."""
    fam, cos = _check(synth.QWEN3_06B, 3, [129, 300, 513], synth_root, ec, "qwen3")
    assert fam == "llama"


# ---- F16 weights (st.lisp:22-30 widening on the device) ----------------------

def _f16_patterns_widened(ec):
    """Every binary16 bit pattern uploaded as an F16 tensor and read back from
    the device as f32."""
    import ctypes as C
    from embedcuda import _lib
    pats = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    shape = np.array([256, 256], np.int64)
    L = ec.lib()
    _lib.check(L.ec_upload_tensor(b"f16.probe", _lib.EC_F16, shape.ctypes.data_as(C.POINTER(C.c_int64)),
                                  2, pats.ctypes.data, pats.nbytes), "upload probe")
    got = np.empty(65536, np.float32)
    dt = C.c_int()
    _lib.check(L.ecdbg_tensor_read(b"f16.probe", got.ctypes.data, got.nbytes, C.byref(dt)), "read")
    assert dt.value == _lib.EC_F32
    ref = np.empty(65536, np.float32)
    oracle.lib().or_f16_to_f32(pats.ctypes.data_as(C.POINTER(C.c_uint16)),
                               ref.ctypes.data_as(C.POINTER(C.c_float)), C.c_int64(65536))
    return pats, got, ref


def test_f16_widening_every_pattern(ec):
    """Subnormals, signed zeros, and exponent 31 (Inf / NaN patterns) ->
    +-most-positive-single-float, bit for bit as st::half-to-float."""
    pats, got, ref = _f16_patterns_widened(ec)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert got[0x7C00] == np.finfo(np.float32).max and got[0xFE00] == -np.finfo(np.float32).max
    assert got[0x0001] == np.float32(2.0 ** -24)  # smallest subnormal


def test_f16_model(synth_root, ec, tmp_path):
    """A 2-layer MiniLM stored as F16, with subnormal halves planted in used
    weights and exponent-31 halves in embedding rows the inputs never touch
    (ids below 1000, positions past the longest sequence)."""
    s = synth.with_layers(synth.MINILM, 2)
    import dataclasses
    s = dataclasses.replace(s, name=s.name + "-f16", dtype="F16")
    w = synth.make_weights(s, 0)
    rng = np.random.default_rng(5)
    sub = np.array([0x0001, 0x0003, 0x03FF, 0x8001, 0x8200, 0x0200], np.uint16)
    for nm in ("encoder.layer.0.attention.self.query.weight", "encoder.layer.1.output.dense.weight",
               "embeddings.word_embeddings.weight"):
        dt, shape, a = w[nm]
        a = a.copy().reshape(-1)
        idx = rng.choice(a.size, 200, replace=False)
        a[idx] = sub[rng.integers(0, len(sub), 200)]
        w[nm] = (dt, shape, a.reshape(shape))
    big = np.array([0x7C00, 0xFC00, 0x7E00, 0xFFFF, 0x7C01], np.uint16)
    dt, shape, a = w["embeddings.word_embeddings.weight"]
    a = a.copy()
    a[1:40] = big[rng.integers(0, len(big), (39, shape[1]))]
    w["embeddings.word_embeddings.weight"] = (dt, shape, a)
    dt, shape, a = w["embeddings.position_embeddings.weight"]
    a = a.copy()
    a[300:] = big[rng.integers(0, len(big), (shape[0] - 300, shape[1]))]
    w["embeddings.position_embeddings.weight"] = (dt, shape, a)
    d = str(tmp_path / "minilm-f16")
    os.makedirs(os.path.join(d, "1_Pooling"))
    import json
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(synth.config_json(s), f)
    with open(os.path.join(d, "1_Pooling", "config.json"), "w") as f:
        json.dump({"word_embedding_dimension": s.hidden, "pooling_mode_mean_tokens": True}, f)
    synth.write_safetensors(os.path.join(d, "model.safetensors"), w)
    fam, cos = _check(s, 0, [1, 5, 64, 130, 256], synth_root, ec, "minilm", d=d)
    assert fam == "bert"


def test_batch_invariance_and_order(synth_root, ec):
    """A sequence's embedding does not depend on its batch-mates or position."""
    d = synth.build_model_dir(synth.MINILM, 0, synth_root)
    model.load_model(d)
    ids, offs = synth.make_inputs("minilm", 64, 0)
    full = model.embed_batch(ids, offs)
    for s in (0, 17, 63):
        one = model.embed(ids[offs[s]:offs[s + 1]])
        assert np.array_equal(one, full[s]) or _cos(one[None], full[s][None])[0] > 0.99999
    again = model.embed_batch(ids, offs)
    assert np.array_equal(full, again)  # deterministic


# batches of at most 16 tokens run the skinny GEMMs + LayerNorm row kernel:
# against the oracle, and against the tcgen05 path (EC_NO_SKINNY) on the
# same batch; 16 tokens exactly, one token, several sequences
@pytest.mark.parametrize("lengths", [[1], [10], [2, 3, 11], [16]])
def test_skinny_small_batches(synth_root, ec, monkeypatch, lengths):
    fam, cos = _check(synth.MINILM, 0, lengths, synth_root, ec, "minilm")
    assert fam == "bert"
    ids, offs = synth.make_short_inputs("minilm", lengths, 0, synth.MINILM.vocab)
    got = model.embed_batch(ids, offs)
    monkeypatch.setenv("EC_NO_SKINNY", "1")
    tc = model.embed_batch(ids, offs)
    assert _cos(got, tc).min() >= 0.9999


def test_skinny_mpnet(synth_root, ec):
    s = synth.with_layers(synth.MPNET_BASE, 2)
    fam, _ = _check(s, 2, [4, 9], synth_root, ec, "mpnet")
    assert fam == "mpnet"


def test_graph_replay(synth_root, ec, monkeypatch):
    """Small host batches replay a captured CUDA graph of the forward: the
    replays (with other lengths captured in between, and new ids of the same
    lengths) equal the launch-by-launch path bit for bit, and the oracle."""
    d = synth.build_model_dir(synth.MINILM, 0, synth_root)
    model.load_model(d)
    ids, offs = synth.make_inputs("minilm", 8, 3)
    rng = np.random.default_rng(5)
    q = [np.concatenate([[101], rng.integers(1000, 30522, 8), [102]]).astype(np.int32) for _ in range(3)]
    got = [model.embed_batch(ids, offs), model.embed(q[0]), model.embed_batch(ids, offs),
           model.embed(q[1]), model.embed(q[2]), model.embed_batch(ids, offs)]
    monkeypatch.setenv("EC_NO_GRAPH", "1")
    ref = [model.embed_batch(ids, offs), model.embed(q[0]), model.embed_batch(ids, offs),
           model.embed(q[1]), model.embed(q[2]), model.embed_batch(ids, offs)]
    for a, b in zip(got, ref):
        assert np.array_equal(a, b)
    om = oracle.OracleModel(d)
    for k, gi in enumerate((1, 3, 4)):
        assert _cos(got[gi][None], om.embed(q[k])[None])[0] >= 0.9999


def test_errors(synth_root, ec):
    from embedcuda import _lib
    d = synth.build_model_dir(synth.MINILM, 0, synth_root)
    model.load_model(d)
    with pytest.raises(_lib.EcError) as e:
        model.embed(np.array([101, 40000, 102], np.int32))  # id outside vocab
    assert e.value.code == _lib.EC_EINVAL
    with pytest.raises(_lib.EcError):
        model.embed(np.arange(600, dtype=np.int32) + 1000)  # past 512 positions
    with pytest.raises(_lib.EcError):
        model.embed_batch(np.zeros(0, np.int32), np.array([0, 0], np.int64))  # empty sequence
    # a sequence that starts before the ids is refused before any id is read
    # (raw call: the host mirror refuses it itself)
    import ctypes as C
    ids = np.arange(10, dtype=np.int32) + 1000
    offs = np.array([-2, 5], np.int64)
    out = np.zeros((1, model.dim()), np.float32)
    rc = _lib.lib().ec_embed_batch(_lib.ptr(ids, C.c_int32), _lib.ptr(offs, C.c_int64), 1,
                                   _lib.ptr(out, C.c_float), out.shape[1])
    assert rc == _lib.EC_EINVAL and "starts at offset" in _lib.last_error()


@pytest.mark.parametrize("unfused", [0, 1, 2])
def test_gemma(synth_root, ec, monkeypatch, unfused):
    """EmbeddingGemma: one sliding (theta 1e4) and one full-attention (theta
    1e6) layer, PLE, per-head q/k/v norms, mean pool + 512 -> 768 projection;
    with the norms / PLE gate fused into GEMM epilogues and without."""
    import dataclasses
    if unfused == 1:      # every Gemma fusion off
        monkeypatch.setenv("EC_NO_FUSED_ROPE", "1")
        monkeypatch.setenv("EC_NO_FUSED_PLE_GATE", "1")
        monkeypatch.setenv("EC_NO_GEMM_RMS", "1")
    elif unfused == 2:    # only the GEMM + RMSNorm epilogues off
        monkeypatch.setenv("EC_NO_GEMM_RMS", "1")
    s = synth.with_layers(synth.GEMMA_EMB, 2, vocab=4096)
    s = dataclasses.replace(s, name=s.name + "-sf", extra=dict(
        s.extra, layer_types=["sliding_attention", "full_attention"]))
    fam, _ = _check(s, 4, [1, 2, 40, 129, 300], synth_root, ec, "gemma")
    assert fam == "gemma"
    assert model.dim() == 768


def test_qwen3_odd_head_count(synth_root, ec):
    """16 q heads + 1 kv head: one 256-wide QKV tile holds the k head and the
    v head, so the fused epilogue rotates one half and leaves the other."""
    import dataclasses
    s = synth.with_layers(synth.QWEN3_06B, 1, vocab=4096)
    s = dataclasses.replace(s, name=s.name + "-kv1", kv_heads=1)
    fam, _ = _check(s, 3, [1, 7, 200, 333], synth_root, ec, "qwen3")
    assert fam == "llama"
