"""End-to-end parity of the encoder forwards against the CPU oracle
(restatement of bert.lisp / llama.lisp) on the same seeded weights and ids.

Tolerance (BF16 tensor-core path): per-vector cosine >= 0.999.
"""
import numpy as np
import pytest

from embedcuda import model, synth
from oracle import oracle

pytestmark = pytest.mark.gpu

COS_BF16 = 0.999


def _cos(a, b):
    return np.sum(a * b, axis=1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


def _check(shape, seed, lengths, synth_root, ec, workload):
    d = synth.build_model_dir(shape, seed, synth_root)
    fam = model.load_model(d)
    ids, offs = synth.make_short_inputs(workload, lengths, seed, shape.vocab)
    got = model.embed_batch(ids, offs)
    ref = oracle.OracleModel(d).embed_batch(ids, offs)
    cos = _cos(got, ref)
    assert np.all(np.isfinite(got))
    assert np.allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    assert cos.min() >= COS_BF16, (fam, cos)
    return fam, cos


# default: the residual between sublayers is the LayerNorm's bf16 output;
# EC_F32_RESIDUAL keeps an fp32 residual stream
@pytest.mark.parametrize("f32_resid", [0, 1])
def test_minilm_full_depth(synth_root, ec, monkeypatch, f32_resid):
    if f32_resid:
        monkeypatch.setenv("EC_F32_RESIDUAL", "1")
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
