"""The CPU oracle (restatement of bert.lisp / llama.lisp / ann.lisp /
kb.lisp) against committed golden vectors and hand-built known answers.

Parity status: the reference has no tests or golden vectors and SBCL is
absent, so the oracle is pinned against Hugging Face transformers run on the
same synthetic weights (tests/golden/make_golden.py) -- an independent
implementation of the same published architectures -- plus exact regression
against its own committed outputs.
"""
import os

import numpy as np
import pytest

from embedcuda import synth
from oracle import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "embed_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLD)


def _case(name):
    if name == "minilm":
        return synth.with_layers(synth.MINILM, 2), 0
    if name == "mpnet":
        return synth.with_layers(synth.MPNET_BASE, 2), 2
    return synth.with_layers(synth.QWEN3_06B, 2, vocab=4096), 3


@pytest.mark.parametrize("name", ["minilm", "mpnet", "qwen3"])
def test_oracle_matches_golden(golden, synth_root, name):
    import hashlib
    s, seed = _case(name)
    d = synth.build_model_dir(s, seed, synth_root)
    om = oracle.OracleModel(d)
    h = hashlib.sha256()
    for k in sorted(om.w):
        h.update(k.encode())
        h.update(np.ascontiguousarray(om.w[k], np.float32).tobytes())
    assert h.digest() == golden[f"{name}_digest"].tobytes(), "synthetic weights drifted"
    ids, offs = golden[f"{name}_ids"], golden[f"{name}_offsets"]
    got = om.embed_batch(ids, offs, threads=4)
    # exact regression against the committed oracle output
    assert np.array_equal(got, golden[f"{name}_oracle"])
    # independent implementation: within the LN-eps placement / erf-approx noise
    hf = golden[f"{name}_hf"]
    cos = np.sum(got * hf, 1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(hf, axis=1))
    assert cos.min() > 0.999999, cos
    assert np.abs(got - hf).max() < 2e-6


def test_mpnet_bucket_table():
    # bert::mpnet-bucket (bert.lisp:324-331): 8 exact, log buckets to 15, +16 for i < j
    assert [oracle.mpnet_bucket(0, j) for j in range(10)] == [0, 17, 18, 19, 20, 21, 22, 23, 24, 24]
    assert [oracle.mpnet_bucket(i, 0) for i in (7, 8, 12, 16, 32, 64, 127, 128, 500)] == \
        [7, 8, 9, 10, 12, 14, 15, 15, 15]


def test_f16_widening_rule():
    # st::half-to-float: exponent 31 (inf / nan) -> +-most-positive-single-float
    import ctypes as C
    src = np.array([0x3C00, 0xC000, 0x7C00, 0xFC00, 0x7E00, 0x0001, 0x0000, 0x8000], np.uint16)
    dst = np.empty(src.size, np.float32)
    oracle.lib().or_f16_to_f32(src.ctypes.data_as(C.POINTER(C.c_uint16)),
                               dst.ctypes.data_as(C.POINTER(C.c_float)), C.c_int64(src.size))
    fmax = np.finfo(np.float32).max
    assert list(dst[:5]) == [1.0, -2.0, fmax, -fmax, fmax]
    assert dst[5] == np.float32(2.0 ** -24) and dst[6] == 0.0


def test_dot_is_sequential_single_float():
    # %dot accumulates left to right in single-float, no fused multiply-add
    a = np.array([1e8, 1.0, -1e8, 1.0], np.float32)
    b = np.ones(4, np.float32)
    assert oracle.dot(a, b) == np.float32(1.0)  # ((1e8 + 1) - 1e8) + 1 = 0 + 1


def test_nearest_centroid_ties_and_negative():
    x = np.array([[1.0, 0.0]], np.float32)
    cent = np.array([[0.0, 1.0], [2.0, 0.0], [2.0, 5.0], [2.0, 0.0]], np.float32)
    assert oracle.assign(x, cent)[0] == 1  # strict >: first of the tied maxima
    neg = np.array([[-5.0, 0.0], [-1.0, 0.0]], np.float32)
    assert oracle.assign(x, neg)[0] == 1


def test_assign_all_is_stable_counting_sort():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((500, 8)).astype(np.float32)
    cent = x[:7]
    counts, lists = oracle.assign_all(x, cent)
    a = oracle.assign(x, cent)
    assert counts.sum() == 500
    o = 0
    for c in range(7):
        ids = lists[o:o + counts[c]]
        assert np.array_equal(ids, np.nonzero(a == c)[0])  # ascending row ids
        o += counts[c]


def test_kmeans_matches_numpy_restatement():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((300, 16)).astype(np.float32)
    sample = rng.permutation(300)[:200]
    k = 5
    cent = x[sample[:k]].copy()
    for _ in range(3):
        a = oracle.assign(x, cent, rows=sample)
        new = cent.copy()
        for c in range(k):
            m = sample[a == c]
            if len(m):
                s = np.zeros(16, np.float32)
                for r in m:  # serial single-float sums in sample order
                    s = (s + x[r]).astype(np.float32)
                new[c] = s / np.float32(len(m))
        cent = new
    assert np.array_equal(oracle.kmeans(x, sample, k, 3), cent)


def test_top_k_ivf_merge_order():
    # two probed lists holding equal scores: the earlier probed list wins ties
    x = np.array([[1, 0], [1, 0], [0, 1], [1, 0]], np.float32)
    cent = np.array([[1, 0], [0.9, 0.1]], np.float32)
    counts = np.array([1, 3], np.uint32)
    lists = np.array([3, 0, 1, 2], np.uint32)
    ids, sc = oracle.top_k_ivf(x, cent, counts, lists, 2, np.array([1, 0], np.float32), 3)
    assert list(ids) == [3, 0, 1] and list(sc) == [1.0, 1.0, 1.0]
    ids, sc = oracle.top_k_brute(x, np.array([1, 0], np.float32), 3)
    assert list(ids) == [0, 1, 3]


def _gemma_numpy(w, t, ids):
    """float64 numpy restatement of gemma::embed (gemma.lisp:306-380) used to
    check the C oracle's Gemma path; same step order, wider arithmetic."""
    H, P, NL = t["hidden_size"], t["hidden_size_per_layer_input"], t["num_hidden_layers"]
    eps = t["rms_norm_eps"]
    pre = "language_model."
    W = {k: np.asarray(v, np.float64) for k, v in w.items()}

    def rms(x, g=None):
        y = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
        return y if g is None else y * g

    def gelu(x):
        return 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))

    S = ids.size
    h = np.sqrt(np.float32(H)).astype(np.float64) * W[pre + "embed_tokens.weight"][ids]
    ple = (h @ W[pre + "ple.per_layer_model_projection.weight"].T) / np.sqrt(H)
    ple = rms(ple.reshape(S, NL, P), W[pre + "ple.per_layer_projection_norm.weight"])
    pos = np.arange(S)[:, None]
    for li in range(NL):
        p = f"{pre}layers.{li}."
        hd = W[p + "self_attn.q_norm.weight"].size
        theta = 1e6 if t["layer_types"][li] == "full_attention" else 1e4
        ang = pos * (1.0 / theta ** (2.0 * np.arange(hd // 2) / hd))
        cos, sin = np.cos(ang)[:, None], np.sin(ang)[:, None]

        def rope(x):
            a, b = x[..., :hd // 2], x[..., hd // 2:]
            return np.concatenate([a * cos - b * sin, a * sin + b * cos], -1)

        x = rms(h, W[p + "input_layernorm.weight"])
        q = (x @ W[p + "self_attn.q_proj.weight"].T).reshape(S, -1, hd)
        k = (x @ W[p + "self_attn.k_proj.weight"].T).reshape(S, -1, hd)
        v = (x @ W[p + "self_attn.v_proj.weight"].T).reshape(S, -1, hd)
        q = rope(rms(q, W[p + "self_attn.q_norm.weight"]))
        k = rope(rms(k, W[p + "self_attn.k_norm.weight"]))
        v = rms(v)
        grp = q.shape[1] // k.shape[1]
        k, v = np.repeat(k, grp, 1), np.repeat(v, grp, 1)
        sc = np.einsum("shd,thd->hst", q, k)            # scale 1.0, bidirectional
        sc = np.exp(sc - sc.max(-1, keepdims=True))
        sc /= sc.sum(-1, keepdims=True)
        ctx = np.einsum("hst,thd->shd", sc, v).reshape(S, -1)
        h = h + rms(ctx @ W[p + "self_attn.o_proj.weight"].T, W[p + "post_attention_layernorm.weight"])
        x = rms(h, W[p + "pre_feedforward_layernorm.weight"])
        f = gelu(x @ W[p + "mlp.gate_proj.weight"].T) * (x @ W[p + "mlp.up_proj.weight"].T)
        h = h + rms(f @ W[p + "mlp.down_proj.weight"].T, W[p + "post_feedforward_layernorm.weight"])
        g = gelu(h @ W[p + "ple_block.per_layer_input_gate.weight"].T) * ple[:, li]
        h = h + rms(g @ W[p + "ple_block.per_layer_projection.weight"].T,
                    W[p + "ple_block.post_per_layer_input_norm.weight"])
        h = h * W[p + "layer_scalar"].reshape(-1)[0]
    h = rms(h, W[pre + "norm.weight"])
    v = W[pre + "embedding_projection.weight"] @ h.mean(0)
    return v / np.linalg.norm(v)


def test_gemma_oracle_matches_float64_restatement(synth_root):
    """The C oracle's gemma::embed (single precision, gemma.lisp's order of
    operations) against a float64 numpy restatement on the same weights:
    two layers, one sliding (theta 1e4) and one full-attention (theta 1e6)."""
    import dataclasses
    import json
    s = synth.with_layers(synth.GEMMA_EMB, 2, vocab=4096)
    s = dataclasses.replace(s, name=s.name + "-sf", extra=dict(
        s.extra, layer_types=["sliding_attention", "full_attention"]))
    d = synth.build_model_dir(s, 4, synth_root)
    om = oracle.OracleModel(d)
    with open(os.path.join(d, "config.json")) as f:
        t = json.load(f)["text_config"]
    ids, offs = synth.make_short_inputs("gemma", [1, 2, 37, 130], 4, s.vocab)
    got = om.embed_batch(ids, offs, threads=4)
    assert got.shape == (4, 768)
    for i in range(4):
        ref = _gemma_numpy(om.w, t, ids[offs[i]:offs[i + 1]])
        cos = float(np.dot(got[i], ref) / np.linalg.norm(got[i]))
        assert cos > 0.99999, (i, cos)
        assert np.abs(got[i] - ref).max() < 1e-4
    # one sequence alone equals the same sequence inside the batch
    one = om.embed(ids[offs[2]:offs[3]])
    assert np.array_equal(one, got[2])
