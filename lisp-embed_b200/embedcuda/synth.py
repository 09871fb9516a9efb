"""Seeded synthetic model directories and inputs for the benchmark workloads.

There are no checkpoints or corpora on the measurement machines, so every
workload is generated from a seed:

* weights: every matrix and embedding table ~ N(0, 0.02) (MPNet's relative
  attention bias too); LayerNorm / RMSNorm gamma = 1, beta = 0; every bias = 0.
  Draws come from ``numpy.random.default_rng(seed)`` in the order of
  ``tensor_specs`` (one ``normal`` call per tensor, float64 -> float32, then
  rounded to BF16 with round-to-nearest-even for BF16 models).
* inputs: ``numpy.random.default_rng((seed, 1))``: first all lengths, then all
  token bodies, sequence by sequence.

The directories use the Hugging Face tensor names that bert.lisp:83-127,
bert.lisp:343-389 and llama.lisp:189-218 read, so the reference loaders and
this library's loader see the same files.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field

import numpy as np

# --------------------------------------------------------------------------
# model shapes


@dataclass
class ModelShape:
    name: str
    model_type: str          # bert | roberta | mpnet | qwen3
    hidden: int
    layers: int
    heads: int
    inter: int
    vocab: int
    max_pos: int
    dtype: str               # F32 | BF16 | F16
    pooling: str             # mean | cls | last
    kv_heads: int = 0
    head_dim: int = 0
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    type_vocab: int = 2
    extra: dict = field(default_factory=dict)


# all-MiniLM-L6-v2 shape.  head_dim = hidden / heads = 32 (bert.lisp:75).
MINILM = ModelShape("minilm-l6", "bert", 384, 6, 12, 1536, 30522, 512, "F32", "mean")
# BERT-base shape (bge/e5-base-like), BF16, CLS pooling.
BERT_BASE = ModelShape("bert-base", "bert", 768, 12, 12, 3072, 30522, 512, "BF16", "cls")
# MPNet-base shape, relative-position attention, F32, mean pooling.
MPNET_BASE = ModelShape("mpnet-base", "mpnet", 768, 12, 12, 3072, 30527, 514, "F32", "mean")
# Qwen3-Embedding-0.6B shape, BF16, last-token pooling.
QWEN3_06B = ModelShape("qwen3-0.6b", "qwen3", 1024, 28, 16, 3072, 151669, 40960, "BF16",
                       "last", kv_heads=8, head_dim=128, rope_theta=1000000.0, rms_eps=1e-6)

# EmbeddingGemma (Gemma-3n text) shape at gemma.lisp's own defaults (hidden
# 512, 24 layers, 4 heads, FFN 2048, PLE 512, output 768; head dim 128 from
# q_norm, one kv head); full_attention every fourth layer.
GEMMA_EMB = ModelShape("embeddinggemma", "embedding_gemma2", 512, 24, 4, 2048, 32768, 2048, "F32",
                       "mean", kv_heads=1, head_dim=128, rms_eps=1e-6,
                       extra={"ple_dim": 512, "out_dim": 768,
                              "layer_types": ["full_attention" if i % 4 == 3 else "sliding_attention"
                                              for i in range(24)]})

SHAPES = {s.name: s for s in (MINILM, BERT_BASE, MPNET_BASE, QWEN3_06B, GEMMA_EMB)}
SEEDS = {"minilm-l6": 0, "bert-base": 1, "mpnet-base": 2, "qwen3-0.6b": 3, "embeddinggemma": 4}


def with_layers(shape: ModelShape, layers: int, vocab: int | None = None) -> ModelShape:
    """Same widths, fewer layers (and optionally a smaller vocab) for tests."""
    d = dict(shape.__dict__)
    d["layers"] = layers
    if "layer_types" in d.get("extra", {}):
        d["extra"] = dict(d["extra"], layer_types=d["extra"]["layer_types"][:layers])
    d["name"] = f"{shape.name}-{layers}l"
    if vocab is not None:
        d["vocab"] = vocab
    return ModelShape(**d)


# --------------------------------------------------------------------------
# tensor specs


def tensor_specs(s: ModelShape):
    """(name, shape, init) in draw order; init is 'normal', 'ones' or 'zeros'."""
    H, F = s.hidden, s.inter
    out = []
    if s.model_type in ("bert", "roberta"):
        out += [("embeddings.word_embeddings.weight", (s.vocab, H), "normal"),
                ("embeddings.position_embeddings.weight", (s.max_pos, H), "normal"),
                ("embeddings.token_type_embeddings.weight", (s.type_vocab, H), "normal"),
                ("embeddings.LayerNorm.weight", (H,), "ones"),
                ("embeddings.LayerNorm.bias", (H,), "zeros")]
        for li in range(s.layers):
            p = f"encoder.layer.{li}."
            for nm in ("query", "key", "value"):
                out += [(p + f"attention.self.{nm}.weight", (H, H), "normal"),
                        (p + f"attention.self.{nm}.bias", (H,), "zeros")]
            out += [(p + "attention.output.dense.weight", (H, H), "normal"),
                    (p + "attention.output.dense.bias", (H,), "zeros"),
                    (p + "attention.output.LayerNorm.weight", (H,), "ones"),
                    (p + "attention.output.LayerNorm.bias", (H,), "zeros"),
                    (p + "intermediate.dense.weight", (F, H), "normal"),
                    (p + "intermediate.dense.bias", (F,), "zeros"),
                    (p + "output.dense.weight", (H, F), "normal"),
                    (p + "output.dense.bias", (H,), "zeros"),
                    (p + "output.LayerNorm.weight", (H,), "ones"),
                    (p + "output.LayerNorm.bias", (H,), "zeros")]
    elif s.model_type == "mpnet":
        out += [("embeddings.word_embeddings.weight", (s.vocab, H), "normal"),
                ("embeddings.position_embeddings.weight", (s.max_pos, H), "normal"),
                ("embeddings.LayerNorm.weight", (H,), "ones"),
                ("embeddings.LayerNorm.bias", (H,), "zeros"),
                ("encoder.relative_attention_bias.weight", (32, s.heads), "normal")]
        for li in range(s.layers):
            p = f"encoder.layer.{li}."
            for nm in ("q", "k", "v", "o"):
                out += [(p + f"attention.attn.{nm}.weight", (H, H), "normal"),
                        (p + f"attention.attn.{nm}.bias", (H,), "zeros")]
            out += [(p + "attention.LayerNorm.weight", (H,), "ones"),
                    (p + "attention.LayerNorm.bias", (H,), "zeros"),
                    (p + "intermediate.dense.weight", (F, H), "normal"),
                    (p + "intermediate.dense.bias", (F,), "zeros"),
                    (p + "output.dense.weight", (H, F), "normal"),
                    (p + "output.dense.bias", (H,), "zeros"),
                    (p + "output.LayerNorm.weight", (H,), "ones"),
                    (p + "output.LayerNorm.bias", (H,), "zeros")]
    elif s.model_type in ("qwen3", "llama", "qwen2", "mistral"):
        hd = s.head_dim or H // s.heads
        kv = s.kv_heads or s.heads
        out += [("embed_tokens.weight", (s.vocab, H), "normal")]
        for li in range(s.layers):
            p = f"layers.{li}."
            out += [(p + "input_layernorm.weight", (H,), "ones"),
                    (p + "post_attention_layernorm.weight", (H,), "ones"),
                    (p + "self_attn.q_proj.weight", (s.heads * hd, H), "normal"),
                    (p + "self_attn.k_proj.weight", (kv * hd, H), "normal"),
                    (p + "self_attn.v_proj.weight", (kv * hd, H), "normal"),
                    (p + "self_attn.o_proj.weight", (H, s.heads * hd), "normal")]
            if s.model_type == "qwen3":
                out += [(p + "self_attn.q_norm.weight", (hd,), "ones"),
                        (p + "self_attn.k_norm.weight", (hd,), "ones")]
            out += [(p + "mlp.gate_proj.weight", (F, H), "normal"),
                    (p + "mlp.up_proj.weight", (F, H), "normal"),
                    (p + "mlp.down_proj.weight", (H, F), "normal")]
        out += [("norm.weight", (H,), "ones")]
    elif s.model_type == "embedding_gemma2":
        hd, kv = s.head_dim, s.kv_heads
        P, O = s.extra["ple_dim"], s.extra["out_dim"]
        pre = "language_model."
        out += [(pre + "embed_tokens.weight", (s.vocab, H), "normal"),
                (pre + "ple.per_layer_model_projection.weight", (s.layers * P, H), "normal"),
                (pre + "ple.per_layer_projection_norm.weight", (P,), "ones"),
                (pre + "norm.weight", (H,), "ones"),
                (pre + "embedding_projection.weight", (O, H), "normal")]
        for li in range(s.layers):
            p = f"{pre}layers.{li}."
            out += [(p + "input_layernorm.weight", (H,), "ones"),
                    (p + "post_attention_layernorm.weight", (H,), "ones"),
                    (p + "pre_feedforward_layernorm.weight", (H,), "ones"),
                    (p + "post_feedforward_layernorm.weight", (H,), "ones"),
                    (p + "self_attn.q_proj.weight", (s.heads * hd, H), "normal"),
                    (p + "self_attn.k_proj.weight", (kv * hd, H), "normal"),
                    (p + "self_attn.v_proj.weight", (kv * hd, H), "normal"),
                    (p + "self_attn.o_proj.weight", (H, s.heads * hd), "normal"),
                    (p + "self_attn.q_norm.weight", (hd,), "ones"),
                    (p + "self_attn.k_norm.weight", (hd,), "ones"),
                    (p + "mlp.gate_proj.weight", (F, H), "normal"),
                    (p + "mlp.up_proj.weight", (F, H), "normal"),
                    (p + "mlp.down_proj.weight", (H, F), "normal"),
                    (p + "ple_block.per_layer_input_gate.weight", (P, H), "normal"),
                    (p + "ple_block.per_layer_projection.weight", (H, P), "normal"),
                    (p + "ple_block.post_per_layer_input_norm.weight", (H,), "ones"),
                    (p + "layer_scalar", (1,), "scalar")]
    else:
        raise ValueError(f"unknown model_type {s.model_type}")
    return out


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rnd = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rnd) >> 16).astype(np.uint16)


def f32_to_f16_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


def make_weights(s: ModelShape, seed: int):
    """dict name -> (dtype string, shape, raw little-endian bytes as ndarray)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape, init in tensor_specs(s):
        if init == "normal":
            a = rng.normal(0.0, 0.02, size=shape).astype(np.float32)
        elif init == "ones":
            a = np.ones(shape, np.float32)
        elif init == "scalar":  # a layer scalar near 1
            a = np.full(shape, 0.5 + rng.random(), np.float32)
        else:
            a = np.zeros(shape, np.float32)
        if s.dtype == "BF16":
            out[name] = ("BF16", shape, f32_to_bf16_bits(a))
        elif s.dtype == "F16":
            out[name] = ("F16", shape, f32_to_f16_bits(a))
        else:
            out[name] = ("F32", shape, a)
    return out


def write_safetensors(path: str, tensors: dict):
    header = {}
    off = 0
    blobs = []
    for name, (dt, shape, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    hj = json.dumps(header, separators=(",", ":")).encode()
    pad = (8 - len(hj) % 8) % 8
    hj += b" " * pad
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def config_json(s: ModelShape) -> dict:
    if s.model_type in ("bert", "roberta", "mpnet"):
        cfg = {"model_type": s.model_type, "hidden_size": s.hidden,
               "num_hidden_layers": s.layers, "num_attention_heads": s.heads,
               "intermediate_size": s.inter, "vocab_size": s.vocab,
               "max_position_embeddings": s.max_pos, "hidden_act": "gelu",
               "layer_norm_eps": 1e-12, "torch_dtype": s.dtype.lower()}
        if s.model_type != "mpnet":
            cfg["type_vocab_size"] = s.type_vocab
        else:
            cfg["relative_attention_num_buckets"] = 32
        return cfg
    hd = s.head_dim or s.hidden // s.heads
    if s.model_type == "embedding_gemma2":
        return {"model_type": "embedding_gemma2",
                "text_config": {"model_type": "embedding_gemma2_text", "hidden_size": s.hidden,
                                "num_hidden_layers": s.layers, "num_attention_heads": s.heads,
                                "num_key_value_heads": s.kv_heads, "head_dim": hd,
                                "intermediate_size": s.inter, "vocab_size": s.vocab,
                                "hidden_size_per_layer_input": s.extra["ple_dim"],
                                "embedding_dim": s.extra["out_dim"], "rms_norm_eps": s.rms_eps,
                                "layer_types": s.extra["layer_types"],
                                "hidden_activation": "gelu_pytorch_tanh"}}
    return {"model_type": s.model_type, "hidden_size": s.hidden,
            "num_hidden_layers": s.layers, "num_attention_heads": s.heads,
            "num_key_value_heads": s.kv_heads or s.heads, "head_dim": hd,
            "intermediate_size": s.inter, "vocab_size": s.vocab,
            "rope_theta": s.rope_theta, "rms_norm_eps": s.rms_eps,
            "max_position_embeddings": s.max_pos, "hidden_act": "silu",
            "torch_dtype": "bfloat16" if s.dtype == "BF16" else "float32"}


def build_model_dir(s: ModelShape, seed: int, root: str) -> str:
    """Write config.json (+ 1_Pooling/config.json for mean pooling) and
    model.safetensors under root/<name>-s<seed>; reuse an existing dir."""
    d = os.path.join(root, f"{s.name}-s{seed}")
    st = os.path.join(d, "model.safetensors")
    done = os.path.join(d, ".complete")
    if os.path.exists(done):
        return d
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(config_json(s), f, indent=1)
    if s.model_type in ("bert", "roberta", "mpnet"):
        os.makedirs(os.path.join(d, "1_Pooling"), exist_ok=True)
        with open(os.path.join(d, "1_Pooling", "config.json"), "w") as f:
            json.dump({"word_embedding_dimension": s.hidden,
                       "pooling_mode_cls_token": s.pooling == "cls",
                       "pooling_mode_mean_tokens": s.pooling == "mean"}, f, indent=1)
    write_safetensors(st, make_weights(s, seed))
    open(done, "w").close()
    return d


# --------------------------------------------------------------------------
# inputs


def make_inputs(workload: str, nseq: int, seed: int, vocab: int | None = None):
    """Token-id batches as (ids int32[total], offsets int64[nseq+1]).

    minilm / bert-base: [CLS]=101 + U[1000, vocab-1] + [SEP]=102, total length
    U{16..256} (minilm) or floor(exp(U[ln 32, ln 512])) (bert-base).
    mpnet: <s>=0 + U[1000, vocab-1] + </s>=2, total length U{64..384}.
    qwen3: body U{128..512} of U[0, 151643) then EOS 151643.
    gemma: <bos>=2 + U[1000, vocab-1] + <eos>=1, total length U{16..512}.
    """
    rng = np.random.default_rng((seed, 1))
    if workload.startswith("minilm"):
        lens = rng.integers(16, 256, size=nseq, endpoint=True)
        lo, hi, pre, post = 1000, (vocab or 30522) - 1, [101], [102]
    elif workload.startswith("bert"):
        lens = np.floor(np.exp(rng.uniform(np.log(32), np.log(512), size=nseq))).astype(np.int64)
        lo, hi, pre, post = 1000, (vocab or 30522) - 1, [101], [102]
    elif workload.startswith("mpnet"):
        lens = rng.integers(64, 384, size=nseq, endpoint=True)
        lo, hi, pre, post = 1000, (vocab or 30527) - 1, [0], [2]
    elif workload.startswith("qwen3"):
        body = rng.integers(128, 512, size=nseq, endpoint=True)
        lens = body + 1
        lo, hi, pre, post = 0, min(151642, (vocab or 151669) - 1), [], [151643]
    elif "gemma" in workload:
        lens = rng.integers(16, 512, size=nseq, endpoint=True)
        lo, hi, pre, post = 1000, (vocab or 32768) - 1, [2], [1]
    else:
        raise ValueError(workload)
    lens = np.asarray(lens, np.int64)
    offsets = np.zeros(nseq + 1, np.int64)
    offsets[1:] = np.cumsum(lens)
    ids = np.empty(int(offsets[-1]), np.int32)
    for i in range(nseq):
        nb = int(lens[i]) - len(pre) - len(post)
        body = rng.integers(lo, hi, size=nb, endpoint=True)
        ids[offsets[i]:offsets[i + 1]] = np.concatenate([pre, body, post]).astype(np.int32)
    return ids, offsets


def make_short_inputs(workload: str, lengths, seed: int, vocab: int):
    """Explicit lengths (for tests): same id distribution as make_inputs."""
    rng = np.random.default_rng((seed, 2))
    if workload.startswith("qwen3"):
        pre, post, lo, hi = [], [min(151643, vocab - 1)], 0, min(151642, vocab - 2)
    elif workload.startswith("mpnet"):
        pre, post, lo, hi = [0], [2], min(1000, vocab - 2), vocab - 1
    elif "gemma" in workload:
        pre, post, lo, hi = [2], [1], min(1000, vocab - 2), vocab - 1
    else:
        pre, post, lo, hi = [101], [102], min(1000, vocab - 2), vocab - 1
    offs = [0]
    chunks = []
    for L in lengths:
        nb = max(0, int(L) - len(pre) - len(post))
        body = rng.integers(lo, hi, size=nb, endpoint=True)
        seq = np.concatenate([pre, body, post]).astype(np.int32)[: max(1, int(L))]
        chunks.append(seq)
        offs.append(offs[-1] + len(seq))
    return np.concatenate(chunks).astype(np.int32), np.asarray(offs, np.int64)


# --------------------------------------------------------------------------
# IVF corpus


def make_ivf_corpus(n: int, dim: int, nclusters: int, seed: int, sigma: float = 0.05):
    """Mixture of `nclusters` Gaussians with centers uniform on the unit sphere,
    each vector L2-normalised.  Returns (vectors f32[n, dim], labels)."""
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((nclusters, dim)).astype(np.float32)
    centers /= np.linalg.norm(centers, axis=1, keepdims=True)
    labels = rng.integers(0, nclusters, size=n)
    x = np.empty((n, dim), np.float32)
    step = 1 << 18
    for s in range(0, n, step):
        e = min(n, s + step)
        blk = centers[labels[s:e]] + sigma * rng.standard_normal((e - s, dim)).astype(np.float32)
        blk /= np.linalg.norm(blk, axis=1, keepdims=True)
        x[s:e] = blk
    return x, labels


def make_ivf_sample(n: int, seed: int) -> np.ndarray:
    """A seeded permutation of all rows: its first k rows initialise k-means
    (ann.lisp:83-86) and the whole permutation is the training sample."""
    return np.random.default_rng((seed, 3)).permutation(n).astype(np.int64)
