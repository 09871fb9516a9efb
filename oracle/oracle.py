"""ctypes front end of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; it is the checker, never the product.  Parity status: UNPINNED
by the reference (no reference tests, no SBCL); oracle.c restates the Lisp.

The model readers here mirror st.lisp (raw dtype widened to F32 exactly as
st:get-tensor does) and the config readers mirror bert:load-model
(bert.lisp:55-80) and llama:load-model (llama.lisp:172-187).
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

F = C.POINTER(C.c_float)


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
                os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.c"))):
            build()
        L = C.CDLL(_LIB_PATH)
        L.or_bert_embed.restype = C.c_int
        L.or_llama_embed.restype = C.c_int
        L.or_embed_batch.restype = C.c_int
        L.or_dot.restype = C.c_float
        L.or_nearest_centroid.restype = C.c_int32
        L.or_top_k_ivf.restype = C.c_int
        L.or_top_k_brute.restype = C.c_int
        L.or_mpnet_bucket.restype = C.c_int
        L.or_gemma_embed.restype = C.c_int
        _lib = L
    return _lib


class BertLayer(C.Structure):
    _fields_ = [(n, F) for n in ("q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "ao_w", "ao_b",
                                 "ao_g", "ao_b2", "ff_w", "ff_b", "o_w", "o_b", "o_g", "o_b2")]


class Bert(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("head_dim", C.c_int), ("inter", C.c_int), ("pooling", C.c_int),
                ("mpnet", C.c_int), ("pos_offset", C.c_int), ("causal", C.c_int),
                ("w_word", F), ("w_pos", F), ("w_type", F), ("emb_g", F), ("emb_b", F),
                ("rel_bias", F), ("L", C.POINTER(BertLayer))]


class LlamaLayer(C.Structure):
    _fields_ = [(n, F) for n in ("in_ln", "post_ln", "q_w", "k_w", "v_w", "o_w", "q_norm",
                                 "k_norm", "gate", "up", "down")]


class Llama(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("inter", C.c_int),
                ("pooling", C.c_int), ("max_pos", C.c_int), ("rope_theta", C.c_double),
                ("eps", C.c_double), ("w_embed", F), ("w_norm", F), ("L", C.POINTER(LlamaLayer))]


class GemmaLayer(C.Structure):
    _fields_ = [("head_dim", C.c_int), ("kv_heads", C.c_int), ("rope_theta", C.c_double)] + \
        [(n, F) for n in ("in_ln", "post_ln", "pre_ff_ln", "post_ff_ln", "q_w", "k_w", "v_w", "o_w",
                          "q_norm", "k_norm", "gate", "up", "down", "ple_gate", "ple_proj",
                          "ple_norm")] + [("scalar", C.c_float)]


class Gemma(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("inter", C.c_int),
                ("ple_dim", C.c_int), ("out_dim", C.c_int), ("max_pos", C.c_int),
                ("eps", C.c_double), ("w_embed", F), ("w_ple_proj", F), ("w_ple_norm", F),
                ("w_norm", F), ("w_out", F), ("L", C.POINTER(GemmaLayer))]


def _fp(a):
    return a.ctypes.data_as(F) if a is not None else None


# ---------------------------------------------------------------------------
# st.lisp mirror


def read_safetensors_f32(path):
    """name -> float32 ndarray, widened per st:get-tensor (st.lisp:32-86)."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name, info in header.items():
            if name == "__metadata__":
                continue
            s, e = info["data_offsets"]
            f.seek(base + s)
            raw = f.read(e - s)
            shape = tuple(info["shape"])
            if info["dtype"] == "F32":
                a = np.frombuffer(raw, np.float32).copy()
            elif info["dtype"] == "BF16":
                a = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)
            elif info["dtype"] == "F16":
                src = np.frombuffer(raw, np.uint16).copy()
                a = np.empty(src.size, np.float32)
                lib().or_f16_to_f32(src.ctypes.data_as(C.POINTER(C.c_uint16)), _fp(a),
                                    C.c_int64(src.size))
            else:
                raise ValueError(f"tensor {name} has unsupported dtype {info['dtype']}")
            out[name] = a.reshape(shape)
    return out


class OracleModel:
    """A loaded model for the oracle: family 'bert' | 'mpnet' | 'llama'."""

    def __init__(self, model_dir):
        with open(os.path.join(model_dir, "config.json")) as f:
            cfg = json.load(f)
        tc = cfg.get("text_config")
        mt = (tc or {}).get("model_type") or cfg.get("model_type")
        self.w = read_safetensors_f32(os.path.join(model_dir, "model.safetensors"))
        self._keep = []
        if mt in ("bert", "roberta", "distilbert", "mpnet"):
            self.kind = 0
            self.family = "mpnet" if mt == "mpnet" else "bert"
            H, heads = cfg["hidden_size"], cfg["num_attention_heads"]
            pool_path = os.path.join(model_dir, "1_Pooling", "config.json")
            pooling = 0
            if os.path.exists(pool_path):
                with open(pool_path) as f:
                    pooling = 1 if json.load(f).get("pooling_mode_mean_tokens") else 0
            m = Bert()
            m.hidden, m.layers, m.heads = H, cfg["num_hidden_layers"], heads
            m.head_dim, m.inter, m.pooling = H // heads, cfg["intermediate_size"], pooling
            m.mpnet = 1 if mt == "mpnet" else 0
            m.pos_offset = 2 if mt == "roberta" else 0
            m.causal = 0
            g = self._get
            m.w_word = g("embeddings.word_embeddings.weight")
            m.w_pos = g("embeddings.position_embeddings.weight")
            m.w_type = None if m.mpnet else g("embeddings.token_type_embeddings.weight", opt=True)
            m.emb_g, m.emb_b = g("embeddings.LayerNorm.weight"), g("embeddings.LayerNorm.bias")
            m.rel_bias = g("encoder.relative_attention_bias.weight") if m.mpnet else None
            layers = (BertLayer * m.layers)()
            for li in range(m.layers):
                p = f"encoder.layer.{li}."
                Lw = layers[li]
                if m.mpnet:
                    names = dict(q_w="attention.attn.q.weight", q_b="attention.attn.q.bias",
                                 k_w="attention.attn.k.weight", k_b="attention.attn.k.bias",
                                 v_w="attention.attn.v.weight", v_b="attention.attn.v.bias",
                                 ao_w="attention.attn.o.weight", ao_b="attention.attn.o.bias",
                                 ao_g="attention.LayerNorm.weight", ao_b2="attention.LayerNorm.bias")
                else:
                    names = dict(q_w="attention.self.query.weight", q_b="attention.self.query.bias",
                                 k_w="attention.self.key.weight", k_b="attention.self.key.bias",
                                 v_w="attention.self.value.weight", v_b="attention.self.value.bias",
                                 ao_w="attention.output.dense.weight",
                                 ao_b="attention.output.dense.bias",
                                 ao_g="attention.output.LayerNorm.weight",
                                 ao_b2="attention.output.LayerNorm.bias")
                names.update(ff_w="intermediate.dense.weight", ff_b="intermediate.dense.bias",
                             o_w="output.dense.weight", o_b="output.dense.bias",
                             o_g="output.LayerNorm.weight", o_b2="output.LayerNorm.bias")
                for field, nm in names.items():
                    setattr(Lw, field, g(p + nm))
            m.L = layers
            self._keep.append(layers)
            self.m = m
            self.dim = H
        elif mt in ("llama", "qwen2", "qwen3", "mistral", "gemma", "gemma2"):
            self.kind = 1
            self.family = "llama"
            m = Llama()
            H, heads = cfg["hidden_size"], cfg["num_attention_heads"]
            m.hidden, m.layers, m.heads = H, cfg["num_hidden_layers"], heads
            m.kv_heads = cfg.get("num_key_value_heads") or heads
            m.head_dim = cfg.get("head_dim") or H // heads
            m.inter = cfg["intermediate_size"]
            m.pooling = 0
            m.max_pos = 1024
            m.rope_theta = float(cfg.get("rope_theta", 10000))
            m.eps = float(cfg.get("rms_norm_eps", 1e-6))
            g = self._get
            m.w_embed, m.w_norm = g("embed_tokens.weight"), g("norm.weight")
            layers = (LlamaLayer * m.layers)()
            for li in range(m.layers):
                p = f"layers.{li}."
                Lw = layers[li]
                Lw.in_ln = g(p + "input_layernorm.weight")
                Lw.post_ln = g(p + "post_attention_layernorm.weight")
                Lw.q_w = g(p + "self_attn.q_proj.weight")
                Lw.k_w = g(p + "self_attn.k_proj.weight")
                Lw.v_w = g(p + "self_attn.v_proj.weight")
                Lw.o_w = g(p + "self_attn.o_proj.weight")
                Lw.q_norm = g(p + "self_attn.q_norm.weight", opt=True)
                Lw.k_norm = g(p + "self_attn.k_norm.weight", opt=True)
                Lw.gate = g(p + "mlp.gate_proj.weight")
                Lw.up = g(p + "mlp.up_proj.weight")
                Lw.down = g(p + "mlp.down_proj.weight")
            m.L = layers
            self._keep.append(layers)
            self.m = m
            self.dim = H
        elif mt in ("embedding_gemma2", "embedding_gemma2_text"):  # model.lisp:41
            # gemma:load-model (gemma.lisp:140-212): text_config fields, weights
            # under language_model., per-layer head dim from q_norm and kv heads
            # from k_proj, RoPE theta 1e6 on full_attention layers
            self.kind = 2
            self.family = "gemma"
            t = tc or cfg
            m = Gemma()
            m.hidden, m.layers = t["hidden_size"], t["num_hidden_layers"]
            m.heads, m.inter = t["num_attention_heads"], t["intermediate_size"]
            m.ple_dim = t.get("hidden_size_per_layer_input") or m.hidden
            m.out_dim = t.get("embedding_dim") or 768
            m.max_pos = 2048
            m.eps = float(t.get("rms_norm_eps") or 1e-6)
            g = self._get
            pre = "language_model."
            m.w_embed = g(pre + "embed_tokens.weight")
            m.w_ple_proj = g(pre + "ple.per_layer_model_projection.weight")
            m.w_ple_norm = g(pre + "ple.per_layer_projection_norm.weight")
            m.w_norm = g(pre + "norm.weight")
            m.w_out = g(pre + "embedding_projection.weight")
            types = t.get("layer_types") or []
            layers = (GemmaLayer * m.layers)()
            for li in range(m.layers):
                p = f"{pre}layers.{li}."
                Lw = layers[li]
                hd = self.w[p + "self_attn.q_norm.weight"].shape[0]
                Lw.head_dim = hd
                Lw.kv_heads = self.w[p + "self_attn.k_proj.weight"].shape[0] // hd
                Lw.rope_theta = 1e6 if li < len(types) and types[li] == "full_attention" else 1e4
                for field, nm in dict(
                        in_ln="input_layernorm.weight", post_ln="post_attention_layernorm.weight",
                        pre_ff_ln="pre_feedforward_layernorm.weight",
                        post_ff_ln="post_feedforward_layernorm.weight",
                        q_w="self_attn.q_proj.weight", k_w="self_attn.k_proj.weight",
                        v_w="self_attn.v_proj.weight", o_w="self_attn.o_proj.weight",
                        q_norm="self_attn.q_norm.weight", k_norm="self_attn.k_norm.weight",
                        gate="mlp.gate_proj.weight", up="mlp.up_proj.weight",
                        down="mlp.down_proj.weight",
                        ple_gate="ple_block.per_layer_input_gate.weight",
                        ple_proj="ple_block.per_layer_projection.weight",
                        ple_norm="ple_block.post_per_layer_input_norm.weight").items():
                    setattr(Lw, field, g(p + nm))
                Lw.scalar = float(self.w[p + "layer_scalar"].reshape(-1)[0])
            m.L = layers
            self._keep.append(layers)
            self.m = m
            self.dim = m.out_dim
        else:
            raise ValueError(f"unsupported model_type {mt}")

    def _get(self, name, opt=False):
        a = self.w.get(name)
        if a is None:
            if opt:
                return None
            raise KeyError(name)
        a = np.ascontiguousarray(a, np.float32)
        self._keep.append(a)
        return _fp(a)

    def embed(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(self.dim, np.float32)
        fn = (lib().or_bert_embed, lib().or_llama_embed, lib().or_gemma_embed)[self.kind]
        rc = fn(C.byref(self.m), ids.ctypes.data_as(C.POINTER(C.c_int32)), C.c_int(ids.size),
                _fp(out))
        if rc:
            raise RuntimeError(f"oracle embed failed rc={rc}")
        return out

    def embed_batch(self, ids, offsets, threads=None, seq_threads=1):
        """One thread per sequence in batches of `threads` (embed.lisp's
        scheme); seq_threads > 1 also splits each sequence's token and head
        loops (for long test sequences; the results do not change)."""
        ids = np.ascontiguousarray(ids, np.int32)
        offsets = np.ascontiguousarray(offsets, np.int64)
        nseq = offsets.size - 1
        out = np.zeros((nseq, self.dim), np.float32)
        threads = threads or os.cpu_count() or 1
        lib().or_set_seq_threads(C.c_int(max(1, int(seq_threads))))
        try:
            rc = lib().or_embed_batch(C.c_int(self.kind), C.byref(self.m),
                                      ids.ctypes.data_as(C.POINTER(C.c_int32)),
                                      offsets.ctypes.data_as(C.POINTER(C.c_int64)), C.c_int(nseq),
                                      C.c_int(self.dim), _fp(out), C.c_int(threads))
        finally:
            lib().or_set_seq_threads(C.c_int(1))
        if rc:
            raise RuntimeError(f"oracle embed_batch failed rc={rc}")
        return out


# ---------------------------------------------------------------------------
# IVF


def _i64(a):
    return a.ctypes.data_as(C.POINTER(C.c_int64))


def _u32(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _i32(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def dot(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return lib().or_dot(_fp(a), _fp(b), C.c_int(a.size))


def assign(vecs, cent, rows=None, threads=None):
    vecs = np.ascontiguousarray(vecs, np.float32)
    cent = np.ascontiguousarray(cent, np.float32)
    k, dim = cent.shape
    nrows = vecs.shape[0] if rows is None else len(rows)
    rows_a = None if rows is None else np.ascontiguousarray(rows, np.int64)
    out = np.empty(nrows, np.int32)
    lib().or_assign(_fp(vecs), _i64(rows_a) if rows_a is not None else None,
                    C.c_int64(nrows), _fp(cent), C.c_int(k), C.c_int(dim), _i32(out),
                    C.c_int(threads or os.cpu_count() or 1))
    return out


def assign_scalar(vecs, cent, rows=None, threads=None):
    """assign() computed one row and one centroid at a time (ann.lisp's loop
    shape; the timed CPU baseline)."""
    vecs = np.ascontiguousarray(vecs, np.float32)
    cent = np.ascontiguousarray(cent, np.float32)
    k, dim = cent.shape
    nrows = vecs.shape[0] if rows is None else len(rows)
    rows_a = None if rows is None else np.ascontiguousarray(rows, np.int64)
    out = np.empty(nrows, np.int32)
    lib().or_assign_scalar(_fp(vecs), _i64(rows_a) if rows_a is not None else None,
                           C.c_int64(nrows), _fp(cent), C.c_int(k), C.c_int(dim), _i32(out),
                           C.c_int(threads or os.cpu_count() or 1))
    return out


def kmeans_update(vecs, sample, assignments, cent):
    vecs = np.ascontiguousarray(vecs, np.float32)
    sample = np.ascontiguousarray(sample, np.int64)
    a = np.ascontiguousarray(assignments, np.int32)
    cent = np.array(cent, np.float32, copy=True, order="C")
    k, dim = cent.shape
    lib().or_kmeans_update(_fp(vecs), _i64(sample), C.c_int64(sample.size), _i32(a),
                           C.c_int(k), C.c_int(dim), _fp(cent))
    return cent


def kmeans(vecs, sample, k, iters, threads=None):
    vecs = np.ascontiguousarray(vecs, np.float32)
    sample = np.ascontiguousarray(sample, np.int64)
    dim = vecs.shape[1]
    cent = np.empty((k, dim), np.float32)
    lib().or_kmeans(_fp(vecs), _i64(sample), C.c_int64(sample.size), C.c_int(k), C.c_int(dim),
                    C.c_int(iters), _fp(cent), C.c_int(threads or os.cpu_count() or 1))
    return cent


def assign_all(vecs, cent, threads=None):
    vecs = np.ascontiguousarray(vecs, np.float32)
    cent = np.ascontiguousarray(cent, np.float32)
    k, dim = cent.shape
    counts = np.empty(k, np.uint32)
    lists = np.empty(vecs.shape[0], np.uint32)
    lib().or_assign_all(_fp(vecs), C.c_int64(vecs.shape[0]), _fp(cent), C.c_int(k),
                        C.c_int(dim), _u32(counts), _u32(lists),
                        C.c_int(threads or os.cpu_count() or 1))
    return counts, lists


def top_k_ivf(vecs, cent, counts, lists, nprobe, q, topk):
    vecs = np.ascontiguousarray(vecs, np.float32)
    cent = np.ascontiguousarray(cent, np.float32)
    counts = np.ascontiguousarray(counts, np.uint32)
    lists = np.ascontiguousarray(lists, np.uint32)
    q = np.ascontiguousarray(q, np.float32)
    ids = np.empty(topk, np.int64)
    sc = np.empty(topk, np.float32)
    r = lib().or_top_k_ivf(_fp(vecs), C.c_int(vecs.shape[1]), _fp(cent), C.c_int(cent.shape[0]),
                           _u32(counts), _u32(lists), C.c_int(nprobe), _fp(q), C.c_int(topk),
                           _i64(ids), _fp(sc))
    return ids[:r], sc[:r]


def top_k_brute(vecs, q, topk, threads=8):
    vecs = np.ascontiguousarray(vecs, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    ids = np.empty(topk, np.int64)
    sc = np.empty(topk, np.float32)
    r = lib().or_top_k_brute(_fp(vecs), C.c_int64(vecs.shape[0]), C.c_int(vecs.shape[1]), _fp(q),
                             C.c_int(topk), C.c_int(threads), _i64(ids), _fp(sc))
    return ids[:r], sc[:r]


def mpnet_bucket(i, j):
    return lib().or_mpnet_bucket(C.c_int(i), C.c_int(j))


def ann_bytes(cent, counts, lists, n):
    """The bytes ann::save-ann writes (ann.lisp:165-187): u32 0x414E4E31, k,
    dim, n (write-u32 of each), then the centroids' f32 bit patterns, the k
    counts and the n row ids, all as little-endian (unsigned-byte 32)."""
    import struct
    cent = np.ascontiguousarray(cent, np.float32)
    k, dim = cent.shape
    return (struct.pack("<4I", 0x414E4E31, k, dim, n) + cent.astype("<f4").tobytes()
            + np.asarray(counts, "<u4").tobytes() + np.asarray(lists, "<u4").tobytes())


def index_bytes(rows):
    """index.bin as embed::write-f32 appends it (embed.lisp:47-57): each row's
    f32 bit patterns, little-endian, no header."""
    return np.ascontiguousarray(rows, np.float32).astype("<f4").tobytes()
