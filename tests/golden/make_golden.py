"""Regenerate tests/golden/embed_golden.npz.

For three small seeded models (MiniLM shape with 2 layers, MPNet shape with
2 layers, Qwen3 shape with 2 layers and a 4096-token vocab) this stores the
token ids, the embeddings computed by Hugging Face transformers (an
independent implementation of the same published architectures, run in fp32
on CPU with the identical synthetic weights) and the embeddings of the CPU
oracle, plus a checksum of the weights so a change in the generator shows up
as a fixture mismatch instead of a silent drift.

    python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "lisp-embed_b200"))

from embedcuda import synth  # noqa: E402
from oracle import oracle  # noqa: E402

CASES = [
    ("minilm", synth.with_layers(synth.MINILM, 2), 0, [1, 5, 17, 64, 130]),
    ("mpnet", synth.with_layers(synth.MPNET_BASE, 2), 2, [2, 9, 65, 140]),
    ("qwen3", synth.with_layers(synth.QWEN3_06B, 2, vocab=4096), 3, [1, 3, 40, 70]),
]


def weights_digest(w):
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(np.ascontiguousarray(w[k], np.float32).tobytes())
    return h.hexdigest()


def hf_embed(name, s, w, ids, offs):
    import torch
    sd = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in w.items()}
    if name == "minilm":
        from transformers import BertConfig, BertModel
        m = BertModel(BertConfig(vocab_size=s.vocab, hidden_size=s.hidden,
                                 num_hidden_layers=s.layers, num_attention_heads=s.heads,
                                 intermediate_size=s.inter, max_position_embeddings=s.max_pos,
                                 layer_norm_eps=1e-12), add_pooling_layer=False)
        pool = "mean"
    elif name == "mpnet":
        from transformers import MPNetConfig, MPNetModel
        m = MPNetModel(MPNetConfig(vocab_size=s.vocab, hidden_size=s.hidden,
                                   num_hidden_layers=s.layers, num_attention_heads=s.heads,
                                   intermediate_size=s.inter, max_position_embeddings=s.max_pos,
                                   layer_norm_eps=1e-12, relative_attention_num_buckets=32,
                                   pad_token_id=1), add_pooling_layer=False)
        pool = "mean"
    else:
        from transformers import Qwen3Config, Qwen3Model
        m = Qwen3Model(Qwen3Config(vocab_size=s.vocab, hidden_size=s.hidden,
                                   num_hidden_layers=s.layers, num_attention_heads=s.heads,
                                   num_key_value_heads=s.kv_heads, head_dim=s.head_dim,
                                   intermediate_size=s.inter, rope_theta=s.rope_theta,
                                   rms_norm_eps=s.rms_eps, max_position_embeddings=40960))
        pool = "last"
    m.load_state_dict(sd, strict=True)
    m.eval()
    out = []
    for i in range(len(offs) - 1):
        x = torch.from_numpy(ids[offs[i]:offs[i + 1]].astype(np.int64))[None]
        with torch.no_grad():
            h = m(input_ids=x).last_hidden_state[0]
        v = h.mean(0) if pool == "mean" else h[-1]
        out.append((v / v.norm()).numpy())
    return np.stack(out).astype(np.float32)


def main():
    root = os.environ.get("EC_SYNTH_DIR", "/tmp/ec_synth")
    data = {}
    for name, s, seed, lens in CASES:
        d = synth.build_model_dir(s, seed, root)
        om = oracle.OracleModel(d)
        wname = "qwen3" if name == "qwen3" else name
        ids, offs = synth.make_short_inputs(wname, lens, seed, s.vocab)
        data[f"{name}_ids"] = ids
        data[f"{name}_offsets"] = offs
        data[f"{name}_oracle"] = om.embed_batch(ids, offs)
        data[f"{name}_hf"] = hf_embed(name, s, om.w, ids, offs)
        data[f"{name}_digest"] = np.frombuffer(bytes.fromhex(weights_digest(om.w)), np.uint8)
    np.savez_compressed(os.path.join(HERE, "embed_golden.npz"), **data)
    print("wrote", os.path.join(HERE, "embed_golden.npz"))


if __name__ == "__main__":
    main()
