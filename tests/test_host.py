"""Host-side logic without a GPU: the seeded workload generator, the
safetensors reader of the host mirror (st.lisp), the ann.bin format
(ann.lisp:4-6, 165-187) and the benchmark's FLOP accounting."""
import json
import os
import struct

import numpy as np

from embedcuda import ann, st, synth


def test_inputs_match_the_workload_spec():
    ids, offs = synth.make_inputs("minilm", 1024, 0)
    lens = np.diff(offs)
    assert len(lens) == 1024 and lens.min() >= 16 and lens.max() <= 256
    first = ids[offs[:-1]]
    last = ids[offs[1:] - 1]
    assert np.all(first == 101) and np.all(last == 102)
    body = np.concatenate([ids[offs[i] + 1:offs[i + 1] - 1] for i in range(1024)])
    assert body.min() >= 1000 and body.max() <= 30521
    ids2, offs2 = synth.make_inputs("minilm", 1024, 0)
    assert np.array_equal(ids, ids2) and np.array_equal(offs, offs2)  # seeded
    q, qo = synth.make_inputs("qwen3", 64, 3)
    ql = np.diff(qo)
    assert ql.min() >= 129 and ql.max() <= 513 and np.all(q[qo[1:] - 1] == 151643)
    b, bo = synth.make_inputs("bert", 512, 1)
    bl = np.diff(bo)
    assert bl.min() >= 32 and bl.max() <= 512
    m, mo = synth.make_inputs("mpnet", 256, 2)
    ml = np.diff(mo)
    assert ml.min() >= 64 and ml.max() <= 384 and np.all(m[mo[:-1]] == 0) and np.all(m[mo[1:] - 1] == 2)


def test_safetensors_layout_and_bf16_rounding(tmp_path):
    s = synth.with_layers(synth.BERT_BASE, 1, vocab=64)
    d = synth.build_model_dir(s, 1, str(tmp_path))
    header, start = st.parse_header(os.path.join(d, "model.safetensors"))
    names = st.tensor_names(header)
    assert "encoder.layer.0.attention.self.query.weight" in names
    info = header["embeddings.word_embeddings.weight"]
    assert info["dtype"] == "BF16" and info["shape"] == [64, 768]
    with open(os.path.join(d, "config.json")) as f:
        cfg = json.load(f)
    assert cfg["model_type"] == "bert" and cfg["hidden_size"] == 768
    assert not os.path.exists(os.path.join(d, "1_Pooling", "config.json")) or \
        not json.load(open(os.path.join(d, "1_Pooling", "config.json")))["pooling_mode_mean_tokens"]
    # round-to-nearest-even to bf16
    a = np.array([1.0, 1.00390625, 1.01171875, -3.0e-39], np.float32)
    bits = synth.f32_to_bf16_bits(a)
    assert list(bits[:3]) == [0x3F80, 0x3F80, 0x3F82]


def test_ann_bin_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    cent = rng.standard_normal((5, 384)).astype(np.float32)
    counts = np.array([3, 0, 2, 1, 4], np.uint32)
    lists = rng.permutation(10).astype(np.uint32)
    p = str(tmp_path / "ann.bin")
    ann.save_ann(p, cent, counts, lists, 10)
    with open(p, "rb") as f:
        assert struct.unpack("<4I", f.read(16)) == (0x414E4E31, 5, 384, 10)
    assert os.path.getsize(p) == 4 * (4 + 5 * 384 + 5 + 10)
    c2, n2, l2 = ann.load_ann(p)
    assert np.array_equal(c2, cent) and np.array_equal(n2, counts) and np.array_equal(l2, lists)


def test_bench_flop_accounting():
    import bench
    offs = np.array([0, 100, 300], np.int64)
    f = bench.algorithmic_flops(synth.MINILM, offs)
    H, F, L = 384, 1536, 6
    want = L * sum(2 * n * (4 * H * H + 2 * H * F) + 4 * n * n * H for n in (100, 200))
    assert f == want
    ids, offsets = synth.make_inputs("minilm", 1024, 0)
    total = bench.algorithmic_flops(synth.MINILM, offsets)
    assert 3.0e12 < total < 3.4e12  # the ~3.18e12 of the workload spec


def test_bench_reference_arm_lines_for_other_workloads():
    """--impl reference prints one JSON line and exits 0 for every workload
    name (the reference arm times the embedding workloads only)."""
    import json
    import subprocess
    import sys
    from conftest import REPO
    for wl in ("ivf", "query", "search", "tokenize"):
        p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", wl,
                            "--steps", "1", "--warmup", "3"], cwd=REPO, capture_output=True,
                           text=True, timeout=300)
        assert p.returncode == 0, p.stderr
        line = json.loads(p.stdout.strip().splitlines()[-1])
        assert line["impl"] == "reference" and "unavailable" in line, wl


def test_bench_search_options():
    import bench
    import sys
    argv = sys.argv
    try:
        sys.argv = ["bench.py", "--workload", "search", "--search-rows", "800000", "--search-k", "1024",
                    "--search-queries", "2500"]
        a = bench.parse_args()
    finally:
        sys.argv = argv
    assert (a.search_rows, a.search_k, a.search_queries) == (800000, 1024, 2500)
    assert bench.SEARCH_NQ == 10_000 and bench.IVF_N == 3_270_000


def test_search_cpu_baseline_threads():
    """The search workload's CPU baseline runs the oracle's kb::top-k-ivf on
    several threads at once; the C restatement is re-entrant, so concurrent
    calls give the single-threaded results."""
    import threading
    import bench
    from oracle import oracle
    x, _ = synth.make_ivf_corpus(4000, 64, 16, seed=4)
    cent = x[:32].copy()
    counts, lists = oracle.assign_all(x, cent)
    qs, _ = synth.make_ivf_corpus(24, 64, 16, seed=5)
    done, el, threads = bench.search_cpu_baseline(x, cent, counts, lists, qs, 8, 10, 5.0, threads=4)
    assert threads == 4 and done == len(qs) and el > 0
    ref = [oracle.top_k_ivf(x, cent, counts, lists, 8, q, 10) for q in qs]
    got = [None] * len(qs)

    def run(i):
        got[i] = oracle.top_k_ivf(x, cent, counts, lists, 8, qs[i], 10)

    th = [threading.Thread(target=run, args=(i,)) for i in range(len(qs))]
    for t in th:
        t.start()
    for t in th:
        t.join()
    for (ri, rs), (gi, gs) in zip(ref, got):
        assert np.array_equal(ri, gi) and np.array_equal(rs, gs)


def test_bench_rank_shards_balanced():
    """N > 1: every rank gets the workload's sequence count from one seeded
    pool, with (nearly) equal token counts, and the shards partition the pool."""
    import bench
    for world in (2, 4, 8):
        tot = []
        seen = 0
        for r in range(world):
            ids, offs = bench.rank_inputs("minilm-l6", 1024, 0, r, world)
            assert len(offs) - 1 == 1024
            tot.append(int(offs[-1]))
            seen += int(offs[-1])
        pool_ids, pool_offs = synth.make_inputs("minilm-l6", 1024 * world, 0)
        assert seen == int(pool_offs[-1])
        assert max(tot) - min(tot) <= 0.01 * max(tot), tot
    ids1, offs1 = bench.rank_inputs("minilm-l6", 1024, 0, 0, 1)
    ref_ids, ref_offs = synth.make_inputs("minilm-l6", 1024, 0)
    assert np.array_equal(ids1, ref_ids) and np.array_equal(offs1, ref_offs)


def test_bench_reference_config_matches_ours():
    """Both arms print the same `config` object for the same run."""
    import bench
    for world in (1, 4):
        ids, offs = bench.rank_inputs("minilm-l6", 1024, 0, 0, world)
        a = bench.workload_config("minilm", world, int(offs[-1]))
        assert a["workload"] == "minilm-l6" and a["parallelism"] == f"dp{world} (sequence shards)"
        assert a["tokens_per_rank"] == int(offs[-1])


def test_mirror_refuses_arrays_the_library_would_misread(monkeypatch):
    """The C calls take raw pointers and counts, so the host mirror checks the
    shapes it knows before any call: query width against the loaded index,
    initial centroids against k x dim, centroid width, the ann arrays'
    lengths, packed offsets within ids, and a caller's output buffer.  Each
    case raises before the library is reached (no GPU needed)."""
    import pytest
    from embedcuda import kb, model

    monkeypatch.setitem(kb._state, "dim", 8)
    with pytest.raises(ValueError, match="index has dim 8"):
        kb.search_brute(np.zeros((2, 7), np.float32), 3)
    with pytest.raises(ValueError, match="index has dim 8"):
        kb.search_ivf(np.zeros((2, 3, 8), np.float32), 3)
    x = np.zeros((10, 8), np.float32)
    with pytest.raises(ValueError, match="ann must be"):
        kb.load_index(x, (np.zeros((4, 7), np.float32), np.zeros(4, np.uint32), np.zeros(10, np.uint32)))
    with pytest.raises(ValueError, match="ann must be"):
        kb.load_index(x, (np.zeros((4, 8), np.float32), np.zeros(3, np.uint32), np.zeros(10, np.uint32)))
    with pytest.raises(ValueError, match="ann must be"):
        kb.load_index(x, (np.zeros((4, 8), np.float32), np.zeros(4, np.uint32), np.zeros(9, np.uint32)))
    sample = np.arange(10, dtype=np.int64)
    with pytest.raises(ValueError, match=r"need \(4, 8\)"):
        ann.kmeans(x, sample, 4, 1, init=np.zeros((3, 8), np.float32))
    with pytest.raises(ValueError, match=r"need \(4, 8\)"):
        ann.build(x, sample, 4, 1, init=np.zeros(32, np.float32))
    with pytest.raises(ValueError, match=r"need \(k, 8\)"):
        ann.assign(x, np.zeros((4, 16), np.float32))
    with pytest.raises(ValueError, match=r"need \(k, 8\)"):
        ann.assign_all(x, np.zeros(32, np.float32))
    ids = np.arange(20, dtype=np.int32)
    for offs in ([0, 5, 21], [0, 9, 5], [-1, 5], []):
        with pytest.raises(ValueError, match="offsets"):
            model.embed_batch(ids, np.array(offs, np.int64))
    monkeypatch.setattr(model, "dim", lambda: 384)
    offs = np.array([0, 5, 20], np.int64)
    for out in (np.zeros((2, 384), np.float64), np.zeros((1, 384), np.float32),
                np.zeros((2, 383), np.float32), np.zeros((384, 2), np.float32).T):
        with pytest.raises(ValueError, match="out must be"):
            model.embed_batch(ids, offs, out=out)


def test_model_configs_parse_with_the_library_json_reader(tmp_path):
    """config.json of every model shape goes through the library's one JSON
    reader (ec_json.h), shared with the tokenizer loader: loading it as a
    tokenizer.json must fail only for the missing "model" key, after a clean
    parse (integers, floats such as 1e-12, nested objects, null)."""
    import ctypes as C
    from embedcuda import _lib
    for name in ("MINILM", "BERT_BASE", "MPNET_BASE", "QWEN3_06B", "GEMMA_EMB"):
        cfg = synth.config_json(getattr(synth, name))
        cfg["rope_scaling"] = None
        cfg["eos_token_id"] = [1, -2, 9223372036854775807]
        p = tmp_path / f"{name}.json"
        p.write_text(json.dumps(cfg, indent=1))
        h = C.c_int()
        rc = _lib.lib().ec_tokenizer_from_json(str(p).encode(), C.byref(h))
        assert rc == _lib.EC_EINVAL and _lib.last_error().endswith("no model"), (name, _lib.last_error())
