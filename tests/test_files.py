"""The index files of the IVF path read and written by the library
(ec_files.cu) against the reference's formats: ann.bin (ann.lisp:165-187,
kb.lisp:283-314) and index.bin (embed.lisp:47-57, kb.lisp:84-129).

The host-only entry points (ec_ann_save / ec_ann_read) run on the CPU; the
rest need a GPU and are marked."""
import struct

import numpy as np
import pytest

from embedcuda import _lib, ann, kb, model, synth
from oracle import oracle


def _toy(k=7, d=12, n=50, seed=0):
    rng = np.random.default_rng(seed)
    cent = rng.standard_normal((k, d)).astype(np.float32)
    a = rng.integers(0, k, n)
    counts = np.bincount(a, minlength=k).astype(np.uint32)
    lists = np.argsort(a, kind="stable").astype(np.uint32)
    return cent, counts, lists, n


def test_ann_save_bytes_match_reference_format(tmp_path):
    cent, counts, lists, n = _toy()
    p = tmp_path / "ann.bin"
    ann.save_ann(p, cent, counts, lists, n)
    assert p.read_bytes() == oracle.ann_bytes(cent, counts, lists, n)


def test_ann_read_round_trip_and_header(tmp_path):
    cent, counts, lists, n = _toy(k=5, d=384, n=1000, seed=3)
    p = tmp_path / "ann.bin"
    p.write_bytes(oracle.ann_bytes(cent, counts, lists, n))
    got = ann.load_ann(p)
    assert got is not None
    assert np.array_equal(got[0], cent) and np.array_equal(got[1], counts)
    assert np.array_equal(got[2], lists)


def test_ann_file_errors(tmp_path):
    cent, counts, lists, n = _toy()
    good = oracle.ann_bytes(cent, counts, lists, n)
    bad_magic = tmp_path / "m.bin"
    bad_magic.write_bytes(b"XXXX" + good[4:])
    assert ann.load_ann(bad_magic) is None            # kb::load-ann ignores it
    import ctypes as C
    k, d, nn = C.c_int(), C.c_int(), C.c_int64()
    rc = _lib.lib().ec_ann_read(str(bad_magic).encode(), C.byref(k), C.byref(d), C.byref(nn),
                                None, None, None)
    assert rc == _lib.EC_EINVAL
    short = tmp_path / "t.bin"
    short.write_bytes(good[:-4])                      # truncated ids
    rc = _lib.lib().ec_ann_read(str(short).encode(), C.byref(k), C.byref(d), C.byref(nn),
                                None, None, None)
    assert rc == _lib.EC_EINVAL
    # k = d = 2^31 - 1 and n = 2^31 + 16: 16 + (k*d + k + n) * 4 wraps around
    # 2^64 to exactly this file's 80 bytes; the header must still be refused
    wrap = tmp_path / "w.bin"
    wrap.write_bytes(struct.pack("<4I", 0x414E4E31, 0x7FFFFFFF, 0x7FFFFFFF, 0x80000010) + bytes(64))
    rc = _lib.lib().ec_ann_read(str(wrap).encode(), C.byref(k), C.byref(d), C.byref(nn),
                                None, None, None)
    assert rc == _lib.EC_EINVAL and "header says k" in _lib.last_error()
    with pytest.raises(_lib.EcError):                 # counts do not sum to n
        ann.save_ann(tmp_path / "c.bin", cent, counts, lists, n + 1)


@pytest.mark.gpu
def test_index_load_files_matches_in_memory(tmp_path, ec):
    x, _ = synth.make_ivf_corpus(20000, 384, 64, seed=4)
    sample = synth.make_ivf_sample(len(x), 4)
    cent = ann.kmeans(x, sample, 64, 3)
    counts, lists = ann.assign_all(x, cent)
    (tmp_path / "index.bin").write_bytes(oracle.index_bytes(x))
    ann.save_ann(tmp_path / "ann.bin", cent, counts, lists, len(x))
    q = x[:5] + 0.01
    kb.load_index(x, (cent, counts, lists))
    want_ivf = kb.search_ivf(q, 10, 32)
    want_flat = kb.search_brute(q, 10)
    n = kb.load_index_files(tmp_path / "index.bin", 384, tmp_path / "ann.bin")
    assert n == len(x)
    got_ivf = kb.search_ivf(q, 10, 32)
    assert np.array_equal(got_ivf[0], want_ivf[0]) and np.array_equal(got_ivf[1], want_ivf[1])
    assert kb.load_index_files(tmp_path / "index.bin", 384) == len(x)   # flat only
    got_flat = kb.search_brute(q, 10)
    assert np.array_equal(got_flat[0], want_flat[0]) and np.array_equal(got_flat[1], want_flat[1])
    with pytest.raises(_lib.EcError):                 # ann.bin of another dimension
        kb.load_index_files(tmp_path / "index.bin", 192, tmp_path / "ann.bin")


@pytest.mark.gpu
def test_ann_build_file_bytes_equal_oracle(tmp_path, ec):
    """ann:run from index.bin to ann.bin: the file equals the oracle's k-means
    + assign-all written in ann::save-ann's format, byte for byte."""
    x, _ = synth.make_ivf_corpus(12000, 256, 32, seed=5)
    sample = synth.make_ivf_sample(len(x), 5)[:6000]
    (tmp_path / "index.bin").write_bytes(oracle.index_bytes(x))
    ann.build_file(tmp_path / "index.bin", 256, 128, 3, sample, tmp_path / "ann.bin")
    cent = oracle.kmeans(x, sample, 128, 3)
    counts, lists = oracle.assign_all(x, cent)
    assert (tmp_path / "ann.bin").read_bytes() == oracle.ann_bytes(cent, counts, lists, len(x))


@pytest.mark.gpu
def test_embed_batch_to_file_appends_rows(tmp_path, ec, synth_root):
    s = synth.with_layers(synth.MINILM, 2)
    model.load_model(synth.build_model_dir(s, 0, synth_root))
    ids, offs = synth.make_short_inputs("minilm", [5, 40, 130], 0, s.vocab)
    p = tmp_path / "index.bin"
    model.embed_batch_to_file(ids, offs, p)
    model.embed_batch_to_file(ids, offs, p)
    rows = model.embed_batch(ids, offs)
    assert p.read_bytes() == oracle.index_bytes(np.concatenate([rows, rows]))
