"""tokenizer.lisp in the library (ec_tokenizer.cu) against the committed
golden ids of its Python restatement (oracle/tokenizer_ref.py) on tokenizers
trained for the purpose (tests/golden/make_tokenizers.py): WordPiece and
byte-level BPE from tokenizer.json, vocab.txt and vocab.json + merges.txt,
GPT-2 and Llama-3 style pre-tokenizers, Unigram scores.  Host-only: no GPU."""
import json
import os

import numpy as np
import pytest

from embedcuda import _lib
from embedcuda.tokenizer import Tokenizer
from oracle import tokenizer_ref as ref

TOK = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tok")


def _p(name):
    return os.path.join(TOK, name)


@pytest.fixture(scope="module")
def texts():
    with open(_p("texts.json"), encoding="utf-8") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def expected():
    with open(_p("expected.json")) as f:
        return json.load(f)


def _bpe_ids():
    with open(_p("bpe_gpt2.json"), encoding="utf-8") as f:
        v = json.load(f)["model"]["vocab"]
    return v["<s>"], v["</s>"]


def _ours(name):
    if name == "wordpiece_json":
        return Tokenizer.from_json(_p("wordpiece.json"))
    if name == "bpe_gpt2_json":
        return Tokenizer.from_json(_p("bpe_gpt2.json"))
    if name == "bpe_llama3_json":
        return Tokenizer.from_json(_p("bpe_llama3.json"))
    if name == "wordpiece_txt":
        return Tokenizer.wordpiece(_p("vocab.txt"))
    if name == "bpe_files":
        bos, eos = _bpe_ids()
        return Tokenizer.bpe(_p("vocab.json"), _p("merges.txt"), lowercase=False, byte_level=True,
                             llama3=True, unk_token="<unk>", bos=bos, eos=eos)
    if name == "unigram":
        return Tokenizer.unigram(_p("unigram.json"))
    raise KeyError(name)


NAMES = ["wordpiece_json", "bpe_gpt2_json", "bpe_llama3_json", "wordpiece_txt", "bpe_files",
         "unigram"]


@pytest.mark.parametrize("name", NAMES)
def test_library_matches_golden(texts, expected, name):
    tk = _ours(name)
    ids, offs = tk.encode_batch(texts)
    got = [ids[offs[i]:offs[i + 1]].tolist() for i in range(len(texts))]
    for i, (g, e) in enumerate(zip(got, expected[name])):
        assert g == e, (name, i, texts[i][:60])
    # one text at a time and a single thread give the same ids
    ids1, offs1 = tk.encode_batch(texts, threads=1)
    assert np.array_equal(ids1, ids) and np.array_equal(offs1, offs)
    assert tk.encode(texts[3]).tolist() == expected[name][3]
    tk.close()


def test_restatement_matches_golden(texts, expected):
    """The oracle itself, recomputed, against its committed output."""
    tk = ref.from_json(_p("bpe_llama3.json"))
    assert [tk.encode(t) for t in texts] == expected["bpe_llama3_json"]
    tk = ref.from_json(_p("wordpiece.json"))
    assert [tk.encode(t) for t in texts] == expected["wordpiece_json"]


def test_restatement_pinned_to_hf_tokenizers(texts):
    """Where tokenizer.lisp and Hugging Face tokenizers do the same thing --
    ASCII text, single spaces, no apostrophes, WordPiece with the usual
    advance (the Lisp's counts the "##") -- the restatement equals HF."""
    hf = pytest.importorskip("tokenizers")
    wp_hf = hf.Tokenizer.from_file(_p("wordpiece.json"))
    bpe_hf = hf.Tokenizer.from_file(_p("bpe_gpt2.json"))
    wp = ref.from_json(_p("wordpiece.json"))
    wp.lisp_advance = False
    bpe = ref.from_json(_p("bpe_gpt2.json"))
    n = 0
    for t in texts[160:240]:
        if "'" in t:
            continue
        assert wp_hf.encode(t).ids == wp.encode(t)
        assert bpe_hf.encode(t).ids == bpe.encode(t)
        n += 1
    assert n >= 30


def test_lisp_quirks_reproduced():
    tk = Tokenizer.from_json(_p("wordpiece.json"))
    r = ref.from_json(_p("wordpiece.json"))
    long_word = "x" * 101                       # > 100 characters -> [UNK]
    assert tk.encode(long_word).tolist() == r.encode(long_word)
    assert r.inv[r.encode(long_word)[1]] == "[UNK]"
    u = Tokenizer.unigram(_p("unigram.json"))   # Viterbi ids looked up as strings -> [UNK]
    ids = u.encode("kato rina").tolist()
    assert len(ids) >= 2 and len(set(ids)) == 1
    tk.close()
    u.close()


def test_truncation_and_decode(texts):
    tk = Tokenizer.from_json(_p("bpe_gpt2.json"))
    r = ref.from_json(_p("bpe_gpt2.json"))
    long = texts[-1]
    ids = tk.encode(long)
    assert len(ids) == 512 and ids.tolist() == r.encode(long)   # BOS + 510 + EOS
    assert tk.decode(ids[:20]) == r.decode(ids[:20].tolist())
    tk.close()


def test_errors():
    tk = Tokenizer.from_json(_p("wordpiece.json"))
    import ctypes as C
    bad = (C.c_char_p * 1)(b"ok \xff\xfe")
    offs = np.zeros(2, np.int64)
    ids = np.zeros(16, np.int32)
    rc = _lib.lib().ec_tokenize(tk.handle, bad, None, 1, _lib.ptr(ids, C.c_int32), 16,
                                _lib.ptr(offs, C.c_int64), 1)
    assert rc == _lib.EC_EINVAL                  # malformed UTF-8
    good = (C.c_char_p * 1)(b"kato rina mose " * 20)
    rc = _lib.lib().ec_tokenize(tk.handle, good, None, 1, _lib.ptr(ids, C.c_int32), 4,
                                _lib.ptr(offs, C.c_int64), 1)
    assert rc == _lib.EC_EINVAL and offs[1] > 4   # the count needed is reported
    # a NULL text: an error unless its length is given as 0 (an empty text);
    # a negative length: an error (neither is read)
    two = (C.c_char_p * 2)(b"kato", None)
    offs3 = np.zeros(3, np.int64)
    rc = _lib.lib().ec_tokenize(tk.handle, two, None, 2, _lib.ptr(ids, C.c_int32), 16,
                                _lib.ptr(offs3, C.c_int64), 1)
    assert rc == _lib.EC_EINVAL and "text 1: NULL" in _lib.last_error()
    for lens, want in (([4, 0], _lib.EC_OK), ([4, 3], _lib.EC_EINVAL), ([-1, 0], _lib.EC_EINVAL)):
        la = np.array(lens, np.int64)
        rc = _lib.lib().ec_tokenize(tk.handle, two, _lib.ptr(la, C.c_int64), 2,
                                    _lib.ptr(ids, C.c_int32), 16, _lib.ptr(offs3, C.c_int64), 1)
        assert rc == want, (lens, _lib.last_error())
    # the empty text yields what encoding "" yields
    assert offs3[2] - offs3[1] == len(tk.encode(""))
    out = C.create_string_buffer(8)
    n = C.c_int64()
    assert _lib.lib().ec_tokenizer_decode(tk.handle, None, 3, out, 8, C.byref(n)) == _lib.EC_EINVAL
    assert _lib.lib().ec_tokenizer_decode(tk.handle, None, -1, out, 8, C.byref(n)) == _lib.EC_EINVAL
    with pytest.raises(_lib.EcError):
        Tokenizer.from_json(_p("texts.json"))    # not a tokenizer.json
    tk.close()
    with pytest.raises(_lib.EcError):
        tk.handle = 12345
        tk.vocab_size()


def test_malformed_files_are_refused(tmp_path):
    """Damaged tokenizer files end in EC_EINVAL with a message, never in an
    exception through the C ABI: an integer that is only a sign or does not
    fit int64, nesting deeper than the reader's limit, a vocabulary id
    outside [0, 2^24) (ids index the decode table)."""
    import ctypes as C

    def load(text, kind="json"):
        p = tmp_path / "t.json"
        p.write_text(text)
        h = C.c_int()
        if kind == "json":
            return _lib.lib().ec_tokenizer_from_json(str(p).encode(), C.byref(h)), h.value
        return _lib.lib().ec_tokenizer_unigram(str(p).encode(), 0, C.byref(h)), h.value

    wp = '{"model": {"type": "WordPiece", "unk_token": "a", "vocab": {"a": 0, "b": %s}}}'
    for bad, msg in (("-", "bad number"), ("+1", "bad number"),
                     ("9223372036854775808", "out of range"), ("99999999999999999999", "out of range"),
                     ("-1", "outside"), ("16777216", "outside"), ("2147483647", "outside")):
        rc, _ = load(wp % bad)
        assert rc == _lib.EC_EINVAL and msg in _lib.last_error(), (bad, _lib.last_error())
    rc, _ = load("[" * 100000)
    assert rc == _lib.EC_EINVAL and "nested too deeply" in _lib.last_error()
    rc, _ = load('{"a": -}', "unigram")
    assert rc == _lib.EC_EINVAL and "bad number" in _lib.last_error()
    # the edges that are valid still load
    rc, h = load(wp % "151668")
    assert rc == _lib.EC_OK and _lib.lib().ec_tokenizer_vocab_size(h) == 151669
    assert _lib.lib().ec_tokenizer_free(h) == _lib.EC_OK
    rc, h = load('{"a": -9223372036854775808, "b": 9223372036854775807}', "unigram")
    assert rc == _lib.EC_OK and _lib.lib().ec_tokenizer_free(h) == _lib.EC_OK


def test_random_texts_match_restatement(texts):
    """Seeded random texts -- ASCII, whitespace runs and Unicode spaces,
    controls, accents, case pairs with special lowering (dotted I, title-case
    digraphs), ligatures, CJK, Hangul, emoji with modifiers, combining marks,
    zero-width space, apostrophes -- through every tokenizer type: the
    library's ids equal the restatement's, or both reject the text (a piece
    with no id and no unknown token).  The Unigram texts use the characters
    of the golden texts, which its fixture's scores cover."""
    rng = np.random.default_rng(11)
    ascii_ = [chr(c) for c in range(32, 127)]
    extra = list("\t\n\r\x0b\x0c   　éÉßñÀçœ"
                 "日本語中文한국어\U0001f600\U0001f44d\U0001f3fd"
                 "’'`0123456789¡¿«»—–…́​"
                 "\x00\x07ǅİıﬁ")
    golden_chars = sorted(set("".join(texts)))

    def gen(alpha, n):
        return ["".join(alpha[int(i)] for i in rng.integers(0, len(alpha), int(rng.integers(0, 60))))
                for _ in range(n)]

    full = ascii_ * 3 + extra
    cases = [
        ("wordpiece_json", ref.from_json(_p("wordpiece.json")), full),
        ("bpe_gpt2_json", ref.from_json(_p("bpe_gpt2.json")), full),
        ("bpe_llama3_json", ref.from_json(_p("bpe_llama3.json")), full),
        ("wordpiece_txt", ref.from_vocab_txt(_p("vocab.txt")), full),
        ("unigram", ref.from_unigram_scores(_p("unigram.json")), golden_chars),
        # pure-ASCII texts take the library's byte-level WordPiece path
        ("wordpiece_json", ref.from_json(_p("wordpiece.json")), ascii_ + list("\t\n\r\x0b\x0c\x00\x07")),
        ("wordpiece_txt", ref.from_vocab_txt(_p("vocab.txt")), ascii_ + list("\t\n\r\x0b\x0c\x00\x07")),
    ]
    for name, theirs, alpha in cases:
        ours = _ours(name)
        for t in gen(alpha, 300):
            try:
                got = ours.encode(t).tolist()
            except _lib.EcError:
                got = None
            try:
                want = theirs.encode(t)
            except (KeyError, ValueError):
                want = None
            assert got == want, (name, t)
        ours.close()
    # words of exactly 100 and 101 characters (the limit past which a word is
    # one unknown piece), ASCII and not
    wp = ref.from_json(_p("wordpiece.json"))
    ours = _ours("wordpiece_json")
    for t in ["ka" * 50 + " x", "ka" * 50 + "k y", "é" + "ka" * 49 + "k z", "é" + "ka" * 50 + " w"]:
        assert ours.encode(t).tolist() == wp.encode(t), t
    ours.close()


def test_encode_batch_from_threads(texts):
    """encode_batch on one tokenizer from several Python threads at once
    (the library call runs without the GIL) gives each caller its own ids."""
    import threading
    tk = _ours("wordpiece_json")
    want = [tk.encode_batch(texts[i::4]) for i in range(4)]
    got = [None] * 4

    def run(i):
        for _ in range(5):
            got[i] = tk.encode_batch(texts[i::4])

    th = [threading.Thread(target=run, args=(i,)) for i in range(4)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    for (wi, wo), (gi, go) in zip(want, got):
        assert np.array_equal(wi, gi) and np.array_equal(wo, go)
    tk.close()
