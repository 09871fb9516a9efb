"""tokenizer.lisp mirror: texts -> token ids in libembedcuda.so (C++, host
threads).  ``Tokenizer.from_json`` is make-tokenizer-from-json
(tokenizer.lisp:515-552), ``wordpiece`` / ``bpe`` / ``unigram`` are
make-tokenizer (:119-197), ``encode`` is tk-encode (:201-244) for one text and
``encode_batch`` for many at once in ec_embed_batch's packed layout."""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import _lib


class Tokenizer:
    def __init__(self, handle):
        self.handle = handle
        self._tls = threading.local()  # per-thread output buffer, reused across calls

    @classmethod
    def from_json(cls, path):
        h = C.c_int()
        _lib.check(_lib.lib().ec_tokenizer_from_json(str(path).encode(), C.byref(h)),
                   "tokenizer_from_json")
        return cls(h.value)

    @classmethod
    def wordpiece(cls, vocab_txt, lowercase=True):
        h = C.c_int()
        _lib.check(_lib.lib().ec_tokenizer_wordpiece(str(vocab_txt).encode(), int(lowercase),
                                                     C.byref(h)), "tokenizer_wordpiece")
        return cls(h.value)

    @classmethod
    def bpe(cls, vocab_json, merges_txt, lowercase=True, byte_level=False, llama3=False,
            cls_token=None, sep_token=None, unk_token=None, bos=None, eos=None):
        h = C.c_int()
        enc = (lambda s: s.encode() if s is not None else None)
        _lib.check(_lib.lib().ec_tokenizer_bpe(str(vocab_json).encode(), str(merges_txt).encode(),
                                               int(lowercase), int(byte_level), int(llama3),
                                               enc(cls_token), enc(sep_token), enc(unk_token),
                                               -1 if bos is None else bos,
                                               -1 if eos is None else eos, C.byref(h)),
                   "tokenizer_bpe")
        return cls(h.value)

    @classmethod
    def unigram(cls, scores_json, lowercase=True):
        h = C.c_int()
        _lib.check(_lib.lib().ec_tokenizer_unigram(str(scores_json).encode(), int(lowercase),
                                                   C.byref(h)), "tokenizer_unigram")
        return cls(h.value)

    def close(self):
        if self.handle:
            _lib.check(_lib.lib().ec_tokenizer_free(self.handle), "tokenizer_free")
            self.handle = 0

    def vocab_size(self):
        return _lib.check(_lib.lib().ec_tokenizer_vocab_size(self.handle), "vocab_size")

    def encode_batch(self, texts, threads=0):
        """(ids int32[total], offsets int64[n + 1]) for a list of str.  The
        texts go over as one UTF-8 buffer with a pointer per text."""
        n = len(texts)
        if all(t.isascii() for t in texts):
            # one encode for the whole batch: ASCII characters are bytes
            lens = np.fromiter((len(t) for t in texts), np.int64, count=n)
            buf = np.frombuffer(("".join(texts) + "\0").encode("ascii"), np.uint8)
        else:
            raw = [t.encode("utf-8") for t in texts]
            lens = np.fromiter((len(b) for b in raw), np.int64, count=n)
            buf = np.frombuffer(b"".join(raw) + b"\0", np.uint8)
        starts = np.zeros(max(n, 1), np.int64)
        if n:
            starts[1:] = np.cumsum(lens)[:-1]
        ptrs = (buf.ctypes.data + starts).astype(np.uint64)
        offs = np.zeros(n + 1, np.int64)
        cap = 512 * n
        ids = getattr(self._tls, "ids", None)
        if ids is None or ids.size < max(cap, 1):
            ids = self._tls.ids = np.empty(max(cap, 1), np.int32)
        _lib.check(_lib.lib().ec_tokenize(self.handle, ptrs.ctypes.data_as(C.POINTER(C.c_char_p)),
                                          _lib.ptr(lens, C.c_int64) if n else None, n,
                                          _lib.ptr(ids, C.c_int32), cap, _lib.ptr(offs, C.c_int64),
                                          threads), "tokenize")
        return ids[:offs[-1]].copy(), offs

    def encode(self, text):
        ids, _ = self.encode_batch([text], threads=1)
        return ids

    def decode(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        n = C.c_int64()
        L = _lib.lib()
        L.ec_tokenizer_decode(self.handle, _lib.ptr(ids, C.c_int32), ids.size, None, 0, C.byref(n))
        buf = C.create_string_buffer(max(n.value, 1))
        _lib.check(L.ec_tokenizer_decode(self.handle, _lib.ptr(ids, C.c_int32), ids.size, buf,
                                         n.value, C.byref(n)), "decode")
        return buf.raw[:n.value].decode("utf-8")
