"""Search scoring -- the kb.lisp mirror (kb.lisp:153-200, 276-368).

``load_index`` keeps index.bin vectors (and ann.bin when given) resident on
the GPUs; ``top_k`` dispatches to ``top_k_ivf`` when an IVF index is loaded
and to ``top_k_brute`` otherwise, returning ``[(row, score), ...]`` in
descending score order like kb::top-k.  Batched variants take [nq, dim].
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib

ann_nprobe = 64  # kb::*ann-nprobe* (kb.lisp:281)
_state = {"ivf": False, "dim": 0}


def load_index(vectors, ann=None):
    """vectors float32[n, dim]; ann = (centroids, counts, lists) or None."""
    x = np.ascontiguousarray(vectors, np.float32)
    if x.ndim != 2:
        raise ValueError("vectors must be float32[n, dim]")
    n, d = x.shape
    if ann is not None:
        # the library reads k x dim centroids, k counts and n list entries
        c, cnt, lst = ann
        c, cnt, lst = np.asarray(c), np.asarray(cnt), np.asarray(lst)
        if c.ndim != 2 or c.shape[1] != d or cnt.size != c.shape[0] or lst.size != n:
            raise ValueError(f"ann must be (centroids[k, {d}], counts[k], lists[{n}])")
    _lib.init()
    if ann is None:
        _lib.check(_lib.lib().ec_index_load(_lib.ptr(x, C.c_float), n, d, None, 0, None, None),
                   "index_load")
        _state.update(ivf=False, dim=d)
        return
    cent, counts, lists = ann
    cent = np.ascontiguousarray(cent, np.float32)
    counts = np.ascontiguousarray(counts, np.uint32)
    lists = np.ascontiguousarray(lists, np.uint32)
    _lib.check(_lib.lib().ec_index_load(_lib.ptr(x, C.c_float), n, d, _lib.ptr(cent, C.c_float),
                                        cent.shape[0], _lib.ptr(counts, C.c_uint32),
                                        _lib.ptr(lists, C.c_uint32)), "index_load")
    _state.update(ivf=True, dim=d)


def load_index_files(index_path, dim, ann_path=None):
    """index.bin (rows of `dim` f32) and optionally ann.bin straight from the
    files into device memory (kb::load-index + kb::load-ann, kb.lisp:84-129,
    283-314, with the dimension passed in).  Returns n."""
    _lib.init()
    n = C.c_int64()
    _lib.check(_lib.lib().ec_index_load_files(str(index_path).encode(), dim,
                                              str(ann_path).encode() if ann_path else None,
                                              C.byref(n)), "index_load_files")
    _state.update(ivf=ann_path is not None, dim=dim)
    return n.value


def _queries(q):
    """float32[nq, dim] queries of the loaded index's width (the library
    reads nq x dim floats and cannot see the array's own width)."""
    q = np.ascontiguousarray(np.atleast_2d(q), np.float32)
    if q.ndim != 2 or (_state["dim"] and q.shape[1] != _state["dim"]):
        raise ValueError(f"queries of shape {q.shape}, the index has dim {_state['dim']}")
    return q


def search_ivf(q, k, nprobe=None):
    q = _queries(q)
    nq = q.shape[0]
    ids = np.empty((nq, k), np.int64)
    sc = np.empty((nq, k), np.float32)
    _lib.check(_lib.lib().ec_ivf_search(_lib.ptr(q, C.c_float), nq, nprobe or ann_nprobe, k,
                                        _lib.ptr(ids, C.c_int64), _lib.ptr(sc, C.c_float)),
               "ivf_search")
    return ids, sc


def search_brute(q, k):
    q = _queries(q)
    nq = q.shape[0]
    ids = np.empty((nq, k), np.int64)
    sc = np.empty((nq, k), np.float32)
    _lib.check(_lib.lib().ec_flat_search(_lib.ptr(q, C.c_float), nq, k, _lib.ptr(ids, C.c_int64),
                                         _lib.ptr(sc, C.c_float)), "flat_search")
    return ids, sc


def _pairs(ids, sc):
    return [(int(i), float(s)) for i, s in zip(ids, sc) if i >= 0]


def top_k_ivf(q, k):
    ids, sc = search_ivf(q, k)
    return _pairs(ids[0], sc[0])


def top_k_brute(q, k):
    ids, sc = search_brute(q, k)
    return _pairs(ids[0], sc[0])


def top_k(q, k):
    """kb::top-k: IVF when an IVF index is loaded, else brute force."""
    return top_k_ivf(q, k) if _state["ivf"] else top_k_brute(q, k)
