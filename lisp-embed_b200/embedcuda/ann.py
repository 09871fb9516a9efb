"""IVF index build -- the ann.lisp mirror (ann.lisp:1-200).

``kmeans`` (ann::kmeans), ``assign_all`` (ann::assign-all), ``build`` (both
in one call), ``save_ann`` / ``load_ann`` (the ann.bin format of
ann.lisp:4-6, 165-187), ``run`` and ``build_file`` (ann:run from index.bin
to ann.bin in the library).
The arithmetic runs in libembedcuda.so; ``sample`` is the explicit list of
training rows whose first k rows initialise the centroids (ann.lisp:83-86).
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from . import _lib

MAGIC = 0x414E4E31  # "ANN1"


def _init_rows(init, k, d):
    """The library reads k x dim initial centroids."""
    init = np.ascontiguousarray(init, np.float32)
    if init.shape != (k, d):
        raise ValueError(f"init of shape {init.shape}, need ({k}, {d})")
    return init


def _check_centroids(centroids, d):
    """The library reads k x dim centroids, dim taken from the vectors."""
    if centroids.ndim != 2 or centroids.shape[1] != d:
        raise ValueError(f"centroids of shape {centroids.shape}, need (k, {d})")


def kmeans(vecs, sample, k, iters, init=None):
    """Train k centroids on vecs[sample] (float32[k, dim])."""
    vecs = np.ascontiguousarray(vecs, np.float32)
    sample = np.ascontiguousarray(sample, np.int64)
    n, d = vecs.shape
    cent = np.empty((k, d), np.float32)
    init_p = None
    if init is not None:
        init = _init_rows(init, k, d)
        init_p = _lib.ptr(init, C.c_float)
    _lib.check(_lib.lib().ec_kmeans(_lib.ptr(vecs, C.c_float), n, d, _lib.ptr(sample, C.c_int64),
                                    sample.size, k, iters, init_p, _lib.ptr(cent, C.c_float)),
               "kmeans")
    return cent


def assign(vecs, centroids, rows=None):
    """Nearest centroid (argmax inner product, ties -> lowest index)."""
    vecs = np.ascontiguousarray(vecs, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    n, d = vecs.shape
    _check_centroids(centroids, d)
    k = centroids.shape[0]
    rp = None
    m = n
    if rows is not None:
        rows = np.ascontiguousarray(rows, np.int64)
        rp = _lib.ptr(rows, C.c_int64)
        m = rows.size
    out = np.empty(m, np.int32)
    _lib.check(_lib.lib().ec_assign(_lib.ptr(vecs, C.c_float), n, d, rp, m,
                                    _lib.ptr(centroids, C.c_float), k, _lib.ptr(out, C.c_int32)),
               "assign")
    return out


def assign_all(vecs, centroids):
    """(counts uint32[k], lists uint32[n]) with ascending row ids per list."""
    vecs = np.ascontiguousarray(vecs, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    n, d = vecs.shape
    _check_centroids(centroids, d)
    k = centroids.shape[0]
    counts = np.empty(k, np.uint32)
    lists = np.empty(n, np.uint32)
    _lib.check(_lib.lib().ec_assign_all(_lib.ptr(vecs, C.c_float), n, d,
                                        _lib.ptr(centroids, C.c_float), k,
                                        _lib.ptr(counts, C.c_uint32), _lib.ptr(lists, C.c_uint32)),
               "assign_all")
    return counts, lists


def build(vecs, sample, k, iters, init=None):
    """kmeans(vecs, sample, k, iters, init) then assign_all with its
    centroids, in one library call (ec_ann_build: on one device the rows
    cross to it once).  Returns (centroids, counts, lists)."""
    vecs = np.ascontiguousarray(vecs, np.float32)
    sample = np.ascontiguousarray(sample, np.int64)
    n, d = vecs.shape
    cent = np.empty((k, d), np.float32)
    counts = np.empty(k, np.uint32)
    lists = np.empty(n, np.uint32)
    init_p = None
    if init is not None:
        init = _init_rows(init, k, d)
        init_p = _lib.ptr(init, C.c_float)
    _lib.check(_lib.lib().ec_ann_build(_lib.ptr(vecs, C.c_float), n, d, _lib.ptr(sample, C.c_int64),
                                       sample.size, k, iters, init_p, _lib.ptr(cent, C.c_float),
                                       _lib.ptr(counts, C.c_uint32), _lib.ptr(lists, C.c_uint32)),
               "ann_build")
    return cent, counts, lists


def save_ann(path, centroids, counts, lists, n):
    """ann.bin: u32 magic, k, dim, n; k*dim f32; k u32 counts; n u32 ids
    (ann::save-ann, ann.lisp:165-187), written by ec_ann_save."""
    cent = np.ascontiguousarray(centroids, np.float32)
    counts = np.ascontiguousarray(counts, np.uint32)
    lists = np.ascontiguousarray(lists, np.uint32)
    k, d = cent.shape
    _lib.check(_lib.lib().ec_ann_save(str(path).encode(), _lib.ptr(cent, C.c_float), k, d, n,
                                      _lib.ptr(counts, C.c_uint32), _lib.ptr(lists, C.c_uint32)),
               "ann_save")


def load_ann(path):
    """(centroids, counts, lists) from ann.bin, or None when the magic differs
    (kb::load-ann, kb.lisp:283-314), read by ec_ann_read."""
    with open(path, "rb") as f:
        head = f.read(4)
    if len(head) < 4 or struct.unpack("<I", head)[0] != MAGIC:
        return None
    k, d, n = C.c_int(), C.c_int(), C.c_int64()
    L = _lib.lib()
    _lib.check(L.ec_ann_read(str(path).encode(), C.byref(k), C.byref(d), C.byref(n), None, None,
                             None), "ann_read")
    cent = np.empty((k.value, d.value), np.float32)
    counts = np.empty(k.value, np.uint32)
    lists = np.empty(n.value, np.uint32)
    _lib.check(L.ec_ann_read(str(path).encode(), C.byref(k), C.byref(d), C.byref(n),
                             _lib.ptr(cent, C.c_float), _lib.ptr(counts, C.c_uint32),
                             _lib.ptr(lists, C.c_uint32)), "ann_read")
    return cent, counts, lists


def build_file(index_path, dim, k, iters, sample, ann_path):
    """ann:run from index.bin to ann.bin inside the library (the vectors are
    read from a mapping of index.bin, never copied into a host array)."""
    sample = np.ascontiguousarray(sample, np.int64)
    _lib.check(_lib.lib().ec_ann_build_file(str(index_path).encode(), dim, k, iters,
                                            _lib.ptr(sample, C.c_int64), sample.size,
                                            str(ann_path).encode()), "ann_build_file")


def run(vecs, k=1024, iters=10, sample=None, seed=None, out_path=None):
    """ann:run: k-means on a sample, then assign every row (ann.lisp:189-200).
    The reference draws the sample with the global random state; here it is
    explicit (or drawn from `seed`)."""
    vecs = np.ascontiguousarray(vecs, np.float32)
    n = vecs.shape[0]
    if sample is None:
        rng = np.random.default_rng(seed)
        sample = rng.choice(n, size=min(100000, n), replace=False)
    cent, counts, lists = build(vecs, sample, k, iters)
    if out_path:
        save_ann(out_path, cent, counts, lists, n)
    return cent, counts, lists
