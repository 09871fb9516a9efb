"""Embedding-model facade -- the model.lisp mirror (model.lisp:6-65).

``load_model(path)`` reads config.json (and 1_Pooling/config.json), uploads
model.safetensors and lets the library dispatch on model_type exactly as
model:load-model does; ``embed`` / ``embed_batch`` replace model:embed for
token-id sequences; ``dim``, ``family`` and ``path`` mirror their namesakes.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib, st

_state = {"family": None, "path": None, "dim": 0}


def load_model(path, devices=None):
    """Load any supported model directory; returns the family keyword
    ('bert' | 'mpnet' | 'llama' | 'gemma')."""
    _lib.init(devices)
    d = path if os.path.isdir(path) else os.path.dirname(path)
    with open(os.path.join(d, "config.json")) as f:
        cfg = f.read()
    pool = None
    pp = os.path.join(d, "1_Pooling", "config.json")
    if os.path.exists(pp):
        with open(pp) as f:
            pool = f.read()
    st_path = path if path.endswith(".safetensors") else os.path.join(d, "model.safetensors")
    st.upload(st_path)
    fam = C.c_int(0)
    dim_ = C.c_int(0)
    _lib.check(_lib.lib().ec_load_model(cfg.encode(), pool.encode() if pool else None,
                                        C.byref(fam), C.byref(dim_)), "load_model")
    _state.update(family=_lib.FAMILIES[fam.value], path=path, dim=dim_.value)
    return _state["family"]


def dim():
    return _lib.check(_lib.lib().ec_dim(), "dim")


def family():
    return _state["family"]


def path():
    return _state["path"]


def embed_batch(ids, offsets, out=None):
    """Embed packed sequences: ids int32[total], offsets int64[nseq + 1].
    Returns float32[nseq, dim], L2-normalised, in input order."""
    ids = np.ascontiguousarray(ids, np.int32)
    offsets = np.ascontiguousarray(offsets, np.int64)
    # the library reads ids[offsets[0] .. offsets[nseq]) and cannot see the
    # length of ids, nor of out
    if offsets.ndim != 1 or offsets.size < 1:
        raise ValueError("offsets must be int64[nseq + 1]")
    if offsets.size > 1 and (offsets[0] < 0 or offsets[-1] > ids.size or
                             bool(np.any(offsets[1:] < offsets[:-1]))):
        raise ValueError(f"offsets must be non-decreasing within [0, {ids.size}]")
    nseq = offsets.size - 1
    D = dim()
    if out is None:
        out = np.empty((nseq, D), np.float32)
    elif (not isinstance(out, np.ndarray) or out.dtype != np.float32 or out.ndim != 2 or
          not out.flags.c_contiguous or not out.flags.writeable or out.shape[0] < nseq or
          out.shape[1] < D):
        raise ValueError(f"out must be a writeable C-contiguous float32[>= {nseq}, >= {D}] array")
    _lib.check(_lib.lib().ec_embed_batch(_lib.ptr(ids, C.c_int32), _lib.ptr(offsets, C.c_int64),
                                         nseq, _lib.ptr(out, C.c_float), out.shape[1]),
               "embed_batch")
    return out


def embed(ids):
    """One sequence of token ids -> float32[dim] (model:embed)."""
    ids = np.ascontiguousarray(ids, np.int32)
    return embed_batch(ids, np.array([0, ids.size], np.int64))[0]


def embed_batch_device(d_ids_ptr, offsets, nseq, d_out_ptr, out_stride, stream=None):
    """Device-resident variant: ids / out are device pointers (ints); the
    work runs on `stream` (a cudaStream_t as int, None = library stream)."""
    offsets = np.ascontiguousarray(offsets, np.int64)
    _lib.check(_lib.lib().ec_embed_batch_device(C.c_void_p(d_ids_ptr), _lib.ptr(offsets, C.c_int64),
                                                nseq, C.c_void_p(d_out_ptr), out_stride,
                                                C.c_void_p(stream) if stream else None),
               "embed_batch_device")


def embed_batch_to_file(ids, offsets, index_path):
    """embed_batch, then the rows appended to index.bin as embed:run writes
    them (embed.lisp:47-57, 99-101)."""
    ids = np.ascontiguousarray(ids, np.int32)
    offsets = np.ascontiguousarray(offsets, np.int64)
    _lib.check(_lib.lib().ec_embed_batch_to_file(ids.ctypes.data_as(C.POINTER(C.c_int32)),
                                                 offsets.ctypes.data_as(C.POINTER(C.c_int64)),
                                                 offsets.size - 1, str(index_path).encode()),
               "embed_batch_to_file")
