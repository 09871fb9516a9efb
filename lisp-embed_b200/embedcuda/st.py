"""Safetensors upload -- the st.lisp mirror (st.lisp:7-94).

``parse_header`` reads the 8-byte little-endian header length and the JSON
header like st:parse-header; ``upload`` hands every tensor's raw bytes and
dtype to ec_upload_tensor, which keeps F32 bit-exact and widens BF16 / F16 on
the device with st:get-tensor's rules (no host widening).
"""
from __future__ import annotations

import ctypes as C
import json

import numpy as np

from . import _lib

_DT = {"F32": _lib.EC_F32, "BF16": _lib.EC_BF16, "F16": _lib.EC_F16}


def parse_header(path):
    """(header dict, data-start offset), as st:parse-header."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
    return header, 8 + n


def tensor_names(header):
    return [k for k in header if k != "__metadata__"]


def upload(path):
    """Upload every tensor of a .safetensors file; returns the names."""
    header, start = parse_header(path)
    L = _lib.lib()
    names = tensor_names(header)
    with open(path, "rb") as f:
        for name in names:
            info = header[name]
            dt = info["dtype"]
            if dt not in _DT:
                raise _lib.EcError(_lib.EC_EINVAL, f"tensor {name} has unsupported dtype {dt}")
            s, e = info["data_offsets"]
            f.seek(start + s)
            raw = np.frombuffer(f.read(e - s), np.uint8)
            if raw.size != e - s:
                raise _lib.EcError(_lib.EC_EINVAL, f"EOF in tensor {name}")
            shape = np.asarray(info["shape"], np.int64)
            _lib.check(L.ec_upload_tensor(name.encode(), _DT[dt],
                                          shape.ctypes.data_as(C.POINTER(C.c_int64)),
                                          int(shape.size), raw.ctypes.data, int(raw.size)),
                       f"upload {name}")
    return names
