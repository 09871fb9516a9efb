"""ctypes binding of libembedcuda.so (include/embedcuda.h).

Loads the in-tree library next to this package and fails loudly when it is
missing or cannot be built: there is no CPU fallback behind this module.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                      # lisp-embed_b200/
REPO = os.path.dirname(ROOT)
LIB_PATH = os.path.join(ROOT, "libembedcuda.so")
HEADER = os.path.join(REPO, "include", "embedcuda.h")

EC_OK, EC_EINVAL, EC_ESTATE, EC_ECUDA, EC_ENOMEM, EC_ETIMEOUT, EC_ENCCL, EC_EUNSUPPORTED = \
    0, -1, -2, -3, -4, -5, -6, -7
EC_F32, EC_BF16, EC_F16 = 0, 1, 2
FAMILIES = {1: "bert", 2: "mpnet", 3: "llama", 4: "gemma"}

_lock = threading.Lock()
_lib = None


class EcError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def build(force: bool = False):
    """Compile libembedcuda.so for sm_100a with the in-tree Makefile."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-j8", "-C", ROOT], check=True)


P = C.c_void_p
I64P = C.POINTER(C.c_int64)
I32P = C.POINTER(C.c_int32)
U32P = C.POINTER(C.c_uint32)
FP = C.POINTER(C.c_float)

_SIGS = {
    "ec_last_error": (C.c_char_p, []),
    "ec_init": (C.c_int, [I32P, C.c_int]),
    "ec_device_count": (C.c_int, []),
    "ec_shutdown": (C.c_int, []),
    "ec_upload_tensor": (C.c_int, [C.c_char_p, C.c_int, I64P, C.c_int, P, C.c_size_t]),
    "ec_load_model": (C.c_int, [C.c_char_p, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "ec_dim": (C.c_int, []),
    "ec_embed_batch": (C.c_int, [I32P, I64P, C.c_int, FP, C.c_int]),
    "ec_embed_batch_device": (C.c_int, [P, I64P, C.c_int, P, C.c_int, P]),
    "ec_kmeans": (C.c_int, [FP, C.c_int64, C.c_int, I64P, C.c_int64, C.c_int, C.c_int, FP, FP]),
    "ec_assign_all": (C.c_int, [FP, C.c_int64, C.c_int, FP, C.c_int, U32P, U32P]),
    "ec_ann_build": (C.c_int, [FP, C.c_int64, C.c_int, I64P, C.c_int64, C.c_int, C.c_int, FP, FP,
                               U32P, U32P]),
    "ec_assign": (C.c_int, [FP, C.c_int64, C.c_int, I64P, C.c_int64, FP, C.c_int, I32P]),
    "ec_index_load": (C.c_int, [FP, C.c_int64, C.c_int, FP, C.c_int, U32P, U32P]),
    "ec_ivf_search": (C.c_int, [FP, C.c_int, C.c_int, C.c_int, I64P, FP]),
    "ec_flat_search": (C.c_int, [FP, C.c_int, C.c_int, I64P, FP]),
    "ec_flat_search_noalloc": (C.c_int, [P, C.c_int64, C.c_int, P, C.c_int, C.c_int, P, P, P]),
    "ec_ann_save": (C.c_int, [C.c_char_p, FP, C.c_int, C.c_int, C.c_int64, U32P, U32P]),
    "ec_ann_read": (C.c_int, [C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int), I64P, FP, U32P,
                              U32P]),
    "ec_index_load_files": (C.c_int, [C.c_char_p, C.c_int, C.c_char_p, I64P]),
    "ec_ann_build_file": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_int, I64P, C.c_int64,
                                    C.c_char_p]),
    "ec_embed_batch_to_file": (C.c_int, [I32P, I64P, C.c_int, C.c_char_p]),
    "ec_tokenizer_from_json": (C.c_int, [C.c_char_p, C.POINTER(C.c_int)]),
    "ec_tokenizer_wordpiece": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(C.c_int)]),
    "ec_tokenizer_bpe": (C.c_int, [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_char_p,
                                   C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "ec_tokenizer_unigram": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(C.c_int)]),
    "ec_tokenizer_free": (C.c_int, [C.c_int]),
    "ec_tokenizer_vocab_size": (C.c_int, [C.c_int]),
    "ec_tokenize": (C.c_int, [C.c_int, C.POINTER(C.c_char_p), I64P, C.c_int, I32P, C.c_int64,
                              I64P, C.c_int]),
    "ec_tokenizer_decode": (C.c_int, [C.c_int, I32P, C.c_int, C.c_char_p, C.c_int64, I64P]),
    "ec_comm_id_size": (C.c_int, []),
    "ec_comm_get_id": (C.c_int, [P]),
    "ec_comm_init": (C.c_int, [C.c_int, C.c_int, P]),
    "ecdbg_gemm": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, P, P, P, C.c_int, C.c_int]),
    "ecdbg_mlp": (C.c_int, [P, P, P, P, P, P, P, P, P, P, C.c_int, C.c_int, C.c_int]),
    "ecdbg_gemm_ln": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, P, P, P, P, P, P]),
    "ecdbg_gemm_norm": (C.c_int, [P, P, C.c_int, C.c_int, C.c_int, P, P, P, P, P, C.c_int,
                                  C.c_float, C.c_float, C.c_int]),
    "ecdbg_profile": (C.c_int, [C.c_int]),
    "ecdbg_profile_read": (C.c_int, [C.c_char_p, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                     C.POINTER(C.c_double), C.POINTER(C.c_longlong)]),
    "ecdbg_launches": (C.c_longlong, []),
    "ecdbg_assign_rows": (C.c_int, [C.POINTER(C.c_longlong), C.POINTER(C.c_longlong), C.c_int]),
    "ecdbg_wait_timeout": (C.c_int, [C.c_int]),
    "ecdbg_kernel_arch": (C.c_int, [C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "ecdbg_tensor_read": (C.c_int, [C.c_char_p, P, C.c_size_t, C.POINTER(C.c_int)]),
    "ecdbg_attention": (C.c_int, [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P, I32P, C.c_int,
                                  C.c_int, C.c_int, C.c_int, C.c_int]),
}


def lib():
    """The loaded library (built on first use if absent)."""
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    return (lib().ec_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str = ""):
    if rc < 0:
        raise EcError(rc, f"{what}: {last_error()}" if what else last_error())
    return rc


def header_symbols(path: str = HEADER):
    """Function names declared in a public header."""
    with open(path) as f:
        src = f.read()
    return sorted(set(re.findall(r"\b(ec[a-z]*_[a-z0-9_]+)\s*\(", src)))


_inited = False


def init(devices=None):
    """ec_init once per process (devices: list of CUDA ordinals or None)."""
    global _inited
    if _inited:
        return
    if devices:
        arr = (C.c_int32 * len(devices))(*devices)
        check(lib().ec_init(arr, len(devices)), "ec_init")
    else:
        check(lib().ec_init(None, 0), "ec_init")
    _inited = True


def shutdown():
    global _inited
    if _inited:
        check(lib().ec_shutdown(), "ec_shutdown")
    _inited = False


def ptr(a, ctype):
    return a.ctypes.data_as(C.POINTER(ctype))
