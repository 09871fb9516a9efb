"""The C ABI without a GPU: the library builds, loads and exports every
symbol its public headers declare; calls fail cleanly (status + message)
when no device is present."""
import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import gpu_available
from embedcuda import _lib

REPO = _lib.REPO


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _lib.header_symbols(os.path.join(REPO, "include", "embedcuda.h"))
    declared += _lib.header_symbols(os.path.join(REPO, "include", "embedcuda_debug.h"))
    assert "ec_embed_batch" in declared and "ec_kmeans" in declared
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(lib, s)


def test_build_targets_sm100a_only():
    """The library's build compiles device code for sm_100a alone (the
    Makefile's one -gencode pair); the GPU test below checks what the
    runtime loaded."""
    with open(os.path.join(REPO, "lisp-embed_b200", "Makefile")) as f:
        mk = f.read()
    gencodes = re.findall(r"-gencode\s+(\S+)", mk)
    assert gencodes == ["arch=compute_100a,code=sm_100a"], gencodes


@pytest.mark.gpu
def test_loaded_device_code_is_sm100(ec):
    ver, ptx = C.c_int(), C.c_int()
    assert ec.lib().ecdbg_kernel_arch(C.byref(ver), C.byref(ptx)) == 0, ec.last_error()
    assert ver.value == 100, ver.value  # the cubin the runtime picked is sm_100


@pytest.mark.skipif(gpu_available(), reason="checks the no-device path")
def test_calls_fail_cleanly_without_device():
    lib = _lib.lib()
    rc = lib.ec_init(None, 0)
    assert rc in (_lib.EC_ECUDA, _lib.EC_EUNSUPPORTED)
    assert _lib.last_error()
    # everything else reports "ec_init first"
    assert lib.ec_dim() == _lib.EC_ESTATE
    assert lib.ec_embed_batch(None, None, 0, None, 0) == _lib.EC_ESTATE
    assert "ec_init" in _lib.last_error()
    shape = (C.c_int64 * 1)(4)
    assert lib.ec_upload_tensor(b"x", _lib.EC_F32, shape, 1, None, 16) == _lib.EC_ESTATE
    # the IVF entry points check the context before their arguments
    assert lib.ec_kmeans(None, 0, 8, None, 0, 4, 1, None, None) == _lib.EC_ESTATE
    assert lib.ec_assign_all(None, 0, 8, None, 4, None, None) == _lib.EC_ESTATE
    assert lib.ec_ann_build(None, 0, 8, None, 0, 4, 1, None, None, None, None) == _lib.EC_ESTATE
    assert "ec_init" in _lib.last_error()
    assert lib.ec_comm_id_size() == 128


def test_header_declares_status_codes():
    with open(os.path.join(REPO, "include", "embedcuda.h")) as f:
        src = f.read()
    for name, val in [("EC_OK", 0), ("EC_EINVAL", -1), ("EC_ESTATE", -2), ("EC_ECUDA", -3),
                      ("EC_ENOMEM", -4), ("EC_ETIMEOUT", -5), ("EC_ENCCL", -6),
                      ("EC_EUNSUPPORTED", -7)]:
        assert f"#define {name} " in src
        assert getattr(_lib, name) == val
