"""Failure detection without faulting a GPU: every failure is made on the
host (bad input, allocation cap, NCCL made unavailable) or by a bounded
device wait that is allowed to run out; the library reports a status code
and stays usable."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import REPO, gpu_available
from embedcuda import _lib

CHILD = r"""
import sys, os, json
sys.path[:0] = [{repo!r}, os.path.join({repo!r}, "lisp-embed_b200")]
from embedcuda import _lib, model, synth
res = {{}}
try:
    _lib.init([0])
    d = synth.build_model_dir(synth.MINILM, 0, {root!r})
    model.load_model(d)
    res["load"] = "ok"
except _lib.EcError as e:
    res["load"] = e.code
print(json.dumps(res))
"""


def test_nccl_unavailable_is_reported(monkeypatch):
    code = ("import sys, os; sys.path[:0]=[%r, os.path.join(%r,'lisp-embed_b200')];"
            "from embedcuda import _lib; import ctypes as C; b=C.create_string_buffer(128);"
            "print(_lib.lib().ec_comm_get_id(b), _lib.last_error())") % (REPO, REPO)
    env = dict(os.environ, EC_FAKE_NCCL_FAIL="1")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=120)
    rc, msg = out.stdout.strip().split(" ", 1)
    assert int(rc) == _lib.EC_ENCCL and "NCCL" in msg


@pytest.mark.gpu
def test_allocation_cap_gives_enomem(synth_root):
    if not gpu_available():
        pytest.skip("no GPU")
    env = dict(os.environ, EC_MAX_BYTES="32M")
    out = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO, root=synth_root)],
                         env=env, capture_output=True, text=True, timeout=300)
    assert '"load": %d' % _lib.EC_ENOMEM in out.stdout, out.stdout + out.stderr


@pytest.mark.gpu
def test_bounded_wait_times_out_and_context_survives(ec):
    rc = ec.lib().ecdbg_wait_timeout(50)
    assert rc == ec.EC_ETIMEOUT, (rc, ec.last_error())
    assert "timed out" in ec.last_error()
    # the context is still usable afterwards
    import torch
    A = torch.randn(256, 384, device="cuda").bfloat16()
    W = torch.randn(384, 384, device="cuda").bfloat16()
    out = torch.empty(256, 384, device="cuda")
    torch.cuda.synchronize()
    assert ec.lib().ecdbg_gemm(A.data_ptr(), W.data_ptr(), 256, 384, 384, None, None,
                               out.data_ptr(), 4, 0) == 0
    assert torch.allclose(out, A.float() @ W.float().t(), rtol=1e-3, atol=1e-2)


@pytest.mark.gpu
def test_bad_inputs_rejected(ec):
    from embedcuda import ann, kb
    x = np.ones((10, 6), np.float32)  # dim not a multiple of 4
    with pytest.raises(_lib.EcError) as e:
        ann.assign(x, x[:2])
    assert e.value.code == _lib.EC_EINVAL
    with pytest.raises(_lib.EcError):
        ann.kmeans(np.ones((10, 8), np.float32), np.arange(3), 5, 1)  # sample < k
    with pytest.raises(_lib.EcError):
        kb.load_index(np.ones((4, 8), np.float32),
                      (np.ones((2, 8), np.float32), np.array([1, 1], np.uint32),
                       np.array([0, 1, 2, 3], np.uint32)))  # counts do not sum to n
