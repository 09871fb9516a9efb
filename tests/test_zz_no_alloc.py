"""ec_flat_search_noalloc: flat search over caller-owned device buffers with
its candidate scratch in the library's static device array.  Results must
equal ec_flat_search (kb::top-k-brute, kb.lisp:186-200) on the same vectors
and queries -- ids exactly, scores exactly (tolerance 0: both run the same
scan and merge kernels) -- on two calls in a row, which share the scratch,
and the oracle's restatement of kb::top-k-brute on a subset of the queries
(also exact: the scan keeps the reference's sequential single-float sums).
The file name sorts last so it also runs after every other GPU test."""
import ctypes as C

import numpy as np
import pytest

from embedcuda import _lib
from oracle import oracle

SCRATCH_BYTES = 16 << 20


def _call(lib, x_ptr, n, d, q_ptr, nq, topk, ids_ptr, sc_ptr, stream=None):
    return lib.ec_flat_search_noalloc(C.c_void_p(x_ptr), C.c_int64(n), d, C.c_void_p(q_ptr), nq, topk,
                                      C.c_void_p(ids_ptr), C.c_void_p(sc_ptr), C.c_void_p(stream))


def _check_against_flat_search(ec, x, q, topk):
    import torch
    from embedcuda import kb
    n, d = x.shape
    nq = q.shape[0]
    kb.load_index(x)
    ref_ids, ref_sc = kb.search_brute(q, topk)
    dx = torch.from_numpy(x).cuda()
    dq = torch.from_numpy(q).cuda()
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row share the scratch
        ids = torch.full((nq, topk), -7, dtype=torch.int64, device="cuda")
        sc = torch.full((nq, topk), float("nan"), dtype=torch.float32, device="cuda")
        rc = _call(ec.lib(), dx.data_ptr(), n, d, dq.data_ptr(), nq, topk, ids.data_ptr(), sc.data_ptr(), st)
        assert rc == 0, ec.last_error()
        torch.cuda.synchronize()
        got_ids, got_sc = ids.cpu().numpy(), sc.cpu().numpy()
        assert np.array_equal(got_ids, ref_ids)
        np.testing.assert_allclose(got_sc, ref_sc, rtol=0, atol=0)
    for i in range(0, nq, max(1, nq // 16)):
        o_ids, o_sc = oracle.top_k_brute(x, q[i], topk)
        r = len(o_ids)
        assert np.array_equal(got_ids[i, :r], o_ids), i
        assert np.array_equal(got_sc[i, :r], o_sc), i
        assert np.all(got_ids[i, r:] == -1)


@pytest.mark.gpu
def test_noalloc_matches_flat_search(ec):
    rng = np.random.default_rng(21)
    x = rng.standard_normal((50000, 384)).astype(np.float32)
    q = rng.standard_normal((300, 384)).astype(np.float32)
    _check_against_flat_search(ec, x, q, 10)


@pytest.mark.gpu
def test_noalloc_ragged_and_fewer_rows_than_topk(ec):
    rng = np.random.default_rng(22)
    x = rng.standard_normal((5, 64)).astype(np.float32)
    q = rng.standard_normal((7, 64)).astype(np.float32)
    _check_against_flat_search(ec, x, q, 10)  # slots past n hold id -1
    x = rng.standard_normal((8193 * 3 + 17, 32)).astype(np.float32)
    x[100] = x[9000]  # a tied pair: lower row id first
    q = rng.standard_normal((33, 32)).astype(np.float32)
    _check_against_flat_search(ec, x, q, 64)


@pytest.mark.gpu
def test_noalloc_at_scratch_limit(ec):
    # 256 chunks x topk 64 x 8 bytes = 128 KiB per query: 128 queries fill the scratch exactly
    rng = np.random.default_rng(23)
    x = rng.standard_normal((256 * 8192, 4)).astype(np.float32)
    q = rng.standard_normal((SCRATCH_BYTES // (256 * 64 * 8), 4)).astype(np.float32)
    _check_against_flat_search(ec, x, q, 64)


def test_noalloc_rejects_oversize_without_launching():
    lib = _lib.lib()
    fake = 4096  # never dereferenced: every case below is rejected before any launch
    # 129 queries x 256 chunks x 64 x 8 bytes is one query past the scratch
    assert _call(lib, fake, 256 * 8192, 4, fake, 129, 64, fake, fake) == _lib.EC_EINVAL
    assert "static scratch" in _lib.last_error() and "at most 128 queries" in _lib.last_error()
    assert _call(lib, fake, 1000, 4, fake, 1, 65, fake, fake) == _lib.EC_EINVAL
    assert _call(lib, fake, 1000, 6, fake, 1, 5, fake, fake) == _lib.EC_EINVAL
    assert _call(lib, fake, 1 << 31, 4, fake, 1, 5, fake, fake) == _lib.EC_EINVAL
    assert _call(lib, fake, 1000, 4, fake, 70000, 1, fake, fake) == _lib.EC_EINVAL
    assert _call(lib, 0, 1000, 4, fake, 1, 5, fake, fake) == _lib.EC_EINVAL
    assert _call(lib, fake, 1000, 4, fake, 0, 5, fake, fake) == _lib.EC_OK  # nothing to do
