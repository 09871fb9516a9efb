"""Multi-rank host logic on CPU (gloo, world size 2 to 4).

ec_kmeans shards the training sample into contiguous ranges, one per rank.
Its default exchange passes the per-cluster accumulators down the ranks in
sample order (rank r continues rank r-1's sums with its own rows; the last
rank divides and broadcasts the centroids; NCCL send / recv / broadcast on
the GPUs): here gloo ranks run that decomposition with the oracle's
arithmetic and must reproduce the single-process Lloyd iterations bit for
bit.  The all-reduce exchange (EC_KMEANS_ALLREDUCE) sums per-rank partial
sums instead: centroids within float32 summation-order noise, assignments
identical except near-ties.  A third test kills one rank between steps and
checks that the survivor's next collective fails with an error instead of
hanging (host-side failure detection).
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _split(n, parts, k):
    per = (n + parts - 1) // parts
    return min(n, per * k), min(n, per * (k + 1))


def _kmeans_chain_rank(rank, world, port, x, sample, k, iters, out):
    import sys
    sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                 "lisp-embed_b200")]
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    d = x.shape[1]
    cent = x[sample[:k]].copy()
    j0, j1 = _split(len(sample), world, rank)
    mine = sample[j0:j1]
    for _ in range(iters):
        a = oracle.assign(x, cent, rows=mine)
        # the accumulators of ranks 0..rank-1, continued in sample order
        buf = np.zeros((k, d + 1), np.float32)
        if rank > 0:
            t = torch.zeros(k, d + 1)
            dist.recv(t, src=rank - 1)
            buf = t.numpy().copy()
        for j, r in enumerate(mine):
            c = a[j]
            buf[c, :d] = (buf[c, :d] + x[r]).astype(np.float32)
            buf[c, d] += 1
        t_cent = torch.from_numpy(cent.copy())
        if rank + 1 < world:
            dist.send(torch.from_numpy(buf), dst=rank + 1)
        else:
            nz = buf[:, d] > 0
            cent[nz] = buf[nz, :d] / buf[nz, d:d + 1]
            t_cent = torch.from_numpy(cent.copy())
        dist.broadcast(t_cent, src=world - 1)
        cent = t_cent.numpy().copy()
    if rank == 0:
        np.save(out, cent)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4])
def test_chained_lloyd_is_bit_identical(tmp_path, world):
    from embedcuda import synth
    from oracle import oracle
    x, _ = synth.make_ivf_corpus(3000, 32, 16, seed=4, sigma=0.2)
    sample = synth.make_ivf_sample(len(x), 4)
    k, iters = 16, 3
    out = str(tmp_path / "cent.npy")
    mp.start_processes(_kmeans_chain_rank, args=(world, _free_port(), x, sample, k, iters, out),
                       nprocs=world, join=True, start_method="spawn")
    assert np.array_equal(np.load(out), oracle.kmeans(x, sample, k, iters))


def _kmeans_rank(rank, world, port, x, sample, k, iters, out):
    import sys
    sys.path[:0] = [os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                    os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                 "lisp-embed_b200")]
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    d = x.shape[1]
    cent = x[sample[:k]].copy()
    j0, j1 = _split(len(sample), world, rank)
    mine = sample[j0:j1]
    for _ in range(iters):
        a = oracle.assign(x, cent, rows=mine)
        buf = np.zeros((k, d + 1), np.float32)
        for c in range(k):
            m = mine[a == c]
            s = np.zeros(d, np.float32)
            for r in m:
                s = (s + x[r]).astype(np.float32)
            buf[c, :d] = s
            buf[c, d] = len(m)
        t = torch.from_numpy(buf)
        dist.all_reduce(t)
        buf = t.numpy()
        nz = buf[:, d] > 0
        cent[nz] = buf[nz, :d] / buf[nz, d:d + 1]
    if rank == 0:
        np.save(out, cent)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_lloyd_matches_single_process(tmp_path):
    from embedcuda import synth
    from oracle import oracle
    x, _ = synth.make_ivf_corpus(3000, 32, 16, seed=4, sigma=0.2)
    sample = synth.make_ivf_sample(len(x), 4)
    k, iters = 16, 3
    out = str(tmp_path / "cent.npy")
    mp.start_processes(_kmeans_rank, args=(2, _free_port(), x, sample, k, iters, out), nprocs=2,
                       join=True, start_method="spawn")
    got = np.load(out)
    ref = oracle.kmeans(x, sample, k, iters)
    assert np.allclose(got, ref, rtol=1e-5, atol=1e-6)
    # assignments with the all-reduced centroids equal the single-process
    # ones except where two centroids tie within 1e-5 relative
    a_got = oracle.assign(x, got)
    a_ref = oracle.assign(x, ref)
    diff = np.nonzero(a_got != a_ref)[0]
    for i in diff:
        s1 = float(x[i] @ ref[a_ref[i]])
        s2 = float(x[i] @ ref[a_got[i]])
        assert abs(s1 - s2) <= 1e-5 * max(abs(s1), 1e-12)


def _dying_rank(rank, world, port, flag):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)  # step 1: both ranks
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        dist.all_reduce(t)  # step 2: the peer is gone
        ok = False
    except Exception:
        ok = True
    with open(flag, "w") as f:
        f.write("error" if ok else "no-error")
    os._exit(0)


def test_dead_rank_fails_next_collective(tmp_path):
    flag = str(tmp_path / "flag")
    ctx = mp.get_context("spawn")
    port = _free_port()
    ps = [ctx.Process(target=_dying_rank, args=(r, 2, port, flag)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("rank did not finish")
    with open(flag) as f:
        assert f.read() == "error"
