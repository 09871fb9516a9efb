"""Multi-GPU paths (run only when two or more GPUs are visible).

* The in-process multi-device split of ec_embed_batch gives the same
  embeddings as one device (no collective: per-sequence work).
* k-means over two devices is bit-identical to the oracle's serial Lloyd
  iterations (ann.lisp:79-125): the per-cluster sums pass from device 0 to
  device 1 in sample order (NCCL send / recv) and device 1 broadcasts the
  centroids.  The all-reduce exchange (EC_KMEANS_ALLREDUCE=1) agrees up to
  float32 summation order.  The same holds with one process per GPU
  (ec_comm_init, each rank passing its contiguous shard of the sample) and,
  with three or four GPUs visible, for the middle ranks of the chain (in
  process and one process per GPU).
* IVF / flat search with the queries split over the devices equals
  kb::top-k-ivf / top-k-brute.
* A device that fails before the first exchange (host-side injection,
  EC_FAKE_COMM_FAIL) makes the call fail at once on every device, no NCCL
  work is left waiting on it, and the next call rebuilds the communicators
  and succeeds.
Every child runs with NVLS off (NCCL_NVLS_ENABLE=0)."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

PRE = r"""
import sys, os, json
import numpy as np
sys.path[:0] = [{repo!r}, os.path.join({repo!r}, "lisp-embed_b200")]
from embedcuda import _lib, model, synth, ann, kb
from oracle import oracle
"""

CHILD = PRE + r"""
_lib.init([0, 1])
d = synth.build_model_dir(synth.with_layers(synth.MINILM, 2), 0, {root!r})
model.load_model(d)
ids, offs = synth.make_inputs("minilm", 256, 5)
two = model.embed_batch(ids, offs)
x, _ = synth.make_ivf_corpus(40000, 384, 64, seed=4)
sample = synth.make_ivf_sample(len(x), 4)
cent2 = ann.kmeans(x, sample, 64, 4)
os.environ["EC_KMEANS_ALLREDUCE"] = "1"
cent_ar = ann.kmeans(x, sample, 64, 4)
del os.environ["EC_KMEANS_ALLREDUCE"]
counts, lists = ann.assign_all(x, cent2)
rc, rl = oracle.assign_all(x, cent2)
np.save({out!r} + "_emb.npy", two)
np.save({out!r} + "_cent.npy", cent2)
np.save({out!r} + "_cent_ar.npy", cent_ar)
kb.load_index(x, (cent2, counts, lists))
qs, _ = synth.make_ivf_corpus(300, 384, 64, seed=21)
ids_, sc_ = kb.search_ivf(qs, 10, nprobe=8)
ivf_ok = True
for i in range(len(qs)):
    rid, rsc = oracle.top_k_ivf(x, cent2, counts, lists, 8, qs[i], 10)
    ivf_ok &= bool(np.array_equal(ids_[i][:len(rid)], rid) and np.array_equal(sc_[i][:len(rsc)], rsc))
kb.load_index(x, None)
fid, fsc = kb.search_brute(qs[:24], 10)
flat_ok = True
for i in range(24):
    rid, rsc = oracle.top_k_brute(x, qs[i], 10)
    flat_ok &= bool(np.array_equal(fid[i], rid) and np.array_equal(fsc[i], rsc))
print(json.dumps({{"lists_equal": bool(np.array_equal(counts, rc) and np.array_equal(lists, rl)),
                  "ivf_search_equal": ivf_ok, "flat_search_equal": flat_ok}}))
"""

FAIL_CHILD = PRE + r"""
_lib.init([0, 1])
x, _ = synth.make_ivf_corpus(20000, 384, 64, seed=4)
sample = synth.make_ivf_sample(len(x), 4)
res = {{}}
os.environ["EC_FAKE_COMM_FAIL"] = "1"
try:
    ann.kmeans(x, sample, 64, 2)
    res["first"] = "ok"
except _lib.EcError as e:
    res["first"] = e.code
    res["msg"] = str(e)
del os.environ["EC_FAKE_COMM_FAIL"]
cent = ann.kmeans(x, sample, 64, 2)
res["second_exact"] = bool(np.array_equal(cent, oracle.kmeans(x, sample, 64, 2)))
_lib.shutdown()
res["shutdown"] = "ok"
print(json.dumps(res))
"""

PROC_CHILD = PRE + r"""
import ctypes as C
import torch.distributed as tdist
from datetime import timedelta
rank, world = int(sys.argv[1]), {world}
store = tdist.TCPStore("127.0.0.1", {port}, world, rank == 0, timeout=timedelta(seconds=120))
_lib.init([rank])
L = _lib.lib()
n = L.ec_comm_id_size()
if rank == 0:
    b = C.create_string_buffer(n)
    _lib.check(L.ec_comm_get_id(b), "comm id")
    store.set("id", b.raw)
uid = C.create_string_buffer(store.get("id"), n)
_lib.check(L.ec_comm_init(rank, world, uid), "comm init")
x, _ = synth.make_ivf_corpus(40000, 384, 64, seed=4)
sample = synth.make_ivf_sample(len(x), 4)
per = (len(sample) + world - 1) // world
mine = sample[rank * per:min(len(sample), (rank + 1) * per)]
init = x[sample[:64]].copy()
cent = ann.kmeans(x, mine, 64, 4, init=init)
if rank == 0:
    np.save({out!r}, cent)
store.set("done%d" % rank, "1")
store.wait(["done%d" % r for r in range(world)])
_lib.shutdown()
print("rank", rank, "ok")
"""


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _env():
    return dict(os.environ, NCCL_NVLS_ENABLE="0", EC_COMM_TIMEOUT_S="60")


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_device_embed_and_kmeans(tmp_path, synth_root):
    out = str(tmp_path / "r")
    p = subprocess.run([sys.executable, "-c", CHILD.format(repo=REPO, root=synth_root, out=out)],
                       capture_output=True, text=True, timeout=900, env=_env())
    assert p.returncode == 0, p.stdout + p.stderr
    assert '"lists_equal": true' in p.stdout
    assert '"ivf_search_equal": true' in p.stdout and '"flat_search_equal": true' in p.stdout
    from embedcuda import _lib, model, synth
    from oracle import oracle
    _lib.init([0])
    d = synth.build_model_dir(synth.with_layers(synth.MINILM, 2), 0, synth_root)
    model.load_model(d)
    ids, offs = synth.make_inputs("minilm", 256, 5)
    one = model.embed_batch(ids, offs)
    two = np.load(out + "_emb.npy")
    assert np.array_equal(one, two)  # no collective: per-sequence results are identical
    x, _ = synth.make_ivf_corpus(40000, 384, 64, seed=4)
    sample = synth.make_ivf_sample(len(x), 4)
    ref = oracle.kmeans(x, sample, 64, 4)
    assert np.array_equal(np.load(out + "_cent.npy"), ref)  # chained sums: bit-identical
    assert np.allclose(np.load(out + "_cent_ar.npy"), ref, rtol=1e-5, atol=1e-6)


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_device_failure_before_exchange_then_recovery():
    p = subprocess.run([sys.executable, "-c", FAIL_CHILD.format(repo=REPO)],
                       capture_output=True, text=True, timeout=600, env=_env())
    assert p.returncode == 0, p.stdout + p.stderr
    import json
    res = json.loads(p.stdout.strip().splitlines()[-1])
    from embedcuda import _lib
    assert res["first"] == _lib.EC_ENCCL, res
    # the call reports the first device's error: the injected failure or the
    # other device's prompt "another rank failed"
    assert "injected" in res["msg"] or "another rank failed" in res["msg"], res
    assert res["second_exact"] and res["shutdown"] == "ok", res


@pytest.mark.skipif(_gpus() < 3, reason="needs three GPUs")
def test_in_process_kmeans_middle_devices_bit_identical():
    """Three or four devices in one process: the middle devices both receive
    the running sums and pass them on."""
    nd = min(_gpus(), 4)
    src = PRE.format(repo=REPO) + f"""
_lib.init(list(range({nd})))
x, _ = synth.make_ivf_corpus(40000, 384, 64, seed=4)
sample = synth.make_ivf_sample(len(x), 4)
cent = ann.kmeans(x, sample, 64, 4)
print(json.dumps({{"exact": bool(np.array_equal(cent, oracle.kmeans(x, sample, 64, 4)))}}))
"""
    p = subprocess.run([sys.executable, "-c", src], capture_output=True, text=True, timeout=600,
                       env=_env())
    assert p.returncode == 0, p.stdout + p.stderr
    assert '"exact": true' in p.stdout, p.stdout


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_process_kmeans_bit_identical(tmp_path):
    """One process per GPU on every visible GPU up to four (two ranks: the
    first and last; more: the middle ranks of the chain too)."""
    import socket
    world = min(_gpus(), 4)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = str(tmp_path / "cent.npy")
    src = PROC_CHILD.format(repo=REPO, port=port, out=out, world=world)
    ps = [subprocess.Popen([sys.executable, "-c", src, str(r)], stdout=subprocess.PIPE,
                           stderr=subprocess.STDOUT, text=True, env=_env()) for r in range(world)]
    outs = []
    for p in ps:
        try:
            outs.append(p.communicate(timeout=600)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            outs.append(p.communicate()[0])
    assert all(p.returncode == 0 for p in ps), outs
    from embedcuda import synth
    from oracle import oracle
    x, _ = synth.make_ivf_corpus(40000, 384, 64, seed=4)
    sample = synth.make_ivf_sample(len(x), 4)
    assert np.array_equal(np.load(out), oracle.kmeans(x, sample, 64, 4))
