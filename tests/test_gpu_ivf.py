"""IVF path parity: assignments, k-means, inverted lists and search results
are compared with the oracle (ann.lisp / kb.lisp restatement).  Scores use
the reference's sequential single-float arithmetic, so results are exact."""
import numpy as np
import pytest

from embedcuda import ann, kb, synth
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def corpus():
    x, _ = synth.make_ivf_corpus(20000, 384, 64, seed=4)
    return x


def test_assign_exact(ec, corpus):
    x = corpus
    rng = np.random.default_rng(0)
    cent = x[rng.choice(len(x), 300, replace=False)]
    got = ann.assign(x, cent)
    ref = oracle.assign(x, cent)
    assert np.array_equal(got, ref)
    rows = rng.choice(len(x), 5000, replace=False)
    assert np.array_equal(ann.assign(x, cent, rows=rows), oracle.assign(x, cent, rows=rows))


def _assign_rows(ec):
    import ctypes as C
    tc, ex = C.c_longlong(), C.c_longlong()
    ec.check(ec.lib().ecdbg_assign_rows(C.byref(tc), C.byref(ex), 1), "assign rows")
    return tc.value, ex.value


# d % 64 == 0 and k % 128 == 0: bf16 tensor-core scores with an error window,
# candidates re-scored exactly; results must equal the exact scan bit for bit
@pytest.mark.parametrize("k", [128, 384, 512])
def test_assign_tensor_core_exact(ec, corpus, k):
    x = corpus
    rng = np.random.default_rng(k)
    cent = x[rng.choice(len(x), k, replace=False)].copy()
    _assign_rows(ec)
    got = ann.assign(x, cent)
    tc, _ = _assign_rows(ec)
    assert tc > 0  # the tensor-core path ran
    assert np.array_equal(got, oracle.assign(x, cent))


def test_assign_tensor_core_ties_and_near_ties(ec, corpus):
    """Duplicated centroids (exact ties: lowest index wins), clusters of
    near-identical centroids (more candidates than one part keeps: those rows
    take the exact scan), rows equal to centroids, a row too large for a
    finite norm."""
    x = corpus[:4000].copy()
    rng = np.random.default_rng(7)
    cent = x[rng.choice(len(x), 256, replace=False)].copy()
    cent[200] = cent[3]                      # exact duplicate, higher index
    cent[201] = cent[3]
    for j in range(10, 16):                  # six near-copies of centroid 9
        cent[j] = cent[9] + 1e-4 * rng.standard_normal(cent.shape[1]).astype(np.float32)
    x[:50] = cent[rng.integers(0, 256, 50)]  # rows sitting on centroids
    x[50] = cent[3]
    x[51] = cent[9]
    x[52, :] = 3e19                          # |x|^2 overflows single-float
    _assign_rows(ec)
    got = ann.assign(x, cent)
    tc, exact = _assign_rows(ec)
    assert tc > 0 and exact > 0
    ref = oracle.assign(x, cent)
    assert np.array_equal(got, ref)
    assert got[50] == 3


def test_kmeans_tensor_core_bit_exact(ec, corpus):
    x = corpus
    sample = synth.make_ivf_sample(len(x), 4)
    _assign_rows(ec)
    got = ann.kmeans(x, sample, 256, 4)
    tc, _ = _assign_rows(ec)
    assert tc > 0
    assert np.array_equal(got, oracle.kmeans(x, sample, 256, 4))


def test_assign_ties_lowest_index(ec):
    x = np.zeros((8, 8), np.float32)
    x[:, 0] = 1.0
    cent = np.zeros((5, 8), np.float32)
    cent[[1, 3, 4], 0] = 2.0  # three tied best centroids
    assert np.all(ann.assign(x, cent) == 1)


def test_kmeans_bit_exact(ec, corpus):
    x = corpus
    sample = synth.make_ivf_sample(len(x), 4)
    got = ann.kmeans(x, sample, 64, 5)
    ref = oracle.kmeans(x, sample, 64, 5)
    assert np.array_equal(got, ref)


def test_kmeans_empty_cluster_kept(ec):
    x = np.eye(8, dtype=np.float32)[:6]
    init = np.zeros((4, 8), np.float32)
    init[0, 0] = init[1, 1] = 1.0
    init[3, 7] = 5.0  # nothing comes closer to it than to others? it wins nothing with x
    init[2] = -1.0
    sample = np.arange(6, dtype=np.int64)
    got = ann.kmeans(x, sample, 4, 3, init=init)
    # cluster 2 never wins a row: it keeps its initial centroid (ann.lisp:118)
    assert np.array_equal(got[2], init[2])


def test_assign_all_lists(ec, corpus):
    x = corpus
    cent = x[:128]
    counts, lists = ann.assign_all(x, cent)
    rc, rl = oracle.assign_all(x, cent)
    assert np.array_equal(counts, rc) and np.array_equal(lists, rl)


# ann:run in one call (ec_ann_build): the rows go up once; the sample is the
# whole corpus in order (k-means rows = the resident copy, its bf16 rows
# reused by the final assignment), a contiguous slice of it, a permutation
# of it or a random subset (both gathered on the device)
@pytest.mark.parametrize("kind", ["all", "slice", "perm", "subset"])
def test_ann_build_one_upload(ec, corpus, kind):
    x = corpus
    n = len(x)
    rng = np.random.default_rng(11)
    sample = {"all": np.arange(n), "slice": np.arange(1000, 15000), "perm": rng.permutation(n),
              "subset": rng.choice(n, 6000, replace=False)}[kind].astype(np.int64)
    k, iters = 256, 3
    cent, counts, lists = ann.build(x, sample, k, iters)
    ref_cent = oracle.kmeans(x, sample, k, iters)
    assert np.array_equal(cent, ref_cent)
    rc, rl = oracle.assign_all(x, ref_cent)
    assert np.array_equal(counts, rc) and np.array_equal(lists, rl)
    # the same as the two calls
    c2 = ann.kmeans(x, sample, k, iters)
    assert np.array_equal(cent, c2)


def test_ann_build_init_and_small_k(ec, corpus):
    # given initial centroids, k below the tensor-core granule (exact scan)
    x = corpus[:3000]
    sample = np.arange(len(x), dtype=np.int64)
    init = np.ascontiguousarray(x[[5, 900, 1700, 2999, 42]])
    cent, counts, lists = ann.build(x, sample, 5, 2, init=init)
    assert np.array_equal(cent, ann.kmeans(x, sample, 5, 2, init=init))
    rc, rl = ann.assign_all(x, cent)
    assert np.array_equal(counts, rc) and np.array_equal(lists, rl)
    assert int(counts.sum()) == len(x)


def test_ivf_and_flat_search(ec, corpus):
    x = corpus
    sample = synth.make_ivf_sample(len(x), 4)
    cent = ann.kmeans(x, sample, 64, 3)
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    qs, _ = synth.make_ivf_corpus(40, 384, 64, seed=99)
    ids, sc = kb.search_ivf(qs, 10, nprobe=8)
    for i in range(len(qs)):
        rid, rsc = oracle.top_k_ivf(x, cent, counts, lists, 8, qs[i], 10)
        assert np.array_equal(ids[i][:len(rid)], rid), i
        assert np.array_equal(sc[i][:len(rsc)], rsc), i
    fid, fsc = kb.search_brute(qs[:8], 10)
    for i in range(8):
        rid, rsc = oracle.top_k_brute(x, qs[i], 10)
        assert np.array_equal(fid[i], rid) and np.array_equal(fsc[i], rsc)
    # kb::top-k pairs
    pairs = kb.top_k(qs[0], 5)
    assert len(pairs) == 5 and all(pairs[j][1] >= pairs[j + 1][1] for j in range(4))


def _check_ivf(x, cent, counts, lists, qs, nprobe, topk):
    ids, sc = kb.search_ivf(qs, topk, nprobe=nprobe)
    for i in range(len(qs)):
        rid, rsc = oracle.top_k_ivf(x, cent, counts, lists, nprobe, qs[i], topk)
        assert np.array_equal(ids[i][:len(rid)], rid), i
        assert np.array_equal(sc[i][:len(rsc)], rsc), i
        assert np.all(ids[i][len(rid):] == -1), i


@pytest.mark.parametrize("topk", [1, 10, 64])
def test_ivf_search_query_batched(ec, corpus, topk):
    """Enough queries that every list gets several 32-query chunks: the
    list-major scan (one CTA per list and query chunk) against kb::top-k-ivf."""
    x = corpus
    cent = x[synth.make_ivf_sample(len(x), 5)[:64]]
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    qs, _ = synth.make_ivf_corpus(400, 384, 64, seed=101)
    _check_ivf(x, cent, counts, lists, qs, 8, topk)


def test_ivf_search_batched_ties_empty_lists_odd_dim(ec):
    """d = 100 (a partial 32-column chunk), every row duplicated (equal scores:
    the earlier list position must win), and centroids that own no rows
    (empty lists probed by many queries)."""
    base, _ = synth.make_ivf_corpus(3000, 100, 16, seed=7)
    x = np.repeat(base, 2, axis=0)
    far = -np.ones((8, 100), np.float32) / 10.0  # attract no rows
    cent = np.concatenate([x[::250][:24], far], axis=0).astype(np.float32)
    counts, lists = ann.assign_all(x, cent)
    assert (counts == 0).sum() >= 1
    kb.load_index(x, (cent, counts, lists))
    qs, _ = synth.make_ivf_corpus(300, 100, 16, seed=8)
    qs = np.concatenate([qs, base[:20]], axis=0)  # exact duplicates of rows
    _check_ivf(x, cent, counts, lists, qs, 32, 10)
    _check_ivf(x, cent, counts, lists, qs, 5, 64)


@pytest.mark.parametrize("nq", [1, 3])
def test_ivf_search_few_queries_tied_probes(ec, corpus, nq):
    """A few queries (the staged-row probe scores, the warp-level merge):
    every centroid duplicated, so probe scores tie in pairs and the nprobe-th
    place falls inside a tie (the radix select's index passes); nprobe 33
    splits a pair, nprobe 32 keeps whole pairs (no index pass)."""
    x = corpus
    base = x[synth.make_ivf_sample(len(x), 9)[:48]]
    cent = np.ascontiguousarray(np.repeat(base, 2, axis=0))
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    rng = np.random.default_rng(nq)
    qs = np.ascontiguousarray(x[rng.choice(len(x), nq, replace=False)])
    for nprobe, topk in [(33, 10), (32, 10), (5, 64), (1, 1)]:
        _check_ivf(x, cent, counts, lists, qs, nprobe, topk)


def test_flat_search_query_batched(ec, corpus):
    x = corpus
    kb.load_index(x, None)
    qs, _ = synth.make_ivf_corpus(40, 384, 64, seed=11)
    qs = np.concatenate([qs, x[100:104]], axis=0)
    for topk in (10, 64):
        fid, fsc = kb.search_brute(qs, topk)
        for i in range(len(qs)):
            rid, rsc = oracle.top_k_brute(x, qs[i], topk)
            assert np.array_equal(fid[i], rid) and np.array_equal(fsc[i], rsc), (topk, i)


@pytest.mark.parametrize("nprobe", [16, 32, 128])
def test_ivf_search_tensor_core_probes(ec, corpus, nprobe):
    """Batches of >= 64 queries with k % 128 == 0 score the probes on the
    tensor cores and re-score the centroids inside the error window exactly:
    the probe order (and so every result) must equal kb::top-k-ivf's."""
    x = corpus
    cent = x[synth.make_ivf_sample(len(x), 6)[:256]]
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    qs, _ = synth.make_ivf_corpus(160, 384, 64, seed=102)
    qs = np.concatenate([qs, x[:16]], axis=0)
    _check_ivf(x, cent, counts, lists, qs, nprobe, 10)


def test_ivf_search_tensor_core_probe_ties_and_fallback(ec, corpus):
    """300 identical centroids (exact ties, decided by the lower index) out
    of 384: queries next to them have more window candidates than the fast
    path keeps and take the exact scoring of every centroid; the others stay
    on the fast path.  Both must give kb::top-k-ivf's results."""
    x = corpus
    rest = x[synth.make_ivf_sample(len(x), 7)[:84]]
    cent = np.concatenate([rest[:40], np.repeat(x[5:6], 300, axis=0), rest[40:]], axis=0).astype(np.float32)
    assert cent.shape[0] == 384
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    near = x[5:6] + 0.01 * np.random.default_rng(3).standard_normal((40, 384)).astype(np.float32)
    far, _ = synth.make_ivf_corpus(60, 384, 64, seed=103)
    qs = np.concatenate([near / np.linalg.norm(near, axis=1, keepdims=True), far], axis=0).astype(np.float32)
    _check_ivf(x, cent, counts, lists, qs, 32, 10)
    _check_ivf(x, cent, counts, lists, qs, 128, 10)


# ---- the IVF workload's own density: k 4096, d 384 ------------------------------

@pytest.fixture(scope="module")
def c5_subset():
    """200,000 rows of the IVF workload's distribution (4096 Gaussian
    clusters, centers uniform on the unit sphere, sigma 0.05, rows
    L2-normalised, seed 4) and its seeded training permutation."""
    x, _ = synth.make_ivf_corpus(200_000, 384, 4096, seed=4)
    return x, synth.make_ivf_sample(len(x), 4)


def test_c5_density_assign_kmeans_lists_exact(ec, c5_subset):
    """At k = 4096, d = 384 the tensor-core window holds many near-tied
    centroids per row: assignments from identical centroids, two Lloyd
    iterations and the final inverted lists must still equal the oracle's
    (ann.lisp:69-158) exactly -- no tie exceptions are needed."""
    x, sample = c5_subset
    k = 4096
    init = x[sample[:k]].copy()
    _assign_rows(ec)
    got = ann.assign(x, init)
    tc, exact = _assign_rows(ec)
    assert tc > 0  # the tensor-core path ran at this density
    assert np.array_equal(got, oracle.assign(x, init))
    cent = ann.kmeans(x, sample, k, 2)
    ref = oracle.kmeans(x, sample, k, 2)
    assert np.array_equal(cent, ref)
    counts, lists = ann.assign_all(x, cent)
    rc, rl = oracle.assign_all(x, ref)
    assert np.array_equal(counts, rc) and np.array_equal(lists, rl)
    # IVF top-10 at nprobe 32 over the same index (kb.lisp:348-364)
    kb.load_index(x, (cent, counts, lists))
    qs, _ = synth.make_ivf_corpus(300, 384, 4096, seed=4)
    _check_ivf(x, cent, counts, lists, qs[:200], 32, 10)
