#!/usr/bin/env python
"""Benchmark of the B200 embedding hot path (one JSON line on rank 0).

Default workload: corpus embedding with the all-MiniLM-L6-v2 shape (6 layers,
hidden 384, 12 heads x 32, FFN 1536, seed-0 random F32 weights run on the
BF16 tensor-core path), 1024 sequences of uniform length 16..256 with
[CLS]/[SEP], mean pooling + L2.  A step is one forward over the whole batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload minilm|bert-base|mpnet|qwen3|gemma]

N > 1 is launched by torch.distributed.run, one process per GPU: every rank
embeds its own 1024-sequence shard (weak scaling, no data-path collective);
`value` is all ranks' sequences / the slowest rank's time.

--impl reference times the reference algorithm on the host cores (the Lisp
cannot run here, so its CPU restatement in oracle/ stands in, threads = all
host cores, one sequence per thread as embed.lisp does).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "lisp-embed_b200"))

import numpy as np  # noqa: E402

WORKLOADS = {
    # name: (shape name, seed, sequences per rank, description)
    "minilm": ("minilm-l6", 0, 1024, "MiniLM-L6 shape, 1024 seqs len U[16,256], mean pool"),
    "bert-base": ("bert-base", 1, 8192, "BERT-base shape BF16, 8192 seqs log-U[32,512], CLS"),
    "mpnet": ("mpnet-base", 2, 4096, "MPNet-base shape, 4096 seqs len U[64,384], mean pool"),
    "qwen3": ("qwen3-0.6b", 3, 2048, "Qwen3-0.6B shape BF16, 2048 seqs len U[128,512]+EOS, last"),
    "gemma": ("embeddinggemma", 4, 2048,
              "EmbeddingGemma shape (24 layers, H 512, PLE 512, out 768), 2048 seqs "
              "len U[16,512], mean pool + projection"),
}
IVF_N, IVF_D, IVF_K, IVF_ITERS, IVF_SEED = 3_270_000, 384, 4096, 20, 4
SEARCH_NQ, SEARCH_NPROBE, SEARCH_TOPK = 10_000, 32, 10


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS) + ["ivf", "query", "search", "tokenize"], default="minilm")
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="bounded CPU-baseline sample length")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--search-rows", type=int, default=IVF_N,
                   help="search workload: index rows (a smaller index for profiling)")
    p.add_argument("--search-k", type=int, default=IVF_K,
                   help="search workload: centroids")
    p.add_argument("--search-queries", type=int, default=SEARCH_NQ,
                   help="search workload: queries per call")
    return p.parse_args()


def algorithmic_flops(shape, offsets):
    """Encoder FLOPs on true lengths: layers * [2 L (4H^2 + 2HF) + 4 L^2 H]
    (BERT family); Qwen3: layers * [2 L (qkv+o+3HF) + 2 * 2 L(L+1)/2 * heads*hd];
    EmbeddingGemma: layers * [2 L (qkv+o+3HF + 3HP) + 4 L^2 heads*hd] (3HP: its
    slice of the per-layer-embedding projection, the PLE gate and projection)."""
    lens = np.diff(offsets).astype(np.float64)
    H, F, Lr = shape.hidden, shape.inter, shape.layers
    if shape.model_type == "qwen3":
        hd, nh, kv = shape.head_dim, shape.heads, shape.kv_heads
        lin = H * (nh * hd + 2 * kv * hd) + nh * hd * H + 3 * H * F
        return float(Lr * np.sum(2 * lens * lin + 2 * nh * hd * lens * (lens + 1)))
    if shape.model_type == "embedding_gemma2":
        hd, nh, kv, P = shape.head_dim, shape.heads, shape.kv_heads, shape.extra["ple_dim"]
        lin = H * (nh * hd + 2 * kv * hd) + nh * hd * H + 3 * H * F + 3 * H * P
        return float(Lr * np.sum(2 * lens * lin + 4 * nh * hd * lens * lens))
    return float(Lr * np.sum(2 * lens * (4 * H * H + 2 * H * F) + 4 * lens * lens * H))


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            j = json.load(f)
        return j, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, \
            "fallback"


def profile_traffic(kind):
    """DRAM bytes per GEMM launch from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", f"{kind}.txt")
    try:
        with open(path) as f:
            for ln in f:
                if ln.startswith("traffic_bytes_per_launch:"):
                    return float(ln.split(":", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock / throttle reasons during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.tmp = None

    def __enter__(self):
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        try:
            with open(self.tmp.name) as f:
                rows = [ln.strip().split(", ") for ln in f if ln.strip()]
            os.unlink(self.tmp.name)
        except OSError:
            return None
        rows = [r for r in rows if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline(model_dir, ids, offsets, seconds):
    """The oracle (CPU restatement of the reference) on all host cores, one
    sequence per thread in batches (embed.lisp:88-105); bounded sample."""
    from oracle import oracle
    om = oracle.OracleModel(model_dir)
    threads = os.cpu_count() or 1
    nseq = len(offsets) - 1
    done = 0
    t0 = time.perf_counter()
    s = 0
    while True:
        b = list(range(s, min(nseq, s + threads)))
        if not b:
            s = 0
            continue
        sub_off = offsets[b[0]:b[-1] + 2] - offsets[b[0]]
        om.embed_batch(ids[offsets[b[0]]:offsets[b[-1] + 1]], sub_off, threads=threads)
        done += len(b)
        s = b[-1] + 1 if b[-1] + 1 < nseq else 0
        if time.perf_counter() - t0 >= seconds:
            break
    el = time.perf_counter() - t0
    return {"value": done / el, "unit": "embeddings/s", "cores": threads, "kind": "port",
            "sample": f"{done} of the workload's sequences in {el:.1f} s "
                      f"({threads} threads, one sequence per thread)"}


def ivf_corpus_torch(n, d, k, seed, device, nqueries=0):
    """The IVF workload generated on the GPU: k centers uniform on the unit
    sphere, x = normalize(center + 0.05 N(0, I)), fp32 (same distribution as
    synth.make_ivf_corpus, drawn with torch's generator for speed).  With
    nqueries > 0 also returns that many queries drawn from the same mixture
    after the corpus (the corpus is unchanged)."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    centers = torch.randn(k, d, generator=g, device=device)
    centers /= centers.norm(dim=1, keepdim=True)
    labels = torch.randint(0, k, (n,), generator=g, device=device)
    x = torch.empty(n, d, device=device)
    step = 1 << 20
    for s0 in range(0, n, step):
        e = min(n, s0 + step)
        blk = centers[labels[s0:e]] + 0.05 * torch.randn(e - s0, d, generator=g, device=device)
        x[s0:e] = blk / blk.norm(dim=1, keepdim=True)
    perm = torch.randperm(n, generator=g, device=device)
    if nqueries <= 0:
        return x, perm
    ql = torch.randint(0, k, (nqueries,), generator=g, device=device)
    q = centers[ql] + 0.05 * torch.randn(nqueries, d, generator=g, device=device)
    return x, perm, q / q.norm(dim=1, keepdim=True)


def run_ivf(args, rank, world, local_rank):
    """IVF build seconds: 20 Lloyd iterations over all 3.27M rows (k 4096,
    init = first k rows of a seeded permutation, ann.lisp:83-86), rows
    sharded over the ranks with one NCCL all-reduce of sums + counts per
    iteration, then the inverted lists of each shard (ann::assign-all).
    Inputs start in host memory; the timed region includes their upload."""
    import ctypes as C
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from embedcuda import _lib, ann
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    x_dev, perm = ivf_corpus_torch(IVF_N, IVF_D, IVF_K, IVF_SEED, "cuda")
    j0 = (IVF_N + world - 1) // world * rank
    j1 = min(IVF_N, j0 + (IVF_N + world - 1) // world)
    mine = perm[j0:j1]
    x_local = x_dev[mine].cpu().numpy()            # this rank's training rows, sample order
    init = x_dev[perm[:IVF_K]].cpu().numpy()        # same on every rank
    del x_dev
    torch.cuda.empty_cache()
    _lib.init([local_rank])
    L = _lib.lib()
    if world > 1:
        idbuf = C.create_string_buffer(L.ec_comm_id_size())
        if rank == 0:
            _lib.check(L.ec_comm_get_id(idbuf), "comm id")
        t = torch.frombuffer(bytearray(idbuf.raw), dtype=torch.uint8).cuda()
        dist.broadcast(t, 0)
        idbuf = C.create_string_buffer(bytes(t.cpu().numpy()), len(idbuf.raw))
        _lib.check(L.ec_comm_init(rank, world, idbuf), "comm init")
    local_sample = np.arange(len(x_local), dtype=np.int64)
    # warm-up: one iteration (module load, NCCL channels)
    ann.kmeans(x_local[:200000], local_sample[:200000], IVF_K, 1, init=init)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    L.ecdbg_profile(1)
    L.ecdbg_assign_rows(None, None, 1)
    t0 = time.perf_counter()
    cent = ann.kmeans(x_local, local_sample, IVF_K, IVF_ITERS, init=init)
    t_km = time.perf_counter() - t0
    counts, lists = ann.assign_all(x_local, cent)
    t_all = time.perf_counter() - t0
    v = [C.c_double(), C.c_double(), C.c_double(), C.c_longlong()]
    L.ecdbg_profile_read(b"gemm", *[C.byref(z) for z in v])
    g_ms, g_flops, g_launches = v[0].value, v[1].value, v[3].value
    L.ecdbg_profile_read(b"rows", *[C.byref(z) for z in v])
    r_ms = v[0].value
    L.ecdbg_profile(0)
    tc_rows, ex_rows = C.c_longlong(), C.c_longlong()
    L.ecdbg_assign_rows(C.byref(tc_rows), C.byref(ex_rows), 0)
    if world > 1:
        tt = torch.tensor([t_km, t_all], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_km, t_all = float(tt[0]), float(tt[1])
    if rank == 0:
        flops = 2.0 * IVF_N * IVF_K * IVF_D * (IVF_ITERS + 1)
        out = {"metric": "IVF build s", "value": t_all, "unit": "s", "n_gpus": world,
               "steps": 1, "warmup": 1, "ms_per_step": 1000 * t_all, "higher_is_better": False,
               "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
               "config": {"workload": "ivf-3.27Mx384", "n": IVF_N, "dim": IVF_D, "k": IVF_K,
                          "iters": IVF_ITERS, "sample": "all rows, seeded permutation",
                          "kmeans_s": t_km, "assign_all_s": t_all - t_km,
                          "parallelism": f"rows sharded over {world} GPU(s), NCCL all-reduce"},
               "achieved_tflops": flops / t_all / 1e12,
               "note": "assignments bit-exact to ann.lisp's sequential single-float scores on "
                       "one GPU: bf16 tensor-core scores with a rigorous error window, "
                       "candidates re-scored exactly, the rest of the rows scanned exactly"}
        peaks, src = measured_peaks()
        achieved = g_flops / (g_ms * 1e-3) / 1e12 if g_ms > 0 else None
        peak = peaks.get("bf16_tflops")
        out["roofline"] = {"bound": "tensor", "kernel": "gemm_tn_bf16_kernel<256, kEpiArgCand> "
                                                       "(assignment scores)",
                           "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                           "frac": achieved / peak if achieved and peak else None,
                           "traffic": None, "launches": g_launches,
                           "peak_source": f"{src} bf16_tflops (burst: each launch ~10 ms)"}
        out["kernel_classes"] = {"assign_gemm_ms": g_ms, "assign_reduce_ms": r_ms}
        out["assign_rows"] = {"tensor_core": tc_rows.value, "exact_scan": ex_rows.value}
        print(json.dumps(out), flush=True)
    _lib.shutdown()
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_query(args, rank, local_rank):
    """p50 ms of one short MiniLM query end to end through the host API:
    ec_embed_batch of ~10 token ids, then ec_ivf_search top-10 with nprobe 32
    over the 3.27M x 384 IVF index (kb:kb-search without the text part)."""
    if rank != 0:
        return 0
    import torch
    from embedcuda import _lib, ann, kb, model, synth
    torch.cuda.set_device(local_rank)
    x_dev, perm = ivf_corpus_torch(IVF_N, IVF_D, IVF_K, IVF_SEED, "cuda")
    x = x_dev.cpu().numpy()
    del x_dev
    torch.cuda.empty_cache()
    perm = perm.cpu().numpy().astype(np.int64)
    _lib.init([local_rank])
    cent = ann.kmeans(x, perm, IVF_K, IVF_ITERS)
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    d = synth.build_model_dir(synth.MINILM, 0, os.environ.get("EC_SYNTH_DIR", "/tmp/ec_synth"))
    model.load_model(d)
    rng = np.random.default_rng(7)
    times = []
    for i in range(101 + args.warmup):
        ids = np.concatenate([[101], rng.integers(1000, 30522, 8), [102]]).astype(np.int32)
        t0 = time.perf_counter()
        q = model.embed(ids)
        ids_, sc = kb.search_ivf(q, 10, nprobe=32)
        el = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(el)
    p50 = 1000 * float(np.median(times))
    out = {"metric": "p50 query ms", "value": p50, "unit": "ms", "n_gpus": 1, "steps": 101,
           "warmup": args.warmup, "ms_per_step": p50, "higher_is_better": False,
           "scaling": "none", "vs_baseline": None, "dtype": "bf16+f32", "data": "synthetic",
           "config": {"workload": "minilm-l6 query (10 ids) + ivf top-10 nprobe 32 over 3.27Mx384",
                      "p90_ms": 1000 * float(np.percentile(times, 90)),
                      "min_ms": 1000 * float(np.min(times))}}
    print(json.dumps(out), flush=True)
    _lib.shutdown()
    return 0




def search_cpu_baseline(x, cent, counts, lists, qs, nprobe, topk, seconds, threads=None):
    """The oracle's kb::top-k-ivf on the host cores: one query per thread at a
    time (the C restatement releases the GIL), for about `seconds`.  Returns
    (queries done, elapsed s, threads)."""
    import threading
    from oracle import oracle
    threads = threads or os.cpu_count() or 1
    lock = threading.Lock()
    state = {"next": 0, "done": 0}
    t0 = time.perf_counter()

    def worker():
        while True:
            with lock:
                i = state["next"]
                if i >= len(qs) or time.perf_counter() - t0 >= seconds:
                    return
                state["next"] = i + 1
            oracle.top_k_ivf(x, cent, counts, lists, nprobe, qs[i], topk)
            with lock:
                state["done"] += 1

    pool = [threading.Thread(target=worker) for _ in range(threads)]
    for t in pool:
        t.start()
    for t in pool:
        t.join()
    return state["done"], time.perf_counter() - t0, threads


def run_search(args, rank, local_rank):
    """Queries/s of batched IVF search (kb::top-k-ivf for a batch): 10,000
    queries from the corpus mixture, nprobe 32, top-10, over the 3.27M x 384
    index (k 4096 from 20 Lloyd iterations).  Each step is one ec_ivf_search
    call on all queries through the host API (queries uploaded, ids and
    scores read back inside the timed region).  Results are bit-identical to
    the reference's sequential single-float scores."""
    if rank != 0:
        return 0
    import ctypes as C
    import torch
    from embedcuda import _lib, ann, kb
    from oracle import oracle
    torch.cuda.set_device(local_rank)
    n, k, nq = args.search_rows, args.search_k, args.search_queries
    x_dev, perm, q_dev = ivf_corpus_torch(n, IVF_D, k, IVF_SEED, "cuda", nq)
    x = x_dev.cpu().numpy()
    qs = q_dev.cpu().numpy()
    del x_dev, q_dev
    torch.cuda.empty_cache()
    perm = perm.cpu().numpy().astype(np.int64)
    _lib.init([local_rank])
    cent = ann.kmeans(x, perm, k, IVF_ITERS)
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    L = _lib.lib()
    for _ in range(args.warmup):
        kb.search_ivf(qs, SEARCH_TOPK, nprobe=SEARCH_NPROBE)
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    smi_index = phys[local_rank] if len(phys) > local_rank and phys[local_rank] else local_rank
    with ClockSampler(smi_index) as clk:
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            ids, sc = kb.search_ivf(qs, SEARCH_TOPK, nprobe=SEARCH_NPROBE)
            times.append(time.perf_counter() - t0)
    el = sum(times) / len(times)
    # one more pass with the scan kernel event-timed (profiling reads the
    # probes back before the scan, so it is kept out of the timed steps)
    L.ecdbg_profile(1)
    kb.search_ivf(qs, SEARCH_TOPK, nprobe=SEARCH_NPROBE)
    v = [C.c_double(), C.c_double(), C.c_double(), C.c_longlong()]
    L.ecdbg_profile_read(b"scan", *[C.byref(z) for z in v])
    L.ecdbg_profile(0)
    scan_ms, scan_flops, scan_bytes = v[0].value, v[1].value, v[2].value
    # spot parity against the oracle (kb::top-k-ivf restated) on a few queries
    for i in range(0, nq, max(1, nq // 4)):
        rid, rsc = oracle.top_k_ivf(x, cent, counts, lists, SEARCH_NPROBE, qs[i], SEARCH_TOPK)
        if not (np.array_equal(ids[i][:len(rid)], rid) and np.array_equal(sc[i][:len(rsc)], rsc)):
            raise SystemExit(f"search parity failed on query {i}")
    # CPU baseline: the oracle's kb::top-k-ivf on all host cores
    done, cpu_el, cpu_threads = 0, 1.0, 1
    if not args.no_cpu_baseline:
        done, cpu_el, cpu_threads = search_cpu_baseline(x, cent, counts, lists, qs, SEARCH_NPROBE,
                                                        SEARCH_TOPK, 10.0)
    peak = None
    clocks = clk.summary()
    sm_max = clocks.get("sm_max_mhz") if clocks else None
    props = torch.cuda.get_device_properties(local_rank)
    if sm_max:
        peak = props.multi_processor_count * 128 * sm_max * 1e6 / 1e12
    achieved = scan_flops / (scan_ms * 1e-3) / 1e12 if scan_ms > 0 else None
    qps = nq / el
    out = {"metric": "queries/s", "value": qps, "unit": "queries/s", "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el,
           "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic",
           "config": {"workload": f"ivf-search-{n / 1e6:g}Mx{IVF_D}", "queries": nq,
                      "nprobe": SEARCH_NPROBE, "topk": SEARCH_TOPK, "k": k, "rows": n,
                      "l2": f"index {n * IVF_D * 4 / 1e9:.1f} GB > L2",
                      "timing": "host wall clock around the synchronous ec_ivf_search call"},
           "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": int(qs.nbytes),
                   "d2h_bytes_per_step": nq * SEARCH_TOPK * 12},
           "roofline": {"bound": "fp32", "kernel": "tile_scan_kernel<true> (list scan)",
                        "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak if achieved and peak else None, "traffic": None,
                        "peak_source": "nominal: SMs x 128 fp32 lanes x max SM clock, one "
                                       "rounded op per lane per clock (the reference's multiply "
                                       "and add are rounded separately, so they cannot fuse)",
                        "scan_ms_per_step": scan_ms,
                        "algorithmic_gb_per_step": scan_bytes / 1e9,
                        "algorithmic_note": "2 FLOP and 4 bytes per probed row and column"},
           "clocks": clocks,
           "cpu_baseline": None if args.no_cpu_baseline else {
                            "value": done / cpu_el, "unit": "queries/s", "cores": cpu_threads,
                            "kind": "port",
                            "sample": f"{done} queries in {cpu_el:.1f} s (oracle kb::top-k-ivf, "
                                      f"one query per thread on {cpu_threads} threads)"}}
    print(json.dumps(out), flush=True)
    _lib.shutdown()
    return 0


def run_reference(args, rank):
    """--impl reference: the oracle port of the reference's CPU path."""
    if rank != 0:
        return 0
    from embedcuda import synth
    shape_name, seed, nseq, desc = WORKLOADS[args.workload]
    shape = synth.SHAPES[shape_name]
    root = os.environ.get("EC_SYNTH_DIR", "/tmp/ec_synth")
    d = synth.build_model_dir(shape, seed, root)
    ids, offsets = synth.make_inputs(shape_name, nseq, seed)
    from oracle import oracle
    om = oracle.OracleModel(d)
    threads = os.cpu_count() or 1
    times, counts = [], []
    pos = 0

    def one_step():
        nonlocal pos
        b0 = pos
        b1 = min(nseq, pos + threads)
        sub_off = offsets[b0:b1 + 1] - offsets[b0]
        t = time.perf_counter()
        om.embed_batch(ids[offsets[b0]:offsets[b1]], sub_off, threads=threads)
        el = time.perf_counter() - t
        pos = b1 if b1 < nseq else 0
        return el, b1 - b0

    for _ in range(args.warmup):
        one_step()
    for _ in range(args.steps):
        el, c = one_step()
        times.append(el)
        counts.append(c)
    tot = sum(times)
    value = sum(counts) / tot
    line = {
        "impl": "reference", "metric": "embeddings/sec", "value": value, "unit": "embeddings/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * tot / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": shape_name, "description": desc, "sequences_per_step": threads,
                   "note": "each step embeds `threads` sequences of the workload"},
        "cpu_baseline": {"value": value, "unit": "embeddings/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x {threads} sequences; SBCL absent, the "
                                   "C restatement of bert.lisp/llama.lisp stands in"},
        "e2e": {"value": value, "unit": "embeddings/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_tokenize(args, rank):
    """tokenizer.lisp's tk-encode on the host: texts/s of ec_tokenize (C++,
    all host threads) over 20,000 synthetic sentences of 16..256 words, with
    the WordPiece tokenizer.json fixture (700-piece vocabulary, lowercase,
    [CLS]/[SEP]).  cpu_baseline: the Python restatement of tokenizer.lisp on
    one thread over a bounded sample (the Lisp itself needs SBCL)."""
    if rank != 0:
        return 0
    import random
    from embedcuda.tokenizer import Tokenizer
    tok_json = os.path.join(REPO, "tests", "golden", "tok", "wordpiece.json")
    rng = random.Random(11)
    syl = ["ka", "to", "ri", "na", "mo", "se", "lu", "pe", "di", "ga", "vo", "stra", "ble",
           "ing", "tion", "er", "ed", "ly", "pre", "un", "re", "ment", "ness"]
    punct = [",", ".", "!", "?", ";", "(", ")"]

    def sentence():
        words = []
        for _ in range(rng.randint(16, 256)):
            r = rng.random()
            words.append(rng.choice(punct) if r < 0.08 else str(rng.randint(0, 9999)) if r < 0.14
                         else "".join(rng.choice(syl) for _ in range(rng.randint(1, 4))))
        return " ".join(words)

    texts = [sentence() for _ in range(20000)]
    tk = Tokenizer.from_json(tok_json)
    for _ in range(args.warmup):
        tk.encode_batch(texts[:2000])
    times = []
    ntok = 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ids, offs = tk.encode_batch(texts)
        times.append(time.perf_counter() - t0)
        ntok = int(offs[-1])
    el = sum(times)
    threads = os.cpu_count() or 1
    value = len(texts) * args.steps / el
    out = {"metric": "texts/s", "value": value, "unit": "texts/s", "n_gpus": 0,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * el / args.steps,
           "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "utf-8",
           "data": "synthetic", "config": {"workload": "tokenize (tk-encode, WordPiece)",
                                           "texts_per_step": len(texts),
                                           "tokens_per_step": ntok, "threads": threads},
           "tokens_per_s": ntok * args.steps / el}
    if not args.no_cpu_baseline:
        from oracle import tokenizer_ref
        r = tokenizer_ref.from_json(tok_json)
        t0 = time.perf_counter()
        done = 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 10.0) and done < len(texts):
            r.encode(texts[done])
            done += 1
        rel = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": done / rel, "unit": "texts/s", "cores": 1, "kind": "port",
                               "sample": f"{done} texts in {rel:.1f} s (Python restatement of "
                                         "tokenizer.lisp, one thread)"}
    print(json.dumps(out), flush=True)
    tk.close()
    return 0


def main():
    args = parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.workload in ("ivf", "query", "search", "tokenize"):
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "reference arm is timed for the embedding workloads only"}))
            return 0
        return run_reference(args, rank)
    if not os.environ.get("EC_KEEP_NCCL_DEBUG"):
        os.environ["NCCL_DEBUG"] = "WARN"
    if args.workload == "ivf":
        return run_ivf(args, rank, world, local_rank)
    if args.workload == "query":
        return run_query(args, rank, local_rank)
    if args.workload == "search":
        return run_search(args, rank, local_rank)
    if args.workload == "tokenize":
        return run_tokenize(args, rank)

    # NCCL's version banner goes to stdout; the benchmark prints one JSON line
    if not os.environ.get("EC_KEEP_NCCL_DEBUG"):
        os.environ["NCCL_DEBUG"] = "WARN"
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))

    from embedcuda import _lib, model, synth
    shape_name, seed, nseq, desc = WORKLOADS[args.workload]
    shape = synth.SHAPES[shape_name]
    root = os.path.join(os.environ.get("EC_SYNTH_DIR", "/tmp/ec_synth"), f"r{rank}")
    mdir = synth.build_model_dir(shape, seed, root)
    _lib.init([local_rank])
    model.load_model(mdir)
    dim = model.dim()
    rseed = seed if rank == 0 else seed * 100003 + 7919 * rank
    ids, offsets = synth.make_inputs(shape_name, nseq, rseed)
    T = int(offsets[-1])
    flops_step = algorithmic_flops(shape, offsets)

    d_ids = torch.from_numpy(ids).cuda()
    d_out = torch.empty((nseq, dim), dtype=torch.float32, device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    L = _lib.lib()

    def step_device():
        model.embed_batch_device(d_ids.data_ptr(), offsets, nseq, d_out.data_ptr(), dim, sptr)

    for _ in range(args.warmup):
        flush.zero_()
        step_device()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    # timed region: K steps, L2 flushed (256 MB write) between them, CUDA
    # events around each step on the stream the library launches on
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    smi_index = phys[local_rank] if len(phys) > local_rank and phys[local_rank] else local_rank
    L.ecdbg_profile(1)
    with ClockSampler(smi_index) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            step_device()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    launches = int(L.ecdbg_launches())
    L.ecdbg_profile(0)
    ms = sum(a.elapsed_time(b) for a, b in ev)
    prof = {}
    import ctypes as C
    for cls in ("gemm", "attention", "rows"):
        v = [C.c_double(), C.c_double(), C.c_double(), C.c_longlong()]
        L.ecdbg_profile_read(cls.encode(), *[C.byref(x) for x in v])
        prof[cls] = {"ms": v[0].value, "flops": v[1].value, "bytes": v[2].value,
                     "launches": v[3].value}
    clocks = clk.summary()

    # end to end through the host API (ec_embed_batch): ids from pinned host
    # memory in, embeddings back to host memory, each step
    h_ids = torch.from_numpy(ids).pin_memory().numpy()
    h_out = np.empty((nseq, dim), np.float32)
    for _ in range(2):
        model.embed_batch(h_ids, offsets, out=h_out)
    e2e_s = 0.0
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        model.embed_batch(h_ids, offsets, out=h_out)
        e2e_s += time.perf_counter() - t0
    nblk = int(np.sum((np.diff(offsets) + 63) // 64))
    h2d = T * 4 + (nseq + 1) * 4 + nblk * 8
    d2h = nseq * dim * 4

    if world > 1:
        t = torch.tensor([ms, e2e_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_s = float(t[0]), float(t[1])
        dist.barrier()

    out = None
    if rank == 0:
        peaks, src = measured_peaks()
        g = prof["gemm"]
        achieved = g["flops"] / (g["ms"] * 1e-3) / 1e12 if g["ms"] > 0 else None
        peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
        traffic = profile_traffic(f"gemm_{args.workload}")
        value = world * nseq * args.steps / (ms * 1e-3)
        step_tflops = flops_step * args.steps / (ms * 1e-3) / 1e12
        out = {
            "metric": "embeddings/sec", "value": value, "unit": "embeddings/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded ids and N(0,0.02) weights of the named shape)",
            "config": {"workload": shape_name, "description": desc, "sequences_per_rank": nseq,
                       "tokens_per_rank": T, "parallelism": f"dp{world} (sequence shards)",
                       "l2": "flushed (256 MB write) between timed steps",
                       "precision": "bf16 tensor-core GEMM/attention, fp32 accumulate, "
                                    "fp32 norms; residual between sublayers: the "
                                    "LayerNorm's bf16 output (BERT/MPNet), fp32 (Qwen3, "
                                    "Gemma)"},
            "e2e": {"value": world * nseq * args.steps / e2e_s, "unit": "embeddings/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "timing": "host wall clock around the synchronous ec_embed_batch call"},
            "roofline": {"bound": "tensor", "kernel": "gemm_tn_bf16 (all GEMM launches)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved / peak) if achieved and peak else None,
                         "traffic": traffic,
                         "peak_source": f"{src} bf16_tflops_sustained (dense cuBLAS, "
                                        "seconds-long loop)",
                         "step_tflops": step_tflops,
                         "step_frac_of_peak": step_tflops / peak if peak else None},
            "kernel_classes": prof,
            "gpu_launches": launches,
            "clocks": clocks,
        }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_baseline(mdir, ids, offsets, args.cpu_seconds)
        except Exception as e:  # the baseline must not sink the GPU number
            out["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if rank == 0:
        print(json.dumps(out), flush=True)
    _lib.shutdown()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
