#!/usr/bin/env python
"""Benchmark of the B200 embedding hot path (one JSON line on rank 0).

Default run: the headline is corpus embedding with the all-MiniLM-L6-v2
shape (6 layers, hidden 384, 12 heads x 32, FFN 1536, seed-0 random F32
weights run on the BF16 tensor-core path), 1024 sequences per rank of uniform
length 16..256 with [CLS]/[SEP], mean pooling + L2.  A step is one forward
over the whole batch.  The same line then carries the other metrics the
benchmark names, each measured in the same run:

  * "qwen3": embeddings/s of the Qwen3-Embedding-0.6B shape (28 layers, GQA
    16:8, BF16), 2048 sequences per rank of 128..512 tokens + EOS;
  * "ivf_build": seconds to build the IVF index over 3.27M x 384 rows
    (k 4096, 20 Lloyd iterations + assign-all), rows sharded over the ranks;
  * "query": p50 ms of one short MiniLM query (10 ids) + IVF top-10 over
    that index, end to end through the host API (rank 0);
  * "inproc_split" (N > 1): rank 0 drives all N devices through one
    ec_embed_batch call (the library's length-balanced split, the path an
    SBCL host takes) while the other ranks wait on the host.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload minilm|bert-base|mpnet|qwen3|gemma|ivf|query|search|tokenize]
                    [--headline-only]

N > 1 is launched by torch.distributed.run, one process per GPU: every rank
embeds its own shard (weak scaling, no data-path collective; the shards are
dealt from one seeded pool so every rank gets the same token count), and
`value` is all ranks' sequences / the slowest rank's device time.

--impl reference times the reference algorithm on the host cores (the Lisp
cannot run here, so its CPU restatement in oracle/ stands in, threads = all
host cores, one sequence per thread as embed.lisp does) on the headline
workload.
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
IVF_TIMED_BUILDS = 3  # timed IVF builds per run; the median is the value
IVF_ROWS = [IVF_N]  # rows of the IVF workload (--ivf-rows: a smaller build for profiling)
PRECISION = ("bf16 tensor-core GEMM/attention, fp32 accumulate, fp32 norms; residual between "
             "sublayers: the LayerNorm's bf16 output (BERT/MPNet), fp32 (Qwen3, Gemma)")


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
    p.add_argument("--headline-only", action="store_true",
                   help="default workload: the MiniLM headline alone")
    p.add_argument("--ivf-rows", type=int, default=IVF_N,
                   help="ivf workload: rows of the corpus (a smaller build for profiling)")
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


class Ranks:
    """Rank layout of one run.  Host-side exchanges (barriers, the max of
    device times, the NCCL id of the library's k-means communicator) go
    through a gloo group, so a rank waiting on another runs no GPU kernel."""

    def __init__(self):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.gloo = None

    def setup(self):
        import torch
        torch.cuda.set_device(self.local_rank)
        if self.world > 1:
            import torch.distributed as dist
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                    device_id=torch.device("cuda", self.local_rank))
            self.gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=900))
        phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
        self.smi_index = (phys[self.local_rank] if len(phys) > self.local_rank and phys[self.local_rank]
                          else self.local_rank)
        return self

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.gloo)

    def max(self, *vals):
        if self.world == 1:
            return vals if len(vals) > 1 else vals[0]
        import torch
        import torch.distributed as dist
        t = torch.tensor(vals, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.gloo)
        out = tuple(float(v) for v in t)
        return out if len(out) > 1 else out[0]

    def sum(self, val):
        if self.world == 1:
            return val
        import torch
        import torch.distributed as dist
        t = torch.tensor([val], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.gloo)
        return float(t[0])

    def bcast_bytes(self, data, n):
        if self.world == 1:
            return data
        import torch
        import torch.distributed as dist
        t = torch.zeros(n, dtype=torch.uint8)
        if self.rank == 0:
            t[:] = torch.frombuffer(bytearray(data), dtype=torch.uint8)
        dist.broadcast(t, 0, group=self.gloo)
        return bytes(t.numpy())

    def finish(self):
        if self.world > 1:
            import torch.distributed as dist
            self.barrier()
            dist.destroy_process_group()


def synth_root():
    return os.environ.get("EC_SYNTH_DIR", "/tmp/ec_synth")


def shared_model_dir(shape, seed, R):
    """The seeded model directory, written once per host (local rank 0) and
    read by every rank."""
    from embedcuda import synth
    if R.local_rank == 0:
        d = synth.build_model_dir(shape, seed, synth_root())
    R.barrier()
    if R.local_rank != 0:
        d = synth.build_model_dir(shape, seed, synth_root())
    return d


def workload_config(workload, world, tokens_rank0):
    """The `config` object of a line: the workload alone (both arms)."""
    shape_name, _, nseq, desc = WORKLOADS[workload]
    return {"workload": shape_name, "description": desc, "sequences_per_rank": nseq,
            "tokens_per_rank": tokens_rank0, "parallelism": f"dp{world} (sequence shards)"}


def rank_inputs(shape_name, nseq, seed, rank, world):
    """This rank's sequences.  One rank: the workload's `nseq` sequences.
    N ranks: a pool of N * nseq sequences from the same seed, sorted by
    length and dealt in a snake order, so every rank gets nseq sequences and
    (nearly) the same token count."""
    from embedcuda import synth
    if world == 1:
        return synth.make_inputs(shape_name, nseq, seed)
    ids, offs = synth.make_inputs(shape_name, nseq * world, seed)
    lens = np.diff(offs)
    order = np.argsort(-lens, kind="stable")
    pos = np.arange(order.size)
    blk, r = pos // world, pos % world
    owner = np.where(blk % 2 == 0, r, world - 1 - r)
    mine = np.sort(order[owner == rank])
    chunks = [ids[offs[i]:offs[i + 1]] for i in mine]
    o = np.zeros(len(mine) + 1, np.int64)
    o[1:] = np.cumsum([len(c) for c in chunks])
    return np.concatenate(chunks).astype(np.int32), o


def embed_measure(R, workload, steps, warmup, profile=True, e2e_steps=None):
    """Device-timed forward steps of one embedding workload on this rank's
    shard (inputs resident in HBM, L2 flushed between steps), then the same
    batch end to end through ec_embed_batch with host buffers.  Returns
    rank 0's dict (None elsewhere)."""
    import ctypes as C
    import torch
    from embedcuda import _lib, model, synth
    shape_name, seed, nseq, desc = WORKLOADS[workload]
    shape = synth.SHAPES[shape_name]
    mdir = shared_model_dir(shape, seed, R)
    _lib.init([R.local_rank])
    model.load_model(mdir)
    dim = model.dim()
    ids, offsets = rank_inputs(shape_name, nseq, seed, R.rank, R.world)
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

    for _ in range(warmup):
        flush.zero_()
        step_device()
    torch.cuda.synchronize()
    R.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    with ClockSampler(R.smi_index) as clk:
        for i in range(steps):
            flush.zero_()
            ev[i][0].record(stream)
            step_device()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    R.barrier()
    launches = None
    prof = {}
    if profile:
        # per-kernel-class times: the same steps again with a CUDA event
        # pair around every launch (the events cost 2-3% of a step, so the
        # throughput above is taken without them)
        L.ecdbg_profile(1)
        for i in range(steps):
            flush.zero_()
            step_device()
        torch.cuda.synchronize()
        launches = int(L.ecdbg_launches())
        L.ecdbg_profile(0)
        for cls in ("gemm", "attention", "rows"):
            v = [C.c_double(), C.c_double(), C.c_double(), C.c_longlong()]
            L.ecdbg_profile_read(cls.encode(), *[C.byref(x) for x in v])
            prof[cls] = {"ms": v[0].value, "flops": v[1].value, "bytes": v[2].value,
                         "launches": v[3].value}
    ms = sum(a.elapsed_time(b) for a, b in ev)
    clocks = clk.summary()
    # end to end through the host API: ids from pinned host memory in,
    # embeddings back to host memory, each step
    h_ids = torch.from_numpy(ids).pin_memory().numpy()
    h_out = np.empty((nseq, dim), np.float32)
    for _ in range(2):
        model.embed_batch(h_ids, offsets, out=h_out)
    e2e_s = 0.0
    ne2e = e2e_steps or steps
    for _ in range(ne2e):
        flush.zero_()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        model.embed_batch(h_ids, offsets, out=h_out)
        e2e_s += time.perf_counter() - t0
    nblk = int(np.sum((np.diff(offsets) + 63) // 64))
    h2d = T * 4 + (nseq + 1) * 4 + nblk * 8
    d2h = nseq * dim * 4
    ms, e2e_per = R.max(ms, e2e_s / ne2e)
    tokens_all = R.sum(float(T))
    if R.rank != 0:
        return None
    peaks, src = measured_peaks()
    peak = peaks.get("bf16_tflops")
    out = {
        "value": R.world * nseq * steps / (ms * 1e-3), "unit": "embeddings/s",
        "ms_per_step": ms / steps, "steps": steps, "warmup": warmup,
        "config": workload_config(workload, R.world, T),
        "tokens_all_ranks": int(tokens_all),
        "l2": "flushed (256 MB write) between timed steps",
        "e2e": {"value": R.world * nseq / e2e_per, "unit": "embeddings/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "timing": "host wall clock around the synchronous ec_embed_batch call"},
        "clocks": clocks,
        "step_tflops": flops_step * steps / (ms * 1e-3) / 1e12,
        "model_dir": mdir, "ids": ids, "offsets": offsets,
    }
    out["step_frac_of_peak"] = out["step_tflops"] / peak if peak else None
    if profile:
        g = prof["gemm"]
        achieved = g["flops"] / (g["ms"] * 1e-3) / 1e12 if g["ms"] > 0 else None
        out["roofline"] = {
            "bound": "tensor", "kernel": "gemm_tn_bf16 / gemm_ln (all GEMM launches)",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": (achieved / peak) if achieved and peak else None,
            "traffic": profile_traffic(f"gemm_{workload}"),
            "peak_source": f"{src} bf16_tflops (burst: GEMM launches of 0.1-1 ms)",
            "timing": "CUDA events on the launching stream around each GEMM launch, in a "
                      "second pass of the same steps right after the timed one",
            "step_tflops": out["step_tflops"], "step_frac_of_peak": out["step_frac_of_peak"]}
        out["kernel_classes"] = prof
        out["gpu_launches"] = launches
    return out


def qwen3_cpu_baseline(model_dir, ids, offsets, seconds):
    """The oracle's llama.lisp forward on all host cores, one sequence per
    thread, over the first 2 of the 28 layers; the time is scaled by 28 / 2
    (every layer does the same work; the embedding gather and final norm are
    negligible)."""
    from oracle import oracle
    om = oracle.OracleModel(model_dir)
    full = om.m.layers
    om.m.layers = 2
    threads = os.cpu_count() or 1
    nseq = len(offsets) - 1
    done, el, s = 0, 0.0, 0
    while el < seconds and s < nseq:
        b1 = min(nseq, s + threads)
        sub = offsets[s:b1 + 1] - offsets[s]
        t0 = time.perf_counter()
        om.embed_batch(ids[offsets[s]:offsets[b1]], sub, threads=threads)
        el += time.perf_counter() - t0
        done += b1 - s
        s = b1
    om.m.layers = full
    scale = full / 2.0
    return {"value": done / (el * scale), "unit": "embeddings/s", "cores": threads, "kind": "port",
            "sample": f"{done} of the workload's sequences through 2 of {full} layers in {el:.1f} s "
                      f"({threads} threads, one sequence per thread), time scaled by {scale:g}"}


def ivf_corpus_host(R):
    """The IVF workload (generated on this rank's GPU with a fixed seed, the
    same on every rank) copied to host memory, and its training permutation."""
    import torch
    x_dev, perm = ivf_corpus_torch(IVF_ROWS[0], IVF_D, IVF_K, IVF_SEED, "cuda")
    x = x_dev.cpu().numpy()
    perm = perm.cpu().numpy().astype(np.int64)
    del x_dev
    torch.cuda.empty_cache()
    return x, perm


def ivf_build_measure(R, x, perm):
    """IVF build seconds: 20 Lloyd iterations over all 3.27M rows (k 4096,
    init = the first k rows of a seeded permutation, ann.lisp:83-86) with the
    rows sharded over the ranks in sample order (the sums chained from rank
    to rank over NCCL, so the centroids equal one device's bit for bit), then
    the inverted lists of each shard (ann::assign-all), both in one
    ec_ann_build call.  Inputs start in host memory; the timed region
    includes their upload.  Returns (rank 0's dict,
    centroids)."""
    import ctypes as C
    import torch
    from embedcuda import _lib, ann
    n = len(x)
    per = (n + R.world - 1) // R.world
    j0, j1 = per * R.rank, min(n, per * (R.rank + 1))
    mine = perm[j0:j1]
    x_local = np.ascontiguousarray(x[mine])  # this rank's training rows, in sample order
    init = np.ascontiguousarray(x[perm[:IVF_K]])
    _lib.init([R.local_rank])
    L = _lib.lib()
    if R.world > 1 and not getattr(R, "comm_ready", False):
        idn = L.ec_comm_id_size()
        idbuf = C.create_string_buffer(idn)
        if R.rank == 0:
            _lib.check(L.ec_comm_get_id(idbuf), "comm id")
        raw = R.bcast_bytes(idbuf.raw, idn)
        _lib.check(L.ec_comm_init(R.rank, R.world, C.create_string_buffer(raw, idn)), "comm init")
        R.comm_ready = True
    local_sample = np.arange(len(x_local), dtype=np.int64)
    # warm-up: the same build with one iteration (module load, NCCL channels,
    # and the first device allocations of these sizes, whose cost varied from
    # milliseconds to ~1 s between processes on the same box)
    ann.build(x_local, local_sample, IVF_K, 1, init=init)
    torch.cuda.synchronize()
    R.barrier()
    L.ecdbg_profile(1)
    L.ecdbg_assign_rows(None, None, 1)
    # three timed builds, the median reported (single builds on these shared
    # hosts were occasionally slowed 2-3x by host-side stalls)
    builds = []
    with ClockSampler(R.smi_index) as clk:
        for _ in range(IVF_TIMED_BUILDS):
            R.barrier()
            t0 = time.perf_counter()
            cent, counts, lists = ann.build(x_local, local_sample, IVF_K, IVF_ITERS, init=init)
            builds.append(time.perf_counter() - t0)
    v = [C.c_double(), C.c_double(), C.c_double(), C.c_longlong()]
    L.ecdbg_profile_read(b"gemm", *[C.byref(z) for z in v])
    g_ms, g_flops, g_launches = v[0].value, v[1].value, v[3].value
    L.ecdbg_profile_read(b"rows", *[C.byref(z) for z in v])
    r_ms = v[0].value
    L.ecdbg_profile(0)
    tc_rows, ex_rows = C.c_longlong(), C.c_longlong()
    L.ecdbg_assign_rows(C.byref(tc_rows), C.byref(ex_rows), 0)
    builds = [R.max(b) for b in builds]
    t_all = float(np.median(builds))
    if R.rank != 0:
        return None, cent
    peaks, src = measured_peaks()
    achieved = g_flops / (g_ms * 1e-3) / 1e12 if g_ms > 0 else None
    peak = peaks.get("bf16_tflops")
    flops = 2.0 * n * IVF_K * IVF_D * (IVF_ITERS + 1)  # one build
    out = {"value": t_all, "unit": "s", "higher_is_better": False, "scaling": "strong",
           "n_gpus": R.world, "dtype": "f32 (bf16 tensor-core scores, exact re-check)",
           "config": {"workload": f"ivf-{n / 1e6:g}Mx{IVF_D}", "n": n, "dim": IVF_D, "k": IVF_K,
                      "iters": IVF_ITERS, "sample": "all rows, seeded permutation",
                      "parallelism": f"rows sharded over {R.world} GPU(s) in sample order",
                      "exchange": "per-cluster sums chained rank to rank (NCCL send/recv), "
                                  "centroids broadcast" if R.world > 1 else "none"},
           "api": "ec_ann_build (kmeans + assign-all, rows uploaded once)",
           "achieved_tflops": flops / t_all / 1e12,
           "roofline": {"bound": "tensor",
                        "kernel": "gemm_tn_bf16_kernel<256, kEpiArgCand> (assignment scores, rank 0)",
                        "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak if achieved and peak else None, "traffic": None,
                        "launches": g_launches, "assign_gemm_ms": g_ms, "assign_reduce_ms": r_ms,
                        "peak_source": f"{src} bf16_tflops (burst)"},
           "builds_s": builds,
           "assign_rows": {"tensor_core": tc_rows.value // len(builds),
                           "exact_scan": ex_rows.value // len(builds)},
           "clocks": clk.summary(),
           "note": "assignments and centroids bit-identical to ann.lisp's sequential "
                   "single-float arithmetic at any rank count"}
    return out, cent


def ivf_cpu_baseline(x, perm, seconds):
    """ann::kmeans on the host cores, timed on a sample and extrapolated: the
    assignment pass one row and one centroid at a time on all threads
    (ann.lisp:90-105) over a slice of rows, and the serial update
    (ann.lisp:107-122) over a slice; build = 21 assignment passes + 20
    updates over all 3.27M rows."""
    from oracle import oracle
    threads = os.cpu_count() or 1
    init = np.ascontiguousarray(x[perm[:IVF_K]])
    rows = 2048
    el_a, done_a = 0.0, 0
    while el_a < 0.6 * seconds and done_a < 64 * rows:
        sl = perm[done_a:done_a + rows]
        t0 = time.perf_counter()
        a = oracle.assign_scalar(x, init, rows=sl, threads=threads)
        el_a += time.perf_counter() - t0
        done_a += rows
    sl = perm[:200000]
    # the serial update's cost does not depend on which cluster a row joins
    a = np.random.default_rng(0).integers(0, IVF_K, len(sl)).astype(np.int32)
    t0 = time.perf_counter()
    oracle.kmeans_update(x, sl, a, init)
    el_u = time.perf_counter() - t0
    n = len(x)
    t_assign = n * el_a / done_a
    t_update = n * el_u / len(sl)
    total = (IVF_ITERS + 1) * t_assign + IVF_ITERS * t_update
    return {"value": total, "unit": "s", "cores": threads, "kind": "port",
            "sample": f"assignment of {done_a} rows on {threads} threads in {el_a:.1f} s and the "
                      f"serial update of {len(sl)} rows in {el_u:.2f} s, extrapolated to "
                      f"{IVF_ITERS + 1} passes and {IVF_ITERS} updates of {n} rows"}


def query_measure(R, x, cent, nq, warmup):
    """p50 ms of one short MiniLM query end to end through the host API
    (rank 0, one GPU): ec_embed_batch of 10 token ids, then ec_ivf_search
    top-10 with nprobe 32 over the 3.27M x 384 IVF index (kb:kb-search after
    the text part)."""
    from embedcuda import ann, kb, model, synth
    counts, lists = ann.assign_all(x, cent)
    kb.load_index(x, (cent, counts, lists))
    model.load_model(synth.build_model_dir(synth.MINILM, 0, synth_root()))
    rng = np.random.default_rng(7)
    times = []
    for i in range(nq + warmup):
        ids = np.concatenate([[101], rng.integers(1000, 30522, 8), [102]]).astype(np.int32)
        t0 = time.perf_counter()
        q = model.embed(ids)
        kb.search_ivf(q, SEARCH_TOPK, nprobe=SEARCH_NPROBE)
        el = time.perf_counter() - t0
        if i >= warmup:
            times.append(el)
    return {"value": 1000 * float(np.median(times)), "unit": "ms", "higher_is_better": False,
            "n_gpus": 1, "queries": nq,
            "p90_ms": 1000 * float(np.percentile(times, 90)),
            "min_ms": 1000 * float(np.min(times)),
            "config": {"workload": "minilm-l6 query (10 ids) + ivf top-10 nprobe 32 over 3.27Mx384"},
            "counts": counts, "lists": lists}


def query_cpu_baseline(x, cent, counts, lists, nq=11):
    """The oracle on the host: bert.lisp's forward of the same 10-id queries
    on one thread, then kb::top-k-ivf (nprobe 32, top-10); p50 of nq."""
    from embedcuda import synth
    from oracle import oracle
    om = oracle.OracleModel(synth.build_model_dir(synth.MINILM, 0, synth_root()))
    rng = np.random.default_rng(7)
    times = []
    for _ in range(nq):
        ids = np.concatenate([[101], rng.integers(1000, 30522, 8), [102]]).astype(np.int32)
        t0 = time.perf_counter()
        q = om.embed(ids)
        oracle.top_k_ivf(x, cent, counts, lists, SEARCH_NPROBE, q, SEARCH_TOPK)
        times.append(time.perf_counter() - t0)
    return {"value": 1000 * float(np.median(times)), "unit": "ms", "cores": 1, "kind": "port",
            "sample": f"p50 of {nq} queries (oracle embed on one thread + kb::top-k-ivf scan)"}


def inproc_split_measure(R, steps):
    """N > 1, rank 0 only: ec_init on all N devices and one ec_embed_batch
    per step over N x 1024 MiniLM sequences from host buffers (the library
    sorts them by length, deals them to the least-loaded device and scatters
    the rows back in input order).  Host wall clock per call."""
    import torch
    from embedcuda import _lib, model, synth
    if torch.cuda.device_count() < R.world:
        return {"skipped": f"{torch.cuda.device_count()} devices visible to rank 0"}
    shape_name, seed, nseq, _ = WORKLOADS["minilm"]
    _lib.init(list(range(R.world)))
    model.load_model(synth.build_model_dir(synth.SHAPES[shape_name], seed, synth_root()))
    ids, offs = synth.make_inputs(shape_name, nseq * R.world, seed)
    h_ids = torch.from_numpy(ids).pin_memory().numpy()
    out = np.empty((len(offs) - 1, model.dim()), np.float32)
    for _ in range(3):
        model.embed_batch(h_ids, offs, out=out)
    t = []
    for _ in range(steps):
        t0 = time.perf_counter()
        model.embed_batch(h_ids, offs, out=out)
        t.append(time.perf_counter() - t0)
    el = sum(t) / len(t)
    _lib.shutdown()
    return {"value": (len(offs) - 1) / el, "unit": "embeddings/s", "n_gpus": R.world,
            "ms_per_step": 1000 * el, "steps": steps, "sequences": len(offs) - 1,
            "tokens": int(offs[-1]),
            "timing": "host wall clock around one ec_embed_batch call over all devices "
                      "(host ids in, host embeddings out)"}


def run_default(args):
    """The headline (MiniLM) line with the other metrics as sub-results."""
    R = Ranks().setup()
    from embedcuda import _lib
    head = embed_measure(R, "minilm", args.steps, args.warmup)
    out = None
    if R.rank == 0:
        out = {"metric": "embeddings/sec", "value": head["value"], "unit": "embeddings/s",
               "n_gpus": R.world, "steps": args.steps, "warmup": args.warmup,
               "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (seeded ids and N(0,0.02) weights of the named shape)",
               "config": head["config"], "precision": PRECISION, "l2": head["l2"],
               "tokens_all_ranks": head["tokens_all_ranks"],
               "e2e": head["e2e"], "roofline": head["roofline"],
               "kernel_classes": head["kernel_classes"], "gpu_launches": head["gpu_launches"],
               "clocks": head["clocks"]}
    extras = not args.headline_only
    if extras:
        q = embed_measure(R, "qwen3", 3, 3, profile=True, e2e_steps=2)
        if R.rank == 0:
            q.pop("ids"), q.pop("offsets"), q.pop("model_dir")
            q.pop("kernel_classes", None), q.pop("gpu_launches", None)
            out["qwen3"] = q
        x, perm = ivf_corpus_host(R)
        ivf, cent = ivf_build_measure(R, x, perm)
        if R.rank == 0:
            out["ivf_build"] = ivf
            qm = query_measure(R, x, cent, 101, 5)
            counts, lists = qm.pop("counts"), qm.pop("lists")
            out["query"] = qm
        # every rank closes the library (and the k-means communicator) together
        R.barrier()
        _lib.shutdown()
        R.barrier()
        if R.world > 1:
            if R.rank == 0:
                out["inproc_split"] = inproc_split_measure(R, args.steps)
            R.barrier()
    if R.rank == 0 and R.world == 1 and not args.no_cpu_baseline:
        try:
            out["cpu_baseline"] = cpu_baseline(head["model_dir"], head["ids"], head["offsets"],
                                               args.cpu_seconds)
        except Exception as e:  # the baseline must not sink the GPU number
            out["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        if extras:
            for key, fn in (
                    ("qwen3", lambda: qwen3_cpu_baseline(
                        _qwen_dir(), *_qwen_inputs(), args.cpu_seconds)),
                    ("ivf_build", lambda: ivf_cpu_baseline(x, perm, args.cpu_seconds)),
                    ("query", lambda: query_cpu_baseline(x, cent, counts, lists))):
                try:
                    out[key]["cpu_baseline"] = fn()
                except Exception as e:
                    out[key]["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
    if R.rank == 0:
        print(json.dumps(out), flush=True)
    _lib.shutdown()
    R.finish()
    return 0


def _qwen_dir():
    from embedcuda import synth
    shape_name, seed, _, _ = WORKLOADS["qwen3"]
    return synth.build_model_dir(synth.SHAPES[shape_name], seed, synth_root())


def _qwen_inputs():
    from embedcuda import synth
    shape_name, seed, nseq, _ = WORKLOADS["qwen3"]
    return synth.make_inputs(shape_name, nseq, seed)


def run_single_embed(args):
    """--workload bert-base | mpnet | qwen3 | gemma: that workload alone."""
    R = Ranks().setup()
    from embedcuda import _lib
    r = embed_measure(R, args.workload, args.steps, args.warmup)
    if R.rank == 0:
        out = {"metric": "embeddings/sec", "value": r["value"], "unit": "embeddings/s",
               "n_gpus": R.world, "steps": args.steps, "warmup": args.warmup,
               "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic (seeded ids and N(0,0.02) weights of the named shape)",
               "config": r["config"], "precision": PRECISION, "l2": r["l2"], "e2e": r["e2e"],
               "roofline": r["roofline"], "kernel_classes": r["kernel_classes"],
               "gpu_launches": r["gpu_launches"], "clocks": r["clocks"]}
        if R.world == 1 and not args.no_cpu_baseline:
            try:
                if args.workload == "qwen3":
                    out["cpu_baseline"] = qwen3_cpu_baseline(r["model_dir"], r["ids"], r["offsets"],
                                                             args.cpu_seconds)
                else:
                    out["cpu_baseline"] = cpu_baseline(r["model_dir"], r["ids"], r["offsets"],
                                                       args.cpu_seconds)
            except Exception as e:
                out["cpu_baseline"] = {"value": None, "error": str(e)[:200]}
        print(json.dumps(out), flush=True)
    _lib.shutdown()
    R.finish()
    return 0


def run_ivf(args):
    """--workload ivf: the IVF build alone (its own line)."""
    R = Ranks().setup()
    from embedcuda import _lib
    x, perm = ivf_corpus_host(R)
    ivf, _ = ivf_build_measure(R, x, perm)
    if R.rank == 0:
        ivf.update(metric="IVF build s", steps=1, warmup=1, ms_per_step=1000 * ivf["value"],
                   vs_baseline=None, data="synthetic")
        if R.world == 1 and not args.no_cpu_baseline:
            ivf["cpu_baseline"] = ivf_cpu_baseline(x, perm, args.cpu_seconds)
        print(json.dumps(ivf), flush=True)
    _lib.shutdown()
    R.finish()
    return 0


def run_query(args):
    """--workload query: the p50 query alone (rank 0)."""
    R = Ranks().setup()
    from embedcuda import _lib, ann
    if R.rank == 0:
        x, perm = ivf_corpus_host(R)
        _lib.init([R.local_rank])
        cent = ann.kmeans(x, perm, IVF_K, IVF_ITERS)
        qm = query_measure(R, x, cent, 101, args.warmup)
        counts, lists = qm.pop("counts"), qm.pop("lists")
        qm.update(metric="p50 query ms", steps=101, warmup=args.warmup, ms_per_step=qm["value"],
                  vs_baseline=None, data="synthetic", dtype="bf16+f32", scaling="none")
        if not args.no_cpu_baseline:
            qm["cpu_baseline"] = query_cpu_baseline(x, cent, counts, lists)
        print(json.dumps(qm), flush=True)
    _lib.shutdown()
    R.finish()
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
    cent, counts, lists = ann.build(x, perm, k, IVF_ITERS)
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


def run_reference(args, rank, world):
    """--impl reference: the oracle port of the reference's CPU path on the
    host cores, on the headline workload (rank 0's shard), one sequence per
    thread in batches of `threads` (embed.lisp:88-105); rank 0 alone."""
    if rank != 0:
        return 0
    from embedcuda import synth
    workload = args.workload if args.workload in WORKLOADS else "minilm"
    shape_name, seed, nseq, desc = WORKLOADS[workload]
    shape = synth.SHAPES[shape_name]
    d = synth.build_model_dir(shape, seed, synth_root())
    ids, offsets = rank_inputs(shape_name, nseq, seed, 0, world)
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
        "config": workload_config(workload, world, int(offsets[-1])),
        "cpu_baseline": {"value": value, "unit": "embeddings/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps x {threads} sequences of the workload "
                                   "(one sequence per thread); SBCL absent, the C restatement "
                                   "of bert.lisp / llama.lisp stands in"},
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
    IVF_ROWS[0] = args.ivf_rows
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if args.workload in ("ivf", "query", "search", "tokenize"):
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "reference arm is timed for the embedding workloads only"}))
            return 0
        return run_reference(args, rank, world)
    # NCCL's version banner goes to stdout; the benchmark prints one JSON line
    if not os.environ.get("EC_KEEP_NCCL_DEBUG"):
        os.environ["NCCL_DEBUG"] = "WARN"
    if args.workload == "minilm":
        return run_default(args)
    if args.workload in WORKLOADS:
        return run_single_embed(args)
    if args.workload == "ivf":
        return run_ivf(args)
    if args.workload == "query":
        return run_query(args)
    if args.workload == "search":
        return run_search(args, rank, local_rank)
    return run_tokenize(args, rank)


if __name__ == "__main__":
    sys.exit(main())
