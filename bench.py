"""Benchmark of the quantized flat-scan path (default).

Default workload (the largest configuration and the
one with 1/2/4/8-GPU numbers): 1-bit codes, N=10,000,000 rows, d=768 (P=1024,
128 B of sign bits per row), a 1,024-centre Gaussian mixture (sigma 0.3),
L2-normalised, seed 4; queryBatch of 1,000 queries from the same mixture;
cosine; k=100 with a 10x oversample (F=1,000) re-ranked in exact fp32.  The
rows are split evenly across the GPUs (one process per GPU, NCCL); a step is
the whole batch: prep, the tcgen05 kind::i8 GEMM + select rounds, (N > 1) one
all-gather of the shards' candidate keys and the global F-th key, the exact
re-rank of each shard's members of the global best F, one all-gather of the
shard records and the merge.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config c1|c2|c3|c4|c5]

value  : queries/s of the whole job, inputs resident in HBM (device timed with
         CUDA events on the launch stream, max over ranks).
e2e    : the same through the public API with host buffers: per step a pinned
         H2D of the batch, the search, a D2H of the results.
roofline: the dominant kernel (the GEMM for the batched configs), its
         algorithmic int8 ops over its own event-timed duration.
--impl reference: the reference's CPU path for the workload -- the WASM-SIMD
         exact fp32 flat scan + topK (src/fallback/kernel.wat, cpu.ts:66-88),
         restated in C (oracle/), one CpuIndex per row shard of at most
         3.5 GiB merged with mergePartials (gpuTopk.ts:160-189), on all host
         threads, a bounded query sample per step.
Single-query configs (c1, c2) keep their own flow (see run_single).
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_ROWS, DIM, N_QUERIES, K, RERANK_FACTOR, SEED = 100_000, 768, 1000, 10, 4, 2
METRIC = "queries/sec at fixed recall@10 (TurboQuant int8 flat scan, N=100k, d=768, k=10, F=40)"
BITS, WORKLOAD = 8, "BASELINE config 2: TurboQuant int8 flat, single-query scans"
# Single-query configurations: queries issued one at a time against one index
# (replicated round-robin so that every scan reads a corpus evicted from L2).
SINGLE = {
    "c2": dict(n=100_000, dim=768, nq=1000, k=10, rf=4, seed=2, bits=8, metric=METRIC,
               workload="BASELINE config 2: TurboQuant int8 flat, single-query scans"),
    "c1": dict(n=20_000, dim=384, nq=100, k=10, rf=1, seed=0, bits=0,
               metric="queries/sec at recall@10 = 1.0 (exact fp32 flat cosine scan, N=20k, d=384, k=10)",
               workload="BASELINE config 1: exact fp32 flat scan (the reference CPU path's WASM-SIMD f32 "
                        "arithmetic), single-query scans"),
}


def _use_single(name):
    """Point the single-query flow at configuration `name`."""
    global N_ROWS, DIM, N_QUERIES, K, RERANK_FACTOR, SEED, METRIC, BITS, WORKLOAD
    c = SINGLE[name]
    N_ROWS, DIM, N_QUERIES, K, RERANK_FACTOR, SEED = c["n"], c["dim"], c["nq"], c["k"], c["rf"], c["seed"]
    METRIC, BITS, WORKLOAD = c["metric"], c["bits"], c["workload"]
UNIT = "queries/s"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _measured_traffic():
    """DRAM bytes of the dominant kernels from ncu captures (profiles/dram_traffic.json)."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    return json.load(open(p)) if os.path.exists(p) else {}


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"])
    return 1590.0


def make_data(torch, device, seed, n, dim):
    """Seeded counter-based (Philox) N(0,1) rows on the GPU, L2-normalised in f64."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((n, dim), generator=g, device=device, dtype=torch.float32)
    x64 = x.double()
    norm = x64.pow(2).sum(1, keepdim=True).sqrt()
    return (x64 / norm).float().contiguous()


class Clocks:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_qps(corpus_np, queries_np, steps, warmup, per_step, threads):
    """The reference CPU path (WASM-SIMD fp32 scan + topK), restated in C."""
    from oracle import oracle as O

    nq = queries_np.shape[0]
    times = []
    for s in range(warmup + steps):
        sel = queries_np[(np.arange(per_step) + s * per_step) % nq]
        t0 = time.perf_counter()
        O.cpu_index_query_batch(corpus_np, DIM, sel, K, threads=threads)
        dt = time.perf_counter() - t0
        if s >= warmup:
            times.append(dt)
    return per_step * len(times) / sum(times), per_step


def recall_at_10(torch, corpus, queries, got_rows):
    exact = (queries.double() @ corpus.double().T).topk(K, dim=1).indices.cpu().numpy()
    hit = 0
    for i in range(exact.shape[0]):
        hit += len(set(exact[i].tolist()) & set(got_rows[i].tolist()))
    return hit / (exact.shape[0] * K)


# Row-sharded configurations: rows split over the ranks,
# one all-gather of shard records per step, merged on every rank.
SHARDED = {
    "c3": dict(bits=4, n=1_000_000, dim=384, kind="mixture", seed=3, nq=10_000, metric="dot", k=10, rf=8,
               scoring="int", workload="BASELINE config 3: TurboQuant int4, queryBatch of 10,000, row-sharded"),
    "c4": dict(bits=1, n=10_000_000, dim=768, kind="mixture", seed=4, nq=1000, metric="cosine", k=100, rf=10,
               scoring="int", workload="BASELINE config 4: 1-bit codes (int8 query x +-1 codes, the popc-equivalent "
                                       "integer dot), queryBatch of 1,000, row-sharded"),
    "c5": dict(bits=8, n=50_000_000, dim=128, kind="iid", seed=5, nq=4096, metric="cosine", k=10, rf=4,
               scoring="int", filter=True,
               workload="BASELINE config 5: TurboQuant int8, queryBatch of 4,096, metadata filter "
                        "{lang: <most common>, year: {$gte: 2020}} as a device predicate + score mask, row-sharded"),
}


def _init_dist(torch):
    """One process per GPU over NCCL; a one-rank group when not under torchrun."""
    import socket
    from datetime import timedelta

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1 and "MASTER_PORT" not in os.environ:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            os.environ["MASTER_PORT"] = str(s.getsockname()[1])
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return dist, world, rank, local


def _exact_top10(torch, dist, x, lo, qs, chunk=1 << 20, keep=None):
    """Global exact fp32 top-10 (rows) of qs over the sharded corpus (rows
    with keep False excluded)."""
    best_v = torch.full((qs.shape[0], 10), -float("inf"), device=qs.device)
    best_r = torch.zeros((qs.shape[0], 10), dtype=torch.int64, device=qs.device)
    for a in range(0, x.shape[0], chunk):
        s = qs @ x[a:a + chunk].T
        if keep is not None:
            s[:, ~keep[a:a + chunk]] = -float("inf")
        v, r = s.topk(min(10, s.shape[1]), dim=1)
        v = torch.cat([best_v, v], 1)
        r = torch.cat([best_r, r + lo + a], 1)
        best_v, i = v.topk(10, dim=1)
        best_r = r.gather(1, i)
    world = dist.get_world_size()
    gv = [torch.empty_like(best_v) for _ in range(world)]
    gr = [torch.empty_like(best_r) for _ in range(world)]
    dist.all_gather(gv, best_v)
    dist.all_gather(gr, best_r)
    v, r = torch.cat(gv, 1), torch.cat(gr, 1)
    _, i = v.topk(10, dim=1)
    return r.gather(1, i).cpu().numpy()


def _c5_keep(torch, dev, cfg, lo, hi):
    """Config-5 metadata of rows [lo, hi) as device columns, and the filter."""
    from browservec_b200 import datagen
    from browservec_b200.filter import DeviceColumns

    year, lang = datagen.metadata(torch, dev, cfg["seed"], lo, hi)
    dc = DeviceColumns(dev)
    dc.set_number_column("year", year)
    dc.set_string_column("lang", lang, [f"lang{i}" for i in range(8)])
    return dc, {"lang": "lang0", "year": {"$gte": 2020}}


def _unpack(torch, words, n):
    bits = (words.view(-1, 1) >> torch.arange(32, device=words.device, dtype=torch.int32)) & 1
    return bits.reshape(-1)[:n].bool()


SHARD_BYTES = int(3.5 * 2 ** 30)  # one wasm32 CpuIndex holds at most ~4 GiB of corpus (cpu.ts:97-104)


def _host_shards(torch, dev, cfg, threads, x=None):
    """The corpus in host memory as row shards of at most 3.5 GiB, at least one
    per host thread, for the reference CPU path (one CpuIndex per shard).  A
    filtered configuration keeps only the rows its filter passes (with their
    global rows).  x: the corpus already on this device (else generated)."""
    from browservec_b200 import datagen

    n, dim = cfg["n"], cfg["dim"]
    step = 1 << 20
    rowmap = None
    if cfg.get("filter"):
        parts, maps = [], []
        for a in range(0, n, step):
            b = min(n, a + step)
            xs = x[a:b] if x is not None else datagen.rows(torch, dev, cfg["kind"], cfg["seed"], a, b, dim)
            dc, flt = _c5_keep(torch, dev, cfg, a, b)
            keep = _unpack(torch, dc.mask(flt), b - a)
            parts.append(xs[keep].cpu().numpy())
            maps.append((torch.nonzero(keep).squeeze(1) + a).cpu().numpy().astype(np.uint32))
        host = np.concatenate(parts)
        rowmap = np.concatenate(maps)
    else:
        host = np.empty((n, dim), np.float32)
        ht = torch.from_numpy(host)
        for a in range(0, n, step):
            b = min(n, a + step)
            xs = x[a:b] if x is not None else datagen.rows(torch, dev, cfg["kind"], cfg["seed"], a, b, dim)
            ht[a:b].copy_(xs)
    m = host.shape[0]
    per = max(1, min(SHARD_BYTES // (dim * 4), -(-m // threads)))
    shards, bases, maps = [], [], []
    for a in range(0, m, per):
        b = min(m, a + per)
        shards.append(host[a:b])
        bases.append(a if rowmap is None else 0)
        maps.append(None if rowmap is None else rowmap[a:b])
    return shards, bases, (maps if rowmap is not None else None)


def _cpu_sharded_qps(shards, bases, maps, cfg, qs_np, threads, per_step, steps, warmup):
    """The reference CPU path over the sharded host corpus: per step
    `per_step` queries, each scanned by every shard's CpuIndex and merged."""
    from oracle import oracle as O

    nq = qs_np.shape[0]
    times = []
    for st in range(warmup + steps):
        sel = qs_np[(np.arange(per_step) + st * per_step) % nq]
        t0 = time.perf_counter()
        O.cpu_sharded_query_batch(shards, bases, cfg["n"], cfg["dim"], sel, cfg["k"], threads=threads, maps=maps)
        dt = time.perf_counter() - t0
        if st >= warmup:
            times.append(dt)
    return per_step * len(times) / sum(times), sum(times)


def _baseline_sample(shards, cfg, threads, per_step):
    kept = sum(a.shape[0] for a in shards)
    what = f"{kept} kept rows of {cfg['n']}" if cfg.get("filter") else f"all {cfg['n']} rows"
    return (f"{per_step} queries per step over {what} x {cfg['dim']} fp32 in {len(shards)} row shards "
            f"(<= 3.5 GiB each, one CpuIndex per shard, {threads} threads), WASM-SIMD exact scan + topK "
            "restated in C (kernel.wat, cpu.ts:66-88, flat.ts:217-239), shards merged with mergePartials "
            "(gpuTopk.ts:160-189)")


def run_sharded(args, name, ds):
    """One row-sharded configuration; returns rank 0's JSON line (else None)."""
    import torch

    from browservec_b200 import datagen
    from browservec_b200.sharded import ShardedIndex, shard_bounds

    cfg = dict(SHARDED[name])
    if args.rows:  # a smaller case of the same configuration (for ncu captures)
        cfg["n"] = args.rows
    if args.queries:
        cfg["nq"] = args.queries
    dist, world, rank, local = ds
    dev = torch.device("cuda", local)
    n, dim, nq, k = cfg["n"], cfg["dim"], cfg["nq"], cfg["k"]
    fetch = min(n, max(k, k * cfg["rf"]))  # src/index.ts:414-417
    lo, hi = shard_bounds(n, world, rank)
    R = {8: 1, 4: 2, 1: 8}[cfg["bits"]]
    P = 1 << (dim - 1).bit_length()
    metric = (f"queries/sec at fixed recall@10 ({cfg['workload']}, N={n}, d={dim}, k={k}, F={fetch})")
    config = {"workload": cfg["workload"], "rows": n, "dim": dim, "padded_dim": P, "bits": cfg["bits"],
              "queries_per_step": nq, "k": k, "fetch": fetch, "metric": cfg["metric"], "scoring": cfg["scoring"],
              "parallelism": f"row shards x{world} + NCCL all-gather merge", "data_kind": cfg["kind"],
              "l2": f"no flush needed: each step reads {(hi - lo) * (P // R + 4) / 1e6:.0f} MB of codes per GPU"
                    + (" (> 126 MB L2)" if (hi - lo) * (P // R + 4) > 126e6 else " (fits in L2)")}
    threads = os.cpu_count() or 1
    if args.impl == "reference":
        if rank == 0:
            shards, bases, maps = _host_shards(torch, dev, cfg, threads)
            qs_np = datagen.rows(torch, dev, cfg["kind"], cfg["seed"], 0, nq, dim,
                                 stream=datagen.STREAM_QUERIES).cpu().numpy()
            torch.cuda.empty_cache()
            per_step = args.cpu_queries or 4
            qps, _ = _cpu_sharded_qps(shards, bases, maps, cfg, qs_np, threads, per_step, args.steps, args.warmup)
            line = {"metric": metric, "value": qps, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": per_step / qps * 1e3, "higher_is_better": True,
                    "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                    "impl": "reference", "config": config,
                    "cpu_baseline": {"value": qps, "unit": UNIT, "cores": threads, "kind": "port",
                                     "sample": _baseline_sample(shards, cfg, threads, per_step)},
                    "e2e": {"value": qps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            return line
        return None

    scoring = args.sharded_scoring or cfg["scoring"]
    batched = scoring != "asym" and not args.per_query
    config["scoring"] = scoring
    config["search"] = ("batched: prep + rounds of (tcgen05 kind::i8 GEMM + select)"
                        + (", all-gather of candidate keys + global F-th key, exact re-rank of the shard's "
                           "members of the global best F" if world > 1 else ", exact re-rank of the best F")
                        + ", all-gather of shard records + merge" if batched else
                        "per query one scan + one tail launch, then one merge launch per step")
    x = datagen.rows(torch, dev, cfg["kind"], cfg["seed"], lo, hi, dim)
    idx = ShardedIndex(dim, n, bits=cfg["bits"], scoring=scoring, metric=cfg["metric"], device=local,
                       batched=batched)
    idx.load(x)
    qs = datagen.rows(torch, dev, cfg["kind"], cfg["seed"], 0, nq, dim, stream=datagen.STREAM_QUERIES)
    dc, flt = _c5_keep(torch, dev, cfg, lo, hi) if cfg.get("filter") else (None, None)
    if dc is not None:
        config["filter"] = "device predicate (bv_filter_mask) evaluated every step, kept rows compacted"
    torch.cuda.synchronize()
    eng_index = idx.engine.index

    def search(qq):
        # the filter's mask is rebuilt every step from the shard's device columns
        return idx.search(qq, k, fetch, dc.mask(flt) if dc is not None else None)

    for _ in range(args.warmup):
        rows, scores, counts = search(qs)
    torch.cuda.synchronize()
    dist.barrier()
    clk = Clocks(local)
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(args.steps):
        rows, scores, counts = search(qs)
    e1.record(cur)
    torch.cuda.synchronize()
    clk_res = clk.stop()
    ms = e0.elapsed_time(e1)
    # The phase breakdown and the GEMM's own device time come from as many
    # further steps run with per-phase events (bv_set_batch_timing), outside
    # the timed region: reading them back synchronises every step.
    prof = {"gemm_ms": 0.0, "gemm_macs": 0.0, "gemm_launches": 0, "select_ms": 0.0, "tail_ms": 0.0,
            "prep_ms": 0.0, "compact_ms": 0.0, "rounds": 0}
    prof_step_ms = 0.0
    if batched:
        eng_index.set_batch_timing(True)
        dist.barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(cur)
        for _ in range(args.steps):
            search(qs)
            pr = eng_index.batch_profile()
            for key in prof:
                prof[key] += pr[key]
        p1.record(cur)
        torch.cuda.synchronize()
        prof_step_ms = p0.elapsed_time(p1) / args.steps
        eng_index.set_batch_timing(False)
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    qps = args.steps * nq / (ms / 1e3)
    # the search's own launches, plus the exchange kernels: batched two-phase
    # (keys threshold, finish's trim, merge), per-query (merge); one rank has
    # no exchange
    launches_per_step = eng_index.last_launches() + (0 if world == 1 else (3 if batched else 1))

    ns = min(nq, 100)
    keep = _unpack(torch, dc.mask(flt), hi - lo) if dc is not None else None
    kept_local = int(keep.sum().item()) if keep is not None else hi - lo
    truth = _exact_top10(torch, dist, x, lo, qs[:ns], keep=keep)

    def recall(rr):
        got = rr[:ns, :10].cpu().numpy()
        return sum(len(set(truth[i].tolist()) & set(got[i].tolist())) for i in range(ns)) / (ns * 10)

    rec = recall(rows)
    query_ms = ms / (args.steps * nq)
    if batched:
        # the dominant kernel: the GEMM, 2 x queries x contracted rows x paddedDim int8 ops,
        # over its own device time (events around each GEMM launch of the timed steps)
        ops = 2.0 * prof["gemm_macs"]
        gemm_s = prof["gemm_ms"] / 1e3
        tops = ops / gemm_s / 1e12 if gemm_s > 0 else 0.0
        peak = 2.0 * tensor_peak()
        # DRAM bytes of the step's GEMM launches, scaled by row tiles from the ncu capture of
        # one config-4 launch (rows of the same padded width only); None for other widths
        traffic = None
        gt = _measured_traffic().get("gemm_c4", {})
        if gt and P == gt["row_bytes"] and kept_local == hi - lo:
            traffic = gt["bytes_per_row_tile"] * (-(-(hi - lo) // 256))
        roofline = {"bound": "tensor", "achieved": tops, "peak": peak, "unit": "TOP/s (int8)",
                    "frac": tops / peak, "traffic": traffic,
                    "traffic_scope": "DRAM bytes of one step's GEMM launches (the span 'achieved' covers), "
                                     "scaled by row tiles from one ncu capture (profiles/gemm_c4_full.md)",
                    "algorithmic_operand_bytes_per_step": float((hi - lo) * P + nq * P),
                    "peak_kind": "int8 dense = 2 x the measured bf16 burst (MEASURED_PEAKS.json bf16_tflops, "
                                 "of measured); no int8 figure is measured on this pool",
                    "kernel": "gemm_kernel (tcgen05.mma kind::i8)",
                    "algorithmic_ops_per_step": ops / args.steps,
                    "gemm_launches_per_step": prof["gemm_launches"] / args.steps,
                    "gemm_ms_per_step": prof["gemm_ms"] / args.steps,
                    "duration": "CUDA events around every GEMM launch of as many profiled steps run after "
                                "the timed region, on its stream"}
        breakdown = {kk: prof[kk] / args.steps for kk in ("prep_ms", "gemm_ms", "select_ms", "tail_ms", "compact_ms")}
        breakdown["other_ms"] = prof_step_ms - sum(breakdown.values())
        breakdown["profiled_step_ms"] = prof_step_ms
        breakdown["note"] = ("phases of steps run with per-phase events after the timed region "
                             "(they synchronise each step); the timed steps ran without them")
        breakdown["rounds"] = prof["rounds"] / args.steps
    else:
        # per-GPU roofline of the scan: codes + scales of the shard, the re-rank rows, the query
        algo_bytes = (hi - lo) * (P // R + 4) + fetch * dim * 4 + dim * 4
        peak, peak_kind = peaks()
        achieved = algo_bytes / (query_ms / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": None,
                    "peak_kind": f"{peak_kind} (copy bandwidth, MEASURED_PEAKS.json hbm_gbs)",
                    "algorithmic_bytes_per_launch": algo_bytes,
                    "duration": "per query per GPU: timed region / queries (scan + tail, all-gather and "
                                "merge amortised)"}
        breakdown = None

    # the reference's own arithmetic (asym: fp32 rotated query x codes), per-query scans, for recall
    also = None
    if scoring != "asym" and not args.no_asym:
        idx.set_scoring("asym", batched=False)
        r2, _, _ = idx.search(qs[:ns], k, fetch, dc.mask(flt) if dc is not None else None)
        also = {"scoring": "asym (reference arithmetic: fp32 rotated query x codes, per-query scans)",
                "recall_at_10": recall(r2), "recall_sample": ns}
        idx.set_scoring(scoring, batched=batched)

    # 1-bit codes: the same batch scored as BASELINE words config 4's prefilter, the
    # popc Hamming distance of the query's sign bits and the codes (+-1 x +-1 on the
    # tensor cores: idot = P - 2 x hamming), timed like the headline
    hamming = None
    if cfg["bits"] == 1 and scoring == "int" and batched and not args.no_hamming:
        idx.set_scoring("hamming", batched=True)
        for _ in range(args.warmup):
            search(qs)
        dist.barrier()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(cur)
        for _ in range(args.steps):
            rh, _, _ = search(qs)
        h1.record(cur)
        torch.cuda.synchronize()
        t = torch.tensor([h0.elapsed_time(h1)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        hms = float(t.item())
        hamming = {"scoring": "hamming (popc of the query's sign bits against the 1-bit codes, as +-1 int8 "
                              "on the tensor cores)",
                   "value": args.steps * nq / (hms / 1e3), "unit": UNIT, "ms_per_step": hms / args.steps,
                   "recall_at_10": recall(rh), "recall_sample": ns}
        idx.set_scoring(scoring, batched=batched)

    # e2e: host queries (pinned) -> device, search, results back to the host, every step
    q_host = qs.cpu().pin_memory()
    e2e_steps = max(1, min(args.steps, 3))
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        qd = q_host.to(dev, non_blocking=True)
        r_, s_, c_ = search(qd)
        r_, s_, c_ = r_.cpu(), s_.cpu(), c_.cpu()
    wall = time.perf_counter() - t0
    t = torch.tensor([wall], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    wall = float(t.item())
    e2e = {"value": e2e_steps * nq / wall, "unit": UNIT, "h2d_bytes_per_step": nq * dim * 4,
           "d2h_bytes_per_step": nq * (2 * k + 1) * 4, "steps": e2e_steps,
           "timing": "host wall clock, max over ranks (pinned H2D of the batch, search, D2H of the results)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        shards, bases, maps = _host_shards(torch, dev, cfg, threads, x=x)
        per = args.cpu_queries or 16
        cqps, _ = _cpu_sharded_qps(shards, bases, maps, cfg, qs.cpu().numpy(), threads, per, 1, 0)
        cpu = {"value": cqps, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": _baseline_sample(shards, cfg, threads, per)}
        del shards
    if rank == 0:
        line = {"metric": metric, "value": qps, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": {"int": "s8", "hamming": "b1"}.get(scoring, "f32xs8"),
                "data": f"synthetic (seeded Philox, {cfg['kind']}, L2-normalised)", "config": config,
                "recall_at_10": rec, "recall_sample": ns, "query_ms": query_ms,
                "gpu_launches": args.steps * launches_per_step, "roofline": roofline, "cpu_baseline": cpu,
                "e2e": e2e, "clocks": clk_res, "also": also, "step_breakdown_ms": breakdown}
        if hamming is not None:
            line["hamming"] = hamming
    idx.destroy()
    return line if rank == 0 else None


METRIC_SHARDED = "queries/sec at fixed recall@10 (row-sharded quantized flat scan)"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scoring", default="int", choices=["asym", "int"])
    ap.add_argument("--also", default="asym", choices=["asym", "int", "none"],
                    help="second scoring mode timed and reported beside the headline")
    ap.add_argument("--replicas", type=int, default=4)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--config", default=None, choices=[*SINGLE, *SHARDED],
                    help="one configuration only (default: config 4 as the headline line, with configs "
                         "1, 2, 3 and 5 measured in the same run under its 'configs' key)")
    ap.add_argument("--cpu-queries", type=int, default=0,
                    help="sharded configs: queries per CPU-baseline sample (default 16, reference arm 4 per step)")
    ap.add_argument("--no-asym", action="store_true", help="sharded configs: skip the asym recall figure")
    ap.add_argument("--no-hamming", action="store_true",
                    help="config 4: skip the Hamming (popc) scoring figure")
    ap.add_argument("--sharded-scoring", default=None, choices=["asym", "int", "hamming"],
                    help="scoring of a sharded config (default: the config's)")
    ap.add_argument("--rows", type=int, default=0, help="sharded configs: corpus rows (default: the config's)")
    ap.add_argument("--queries", type=int, default=0,
                    help="sharded configs: batch size; single configs: queries per step (default: the config's)")
    ap.add_argument("--per-query", action="store_true",
                    help="sharded configs: per-query scans instead of the batched tensor-core path")
    args = ap.parse_args()
    import torch

    ds = _init_dist(torch)
    dist, world, rank, local = ds
    try:
        if args.config is not None:
            line = run_config(args, args.config, ds)
        else:
            line = run_config(args, "c4", ds)
            if args.impl == "ours":
                extra = {}
                for name in ("c3", "c5", "c2", "c1"):
                    sub = argparse.Namespace(**vars(args))
                    try:
                        r = run_config(sub, name, ds)
                        if r is not None:
                            extra[name] = _summary(r)
                    except Exception as e:  # a failing side configuration must not lose the headline
                        extra[name] = {"error": f"{type(e).__name__}: {e}"[:400]}
                    torch.cuda.empty_cache()
                if line is not None:
                    line["configs"] = extra
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        dist.destroy_process_group()


def _summary(line):
    """The figures of one configuration's line kept under the headline's 'configs'."""
    keys = ("metric", "value", "unit", "ms_per_step", "dtype", "recall_at_10", "recall_sample", "gpu_launches",
            "roofline", "cpu_baseline", "e2e", "also", "hamming", "step_breakdown_ms", "clocks")
    out = {k: line[k] for k in keys if k in line}
    out["config"] = line.get("config")
    return out


def run_config(args, name, ds):
    if name in SHARDED:
        return run_sharded(args, name, ds)
    return run_single(args, name, ds)


def run_single(args, name, ds):
    """One single-query configuration (replicas per GPU); returns rank 0's
    JSON line (else None)."""
    args.config = name
    _use_single(args.config)
    if args.queries:  # a shorter step (for ncu captures); the timed line then says so in its config
        global N_QUERIES
        N_QUERIES = args.queries
    if BITS == 0:  # the exact index has one scoring
        args.scoring, args.also = "asym", "none"
    corpus_mb = N_ROWS * (DIM * 4 if BITS == 0 else (1 << (DIM - 1).bit_length()) + 4) / 1e6
    args.replicas = max(args.replicas, int(130.0 / corpus_mb) + 1)

    import torch

    dist, world, rank, local = ds
    if world == 1:
        dist = None  # replicas need no collective on one GPU
    dev = torch.device("cuda", local)
    fetch = min(N_ROWS, max(K, K * RERANK_FACTOR))  # src/index.ts:414-417
    config = {"workload": WORKLOAD, "rows": N_ROWS, "dim": DIM, "bits": BITS,
              "padded_dim": 1 << (DIM - 1).bit_length(), "queries_per_step": N_QUERIES,
              "k": K, "fetch": fetch, "metric": "cosine", "scoring": args.scoring if BITS else "exact fp32",
              "parallelism": f"replicas x{max(world, 1)}",
              "l2": f"corpus replicated x{args.replicas} ({args.replicas * corpus_mb:.0f} MB > 126 MB L2), "
                    "query i scans replica i % replicas",
              "submission": "one bv_search_async_n call per step: a single-query scan per entry"}

    if args.impl == "reference":
        if rank != 0:
            return None
        corpus = make_data(torch, dev, SEED, N_ROWS, DIM)
        queries = make_data(torch, dev, SEED + 1, N_QUERIES, DIM)
        c_np, q_np = corpus.cpu().numpy(), queries.cpu().numpy()
        threads = os.cpu_count() or 1
        qps, per_step = cpu_reference_qps(c_np, q_np, args.steps, args.warmup, max(threads, 8), threads)
        line = {"metric": METRIC, "value": qps, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": per_step / qps * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                "config": config,
                "cpu_baseline": {"value": qps, "unit": UNIT, "cores": threads, "kind": "port",
                                 "sample": f"{per_step} queries per step over the full {N_ROWS} x {DIM} fp32 corpus "
                                           "(WASM-SIMD scan restated in C, one query per thread)"},
                "e2e": {"value": qps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        return line

    from browservec_b200.index import AddonQuantIndex, AsyncSearchList, PreparedSearch

    corpus = make_data(torch, dev, SEED, N_ROWS, DIM)
    queries = make_data(torch, dev, SEED + 1, N_QUERIES, DIM)
    out_rows = torch.zeros((N_QUERIES, K), dtype=torch.int32, device=dev)
    out_scores = torch.zeros((N_QUERIES, K), dtype=torch.float32, device=dev)
    out_counts = torch.zeros((N_QUERIES,), dtype=torch.int32, device=dev)
    # One explicit stream for every launch and both timing events (never the
    # legacy default stream, whose handle 0 would select each index's own stream).
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    assert sp != 0

    def build(scoring):
        reps = []
        for _ in range(args.replicas):
            ix = AddonQuantIndex(DIM, bits=BITS, scoring=scoring, device=local)
            torch.cuda.synchronize()
            ix.append_device(corpus.data_ptr(), N_ROWS, torch.cuda.current_stream().cuda_stream)
            reps.append(ix)
        torch.cuda.synchronize()
        return reps

    lists = {}

    def step(reps):
        # one bv_search_async_n call submits the step's N_QUERIES single-query
        # scans, query i on replica i % replicas (argument array built once)
        key = id(reps)
        if key not in lists:
            lists[key] = AsyncSearchList([(reps[i % len(reps)], queries[i].data_ptr(), K, fetch, True,
                                           out_rows[i].data_ptr(), out_scores[i].data_ptr(),
                                           out_counts[i:].data_ptr()) for i in range(N_QUERIES)])
        lists[key].submit(sp)

    def timed(reps, clocks=False):
        for _ in range(args.warmup):
            step(reps)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        clk = Clocks(local) if clocks else None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step(reps)
        e1.record(stream)
        torch.cuda.synchronize()
        clk_res = clk.stop() if clk else None
        ms = e0.elapsed_time(e1)
        if dist:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        rec = recall_at_10(torch, corpus, queries, out_rows.cpu().numpy())
        return ms, rec, clk_res

    reps = build(args.scoring)
    ms, rec, clk = timed(reps, clocks=True)
    launches = args.steps * N_QUERIES * reps[0].last_launches()
    qps = max(world, 1) * args.steps * N_QUERIES / (ms / 1e3)
    query_ms = ms / (args.steps * N_QUERIES)

    # roofline: algorithmic bytes of one query (codes + scales + re-rank rows + query)
    if BITS == 0:
        algo_bytes = N_ROWS * DIM * 4 + DIM * 4
    else:
        algo_bytes = N_ROWS * ((1 << (DIM - 1).bit_length()) * BITS // 8 + 4) + fetch * DIM * 4 + DIM * 4
    peak, peak_kind = peaks()
    achieved = algo_bytes / (query_ms / 1e3) / 1e9
    traffic = None
    if BITS == 8 and N_ROWS == 100_000:
        traffic = _measured_traffic().get("scan_c2", {}).get(args.scoring)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic,
                "peak_kind": f"{peak_kind} (copy bandwidth, MEASURED_PEAKS.json hbm_gbs)",
                "algorithmic_bytes_per_launch": algo_bytes,
                "duration": "per query: timed region / queries (scan + tail kernels, PDL-overlapped)"}

    # e2e through the host API (host buffers, H2D + D2H + sync per query)
    e2e = None
    if not args.no_e2e:
        q_np = queries.cpu().numpy()
        calls = [PreparedSearch(ix, 1, K, fetch, True) for ix in reps]  # host buffers, one query per call
        for i in range(min(64, N_QUERIES)):
            calls[i % len(calls)](q_np[i:i + 1])
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e2e_steps = max(1, min(args.steps, 3))
        for _ in range(e2e_steps):
            for i in range(N_QUERIES):
                calls[i % len(calls)](q_np[i:i + 1])
        wall = time.perf_counter() - t0
        if dist:
            t = torch.tensor([wall], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            wall = float(t.item())
        out_words = 2 * K + 1
        e2e = {"value": max(world, 1) * e2e_steps * N_QUERIES / wall, "unit": UNIT,
               "h2d_bytes_per_step": N_QUERIES * DIM * 4, "d2h_bytes_per_step": N_QUERIES * out_words * 4,
               "steps": e2e_steps, "timing": "host wall clock around synchronous bv_search calls (one query "
                                             "per call, host buffers, PreparedSearch)"}
    for ix in reps:
        ix.destroy()

    also = None
    if args.also != "none" and args.also != args.scoring:
        reps2 = build(args.also)
        ms2, rec2, _ = timed(reps2)
        also = {"scoring": args.also, "value": max(world, 1) * args.steps * N_QUERIES / (ms2 / 1e3),
                "unit": UNIT, "recall_at_10": rec2, "ms_per_step": ms2 / args.steps}
        for ix in reps2:
            ix.destroy()

    cpu = None
    if rank == 0 and not args.no_cpu and world == 1:
        threads = os.cpu_count() or 1
        c_np, q_np = corpus.cpu().numpy(), queries.cpu().numpy()
        cqps, per = cpu_reference_qps(c_np, q_np, 1, 0, max(threads, 8), threads)
        cpu = {"value": cqps, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{per} queries over the full {N_ROWS} x {DIM} fp32 corpus, WASM-SIMD exact scan "
                         "restated in C (src/fallback/kernel.wat), one query per thread"}

    if rank == 0:
        line = {"metric": METRIC, "value": qps, "unit": UNIT, "n_gpus": max(world, 1), "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32" if BITS == 0 else ("s8" if args.scoring == "int" else "f32xs8"),
                "data": "synthetic (seeded Philox N(0,1), L2-normalised)", "config": config,
                "recall_at_10": rec, "query_ms": query_ms, "gpu_launches": launches,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk, "also": also}
        return line
    return None


if __name__ == "__main__":
    main()
