#!/usr/bin/env python
"""SVA decode benchmark on B200: microseconds per query at 2^20 cached keys (summon + verify).

Workload (in the 9-head shape the reference publishes its million-key numbers
on): 2^20 cached keys per head, 9 independent heads, head_dim 64, rank 64, bf16 K/V ~ N(0,1)
with 64 planted near-duplicates per head, PQ codes 4x64 (default) or 1x256, shortlist 2048,
budget 512, one query token.  A "query" is one decode token over all 9 heads.

A step is one CUDA-graph replay of ``--queries-per-step`` decode calls.  The graph cycles over
``--sets`` independent 9-head catalogs so that consecutive queries touch disjoint memory (each
query touches ~44 MB; four sets ~176 MB > the 126 MB L2), i.e. every query runs against a cold
L2.  Inputs are resident in HBM before timing; the catalog is built by the CUDA write path.

Multi-GPU (``torchrun --nproc-per-node N``): the catalog is sharded by key range; every rank
summons, rescores and partially verifies its range, and the exact global result comes from three
NCCL all-gathers between the stages (sva_b200.sharded).  ``value`` is the max over ranks.

``--impl reference`` times the CPU restatement of the reference path (oracle/cpu_baseline.py,
the reference itself is PyTorch code that cannot be shipped to the GPU host) on the same
configuration with all host threads.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SVA decode us/query @1M keys (summon+verify)"
UNIT = "us/query"
# reference, H100, 9 heads: docs/snapshots/compact_summon_frontier_snapshot_2026-05-14.md:41,45
PUBLISHED_US = {"4x64": 1028.0, "1x256": 649.0}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="sva_b200", choices=["sva_b200", "reference"])
    ap.add_argument("--keys", type=int, default=1 << 20)
    ap.add_argument("--heads", type=int, default=9)
    ap.add_argument("--pq", default="4x64", choices=["4x64", "1x256", "2x256"])
    ap.add_argument("--shortlist", type=int, default=2048)
    ap.add_argument("--budget", type=int, default=512)
    ap.add_argument("--sets", type=int, default=4)
    ap.add_argument("--queries-per-step", type=int, default=256)
    ap.add_argument("--e2e-queries", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--throughput-heads", type=int, default=64,
                    help="heads per launch of the throughput-mode measurement (0: skip)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-inverted", dest="inverted", action="store_false",
                    help="skip the static inverted-index summon measurement")
    ap.add_argument("--no-ragged", dest="ragged", action="store_false",
                    help="skip the config-5 ragged paged batch measurement")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg3", "cfg4"],
                    help="cfg2: million-key decode (default); cfg3 / cfg4: model-level decode tokens/s")
    ap.add_argument("--model-prefill", type=int, default=None, help="prompt tokens (cfg3: 8192, cfg4: 32768)")
    ap.add_argument("--model-decode", type=int, default=None, help="decode steps (cfg3: 256, cfg4: 64)")
    return ap.parse_args()


def pq_shape(pq: str):
    s, c = pq.split("x")
    return int(s), int(c)


def algorithmic_bytes(args) -> dict:
    """Algorithmic HBM bytes per query (one token, all heads), reference dtypes: uint8 codes, fp32
    codebooks / projections / k_low, bf16 K and V."""
    s, c = pq_shape(args.pq)
    rank = 64
    per_head = {
        "codes": args.keys * s,
        "codebooks": c * rank * 4,
        "q_proj": 64 * rank * 4,
        "rescore": args.shortlist * rank * 4,
        "verify": args.budget * 64 * 2 * 2,
    }
    per_query = {k: v * args.heads for k, v in per_head.items()}
    per_query["total"] = sum(per_query.values())
    return per_query


# ---------------------------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines: list[str] = []
        self._thread = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        if self.gpu_id:
            cmd += ["-i", self.gpu_id]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._thread:
            self._thread.join(timeout=2)
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "power_w_max": max(power) if power else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profile_traffic(workload: str, kernel: str):
    """DRAM traffic per launch from a committed ncu summary (profiles/traffic.json), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d.get(workload, {}).get(kernel)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------------------------------------
# CPU baseline (oracle port) -- used by --impl reference and by the cpu_baseline field
# ---------------------------------------------------------------------------------------------

def cpu_problem(args, seed: int):
    """Host-side 9-head catalog drawn like the reference's million-key benchmark (random codes and
    low-rank keys, experiments/sva_million_cached_decode_benchmark.py:97-136)."""
    s, c = pq_shape(args.pq)
    rng = np.random.default_rng(seed)
    heads, keys, d, r = args.heads, args.keys, 64, 64
    f32 = np.float32
    q = rng.standard_normal((heads, d), dtype=f32)
    q_proj = rng.standard_normal((heads, d, r), dtype=f32) * f32(0.125)
    codebooks = rng.standard_normal((heads, s, c, r // s), dtype=f32)
    codes = rng.integers(0, c, (heads, keys, s), dtype=np.uint8)
    k_low = rng.standard_normal((heads, keys, r), dtype=f32)

    def bf16_bits(shape):
        x = rng.standard_normal(shape, dtype=f32)
        return (x.view(np.uint32) >> 16).astype(np.uint16)

    kv_k = bf16_bits((heads, keys, d))
    kv_v = bf16_bits((heads, keys, d))
    return q, q_proj, np.ones(heads, dtype=f32), codebooks, codes, k_low, kv_k, kv_v


def run_cpu_decoder(args, steps: int, warmup: int, seconds: float | None):
    from oracle.cpu_baseline import CpuDecoder

    q, q_proj, scale, codebooks, codes, k_low, kk, vv = cpu_problem(args, args.seed + 101)
    threads = os.cpu_count() or 1
    dec = CpuDecoder(q_proj, scale, codebooks, codes, k_low, kk, vv, groups=1, threads=threads)
    for _ in range(warmup):
        dec(q, args.shortlist, args.budget, 0.125, "bf16", 1)
    times = []
    t_end = None if seconds is None else time.perf_counter() + seconds
    for i in range(steps):
        t0 = time.perf_counter()
        dec(q, args.shortlist, args.budget, 0.125, "bf16", 1)
        times.append(time.perf_counter() - t0)
        if t_end is not None and time.perf_counter() > t_end and i >= 1:
            break
    dec.close()
    return times, dec.threads


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    times, threads = run_cpu_decoder(args, args.steps, args.warmup, None)
    us = 1e6 * sum(times) / len(times)
    s, c = pq_shape(args.pq)
    line = {
        "metric": METRIC, "value": round(us, 2), "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": round(us / 1000.0, 4),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random catalog as in the reference million-key benchmark)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": round(us, 2), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.heads} heads x {args.keys} keys ({args.pq}), 1 query token per step"},
        "e2e": {"value": round(us, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


def workload_config(args, world: int) -> dict:
    return {
        "workload": f"cfg2 million-key decode: {args.keys} keys x {args.heads} heads, {args.pq} codes, "
                    f"shortlist {args.shortlist}, budget {args.budget}, q=1",
        "keys": args.keys, "heads": args.heads, "pq": args.pq, "shortlist": args.shortlist, "budget": args.budget,
        "head_dim": 64, "rank_dim": 64, "queries_per_step": args.queries_per_step,
        "parallelism": "single GPU" if world == 1 else f"key-range shards x{world}",
        "l2": f"{args.sets} rotating catalogs per graph ({args.sets} x ~{algorithmic_bytes(args)['total'] / 1e6:.0f} MB "
              f"touched per cycle > 126 MB L2)",
    }


# ---------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------

def build_sets(args, device, rank: int, world: int):
    """Per set: q [H,1,D], K/V [H,L_local,D] bf16, k_low [H,L_local,R], codes [H,L_local,S] for this
    rank's key range; artifacts shared across ranks (same seed)."""
    import torch

    from sva_b200 import kernels

    s, c = pq_shape(args.pq)
    heads, keys, d, r = args.heads, args.keys, 64, 64
    lo = keys * rank // world
    hi = keys * (rank + 1) // world
    sets = []
    build_ms = 0.0
    for si in range(args.sets):
        cpu_gen = torch.Generator().manual_seed(args.seed * 1000 + si)
        q = torch.randn(heads, 1, d, generator=cpu_gen).to(torch.bfloat16)
        q_proj = (torch.randn(heads, d, r, generator=cpu_gen) * 0.125).to(torch.bfloat16).float()
        k_proj = (torch.randn(heads, d, r, generator=cpu_gen) * 0.125).to(torch.bfloat16).float()
        cb = torch.randn(heads, s, c, r // s, generator=cpu_gen).to(torch.bfloat16).float()
        planted = torch.stack([torch.randperm(keys, generator=cpu_gen)[:64] for _ in range(heads)])
        noise = torch.randn(heads, 64, d, generator=cpu_gen)
        gen = torch.Generator(device=device).manual_seed(args.seed * 1000 + si + 7)
        kk = torch.empty(heads, hi - lo, d, dtype=torch.bfloat16, device=device)
        vv = torch.empty(heads, hi - lo, d, dtype=torch.bfloat16, device=device)
        for h in range(heads):
            kk[h] = torch.randn(hi - lo, d, generator=gen, device=device).to(torch.bfloat16)
            vv[h] = torch.randn(hi - lo, d, generator=gen, device=device).to(torch.bfloat16)
            sel = (planted[h] >= lo) & (planted[h] < hi)
            pos = (planted[h][sel] - lo).to(device)
            kk[h, pos] = (0.9 * q[h, 0].float()[None, :] + 0.1 * noise[h][sel]).to(torch.bfloat16).to(device)
        q = q.to(device)
        q_proj, k_proj, cb = q_proj.to(device), k_proj.to(device), cb.to(device)
        k_low = torch.empty(heads, hi - lo, r, dtype=torch.float32, device=device)
        codes = torch.empty(heads, hi - lo, s, dtype=torch.uint8, device=device)
        tc = kernels.tensor_core_write_ok(kk, k_proj)
        status = torch.zeros(1, dtype=torch.int32, device=device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        kernels.catalog_encode(kk, k_proj, cb, 0, hi - lo, k_low, codes, tensor_cores=tc, status=status)
        e1.record()
        torch.cuda.synchronize()
        if int(status.item()) != 0:
            raise RuntimeError("tensor-core write path timed out")
        build_ms += e0.elapsed_time(e1)
        if si == 0:
            # the exact CUDA-core write path, timed once for comparison (into scratch buffers)
            k2, c2 = torch.empty_like(k_low), torch.empty_like(codes)
            e0.record()
            kernels.catalog_encode(kk, k_proj, cb, 0, hi - lo, k2, c2, tensor_cores=False)
            e1.record()
            torch.cuda.synchronize()
            exact_ms = e0.elapsed_time(e1)
            del k2, c2
        scale = torch.ones(heads, dtype=torch.float32, device=device)
        sets.append(dict(q=q, q_proj=q_proj, scale=scale, cb=cb, codes=codes, k_low=k_low, keys=kk, values=vv,
                         out=torch.empty(heads, 1, d, dtype=torch.bfloat16, device=device), offset=lo))
    write = {"tensor_cores": bool(tc), "ms_per_set": build_ms / args.sets, "exact_ms_per_set": exact_ms}
    return sets, write, (hi - lo)


def inverted_measure(args, sets, device) -> dict:
    """The static inverted-index summon (reference sva/llama.py:427-576) on the same catalogs: the
    posting lists of every set are built once (not timed), then decode_inverted runs one query
    token per head with the serving defaults (8 cells per subspace, budget = min = mid budget),
    eager calls over the rotating sets, device-timed after 3 warm-ups."""
    import torch

    from sva_b200 import kernels

    post = [kernels.postings_build(st["codes"], int(st["cb"].shape[2])) for st in sets]
    outs = [torch.empty(st["q"].shape[0], st["q"].shape[2], dtype=st["q"].dtype, device=device) for st in sets]
    stats = torch.zeros(8, dtype=torch.int64, device=device)
    cells = 8

    def one(i, st_stats=None):
        k = i % len(sets)
        st = sets[k]
        kernels.decode_inverted(st["q"][:, 0, :], st["q_proj"], st["scale"], st["cb"], st["codes"], post[k],
                                st["k_low"], st["keys"], st["values"], args.budget, cells, args.budget, args.budget,
                                dynamic=False, softmax_scale=0.125, out=outs[k], stats=st_stats)

    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    n = 32
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(n):
        one(i, stats)
    e.record()
    torch.cuda.synchronize()
    st = stats.cpu().tolist()
    return {"summon": "inverted_static", "us_per_query": round(1000.0 * s.elapsed_time(e) / n, 2),
            "cells_per_subspace": cells, "budget": args.budget, "queries": n,
            "cell_visits_per_query": round(st[5] / n, 1), "verified_per_query": round(st[4] / n, 1),
            "timing": "eager calls over the rotating catalog sets, device clock"}


def throughput_measure(args, device, peak: float) -> dict:
    """Throughput mode (one GPU): many independent (head, query) problems per launch, here
    ``--throughput-heads`` heads of 2^20 keys decoded by one call, so that the per-problem latency
    chains overlap and the scan streams at bandwidth.  One catalog of that many heads (its codes
    alone exceed L2); a CUDA graph of 8 calls; device-timed over 5 replays after 3 warm-ups."""
    import copy

    import torch

    from sva_b200 import kernels

    targs = copy.copy(args)
    targs.heads, targs.sets = args.throughput_heads, 1
    sets, _, _ = build_sets(targs, device, 0, 1)
    st = sets[0]

    def call():
        kernels.decode(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"],
                       st["values"], args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1, out=st["out"])

    call()
    torch.cuda.synchronize()
    calls = 8
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(calls):
                call()
    torch.cuda.synchronize()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = 1000.0 * e0.elapsed_time(e1) / (reps * calls)
    nbytes = algorithmic_bytes(targs)["total"]
    gbs = nbytes / (us * 1e-6) / 1e9
    del graph, sets, st
    torch.cuda.empty_cache()
    return {"heads_per_launch": targs.heads, "us_per_launch": round(us, 2), "us_per_head": round(us / targs.heads, 3),
            "algorithmic_bytes_per_launch": int(nbytes), "achieved_gbs": round(gbs, 1), "peak_gbs": peak,
            "frac": round(gbs / peak, 4), "keys": args.keys, "pq": args.pq}


def ragged_paged_set(device, n_seqs: int = 64, page_keys: int = 256, seed: int = 3, heads: int = 9, kv_heads: int = 3,
                     lo: int = 4096, hi: int = 131072):
    """n_seqs sequences with cached lengths drawn log-uniform in [lo, hi]
    (seed 3), 9 query / 3 KV heads, head_dim 64, bf16 K/V ~ N(0,1), 4x64 codes, in page pools of
    page_keys keys handed out in a shuffled order (page tables [n_seqs, max_pages]).  Pools are
    head-major ([heads, pages * page_keys, ...]) so that the write path encodes them in one call;
    the decode sees them through [pages, heads, page_keys, ...] views."""
    import torch

    from sva_b200 import kernels

    gen = torch.Generator().manual_seed(seed)
    u = torch.rand(n_seqs, generator=gen, dtype=torch.float64)
    lengths = torch.exp(math.log(lo) + u * (math.log(hi) - math.log(lo))).floor().long().clamp(lo, hi)
    pages_per = (lengths + page_keys - 1) // page_keys
    total_pages = int(pages_per.sum())
    perm = torch.randperm(total_pages, generator=gen).to(torch.int32)
    table = torch.zeros(n_seqs, int(pages_per.max()), dtype=torch.int32)
    k = 0
    for b in range(n_seqs):
        n = int(pages_per[b])
        table[b, :n] = perm[k:k + n]
        k += n
    d, r, s, c = 64, 64, 4, 64
    q = torch.randn(n_seqs, heads, 1, d, generator=gen).to(torch.bfloat16)
    q_proj = (torch.randn(heads, d, r, generator=gen) * 0.125).to(torch.bfloat16).float()
    k_proj = (torch.randn(heads, d, r, generator=gen) * 0.125).to(torch.bfloat16).float()
    cb = torch.randn(heads, s, c, r // s, generator=gen).to(torch.bfloat16).float()
    rows = total_pages * page_keys
    dgen = torch.Generator(device=device).manual_seed(seed + 11)
    keys = torch.randn(kv_heads, rows, d, generator=dgen, device=device).to(torch.bfloat16)
    values = torch.randn(kv_heads, rows, d, generator=dgen, device=device).to(torch.bfloat16)
    k_low = torch.empty(heads, rows, r, dtype=torch.float32, device=device)
    codes = torch.empty(heads, rows, s, dtype=torch.uint8, device=device)
    q_proj, k_proj, cb = q_proj.to(device), k_proj.to(device), cb.to(device)
    kernels.catalog_encode(keys, k_proj, cb, 0, rows, k_low, codes)

    def pages_view(t):
        return t.view(t.shape[0], total_pages, page_keys, t.shape[-1]).permute(1, 0, 2, 3)

    return dict(q=q.to(device), q_proj=q_proj, scale=torch.ones(heads, device=device), cb=cb,
                codes=pages_view(codes), k_low=pages_view(k_low), keys=pages_view(keys), values=pages_view(values),
                table=table.to(device), lengths=lengths.tolist(), seq_lens=lengths.to(device),
                flat=dict(codes=codes, k_low=k_low, keys=keys, values=values), page_keys=page_keys,
                total_pages=total_pages)


def ragged_measure(args, device, peak: float) -> dict:
    """Config 5 on one GPU: one step decodes one query token of each of the 64 sequences (all 9
    heads) in a single sva_decode_batched call over the paged catalog; device-timed CUDA-graph
    replays after 3 warm-ups.  Before timing, two sequences are checked against the
    single-sequence decode of their own rows (identical shortlists, final sets and outputs)."""
    import torch

    from sva_b200 import _lib, kernels

    st = ragged_paged_set(device)
    n_seqs, heads = st["q"].shape[0], st["q"].shape[1]
    lmax = max(st["lengths"])
    out = torch.empty(n_seqs, heads, 1, 64, dtype=torch.bfloat16, device=device)

    def call(**kw):
        return kernels.decode_batched(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"],
                                      st["keys"], st["values"], args.shortlist, args.budget, seq_lens=st["seq_lens"],
                                      page_table=st["table"], max_len=lmax, softmax_scale=0.125, logits_mode=1,
                                      **kw)

    # consistency with single-sequence decodes (gathered rows of the sequence's pages)
    _, sl, fin = call(out=out, want_shortlist=True, want_final=True)
    torch.cuda.synchronize()
    parity = "ok"
    pk = st["page_keys"]
    for b in (0, n_seqs - 1):
        n = st["lengths"][b]
        pages = st["table"][b, : (n + pk - 1) // pk].long()
        idx = (pages[:, None] * pk + torch.arange(pk, device=device)[None, :]).reshape(-1)[:n]
        f = st["flat"]
        o1, s1, f1 = kernels.decode(st["q"][b], st["q_proj"], st["scale"], st["cb"], f["codes"][:, idx].contiguous(),
                                    f["k_low"][:, idx].contiguous(), f["keys"][:, idx].contiguous(),
                                    f["values"][:, idx].contiguous(), args.shortlist, args.budget, softmax_scale=0.125,
                                    logits_mode=1, want_shortlist=True, want_final=True)
        torch.cuda.synchronize()
        if not (torch.equal(s1, sl[b]) and torch.equal(f1, fin[b]) and torch.equal(o1, out[b])):
            parity = f"mismatch in sequence {b}"
    calls = 8
    prof = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(4)]
    for e in prof:
        e.record()
    torch.cuda.synchronize()
    handles = ctypes_voidp_array([e.cuda_event for e in prof[1:]])
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        call(out=out)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(calls):
                if i == 0:
                    prof[0].record()
                    _lib.load().sva_profile_events(handles, 3)
                try:
                    call(out=out)
                finally:
                    if i == 0:
                        _lib.load().sva_profile_events(None, 0)
    torch.cuda.synchronize()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    reps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kern = []
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = 1000.0 * e0.elapsed_time(e1) / (reps * calls)
    graph.replay()
    torch.cuda.synchronize()
    kern = [round(1000.0 * prof[j].elapsed_time(prof[j + 1]), 2) for j in range(3)]
    total_keys = sum(st["lengths"])
    sl_eff = sum(min(args.shortlist, n) for n in st["lengths"])
    b_eff = sum(min(args.budget, args.shortlist, n) for n in st["lengths"])
    nbytes = heads * (total_keys * 4 + sl_eff * 64 * 4 + b_eff * 64 * 2 * 2) + heads * (64 * 64 * 4 + 64 * 64 * 4)
    gbs = nbytes / (us * 1e-6) / 1e9
    del graph
    return {"workload": f"cfg5 ragged paged decode: {n_seqs} sequences, lengths log-uniform in [4096, 131072] "
                        f"(total {total_keys} keys), 9 query / 3 KV heads, 4x64 codes, {pk}-key pages, "
                        f"shortlist {args.shortlist}, budget {args.budget}, one token per sequence per step",
            "us_per_step": round(us, 2), "tokens_per_s": round(n_seqs / (us * 1e-6), 1),
            "us_per_token": round(us / n_seqs, 3), "algorithmic_bytes_per_step": int(nbytes),
            "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "frac": round(gbs / peak, 4),
            "kernel_us_first_call": dict(zip(["prep", "scan", "finish"], kern)), "gpu_launches_per_step": 3,
            "parity": parity, "total_keys": total_keys, "pages": st["total_pages"],
            "timing": "CUDA graph of 8 steps, 5 replays after 3 warm-ups, device clock"}


def write_path_summary(args, write: dict, local_keys: int, peak: float) -> dict:
    """The catalog write of one set (all heads): keys/s, projection TFLOP/s and the fraction of
    the measured HBM peak its algorithmic bytes reach (K read as bf16, k_low fp32 written, codes)."""
    s, _ = pq_shape(args.pq)
    keys = args.heads * local_keys
    flops = 2.0 * keys * 64 * 64
    nbytes = keys * (64 * 2 + 64 * 4 + s)
    out = {"path": "tcgen05 projection + CUDA-core assignment" if write["tensor_cores"] else "exact CUDA-core"}
    for name, ms in (("", write["ms_per_set"]), ("exact_", write["exact_ms_per_set"])):
        out[name + "ms_per_set"] = round(ms, 3)
        out[name + "keys_per_s"] = round(keys / (ms * 1e-3), 1)
        out[name + "projection_tflops"] = round(flops / (ms * 1e-3) / 1e12, 3)
        out[name + "hbm_frac"] = round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)
    out["algorithmic_bytes_per_set"] = int(nbytes)
    return out


def gpu_arm(args):
    import torch

    from sva_b200 import _lib, kernels

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (B200); use --impl reference for the CPU baseline")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        group = dist.group.WORLD
    lib = _lib.load()
    sets, write, local_keys = build_sets(args, device, rank, world)

    if world == 1:
        def one_query(st):
            kernels.decode(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"],
                           st["values"], args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1, out=st["out"])
    else:
        from sva_b200 import sharded

        shard = sharded.ShardedDecoder(group, heads=args.heads, head_dim=64, shortlist=args.shortlist,
                                       budget=args.budget, device=device)

        def one_query(st):
            shard.decode(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"],
                         st["values"], key_offset=st["offset"], out=st["out"], logits_mode=1)

    # warm the workspace / communicators outside capture
    for st in sets:
        one_query(st)
    torch.cuda.synchronize()

    grid_schedule = local_keys > 32768 or world > 1  # shards always run prep + scan + top
    n_prof = 3 if grid_schedule else 1
    prof = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(n_prof + 1)]
    for e in prof:  # torch creates the CUDA event on its first record
        e.record()
    torch.cuda.synchronize()
    handles = ctypes_voidp_array([e.cuda_event for e in prof[1:]])
    if not all(e.cuda_event for e in prof):
        raise RuntimeError("profiling events were not created")
    graph = torch.cuda.CUDAGraph()
    qps = args.queries_per_step
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for i in range(qps):
                st = sets[i % len(sets)]
                if i == 0:
                    prof[0].record()
                    lib.sva_profile_events(handles, n_prof)
                try:
                    one_query(st)
                finally:
                    if i == 0:
                        lib.sva_profile_events(None, 0)
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if group is not None:
        torch.distributed.barrier(group)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kern = []
    gpu_id = None
    try:
        gpu_id = str(torch.cuda.get_device_properties(device).uuid)
        gpu_id = gpu_id if gpu_id.startswith("GPU-") else "GPU-" + gpu_id
    except Exception:
        gpu_id = str(local_rank)
    sampler = ClockSampler(gpu_id)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    cur = torch.cuda.current_stream(device)
    for i in range(args.steps):
        starts[i].record(cur)
        graph.replay()
        ends[i].record(cur)
        ends[i].synchronize()
        kern.append([prof[j].elapsed_time(prof[j + 1]) for j in range(n_prof)])
    torch.cuda.synchronize()
    wall = time.perf_counter() - t_wall
    clocks = sampler.stop()
    step_ms = [starts[i].elapsed_time(ends[i]) for i in range(args.steps)]
    ms_step = sum(step_ms) / len(step_ms)
    if group is not None:
        t = torch.tensor([ms_step], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
        ms_step = float(t.item())
    us_query = 1000.0 * ms_step / qps

    # per-kernel timing (first query of every replay)
    ab = algorithmic_bytes(args)
    local_frac = local_keys / args.keys
    if grid_schedule:
        # third launch: finish on one GPU (rescore + verify); on shards the local top select
        # (its rescore / verify stages follow the all-gathers and are not separately timed)
        names = ["prep", "scan", "finish" if world == 1 else "top"]
        kernel_bytes = {
            # prep reads the projections and codebooks (and a 16384-key sample of the codes)
            "prep": ab["codebooks"] + ab["q_proj"],
            # scan is the single pass over the codes
            "scan": ab["codes"] * local_frac,
            # finish gathers the shortlist's k_low rows and the budget's K and V rows
            "finish": ab["rescore"] + ab["verify"],
            # top reads the scan's candidates (about 2x the shortlist, 8 bytes each)
            "top": 2 * args.shortlist * 8 * args.heads,
        }
    else:
        names = ["fused"]
        kernel_bytes = {"fused": ab["total"] * local_frac}
    kmeans = [sum(k[j] for k in kern) / len(kern) for j in range(n_prof)]
    dom = max(range(n_prof), key=lambda j: kmeans[j])
    if world > 1:
        dom = names.index("scan")  # the kernel whose work the shards divide
    peak, peak_kind = measured_peaks()
    achieved = kernel_bytes[names[dom]] / (kmeans[dom] * 1e-3) / 1e9
    workload_key = f"{args.pq}_{args.heads}h_{args.keys}"
    traffic = profile_traffic(workload_key, names[dom])
    roofline = {
        "bound": "hbm", "kernel": names[dom], "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
        "algorithmic_bytes_per_launch": int(kernel_bytes[names[dom]]), "traffic": traffic,
        "kernel_us": {n: round(1000 * m, 2) for n, m in zip(names, kmeans)},
        "kernel_share": {n: round(m / sum(kmeans), 3) for n, m in zip(names, kmeans)},
    }
    step_gbs = ab["total"] * local_frac / (us_query * 1e-6) / 1e9
    step_roofline = {"algorithmic_bytes_per_query": int(ab["total"] * local_frac), "achieved": round(step_gbs, 1),
                     "frac": round(step_gbs / peak, 4), "peak_kind": peak_kind}

    # end to end through the public op with pinned host buffers
    host_query = None
    if world == 1:
        def host_query(st, hq, ho):
            kernels.decode(hq, st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"],
                           st["values"], args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1, out=ho)
    e2e = e2e_measure(args, sets, one_query, device, group, host_query)

    line = {
        "metric": METRIC, "value": round(us_query, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": round(us_query / PUBLISHED_US[args.pq], 5) if args.pq in PUBLISHED_US else None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 K/V, 64 planted keys/head, catalog built on GPU)",
        "config": workload_config(args, world),
        "gpu_launches": None, "roofline": roofline, "step_roofline": step_roofline, "clocks": clocks, "e2e": e2e,
        "write_path": write_path_summary(args, write, local_keys, peak),
        "wall_s_timed": round(wall, 3),
    }
    launches_per_query = 3 if grid_schedule else 1
    if world > 1:
        launches_per_query = 3 + shard.extra_launches
    line["gpu_launches"] = launches_per_query * qps * args.steps
    if world == 1 and args.throughput_heads > 0:
        line["throughput"] = throughput_measure(args, device, peak)
    if world == 1 and args.inverted:
        line["inverted_static"] = inverted_measure(args, sets, device)
    if world == 1 and args.ragged:
        line["ragged_paged"] = ragged_measure(args, device, peak)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        times, threads = run_cpu_decoder(args, 1000, 1, args.cpu_seconds)
        cpu_us = 1e6 * sum(times) / len(times)
        line["cpu_baseline"] = {"value": round(cpu_us, 1), "unit": UNIT, "cores": threads, "kind": "port",
                                "sample": f"{len(times)} query tokens x {args.heads} heads x {args.keys} keys "
                                          f"({args.pq}), random catalog"}
    if rank == 0:
        emit(line)
    if group is not None:
        del graph
        torch.distributed.barrier(group)
        torch.distributed.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------------------------
# model-level decode (BASELINE configs 3 and 4): tokens/s through patch_llama_attention
# ---------------------------------------------------------------------------------------------

def smollm2_model(device, layers: int = 30):
    """Random-init Llama with the SmolLM2-135M shape (seed 0), bf16, SDPA attention for the
    unpatched layers."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=49152, hidden_size=576, intermediate_size=1536, num_hidden_layers=layers,
                      num_attention_heads=9, num_key_value_heads=3, head_dim=64, max_position_embeddings=65536,
                      rope_theta=100000.0, rms_norm_eps=1e-5, tie_word_embeddings=True, attn_implementation="sdpa")
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval().to(torch.bfloat16).to(device)


def random_bundle(n_layers: int, shortlist: int, budget: int, seed: int = 7):
    """Frozen random-init 2x256 artifacts for every layer (bf16 values, as real bundles store)."""
    import torch

    from sva_b200 import SVAArtifactBundle, SVALayerArtifacts

    gen = torch.Generator().manual_seed(seed)
    layers = {}
    for i in range(n_layers):
        layers[i] = SVALayerArtifacts((torch.randn(9, 64, 64, generator=gen) * 0.125).to(torch.bfloat16),
                                      (torch.randn(9, 64, 64, generator=gen) * 0.125).to(torch.bfloat16),
                                      torch.zeros(9), torch.randn(9, 2, 256, 32, generator=gen).to(torch.bfloat16),
                                      0.0, 0.0, "qk")
    manifest = {"schema_version": 1, "artifact_type": "summon_verify_attention", "rank_dim": 64,
                "coarse_subspaces": 2, "coarse_codewords": 256, "default_shortlist": shortlist,
                "default_budget": budget, "layer_count": n_layers, "layers": list(range(n_layers))}
    return SVAArtifactBundle(manifest=manifest, layers=layers)


def passkey_prompt(batch: int, context: int, seed: int = 2, digit_ids=tuple(range(48, 58))):
    """config 4 prompts: uniform random ids, a random 5-digit string of digit-token ids (ids 48-57
    stand for the digits of the random-init vocabulary) inserted at a seeded position and repeated
    at the end; ``context`` tokens in total."""
    import torch

    gen = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 49152, (batch, context), generator=gen)
    for b in range(batch):
        digits = torch.tensor([digit_ids[int(d)] for d in torch.randint(0, 10, (5,), generator=gen)])
        pos = int(torch.randint(0, context - 10, (1,), generator=gen))
        ids[b, pos:pos + 5] = digits
        ids[b, -5:] = digits
    return ids


def eager_decode(model, prompt, steps: int, device):
    """Prefill the prompt, then `steps` greedy tokens through the model's eager forward over HF's
    DynamicCache (the reference's way).  Returns (prefill_ms, decode_ms): device time of each."""
    import torch
    from transformers import DynamicCache

    with torch.no_grad():
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        out = model(input_ids=prompt.to(device), use_cache=True, past_key_values=DynamicCache(config=model.config),
                    logits_to_keep=1)
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        e1.record()
        cache = out.past_key_values
        for _ in range(steps - 1):
            out = model(input_ids=tok, use_cache=True, past_key_values=cache, logits_to_keep=1)
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
        e2.record()
        torch.cuda.synchronize()
    return e0.elapsed_time(e1), e1.elapsed_time(e2)


def graphed_decode(model, prompt, steps: int, device):
    """The same greedy decode with the per-token step captured in a CUDA graph over a StaticCache
    (sva_b200.serving.GraphedGreedyDecoder).  Returns (prefill_ms, decode_ms, e2e_ms, tokens):
    decode_ms is the device time of `steps` graph replays; e2e_ms the same replays where every
    step also moves its tokens device -> pinned host -> device (a host-driven generation loop)."""
    import torch

    from sva_b200.serving import GraphedGreedyDecoder

    batch = prompt.shape[0]
    dec = GraphedGreedyDecoder(model, batch, prompt.shape[1] + 2 * steps + 4)
    with torch.no_grad():
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        first = dec.prefill(prompt)
        e1.record()
        torch.cuda.synchronize()
        prefill_ms = e0.elapsed_time(e1)
        dec.capture()
        toks = [first, dec.warm_token]
        e0.record()
        for _ in range(steps):
            dec.step()
        e1.record()
        torch.cuda.synchronize()
        decode_ms = e0.elapsed_time(e1)
        toks.append(dec.tok.clone())
        host = torch.empty_like(dec.tok, device="cpu").pin_memory()
        e0.record()
        for _ in range(steps):
            nxt = dec.step()
            host.copy_(nxt, non_blocking=True)
            dec.tok.copy_(host, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)
    dec.release()
    return prefill_ms, decode_ms, e2e_ms, torch.cat(toks, 1)


def model_arm(args):
    """--workload cfg3 / cfg4: decode tokens/s of the patched random-init SmolLM2-shaped model."""
    import torch

    from sva_b200 import patch_llama_attention
    from sva_b200.adapter import wrap_socket_layers_with_adapters

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    model = smollm2_model(device)
    if args.workload == "cfg3":
        gen = torch.Generator().manual_seed(1)
        prompt = torch.randint(0, 49152, (1, args.model_prefill), generator=gen)
        settings = [(2048, 512, list(range(30)), False)]
        steps, batch = args.model_decode, 1
    else:
        prompt = passkey_prompt(8, args.model_prefill)
        settings = [(8192, 2048, [26, 27, 28, 29], True), (512, 128, [26, 27, 28, 29], True)]
        steps, batch = args.model_decode, 8
    # warm-up (kernel loading, library heuristics) on a short prompt, then the unpatched model
    eager_decode(model, prompt[:, :256], 4, device)
    pf, _, _, _ = graphed_decode(model, prompt, steps, device)
    _, dm, _, _ = graphed_decode(model, prompt, steps, device)
    full = {"prefill_ms": round(pf, 1), "decode_ms_per_step": round(dm / steps, 3),
            "tokens_per_s": round(batch * steps / (dm * 1e-3), 1), "path": "full attention, graphed step"}
    runs = []
    clocks = None
    for shortlist, budget, layers, adapter in settings:
        handle = patch_llama_attention(model, random_bundle(30, shortlist, budget), layers=layers,
                                       allow_batch=batch > 1)
        if adapter:
            wrap_socket_layers_with_adapters(model, layers, rank=16, scale=1.0)
            gen = torch.Generator().manual_seed(4)
            with torch.no_grad():
                for i in layers:
                    a = model.model.layers[i].self_attn
                    a.down.weight.copy_(torch.randn(a.down.weight.shape, generator=gen) * 0.02)
                    a.up.weight.copy_(torch.randn(a.up.weight.shape, generator=gen) * 0.02)
        eager_steps = min(steps, 16)
        epf, edm = eager_decode(model, prompt, eager_steps, device)
        handle.reset_catalogs()
        sampler = ClockSampler(None)
        sampler.start()
        pf, dm, em, toks = graphed_decode(model, prompt, steps, device)
        clocks = sampler.stop()
        summary = handle.stats.summary()
        handle.unpatch()
        n_tok = batch * steps
        runs.append({"shortlist": shortlist, "budget": budget, "patched_layers": len(layers), "adapter": adapter,
                     "prefill_ms": round(pf, 1), "decode_ms_per_step": round(dm / steps, 3),
                     "tokens_per_s": round(n_tok / (dm * 1e-3), 1), "e2e_tokens_per_s": round(n_tok / (em * 1e-3), 1),
                     "eager_prefill_ms": round(epf, 1), "eager_decode_ms_per_step": round(edm / (eager_steps - 1), 3),
                     "eager_tokens_per_s": round(batch * (eager_steps - 1) / (edm * 1e-3), 1),
                     "avg_summoned": summary.get("avg_summoned"), "avg_verified": summary.get("avg_verified")})
    head = runs[0]
    line = {
        "metric": "decode tok/s" + (" @32k" if args.workload == "cfg4" else " @8k"), "value": head["tokens_per_s"],
        "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": 1,
        "ms_per_step": head["decode_ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init SmolLM2-135M-shaped model and artifacts, random token ids)",
        "config": {"workload": (f"cfg3: 30-layer SmolLM2-135M shape, all layers SVA 2x256 (2048/512), prefill "
                                f"{args.model_prefill}, greedy decode {steps}, batch 1") if args.workload == "cfg3" else
                   (f"cfg4: late4 socket (layers 26-29 SVA + rank-16 residual adapters), context "
                    f"{args.model_prefill}, batch 8, greedy decode {steps}; shortlist/budget 8192/2048 and 512/128"),
                   "path": "HF LlamaForCausalLM patched by sva_b200.patch_llama_attention; per-token step in one CUDA "
                           "graph over a StaticCache (sva_b200.serving.GraphedGreedyDecoder); eager DynamicCache "
                           "loop reported beside it"},
        "e2e": {"value": head["e2e_tokens_per_s"], "unit": "tokens/s", "h2d_bytes_per_step": 8 * batch,
                "d2h_bytes_per_step": 8 * batch},
        "runs": runs, "full_attention": full, "clocks": clocks, "gpu_launches": None,
    }
    emit(line)
    return 0


def ctypes_voidp_array(vals):
    import ctypes

    arr = (ctypes.c_void_p * len(vals))(*vals)
    return arr


def e2e_measure(args, sets, one_query, device, group, host_query=None):
    """Each step moves the query token of every head from pinned host memory to the GPU, runs the
    public decode op, and moves the output back to pinned host memory; time per query on the
    device clock.  With host_query (one GPU), the public op is given the pinned host tensors
    themselves and its kernels read q from and write out to host memory; otherwise the step
    copies them with torch around the op."""
    import torch

    n = args.e2e_queries
    st_list = [sets[i % len(sets)] for i in range(n)]
    host_q = [st["q"].cpu().pin_memory() for st in sets]
    host_out = [torch.empty_like(st["out"], device="cpu").pin_memory() for st in sets]
    for i in range(4):
        st = st_list[i % len(st_list)]
        if host_query is not None:
            host_query(st, host_q[i % len(sets)], host_out[i % len(sets)])
        else:
            one_query(st)
    torch.cuda.synchronize()
    if group is not None:
        torch.distributed.barrier(group)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(n):
        st = st_list[i]
        k = i % len(sets)
        if host_query is not None:
            host_query(st, host_q[k], host_out[k])
        else:
            st["q"].copy_(host_q[k], non_blocking=True)
            one_query(st)
            host_out[k].copy_(st["out"], non_blocking=True)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    if group is not None:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
        ms = float(t.item())
    qbytes = sets[0]["q"].numel() * sets[0]["q"].element_size()
    obytes = sets[0]["out"].numel() * sets[0]["out"].element_size()
    return {"value": round(1000.0 * ms / n, 3), "unit": UNIT, "h2d_bytes_per_step": qbytes,
            "d2h_bytes_per_step": obytes, "queries": n,
            "path": ("sva_b200.kernels.decode (eager calls per query) given pinned host q and out; its kernels "
                     "read q from and write out to host memory" if host_query is not None else
                     "sva_b200.sharded.ShardedDecoder.decode (eager calls per query) with torch copies of pinned "
                     "host q and out around it")}


# The JSON line is the only thing bench.py writes to its standard output: file descriptor 1 is
# pointed at stderr for everything else (NCCL's version banner, library messages), and the line
# goes to a duplicate of the original stdout.
_JSON_OUT = None


def emit(line: dict) -> None:
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    args = parse_args()
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload in ("cfg3", "cfg4"):
        if args.model_prefill is None:
            args.model_prefill = 8192 if args.workload == "cfg3" else 32768
        if args.model_decode is None:
            args.model_decode = 256 if args.workload == "cfg3" else 64
        return model_arm(args)
    return gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
