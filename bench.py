#!/usr/bin/env python
"""SVA decode benchmark on B200: microseconds per query at 2^20 cached keys (summon + verify).

Workload (in the 9-head shape the reference publishes its million-key numbers
on): ``--sequences`` independent caches ("sequences", 16 by default) of 2^20 keys per head, 9
heads each, head_dim 64, rank 64, bf16 K/V ~ N(0,1) with 64 planted near-duplicates per head,
4x64 codes (default) or 1x256, shortlist 2048, budget 512.  A query is one decode token of one
sequence over its 9 heads.

Headline (``value``, every N): serving mode.  One decode call takes the next token of every
sequence (16 queries, 144 (head, query) problems); a step is ``--tokens-per-step`` such calls
(256 queries), and value = step time / queries.  Each call touches 16 x ~44 MB, far more than
the 126 MB L2.  On one GPU the step is one CUDA-graph replay of sva_decode_batched calls; on N
GPUs (``torchrun --nproc-per-node N``) every sequence's keys are split by key range and each call
runs the batched shard stages with three NCCL all-gathers (sva_b200.sharded.BatchedShardedDecoder);
value is the max over ranks.  Inputs are resident in HBM; catalogs are built by the CUDA write path.

Beside it (one GPU): ``latency``, the decode of one query at a time (a 256-query graph over the
first four sequences: the single-sequence latency), ``ragged_paged`` (config 5: 64 ragged
sequences in a paged catalog; at N > 1 page-dealt over the ranks), ``inverted_static`` (the
static inverted-index summon), ``write_path`` and ``cpu_baseline``.

``--impl reference`` times the CPU restatement of the reference path (oracle/cpu_baseline.py;
the reference itself is PyTorch code that cannot be shipped to the GPU host) on the same
configuration with all host threads.  ``--workload cfg3 / cfg4`` measure model-level decode
tokens/s instead (see model_arm).
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
    ap.add_argument("--sequences", type=int, default=16, help="independent million-key caches decoded together")
    ap.add_argument("--tokens-per-step", type=int, default=16, help="serving calls (tokens of every sequence) per step")
    ap.add_argument("--sets", type=int, default=4, help="sequences the latency measurement rotates over")
    ap.add_argument("--queries-per-step", type=int, default=256, help="queries per step of the latency measurement")
    ap.add_argument("--e2e-queries", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-1x256", dest="alt_pq", action="store_false",
                    help="skip the 1x256-code serving and latency measurement of the same sequences")
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
        # nvidia-smi can take a second to start on a many-GPU box: wait for its first sample
        deadline = time.time() + 10.0
        while not self.lines and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self) -> None:
        """Call at the start of the timed region: stop() reports the samples taken from here on."""
        self._mark = len(self.lines)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        # a short timed region may end between two samples: take at least two after the mark
        first = getattr(self, "_mark", 0)
        deadline = time.time() + 1.0
        while len(self.lines) < first + 2 and time.time() < deadline and self.proc.poll() is None:
            time.sleep(0.01)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._thread:
            self._thread.join(timeout=2)
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[first:]:
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
        "workload": f"cfg2 million-key decode, serving mode: {args.sequences} sequences x {args.keys} keys x "
                    f"{args.heads} heads, {args.pq} codes, shortlist {args.shortlist}, budget {args.budget}; one call "
                    f"decodes one token of every sequence, {args.tokens_per_step} calls per step",
        "keys": args.keys, "heads": args.heads, "pq": args.pq, "shortlist": args.shortlist, "budget": args.budget,
        "head_dim": 64, "rank_dim": 64, "sequences": args.sequences,
        "queries_per_step": args.sequences * args.tokens_per_step,
        "parallelism": "single GPU" if world == 1 else f"key-range shards x{world}",
        "l2": f"every call touches {args.sequences} x ~{algorithmic_bytes(args)['total'] / 1e6:.0f} MB > 126 MB L2",
    }


def build_batch(args, device, rank: int, world: int, keep_full_first: bool = False):
    """The serving batch for this rank: q [N, H, 1, D], artifacts shared by the sequences (one
    layer), and this rank's key range [lo, hi) of every sequence: codes [N, H, L_r, S], k_low
    [N, H, L_r, R], keys / values [N, H, L_r, D] (one KV head per query head).  Every rank draws
    the same full caches (seeded per sequence on the device) and keeps its slice, so the shards
    are exactly the one-GPU data.  With keep_full_first, sequence 0's full arrays are returned too
    (the parity check of the sharded runs)."""
    import torch

    from sva_b200 import kernels

    s_sub, c = pq_shape(args.pq)
    n, heads, keys, d, r = args.sequences, args.heads, args.keys, 64, 64
    lo, hi = keys * rank // world, keys * (rank + 1) // world
    gen = torch.Generator().manual_seed(args.seed * 1000 + 17)
    q = torch.randn(n, heads, 1, d, generator=gen).to(torch.bfloat16)
    q_proj = (torch.randn(heads, d, r, generator=gen) * 0.125).to(torch.bfloat16).float().to(device)
    k_proj = (torch.randn(heads, d, r, generator=gen) * 0.125).to(torch.bfloat16).float().to(device)
    cb = torch.randn(heads, s_sub, c, r // s_sub, generator=gen).to(torch.bfloat16).float().to(device)
    planted = torch.stack([torch.stack([torch.randperm(keys, generator=gen)[:64] for _ in range(heads)])
                           for _ in range(n)])
    noise = torch.randn(n, heads, 64, d, generator=gen)
    L = hi - lo
    kk = torch.empty(n, heads, L, d, dtype=torch.bfloat16, device=device)
    vv = torch.empty(n, heads, L, d, dtype=torch.bfloat16, device=device)
    k_low = torch.empty(n, heads, L, r, dtype=torch.float32, device=device)
    codes = torch.empty(n, heads, L, s_sub, dtype=torch.uint8, device=device)
    full_first = None
    write = {}
    for i in range(n):
        dgen = torch.Generator(device=device).manual_seed(args.seed * 1000 + i + 7)
        fk = torch.empty(heads, keys, d, dtype=torch.bfloat16, device=device)
        fv = torch.empty(heads, keys, d, dtype=torch.bfloat16, device=device)
        for h in range(heads):
            fk[h] = torch.randn(keys, d, generator=dgen, device=device).to(torch.bfloat16)
            fv[h] = torch.randn(keys, d, generator=dgen, device=device).to(torch.bfloat16)
            fk[h, planted[i, h].to(device)] = (0.9 * q[i, h, 0].float()[None, :] + 0.1 * noise[i, h]).to(
                torch.bfloat16).to(device)
        kk[i], vv[i] = fk[:, lo:hi], fv[:, lo:hi]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        kernels.catalog_encode(kk[i], k_proj, cb, 0, L, k_low[i], codes[i])
        e1.record()
        if i == 0:
            torch.cuda.synchronize()
            write["exact_ms_per_set"] = e0.elapsed_time(e1)
            # the tensor-core write path of the same keys, into scratch buffers (reported only)
            tc = kernels.tensor_core_write_ok(kk[0], k_proj)
            write["tensor_cores"] = bool(tc)
            if tc:
                k2, c2 = torch.empty_like(k_low[0]), torch.empty_like(codes[0])
                status = torch.zeros(1, dtype=torch.int32, device=device)
                e0.record()
                kernels.catalog_encode(kk[0], k_proj, cb, 0, L, k2, c2, tensor_cores=True, status=status)
                e1.record()
                torch.cuda.synchronize()
                write["tc_ms_per_set"] = e0.elapsed_time(e1)
                del k2, c2
            if keep_full_first and world > 1:
                fl = torch.empty(heads, keys, r, dtype=torch.float32, device=device)
                fc = torch.empty(heads, keys, s_sub, dtype=torch.uint8, device=device)
                kernels.catalog_encode(fk, k_proj, cb, 0, keys, fl, fc)
                full_first = dict(keys=fk, values=fv, k_low=fl, codes=fc)
        del fk, fv
    torch.cuda.synchronize()
    return dict(q=q.to(device), q_proj=q_proj, scale=torch.ones(heads, dtype=torch.float32, device=device), cb=cb,
                codes=codes, k_low=k_low, keys=kk, values=vv, offset=lo, write=write, full_first=full_first,
                k_proj=k_proj)


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
    us = 1000.0 * s.elapsed_time(e) / n
    # algorithmic bytes: every visited posting entry (4-byte id) and its k_low row (256 bytes), and
    # the verify's K and V rows of the budget (bf16)
    entries = st[1] / n
    nbytes = entries * (4 + 64 * 4) + st[4] / n * 64 * 2 * 2
    peak, peak_kind = measured_peaks()
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"summon": "inverted_static", "us_per_query": round(us, 2),
            "cells_per_subspace": cells, "budget": args.budget, "queries": n,
            "cell_visits_per_query": round(st[5] / n, 1), "posting_entries_per_query": round(entries, 1),
            "verified_per_query": round(st[4] / n, 1),
            "roofline": {"bound": "hbm", "algorithmic_bytes_per_query": int(nbytes), "achieved": round(gbs, 1),
                         "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4), "peak_kind": peak_kind},
            "timing": "eager calls over the rotating catalog sets, device clock"}


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


def ragged_sharded_measure(args, device, peak: float, group) -> dict:
    """Config 5 on N GPUs: the pages of every sequence are dealt round-robin over the ranks (global
    page g of a sequence on rank g % N); each call runs the batched shard stages over the rank's own
    pages with three NCCL all-gathers (page-dealt BatchedShardedDecoder).  Every rank draws the
    same page pool and keeps a page table of its own pages only.  Rank 0 checks the result against
    the one-GPU batched decode of all pages before timing; eager calls, device-timed, max over
    ranks."""
    import torch
    import torch.distributed as dist

    from sva_b200 import kernels, sharded

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    st = ragged_paged_set(device)
    pk = st["page_keys"]
    n_seqs, heads = st["q"].shape[0], st["q"].shape[1]
    table = st["table"].cpu()
    rows, lens = [], []
    for b, n in enumerate(st["lengths"]):
        n_pages = (n + pk - 1) // pk
        mine = list(range(rank, n_pages, world))
        rows.append([int(table[b, g]) for g in mine])
        last = n - (n_pages - 1) * pk
        lens.append(sum(pk if g < n_pages - 1 else last for g in mine))
    width = max(1, max(len(x) for x in rows))
    local = torch.zeros(n_seqs, width, dtype=torch.int32)
    for b, x in enumerate(rows):
        if x:
            local[b, :len(x)] = torch.tensor(x, dtype=torch.int32)
    local = local.to(device)
    seq_lens = torch.tensor(lens, dtype=torch.int64, device=device)
    dec = sharded.BatchedShardedDecoder(group, args.shortlist, args.budget, device)
    out = torch.empty(n_seqs, heads, 1, 64, dtype=torch.bfloat16, device=device)

    def call(saturated=None):
        dec.decode(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"], st["values"],
                   seq_lens=seq_lens, page_table=local, max_len=width * pk, page_dealt=True, out=out, logits_mode=1,
                   softmax_scale=0.125, saturated=saturated)

    call()
    torch.cuda.synchronize()
    parity = None
    if rank == 0:
        ref = kernels.decode_batched(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"],
                                     st["values"], args.shortlist, args.budget, seq_lens=st["seq_lens"],
                                     page_table=st["table"], max_len=max(st["lengths"]), softmax_scale=0.125,
                                     logits_mode=1)
        torch.cuda.synchronize()
        parity = "ok" if torch.equal(ref, out) else "MISMATCH"
    # 8 calls (kernels and all-gathers) in one CUDA graph; saturation flags read once per replay
    calls = 8
    flags = torch.zeros(calls, dtype=torch.int32, device=device)
    ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(7)]
    for e in ev:
        e.record()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    gstream = torch.cuda.Stream(device)
    with torch.cuda.stream(gstream):
        call()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=gstream):
            flags.zero_()
            for i in range(calls):
                dec.stage_events = ev if i == 0 else None
                call(flags[i:i + 1])
            dec.stage_events = None
    torch.cuda.synchronize()
    repeats = 0
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier(group)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        graph.replay()
        bad = int(flags.sum().item())
        if bad:
            repeats += bad
            with dec.full_width():
                for _ in range(bad):
                    call()
    e1.record()
    torch.cuda.synchronize()
    us = 1000.0 * e0.elapsed_time(e1) / (reps * calls)
    t = torch.tensor([us], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    us = float(t.item())
    del graph
    names = ["summon", "gather_top", "rescore", "gather_records", "verify_gather_partials", "combine"]
    stages = {n: round(1000.0 * ev[j].elapsed_time(ev[j + 1]), 2) for j, n in enumerate(names)}
    total_keys = sum(st["lengths"])
    sl_eff = sum(min(args.shortlist, n) for n in st["lengths"])
    b_eff = sum(min(args.budget, args.shortlist, n) for n in st["lengths"])
    nbytes = heads * (total_keys * 4 + sl_eff * 64 * 4 + b_eff * 64 * 2 * 2) + heads * (64 * 64 * 4 + 64 * 64 * 4)
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": f"cfg5 ragged paged decode, page-dealt over {world} GPUs: {n_seqs} sequences (total "
                        f"{total_keys} keys), 9 query / 3 KV heads, 4x64 codes, {pk}-key pages",
            "us_per_step": round(us, 2), "tokens_per_s": round(n_seqs / (us * 1e-6), 1),
            "algorithmic_bytes_per_step": int(nbytes), "achieved_gbs_aggregate": round(gbs, 1),
            "frac_of_n_gpu_peak": round(gbs / (peak * world), 4), "stage_us_rank0_view": stages,
            "exchange_width": dec.width, "saturation_repeats": repeats, "parity": parity,
            "timing": "CUDA graph of 8 calls (kernels + NCCL all-gathers), 3 replays after 3 warm-ups, device clock, "
                      "max over ranks; stage times from events captured in the first call"}


def inverted_sharded_measure(args, batch, device, group) -> dict:
    """The static inverted-index summon with every sequence's static catalog split by key range
    (ShardedInvertedDecoder: the ranks' top-budget candidate records, then the fp64 partial
    outputs, two NCCL all-gathers), over the first --sets sequences; posting lists over each
    rank's keys built once, the global largest list from one all-reduce; eager calls,
    device-timed, max over ranks.  Rank 0 checks sequence 0 against the one-GPU static decode."""
    import torch
    import torch.distributed as dist

    from sva_b200 import kernels, sharded

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    C = int(batch["cb"].shape[2])
    seqs = [seq_view(batch, i) for i in range(args.sets)]
    posts = [kernels.postings_build(st["codes"], C) for st in seqs]
    gmax = [sharded.global_max_bucket(pp, group) for pp in posts]
    dec = sharded.ShardedInvertedDecoder(group, args.budget, cells=8)
    outs = [torch.empty(st["q"].shape[0], st["q"].shape[2], dtype=st["q"].dtype, device=device) for st in seqs]
    holds = rank == world - 1

    def one(i):
        st = seqs[i % len(seqs)]
        dec.decode(st["q"][:, 0, :], st["q_proj"], st["scale"], st["cb"], st["codes"], posts[i % len(seqs)],
                   st["k_low"], st["keys"], st["values"], key_offset=batch["offset"], holds_current=holds,
                   global_max_bucket=gmax[i % len(seqs)], out=outs[i % len(seqs)], softmax_scale=0.125)

    one(0)
    torch.cuda.synchronize()
    parity = None
    if rank == 0 and batch.get("full_first") is not None:
        f = batch["full_first"]
        fp = kernels.postings_build(f["codes"], C)
        ref = kernels.decode_inverted(batch["q"][0][:, 0, :], batch["q_proj"], batch["scale"], batch["cb"], f["codes"],
                                      fp, f["k_low"], f["keys"], f["values"], args.budget, 8, args.budget, args.budget,
                                      dynamic=False, softmax_scale=0.125)
        torch.cuda.synchronize()
        parity = "ok" if torch.equal(ref, outs[0]) else "MISMATCH"
    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    dist.barrier(group)
    n = 16
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(n):
        one(i)
    e1.record()
    torch.cuda.synchronize()
    us = 1000.0 * e0.elapsed_time(e1) / n
    t = torch.tensor([us], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return {"summon": "inverted_static, key-range shards", "us_per_query": round(float(t.item()), 2),
            "cells_per_subspace": 8, "budget": args.budget, "queries": n, "parity": parity,
            "timing": "eager calls over the first sequences, device clock, max over ranks"}


def write_path_summary(args, write: dict, local_keys: int, peak: float) -> dict:
    """The catalog write of one sequence (all heads): keys/s, projection TFLOP/s and the fraction of
    the measured HBM peak its algorithmic bytes reach (K read as bf16, k_low fp32 written, codes)."""
    s, _ = pq_shape(args.pq)
    keys = args.heads * local_keys
    flops = 2.0 * keys * 64 * 64
    nbytes = keys * (64 * 2 + 64 * 4 + s)
    import torch

    c = pq_shape(args.pq)[1]
    # the exact path is bound by fp32 CUDA-core issue: every product and every sum is its own
    # rounded instruction (no fused multiply-add), per key and head 2*D*R for the projection,
    # 2*R*C for the codeword dot products, 2*R for |x|^2 and 3*S*C for the distances
    ops = keys * (2.0 * 64 * 64 + 2.0 * 64 * c + 2.0 * 64 + 3.0 * s * c)
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    op_peak = sms * 128 * 1.965e9
    out = {"path": "exact CUDA-core projection and assignment (the adapter's default)"}
    for name, key in (("exact_", "exact_ms_per_set"), ("tc_", "tc_ms_per_set")):
        ms = write.get(key)
        if ms is None:
            continue
        out[name + "ms_per_set"] = round(ms, 3)
        out[name + "keys_per_s"] = round(keys / (ms * 1e-3), 1)
        out[name + "projection_tflops"] = round(flops / (ms * 1e-3) / 1e12, 3)
        out[name + "hbm_frac"] = round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)
    if write.get("exact_ms_per_set"):
        out["exact_fp32_ops_per_set"] = int(ops)
        out["exact_cuda_core_frac"] = round(ops / (write["exact_ms_per_set"] * 1e-3) / op_peak, 4)
        out["cuda_core_peak"] = f"{sms} SMs x 128 fp32 lanes x 1.965 GHz (nominal max clock)"
    out["algorithmic_bytes_per_set"] = int(nbytes)
    return out


def seq_view(batch, i: int) -> dict:
    """Sequence i of the serving batch as single-sequence decode arguments."""
    return dict(q=batch["q"][i], q_proj=batch["q_proj"], scale=batch["scale"], cb=batch["cb"], codes=batch["codes"][i],
                k_low=batch["k_low"][i], keys=batch["keys"][i], values=batch["values"][i])


def profiled_graph(calls, n_calls: int, device, n_prof: int):
    """A CUDA graph of n_calls calls whose first call records the library's per-kernel events."""
    import torch

    from sva_b200 import _lib

    prof = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(n_prof + 1)]
    for e in prof:
        e.record()
    torch.cuda.synchronize()
    handles = ctypes_voidp_array([e.cuda_event for e in prof[1:]])
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        calls(0)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(n_calls):
                if i == 0:
                    prof[0].record()
                    _lib.load().sva_profile_events(handles, n_prof)
                try:
                    calls(i)
                finally:
                    if i == 0:
                        _lib.load().sva_profile_events(None, 0)
    torch.cuda.synchronize()
    return graph, prof


def latency_measure(args, batch, device, peak: float) -> dict:
    """One query at a time (the single-sequence decode latency): a CUDA graph of
    --queries-per-step single-sequence decodes cycling over the first --sets sequences (each query
    touches ~44 MB and the cycle ~176 MB > L2), device-timed after warm-up, with the per-kernel
    split of the first query and the end-to-end decode with pinned host q and out."""
    import torch

    from sva_b200 import kernels

    sets = [seq_view(batch, i) for i in range(min(args.sets, args.sequences))]
    outs = [torch.empty_like(st["q"]) for st in sets]

    def one(i, q=None, out=None):
        st = sets[i % len(sets)]
        kernels.decode(st["q"] if q is None else q, st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"],
                       st["keys"], st["values"], args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1,
                       out=outs[i % len(sets)] if out is None else out)

    qps = args.queries_per_step
    graph, prof = profiled_graph(one, qps, device, 3)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(2, args.steps // 2)
    kern = []
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = 1000.0 * e0.elapsed_time(e1) / (reps * qps)
    graph.replay()
    torch.cuda.synchronize()
    kern = {n: round(1000.0 * prof[j].elapsed_time(prof[j + 1]), 2) for j, n in enumerate(["prep", "scan", "finish"])}
    del graph
    ab = algorithmic_bytes(args)
    kb = {"prep": ab["codebooks"] + ab["q_proj"], "scan": ab["codes"], "finish": ab["rescore"] + ab["verify"]}
    dom = max(kern, key=kern.get)
    # end to end: pinned host q and out handed to the public op, read / written by its kernels
    hq = [st["q"].cpu().pin_memory() for st in sets]
    ho = [torch.empty_like(st["q"], device="cpu").pin_memory() for st in sets]
    for i in range(4):
        one(i, hq[i % len(sets)], ho[i % len(sets)])
    torch.cuda.synchronize()
    n = args.e2e_queries
    e0.record()
    for i in range(n):
        one(i, hq[i % len(sets)], ho[i % len(sets)])
    e1.record()
    torch.cuda.synchronize()
    e2e = 1000.0 * e0.elapsed_time(e1) / n
    gbs = ab["total"] / (us * 1e-6) / 1e9
    return {"us_per_query": round(us, 3), "e2e_us_per_query": round(e2e, 3),
            "kernel_us_first_query": kern, "kernel_share": {k: round(v / sum(kern.values()), 3) for k, v in kern.items()},
            "dominant": dom, "dominant_achieved_gbs": round(kb[dom] / (kern[dom] * 1e-6) / 1e9, 1),
            "algorithmic_bytes_per_query": int(ab["total"]), "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
            "vs_published_h100": round(us / PUBLISHED_US[args.pq], 5) if args.pq in PUBLISHED_US else None,
            "timing": f"CUDA graph of {qps} single-query decodes over {len(sets)} sequences, device clock; e2e: "
                      f"{n} eager calls with pinned host q / out"}


def pq_1x256_measure(args, batch, device, peak: float) -> dict:
    """The same sequences with 1x256 codes (the reference's best published PQ setting, 0.649 ms on
    an H100): a 1x256 codebook per head, every sequence's codes written by the library, then the
    serving call (CUDA graph of --tokens-per-step calls) and the single-query latency (CUDA graph
    of 64 queries over --sets sequences), device-timed after warm-ups; sequence 0 of a serving
    call is checked against its single-sequence decode."""
    import argparse

    import torch

    from sva_b200 import kernels

    heads, n, L = args.heads, args.sequences, int(batch["codes"].shape[2])
    gen = torch.Generator().manual_seed(args.seed * 1000 + 256)
    cb = torch.randn(heads, 1, 256, 64, generator=gen).to(torch.bfloat16).float().to(device)
    codes = torch.empty(n, heads, L, 1, dtype=torch.uint8, device=device)
    for i in range(n):
        kernels.catalog_encode(batch["keys"][i], batch["k_proj"], cb, 0, L, None, codes[i])
    out = torch.empty_like(batch["q"])

    def serve(i=0):
        kernels.decode_batched(batch["q"], batch["q_proj"], batch["scale"], cb, codes, batch["k_low"], batch["keys"],
                               batch["values"], args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1,
                               out=out)

    def timed(graph, reps):
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return 1000.0 * e0.elapsed_time(e1) / reps

    calls = args.tokens_per_step
    graph, _ = profiled_graph(lambda i: serve(), calls, device, 3)
    serve_us = timed(graph, max(2, args.steps // 2)) / (calls * n)
    del graph
    st0 = dict(seq_view(batch, 0), cb=cb, codes=codes[0])
    ref = kernels.decode(st0["q"], st0["q_proj"], st0["scale"], cb, codes[0], st0["k_low"], st0["keys"], st0["values"],
                         args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1)
    torch.cuda.synchronize()
    parity = bool(torch.equal(ref, out[0]))
    sets = [dict(seq_view(batch, i), codes=codes[i]) for i in range(min(args.sets, n))]
    outs = [torch.empty_like(x["q"]) for x in sets]

    def one(i):
        x = sets[i % len(sets)]
        kernels.decode(x["q"], x["q_proj"], x["scale"], cb, x["codes"], x["k_low"], x["keys"], x["values"],
                       args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1, out=outs[i % len(sets)])

    graph, _ = profiled_graph(one, 64, device, 3)
    lat_us = timed(graph, max(2, args.steps // 2)) / 64
    del graph, codes
    ab = algorithmic_bytes(argparse.Namespace(**{**vars(args), "pq": "1x256"}))
    return {"serving_us_per_query": round(serve_us, 3), "latency_us_per_query": round(lat_us, 3),
            "vs_published_h100": round(lat_us / PUBLISHED_US["1x256"], 5),
            "algorithmic_bytes_per_query": int(ab["total"]),
            "serving_frac": round(ab["total"] / (serve_us * 1e-6) / 1e9 / peak, 4),
            "parity": ("ok" if parity else "MISMATCH") + ": sequence 0 of the serving call vs its single-sequence decode",
            "timing": f"CUDA graphs ({calls} serving calls of {n} sequences; 64 single queries), device clock"}


def cpu_parity_and_baseline(args, batch, device) -> tuple[dict, str]:
    """The cpu_baseline leg: the oracle's threaded CPU decoder on sequence 0's own catalog (copied to
    the host), timed on all host threads over a bounded sample, and its final sets and outputs
    compared with the GPU's decode of the same sequence (the bench's parity check)."""
    import torch

    from oracle.cpu_baseline import CpuDecoder
    from sva_b200 import kernels

    st = seq_view(batch, 0)
    out, _, fin = kernels.decode(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"],
                                 st["values"], args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1,
                                 want_final=True)
    torch.cuda.synchronize()
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    q = st["q"].float().cpu().numpy()[:, 0]
    dec = CpuDecoder(st["q_proj"].cpu().numpy(), st["scale"].cpu().numpy(), st["cb"].cpu().numpy(),
                     st["codes"].cpu().numpy(), st["k_low"].cpu().numpy(), bits(st["keys"]), bits(st["values"]),
                     groups=1, threads=os.cpu_count() or 1)
    ref_out, ref_fin = dec(q, args.shortlist, args.budget, 0.125, "bf16", 1, want_final=True)
    got_fin = fin.cpu().numpy()
    ok_sets = all(np.array_equal(got_fin[h, 0][got_fin[h, 0] >= 0], ref_fin[h]) for h in range(args.heads))
    err = float(np.abs(out.float().cpu().numpy()[:, 0] - ref_out).max())
    parity = ("ok" if ok_sets and err <= 2e-2 else "MISMATCH") + (
        f": final sets {'bit-exact' if ok_sets else 'differ'} vs the CPU oracle decoder on sequence 0, "
        f"max |out - oracle| = {err:.2e} (bf16 tolerance 2e-2)")
    times = []
    t_end = time.perf_counter() + args.cpu_seconds
    while True:
        t0 = time.perf_counter()
        dec(q, args.shortlist, args.budget, 0.125, "bf16", 1)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and len(times) >= 2:
            break
    dec.close()
    cpu_us = 1e6 * sum(times) / len(times)
    return ({"value": round(cpu_us, 1), "unit": UNIT, "cores": dec.threads, "kind": "port",
             "sample": f"{len(times)} query tokens x {args.heads} heads x {args.keys} keys ({args.pq}) of sequence 0's "
                       f"catalog"}, parity)


def gpu_arm(args):
    import torch

    from sva_b200 import kernels

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
    batch = build_batch(args, device, rank, world, keep_full_first=(rank == 0))
    local_keys = int(batch["codes"].shape[2])
    out = torch.empty_like(batch["q"])
    peak, peak_kind = measured_peaks()

    if world == 1:
        def serve(i=0, q=None, o=None):
            return kernels.decode_batched(batch["q"] if q is None else q, batch["q_proj"], batch["scale"], batch["cb"],
                                          batch["codes"], batch["k_low"], batch["keys"], batch["values"],
                                          args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1,
                                          out=out if o is None else o)
        shard = None
    else:
        from sva_b200 import sharded

        shard = sharded.BatchedShardedDecoder(group, args.shortlist, args.budget, device)

        def serve(i=0, q=None, o=None):
            return shard.decode(batch["q"] if q is None else q, batch["q_proj"], batch["scale"], batch["cb"],
                                batch["codes"], batch["k_low"], batch["keys"], batch["values"],
                                key_offset=batch["offset"], out=out if o is None else o, logits_mode=1,
                                softmax_scale=0.125)

    # parity before timing: sequence 0 of a serving call against the one-GPU single-sequence decode
    serve()
    torch.cuda.synchronize()
    parity_serve = None
    if rank == 0:
        if world == 1:
            st = seq_view(batch, 0)
            ref = kernels.decode(st["q"], st["q_proj"], st["scale"], st["cb"], st["codes"], st["k_low"], st["keys"],
                                 st["values"], args.shortlist, args.budget, softmax_scale=0.125, logits_mode=1)
        else:
            f = batch["full_first"]
            ref = kernels.decode(batch["q"][0], batch["q_proj"], batch["scale"], batch["cb"], f["codes"], f["k_low"],
                                 f["keys"], f["values"], args.shortlist, args.budget, softmax_scale=0.125,
                                 logits_mode=1)
        torch.cuda.synchronize()
        parity_serve = bool(torch.equal(ref, out[0]))

    calls = args.tokens_per_step
    n_q = args.sequences * calls
    kern = None
    repeats = [0]
    if world == 1:
        graph, prof = profiled_graph(lambda i: serve(), calls, device, 3)
        run_step = graph.replay
    else:
        # the step's sharded calls (kernels and NCCL all-gathers) in one CUDA graph; each call ORs
        # its saturation flag into its own slot, read once per step; a flagged call is repeated
        # at full width inside the step (exactness), and counted
        flags = torch.zeros(calls, dtype=torch.int32, device=device)
        stage_ev = [torch.cuda.Event(enable_timing=True, external=True) for _ in range(7)]
        for e in stage_ev:
            e.record()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        gstream = torch.cuda.Stream(device)
        with torch.cuda.stream(gstream):
            serve()  # warm the workspaces on the capture stream
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=gstream):
                flags.zero_()
                for i in range(calls):
                    shard.stage_events = stage_ev if i == 0 else None
                    shard.decode(batch["q"], batch["q_proj"], batch["scale"], batch["cb"], batch["codes"],
                                 batch["k_low"], batch["keys"], batch["values"], key_offset=batch["offset"], out=out,
                                 logits_mode=1, softmax_scale=0.125, saturated=flags[i:i + 1])
                shard.stage_events = None
        torch.cuda.synchronize()

        def run_step():
            graph.replay()
            bad = int(flags.sum().item())
            if bad:
                repeats[0] += bad
                with shard.full_width():
                    for _ in range(bad):
                        serve()
    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    if group is not None:
        torch.distributed.barrier(group)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
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
    sampler.mark()
    t_wall = time.perf_counter()
    cur = torch.cuda.current_stream(device)
    for i in range(args.steps):
        starts[i].record(cur)
        run_step()
        ends[i].record(cur)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t_wall
    clocks = sampler.stop()
    ms_step = sum(starts[i].elapsed_time(ends[i]) for i in range(args.steps)) / args.steps
    if group is not None:
        t = torch.tensor([ms_step], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
        ms_step = float(t.item())
    us_query = 1000.0 * ms_step / n_q

    ab = algorithmic_bytes(args)
    local_frac = local_keys / args.keys
    per_call = {k: v * args.sequences for k, v in ab.items()}
    if world == 1:
        graph.replay()
        torch.cuda.synchronize()
        kus = {n: 1000.0 * prof[j].elapsed_time(prof[j + 1]) for j, n in enumerate(["prep", "scan", "finish"])}
        kernel_bytes = {"prep": per_call["codebooks"] + per_call["q_proj"], "scan": per_call["codes"],
                        "finish": per_call["rescore"] + per_call["verify"]}
        dom = max(kus, key=kus.get)
        achieved = kernel_bytes[dom] / (kus[dom] * 1e-6) / 1e9
        roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                    "algorithmic_bytes_per_launch": int(kernel_bytes[dom]),
                    "traffic": profile_traffic(f"serve_{args.pq}_{args.sequences}x{args.heads}h_{args.keys}", dom),
                    "kernel_us": {n: round(v, 2) for n, v in kus.items()},
                    "kernel_share": {n: round(v / sum(kus.values()), 3) for n, v in kus.items()}}
        del graph
    else:
        # per-stage device times of the first call of a replay (summon = prep + scan + local top;
        # gathers = NCCL all-gathers), from events captured in the graph
        graph.replay()
        torch.cuda.synchronize()
        ev = stage_ev
        names = ["summon", "gather_top", "rescore", "gather_records", "verify_gather_partials", "combine"]
        stages = {n: round(1000.0 * ev[j].elapsed_time(ev[j + 1]), 2) for j, n in enumerate(names)}
        scan_bytes = per_call["codes"] * local_frac
        achieved = scan_bytes / (stages["summon"] * 1e-6) / 1e9
        roofline = {"bound": "hbm", "kernel": "summon (prep + scan + local top, this rank's key range)",
                    "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "peak_kind": peak_kind, "algorithmic_bytes_per_launch": int(scan_bytes), "traffic": None,
                    "stage_us": stages, "exchange_width": shard.width, "saturation_repeats": repeats[0]}
    step_bytes = ab["total"] * local_frac
    step_gbs = step_bytes / (us_query * 1e-6) / 1e9
    step_roofline = {"algorithmic_bytes_per_query": int(step_bytes), "achieved": round(step_gbs, 1),
                     "frac": round(step_gbs / peak, 4), "peak_kind": peak_kind}
    e2e = e2e_measure(args, batch, serve, device, group)

    line = {
        "metric": METRIC, "value": round(us_query, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": round(us_query / PUBLISHED_US[args.pq], 5) if args.pq in PUBLISHED_US else None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 K/V, 64 planted keys/head, catalog built on GPU)",
        "config": workload_config(args, world),
        "gpu_launches": calls * args.steps * (3 if world == 1 else 6),
        "roofline": roofline, "step_roofline": step_roofline, "clocks": clocks, "e2e": e2e,
        "parity": ("ok" if parity_serve else "MISMATCH") + ": sequence 0 of the serving call vs the one-GPU "
                  "single-sequence decode (bit-identical output)" if rank == 0 else None,
        "write_path": write_path_summary(args, batch["write"], local_keys, peak),
        "wall_s_timed": round(wall, 3),
    }
    if world == 1:
        line["latency"] = latency_measure(args, batch, device, peak)
        if args.pq == "4x64" and args.alt_pq:
            line["pq_1x256"] = pq_1x256_measure(args, batch, device, peak)
        if args.inverted:
            line["inverted_static"] = inverted_measure(args, [seq_view(batch, i) for i in range(args.sets)], device)
    elif args.inverted:
        line["inverted_static"] = inverted_sharded_measure(args, batch, device, group)
    batch["full_first"] = None
    torch.cuda.empty_cache()
    if args.ragged:
        line["ragged_paged"] = ragged_measure(args, device, peak) if world == 1 else \
            ragged_sharded_measure(args, device, peak, group)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"], line["oracle_parity"] = cpu_parity_and_baseline(args, batch, device)
    if rank == 0:
        emit(line)
    if group is not None:
        del graph  # a graph holding NCCL calls is released before the process group
        torch.cuda.synchronize()
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
        sampler.mark()
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


def e2e_measure(args, batch, serve, device, group):
    """Serving calls through the public op with every call's queries in pinned host memory and its
    outputs returned there, device-timed per query.  One GPU: decode_batched is given the pinned
    host tensors themselves and its kernels read q and write out over PCIe; shards: the queries and
    outputs are copied with torch around BatchedShardedDecoder.decode."""
    import torch

    host_q = batch["q"].cpu().pin_memory()
    host_o = torch.empty_like(batch["q"], device="cpu").pin_memory()
    dev_q = torch.empty_like(batch["q"])
    dev_o = torch.empty_like(batch["q"])
    world = 1 if group is None else torch.distributed.get_world_size(group)

    def one():
        if world == 1:
            serve(q=host_q, o=host_o)
        else:
            dev_q.copy_(host_q, non_blocking=True)
            serve(q=dev_q, o=dev_o)
            host_o.copy_(dev_o, non_blocking=True)

    for _ in range(3):
        one()
    torch.cuda.synchronize()
    if group is not None:
        torch.distributed.barrier(group)
    n = max(1, args.e2e_queries // args.sequences)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(n):
        one()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e)
    if group is not None:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX, group=group)
        ms = float(t.item())
    nbytes = batch["q"].numel() * batch["q"].element_size()
    return {"value": round(1000.0 * ms / (n * args.sequences), 3), "unit": UNIT, "h2d_bytes_per_step": nbytes,
            "d2h_bytes_per_step": nbytes, "calls": n,
            "path": ("sva_b200.kernels.decode_batched (eager calls) given pinned host q and out; its kernels read q "
                     "from and write out to host memory" if world == 1 else
                     "sva_b200.sharded.BatchedShardedDecoder.decode (eager calls) with torch copies of pinned host q "
                     "and out around it")}


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
