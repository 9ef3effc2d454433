"""The key-range shard protocol of sva_b200.sharded on CPU ranks (gloo, world size 2 and 3).

Each rank holds a key range of a seeded config-1 cache.  ShardedDecoder runs its stages and
all-gathers with a host backend that restates every stage with the oracle's arithmetic
(coarse ADC keys, canonical selections, rank scores, logits, rounded weights, fp64 sums).  The
gathered result must equal the oracle's single-device scan decode over all keys: the same
shortlist and final sets, and the same output.  The CUDA stage kernels are checked against the
single-GPU kernel in tests/test_gpu_sharded.py.
"""

from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sva_oracle as O
from sva_b200.sharded import ShardCall, ShardedDecoder
from tests.golden.inputs import config1

KEY_LEN = 6000
SHORTLIST, BUDGET = 512, 128


def _comp(keys32: np.ndarray, idx: np.ndarray) -> np.ndarray:
    return (keys32.astype(np.uint64) << np.uint64(32)) | ((~idx.astype(np.uint64)) & np.uint64(0xFFFFFFFF))


def _as_u64(t: torch.Tensor) -> np.ndarray:
    return t.numpy().view(np.uint64)


class HostShardBackend:
    """The four stages restated on the host with the oracle's arithmetic (test infrastructure)."""

    launches_per_decode = 6

    def prepare(self, q, q_proj, scale, codebooks, codes, k_low, keys, values, *, shortlist, budget, key_offset,
                out=None, logits_mode=0, softmax_scale=None, stats=None):
        st = dict(q=q[:, 0].float().numpy(), q_proj=q_proj.numpy(), scale=scale.numpy(), cb=codebooks.numpy(),
                  codes=codes.numpy().astype(np.int64), k_low=k_low.numpy(), keys=keys.float().numpy(),
                  values=values.float().numpy(), budget=budget, scaling=softmax_scale, logits_mode=logits_mode)
        n_heads, _, d = q.shape
        if out is None:
            out = torch.empty(n_heads, 1, d, dtype=q.dtype)
        c = ShardCall(st, out, key_offset, n_heads, d, shortlist, torch.device("cpu"))
        ql = O.query_low(st["q"][:, None, :], st["q_proj"], np.zeros(n_heads, np.float32), st["scale"])
        st["ql"] = ql[:, 0]
        st["adc"] = O.adc_scores(O.build_lut(ql, st["cb"]), st["codes"], st["q_proj"].shape[-1])[:, 0]
        return c

    def summon(self, c):
        st = c.args
        top = np.zeros((c.heads, c.shortlist), dtype=np.uint64)
        for h in range(c.heads):
            sel = O.topk_canonical(st["adc"][h], c.shortlist)
            top[h, : sel.shape[0]] = _comp(O.ordered_key(st["adc"][h][sel]), sel + c.key_offset)
        return torch.from_numpy(top.view(np.int64))

    def rescore(self, c, gathered_top, world, rank):
        st = c.args
        g = _as_u64(gathered_top)  # [W, H, SL]
        rec = np.zeros((c.heads, c.shortlist, 4), dtype=np.uint32)
        rank_dim = st["q_proj"].shape[-1]
        groups = c.heads // st["keys"].shape[0]
        for h in range(c.heads):
            allc = g[:, h].reshape(-1)
            live = np.sort(allc[allc != 0])[::-1]
            thr = live[min(c.shortlist, live.shape[0]) - 1]
            st.setdefault("shortlist", {})[h] = np.sort(((~live[live >= thr]) & np.uint64(0xFFFFFFFF)).astype(np.int64))
            own = g[rank, h]
            own = own[(own != 0) & (own >= thr)]
            gidx = ((~own) & np.uint64(0xFFFFFFFF)).astype(np.int64)
            lidx = gidx - c.key_offset
            rs = O.tree_dot(st["k_low"][h, lidx], st["ql"][h][None, :]) / np.float32(math.sqrt(rank_dim))
            rc = _comp(O.ordered_key(rs), gidx)
            lg = _logits(st, h // groups, h, lidx)
            rec[h, : own.shape[0], 0] = (rc & np.uint64(0xFFFFFFFF)).astype(np.uint32)
            rec[h, : own.shape[0], 1] = (rc >> np.uint64(32)).astype(np.uint32)
            rec[h, : own.shape[0], 2] = lg.astype(np.float32).view(np.uint32)
        return torch.from_numpy(rec.view(np.int32))

    def verify(self, c, gathered_records, world, rank):
        st = c.args
        g = gathered_records.numpy().view(np.uint32)  # [W, H, SL, 4]
        dtype = _dtype(c.out)
        groups = c.heads // st["keys"].shape[0]
        part = np.zeros((c.heads, c.head_dim), dtype=np.float64)
        for h in range(c.heads):
            comp = (g[:, h, :, 1].astype(np.uint64) << np.uint64(32)) | g[:, h, :, 0].astype(np.uint64)
            lg = g[:, h, :, 2].copy().view(np.float32)
            live = np.sort(comp[comp != 0])[::-1]
            b = min(st["budget"], live.shape[0])
            thr = live[b - 1]
            fin = (comp != 0) & (comp >= thr)
            st.setdefault("final", {})[h] = np.sort(((~comp[fin]) & np.uint64(0xFFFFFFFF)).astype(np.int64))
            m = lg[fin].max()
            denom = np.exp((lg[fin] - m).astype(np.float64)).sum()  # fp64, as the oracle's verify_one
            own = fin[rank]
            gidx = ((~comp[rank][own]) & np.uint64(0xFFFFFFFF)).astype(np.int64)
            w = O.round_to((np.exp((lg[rank][own] - m).astype(np.float64)) / denom).astype(np.float32), dtype)
            v = st["values"][h // groups][gidx - c.key_offset]
            part[h] = O.round_to(w[:, None] * v, dtype).astype(np.float64).sum(axis=0)
        return torch.from_numpy(part)

    def combine(self, c, gathered_partials, world):
        tot = gathered_partials.numpy().sum(axis=0)  # rank order
        out = O.round_to(tot.astype(np.float32), _dtype(c.out))
        c.out[:, 0] = torch.from_numpy(out).to(c.out.dtype)
        return c.out


def _dtype(t: torch.Tensor) -> str:
    return {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[t.dtype]


def _logits(st, kvh, h, lidx):
    q = st["q"][h]
    k_sel = st["keys"][kvh][lidx]
    if st["logits_mode"] == 1 and st["keys"].dtype != np.float32:
        raise AssertionError("the host backend holds float32 copies")
    return O.tree_dot(k_sel, q[None, :]) * np.float32(st["scaling"])


def _case():
    case = config1(key_len=KEY_LEN)
    groups = case.n_heads // case.n_kv_heads
    k_low, codes = O.build_catalog(case.keys[0].numpy(), case.k_proj.numpy(), case.codebooks.numpy(), groups)
    return case, k_low, codes


def _rank_main(rank: int, world: int, port: int, bounds: list[int], results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case, k_low, codes = _case()
        lo, hi = bounds[rank], bounds[rank + 1]
        dec = ShardedDecoder(dist.group.WORLD, heads=case.n_heads, head_dim=64, shortlist=SHORTLIST, budget=BUDGET,
                             backend=HostShardBackend())
        backend = dec.backend
        calls = []
        prepare = backend.prepare
        backend.prepare = lambda *a, **k: calls.append(prepare(*a, **k)) or calls[-1]
        out = dec.decode(case.q[0], case.q_proj, torch.ones(case.n_heads), case.codebooks,
                         torch.from_numpy(codes[:, lo:hi].astype(np.uint8)), torch.from_numpy(k_low[:, lo:hi]),
                         case.keys[0][:, lo:hi], case.values[0][:, lo:hi], key_offset=lo, softmax_scale=0.125)
        st = calls[0].args
        results[rank] = (out[:, 0].numpy().copy(), st["shortlist"], st["final"])
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("bounds", [[0, 2500, KEY_LEN], [0, 100, 4100, KEY_LEN]])
def test_gloo_ranks_reproduce_the_single_device_decode(bounds):
    world = len(bounds) - 1
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_rank_main, args=(world, _free_port(), bounds, results), nprocs=world,
                           start_method="spawn", join=True)
        outs = [results[r] for r in range(world)]
    case, k_low, codes = _case()
    ref = O.scan_decode(case.q[0].numpy(), case.q_proj.numpy(), case.logit_scale.numpy(), case.codebooks.numpy(),
                        codes, k_low, case.keys[0].numpy(), case.values[0].numpy(), SHORTLIST, BUDGET, 0.125, "f32", 0,
                        scale=np.ones(case.n_heads, np.float32))
    for r in range(world):
        out, sl, fin = outs[r]
        for h in range(case.n_heads):
            np.testing.assert_array_equal(sl[h], ref.shortlist[h][0], err_msg=f"rank {r} shortlist head {h}")
            np.testing.assert_array_equal(fin[h], np.sort(ref.final[h][0]), err_msg=f"rank {r} final head {h}")
        np.testing.assert_allclose(out, ref.out[:, 0], rtol=1e-5, atol=1e-6, err_msg=f"rank {r}")
        np.testing.assert_array_equal(out, outs[0][0])
