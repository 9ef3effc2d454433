"""Batched shards on one GPU (sva_shard_batched_*): the ranks of a sharded batch decode run one
after another on one device, the all-gathers are emulated by stacking their outputs in rank
order, and every sequence's output must equal the one-GPU batched decode of the whole caches
(bf16: bit-identical, its fp64 sums of rounded products are exact).

* key-range shards of a ragged batch, with the narrow first exchange;
* page-dealt shards of a paged ragged batch (config 5's layout) at 2 and 4 ranks;
* an exchange width below the ranks' shares of the shortlist: the rescore stage must flag
  saturation, and the full-width repeat gives the exact result.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from sva_b200 import _lib, kernels
from sva_b200.sharded import default_exchange_width
from tests.test_gpu_batched import H, HKV, D, make_batch, paged

pytestmark = pytest.mark.gpu


def run_ranks(rank_inputs, shortlist=2048, budget=512, width=None, page_dealt=False):
    """rank_inputs[r] = dict(q, q_proj, scale, cb, codes, k_low, keys, values, seq_lens, table, max_len,
    key_offset).  Returns (outputs of every rank, saturation flag of the first pass, width used)."""
    world = len(rank_inputs)
    lib = _lib.load()
    width = default_exchange_width(shortlist, world) if width is None else width
    args = []
    for r, x in enumerate(rank_inputs):
        a, lay, out = kernels.batched_args(x["q"], x["q_proj"], x["scale"], x["cb"], x["codes"], x["k_low"],
                                           x["keys"], x["values"], shortlist, budget, seq_lens=x["seq_lens"],
                                           page_table=x.get("table"), max_len=x["max_len"], softmax_scale=0.125,
                                           logits_mode=1)
        m = _lib.ShardMap()
        m.key_offset = x.get("key_offset", 0)
        m.page_world = world if page_dealt else 0
        m.page_rank = r if page_dealt else 0
        args.append((a, lay, m, out))
    P = int(rank_inputs[0]["q"].shape[0] * rank_inputs[0]["q"].shape[1])
    first_flag = None
    for attempt in range(2):
        tops, wss = [], []
        for a, lay, m, _ in args:
            ws_bytes = int(lib.sva_shard_batched_workspace_size(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m),
                                                                width))
            assert ws_bytes > 0, _lib.load().sva_last_error()
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
            top = torch.empty(P, width, dtype=torch.int64, device="cuda")
            _lib.check(lib.sva_shard_batched_summon(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m), width,
                                                    top.data_ptr(), ws.data_ptr(), ws_bytes, None))
            tops.append(top)
            wss.append((ws, ws_bytes))
        g_top = torch.stack(tops)
        recs = []
        sat = torch.zeros(1, dtype=torch.int32, device="cuda")
        for r, (a, lay, m, _) in enumerate(args):
            rec = torch.empty(P, width, 4, dtype=torch.int32, device="cuda")
            _lib.check(lib.sva_shard_batched_rescore(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m), width,
                                                     world, r, g_top.data_ptr(), rec.data_ptr(), sat.data_ptr(),
                                                     wss[r][0].data_ptr(), wss[r][1], None))
            recs.append(rec)
        flag = int(sat.item())
        if first_flag is None:
            first_flag = flag
        if flag == 0 or width >= shortlist:
            break
        width = shortlist
    g_rec = torch.stack(recs)
    parts = []
    for r, (a, lay, m, _) in enumerate(args):
        part = torch.empty(P, D, dtype=torch.float64, device="cuda")
        _lib.check(lib.sva_shard_batched_verify(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m), width, world, r,
                                                g_rec.data_ptr(), part.data_ptr(), None))
        parts.append(part)
    g_part = torch.stack(parts)
    for a, lay, m, out in args:
        _lib.check(lib.sva_shard_batched_combine(ctypes.byref(a), ctypes.byref(lay), world, g_part.data_ptr(), None))
    torch.cuda.synchronize()
    return [x[3] for x in args], first_flag, width


def key_range_ranks(batch, world):
    """Rank r holds global keys [o_r, o_{r+1}) of every sequence (o_r = r * Lmax / world)."""
    lmax = max(batch["lengths"])
    ranks = []
    for r in range(world):
        lo, hi = lmax * r // world, lmax * (r + 1) // world
        lens = [max(0, min(n, hi) - lo) for n in batch["lengths"]]
        ranks.append(dict(q=batch["q"], q_proj=batch["q_proj"], scale=batch["scale"], cb=batch["cb"],
                          codes=batch["codes"][:, :, lo:hi].contiguous(), k_low=batch["k_low"][:, :, lo:hi].contiguous(),
                          keys=batch["keys"][:, :, lo:hi].contiguous(), values=batch["values"][:, :, lo:hi].contiguous(),
                          seq_lens=torch.tensor(lens, dtype=torch.int64, device="cuda"), max_len=max(1, hi - lo),
                          key_offset=lo))
    return ranks


def page_dealt_ranks(batch, pools, table, world, page_keys):
    """Rank r holds global pages g = r, r + world, ... of every sequence as its local pages 0, 1, ..."""
    ranks = []
    for r in range(world):
        lens, rows = [], []
        for b, n in enumerate(batch["lengths"]):
            n_pages = (n + page_keys - 1) // page_keys
            mine = list(range(r, n_pages, world))
            rows.append([int(table[b, g]) for g in mine])
            last = n - (n_pages - 1) * page_keys
            lens.append(sum(page_keys if g < n_pages - 1 else last for g in mine))
        width = max(1, max(len(x) for x in rows))
        t = torch.zeros(len(rows), width, dtype=torch.int32)
        for b, x in enumerate(rows):
            t[b, :len(x)] = torch.tensor(x, dtype=torch.int32) if x else 0
        ranks.append(dict(q=batch["q"], q_proj=batch["q_proj"], scale=batch["scale"], cb=batch["cb"],
                          codes=pools["codes"], k_low=pools["k_low"], keys=pools["keys"], values=pools["values"],
                          seq_lens=torch.tensor(lens, dtype=torch.int64, device="cuda"), table=t.cuda(),
                          max_len=max(1, width * page_keys)))
    return ranks


def one_gpu(batch):
    return kernels.decode_batched(batch["q"], batch["q_proj"], batch["scale"], batch["cb"], batch["codes"],
                                  batch["k_low"], batch["keys"], batch["values"], 2048, 512, seq_lens=batch["seq_lens"],
                                  max_len=max(batch["lengths"]), softmax_scale=0.125, logits_mode=1)


@pytest.mark.parametrize("world", [2, 3])
def test_key_range_shards_of_a_batch(world):
    """Equal lengths: every rank holds about 1 / world of each shortlist, the narrow exchange
    suffices (no repeat) and the result is exact."""
    batch = make_batch([60000, 60000, 60000], seed=31)
    want = one_gpu(batch)
    outs, flag, width = run_ranks(key_range_ranks(batch, world))
    assert flag == 0 and width < 2048
    for r, out in enumerate(outs):
        assert torch.equal(out, want), f"rank {r}"


@pytest.mark.parametrize("world", [2, 3])
def test_key_range_shards_of_a_ragged_batch(world):
    """Ragged lengths: a short sequence lies in one rank's range, which then holds its whole
    shortlist; the repeat at full width (when flagged) keeps the result exact."""
    batch = make_batch([50000, 70001, 33000], seed=31)
    want = one_gpu(batch)
    outs, flag, width = run_ranks(key_range_ranks(batch, world))
    for r, out in enumerate(outs):
        assert torch.equal(out, want), f"rank {r}"


@pytest.mark.parametrize("world,page_keys", [(2, 256), (4, 256), (3, 1024)])
def test_page_dealt_shards_of_a_paged_batch(world, page_keys):
    batch = make_batch([40000, 5000, 70001, 12345], seed=33)
    want = one_gpu(batch)
    pools, table = paged(batch, page_keys)
    outs, flag, _ = run_ranks(page_dealt_ranks(batch, pools, table.cpu(), world, page_keys), page_dealt=True)
    assert flag == 0
    for r, out in enumerate(outs):
        assert torch.equal(out, want), f"rank {r}"


def test_saturation_repeats_at_full_width():
    """An exchange width below every rank's share of the shortlist (600 of ~1024 members per rank
    at 2 ranks): the rescore stage must flag the first pass, and the full-width repeat must give
    the exact result."""
    batch = make_batch([60000, 45000], seed=35)
    want = one_gpu(batch)
    outs, flag, width = run_ranks(key_range_ranks(batch, 2), width=600)
    assert flag == 1 and width == 2048
    for out in outs:
        assert torch.equal(out, want)
