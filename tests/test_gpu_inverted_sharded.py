"""Key-range shards of the static inverted-index summon (sva_inverted_shard_*), emulated on one GPU:
the ranks run one after another, the all-gathers are emulated by stacking their outputs in rank
order, and the result must equal sva_decode_inverted over the whole static catalog (reference
sva/llama.py:427-576): bf16 outputs bit-identical (fp64 sums of rounded products are exact).
Cases: 4x64 and 2x256 codes, 2 to 4 ranks, uneven ranges, with and without adaptive budgets.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from sva_b200 import _lib, kernels

pytestmark = pytest.mark.gpu


def catalog(n_heads, n_keys, subspaces, codewords, seed):
    gen = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    q = torch.randn(n_heads, 64, generator=gen).to(torch.bfloat16).to(dev)
    q_proj = (torch.randn(n_heads, 64, 64, generator=gen) * 0.125).to(torch.bfloat16).float().to(dev)
    k_proj = (torch.randn(n_heads, 64, 64, generator=gen) * 0.125).to(torch.bfloat16).float().to(dev)
    cb = torch.randn(n_heads, subspaces, codewords, 64 // subspaces, generator=gen).to(torch.bfloat16).float().to(dev)
    keys = torch.randn(n_heads, n_keys, 64, generator=gen).to(torch.bfloat16).to(dev)
    values = torch.randn(n_heads, n_keys, 64, generator=gen).to(torch.bfloat16).to(dev)
    k_low = torch.empty(n_heads, n_keys, 64, device=dev)
    codes = torch.empty(n_heads, n_keys, subspaces, dtype=torch.uint8, device=dev)
    kernels.catalog_encode(keys, k_proj, cb, 0, n_keys, k_low, codes)
    return dict(q=q, q_proj=q_proj, scale=torch.ones(n_heads, device=dev), cb=cb, keys=keys, values=values,
                k_low=k_low, codes=codes)


def shard_decode(c, bounds, budget, min_budget, mid_budget, cells=8):
    world = len(bounds) - 1
    lib = _lib.load()
    C = int(c["cb"].shape[2])
    ranks = []
    counts = None
    for r in range(world):
        lo, hi = bounds[r], bounds[r + 1]
        loc = {k: c[k][:, lo:hi].contiguous() for k in ("codes", "k_low", "keys", "values")}
        post = kernels.postings_build(loc["codes"], C)
        counts = post.counts.to(torch.int64) if counts is None else counts + post.counts.to(torch.int64)
        ranks.append((lo, hi, loc, post))
    gmax = counts.max().to(torch.int32).reshape(1)
    recs, args = [], []
    for r, (lo, hi, loc, post) in enumerate(ranks):
        a, out = kernels.inverted_args(c["q"], c["q_proj"], c["scale"], c["cb"], loc["codes"], post, loc["k_low"],
                                       loc["keys"], loc["values"], budget, cells, min_budget, mid_budget,
                                       softmax_scale=0.125, max_bucket=gmax)
        ws_bytes = int(lib.sva_inverted_shard_workspace_size(ctypes.byref(a)))
        assert ws_bytes > 0, lib.sva_last_error()
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        rec = torch.empty(c["q"].shape[0], budget, 4, dtype=torch.int32, device="cuda")
        holds = int(r == world - 1)
        _lib.check(lib.sva_inverted_shard_summon(ctypes.byref(a), lo, holds, rec.data_ptr(), ws.data_ptr(), ws_bytes,
                                                 None))
        recs.append(rec)
        args.append((a, out, ws, ws_bytes, lo, holds, loc, post))
    g_rec = torch.stack(recs)
    parts = []
    for r, (a, out, ws, ws_bytes, lo, holds, loc, post) in enumerate(args):
        part = torch.empty(c["q"].shape[0], 64, dtype=torch.float64, device="cuda")
        _lib.check(lib.sva_inverted_shard_verify(ctypes.byref(a), lo, holds, world, r, g_rec.data_ptr(),
                                                 part.data_ptr(), ws.data_ptr(), ws_bytes, None))
        parts.append(part)
    g_part = torch.stack(parts)
    outs = []
    for a, out, *_ in args:
        _lib.check(lib.sva_inverted_shard_combine(ctypes.byref(a), world, g_part.data_ptr(), None))
        outs.append(out)
    torch.cuda.synchronize()
    return outs


def one_gpu(c, budget, min_budget, mid_budget, cells=8):
    post = kernels.postings_build(c["codes"], int(c["cb"].shape[2]))
    return kernels.decode_inverted(c["q"], c["q_proj"], c["scale"], c["cb"], c["codes"], post, c["k_low"], c["keys"],
                                   c["values"], budget, cells, min_budget, mid_budget, dynamic=False, softmax_scale=0.125)


@pytest.mark.parametrize("subspaces,codewords,bounds", [(4, 64, [0, 30000, 60000]),
                                                        (4, 64, [0, 10000, 35000, 41000, 60000]),
                                                        (2, 256, [0, 25000, 60000])])
def test_sharded_static_inverted_matches_one_gpu(subspaces, codewords, bounds):
    c = catalog(3, 60000, subspaces, codewords, seed=subspaces * 100 + len(bounds))
    want = one_gpu(c, 512, 512, 512)
    for r, got in enumerate(shard_decode(c, bounds, 512, 512, 512)):
        assert torch.equal(got, want), f"rank {r}"


def test_sharded_static_inverted_adaptive_budgets():
    c = catalog(4, 40000, 2, 256, seed=7)
    want = one_gpu(c, 256, 64, 128, cells=4)
    for r, got in enumerate(shard_decode(c, [0, 13000, 40000], 256, 64, 128, cells=4)):
        assert torch.equal(got, want), f"rank {r}"
