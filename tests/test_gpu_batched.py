"""Batched, ragged and paged scan decode (sva_decode_batched).

The reference decodes one sequence per call (sva/llama.py:182-183); a batch of B sequences is,
by definition, B independent calls of sva/llama.py:171-328.  So every problem of a batched call
must reproduce the single-sequence decode of its own sequence exactly (same shortlist and final
sets, bit-identical outputs), whatever the lengths of the other sequences and whether the catalog
and the K/V cache are contiguous per sequence or spread over a shuffled page pool.  The
single-sequence path itself is checked against the oracle and the reference's fixtures in
test_gpu_decode.py; one sequence per case is also checked against the oracle here.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sva_oracle as O

pytestmark = pytest.mark.gpu

H, HKV, D, R = 6, 2, 64, 64


def make_batch(lengths, subspaces=4, codewords=64, dtype=torch.bfloat16, n_q=1, seed=0):
    """Sequences of the given lengths with their own K/V (N(0,1)) and catalogs, in padded
    [B, H, Lmax, ...] buffers; shared artifacts (one layer)."""
    from sva_b200 import kernels

    gen = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    B, lmax = len(lengths), max(lengths)
    q = torch.randn(B, H, n_q, D, generator=gen).to(dtype).to(dev)
    q_proj = (torch.randn(H, D, R, generator=gen) * 0.125).to(torch.bfloat16).float().to(dev)
    k_proj = (torch.randn(H, D, R, generator=gen) * 0.125).to(torch.bfloat16).float().to(dev)
    cb = torch.randn(H, subspaces, codewords, R // subspaces, generator=gen).to(torch.bfloat16).float().to(dev)
    scale = torch.ones(H, device=dev)
    keys = torch.zeros(B, HKV, lmax, D, dtype=dtype, device=dev)
    values = torch.zeros(B, HKV, lmax, D, dtype=dtype, device=dev)
    codes = torch.zeros(B, H, lmax, subspaces, dtype=torch.uint8, device=dev)
    k_low = torch.zeros(B, H, lmax, R, dtype=torch.float32, device=dev)
    for b, n in enumerate(lengths):
        keys[b, :, :n] = torch.randn(HKV, n, D, generator=gen).to(dtype).to(dev)
        values[b, :, :n] = torch.randn(HKV, n, D, generator=gen).to(dtype).to(dev)
        kernels.catalog_encode(keys[b], k_proj, cb, 0, n, k_low[b], codes[b])
    seq_lens = torch.tensor(lengths, dtype=torch.int64, device=dev)
    return dict(q=q, q_proj=q_proj, scale=scale, cb=cb, keys=keys, values=values, codes=codes, k_low=k_low,
                seq_lens=seq_lens, lengths=list(lengths))


def paged(batch, page_keys=256, seed=1):
    """The same catalogs and caches moved into page pools in a shuffled page order."""
    lengths = batch["lengths"]
    pages_per = [(n + page_keys - 1) // page_keys for n in lengths]
    total = sum(pages_per)
    perm = torch.randperm(total, generator=torch.Generator().manual_seed(seed)).tolist()
    max_pages = max(pages_per)
    table = torch.zeros(len(lengths), max_pages, dtype=torch.int32)
    dev = batch["q"].device
    S = batch["codes"].shape[-1]
    pools = dict(codes=torch.zeros(total, H, page_keys, S, dtype=torch.uint8, device=dev),
                 k_low=torch.zeros(total, H, page_keys, R, dtype=torch.float32, device=dev),
                 keys=torch.zeros(total, HKV, page_keys, D, dtype=batch["keys"].dtype, device=dev),
                 values=torch.zeros(total, HKV, page_keys, D, dtype=batch["keys"].dtype, device=dev))
    k = 0
    for b, n in enumerate(lengths):
        for j in range(pages_per[b]):
            phys = perm[k]
            k += 1
            table[b, j] = phys
            lo, hi = j * page_keys, min(n, (j + 1) * page_keys)
            for name in pools:
                pools[name][phys, :, : hi - lo] = batch[name][b, :, lo:hi]
    return pools, table.to(dev)


def run_batched(batch, pools=None, table=None, **kw):
    from sva_b200 import kernels

    src = batch if pools is None else pools
    return kernels.decode_batched(batch["q"], batch["q_proj"], batch["scale"], batch["cb"], src["codes"],
                                  src["k_low"], src["keys"], src["values"], 2048, 512, seq_lens=batch["seq_lens"],
                                  page_table=table, max_len=max(batch["lengths"]), softmax_scale=0.125,
                                  logits_mode=1, want_shortlist=True, want_final=True, **kw)


def run_single(batch, b):
    from sva_b200 import kernels

    n = batch["lengths"][b]
    return kernels.decode(batch["q"][b], batch["q_proj"], batch["scale"], batch["cb"], batch["codes"][b, :, :n],
                          batch["k_low"][b, :, :n], batch["keys"][b, :, :n], batch["values"][b, :, :n], 2048, 512,
                          softmax_scale=0.125, logits_mode=1, want_shortlist=True, want_final=True)


def check_against_single(batch, res):
    """Selections bit-identical; outputs bit-identical for bf16 (its fp64 sums of rounded products
    are exact), within 1e-6 for fp32, where a sequence that one call decodes in the one-CTA
    schedule and the other in the grid schedule adds its fp64 partial sums in another order."""
    out, sl, fin = res
    torch.cuda.synchronize()
    for b in range(len(batch["lengths"])):
        o1, s1, f1 = run_single(batch, b)
        torch.cuda.synchronize()
        assert torch.equal(sl[b], s1), f"shortlist of sequence {b}"
        assert torch.equal(fin[b], f1), f"final set of sequence {b}"
        if out.dtype == torch.bfloat16:
            assert torch.equal(out[b], o1), f"output of sequence {b}"
        else:
            torch.testing.assert_close(out[b], o1, rtol=1e-6, atol=1e-6)


def check_one_against_oracle(batch, res, b):
    out, sl, fin = res
    n = batch["lengths"][b]
    kl = batch["k_low"][b, :, :n].cpu().numpy()
    cd = batch["codes"][b, :, :n].cpu().numpy().astype(np.int64)
    ref = O.scan_decode(batch["q"][b].float().cpu().numpy(), batch["q_proj"].cpu().numpy(), np.zeros(H, np.float32),
                        batch["cb"].cpu().numpy(), cd, kl, batch["keys"][b, :, :n].float().cpu().numpy(),
                        batch["values"][b, :, :n].float().cpu().numpy(), 2048, 512, 0.125, "bf16", 1)
    sl, fin = sl.cpu().numpy(), fin.cpu().numpy()
    for h in range(H):
        for t in range(sl.shape[2]):
            np.testing.assert_array_equal(sl[b, h, t][sl[b, h, t] >= 0], ref.shortlist[h][t])
            np.testing.assert_array_equal(fin[b, h, t][fin[b, h, t] >= 0], np.sort(ref.final[h][t]))
    np.testing.assert_allclose(out[b].float().cpu().numpy(), ref.out, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("lengths", [[5000, 40000, 70001, 33000], [300, 1000, 4096, 2049]])
def test_ragged_batch_matches_single_sequence_decodes(lengths):
    batch = make_batch(lengths)
    res = run_batched(batch)
    check_against_single(batch, res)
    check_one_against_oracle(batch, res, 0)


@pytest.mark.parametrize("lengths,page_keys", [([5000, 40000, 70001, 33000], 256), ([300, 1000, 4096, 2049], 64),
                                               ([66000, 1 << 17], 1024)])
def test_paged_batch_matches_unpaged(lengths, page_keys):
    batch = make_batch(lengths, seed=3)
    want = run_batched(batch)
    pools, table = paged(batch, page_keys)
    got = run_batched(batch, pools, table)
    torch.cuda.synchronize()
    for w, g in zip(want, got):
        assert torch.equal(w, g)
    check_against_single(batch, want)


def test_batched_one_by_one_subspace_and_fp32():
    """1x256 codes and fp32 caches (another scan variant and the fp32 verify)."""
    batch = make_batch([9000, 50000], subspaces=1, codewords=256, dtype=torch.float32, seed=5)
    res = run_batched(batch)
    check_against_single(batch, res)
    pools, table = paged(batch, 512)
    got = run_batched(batch, pools, table)
    for w, g in zip(res, got):
        assert torch.equal(w, g)


def test_batched_multi_token_causal():
    """T = 3 query tokens per sequence with the default causal lengths (seq_len - T + t + 1)."""
    batch = make_batch([3000, 45000], n_q=3, seed=7)
    res = run_batched(batch)
    check_against_single(batch, res)


def test_batched_rejects_bad_pages():
    from sva_b200 import kernels

    batch = make_batch([1000, 2000], seed=9)
    pools, table = paged(batch, 64)
    bad = {k: v[:, :, :48] for k, v in pools.items()}  # 48-key pages: not a power of two
    with pytest.raises(ValueError):
        kernels.decode_batched(batch["q"], batch["q_proj"], batch["scale"], batch["cb"], bad["codes"], bad["k_low"],
                               bad["keys"], bad["values"], 2048, 512, seq_lens=batch["seq_lens"], page_table=table)


def test_wide_finish_matches_cluster_finish():
    """Launches of at least 64 problems finish with one CTA per problem instead of one cluster per
    problem; both must select and compute the same.  64 independent heads of 40000 keys in one
    call (one-CTA finish) against the same heads in calls of 8 (cluster finish), plus the oracle
    for two heads."""
    from sva_b200 import kernels

    gen = torch.Generator().manual_seed(21)
    dev = torch.device("cuda")
    n_heads, n_keys, S, C = 64, 40000, 4, 64
    q = torch.randn(n_heads, 1, D, generator=gen).to(torch.bfloat16).to(dev)
    q_proj = (torch.randn(n_heads, D, R, generator=gen) * 0.125).to(torch.bfloat16).float().to(dev)
    k_proj = (torch.randn(n_heads, D, R, generator=gen) * 0.125).to(torch.bfloat16).float().to(dev)
    cb = torch.randn(n_heads, S, C, R // S, generator=gen).to(torch.bfloat16).float().to(dev)
    keys = torch.randn(n_heads, n_keys, D, generator=gen).to(torch.bfloat16).to(dev)
    values = torch.randn(n_heads, n_keys, D, generator=gen).to(torch.bfloat16).to(dev)
    k_low = torch.empty(n_heads, n_keys, R, device=dev)
    codes = torch.empty(n_heads, n_keys, S, dtype=torch.uint8, device=dev)
    kernels.catalog_encode(keys, k_proj, cb, 0, n_keys, k_low, codes)
    scale = torch.ones(n_heads, device=dev)
    out, sl, fin = kernels.decode(q, q_proj, scale, cb, codes, k_low, keys, values, 2048, 512, softmax_scale=0.125,
                                  logits_mode=1, want_shortlist=True, want_final=True)
    for h0 in range(0, n_heads, 8):
        hs = slice(h0, h0 + 8)
        o8, s8, f8 = kernels.decode(q[hs], q_proj[hs], scale[hs], cb[hs], codes[hs], k_low[hs], keys[hs], values[hs],
                                    2048, 512, softmax_scale=0.125, logits_mode=1, want_shortlist=True,
                                    want_final=True)
        torch.cuda.synchronize()
        assert torch.equal(s8, sl[hs]) and torch.equal(f8, fin[hs]) and torch.equal(o8, out[hs]), h0
    cd = codes.cpu().numpy().astype(np.int64)
    for h in (0, 63):
        ref = O.scan_decode(q[h:h + 1].float().cpu().numpy(), q_proj[h:h + 1].cpu().numpy(), np.zeros(1, np.float32),
                            cb[h:h + 1].cpu().numpy(), cd[h:h + 1], k_low[h:h + 1].cpu().numpy(),
                            keys[h:h + 1].float().cpu().numpy(), values[h:h + 1].float().cpu().numpy(), 2048, 512,
                            0.125, "bf16", 1)
        np.testing.assert_array_equal(fin[h, 0][fin[h, 0] >= 0].cpu().numpy(), np.sort(ref.final[0][0]))
        np.testing.assert_allclose(out[h].float().cpu().numpy(), ref.out[0], rtol=2e-2, atol=2e-2)
