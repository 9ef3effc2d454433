"""GPU parity of the inverted-index path (sva_postings_build, sva_decode_inverted, sva_top_unique).

Postings, selections and validity flags must be bit-identical to the CPU oracle and to the
reference fixtures (tests/golden/golden_v1.npz, produced by running the reference's own
_inverted_static_decode_attention); outputs within 1e-3 (fp32) / 2e-2 (bf16).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sva_oracle as O
from tests.golden.inputs import config1, config2
from tests.helpers import gpu_catalog, oracle_catalog, to_np, tolerance

pytestmark = pytest.mark.gpu

GOLDEN = np.load(__file__.replace("test_gpu_inverted.py", "golden/golden_v1.npz"))

STATIC_CASES = {
    "static_cfg1": (lambda: config1(key_len=4096), dict(cells=8)),
    "static_4x64": (lambda: config2(key_len=1 << 14, subspaces=4, codewords=64, n_planted=16), dict(cells=8)),
    "static_adaptive": (lambda: config1(key_len=2048, seed=5),
                        dict(cells=4, adaptive_min_budget=64, adaptive_mid_budget=128)),
}


def _budgets(budget: int, key_len: int, amin, amid):
    max_budget = min(budget, key_len)
    min_budget = min(amin or max_budget, max_budget, key_len)
    mid_budget = min(amid or max(min_budget, max_budget // 2), max_budget, key_len)
    return max_budget, min_budget, mid_budget


def _run_gpu(case, plen, cells, amin=None, amid=None, dynamic=False, stats=None):
    from sva_b200 import kernels

    dev = "cuda"
    k_low, codes = gpu_catalog(case)
    post = kernels.postings_build(codes, int(case.codebooks.shape[2]), key_len=plen)
    budget = min(case.budget, case.shortlist, case.key_len)
    bmax, bmin, bmid = _budgets(budget, case.key_len, amin, amid)
    res = kernels.decode_inverted(
        case.q[0, :, 0].to(dev), case.q_proj.to(dev), kernels.sva_scale(case.logit_scale).to(dev),
        case.codebooks.to(dev), codes, post, k_low, case.keys[0].to(dev), case.values[0].to(dev), bmax, cells, bmin,
        bmid, dynamic=dynamic, softmax_scale=float(case.q.shape[-1]) ** -0.5, want_selection=True, stats=stats)
    return res, post, codes


@pytest.mark.parametrize("name", sorted(STATIC_CASES))
def test_postings_match_oracle(name):
    make, _ = STATIC_CASES[name]
    case = make()
    plen = case.key_len - int(GOLDEN[f"{name}_tail"])
    _, codes_ref = oracle_catalog(case)
    counts, offsets, ids = O.build_postings(codes_ref[:, :plen], case.codebooks.shape[2])
    from sva_b200 import kernels

    _, codes = gpu_catalog(case)
    post = kernels.postings_build(codes, int(case.codebooks.shape[2]), key_len=plen)
    np.testing.assert_array_equal(post.counts.cpu().numpy(), counts)
    np.testing.assert_array_equal(post.offsets.cpu().numpy(), offsets)
    np.testing.assert_array_equal(post.ids.cpu().numpy()[..., :plen], ids)
    assert int(post.max_bucket.item()) == int(counts.max())
    np.testing.assert_array_equal(post.counts.cpu().numpy(), GOLDEN[f"{name}_counts"])


@pytest.mark.parametrize("name", sorted(STATIC_CASES))
def test_static_inverted_matches_reference(name):
    make, kw = STATIC_CASES[name]
    case = make()
    tail = int(GOLDEN[f"{name}_tail"])
    plen = case.key_len - tail
    stats = torch.zeros(8, dtype=torch.int64, device="cuda")
    (out, sel_idx, sel_valid, sel_score, budgets), post, codes = _run_gpu(
        case, plen, kw["cells"], kw.get("adaptive_min_budget"), kw.get("adaptive_mid_budget"), stats=stats)
    sel_idx, sel_valid = sel_idx.cpu().numpy(), sel_valid.cpu().numpy().astype(bool)
    # oracle on the same catalog
    k_low_ref, codes_ref = oracle_catalog(case)
    post_ref = O.build_postings(codes_ref[:, :plen], case.codebooks.shape[2])
    budget = min(case.budget, case.shortlist, case.key_len)
    dtype = "f32" if case.q.dtype == torch.float32 else "bf16"
    o_out, o_sel, o_valid, o_scores, o_budgets, o_stats = O.static_decode(
        to_np(case.q[0])[:, 0], case.q_proj.numpy(), case.logit_scale.numpy(), case.codebooks.numpy(), post_ref, plen,
        k_low_ref, to_np(case.keys[0]), to_np(case.values[0]), budget, scaling=0.125, dtype=dtype, **kw)
    for h in range(case.n_heads):
        n = o_sel[h].shape[0]
        np.testing.assert_array_equal(sel_valid[h, :n], o_valid[h])
        np.testing.assert_array_equal(sel_idx[h, :n][o_valid[h]], o_sel[h][o_valid[h]])
        assert not sel_valid[h, n:].any()
        gv = GOLDEN[f"{name}_sel_valid"][h]
        np.testing.assert_array_equal(sel_valid[h, :gv.shape[0]], gv)
        np.testing.assert_array_equal(sel_idx[h, :gv.shape[0]][gv], GOLDEN[f"{name}_sel_idx"][h][gv])
    assert budgets.cpu().tolist() == o_budgets
    rtol, atol = tolerance(case)
    np.testing.assert_allclose(to_np(out), o_out, rtol=rtol, atol=atol)
    np.testing.assert_allclose(to_np(out), GOLDEN[f"{name}_out"], rtol=rtol, atol=atol)
    s = stats.cpu().tolist()
    assert s[0] == case.n_heads
    assert s[1] == o_stats["summoned"]
    assert s[2] == o_stats["refill_pool"] == int(GOLDEN[f"{name}_refill"]) * case.n_heads
    assert s[4] == o_stats["verified"]
    assert s[5] == o_stats["cell_visits"]


@pytest.mark.parametrize("cells,amin,amid", [(2, None, None), (4, 8, 16)])
def test_dynamic_inverted_matches_oracle(cells, amin, amid):
    case = config1(key_len=1500, seed=7)
    case.budget = 64
    (out, sel_idx, sel_valid, _, budgets), _, _ = _run_gpu(case, case.key_len, cells, amin, amid, dynamic=True)
    k_low_ref, codes_ref = oracle_catalog(case)
    post_ref = O.build_postings(codes_ref, case.codebooks.shape[2])
    bmax = min(64, case.key_len)
    o_out, o_sel, o_stats = O.dynamic_inverted_decode(
        to_np(case.q[0])[:, 0], case.q_proj.numpy(), case.logit_scale.numpy(), case.codebooks.numpy(), post_ref,
        k_low_ref, to_np(case.keys[0]), to_np(case.values[0]), bmax, cells, 0.125, "f32",
        adaptive_min_budget=amin, adaptive_mid_budget=amid)
    sel_idx = sel_idx.cpu().numpy()
    for h in range(case.n_heads):
        b = int(budgets[h].item())
        np.testing.assert_array_equal(sel_idx[h, :b], o_sel[h])
    np.testing.assert_allclose(to_np(out), o_out, rtol=1e-3, atol=1e-3)


def test_top_unique_golden_vector():
    """The reference's only exact golden vector (tests/test_sva_llama_adapter.py:58-73)."""
    from sva_b200 import kernels

    idx = torch.tensor([[4, 4, 3, 3, 2, 1]], device="cuda")
    scores = torch.tensor([[9.0, 8.5, 8.0, 7.5, 7.0, 6.0]], device="cuda")
    valid = torch.ones_like(idx, dtype=torch.bool)
    sel, sc, sv, refill = kernels.top_unique(idx, scores, valid, budget=3, refill_factor=2)
    assert refill == 6
    assert sel[sv].tolist() == [4, 3, 2]
    assert sc[sv].tolist() == [9.0, 8.0, 7.0]


@pytest.mark.parametrize("width,budget", [(37, 8), (600, 100), (4096, 512)])
def test_top_unique_matches_oracle(width, budget):
    from sva_b200 import kernels

    gen = torch.Generator().manual_seed(width)
    rows = 3
    idx = torch.randint(0, width // 3 + 1, (rows, width), generator=gen)
    scores = torch.randint(0, 40, (rows, width), generator=gen).float() / 4  # many ties
    # duplicates of one key share its score, as in the reference's candidate lists
    scores = torch.gather(torch.randn(rows, width // 3 + 1, generator=gen), 1, idx)
    valid = torch.rand(rows, width, generator=gen) > 0.2
    sel, sc, sv, refill = kernels.top_unique(idx.cuda(), scores.cuda(), valid.cuda(), budget)
    o_sel, o_sc, o_sv, o_refill = O.top_unique_candidates(idx.numpy(), scores.numpy(), valid.numpy(), budget)
    assert refill == o_refill
    for r in range(rows):
        np.testing.assert_array_equal(sv[r].cpu().numpy(), o_sv[r])
        np.testing.assert_array_equal(sel[r].cpu().numpy()[o_sv[r]], o_sel[r][o_sv[r]])
        np.testing.assert_array_equal(sc[r].cpu().numpy()[o_sv[r]], o_sc[r][o_sv[r]])


def test_incremental_postings_match_rebuild():
    """Appending keys one or a few at a time (sva_postings_append, the dynamic mode's per-token
    update, reference sva/llama.py:659-693) leaves every cell's list equal to a fresh build over
    all keys, ascending; a dynamic inverted decode over the appended lists equals one over the
    rebuilt lists; and an append past a cell's room is refused through the overflow flag."""
    from sva_b200 import kernels

    case = config1(key_len=6000)
    k_low, codes = gpu_catalog(case)
    C = int(case.codebooks.shape[2])
    start = 5000
    post = kernels.postings_padded(codes, C, start)
    cap0 = post.cap
    pos, steps = start, [1, 3, 1, 7, 2]
    while pos < 6000:
        n = min(steps[pos % len(steps)], 6000 - pos)
        kernels.postings_append(codes, post, pos, n)
        pos += n
    ref = kernels.postings_build(codes, C, key_len=6000)
    torch.cuda.synchronize()
    assert int(post.overflow.item()) == 0
    assert torch.equal(post.counts, ref.counts)
    assert int(post.max_bucket.item()) == int(ref.max_bucket.item())
    cnt, off = ref.counts.cpu().numpy(), ref.offsets.cpu().numpy()
    ids_a, ids_r = post.ids.cpu().numpy(), ref.ids.cpu().numpy()
    for h in range(cnt.shape[0]):
        for s in range(cnt.shape[1]):
            for c in range(C):
                n = cnt[h, s, c]
                np.testing.assert_array_equal(ids_a[h, s, c * cap0:c * cap0 + n],
                                              ids_r[h, s, off[h, s, c]:off[h, s, c] + n])
    dev = codes.device
    args = (case.q[0][:, 0].to(dev), case.q_proj.to(dev), kernels.sva_scale(case.logit_scale).to(dev),
            case.codebooks.to(dev), codes)
    tail = (k_low, case.keys[0].to(dev), case.values[0].to(dev), 512, 8, 512, 512)
    got = kernels.decode_inverted(*args, post, *tail, dynamic=True, softmax_scale=0.125)
    want = kernels.decode_inverted(*args, ref, *tail, dynamic=True, softmax_scale=0.125)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    # cells sized for the first 5000 keys: an append past a cell's room is refused and flagged
    cap = int(kernels.postings_build(codes, C, key_len=5000).max_bucket.item())
    tight = kernels.postings_padded(codes, C, 5000, cap=cap)
    kernels.postings_append(codes, tight, 5000, 1000)
    torch.cuda.synchronize()
    assert int(tight.overflow.item()) == int(bool((ref.counts > cap).any()))
    assert bool((tight.counts <= cap).all())
    with pytest.raises(ValueError):
        kernels.postings_padded(codes, C, 6000, cap=cap - 1)
