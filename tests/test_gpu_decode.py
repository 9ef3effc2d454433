"""GPU parity of the write path and the scan summon -> verify decode (sva_catalog_encode, sva_decode).

The CUDA path and the CPU oracle implement the same canonical arithmetic and tie rule, so
codes, k_low, shortlists and final indices must be bit-identical; attention outputs are
compared within 1e-3 (fp32) / 2e-2 (bf16).  The reference's own golden outputs are checked
directly as well (tests/golden/golden_v1.npz).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sva_oracle as O
from tests.golden.inputs import config1, config2
from tests.helpers import (cached_case, gpu_catalog, gpu_decode, oracle_decode, to_np, tolerance, unpad)

pytestmark = pytest.mark.gpu

GOLDEN = np.load(__file__.replace("test_gpu_decode.py", "golden/golden_v1.npz"))
CASES = ["cfg1", "cfg2s_1x256", "cfg2s_4x64"]


@pytest.mark.parametrize("name", CASES)
def test_catalog_bit_exact(name):
    case, (k_low_ref, codes_ref) = cached_case(name)
    k_low, codes = gpu_catalog(case)
    np.testing.assert_array_equal(k_low.cpu().numpy(), k_low_ref)
    np.testing.assert_array_equal(codes.cpu().numpy(), codes_ref.astype(np.uint8))
    np.testing.assert_array_equal(codes.cpu().numpy(), GOLDEN[f"{name}_codes"])


@pytest.mark.parametrize("name", CASES)
def test_decode_matches_oracle_and_reference(name):
    case, (k_low_ref, codes_ref) = cached_case(name)
    k_low, codes = gpu_catalog(case)
    out, sl, fin = gpu_decode(case, k_low, codes)
    torch.cuda.synchronize()
    ref = oracle_decode(case, k_low_ref, codes_ref)
    sl, fin = sl.cpu().numpy(), fin.cpu().numpy()
    rtol, atol = tolerance(case)
    for h in range(case.n_heads):
        np.testing.assert_array_equal(unpad(sl[h, 0]), ref.shortlist[h][0])
        np.testing.assert_array_equal(unpad(fin[h, 0]), np.sort(ref.final[h][0]))
        # and the reference's golden selection (canonical tie rule on its own scores)
        np.testing.assert_array_equal(unpad(sl[h, 0]), GOLDEN[f"{name}_shortlist_canon"][h])
        np.testing.assert_array_equal(unpad(fin[h, 0]), np.sort(GOLDEN[f"{name}_final_canon"][h]))
    got = to_np(out)[:, 0]
    np.testing.assert_allclose(got, ref.out[:, 0], rtol=rtol, atol=atol)
    np.testing.assert_allclose(got, GOLDEN[f"{name}_out_canon"], rtol=rtol, atol=atol)


@pytest.mark.parametrize("name", CASES)
def test_shortlist_bit_exact_with_reference_lut(name):
    """Staged parity: the reference's own fp32 LUT and codes in, the reference shortlist out."""
    case, (k_low_ref, _) = cached_case(name)
    k_low = torch.from_numpy(k_low_ref).cuda()
    codes = torch.from_numpy(GOLDEN[f"{name}_codes"]).cuda()
    lut = torch.from_numpy(GOLDEN[f"{name}_lut"]).cuda().contiguous()
    _, sl, _ = gpu_decode(case, k_low, codes, lut_override=lut)
    sl = sl.cpu().numpy()
    for h in range(case.n_heads):
        np.testing.assert_array_equal(unpad(sl[h, 0]), GOLDEN[f"{name}_shortlist_canon"][h])


@pytest.mark.parametrize("logits_mode", [0, 1])
def test_fp32_and_dtype_logits_modes(logits_mode):
    case, (k_low_ref, codes_ref) = cached_case("cfg2s_4x64")
    k_low, codes = gpu_catalog(case)
    out, _, fin = gpu_decode(case, k_low, codes, logits_mode=logits_mode)
    ref = oracle_decode(case, k_low_ref, codes_ref, logits_mode=logits_mode)
    np.testing.assert_allclose(to_np(out)[:, 0], ref.out[:, 0], rtol=2e-2, atol=2e-2)


def _small_case(key_len, n_heads=3, n_kv=1, seed=3, dtype=torch.float32, subspaces=2, codewords=16, head_dim=64,
                rank=64):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(1, n_heads, 1, head_dim, generator=gen).to(dtype)
    keys = torch.randn(1, n_kv, key_len, head_dim, generator=gen).to(dtype)
    values = torch.randn(1, n_kv, key_len, head_dim, generator=gen).to(dtype)
    from tests.golden.inputs import DecodeCase

    return DecodeCase("small", q, keys, values, torch.randn(n_heads, head_dim, rank, generator=gen) * 0.125,
                      torch.randn(n_heads, head_dim, rank, generator=gen) * 0.125, torch.randn(n_heads, generator=gen) * 0.3,
                      torch.randn(n_heads, subspaces, codewords, rank // subspaces, generator=gen), 64, 16,
                      torch.zeros(n_kv, 0, dtype=torch.long))


@pytest.mark.parametrize("key_len,shortlist,budget", [(1, 4, 2), (5, 4, 2), (37, 64, 16), (300, 64, 80), (3000, 200, 50)])
def test_edge_sizes(key_len, shortlist, budget):
    case = _small_case(key_len)
    k_low_ref, codes_ref = O.build_catalog(to_np(case.keys[0]), case.k_proj.numpy(), case.codebooks.numpy(), 3)
    k_low, codes = gpu_catalog(case)
    np.testing.assert_array_equal(codes.cpu().numpy(), codes_ref)
    out, sl, fin = gpu_decode(case, k_low, codes, shortlist=shortlist, budget=budget)
    ref = oracle_decode(case, k_low_ref, codes_ref, shortlist=shortlist, budget=budget)
    for h in range(case.n_heads):
        np.testing.assert_array_equal(unpad(sl.cpu().numpy()[h, 0]), ref.shortlist[h][0])
        np.testing.assert_array_equal(unpad(fin.cpu().numpy()[h, 0]), np.sort(ref.final[h][0]))
    np.testing.assert_allclose(to_np(out)[:, 0], ref.out[:, 0], rtol=1e-4, atol=1e-5)


def test_tiny_shapes_head_dim_8_rank_4():
    """The reference unit-test geometry: head_dim 8, rank 4, 2x8 codes."""
    case = _small_case(6, n_heads=2, n_kv=2, head_dim=8, rank=4, subspaces=2, codewords=8)
    k_low_ref, codes_ref = O.build_catalog(to_np(case.keys[0]), case.k_proj.numpy(), case.codebooks.numpy(), 1)
    k_low, codes = gpu_catalog(case)
    np.testing.assert_array_equal(k_low.cpu().numpy(), k_low_ref)
    np.testing.assert_array_equal(codes.cpu().numpy(), codes_ref)
    out, sl, fin = gpu_decode(case, k_low, codes, shortlist=4, budget=2)
    ref = oracle_decode(case, k_low_ref, codes_ref, shortlist=4, budget=2)
    for h in range(2):
        np.testing.assert_array_equal(unpad(sl.cpu().numpy()[h, 0]), ref.shortlist[h][0])
        np.testing.assert_array_equal(unpad(fin.cpu().numpy()[h, 0]), np.sort(ref.final[h][0]))
    np.testing.assert_allclose(to_np(out)[:, 0], ref.out[:, 0], rtol=1e-4, atol=1e-5)


def test_prefill_causal_and_mask():
    """T > 1 query tokens with the default causal rule and with an explicit allowed mask."""
    case = _small_case(400, n_heads=2, n_kv=1)
    gen = torch.Generator().manual_seed(9)
    q = torch.randn(2, 24, 64, generator=gen)
    k_low_ref, codes_ref = O.build_catalog(to_np(case.keys[0]), case.k_proj.numpy(), case.codebooks.numpy(), 2)
    k_low, codes = gpu_catalog(case)
    out, sl, fin = gpu_decode(case, k_low, codes, q=q, shortlist=64, budget=16)
    ref = oracle_decode(case, k_low_ref, codes_ref, q=q, shortlist=64, budget=16)
    for h in range(2):
        for t in range(24):
            np.testing.assert_array_equal(unpad(sl.cpu().numpy()[h, t]), ref.shortlist[h][t])
            np.testing.assert_array_equal(unpad(fin.cpu().numpy()[h, t]), np.sort(ref.final[h][t]))
    np.testing.assert_allclose(to_np(out), ref.out, rtol=1e-4, atol=1e-5)
    mask = torch.rand(24, 400, generator=gen) > 0.7
    mask_dev = mask.to(torch.uint8).cuda()
    out, sl, fin = gpu_decode(case, k_low, codes, q=q, shortlist=64, budget=16, allowed_mask=mask_dev,
                              allowed_len=torch.full((24,), 400, dtype=torch.int64, device="cuda"))
    ref = oracle_decode(case, k_low_ref, codes_ref, q=q, shortlist=64, budget=16, allowed_mask=mask.numpy())
    for h in range(2):
        for t in range(24):
            np.testing.assert_array_equal(unpad(sl.cpu().numpy()[h, t]), ref.shortlist[h][t])
            np.testing.assert_array_equal(unpad(fin.cpu().numpy()[h, t]), np.sort(ref.final[h][t]))
    np.testing.assert_allclose(to_np(out), ref.out, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("key_len", [20000, 70000])
def test_all_scores_tied_picks_lowest_indices(key_len):
    """A zero query makes every ADC and rank score 0: the canonical rule keeps the lowest key
    indices.  At 70000 keys (grid schedule) the tie overflows the candidate buffer and exercises
    the exact streaming fallback."""
    case = _small_case(key_len, n_heads=1, n_kv=1)
    k_low, codes = gpu_catalog(case)
    q = torch.zeros(1, 1, 64)
    _, sl, fin = gpu_decode(case, k_low, codes, q=q, shortlist=2048, budget=512)
    np.testing.assert_array_equal(unpad(sl.cpu().numpy()[0, 0]), np.arange(2048))
    np.testing.assert_array_equal(unpad(fin.cpu().numpy()[0, 0]), np.arange(512))


@pytest.mark.parametrize("subspaces,codewords", [(1, 256), (4, 64)])
def test_million_keys(subspaces, codewords):
    """Config 2 at full size (2^20 keys, bf16): GPU catalog, oracle decode on the GPU catalog, and
    a sampled nearest-codeword / projection check of the catalog against the oracle.  (Recall of
    the planted near-duplicates depends on the random codebooks, not on the kernels, so it is not
    asserted.)"""
    case = config2(key_len=1 << 20, subspaces=subspaces, codewords=codewords)
    k_low, codes = gpu_catalog(case)
    out, sl, fin = gpu_decode(case, k_low, codes)
    kl, cd = k_low.cpu().numpy(), codes.cpu().numpy().astype(np.int64)
    rng = np.random.default_rng(0)
    rows = rng.choice(case.key_len, 4096, replace=False)
    sub = 64 // subspaces
    for s in range(subspaces):
        lab = O.assign_to_centroids(kl[0, rows, s * sub:(s + 1) * sub], case.codebooks.numpy()[0, s])
        np.testing.assert_array_equal(cd[0, rows, s], lab)
    proj = O.project_keys(to_np(case.keys[0])[:, rows], case.k_proj.numpy(), 1)
    np.testing.assert_array_equal(kl[0, rows], proj[0])
    ref = oracle_decode(case, kl, cd)
    np.testing.assert_array_equal(unpad(sl.cpu().numpy()[0, 0]), ref.shortlist[0][0])
    np.testing.assert_array_equal(unpad(fin.cpu().numpy()[0, 0]), np.sort(ref.final[0][0]))
    np.testing.assert_allclose(to_np(out)[:, 0], ref.out[:, 0], rtol=2e-2, atol=2e-2)


def test_stats_counters():
    case, (k_low_ref, codes_ref) = cached_case("cfg1")
    k_low, codes = gpu_catalog(case)
    stats = torch.zeros(8, dtype=torch.int64, device="cuda")
    gpu_decode(case, k_low, codes, stats=stats)
    s = stats.cpu().tolist()
    assert s[0] == 9 and s[1] == 9 * 2048 and s[3] == 9 * 512 and s[4] == 9 * 512


def test_cpu_tensors_are_rejected():
    from sva_b200 import kernels

    case, _ = cached_case("cfg1")
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.decode(case.q[0], case.q_proj, case.logit_scale, case.codebooks, torch.zeros(9, 8, 2, dtype=torch.uint8),
                       torch.zeros(9, 8, 64), case.keys[0], case.values[0], 4, 2)


def _decode_with(case, k_low, codes, q, out=None):
    from sva_b200 import kernels

    dev = codes.device
    return kernels.decode(q, case.q_proj.to(dev), kernels.sva_scale(case.logit_scale).to(dev), case.codebooks.to(dev),
                          codes, k_low, case.keys[0].to(dev), case.values[0].to(dev), case.shortlist, case.budget,
                          softmax_scale=float(case.q.shape[-1]) ** -0.5, logits_mode=1, out=out)


@pytest.mark.parametrize("name", ["cfg1", "cfg2s_4x64"])
def test_pinned_host_query_and_output(name):
    """q and out in pinned host memory: the kernels read and write them over PCIe; the output
    equals the one computed with device buffers bit for bit, on both schedules."""
    case, _ = cached_case(name)
    k_low, codes = gpu_catalog(case)
    out_dev = _decode_with(case, k_low, codes, case.q[0].cuda())
    q_host = case.q[0].clone().pin_memory()
    out_host = torch.full(tuple(out_dev.shape), float("nan"), dtype=out_dev.dtype).pin_memory()
    for _ in range(2):  # two calls in a row on the same host buffers
        got = _decode_with(case, k_low, codes, q_host, out=out_host)
        torch.cuda.synchronize()
        assert got.data_ptr() == out_host.data_ptr()
        np.testing.assert_array_equal(to_np(out_host), to_np(out_dev))


def test_unpinned_host_query_is_rejected():
    case, _ = cached_case("cfg1")
    k_low, codes = gpu_catalog(case)
    with pytest.raises(ValueError, match="pinned host tensor"):
        _decode_with(case, k_low, codes, case.q[0].clone())


def test_chained_decodes_query_aliases_previous_output():
    """Two back-to-back decodes on one stream where the second call's query is the first call's
    output buffer: the dependent launches of the second call must read the query only after the
    first call has written it.  Compared with the same two calls separated by a synchronize."""
    case, _ = cached_case("cfg2s_4x64")  # 2^16 keys: the grid schedule
    k_low, codes = gpu_catalog(case)
    q0 = case.q[0].cuda()

    def run(q, out):
        from sva_b200 import kernels

        return kernels.decode(q, case.q_proj.cuda(), kernels.sva_scale(case.logit_scale).cuda(), case.codebooks.cuda(),
                              codes, k_low, case.keys[0].cuda(), case.values[0].cuda(), 2048, 512,
                              softmax_scale=0.125, logits_mode=1, out=out)

    for _ in range(3):
        out1 = torch.empty_like(q0)
        out2 = torch.empty_like(q0)
        run(q0, out1)
        run(out1, out2)  # no synchronisation between the calls
        torch.cuda.synchronize()
        ref1 = torch.empty_like(q0)
        run(q0, ref1)
        torch.cuda.synchronize()
        ref2 = torch.empty_like(q0)
        run(ref1.clone(), ref2)
        torch.cuda.synchronize()
        assert torch.equal(out1, ref1)
        assert torch.equal(out2, ref2)


@pytest.mark.parametrize("name", ["cfg1", "cfg2s_4x64"])
def test_catalog_appends_match_full_build(name):
    """Decode-step appends (one CTA per key and head for up to 8 keys, host or device start row)
    write exactly the rows of the full catalog build."""
    from sva_b200 import kernels

    case, (k_low_ref, codes_ref) = cached_case(name)
    keys = case.keys[0].cuda()
    n = 300
    k_low = torch.zeros(case.n_heads, n, 64, device="cuda")
    codes = torch.zeros(case.n_heads, n, case.codebooks.shape[1], dtype=torch.uint8, device="cuda")
    kp, cb = case.k_proj.cuda(), case.codebooks.cuda()
    pos = 0
    for i, count in enumerate([1, 2, 3, 8, 5, 1, 7, 4] * 20):
        if pos >= n:
            break
        count = min(count, n - pos)
        if i % 2:
            kernels.catalog_encode(keys, kp, cb, pos, count, k_low, codes)
        else:
            start = torch.tensor([pos], dtype=torch.int64, device="cuda")
            kernels.catalog_encode_at(keys, kp, cb, start, count, n, k_low, codes)
        pos += count
    # a device start past the limit writes nothing
    kernels.catalog_encode_at(keys, kp, cb, torch.tensor([n], dtype=torch.int64, device="cuda"), 4, n, k_low, codes)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(k_low.cpu().numpy(), k_low_ref[:, :n])
    np.testing.assert_array_equal(codes.cpu().numpy(), codes_ref[:, :n].astype(np.uint8))
