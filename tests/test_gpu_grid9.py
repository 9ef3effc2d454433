"""Parity at the benchmark's own shape: 9 independent heads x 2^20 bf16 keys, 4x64 and 1x256 codes,
shortlist 2048, budget 512, one query token (the million-key grid schedule: prep -> scan ->
finish over 9 problems in one call).

The catalog is built on the GPU by the exact write path and spot-checked against the oracle's
projection and nearest-codeword rules; the decode is then checked against the oracle run on the
same catalog (oracle.sva_oracle.scan_decode_rows, which fetches the k_low / K / V rows it needs
from the device): shortlists and final sets bit-exact, outputs within 2e-2 (bf16).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sva_oracle as O

pytestmark = pytest.mark.gpu

HEADS, KEYS, D, R = 9, 1 << 20, 64, 64


def bench_like_set(subspaces: int, codewords: int, seed: int = 0):
    """A 9-head catalog drawn like bench.py's (seeded N(0,1) bf16 K/V with 64 planted keys per
    head), generated on the device."""
    from sva_b200 import kernels

    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(HEADS, 1, D, generator=gen).to(torch.bfloat16)
    q_proj = (torch.randn(HEADS, D, R, generator=gen) * 0.125).to(torch.bfloat16).float()
    k_proj = (torch.randn(HEADS, D, R, generator=gen) * 0.125).to(torch.bfloat16).float()
    cb = torch.randn(HEADS, subspaces, codewords, R // subspaces, generator=gen).to(torch.bfloat16).float()
    planted = torch.stack([torch.randperm(KEYS, generator=gen)[:64] for _ in range(HEADS)])
    noise = torch.randn(HEADS, 64, D, generator=gen)
    dgen = torch.Generator(device=dev).manual_seed(seed + 7)
    keys = torch.randn(HEADS, KEYS, D, generator=dgen, device=dev).to(torch.bfloat16)
    values = torch.randn(HEADS, KEYS, D, generator=dgen, device=dev).to(torch.bfloat16)
    for h in range(HEADS):
        keys[h, planted[h].to(dev)] = (0.9 * q[h, 0].float()[None, :] + 0.1 * noise[h]).to(torch.bfloat16).to(dev)
    q, q_proj, k_proj, cb = q.to(dev), q_proj.to(dev), k_proj.to(dev), cb.to(dev)
    k_low = torch.empty(HEADS, KEYS, R, dtype=torch.float32, device=dev)
    codes = torch.empty(HEADS, KEYS, subspaces, dtype=torch.uint8, device=dev)
    kernels.catalog_encode(keys, k_proj, cb, 0, KEYS, k_low, codes)
    return dict(q=q, q_proj=q_proj, k_proj=k_proj, cb=cb, keys=keys, values=values, k_low=k_low, codes=codes)


@pytest.mark.parametrize("subspaces,codewords", [(4, 64), (1, 256)])
def test_nine_heads_million_keys_grid(subspaces, codewords):
    from sva_b200 import kernels

    st = bench_like_set(subspaces, codewords)
    scale = torch.ones(HEADS, dtype=torch.float32, device="cuda")
    out, sl, fin = kernels.decode(st["q"], st["q_proj"], scale, st["cb"], st["codes"], st["k_low"], st["keys"],
                                  st["values"], 2048, 512, softmax_scale=0.125, logits_mode=1, want_shortlist=True,
                                  want_final=True)
    torch.cuda.synchronize()
    codes = st["codes"].cpu().numpy()
    # catalog spot check: projection and nearest codeword of sampled rows of every head
    rows = np.random.default_rng(1).choice(KEYS, 512, replace=False)
    rows_t = torch.from_numpy(rows).cuda()
    sub = R // subspaces
    for h in range(HEADS):
        kl = st["k_low"][h, rows_t].cpu().numpy()
        x = st["keys"][h, rows_t].float().cpu().numpy()
        np.testing.assert_array_equal(kl, O.project_keys(x[None], st["k_proj"][h:h + 1].cpu().numpy(), 1)[0])
        for s in range(subspaces):
            lab = O.assign_to_centroids(kl[:, s * sub:(s + 1) * sub], st["cb"][h, s].cpu().numpy())
            np.testing.assert_array_equal(codes[h, rows, s], lab)

    def k_low_rows(h, idx):
        return st["k_low"][h, torch.from_numpy(np.ascontiguousarray(idx)).cuda()].cpu().numpy()

    def kv_rows(h, idx):
        i = torch.from_numpy(np.ascontiguousarray(idx)).cuda()
        return st["keys"][h, i].float().cpu().numpy(), st["values"][h, i].float().cpu().numpy()

    ref = O.scan_decode_rows(st["q"][:, 0].float().cpu().numpy(), st["q_proj"].cpu().numpy(), np.zeros(HEADS, np.float32),
                             st["cb"].cpu().numpy(), codes, k_low_rows, kv_rows, 2048, 512, 0.125, "bf16", 1)
    sl, fin = sl.cpu().numpy(), fin.cpu().numpy()
    for h in range(HEADS):
        np.testing.assert_array_equal(sl[h, 0][sl[h, 0] >= 0], ref.shortlist[h][0])
        np.testing.assert_array_equal(fin[h, 0][fin[h, 0] >= 0], np.sort(ref.final[h][0]))
    np.testing.assert_allclose(out.float().cpu().numpy()[:, 0], ref.out[:, 0], rtol=2e-2, atol=2e-2)
