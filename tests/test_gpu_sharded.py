"""Key-range shards on one GPU: the four stage kernels run once per emulated rank, the
all-gathers are emulated by stacking the ranks' outputs in rank order, and the result must
equal sva_decode over the concatenated keys: the same shortlist and final sets (bit-exact)
and the same output (up to the order of exact fp64 sums).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from sva_b200 import kernels
from sva_b200.sharded import CudaShardBackend
from tests.golden.inputs import config1, config2
from tests.helpers import gpu_catalog, gpu_decode, unpad

pytestmark = pytest.mark.gpu


def _u64(lo: torch.Tensor, hi: torch.Tensor) -> np.ndarray:
    lo = lo.cpu().numpy().view(np.uint32).astype(np.uint64)
    hi = hi.cpu().numpy().view(np.uint32).astype(np.uint64)
    return (hi << np.uint64(32)) | lo


def emulated_shards(case, k_low, codes, bounds, logits_mode=1):
    """Run the sharded decode with ranks [bounds[r], bounds[r+1]) on one GPU."""
    dev = codes.device
    world = len(bounds) - 1
    q = case.q[0].to(dev)
    q_proj, cb = case.q_proj.to(dev), case.codebooks.to(dev)
    scale = kernels.sva_scale(case.logit_scale).to(dev)
    keys, values = case.keys[0].to(dev), case.values[0].to(dev)
    calls, backends = [], []
    for r in range(world):
        lo, hi = bounds[r], bounds[r + 1]
        be = CudaShardBackend()
        c = be.prepare(q, q_proj, scale, cb, codes[:, lo:hi].contiguous(), k_low[:, lo:hi].contiguous(),
                       keys[:, lo:hi].contiguous(), values[:, lo:hi].contiguous(), shortlist=case.shortlist,
                       budget=case.budget, key_offset=lo, logits_mode=logits_mode,
                       softmax_scale=float(case.q.shape[-1]) ** -0.5)
        calls.append(c)
        backends.append(be)
    g_top = torch.stack([be.summon(c) for be, c in zip(backends, calls)])
    g_rec = torch.stack([be.rescore(c, g_top, world, r) for r, (be, c) in enumerate(zip(backends, calls))])
    g_part = torch.stack([be.verify(c, g_rec, world, r) for r, (be, c) in enumerate(zip(backends, calls))])
    outs = [be.combine(c, g_part, world).clone() for be, c in zip(backends, calls)]
    torch.cuda.synchronize()
    return outs, g_top, g_rec


def sets_from_records(g_rec: torch.Tensor, budget: int):
    """Global shortlist (all live records) and final set (top budget by rank composite) per head."""
    comp = _u64(g_rec[..., 0], g_rec[..., 1])  # [W, H, SL]
    n_heads = comp.shape[1]
    sls, fins = [], []
    for h in range(n_heads):
        c = comp[:, h].reshape(-1)
        c = c[c != 0]
        idx = (~c) & np.uint64(0xFFFFFFFF)
        sls.append(np.sort(idx.astype(np.int64)))
        order = np.argsort(c)[::-1][: min(budget, c.shape[0])]
        fins.append(np.sort(idx[order].astype(np.int64)))
    return sls, fins


@pytest.mark.parametrize("name,bounds_frac", [
    ("cfg2_9h_4x64", (0, 0.5, 1.0)),
    ("cfg2_9h_4x64", (0, 0.13, 0.61, 1.0)),
    ("cfg2_1h_1x256", (0, 0.25, 0.5, 0.75, 1.0)),
    ("cfg2_1h_1x256", (0, 0.001, 1.0)),  # a rank holding fewer keys than the shortlist
    ("cfg1", (0, 0.5, 1.0)),
])
def test_sharded_equals_single_gpu(name, bounds_frac):
    if name == "cfg1":
        case = config1()
    elif name == "cfg2_9h_4x64":
        case = config2(key_len=300_000, subspaces=4, codewords=64, n_heads=9)
    else:
        case = config2(key_len=1 << 20, subspaces=1, codewords=256, n_heads=1)
    k_low, codes = gpu_catalog(case)
    out, sl, fin = gpu_decode(case, k_low, codes)
    bounds = [int(round(f * case.key_len)) for f in bounds_frac]
    outs, g_top, g_rec = emulated_shards(case, k_low, codes, bounds)
    sls, fins = sets_from_records(g_rec, case.budget)
    sl_np, fin_np = sl.cpu().numpy(), fin.cpu().numpy()
    for h in range(case.n_heads):
        np.testing.assert_array_equal(sls[h], unpad(sl_np[h, 0]), err_msg=f"shortlist head {h}")
        np.testing.assert_array_equal(fins[h], unpad(fin_np[h, 0]), err_msg=f"final head {h}")
    ref = out[:, 0].float().cpu()
    for r, o in enumerate(outs):
        got = o[:, 0].float().cpu()
        torch.testing.assert_close(got, ref, rtol=1e-3, atol=1e-3, msg=f"rank {r}")
        assert (got == ref).float().mean().item() >= 0.99, "outputs should agree bit for bit"


def test_sharded_rejects_masks_and_multi_token():
    case = config1(key_len=4096)
    k_low, codes = gpu_catalog(case)
    dev = codes.device
    be = CudaShardBackend()
    q2 = case.q[0].to(dev).expand(-1, 2, -1).contiguous()
    with pytest.raises(ValueError):
        be.prepare(q2, case.q_proj.to(dev), kernels.sva_scale(case.logit_scale).to(dev), case.codebooks.to(dev),
                   codes, k_low, case.keys[0].to(dev), case.values[0].to(dev), shortlist=64, budget=16, key_offset=0)
