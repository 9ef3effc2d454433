"""The tcgen05 write path (sva_catalog_encode_tc) against fp64 and the exact path.

* k_low: bf16 keys times a bf16-valued projection, so every product is exact and the tensor-core
  result may differ from the fp64 product only by fp32 accumulation error (bound in the test).
* codes: bit-identical to the oracle's nearest-codeword assignment applied to the tensor-core
  k_low (the assignment arithmetic is shared with the exact path).  Against the exact path's
  codes, any difference must be a near tie: the two codewords' fp64 distances to the fp64 k_low
  agree to within the fp32 rounding of that k_low.
* Only rows [start, start + count) are written; GQA heads read their KV head.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sva_oracle as O
from sva_b200 import _lib, kernels

pytestmark = pytest.mark.gpu


def _case(seed, n_heads, n_kv, key_len, subspaces, codewords, head_dim=64, rank=64):
    g = torch.Generator().manual_seed(seed)
    keys = torch.randn(n_kv, key_len, head_dim, generator=g).to(torch.bfloat16)
    k_proj = (torch.randn(n_heads, head_dim, rank, generator=g) * 0.125).to(torch.bfloat16).float()
    cb = torch.randn(n_heads, subspaces, codewords, rank // subspaces, generator=g).to(torch.bfloat16).float()
    return keys, k_proj, cb


def _encode(keys, k_proj, cb, start, count, tensor_cores, sentinel=True):
    dev = torch.device("cuda")
    n_heads, rank = k_proj.shape[0], k_proj.shape[-1]
    cap = keys.shape[1]
    k_low = torch.full((n_heads, cap, rank), float("nan") if sentinel else 0.0, dtype=torch.float32, device=dev)
    codes = torch.full((n_heads, cap, cb.shape[1]), 255, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    assert kernels.tensor_core_write_ok(keys.to(dev), k_proj.to(dev)) or not tensor_cores
    kernels.catalog_encode(keys.to(dev), k_proj.to(dev), cb.to(dev), start, count, k_low, codes,
                           tensor_cores=tensor_cores, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return k_low.cpu().numpy(), codes.cpu().numpy()


@pytest.mark.parametrize("n_heads,n_kv,key_len,S,C,start,count", [
    (9, 9, 70_000, 4, 64, 0, 70_000),
    (9, 3, 20_000, 2, 256, 0, 20_000),          # GQA: three query heads per KV head
    (1, 1, 1 << 16, 1, 256, 1000, 50_001),      # a ragged range inside a larger buffer
])
def test_tensor_core_catalog(n_heads, n_kv, key_len, S, C, start, count):
    keys, k_proj, cb = _case(7, n_heads, n_kv, key_len, S, C)
    kl_tc, codes_tc = _encode(keys, k_proj, cb, start, count, True)
    kl_ex, codes_ex = _encode(keys, k_proj, cb, start, count, False)
    sl = slice(start, start + count)
    groups = n_heads // n_kv
    # rows outside the range untouched
    if start > 0:
        assert np.isnan(kl_tc[:, :start]).all() and (codes_tc[:, :start] == 255).all()
    if start + count < key_len:
        assert np.isnan(kl_tc[:, start + count:]).all() and (codes_tc[:, start + count:] == 255).all()
    k64 = keys.double().numpy()
    p64 = k_proj.double().numpy()
    near_ties = 0
    for h in range(n_heads):
        x = k64[h // groups, sl]
        ref = x @ p64[h]
        bound = np.abs(x) @ np.abs(p64[h]) * (64 * 2.0 ** -24) + 1e-30
        err = np.abs(kl_tc[h, sl].astype(np.float64) - ref)
        assert (err <= bound).all(), f"head {h}: max err / bound {np.max(err / bound):.3f}"
        # codes equal the shared assignment applied to the tensor-core k_low
        want = O.encode_product_keys(kl_tc[h:h + 1, sl], cb[h:h + 1].numpy())[0]
        np.testing.assert_array_equal(codes_tc[h, sl], want.astype(np.uint8))
        # against the exact path: only near ties may differ
        diff = np.argwhere(codes_tc[h, sl] != codes_ex[h, sl])
        sub = k_proj.shape[-1] // S
        for i, s in diff:
            xs = ref[i, s * sub:(s + 1) * sub]
            c64 = cb[h, s].double().numpy()
            d = ((xs[None, :] - c64) ** 2).sum(axis=1)
            a, b = int(codes_tc[h, start + i, s]), int(codes_ex[h, start + i, s])
            scale = (xs ** 2).sum() + (c64[[a, b]] ** 2).sum(axis=1).max()
            assert abs(d[a] - d[b]) <= 1e-5 * scale, f"head {h} key {i} subspace {s} is not a near tie"
            near_ties += 1
    assert near_ties <= max(4, count * n_heads * S // 20_000)


def test_tensor_core_catalog_rejects_fp32_keys():
    keys, k_proj, cb = _case(1, 1, 1, 256, 4, 64)
    dev = torch.device("cuda")
    k_low = torch.empty(1, 256, 64, device=dev)
    codes = torch.empty(1, 256, 4, dtype=torch.uint8, device=dev)
    with pytest.raises(TypeError):
        kernels.catalog_encode(keys.float().to(dev), k_proj.to(dev), cb.to(dev), 0, 256, k_low, codes,
                               tensor_cores=True)
    assert b"bf16" in _lib.load().sva_last_error()
