"""Bit-exact parity of the register-tiled bulk write path (catalog_encode_reg_kernel: head_dim =
rank_dim = 64, subspaces of 8, 16 or 32 values) with the CPU oracle's build_catalog (reference
sva/llama.py:598,615 and sva/ops.py:10-47): k_low and codes identical for fp32, bf16 and fp16
keys, grouped heads, key ranges that start and end inside a tile, row strides that rule out
vector loads, and an output buffer whose alignment rules out vector stores.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sva_oracle as O
from sva_b200 import kernels

pytestmark = pytest.mark.gpu


def _case(dtype, n_kv, groups, key_len, subspaces, codewords, seed):
    gen = torch.Generator().manual_seed(seed)
    n_heads = n_kv * groups
    keys = torch.randn(n_kv, key_len, 64, generator=gen).to(dtype)
    k_proj = (torch.randn(n_heads, 64, 64, generator=gen) * 0.125).to(torch.bfloat16).float()
    cb = torch.randn(n_heads, subspaces, codewords, 64 // subspaces, generator=gen).to(torch.bfloat16).float()
    return keys, k_proj, cb


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("subspaces,codewords", [(4, 64), (2, 256), (8, 32)])
def test_register_write_path_bit_exact(dtype, subspaces, codewords):
    keys, k_proj, cb = _case(dtype, 3, 3, 3001, subspaces, codewords, seed=subspaces * 7 + codewords)
    n_heads = 9
    dev = torch.device("cuda")
    kd = keys.contiguous().to(dev)
    k_low = torch.full((n_heads, 3100, 64), float("nan"), device=dev)
    codes = torch.full((n_heads, 3100, subspaces), 255, dtype=torch.uint8, device=dev)
    # a range starting and ending inside a tile, then the head of the cache
    kernels.catalog_encode(kd, k_proj.to(dev), cb.to(dev), 77, 3001 - 77, k_low, codes)
    kernels.catalog_encode(kd, k_proj.to(dev), cb.to(dev), 0, 77, k_low, codes)
    torch.cuda.synchronize()
    k_ref, c_ref = O.build_catalog(keys.float().numpy(), k_proj.numpy(), cb.numpy(), 3)
    np.testing.assert_array_equal(k_low[:, :3001].cpu().numpy(), k_ref)
    np.testing.assert_array_equal(codes[:, :3001].cpu().numpy(), c_ref.astype(np.uint8))
    # rows past the range are untouched
    assert torch.isnan(k_low[:, 3001:]).all() and (codes[:, 3001:] == 255).all()


def test_register_write_path_unaligned_rows_and_outputs():
    """Key rows 66 elements apart (no 16-byte vector loads) and a k_low buffer that starts 4 bytes
    past a 16-byte boundary (no vector stores)."""
    keys, k_proj, cb = _case(torch.bfloat16, 2, 2, 1500, 4, 64, seed=5)
    dev = torch.device("cuda")
    padded = torch.zeros(2, 1500, 66, dtype=torch.bfloat16, device=dev)
    padded[:, :, :64] = keys.to(dev)
    kd = padded[:, :, :64]  # a strided view: rows 66 elements apart
    assert kd.stride(1) == 66
    flat = torch.zeros(4 * 1500 * 64 + 2, device=dev)
    k_low = flat[1:1 + 4 * 1500 * 64].view(4, 1500, 64)  # 4-byte aligned, not 16
    codes = torch.empty(4, 1500, 4, dtype=torch.uint8, device=dev)
    kernels.catalog_encode(kd, k_proj.to(dev), cb.to(dev), 0, 1500, k_low, codes)
    torch.cuda.synchronize()
    k_ref, c_ref = O.build_catalog(keys.float().numpy(), k_proj.numpy(), cb.numpy(), 2)
    np.testing.assert_array_equal(k_low.cpu().numpy(), k_ref)
    np.testing.assert_array_equal(codes.cpu().numpy(), c_ref.astype(np.uint8))


def test_register_write_path_device_start():
    """sva_catalog_encode_at with more than the append kernel's key count: the bulk kernel reads
    its start row on the device and stops at the limit."""
    keys, k_proj, cb = _case(torch.bfloat16, 3, 1, 900, 4, 64, seed=9)
    dev = torch.device("cuda")
    kd = keys.contiguous().to(dev)
    k_low = torch.zeros(3, 900, 64, device=dev)
    codes = torch.zeros(3, 900, 4, dtype=torch.uint8, device=dev)
    start = torch.tensor([300], dtype=torch.int64, device=dev)
    kernels.catalog_encode_at(kd, k_proj.to(dev), cb.to(dev), start, 700, 900, k_low, codes)
    torch.cuda.synchronize()
    k_ref, c_ref = O.build_catalog(keys.float().numpy(), k_proj.numpy(), cb.numpy(), 1)
    np.testing.assert_array_equal(k_low[:, 300:].cpu().numpy(), k_ref[:, 300:])
    np.testing.assert_array_equal(codes[:, 300:].cpu().numpy(), c_ref[:, 300:].astype(np.uint8))
    assert (k_low[:, :300] == 0).all() and (codes[:, :300] == 0).all()
