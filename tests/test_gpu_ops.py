"""GPU parity of the operator surface of the reference's sva/ops.py (sva_b200.ops).

assign_to_centroids, encode_product_keys and product_quantized_scores run the CUDA kernels
behind sva_assign_centroids / sva_pq_scores.  They use the canonical arithmetic of the oracle
(sequential fp32 dot products, lowest index on ties), so labels, codes and scores must be
bit-identical to oracle/sva_oracle.py; codes are also checked against the reference's own codes
(tests/golden/golden_v1.npz), and scores against scores built from the reference's own LUT
within fp32 rounding.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import sva_oracle as O
from tests.helpers import cached_case

pytestmark = pytest.mark.gpu

GOLDEN = np.load(__file__.replace("test_gpu_ops.py", "golden/golden_v1.npz"))
CASES = ["cfg1", "cfg2s_1x256", "cfg2s_4x64"]


@pytest.mark.parametrize("dim,codewords,n", [(32, 256, 5000), (16, 64, 4099), (64, 256, 1), (7, 3, 777)])
def test_assign_to_centroids_matches_oracle(dim, codewords, n):
    from sva_b200 import ops

    gen = torch.Generator().manual_seed(dim * 1000 + codewords)
    x = torch.randn(n, dim, generator=gen)
    cents = torch.randn(codewords, dim, generator=gen)
    # duplicated centroids: the lowest index must win the tie
    cents[codewords // 2] = cents[0]
    got = ops.assign_to_centroids(x.cuda(), cents.cuda())
    assert got.dtype == torch.int64 and got.device.type == "cuda"
    np.testing.assert_array_equal(got.cpu().numpy(), O.assign_to_centroids(x.numpy(), cents.numpy()))


def test_assign_to_centroids_strided_rows():
    """A column slice of a wider matrix (the per-subspace view encode_product_keys passes)."""
    from sva_b200 import ops

    gen = torch.Generator().manual_seed(11)
    wide = torch.randn(3000, 64, generator=gen)
    cents = torch.randn(64, 16, generator=gen)
    got = ops.assign_to_centroids(wide.cuda()[:, 16:32], cents.cuda())
    np.testing.assert_array_equal(got.cpu().numpy(), O.assign_to_centroids(wide[:, 16:32].numpy(), cents.numpy()))


@pytest.mark.parametrize("name", CASES)
def test_encode_product_keys_matches_reference_codes(name):
    from sva_b200 import ops

    case, (k_low_ref, codes_ref) = cached_case(name)
    got = ops.encode_product_keys(torch.from_numpy(k_low_ref).cuda(), case.codebooks.cuda())
    assert got.dtype == torch.int64 and tuple(got.shape) == codes_ref.shape
    got = got.cpu().numpy()
    np.testing.assert_array_equal(got, codes_ref)
    np.testing.assert_array_equal(got, GOLDEN[f"{name}_codes"].astype(np.int64))


def test_encode_product_keys_rejects_bad_rank():
    from sva_b200 import ops

    with pytest.raises(ValueError):
        ops.encode_product_keys(torch.zeros(1, 8, 30, device="cuda"), torch.zeros(1, 4, 16, 7, device="cuda"))


@pytest.mark.parametrize("name", CASES)
def test_product_quantized_scores(name):
    from sva_b200 import ops

    case, (_, codes_ref) = cached_case(name)
    q_low = GOLDEN[f"{name}_q_low"]  # the reference's own q_low [H, 1, R]
    rank = q_low.shape[-1]
    got = ops.product_quantized_scores(torch.from_numpy(q_low).cuda(), case.codebooks.cuda(),
                                       torch.from_numpy(codes_ref).cuda(), rank)
    assert got.dtype == torch.float32 and tuple(got.shape) == (q_low.shape[0], 1, codes_ref.shape[1])
    got = got.cpu().numpy()
    # bit-exact against the oracle's canonical LUT and ADC order
    want = O.adc_scores(O.build_lut(q_low, case.codebooks.numpy()), codes_ref, rank)
    np.testing.assert_array_equal(got, want)
    # and within fp32 rounding of the scores built from the reference's own LUT
    ref = O.adc_scores(GOLDEN[f"{name}_lut"], codes_ref, rank)
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-4)


def test_product_quantized_scores_multi_token_int64_codes():
    """Several query tokens, int64 codes (the dtype encode_product_keys returns), 8 subspaces."""
    from sva_b200 import ops

    gen = torch.Generator().manual_seed(5)
    q_low = torch.randn(2, 3, 64, generator=gen)
    cb = torch.randn(2, 8, 32, 8, generator=gen)
    codes = torch.randint(0, 32, (2, 4097, 8), generator=gen)
    got = ops.product_quantized_scores(q_low.cuda(), cb.cuda(), codes.cuda(), 64).cpu().numpy()
    want = O.adc_scores(O.build_lut(q_low.numpy(), cb.numpy()), codes.numpy(), 64)
    np.testing.assert_array_equal(got, want)
    assert math.isclose(float(np.abs(got).max()), float(np.abs(want).max()))
