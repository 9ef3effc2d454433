"""Core SVA tensor operations on the GPU (signatures of the reference's sva/ops.py).

Every function runs a CUDA kernel of libsva_b200.so on CUDA tensors and raises on CPU
tensors; there is no CPU fallback.  Results use the canonical arithmetic of the kernels
(sequential fp32 dot products, lowest index on ties), which the reference's own outputs
match up to summation-order ulps.
"""

from __future__ import annotations

import torch

from . import kernels


@torch.no_grad()
def assign_to_centroids(x: torch.Tensor, centroids: torch.Tensor, chunk_size: int = 8192) -> torch.Tensor:
    """Nearest centroid of every row of ``x`` by (|x|^2 - 2 x.c) + |c|^2 (reference sva/ops.py:10-21).

    ``chunk_size`` is accepted for signature compatibility; the kernel needs no chunking.
    """
    del chunk_size
    return kernels.assign_centroids(x, centroids.to(x.device))


@torch.no_grad()
def encode_product_keys(k_low: torch.Tensor, codebooks: torch.Tensor, chunk_size: int = 8192) -> torch.Tensor:
    """Product-quantised codes [H, L, S] (int64) of low-rank keys [H, L, R] (reference sva/ops.py:24-47)."""
    del chunk_size
    n_heads, _, rank_dim = k_low.shape
    subspaces = codebooks.shape[1]
    if rank_dim % subspaces != 0:
        raise ValueError(f"rank_dim={rank_dim} must be divisible by subspaces={subspaces}.")
    sub = rank_dim // subspaces
    out = torch.empty(n_heads, k_low.shape[1], subspaces, dtype=torch.int64, device=k_low.device)
    cb = codebooks.to(k_low.device)
    for h in range(n_heads):
        for s in range(subspaces):
            out[h, :, s] = kernels.assign_centroids(k_low[h, :, s * sub:(s + 1) * sub], cb[h, s])
    return out


@torch.no_grad()
def product_quantized_scores(q_low: torch.Tensor, codebooks: torch.Tensor, codes: torch.Tensor,
                             rank_dim: int) -> torch.Tensor:
    """ADC scores [H, T, L]: sum over subspaces of (q part . codeword), / sqrt(rank) (reference sva/ops.py:50-71)."""
    codes_u8 = codes.to(device=q_low.device, dtype=torch.uint8)
    return kernels.pq_scores(q_low, codebooks.to(q_low.device), codes_u8, rank_dim)
