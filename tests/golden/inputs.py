"""Seeded synthetic inputs for the SVA decode configurations (test infrastructure).

The draw order of every recipe is fixed, and all draws use a CPU ``torch.Generator`` so that
the reference (run in the build container), the numpy oracle and the CUDA path (after a copy
to the device) see identical bytes.  These recipes stand in for the reference's benchmark
inputs: the reference's million-key benchmark draws iid normal caches
(experiments/sva_million_cached_decode_benchmark.py:97-136); the planted near-duplicate keys
follow the configuration text of this build (0.9 * q + 0.1 * noise).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class DecodeCase:
    name: str
    q: torch.Tensor            # [1, H, 1, D]
    keys: torch.Tensor         # [1, Hkv, L, D]
    values: torch.Tensor       # [1, Hkv, L, D]
    q_proj: torch.Tensor       # [H, D, R] float32
    k_proj: torch.Tensor       # [H, D, R] float32
    logit_scale: torch.Tensor  # [H] float32
    codebooks: torch.Tensor    # [H, S, C, R/S] float32
    shortlist: int
    budget: int
    planted: torch.Tensor      # [Hkv, n_planted] positions

    @property
    def n_heads(self) -> int:
        return int(self.q.shape[1])

    @property
    def n_kv_heads(self) -> int:
        return int(self.keys.shape[1])

    @property
    def key_len(self) -> int:
        return int(self.keys.shape[2])


def _plant(gen: torch.Generator, q: torch.Tensor, keys: torch.Tensor, n_planted: int, dtype: torch.dtype):
    """Overwrite ``n_planted`` seeded positions per KV head with 0.9*q + 0.1*noise.

    The query used for KV head g is query head g * groups (the first head of the group).
    """
    n_heads = q.shape[1]
    n_kv, length, head_dim = keys.shape[1:]
    groups = n_heads // n_kv
    positions = torch.stack([torch.randperm(length, generator=gen)[:n_planted] for _ in range(n_kv)])
    noise = torch.randn(n_kv, n_planted, head_dim, generator=gen)
    for g in range(n_kv):
        base = q[0, g * groups, 0].float()
        keys[0, g, positions[g]] = (0.9 * base[None, :] + 0.1 * noise[g]).to(dtype)
    return positions


def config1(seed: int = 0, key_len: int = 8192) -> DecodeCase:
    """Single-layer fp32 op: 9 query / 3 KV heads, head_dim 64, rank 64, 2x256 codes."""
    gen = torch.Generator().manual_seed(seed)
    n_heads, n_kv, head_dim, rank, subspaces, codewords = 9, 3, 64, 64, 2, 256
    q = torch.randn(1, n_heads, 1, head_dim, generator=gen)
    keys = torch.randn(1, n_kv, key_len, head_dim, generator=gen)
    values = torch.randn(1, n_kv, key_len, head_dim, generator=gen)
    planted = _plant(gen, q, keys, 16, torch.float32)
    q_proj = torch.randn(n_heads, head_dim, rank, generator=gen) * 0.125
    k_proj = torch.randn(n_heads, head_dim, rank, generator=gen) * 0.125
    codebooks = torch.randn(n_heads, subspaces, codewords, rank // subspaces, generator=gen)
    return DecodeCase("config1", q, keys, values, q_proj, k_proj, torch.zeros(n_heads), codebooks, 2048, 512, planted)


def config2(seed: int = 0, key_len: int = 1 << 20, subspaces: int = 4, codewords: int = 64, n_heads: int = 1,
            n_planted: int = 64) -> DecodeCase:
    """Million-key bf16 lookup: ``n_heads`` independent heads (one KV head each), rank 64.

    Projections and codebooks are rounded to bf16 values (real bundles store bf16 artifacts).
    """
    gen = torch.Generator().manual_seed(seed)
    head_dim, rank = 64, 64
    n_kv = n_heads
    q = torch.randn(1, n_heads, 1, head_dim, generator=gen).to(torch.bfloat16)
    keys = torch.randn(1, n_kv, key_len, head_dim, generator=gen).to(torch.bfloat16)
    values = torch.randn(1, n_kv, key_len, head_dim, generator=gen).to(torch.bfloat16)
    planted = _plant(gen, q, keys, n_planted, torch.bfloat16)
    q_proj = (torch.randn(n_heads, head_dim, rank, generator=gen) * 0.125).to(torch.bfloat16).float()
    k_proj = (torch.randn(n_heads, head_dim, rank, generator=gen) * 0.125).to(torch.bfloat16).float()
    codebooks = torch.randn(n_heads, subspaces, codewords, rank // subspaces, generator=gen).to(torch.bfloat16).float()
    return DecodeCase(f"config2_{subspaces}x{codewords}", q, keys, values, q_proj, k_proj, torch.zeros(n_heads),
                      codebooks, 2048, 512, planted)


def tiny_bundle_tensors(seed: int = 11):
    """The two-layer rank-4 artifact of the reference unit tests (tests/test_sva_llama_adapter.py:28-54)."""
    gen = torch.Generator().manual_seed(seed)
    layers = {}
    for layer_idx in range(2):
        layers[layer_idx] = dict(
            q_proj=torch.randn(2, 8, 4, generator=gen),
            k_proj=torch.randn(2, 8, 4, generator=gen),
            logit_scale=torch.zeros(2),
            coarse_codebooks=torch.randn(2, 2, 8, 2, generator=gen),
        )
    return layers


def tiny_manifest() -> dict:
    return {
        "schema_version": 1,
        "artifact_type": "summon_verify_attention",
        "rank_dim": 4,
        "coarse_subspaces": 2,
        "coarse_codewords": 8,
        "default_shortlist": 4,
        "default_budget": 2,
        "layer_count": 2,
        "layers": [0, 1],
    }
