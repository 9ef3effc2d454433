"""Shared helpers for the GPU parity tests: run the CUDA path and the CPU oracle on one case."""

from __future__ import annotations

from functools import lru_cache

import numpy as np
import torch

from oracle import sva_oracle as O
from tests.golden.inputs import DecodeCase


def dtype_name(t: torch.Tensor) -> str:
    return {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}[t.dtype]


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def gpu_catalog(case: DecodeCase, device="cuda"):
    from sva_b200 import kernels

    keys = case.keys[0].to(device)
    n_heads, key_len = case.n_heads, case.key_len
    rank = int(case.k_proj.shape[-1])
    subspaces = int(case.codebooks.shape[1])
    k_low = torch.empty(n_heads, key_len, rank, dtype=torch.float32, device=device)
    codes = torch.empty(n_heads, key_len, subspaces, dtype=torch.uint8, device=device)
    kernels.catalog_encode(keys, case.k_proj.to(device), case.codebooks.to(device), 0, key_len, k_low, codes)
    return k_low, codes


def gpu_decode(case: DecodeCase, k_low: torch.Tensor, codes: torch.Tensor, device="cuda", logits_mode: int = 1,
               shortlist: int | None = None, budget: int | None = None, q: torch.Tensor | None = None, **kw):
    from sva_b200 import kernels

    q = (case.q[0] if q is None else q).to(device)
    return kernels.decode(
        q, case.q_proj.to(device), kernels.sva_scale(case.logit_scale).to(device), case.codebooks.to(device), codes,
        k_low, case.keys[0].to(device), case.values[0].to(device), case.shortlist if shortlist is None else shortlist,
        case.budget if budget is None else budget, softmax_scale=float(case.q.shape[-1]) ** -0.5,
        logits_mode=logits_mode, want_shortlist=True, want_final=True, **kw)


def oracle_catalog(case: DecodeCase):
    groups = case.n_heads // case.n_kv_heads
    return O.build_catalog(to_np(case.keys[0]), case.k_proj.numpy(), case.codebooks.numpy(), groups)


def oracle_decode(case: DecodeCase, k_low: np.ndarray, codes: np.ndarray, logits_mode: int = 1,
                  shortlist: int | None = None, budget: int | None = None, q: torch.Tensor | None = None, **kw):
    q = case.q[0] if q is None else q
    return O.scan_decode(to_np(q), case.q_proj.numpy(), case.logit_scale.numpy(), case.codebooks.numpy(),
                         np.asarray(codes, dtype=np.int64), k_low, to_np(case.keys[0]), to_np(case.values[0]),
                         case.shortlist if shortlist is None else shortlist, case.budget if budget is None else budget,
                         float(case.q.shape[-1]) ** -0.5, dtype_name(case.q), logits_mode,
                         scale=case.logit_scale.float().exp().clamp(0.01, 100.0).numpy(), **kw)


def tolerance(case: DecodeCase):
    return (1e-3, 1e-3) if case.q.dtype == torch.float32 else (2e-2, 2e-2)


def unpad(row: np.ndarray) -> np.ndarray:
    return row[row >= 0]


@lru_cache(maxsize=None)
def cached_case(name: str):
    from tests.golden.inputs import config1, config2

    table = {
        "cfg1": lambda: config1(),
        "cfg2s_1x256": lambda: config2(key_len=1 << 16, subspaces=1, codewords=256),
        "cfg2s_4x64": lambda: config2(key_len=1 << 16, subspaces=4, codewords=64),
    }
    case = table[name]()
    return case, oracle_catalog(case)
