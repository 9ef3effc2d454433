"""Key-range sharded scan decode over torch.distributed, one process per GPU.

The million-key caches of the reference's scan path (sva/llama.py:171-328, one device) are split
by key range: rank r holds keys [key_offset, key_offset + L_r) of every head (codes, k_low, K,
V).  One decode of one token per head runs four stages of CUDA kernels with three all-gathers
between them (include/sva_b200.h, "Key-range shards"):

  summon  -> all-gather of the local top-SL coarse composites [W, H, SL]
  rescore -> all-gather of the (rank composite, logit) records of the global shortlist's
             members [W, H, SL, 4]
  verify  -> all-gather of the fp64 partial outputs [W, H, D]
  combine -> the output

Every rank takes the same collectives in the same order.  Shortlist and final sets equal the
single-GPU decode over the concatenated keys (same per-key arithmetic, exact selections under
the canonical tie rule), and the output equals it up to the order of exact fp64 sums.

The stage kernels sit behind a backend object so that the protocol itself can be exercised
with CPU ranks (``gloo``) and a host-side backend in the tests; the product backend is
:class:`CudaShardBackend`, and there is no fallback.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from . import _lib, kernels


@dataclass
class ShardCall:
    """One rank's view of one sharded decode (the per-stage state the backend keeps)."""

    args: Any
    out: torch.Tensor
    key_offset: int
    heads: int
    head_dim: int
    shortlist: int
    device: torch.device
    workspace: torch.Tensor | None = None
    ws_bytes: int = 0
    tensors: tuple = ()  # the inputs whose pointers ``args`` holds, kept alive for the call


class CudaShardBackend:
    """The stage kernels of libsva_b200 (sva_shard_summon / _rescore / _verify / _combine)."""

    launches_per_decode = 6  # prep, scan, top, rescore, verify, combine

    def __init__(self) -> None:
        self._ws = kernels.Workspace()

    def prepare(self, q, q_proj, scale, codebooks, codes, k_low, keys, values, *, shortlist: int, budget: int,
                key_offset: int, out=None, logits_mode: int = 0, softmax_scale: float | None = None,
                stats=None) -> ShardCall:
        if q.dim() != 3 or q.shape[1] != 1:
            raise ValueError("sharded decode takes one query token per head: q [H, 1, D]")
        a, out = kernels.decode_args(q, q_proj, scale, codebooks, codes, k_low, keys, values, shortlist, budget,
                                     softmax_scale, logits_mode, out=out, stats=stats)
        lib = _lib.load()
        ws_bytes = int(lib.sva_shard_workspace_size(ctypes.byref(a)))
        if ws_bytes == 0:
            _lib.check(lib.sva_shard_summon(ctypes.byref(a), int(key_offset), None, None, 0, None))
        ws = self._ws.get(q.device, ws_bytes)
        keep = (q, q_proj, scale, codebooks, codes, k_low, keys, values, stats)
        return ShardCall(a, out, int(key_offset), int(q.shape[0]), int(q.shape[2]), int(shortlist), q.device, ws,
                         ws_bytes, keep)

    def summon(self, c: ShardCall) -> torch.Tensor:
        top = torch.empty(c.heads, c.shortlist, dtype=torch.int64, device=c.device)
        lib = _lib.load()
        _lib.check(lib.sva_shard_summon(ctypes.byref(c.args), c.key_offset, top.data_ptr(), c.workspace.data_ptr(),
                                        c.ws_bytes, kernels._stream(c.device)))
        return top

    def rescore(self, c: ShardCall, gathered_top: torch.Tensor, world: int, rank: int) -> torch.Tensor:
        rec = torch.empty(c.heads, c.shortlist, 4, dtype=torch.int32, device=c.device)
        lib = _lib.load()
        _lib.check(lib.sva_shard_rescore(ctypes.byref(c.args), c.key_offset, world, rank, gathered_top.data_ptr(),
                                         rec.data_ptr(), c.workspace.data_ptr(), c.ws_bytes,
                                         kernels._stream(c.device)))
        return rec

    def verify(self, c: ShardCall, gathered_records: torch.Tensor, world: int, rank: int) -> torch.Tensor:
        part = torch.empty(c.heads, c.head_dim, dtype=torch.float64, device=c.device)
        lib = _lib.load()
        _lib.check(lib.sva_shard_verify(ctypes.byref(c.args), c.key_offset, world, rank, gathered_records.data_ptr(),
                                        part.data_ptr(), kernels._stream(c.device)))
        return part

    def combine(self, c: ShardCall, gathered_partials: torch.Tensor, world: int) -> torch.Tensor:
        lib = _lib.load()
        _lib.check(lib.sva_shard_combine(ctypes.byref(c.args), world, gathered_partials.data_ptr(),
                                         kernels._stream(c.device)))
        return c.out


class ShardedDecoder:
    """Exact scan decode over a key-range sharded catalog (see the module docstring).

    ``group`` is the process group of the ranks that hold the shards (rank order = key order is
    not required: the global indices travel with the candidates).  ``decode`` takes this rank's
    arrays: q [H, 1, D]; codes [H, L_r, S] uint8; k_low [H, L_r, R] fp32; keys / values
    [Hkv, L_r, D]; ``key_offset`` the global index of local key 0.  Returns out [H, 1, D].
    """

    def __init__(self, group, heads: int, head_dim: int, shortlist: int, budget: int,
                 device: torch.device | None = None, backend=None) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.heads, self.head_dim = int(heads), int(head_dim)
        self.shortlist, self.budget = int(shortlist), int(budget)
        self.device = device
        self.backend = backend if backend is not None else CudaShardBackend()
        self.extra_launches = getattr(self.backend, "launches_per_decode", 6) - 3
        self._nccl = group is not None and dist.get_backend(group) == "nccl"

    def _gather(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t.unsqueeze(0)
        out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        if self._nccl:
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        else:
            dist.all_gather(list(out.unbind(0)), t.contiguous(), group=self.group)
        return out

    def decode(self, q, q_proj, scale, codebooks, codes, k_low, keys, values, *, key_offset: int, out=None,
               logits_mode: int = 0, softmax_scale: float | None = None, stats=None) -> torch.Tensor:
        call = self.backend.prepare(q, q_proj, scale, codebooks, codes, k_low, keys, values,
                                    shortlist=self.shortlist, budget=self.budget, key_offset=key_offset, out=out,
                                    logits_mode=logits_mode, softmax_scale=softmax_scale, stats=stats)
        top = self.backend.summon(call)
        records = self.backend.rescore(call, self._gather(top), self.world, self.rank)
        partial = self.backend.verify(call, self._gather(records), self.world, self.rank)
        return self.backend.combine(call, self._gather(partial), self.world)
