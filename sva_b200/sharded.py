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
import math
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


def default_exchange_width(shortlist: int, world: int) -> int:
    """Entries each rank sends per problem in the first exchange: the expected share of the
    global shortlist, shortlist / world, plus eight standard deviations of a binomial share plus
    32, capped at the shortlist.  A rank holding more members than that (keys clustered in one
    shard) makes the decode repeat the exchange at full width, so the width only affects speed."""
    if world <= 1:
        return int(shortlist)
    share = shortlist / world
    return int(min(shortlist, math.ceil(share + 8.0 * math.sqrt(share) + 32)))


class BatchedShardedDecoder:
    """Exact scan decode of a batch of sequences whose catalogs are sharded across ranks
    (sva_shard_batched_*, include/sva_b200.h "Batched shards").

    Each call decodes one token of every sequence (q [B, H, 1, D]) in four stages with three
    all-gathers; the first two exchange ``exchange_width`` entries per problem instead of the
    whole shortlist.  ``page_dealt`` selects the page-dealt numbering (global page g of every
    sequence on rank g % world; needs a paged layout) instead of key ranges starting at
    ``key_offset``.  The shortlist, final sets and outputs equal a one-GPU decode of the whole
    caches (outputs up to the order of exact fp64 sums); when a rank holds more shortlist members
    than the exchange width, the rescore stage flags it and the call repeats the first two
    exchanges at full width (``check_saturation``; each call then reads one flag on the host).
    """

    def __init__(self, group, shortlist: int, budget: int, device: torch.device, exchange_width: int | None = None,
                 check_saturation: bool = True) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.shortlist, self.budget = int(shortlist), int(budget)
        self.device = device
        self.width = int(exchange_width) if exchange_width else default_exchange_width(self.shortlist, self.world)
        self.check_saturation = bool(check_saturation)
        self._ws = kernels.Workspace()
        self._nccl = group is not None and dist.get_backend(group) == "nccl"
        self.fallbacks = 0
        self.stage_events = None  # optional list of 7 CUDA events recorded between the stages

    def full_width(self):
        """Context manager: calls inside it exchange the whole shortlist (never saturate)."""
        import contextlib

        @contextlib.contextmanager
        def ctx():
            saved = self.width
            self.width = self.shortlist
            try:
                yield self
            finally:
                self.width = saved

        return ctx()

    def _gather(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t.unsqueeze(0)
        out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        if self._nccl:
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        else:
            dist.all_gather(list(out.unbind(0)), t.contiguous(), group=self.group)
        return out

    def _mark(self, i: int) -> None:
        if self.stage_events is not None:
            self.stage_events[i].record()

    def decode(self, q, q_proj, scale, codebooks, codes, k_low, keys, values, *, seq_lens=None, page_table=None,
               max_len=None, key_offset: int = 0, page_dealt: bool = False, out=None, logits_mode: int = 0,
               softmax_scale: float | None = None, stats=None, saturated: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's local arrays in decode_batched's layouts; returns out [B, H, 1, D].

        With ``saturated`` (an int32 device tensor of one element, zeroed by the caller) the call
        reads nothing back on the host: it runs at the exchange width only and ORs the rescore
        stage's flag into ``saturated``, so that it can be captured in a CUDA graph; a caller that
        finds the flag set must repeat the call with ``full_width()`` in effect.
        """
        if q.dim() != 4 or q.shape[2] != 1:
            raise ValueError("batched sharded decode takes one query token per sequence and head: q [B, H, 1, D]")
        a, lay, out = kernels.batched_args(q, q_proj, scale, codebooks, codes, k_low, keys, values, self.shortlist,
                                           self.budget, seq_lens=seq_lens, page_table=page_table, max_len=max_len,
                                           softmax_scale=softmax_scale, logits_mode=logits_mode, out=out,
                                           stats=stats)
        m = _lib.ShardMap()
        m.key_offset = int(key_offset)
        m.page_world = self.world if page_dealt else 0
        m.page_rank = self.rank if page_dealt else 0
        lib = _lib.load()
        P = int(q.shape[0] * q.shape[1])
        D = int(q.shape[3])
        stream = kernels._stream(q.device)
        width = min(self.width, self.shortlist)
        self._mark(0)
        for attempt in range(2):
            ws_bytes = int(lib.sva_shard_batched_workspace_size(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m),
                                                                width))
            if ws_bytes == 0:
                _lib.check(lib.sva_shard_batched_summon(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m), width,
                                                        None, None, 0, None))
            ws = self._ws.get(q.device, ws_bytes)
            top = torch.empty(P, width, dtype=torch.int64, device=q.device)
            _lib.check(lib.sva_shard_batched_summon(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m), width,
                                                    top.data_ptr(), ws.data_ptr(), ws_bytes, stream))
            self._mark(1)
            g_top = self._gather(top)
            self._mark(2)
            rec = torch.empty(P, width, 4, dtype=torch.int32, device=q.device)
            sat = saturated if saturated is not None else torch.zeros(1, dtype=torch.int32, device=q.device)
            _lib.check(lib.sva_shard_batched_rescore(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m), width,
                                                     self.world, self.rank, g_top.data_ptr(), rec.data_ptr(),
                                                     sat.data_ptr(), ws.data_ptr(), ws_bytes, stream))
            self._mark(3)
            # every rank reads the same flag (it is computed from the same gathered lists)
            if (saturated is not None or width >= self.shortlist or not self.check_saturation
                    or int(sat.item()) == 0):
                break
            self.fallbacks += 1
            width = self.shortlist
        g_rec = self._gather(rec)
        self._mark(4)
        part = torch.empty(P, D, dtype=torch.float64, device=q.device)
        _lib.check(lib.sva_shard_batched_verify(ctypes.byref(a), ctypes.byref(lay), ctypes.byref(m), width,
                                                self.world, self.rank, g_rec.data_ptr(), part.data_ptr(), stream))
        g_part = self._gather(part)
        self._mark(5)
        _lib.check(lib.sva_shard_batched_combine(ctypes.byref(a), ctypes.byref(lay), self.world, g_part.data_ptr(),
                                                 stream))
        self._mark(6)
        return out


class ShardedInvertedDecoder:
    """Exact static inverted-index decode (reference sva/llama.py:427-576) over a key-range sharded
    static catalog (sva_inverted_shard_*, include/sva_b200.h): one token per head, two
    all-gathers (the ranks' top-budget candidate records, then the fp64 partial outputs).

    Each rank passes its own codes / k_low / keys / values and posting lists over its keys
    [key_offset, key_offset + L_r); ``global_max_bucket`` is the largest posting list of the whole
    catalog (``global_max_bucket(postings, group)`` computes it once per catalog), and the rank
    holding the global last key must pass ``holds_current=True``.
    """

    def __init__(self, group, budget: int, cells: int = 8, min_budget: int | None = None,
                 mid_budget: int | None = None, low_margin: float = 0.35, high_margin: float = 0.70) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.budget, self.cells = int(budget), int(cells)
        self.min_budget = int(min_budget or budget)
        self.mid_budget = int(mid_budget or max(self.min_budget, budget // 2))
        self.low_margin, self.high_margin = float(low_margin), float(high_margin)
        self._ws = kernels.Workspace()
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

    def decode(self, q, q_proj, scale, codebooks, codes, postings, k_low, keys, values, *, key_offset: int,
               holds_current: bool, global_max_bucket: torch.Tensor, out=None, softmax_scale=None, stats=None):
        a, out = kernels.inverted_args(q, q_proj, scale, codebooks, codes, postings, k_low, keys, values, self.budget,
                                       self.cells, self.min_budget, self.mid_budget, self.low_margin,
                                       self.high_margin, False, 2, None, None, softmax_scale, out, stats,
                                       max_bucket=global_max_bucket)
        lib = _lib.load()
        ws_bytes = int(lib.sva_inverted_shard_workspace_size(ctypes.byref(a)))
        if ws_bytes == 0:
            _lib.check(lib.sva_inverted_shard_summon(ctypes.byref(a), int(key_offset), int(holds_current), None, None,
                                                     0, None))
        ws = self._ws.get(q.device, ws_bytes)
        stream = kernels._stream(q.device)
        H = int(q.shape[0])
        rec = torch.empty(H, self.budget, 4, dtype=torch.int32, device=q.device)
        _lib.check(lib.sva_inverted_shard_summon(ctypes.byref(a), int(key_offset), int(holds_current), rec.data_ptr(),
                                                 ws.data_ptr(), ws_bytes, stream))
        g_rec = self._gather(rec)
        part = torch.empty(H, int(q.shape[1]), dtype=torch.float64, device=q.device)
        _lib.check(lib.sva_inverted_shard_verify(ctypes.byref(a), int(key_offset), int(holds_current), self.world,
                                                 self.rank, g_rec.data_ptr(), part.data_ptr(), ws.data_ptr(), ws_bytes,
                                                 stream))
        g_part = self._gather(part)
        _lib.check(lib.sva_inverted_shard_combine(ctypes.byref(a), self.world, g_part.data_ptr(), stream))
        return out


def global_max_bucket(postings, group) -> torch.Tensor:
    """The largest posting list of a key-range sharded catalog: the maximum over (head, subspace,
    cell) of the cell sizes summed over the ranks (one all-reduce of the counts)."""
    counts = postings.counts.to(torch.int64).clone()
    if group is not None and dist.get_world_size(group) > 1:
        dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
    return counts.max().to(torch.int32).reshape(1)
