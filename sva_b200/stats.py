"""Runtime accounting with device-side counters (API of the reference's sva/stats.py:13-54).

The CUDA kernels add their per-query counts (queries, summoned, refill pool, exact-scored,
verified, cell visits) into a small int64 tensor per patched layer on its own device, so a
decode step performs no host synchronisation for bookkeeping.  The host-side totals are
brought up to date lazily, with one device read per layer, whenever ``totals``, ``by_layer``,
``ratio`` or ``summary`` is used.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Iterable

import torch

from . import _lib

DEVICE_STAT_NAMES = {
    _lib.STAT_QUERIES: "queries",
    _lib.STAT_SUMMONED: "summoned",
    _lib.STAT_REFILL_POOL: "refill_pool",
    _lib.STAT_EXACT_SCORED: "exact_scored",
    _lib.STAT_VERIFIED: "verified",
    _lib.STAT_CELL_VISITS: "cell_visits",
}


def _float_stats() -> defaultdict[str, float]:
    return defaultdict(float)


class SVAStats:
    """Mutable aggregate statistics recorded by patched attention layers."""

    def __init__(self) -> None:
        self._totals: defaultdict[str, float] = _float_stats()
        self._by_layer: defaultdict[int, defaultdict[str, float]] = defaultdict(_float_stats)
        self._device: dict[int, torch.Tensor] = {}

    # -- device counters -----------------------------------------------------------------
    def device_counters(self, layer_idx: int, device: torch.device) -> torch.Tensor:
        """The int64 counter block the kernels of ``layer_idx`` accumulate into."""
        buf = self._device.get(layer_idx)
        if buf is None or buf.device != torch.device(device):
            if buf is not None:
                self._flush_one(layer_idx, buf)
            buf = torch.zeros(_lib.STAT_COUNT, dtype=torch.int64, device=device)
            self._device[layer_idx] = buf
        return buf

    def _flush_one(self, layer_idx: int, buf: torch.Tensor) -> None:
        vals = buf.tolist()
        buf.zero_()
        add = {name: float(vals[i]) for i, name in DEVICE_STAT_NAMES.items() if vals[i]}
        if add:
            self._add(layer_idx, add)

    def flush(self) -> None:
        for layer_idx, buf in list(self._device.items()):
            self._flush_one(layer_idx, buf)

    # -- reference API ---------------------------------------------------------------------
    @property
    def totals(self) -> defaultdict[str, float]:
        self.flush()
        return self._totals

    @property
    def by_layer(self) -> defaultdict[int, defaultdict[str, float]]:
        self.flush()
        return self._by_layer

    def reset(self) -> None:
        for buf in self._device.values():
            buf.zero_()
        self._totals.clear()
        self._by_layer.clear()

    def _add(self, layer_idx: int, values: dict[str, float]) -> None:
        layer = self._by_layer[layer_idx]
        for key, value in values.items():
            self._totals[key] += value
            layer[key] += value

    def add(self, layer_idx: int, values: dict[str, float]) -> None:
        self._add(layer_idx, values)

    def ratio(self, numerator: str, denominator: str = "queries") -> float:
        totals = self.totals
        total = totals.get(denominator, 0.0)
        if total <= 0:
            return float("nan")
        return totals.get(numerator, 0.0) / total

    def summary(self) -> dict[str, float]:
        totals = self.totals
        keys: Iterable[tuple[str, str, str]] = (
            ("avg_summoned", "summoned", "queries"),
            ("avg_refill_pool", "refill_pool", "queries"),
            ("avg_exact_scored", "exact_scored", "queries"),
            ("avg_verified", "verified", "queries"),
            ("avg_cell_visits", "cell_visits", "queries"),
            ("avg_static_catalog_ms", "static_catalog_ms", "profile_calls"),
            ("avg_static_refill_ms", "static_refill_ms", "profile_calls"),
            ("avg_static_budget_ms", "static_budget_ms", "profile_calls"),
            ("avg_static_gather_ms", "static_gather_ms", "profile_calls"),
            ("avg_static_exact_score_ms", "static_exact_score_ms", "profile_calls"),
            ("avg_static_aggregate_ms", "static_aggregate_ms", "profile_calls"),
            ("avg_static_total_ms", "static_total_ms", "profile_calls"),
            ("avg_static_projection_ms", "static_projection_ms", "profile_outer_calls"),
            ("avg_static_key_catalog_ms", "static_key_catalog_ms", "profile_outer_calls"),
            ("avg_static_outer_total_ms", "static_outer_total_ms", "profile_outer_calls"),
        )
        out = {"queries": totals.get("queries", 0.0)}
        for name, num, den in keys:
            out[name] = self.ratio(num, den)
        return out
