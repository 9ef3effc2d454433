"""Multi-threaded CPU decode used as the timed CPU baseline (TEST / BENCH INFRASTRUCTURE ONLY).

Same algorithm and canonical rules as ``oracle.sva_oracle.scan_decode`` (reference
sva/llama.py:171-328 and experiments/sva_million_cached_decode_benchmark.py:224-249), organised
for speed on the host: an O(n) partition-based canonical top-k and one worker thread per
(head, query) problem (numpy releases the GIL in the heavy calls).  Only ``bench.py`` (the
``cpu_baseline`` field and ``--impl reference``) and the tests use it.
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .sva_oracle import (bf16_bits_to_f32, build_lut, ordered_key, query_low, topk_canonical, tree_dot,
                         verify_one)


def topk_canonical_fast(scores: np.ndarray, k: int) -> np.ndarray:
    """``topk_canonical`` (score desc, index asc) in O(n) for NaN-free scores."""
    n = scores.shape[0]
    if k >= n:
        return topk_canonical(scores, k)
    keys = ordered_key(scores)
    kth = np.partition(keys, n - k)[n - k]
    above = np.flatnonzero(keys > kth)
    ties = np.flatnonzero(keys == kth)[: k - above.shape[0]]
    sel = np.concatenate([above, ties])
    return sel[np.lexsort((sel, ~keys[sel]))]


def adc_scores_one(lut_h: np.ndarray, codes_h: np.ndarray, rank: int) -> np.ndarray:
    """ADC scores of one (head, query): lut_h [S, C], codes_h [L, S] -> [L]."""
    acc = np.zeros(codes_h.shape[0], dtype=np.float32)
    for s in range(lut_h.shape[0]):
        acc = acc + np.take(lut_h[s], codes_h[:, s])
    return acc / np.float32(math.sqrt(rank))


def _rows(arr: np.ndarray, idx: np.ndarray) -> np.ndarray:
    rows = arr[idx]
    return bf16_bits_to_f32(rows) if rows.dtype == np.uint16 else rows.astype(np.float32)


def decode_problem(q: np.ndarray, q_proj_h: np.ndarray, scale_h: np.float32, codebooks_h: np.ndarray,
                   codes_h: np.ndarray, k_low_h: np.ndarray, keys_kv: np.ndarray, values_kv: np.ndarray,
                   shortlist: int, budget: int, scaling: float, dtype: str, logits_mode: int) -> np.ndarray:
    """One (head, query token) decode; keys/values may be float32 or bf16 bit patterns (uint16)."""
    rank = q_proj_h.shape[-1]
    ql = query_low(q[None, None, :], q_proj_h[None], None, np.asarray([scale_h], dtype=np.float32))
    lut = build_lut(ql, codebooks_h[None])[0, 0]
    scores = adc_scores_one(lut, codes_h, rank)
    key_len = codes_h.shape[0]
    sl = topk_canonical_fast(scores, min(shortlist, key_len))
    rs = tree_dot(k_low_h[sl], ql[0, 0][None, :]) / np.float32(math.sqrt(rank))
    keep = topk_canonical(rs, min(budget, sl.shape[0]))
    fin = sl[keep]
    ks = _rows(keys_kv, fin)
    vs = _rows(values_kv, fin)
    return verify_one(q, ks, vs, np.arange(fin.shape[0]), scaling, dtype, logits_mode)


class CpuDecoder:
    """Threaded CPU decode of H heads x 1 query over a resident catalog.

    Each head's key range is split into ``chunks`` pieces scored in parallel; every piece keeps
    its canonical top-``shortlist`` and the per-head merge takes the canonical top-``shortlist``
    of the union, which contains the global one (so the result is exact).
    """

    def __init__(self, q_proj, scale, codebooks, codes, k_low, keys, values, groups: int, threads: int | None = None):
        self.q_proj, self.scale, self.codebooks = q_proj, scale, codebooks
        self.codes, self.k_low, self.keys, self.values = codes, k_low, keys, values
        self.groups = groups
        self.threads = threads or (os.cpu_count() or 1)
        self.pool = ThreadPoolExecutor(max_workers=self.threads)
        n_heads = q_proj.shape[0]
        self.chunks = max(1, self.threads // n_heads)

    def __call__(self, q: np.ndarray, shortlist: int, budget: int, scaling: float, dtype: str,
                 logits_mode: int = 1, want_final: bool = False):
        """Outputs [H, D] (and, with want_final, every head's final key set, ascending)."""
        n_heads, _, rank = self.q_proj.shape
        key_len = self.codes.shape[1]
        sl_cap = min(shortlist, key_len)
        qls = [query_low(q[h][None, None, :], self.q_proj[h][None], None,
                         np.asarray([self.scale[h]], dtype=np.float32)) for h in range(n_heads)]
        luts = [build_lut(qls[h], self.codebooks[h][None])[0, 0] for h in range(n_heads)]
        bounds = np.linspace(0, key_len, self.chunks + 1).astype(np.int64)

        def piece(arg):
            h, c = arg
            lo, hi = int(bounds[c]), int(bounds[c + 1])
            sc = adc_scores_one(luts[h], self.codes[h, lo:hi], rank)
            sel = topk_canonical_fast(sc, min(sl_cap, hi - lo))
            return sel + lo, sc[sel]

        parts = list(self.pool.map(piece, [(h, c) for h in range(n_heads) for c in range(self.chunks)]))

        def finish(h):
            idx = np.concatenate([parts[h * self.chunks + c][0] for c in range(self.chunks)])
            sc = np.concatenate([parts[h * self.chunks + c][1] for c in range(self.chunks)])
            keys = ordered_key(sc)
            sl = idx[np.lexsort((idx, ~keys))[:sl_cap]]
            ql = qls[h][0, 0]
            rs = tree_dot(self.k_low[h][sl], ql[None, :]) / np.float32(math.sqrt(rank))
            keep = topk_canonical(rs, min(budget, sl.shape[0]))
            fin = sl[keep]
            kv = h // self.groups
            out = verify_one(q[h], _rows(self.keys[kv], fin), _rows(self.values[kv], fin),
                             np.arange(fin.shape[0]), scaling, dtype, logits_mode)
            return out, np.sort(fin)

        res = list(self.pool.map(finish, range(n_heads)))
        outs = np.stack([r[0] for r in res])
        return (outs, [r[1] for r in res]) if want_final else outs

    def close(self) -> None:
        self.pool.shutdown(wait=True)
