"""CPU oracle for the SVA summon -> verify decode path (TEST INFRASTRUCTURE ONLY).

This module is a numpy restatement of the reference algorithm (asystemoffields/sva,
``sva/ops.py`` and ``sva/llama.py``).  It exists so that tests, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` can check or time the
CUDA product path.  Nothing in the ``sva_b200`` package imports it; the product path has no
CPU fallback.

Two things are made canonical here, and the CUDA kernels implement exactly the same rules,
so that every integer output (codes, shortlist, final indices, postings) is bit-exact
between the oracle and the GPU:

* Tie rule.  Every ``topk`` of the reference is replaced by "score descending, then key
  index ascending".  The reference's CPU ``torch.topk`` breaks ties in an unspecified order;
  the golden fixtures under ``tests/golden`` pin this oracle against the reference with the
  same canonical rule applied to the reference's own scores.
* Summation order.  fp32 dot products follow one of two fixed orders with every multiply and
  add rounded separately (no fused multiply-add):

  - ``seq_dot``: ``acc = 0; for i: acc = acc + a[i] * b[i]`` (query projection, LUT,
    nearest-codeword distances, key projection of the exact write path);
  - ``tree_dot``: 16 lanes, lane ``j`` sums elements ``4j..4j+3`` sequentially, then the
    lanes are combined by a butterfly ``xor 8, 4, 2, 1`` (exact rank rescore and fp32
    verify logits; this is the order of a 16-lane shuffle reduction on the GPU).

The reference computes the same quantities with MKL / vectorised torch reductions whose
order is CPU-dependent, so oracle-vs-reference agreement on fp32 intermediates is to a few
ulps, and integer outputs agree except where two candidates sit within those ulps of the
selection boundary (the tests count such cases).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

F32 = np.float32
FINFO_MIN = np.float32(np.finfo(np.float32).min)


# ----------------------------------------------------------------------------------------
# dtype helpers
# ----------------------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bfloat16 bit patterns (uint16) to float32 exactly."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return rounded.astype(np.uint32).view(np.float32)


def round_to_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_to_bf16(x)
    if dtype == "f16":
        return round_to_f16(x)
    return np.asarray(x, dtype=np.float32)


# ----------------------------------------------------------------------------------------
# canonical fp32 arithmetic
# ----------------------------------------------------------------------------------------

def seq_dot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Sequential fp32 dot over the last axis: ((0 + a0*b0) + a1*b1) + ...; broadcasts."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    n = a.shape[-1]
    assert b.shape[-1] == n
    acc = np.zeros(np.broadcast_shapes(a.shape[:-1], b.shape[:-1]), dtype=np.float32)
    for i in range(n):
        acc = acc + a[..., i] * b[..., i]
    return acc


def tree_dot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """16-lane fp32 dot over the last axis (length <= 64, see module docstring)."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    n = a.shape[-1]
    assert b.shape[-1] == n and n <= 64
    shape = np.broadcast_shapes(a.shape[:-1], b.shape[:-1])
    lanes = []
    for j in range(16):
        p = np.zeros(shape, dtype=np.float32)
        for i in range(4 * j, min(4 * j + 4, n)):
            p = p + a[..., i] * b[..., i]
        lanes.append(p)
    for step in (8, 4, 2, 1):
        lanes = [lanes[j] + lanes[j ^ step] for j in range(16)]
    return lanes[0]


def ordered_key(scores: np.ndarray) -> np.ndarray:
    """Map float32 scores to uint32 keys whose unsigned order equals the float order.

    -0.0 is folded onto +0.0 first so that the two compare equal, as they do for topk.
    """
    u = np.ascontiguousarray(scores, dtype=np.float32).view(np.uint32).copy()
    u[u == 0x80000000] = 0
    neg = (u & 0x80000000) != 0
    return np.where(neg, ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def topk_canonical(scores: np.ndarray, k: int, valid: np.ndarray | None = None) -> np.ndarray:
    """Indices of the top-k entries of a 1-D score array, score desc then index asc.

    Invalid entries are never selected; fewer than k indices come back if fewer are valid.
    """
    scores = np.asarray(scores, dtype=np.float32)
    idx = np.arange(scores.shape[0], dtype=np.int64)
    if valid is not None:
        idx = idx[np.asarray(valid, dtype=bool)]
    keys = ordered_key(scores[idx])
    # lexsort: last key is primary -> primary = key descending, secondary = index ascending.
    order = np.lexsort((idx, ~keys))
    return idx[order[: min(k, idx.shape[0])]]


# ----------------------------------------------------------------------------------------
# write path: key catalog (reference sva/llama.py:578-624, sva/ops.py:10-47)
# ----------------------------------------------------------------------------------------

def project_keys(keys_f32: np.ndarray, k_proj: np.ndarray, groups: int) -> np.ndarray:
    """k_low[h, l, :] = K[h // groups, l, :] . Kproj[h]  (reference sva/llama.py:598,615).

    keys_f32: [Hkv, L, D]; k_proj: [H, D, R] -> [H, L, R] float32, seq_dot order over D.
    """
    n_heads, head_dim, rank = k_proj.shape
    out = np.empty((n_heads, keys_f32.shape[1], rank), dtype=np.float32)
    for h in range(n_heads):
        x = keys_f32[h // groups]
        acc = np.zeros((x.shape[0], rank), dtype=np.float32)
        for d in range(head_dim):
            acc = acc + x[:, d : d + 1] * k_proj[h, d][None, :].astype(np.float32)
        out[h] = acc
    return out


def assign_to_centroids(x: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """Nearest centroid by (|x|^2 - 2 x.c) + |c|^2, lowest index on ties.

    Follows reference sva/ops.py:10-21 (distance expansion and evaluation order).
    """
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(centroids, dtype=np.float32)
    xn = seq_dot(x, x)  # [N]
    cn = seq_dot(c, c)  # [C]
    best = np.zeros(x.shape[0], dtype=np.int64)
    best_d = None
    for ci in range(c.shape[0]):
        xc = seq_dot(x, c[ci][None, :])
        dist = (xn - np.float32(2.0) * xc) + cn[ci]
        if best_d is None:
            best_d = dist
        else:
            better = dist < best_d
            best = np.where(better, ci, best)
            best_d = np.where(better, dist, best_d)
    return best


def encode_product_keys(k_low: np.ndarray, codebooks: np.ndarray) -> np.ndarray:
    """codes[h, l, s] = nearest codeword of subspace s (reference sva/ops.py:24-47)."""
    n_heads, length, rank = k_low.shape
    subspaces = codebooks.shape[1]
    sub = rank // subspaces
    codes = np.empty((n_heads, length, subspaces), dtype=np.int64)
    for h in range(n_heads):
        for s in range(subspaces):
            codes[h, :, s] = assign_to_centroids(k_low[h, :, s * sub : (s + 1) * sub], codebooks[h, s])
    return codes


def build_catalog(keys_f32: np.ndarray, k_proj: np.ndarray, codebooks: np.ndarray, groups: int):
    k_low = project_keys(keys_f32, k_proj, groups)
    return k_low, encode_product_keys(k_low, codebooks)


# ----------------------------------------------------------------------------------------
# summon (reference sva/llama.py:211, sva/ops.py:50-71, sva/llama.py:270-302)
# ----------------------------------------------------------------------------------------

def query_low(q_f32: np.ndarray, q_proj: np.ndarray, logit_scale: np.ndarray, scale: np.ndarray | None = None) -> np.ndarray:
    """q_low[h, t, :] = (q[h, t, :] . Qproj[h]) * clamp(exp(logit_scale[h]), 0.01, 100).

    Reference sva/llama.py:69-73 (scale buffer) and :211 (einsum then scale).  ``scale`` may be
    given precomputed (the reference computes it once with torch at patch time).
    """
    if scale is None:
        scale = sva_scale(logit_scale)
    scale = np.asarray(scale, dtype=np.float32)
    n_heads, n_q, head_dim = q_f32.shape
    rank = q_proj.shape[-1]
    out = np.empty((n_heads, n_q, rank), dtype=np.float32)
    for h in range(n_heads):
        acc = np.zeros((n_q, rank), dtype=np.float32)
        for d in range(head_dim):
            acc = acc + q_f32[h, :, d : d + 1] * q_proj[h, d][None, :].astype(np.float32)
        out[h] = acc * scale[h]
    return out


def sva_scale(logit_scale: np.ndarray) -> np.ndarray:
    return np.clip(np.exp(np.asarray(logit_scale, dtype=np.float32)), np.float32(0.01), np.float32(100.0)).astype(np.float32)


def build_lut(q_low: np.ndarray, codebooks: np.ndarray) -> np.ndarray:
    """lut[h, t, s, c] = q_low[h, t, s-part] . codebook[h, s, c]  (reference sva/ops.py:68)."""
    n_heads, n_q, rank = q_low.shape
    subspaces, codewords, sub = codebooks.shape[1:]
    parts = q_low.reshape(n_heads, n_q, subspaces, 1, sub)
    return seq_dot(parts, codebooks[:, None, :, :, :].astype(np.float32))


def adc_scores(lut: np.ndarray, codes: np.ndarray, rank: int) -> np.ndarray:
    """scores[h, t, l] = (sum over s ascending of lut[h, t, s, codes[h, l, s]]) / sqrt(rank).

    Reference sva/ops.py:64-71: accumulation starts from zeros, one subspace at a time.
    """
    n_heads, n_q, subspaces, _ = lut.shape
    length = codes.shape[1]
    scores = np.zeros((n_heads, n_q, length), dtype=np.float32)
    for h in range(n_heads):
        for s in range(subspaces):
            scores[h] = scores[h] + lut[h, :, s][:, codes[h, :, s]]
    return scores / np.float32(math.sqrt(rank))


@dataclass
class DecodeResult:
    out: np.ndarray            # [H, T, D] float32 (already rounded to the value dtype)
    q_low: np.ndarray          # [H, T, R]
    lut: np.ndarray            # [H, T, S, C]
    shortlist: list            # [H][T] -> int64 array, ascending key index
    final: list                # [H][T] -> int64 array, rank-score desc / index asc
    rank_scores: list          # [H][T] -> float32 array aligned with ``final``
    n_summoned: int
    n_verified: int


def allowed_lengths(key_len: int, n_q: int) -> np.ndarray:
    """Causal allowed length per query when no mask is given (reference sva/llama.py:191-198)."""
    return np.asarray([key_len - n_q + t + 1 for t in range(n_q)], dtype=np.int64)


def verify_one(q_f32: np.ndarray, keys_f32: np.ndarray, values_f32: np.ndarray, idx: np.ndarray,
               scaling: float, dtype: str, logits_mode: int) -> np.ndarray:
    """Exact attention over the selected keys (reference sva/llama.py:304-317 and :532-553).

    logits_mode 0: fp32 logits (static path, million-key benchmark); 1: logits computed in the
    value dtype as the reference scan path does (bf16 products, fp32 accumulation rounded to
    the dtype, then the scale).  Weights and the weighted sum follow the reference: softmax in
    fp32, weights rounded to the dtype, products rounded to the dtype, fp32 sum rounded to the
    dtype.
    """
    head_dim = q_f32.shape[-1]
    if idx.shape[0] == 0:
        return np.zeros(head_dim, dtype=np.float32)
    k_sel = keys_f32[idx]
    v_sel = values_f32[idx]
    if logits_mode == 1 and dtype != "f32":
        prods = round_to(k_sel * q_f32[None, :], dtype)
        logits = round_to(prods.astype(np.float64).sum(axis=-1).astype(np.float32), dtype)
        logits = round_to(logits * np.float32(scaling), dtype)
    else:
        logits = tree_dot(k_sel, q_f32[None, :]) * np.float32(scaling)
    m = logits.max()
    e = np.exp((logits - m).astype(np.float64))
    w = (e / e.sum()).astype(np.float32)
    w = round_to(w, dtype)
    prods = round_to(w[:, None] * v_sel, dtype)
    return round_to(prods.astype(np.float64).sum(axis=0).astype(np.float32), dtype)


def scan_decode(q_f32: np.ndarray, q_proj: np.ndarray, logit_scale: np.ndarray, codebooks: np.ndarray,
                codes: np.ndarray, k_low: np.ndarray, keys_f32: np.ndarray, values_f32: np.ndarray,
                shortlist: int, budget: int, scaling: float, dtype: str = "f32", logits_mode: int = 0,
                allowed_len: np.ndarray | None = None, allowed_mask: np.ndarray | None = None,
                lut_override: np.ndarray | None = None, scale: np.ndarray | None = None) -> DecodeResult:
    """Scan summon -> rank-64 rescore -> exact verify (reference sva/llama.py:171-328).

    q_f32 [H, T, D]; codes [H, L, S]; k_low [H, L, R]; keys/values [Hkv, L, D] (float32 copies
    of the cache values).  allowed_mask [T, L] (bool) overrides allowed_len.
    """
    n_heads, n_q, head_dim = q_f32.shape
    rank = q_proj.shape[-1]
    n_kv = keys_f32.shape[0]
    groups = n_heads // n_kv
    key_len = codes.shape[1]
    ql = query_low(q_f32, q_proj, logit_scale, scale)
    lut = build_lut(ql, codebooks) if lut_override is None else np.asarray(lut_override, dtype=np.float32)
    scores = adc_scores(lut, codes, rank)
    sl_cap = min(shortlist, key_len)
    b_cap = min(budget, sl_cap)
    if allowed_len is None:
        allowed_len = allowed_lengths(key_len, n_q)
    out = np.zeros((n_heads, n_q, head_dim), dtype=np.float32)
    sl_all, fin_all, rs_all = [], [], []
    n_summoned = 0
    n_verified = 0
    for h in range(n_heads):
        sl_h, fin_h, rs_h = [], [], []
        for t in range(n_q):
            if allowed_mask is not None:
                valid = np.asarray(allowed_mask[t], dtype=bool)
            else:
                valid = np.arange(key_len) < allowed_len[t]
            sl = topk_canonical(scores[h, t], sl_cap, valid)
            rank_scores = tree_dot(k_low[h, sl], ql[h, t][None, :]) / np.float32(math.sqrt(rank))
            keep = topk_canonical(rank_scores, b_cap)
            fin = sl[keep]
            n_summoned += sl.shape[0]
            n_verified += fin.shape[0]
            out[h, t] = verify_one(q_f32[h, t], keys_f32[h // groups], values_f32[h // groups], fin,
                                   scaling, dtype, logits_mode)
            sl_h.append(np.sort(sl))
            fin_h.append(fin)
            rs_h.append(rank_scores[keep])
        sl_all.append(sl_h)
        fin_all.append(fin_h)
        rs_all.append(rs_h)
    return DecodeResult(out, ql, lut, sl_all, fin_all, rs_all, n_summoned, n_verified)


def scan_decode_rows(q_f32: np.ndarray, q_proj: np.ndarray, logit_scale: np.ndarray, codebooks: np.ndarray,
                     codes: np.ndarray, k_low_rows, kv_rows, shortlist: int, budget: int, scaling: float,
                     dtype: str = "f32", logits_mode: int = 0, key_len: np.ndarray | None = None) -> DecodeResult:
    """scan_decode for one query token per head on catalogs too large to copy to the host whole.

    The same steps as scan_decode (reference sva/llama.py:171-328), with the rows a step needs
    fetched on demand: ``k_low_rows(h, idx) -> [n, R]`` float32 and ``kv_rows(h, idx) -> (K, V)``
    [n, D] float32 (the query head's KV head rows).  q_f32 [H, D]; codes [H, L, S].  ``key_len``
    [H] (optional) limits head h to keys [0, key_len[h]) (ragged batches).
    """
    n_heads, head_dim = q_f32.shape
    rank = q_proj.shape[-1]
    ql = query_low(q_f32[:, None, :], q_proj, logit_scale)
    lut = build_lut(ql, codebooks)
    out = np.zeros((n_heads, 1, head_dim), dtype=np.float32)
    sl_all, fin_all, rs_all = [], [], []
    n_summoned = n_verified = 0
    for h in range(n_heads):
        length = codes.shape[1] if key_len is None else int(key_len[h])
        scores = adc_scores(lut[h : h + 1], codes[h : h + 1, :length], rank)[0, 0]
        sl_cap = min(shortlist, length)
        sl = topk_canonical(scores, sl_cap)
        rank_scores = tree_dot(k_low_rows(h, sl), ql[h, 0][None, :]) / np.float32(math.sqrt(rank))
        keep = topk_canonical(rank_scores, min(budget, sl_cap))
        fin = sl[keep]
        k_sel, v_sel = kv_rows(h, fin)
        out[h, 0] = verify_one(q_f32[h], k_sel, v_sel, np.arange(fin.shape[0]), scaling, dtype, logits_mode)
        n_summoned += sl.shape[0]
        n_verified += fin.shape[0]
        sl_all.append([np.sort(sl)])
        fin_all.append([fin])
        rs_all.append([rank_scores[keep]])
    return DecodeResult(out, ql, lut, sl_all, fin_all, rs_all, n_summoned, n_verified)


# ----------------------------------------------------------------------------------------
# static inverted index (reference sva/llama.py:83-116, 427-576, 626-657)
# ----------------------------------------------------------------------------------------

def build_postings(codes: np.ndarray, codewords: int):
    """CSR posting lists per (head, subspace): counts [H,S,C], offsets [H,S,C+1], ids [H,S,L].

    Within a cell, key ids are in ascending order (a stable counting sort).  The reference
    (sva/llama.py:626-657) stores the same lists padded to the largest bucket; the order inside
    a bucket does not change any decode result.
    """
    n_heads, length, subspaces = codes.shape
    counts = np.zeros((n_heads, subspaces, codewords), dtype=np.int64)
    offsets = np.zeros((n_heads, subspaces, codewords + 1), dtype=np.int64)
    ids = np.zeros((n_heads, subspaces, length), dtype=np.int64)
    for h in range(n_heads):
        for s in range(subspaces):
            lab = codes[h, :, s].astype(np.int64)
            counts[h, s] = np.bincount(lab, minlength=codewords)
            offsets[h, s, 1:] = np.cumsum(counts[h, s])
            ids[h, s] = np.argsort(lab, kind="stable")
    return counts, offsets, ids


def top_unique_candidates(candidate_idx: np.ndarray, candidate_scores: np.ndarray, candidate_valid: np.ndarray,
                          budget: int, refill_factor: int = 2):
    """Refill-and-dedupe selection (reference sva/llama.py:83-116) under the canonical tie rule.

    Rows are independent.  Entries are ordered by (masked score desc, key idx asc, position asc);
    the first ``refill`` entries form the window; within the window each key keeps its first
    valid entry; the ``min(budget, refill)`` best unique entries are returned in order.
    Returns (selected_idx, selected_scores, selected_valid, refill_count) as lists per row plus
    the refill count; invalid slots carry FINFO_MIN scores.
    """
    rows, width = candidate_idx.shape
    if width == 0 or budget <= 0:
        return [np.zeros(0, np.int64)] * rows, [np.zeros(0, np.float32)] * rows, [np.zeros(0, bool)] * rows, 0
    refill = min(width, max(budget, budget * refill_factor))
    selected_count = min(budget, refill)
    sel_idx, sel_scores, sel_valid = [], [], []
    for r in range(rows):
        idx = candidate_idx[r].astype(np.int64)
        valid = candidate_valid[r].astype(bool)
        masked = np.where(valid, candidate_scores[r].astype(np.float32), FINFO_MIN).astype(np.float32)
        keys = ordered_key(masked)
        pos = np.arange(width)
        order = np.lexsort((pos, idx, ~keys))[:refill]
        w_idx, w_scores, w_valid = idx[order], masked[order], valid[order]
        seen = set()
        uniq = np.zeros(refill, dtype=bool)
        for j in range(refill):
            if w_valid[j] and int(w_idx[j]) not in seen:
                uniq[j] = True
            seen.add(int(w_idx[j]))
        u_scores = np.where(uniq, w_scores, FINFO_MIN).astype(np.float32)
        u_keys = ordered_key(u_scores)
        order2 = np.lexsort((w_idx, ~u_keys))[:selected_count]
        sel_idx.append(w_idx[order2])
        sel_scores.append(u_scores[order2])
        sel_valid.append(uniq[order2])
    return sel_idx, sel_scores, sel_valid, refill


def top_cells(lut: np.ndarray, cells: int, rank: int) -> np.ndarray:
    """Top ``cells`` codewords per subspace by lut/sqrt(rank), codeword asc on ties."""
    code_scores = lut / np.float32(math.sqrt(rank))
    subspaces = lut.shape[0]
    return np.stack([topk_canonical(code_scores[s], cells) for s in range(subspaces)])


def _adaptive_budget(scores_sorted: np.ndarray, rank_count: int, min_budget: int, mid_budget: int, max_budget: int,
                     low: float, high: float, degenerate: int) -> int:
    """Margin rule shared by both inverted variants (reference sva/llama.py:393-400, 508-523)."""
    if rank_count > 1:
        margin_ref = min(min_budget, rank_count) - 1
        margin = np.float32(scores_sorted[0] - scores_sorted[margin_ref])
        if margin >= np.float32(high):
            b = min_budget
        elif margin >= np.float32(low):
            b = mid_budget
        else:
            b = max_budget
        return min(b, rank_count)
    return degenerate


def static_decode(q_f32: np.ndarray, q_proj: np.ndarray, logit_scale: np.ndarray, codebooks: np.ndarray,
                  postings, postings_len: int, k_low: np.ndarray, keys_f32: np.ndarray,
                  values_f32: np.ndarray, budget: int, cells: int, scaling: float, dtype: str = "f32",
                  refill_factor: int = 2, allowed_len: int | None = None,
                  adaptive_min_budget: int | None = None, adaptive_mid_budget: int | None = None,
                  adaptive_low_margin: float = 0.35, adaptive_high_margin: float = 0.70):
    """Static inverted-index decode for one query token (reference sva/llama.py:427-576).

    ``budget`` is the already-clamped budget (min(budget, shortlist, key_len)).  The candidate
    list is laid out as the reference lays it out (subspace-major, cells in top-cell order,
    posting slots padded to the largest bucket, then the tail or the current key) and the
    refill selection is ``top_unique_candidates``.
    Returns (out [H, D], selected idx per head, refill-valid per head (before the budget
    cut), rank scores per head, budget per head, stats).
    """
    counts, offsets, ids = postings
    n_heads = q_f32.shape[0]
    rank = q_proj.shape[-1]
    key_len = k_low.shape[1]
    groups = n_heads // keys_f32.shape[0]
    subspaces, codewords = codebooks.shape[1], codebooks.shape[2]
    if allowed_len is None:
        allowed_len = key_len
    min_budget = min(adaptive_min_budget or budget, budget, key_len)
    mid_budget = min(adaptive_mid_budget or max(min_budget, budget // 2), budget, key_len)
    max_budget = min(budget, key_len)
    cells = min(cells, codewords)
    ql = query_low(q_f32[:, None, :], q_proj, logit_scale)[:, 0]
    lut = build_lut(ql[:, None, :], codebooks)[:, 0]
    max_bucket = max(1, int(counts.max()))
    tail_start = min(max(postings_len, 0), key_len)
    outs = np.zeros(q_f32.shape, dtype=np.float32)
    sel_all, valid_all, score_all, budget_all = [], [], [], []
    summoned = verified = refill_total = 0
    for h in range(n_heads):
        tc = top_cells(lut[h], cells, rank)
        cand, cvalid = [], []
        for s in range(subspaces):
            for c in tc[s]:
                n = int(counts[h, s, c])
                lst = np.zeros(max_bucket, dtype=np.int64)
                lst[:n] = ids[h, s, offsets[h, s, c] : offsets[h, s, c] + n]
                cand.append(lst)
                cvalid.append((np.arange(max_bucket) < n) & (lst < allowed_len))
        if tail_start < key_len:
            tail = np.arange(tail_start, key_len, dtype=np.int64)
        else:
            tail = np.asarray([key_len - 1], dtype=np.int64)
        cand.append(tail)
        cvalid.append(tail < allowed_len)
        cand = np.concatenate(cand)
        cvalid = np.concatenate(cvalid)
        summoned += int(cvalid.sum())
        cscores = tree_dot(k_low[h, cand], ql[h][None, :]) / np.float32(math.sqrt(rank))
        si, ss, sv, refill = top_unique_candidates(cand[None, :], cscores[None, :], cvalid[None, :], max_budget,
                                                   refill_factor)
        s_idx, s_scores, s_valid = si[0], ss[0], sv[0]
        refill_total += refill
        rank_count = s_idx.shape[0]
        b_h = _adaptive_budget(s_scores, rank_count, min_budget, mid_budget, max_budget,
                               adaptive_low_margin, adaptive_high_margin, 1)
        use = s_valid & (np.arange(rank_count) < b_h)
        verified += int(use.sum())
        outs[h] = verify_one(q_f32[h], keys_f32[h // groups], values_f32[h // groups], s_idx[use], scaling,
                             dtype, 0)
        sel_all.append(s_idx)
        valid_all.append(s_valid)
        score_all.append(s_scores)
        budget_all.append(b_h)
    stats = {"summoned": summoned, "refill_pool": refill_total, "exact_scored": verified, "verified": verified,
             "queries": n_heads, "cell_visits": n_heads * subspaces * cells}
    return outs, sel_all, valid_all, score_all, budget_all, stats


def dynamic_inverted_decode(q_f32: np.ndarray, q_proj: np.ndarray, logit_scale: np.ndarray, codebooks: np.ndarray,
                            postings, k_low: np.ndarray, keys_f32: np.ndarray, values_f32: np.ndarray, budget: int,
                            cells: int, scaling: float, dtype: str = "f32", allowed_len: int | None = None,
                            adaptive_min_budget: int | None = None, adaptive_mid_budget: int | None = None,
                            adaptive_low_margin: float = 0.35, adaptive_high_margin: float = 0.70):
    """Dynamic inverted decode for one query token (reference sva/llama.py:330-425).

    Candidates are the unique allowed keys of the top cells plus the current key; all of them
    are ranked (no refill window).  Postings must cover every key.
    """
    counts, offsets, ids = postings
    n_heads = q_f32.shape[0]
    rank = q_proj.shape[-1]
    key_len = k_low.shape[1]
    groups = n_heads // keys_f32.shape[0]
    subspaces, codewords = codebooks.shape[1], codebooks.shape[2]
    if allowed_len is None:
        allowed_len = key_len
    min_budget = min(adaptive_min_budget or budget, budget, key_len)
    mid_budget = min(adaptive_mid_budget or max(min_budget, budget // 2), budget, key_len)
    max_budget = min(budget, key_len)
    cells = min(cells, codewords)
    ql = query_low(q_f32[:, None, :], q_proj, logit_scale)[:, 0]
    lut = build_lut(ql[:, None, :], codebooks)[:, 0]
    outs = np.zeros(q_f32.shape, dtype=np.float32)
    sel_all = []
    summoned = verified = 0
    for h in range(n_heads):
        tc = top_cells(lut[h], cells, rank)
        cand = [ids[h, s, offsets[h, s, c] : offsets[h, s, c] + counts[h, s, c]] for s in range(subspaces) for c in tc[s]]
        cand = np.concatenate(cand + [np.zeros(0, np.int64)])
        cand = cand[cand < allowed_len]
        if key_len - 1 < allowed_len:
            cand = np.concatenate([cand, [key_len - 1]])
        cand = np.unique(cand)
        if cand.shape[0] == 0:
            cand = np.asarray([min(allowed_len, key_len) - 1], dtype=np.int64)
        cscores = tree_dot(k_low[h, cand], ql[h][None, :]) / np.float32(math.sqrt(rank))
        rank_count = min(max_budget, cand.shape[0])
        order = topk_canonical(cscores, rank_count)
        b_h = _adaptive_budget(cscores[order], rank_count, min_budget, mid_budget, max_budget,
                               adaptive_low_margin, adaptive_high_margin, min(min_budget, rank_count))
        fin = cand[order[:b_h]]
        outs[h] = verify_one(q_f32[h], keys_f32[h // groups], values_f32[h // groups], fin, scaling, dtype, 0)
        summoned += cand.shape[0]
        verified += b_h
        sel_all.append(fin)
    stats = {"summoned": summoned, "exact_scored": verified, "verified": verified, "queries": n_heads,
             "cell_visits": n_heads * subspaces * cells}
    return outs, sel_all, stats
