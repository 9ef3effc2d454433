"""Torch-facing wrappers of the C ABI (CUDA tensors only; no CPU fallback).

Each function checks devices, dtypes and layouts, passes raw device pointers and element
strides to libsva_b200.so on the current CUDA stream, and maps error codes to exceptions.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError as exc:
        raise TypeError(f"sva_b200 supports float32, bfloat16 and float16 tensors, got {dtype}") from exc


def _cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise RuntimeError(f"sva_b200 runs on CUDA devices only; {name} is on {t.device}")
    return t


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_host_ok: dict[int, bool] = {}


def _cuda_or_host(t: torch.Tensor, name: str) -> None:
    """A CUDA tensor, or a page-locked host tensor that device code can address (checked once
    per allocation through sva_host_buffer_device_accessible)."""
    if t.is_cuda:
        return
    if t.device.type == "cpu" and t.is_pinned():
        base = t.untyped_storage().data_ptr()
        ok = _host_ok.get(base)
        if ok is None:
            ok = bool(_lib.load().sva_host_buffer_device_accessible(ctypes.c_void_p(base)))
            _host_ok[base] = ok
        if ok:
            return
    raise ValueError(f"{name} must be a CUDA tensor or a pinned host tensor that the GPU can address")


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class Workspace:
    """Grow-only device scratch buffer reused across calls (one per device and purpose)."""

    def __init__(self) -> None:
        self._buf: dict[torch.device, torch.Tensor] = {}

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        buf = self._buf.get(device)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._buf[device] = buf
        return buf


_decode_ws = Workspace()


def tensor_core_write_ok(keys: torch.Tensor, k_proj: torch.Tensor) -> bool:
    """Whether the tcgen05 write path applies: bf16 keys with 16-byte aligned rows, head_dim a
    multiple of 16 up to 128, rank a multiple of 16 up to 64, and a key projection whose values
    are bf16 numbers (so rounding it to bf16 changes nothing)."""
    head_dim, rank = int(keys.shape[-1]), int(k_proj.shape[-1])
    if keys.dtype != torch.bfloat16 or head_dim % 16 or head_dim > 128 or rank % 16 or rank > 64:
        return False
    if keys.data_ptr() % 16 or (keys.stride(-2) * 2) % 16 or (keys.stride(0) * 2) % 16:
        return False
    return bool(torch.equal(k_proj, k_proj.to(torch.bfloat16).to(k_proj.dtype)))


def catalog_encode(keys: torch.Tensor, k_proj: torch.Tensor, codebooks: torch.Tensor, start: int, count: int,
                   k_low: torch.Tensor | None, codes: torch.Tensor | None, n_heads: int | None = None,
                   tensor_cores: bool = False, status: torch.Tensor | None = None) -> None:
    """Write k_low / codes rows [start, start+count) of every query head.

    keys [Hkv, L, D] (rows contiguous), k_proj [H, D, R] fp32, codebooks [H, S, C, R/S] fp32,
    k_low [H, cap, R] fp32 (contiguous rows), codes [H, cap, S] uint8.  ``tensor_cores`` selects
    the tcgen05 projection (sva_catalog_encode_tc; see ``tensor_core_write_ok``) instead of the
    exact sequential-order CUDA-core projection; ``status`` (int32 device scalar) receives its
    timeout flag.
    """
    _cuda(keys, "keys")
    if keys.stride(-1) != 1:
        raise ValueError("keys rows must be contiguous")
    n_heads = int(k_proj.shape[0]) if n_heads is None else n_heads
    n_kv, _, head_dim = keys.shape
    rank = int(k_proj.shape[-1])
    subspaces, codewords = int(codebooks.shape[1]), int(codebooks.shape[2])
    k_proj = k_proj.contiguous()
    codebooks = codebooks.contiguous()
    for name, t in (("k_low", k_low), ("codes", codes)):
        if t is not None:
            _cuda(t, name)
            if not (t.stride(-1) == 1 and t.stride(-2) == t.shape[-1]):
                raise ValueError(f"{name} rows must be contiguous")
    lib = _lib.load()
    common = (keys.data_ptr(), dtype_code(keys.dtype), keys.stride(0), keys.stride(1), n_heads, n_kv, head_dim, rank,
              k_proj.data_ptr(), codebooks.data_ptr(), subspaces, codewords, int(start), int(count), _ptr(k_low),
              0 if k_low is None else k_low.stride(0), _ptr(codes), 0 if codes is None else codes.stride(0))
    if tensor_cores:
        rc = lib.sva_catalog_encode_tc(*common, _ptr(status), _stream(keys.device))
    else:
        rc = lib.sva_catalog_encode(*common, _stream(keys.device))
    _lib.check(rc)


def catalog_encode_at(keys: torch.Tensor, k_proj: torch.Tensor, codebooks: torch.Tensor, start: torch.Tensor,
                      count: int, limit: int, k_low: torch.Tensor, codes: torch.Tensor,
                      n_heads: int | None = None) -> None:
    """catalog_encode of rows [start, start + count) with ``start`` an int64 device scalar read by
    the kernel (sva_catalog_encode_at): capturable in a CUDA graph whose replays append at a moving
    position.  Rows at or beyond ``limit`` are skipped."""
    _cuda(keys, "keys")
    _cuda(start, "start")
    if start.dtype != torch.int64:
        raise TypeError("start must be an int64 tensor")
    if keys.stride(-1) != 1:
        raise ValueError("keys rows must be contiguous")
    n_heads = int(k_proj.shape[0]) if n_heads is None else n_heads
    n_kv, _, head_dim = keys.shape
    for name, t in (("k_low", k_low), ("codes", codes)):
        _cuda(t, name)
        if not (t.stride(-1) == 1 and t.stride(-2) == t.shape[-1]):
            raise ValueError(f"{name} rows must be contiguous")
    rc = _lib.load().sva_catalog_encode_at(
        keys.data_ptr(), dtype_code(keys.dtype), keys.stride(0), keys.stride(1), n_heads, n_kv, head_dim,
        int(k_proj.shape[-1]), k_proj.data_ptr(), codebooks.data_ptr(), int(codebooks.shape[1]),
        int(codebooks.shape[2]), start.data_ptr(), int(count), int(limit), k_low.data_ptr(), k_low.stride(0),
        codes.data_ptr(), codes.stride(0), _stream(keys.device))
    _lib.check(rc)


def assign_centroids(x: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    _cuda(x, "x")
    x = x.float()
    if x.stride(-1) != 1:
        x = x.contiguous()
    cent = centroids.float().contiguous()
    labels = torch.empty(x.shape[0], dtype=torch.int64, device=x.device)
    rc = _lib.load().sva_assign_centroids(x.data_ptr(), x.shape[0], x.shape[1], x.stride(0), cent.data_ptr(),
                                          cent.shape[0], labels.data_ptr(), _stream(x.device))
    _lib.check(rc)
    return labels


def pq_scores(q_low: torch.Tensor, codebooks: torch.Tensor, codes_u8: torch.Tensor, rank_dim: int) -> torch.Tensor:
    _cuda(q_low, "q_low")
    q_low = q_low.float().contiguous()
    codebooks = codebooks.float().contiguous()
    codes_u8 = codes_u8.contiguous()
    n_heads, n_q, _ = q_low.shape
    key_len = int(codes_u8.shape[1])
    out = torch.empty(n_heads, n_q, key_len, dtype=torch.float32, device=q_low.device)
    rc = _lib.load().sva_pq_scores(q_low.data_ptr(), n_heads, n_q, rank_dim, codebooks.data_ptr(),
                                   codebooks.shape[1], codebooks.shape[2], codes_u8.data_ptr(), key_len,
                                   out.data_ptr(), _stream(q_low.device))
    _lib.check(rc)
    return out


def decode_args(q: torch.Tensor, q_proj: torch.Tensor, scale: torch.Tensor, codebooks: torch.Tensor,
                codes: torch.Tensor, k_low: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, shortlist: int,
                budget: int, softmax_scale: float | None = None, logits_mode: int = 0,
                allowed_len: torch.Tensor | None = None, allowed_mask: torch.Tensor | None = None,
                lut_override: torch.Tensor | None = None, out: torch.Tensor | None = None,
                stats: torch.Tensor | None = None) -> tuple[_lib.DecodeArgs, torch.Tensor]:
    """Validated sva_decode_args for the tensors of a decode call, and the output tensor."""
    for name, t in (("codes", codes), ("k_low", k_low), ("keys", keys), ("values", values)):
        _cuda(t, name)
    dev = codes.device
    _cuda_or_host(q, "q")
    if out is not None:
        _cuda_or_host(out, "out")
    n_heads, n_q, head_dim = q.shape
    n_kv = int(keys.shape[0])
    key_len = int(codes.shape[1])
    rank = int(q_proj.shape[-1])
    if q.stride(-1) != 1 or keys.stride(-1) != 1 or values.stride(-1) != 1:
        raise ValueError("q, keys and values must have contiguous rows")
    if codes.dtype != torch.uint8 or codes.stride(-1) != 1 or codes.stride(-2) != codes.shape[-1]:
        raise ValueError("codes must be uint8 with contiguous [L, S] rows per head")
    if k_low.dtype != torch.float32 or k_low.stride(-1) != 1 or k_low.stride(-2) != rank:
        raise ValueError("k_low must be float32 with contiguous [L, R] rows per head")
    if keys.dtype != q.dtype or values.dtype != q.dtype:
        raise TypeError("q, keys and values must share a dtype")
    if out is None:
        out = torch.empty(n_heads, n_q, head_dim, dtype=q.dtype, device=dev)
    a = _lib.DecodeArgs()
    a.n_heads, a.n_kv_heads, a.n_queries, a.head_dim = n_heads, n_kv, n_q, head_dim
    a.rank_dim, a.subspaces, a.codewords = rank, int(codebooks.shape[1]), int(codebooks.shape[2])
    a.shortlist, a.budget = int(shortlist), int(budget)
    a.qkv_dtype = dtype_code(q.dtype)
    a.logits_mode = int(logits_mode)
    a.softmax_scale = float(head_dim ** -0.5 if softmax_scale is None else softmax_scale)
    a.key_len = key_len
    a.query, a.q_head_stride, a.q_row_stride = q.data_ptr(), q.stride(0), q.stride(1)
    a.q_proj = q_proj.data_ptr()
    a.scale = scale.data_ptr()
    a.codebooks = codebooks.data_ptr()
    a.lut_override = _ptr(lut_override)
    a.codes, a.codes_head_stride = codes.data_ptr(), codes.stride(0)
    a.k_low, a.k_low_head_stride = k_low.data_ptr(), k_low.stride(0)
    a.keys, a.k_head_stride, a.k_row_stride = keys.data_ptr(), keys.stride(0), keys.stride(1)
    a.values, a.v_head_stride, a.v_row_stride = values.data_ptr(), values.stride(0), values.stride(1)
    a.allowed_len = _ptr(allowed_len)
    a.allowed_mask = _ptr(allowed_mask)
    a.mask_row_stride = 0 if allowed_mask is None else allowed_mask.stride(0)
    a.out, a.out_head_stride, a.out_row_stride = out.data_ptr(), out.stride(0), out.stride(1)
    a.stats = _ptr(stats)
    return a, out


def decode(q: torch.Tensor, q_proj: torch.Tensor, scale: torch.Tensor, codebooks: torch.Tensor, codes: torch.Tensor,
           k_low: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, shortlist: int, budget: int,
           softmax_scale: float | None = None, logits_mode: int = 0, allowed_len: torch.Tensor | None = None,
           allowed_mask: torch.Tensor | None = None, lut_override: torch.Tensor | None = None,
           out: torch.Tensor | None = None, want_shortlist: bool = False, want_final: bool = False,
           stats: torch.Tensor | None = None):
    """Scan summon -> rescore -> verify for H heads x T tokens (see include/sva_b200.h).

    q [H, T, D]; codes [H, L, S] uint8 (rows contiguous); k_low [H, L, R] fp32 (rows
    contiguous); keys/values [Hkv, L, D].  Returns out [H, T, D] (and the shortlist / final
    index tensors when requested, [H, T, shortlist] / [H, T, budget] int32, ascending, -1 padded).
    q and out may be pinned host tensors: the kernels then read q from and write out to host
    memory directly, so a host caller needs no separate copies for them.  A new output is
    allocated on the device of the catalog.
    """
    a, out = decode_args(q, q_proj, scale, codebooks, codes, k_low, keys, values, shortlist, budget, softmax_scale,
                         logits_mode, allowed_len, allowed_mask, lut_override, out, stats)
    dev = codes.device
    n_heads, n_q, _ = q.shape
    sl_out = fin_out = None
    if want_shortlist:
        sl_out = torch.empty(n_heads, n_q, int(shortlist), dtype=torch.int32, device=dev)
        a.shortlist_out = sl_out.data_ptr()
    if want_final:
        fin_out = torch.empty(n_heads, n_q, int(budget), dtype=torch.int32, device=dev)
        a.final_out = fin_out.data_ptr()
    lib = _lib.load()
    ws_bytes = int(lib.sva_decode_workspace_size(ctypes.byref(a)))
    ws = _decode_ws.get(dev, ws_bytes)
    rc = lib.sva_decode(ctypes.byref(a), _ptr(ws), ws_bytes, _stream(dev))
    _lib.check(rc)
    if want_shortlist or want_final:
        return out, sl_out, fin_out
    return out


def batched_args(q: torch.Tensor, q_proj: torch.Tensor, scale: torch.Tensor, codebooks: torch.Tensor,
                 codes: torch.Tensor, k_low: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, shortlist: int,
                 budget: int, *, seq_lens: torch.Tensor | None = None, page_table: torch.Tensor | None = None,
                 max_len: int | None = None, softmax_scale: float | None = None, logits_mode: int = 0,
                 allowed_len: torch.Tensor | None = None, allowed_mask: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, stats: torch.Tensor | None = None):
    """Validated (sva_decode_args, sva_batch_layout, out) for the tensors of a batched call (see
    decode_batched for the layouts)."""
    for name, t in (("codes", codes), ("k_low", k_low), ("keys", keys), ("values", values)):
        _cuda(t, name)
    _cuda_or_host(q, "q")
    if out is not None:
        _cuda_or_host(out, "out")
    if q.dim() != 4 or codes.dim() != 4 or k_low.dim() != 4 or keys.dim() != 4 or values.dim() != 4:
        raise ValueError("decode_batched takes 4-d q, codes, k_low, keys and values")
    dev = codes.device
    n_seqs, n_heads, n_q, head_dim = q.shape
    n_kv = int(keys.shape[1])
    rank = int(q_proj.shape[-1])
    if q.stride(-1) != 1 or keys.stride(-1) != 1 or values.stride(-1) != 1:
        raise ValueError("q, keys and values must have contiguous rows")
    if codes.dtype != torch.uint8 or codes.stride(-1) != 1 or codes.stride(-2) != codes.shape[-1]:
        raise ValueError("codes must be uint8 with contiguous rows")
    if k_low.dtype != torch.float32 or k_low.stride(-1) != 1 or k_low.stride(-2) != rank:
        raise ValueError("k_low must be float32 with contiguous rows")
    if keys.dtype != q.dtype or values.dtype != q.dtype:
        raise TypeError("q, keys and values must share a dtype")
    paged = page_table is not None
    if paged:
        _cuda(page_table, "page_table")
        if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.stride(-1) != 1:
            raise ValueError("page_table must be an int32 [B, max_pages] tensor with contiguous rows")
        page_keys = int(codes.shape[2])
        if max_len is None:
            max_len = int(page_table.shape[1]) * page_keys
    else:
        page_keys = 0
        if max_len is None:
            max_len = int(codes.shape[2])
    if seq_lens is not None:
        _cuda(seq_lens, "seq_lens")
        if seq_lens.dtype != torch.int64 or seq_lens.numel() != n_seqs:
            raise ValueError("seq_lens must be an int64 tensor of B entries")
    if out is None:
        out = torch.empty(n_seqs, n_heads, n_q, head_dim, dtype=q.dtype, device=dev)
    a = _lib.DecodeArgs()
    a.n_heads, a.n_kv_heads, a.n_queries, a.head_dim = n_heads, n_kv, n_q, head_dim
    a.rank_dim, a.subspaces, a.codewords = rank, int(codebooks.shape[1]), int(codebooks.shape[2])
    a.shortlist, a.budget = int(shortlist), int(budget)
    a.qkv_dtype = dtype_code(q.dtype)
    a.logits_mode = int(logits_mode)
    a.softmax_scale = float(head_dim ** -0.5 if softmax_scale is None else softmax_scale)
    a.key_len = int(max_len)
    a.query, a.q_head_stride, a.q_row_stride = q.data_ptr(), q.stride(1), q.stride(2)
    a.q_proj, a.scale, a.codebooks = q_proj.data_ptr(), scale.data_ptr(), codebooks.data_ptr()
    a.codes, a.codes_head_stride = codes.data_ptr(), codes.stride(1)
    a.k_low, a.k_low_head_stride = k_low.data_ptr(), k_low.stride(1)
    a.keys, a.k_head_stride, a.k_row_stride = keys.data_ptr(), keys.stride(1), keys.stride(2)
    a.values, a.v_head_stride, a.v_row_stride = values.data_ptr(), values.stride(1), values.stride(2)
    a.allowed_len = _ptr(allowed_len)
    a.allowed_mask = _ptr(allowed_mask)
    a.mask_row_stride = 0 if allowed_mask is None else allowed_mask.stride(0)
    a.out, a.out_head_stride, a.out_row_stride = out.data_ptr(), out.stride(1), out.stride(2)
    a.stats = _ptr(stats)
    lay = _lib.BatchLayout()
    lay.n_seqs, lay.page_keys = n_seqs, page_keys
    lay.seq_lens = _ptr(seq_lens)
    lay.page_table = _ptr(page_table)
    lay.page_table_stride = 0 if page_table is None else page_table.stride(0)
    lay.q_seq_stride, lay.out_seq_stride = q.stride(0), out.stride(0)
    lay.codes_page_stride, lay.k_low_page_stride = codes.stride(0), k_low.stride(0)
    lay.k_page_stride, lay.v_page_stride = keys.stride(0), values.stride(0)
    return a, lay, out


def decode_batched(q: torch.Tensor, q_proj: torch.Tensor, scale: torch.Tensor, codebooks: torch.Tensor,
                   codes: torch.Tensor, k_low: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, shortlist: int,
                   budget: int, *, seq_lens: torch.Tensor | None = None, page_table: torch.Tensor | None = None,
                   max_len: int | None = None, softmax_scale: float | None = None, logits_mode: int = 0,
                   allowed_len: torch.Tensor | None = None, allowed_mask: torch.Tensor | None = None,
                   out: torch.Tensor | None = None, want_shortlist: bool = False, want_final: bool = False,
                   stats: torch.Tensor | None = None):
    """Scan decode of B sequences in one call (sva_decode_batched, see include/sva_b200.h).

    q [B, H, T, D]; q_proj / scale / codebooks are shared by the sequences (one layer).
    Unpaged (``page_table`` None): codes [B, H, L, S], k_low [B, H, L, R], keys / values
    [B, Hkv, L, D], with L the longest sequence.  Paged: codes [pages, H, page_keys, S], k_low
    [pages, H, page_keys, R], keys / values [pages, Hkv, page_keys, D] page pools and page_table
    [B, max_pages] int32 (page of every page_keys-key block of each sequence).  ``seq_lens`` [B]
    int64 (device) gives each sequence's keys (None: all L, or all ``max_len``); ``max_len`` (host
    int) bounds them (default: L, or max_pages * page_keys).  ``allowed_len`` [B, T] int64 and
    ``allowed_mask`` [B * T, >= L] uint8 as for ``decode``.  Returns out [B, H, T, D] (and
    shortlist / final index tensors [B, H, T, shortlist] / [B, H, T, budget] when requested).
    As for ``decode``, q and out may be page-locked host tensors that the GPU can address.
    """
    a, lay, out = batched_args(q, q_proj, scale, codebooks, codes, k_low, keys, values, shortlist, budget,
                               seq_lens=seq_lens, page_table=page_table, max_len=max_len,
                               softmax_scale=softmax_scale, logits_mode=logits_mode, allowed_len=allowed_len,
                               allowed_mask=allowed_mask, out=out, stats=stats)
    dev = codes.device
    n_seqs, n_heads, n_q, _ = q.shape
    sl_out = fin_out = None
    if want_shortlist:
        sl_out = torch.empty(n_seqs, n_heads, n_q, int(shortlist), dtype=torch.int32, device=dev)
        a.shortlist_out = sl_out.data_ptr()
    if want_final:
        fin_out = torch.empty(n_seqs, n_heads, n_q, int(budget), dtype=torch.int32, device=dev)
        a.final_out = fin_out.data_ptr()
    lib = _lib.load()
    ws_bytes = int(lib.sva_decode_batched_workspace_size(ctypes.byref(a), ctypes.byref(lay)))
    ws = _decode_ws.get(dev, ws_bytes)
    rc = lib.sva_decode_batched(ctypes.byref(a), ctypes.byref(lay), _ptr(ws), ws_bytes, _stream(dev))
    _lib.check(rc)
    if want_shortlist or want_final:
        return out, sl_out, fin_out
    return out


def sva_scale(logit_scale: torch.Tensor) -> torch.Tensor:
    """clamp(exp(logit_scale), 0.01, 100) computed as the reference does (sva/llama.py:69-73)."""
    return logit_scale.detach().float().exp().clamp(0.01, 100.0)


def sqrt_rank(rank_dim: int) -> float:
    return math.sqrt(rank_dim)


_post_ws = Workspace()
_inv_ws = Workspace()


class Postings:
    """Device posting lists of one catalog: CSR (sva_postings_build) or, with ``cap``, the padded
    layout of sva_postings_append (cell c of every (head, subspace) owns ``cap`` id slots)."""

    def __init__(self, counts, offsets, ids, max_bucket, key_len: int, cap: int | None = None):
        self.counts, self.offsets, self.ids, self.max_bucket = counts, offsets, ids, max_bucket
        self.key_len = int(key_len)
        self.cap = cap
        self.overflow = None


def postings_build(codes: torch.Tensor, codewords: int, key_len: int | None = None) -> Postings:
    """Posting lists of keys [0, key_len) of codes [H, L, S] uint8 (reference sva/llama.py:626-657)."""
    _cuda(codes, "codes")
    if codes.dtype != torch.uint8 or codes.stride(-1) != 1 or codes.stride(-2) != codes.shape[-1]:
        raise ValueError("codes must be uint8 with contiguous [L, S] rows per head")
    n_heads, cap, subspaces = codes.shape
    key_len = cap if key_len is None else int(key_len)
    dev = codes.device
    counts = torch.empty(n_heads, subspaces, codewords, dtype=torch.int32, device=dev)
    offsets = torch.empty(n_heads, subspaces, codewords + 1, dtype=torch.int32, device=dev)
    ids = torch.empty(n_heads, subspaces, max(key_len, 1), dtype=torch.int32, device=dev)
    max_bucket = torch.empty(1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws_bytes = int(lib.sva_postings_workspace_size(n_heads, subspaces, codewords, key_len))
    ws = _post_ws.get(dev, ws_bytes)
    rc = lib.sva_postings_build(codes.data_ptr(), codes.stride(0), n_heads, subspaces, codewords, key_len,
                                counts.data_ptr(), offsets.data_ptr(), ids.data_ptr(), ids.shape[-1],
                                max_bucket.data_ptr(), _ptr(ws), ws_bytes, _stream(dev))
    _lib.check(rc)
    return Postings(counts, offsets, ids, max_bucket, key_len)


def postings_padded(codes: torch.Tensor, codewords: int, key_len: int, cap: int | None = None) -> Postings:
    """Posting lists of keys [0, key_len) in the padded layout with ``cap`` slots per cell (at least
    the largest list; None: twice the largest list, at least 64 more): the CSR build, then each
    list moved to its cell's slots.  Reads the largest list size on the host."""
    csr = postings_build(codes, codewords, key_len=key_len)
    largest = int(csr.max_bucket.item())
    if cap is None:
        cap = max(2 * largest, largest + 64)
    if largest > cap:
        raise ValueError(f"postings_padded: the largest list has {largest} keys, more than cap={cap}")
    n_heads, subspaces, _ = csr.counts.shape
    dev = codes.device
    offsets = (torch.arange(codewords + 1, device=dev, dtype=torch.int32) * cap).expand(n_heads, subspaces, -1)
    offsets = offsets.contiguous()
    ids = torch.zeros(n_heads, subspaces, codewords * cap, dtype=torch.int32, device=dev)
    if key_len > 0:
        pos = torch.arange(key_len, device=dev, dtype=torch.int32).expand(n_heads, subspaces, -1).contiguous()
        # cell of every CSR position, and its slot inside the cell
        cell = torch.searchsorted(csr.offsets[..., 1:].contiguous(), pos, right=True)
        slot = pos - torch.gather(csr.offsets, 2, cell)
        ids.scatter_(2, (cell * cap + slot).to(torch.int64), csr.ids[..., :key_len])
    out = Postings(csr.counts, offsets, ids, csr.max_bucket, key_len, cap=int(cap))
    out.overflow = torch.zeros(1, dtype=torch.int32, device=dev)
    out.largest_at_build = largest
    return out


def postings_append(codes: torch.Tensor, postings: Postings, start: int, count: int) -> None:
    """Appends keys [start, start + count) of codes [H, L, S] to padded posting lists in place
    (sva_postings_append; reference sva/llama.py:659-693)."""
    if postings.cap is None:
        raise ValueError("postings_append needs the padded layout (postings_padded)")
    n_heads, _, subspaces = codes.shape
    codewords = int(postings.counts.shape[-1])
    rc = _lib.load().sva_postings_append(codes.data_ptr(), codes.stride(0), n_heads, subspaces, codewords, int(start),
                                         int(count), postings.counts.data_ptr(), postings.offsets.data_ptr(),
                                         postings.ids.data_ptr(), postings.ids.shape[-1],
                                         postings.max_bucket.data_ptr(), postings.overflow.data_ptr(),
                                         _stream(codes.device))
    _lib.check(rc)
    postings.key_len = int(start + count)


def inverted_args(q: torch.Tensor, q_proj: torch.Tensor, scale: torch.Tensor, codebooks: torch.Tensor,
                  codes: torch.Tensor, postings: Postings, k_low: torch.Tensor, keys: torch.Tensor,
                  values: torch.Tensor, budget: int, cells: int, min_budget: int, mid_budget: int,
                  low_margin: float = 0.35, high_margin: float = 0.70, dynamic: bool = False, refill_factor: int = 2,
                  allowed_len: int | None = None, allowed_mask: torch.Tensor | None = None,
                  softmax_scale: float | None = None, out: torch.Tensor | None = None,
                  stats: torch.Tensor | None = None, max_bucket: torch.Tensor | None = None):
    """Validated (sva_inverted_args, out) for decode_inverted's tensors; ``max_bucket`` (device int32)
    overrides the postings' own largest bucket (the shards pass the global one)."""
    for name, t in (("q", q), ("codes", codes), ("k_low", k_low), ("keys", keys), ("values", values)):
        _cuda(t, name)
    dev = q.device
    n_heads, head_dim = q.shape
    key_len = int(k_low.shape[1])
    if out is None:
        out = torch.empty(n_heads, head_dim, dtype=q.dtype, device=dev)
    a = _lib.InvertedArgs()
    a.n_heads, a.n_kv_heads, a.head_dim = n_heads, int(keys.shape[0]), head_dim
    a.rank_dim, a.subspaces, a.codewords = int(q_proj.shape[-1]), int(codebooks.shape[1]), int(codebooks.shape[2])
    a.budget, a.cells, a.refill_factor, a.dynamic = int(budget), int(cells), int(refill_factor), int(bool(dynamic))
    a.min_budget, a.mid_budget = int(min_budget), int(mid_budget)
    a.qkv_dtype = dtype_code(q.dtype)
    a.low_margin, a.high_margin = float(low_margin), float(high_margin)
    a.softmax_scale = float(head_dim ** -0.5 if softmax_scale is None else softmax_scale)
    a.key_len = key_len
    a.postings_len = postings.key_len
    a.allowed_len = key_len if allowed_len is None else int(allowed_len)
    a.allowed_mask = _ptr(allowed_mask)
    a.query, a.q_head_stride = q.data_ptr(), q.stride(0)
    a.q_proj, a.scale, a.codebooks = q_proj.data_ptr(), scale.data_ptr(), codebooks.data_ptr()
    a.codes, a.codes_head_stride = codes.data_ptr(), codes.stride(0)
    a.post_counts, a.post_offsets = postings.counts.data_ptr(), postings.offsets.data_ptr()
    a.post_ids, a.post_ids_sub_stride = postings.ids.data_ptr(), postings.ids.shape[-1]
    a.max_bucket = (postings.max_bucket if max_bucket is None else max_bucket).data_ptr()
    a.k_low, a.k_low_head_stride = k_low.data_ptr(), k_low.stride(0)
    a.keys, a.k_head_stride, a.k_row_stride = keys.data_ptr(), keys.stride(0), keys.stride(1)
    a.values, a.v_head_stride, a.v_row_stride = values.data_ptr(), values.stride(0), values.stride(1)
    a.out, a.out_head_stride = out.data_ptr(), out.stride(0)
    a.stats = _ptr(stats)
    return a, out


def decode_inverted(q: torch.Tensor, q_proj: torch.Tensor, scale: torch.Tensor, codebooks: torch.Tensor,
                    codes: torch.Tensor, postings: Postings, k_low: torch.Tensor, keys: torch.Tensor,
                    values: torch.Tensor, budget: int, cells: int, min_budget: int, mid_budget: int,
                    low_margin: float = 0.35, high_margin: float = 0.70, dynamic: bool = False,
                    refill_factor: int = 2, allowed_len: int | None = None, allowed_mask: torch.Tensor | None = None,
                    softmax_scale: float | None = None,
                    out: torch.Tensor | None = None, want_selection: bool = False, stats: torch.Tensor | None = None):
    """Inverted-index decode of one token per head (reference sva/llama.py:427-576 / :330-425).

    q [H, D]; codes [H, >=postings_len, S]; k_low [H, L, R]; keys/values [Hkv, L, D].  ``budget``,
    ``min_budget`` and ``mid_budget`` are already clamped as the reference clamps them.
    """
    a, out = inverted_args(q, q_proj, scale, codebooks, codes, postings, k_low, keys, values, budget, cells,
                           min_budget, mid_budget, low_margin, high_margin, dynamic, refill_factor, allowed_len,
                           allowed_mask, softmax_scale, out, stats)
    dev = q.device
    n_heads = q.shape[0]
    sel = None
    if want_selection:
        sel = (torch.empty(n_heads, int(budget), dtype=torch.int32, device=dev),
               torch.empty(n_heads, int(budget), dtype=torch.uint8, device=dev),
               torch.empty(n_heads, int(budget), dtype=torch.float32, device=dev),
               torch.empty(n_heads, dtype=torch.int32, device=dev))
        a.sel_idx_out, a.sel_valid_out, a.sel_score_out, a.budget_out = (t.data_ptr() for t in sel)
    lib = _lib.load()
    ws_bytes = int(lib.sva_inverted_workspace_size(ctypes.byref(a)))
    if ws_bytes == 0:
        raise ValueError("sva_b200: invalid inverted decode arguments")
    ws = _inv_ws.get(dev, ws_bytes)
    rc = lib.sva_decode_inverted(ctypes.byref(a), _ptr(ws), ws_bytes, _stream(dev))
    _lib.check(rc)
    return (out, *sel) if want_selection else out


def top_unique(candidate_idx: torch.Tensor, candidate_scores: torch.Tensor, candidate_valid: torch.Tensor,
               budget: int, refill_factor: int = 2):
    """Refill-and-dedupe selection on explicit rows (reference sva/llama.py:83-116)."""
    for name, t in (("candidate_idx", candidate_idx), ("candidate_scores", candidate_scores),
                    ("candidate_valid", candidate_valid)):
        _cuda(t, name)
    dev = candidate_idx.device
    rows, width = candidate_idx.shape
    idx = candidate_idx.to(torch.int64).contiguous()
    scores = candidate_scores.to(torch.float32).contiguous()
    valid = candidate_valid.to(torch.uint8).contiguous()
    if width == 0 or budget <= 0:
        return candidate_idx[:, :0], candidate_scores[:, :0], candidate_valid[:, :0], 0
    refill = min(width, max(budget, budget * refill_factor))
    sel_count = min(budget, refill)
    sel_idx = torch.empty(rows, sel_count, dtype=torch.int64, device=dev)
    sel_scores = torch.empty(rows, sel_count, dtype=torch.float32, device=dev)
    sel_valid = torch.empty(rows, sel_count, dtype=torch.uint8, device=dev)
    refill_out = ctypes.c_int32(0)
    rc = _lib.load().sva_top_unique(idx.data_ptr(), scores.data_ptr(), valid.data_ptr(), rows, width, int(budget),
                                    int(refill_factor), sel_idx.data_ptr(), sel_scores.data_ptr(), sel_valid.data_ptr(),
                                    ctypes.byref(refill_out), _stream(dev))
    _lib.check(rc)
    return sel_idx, sel_scores.to(candidate_scores.dtype), sel_valid.bool(), int(refill_out.value)
