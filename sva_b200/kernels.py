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


def catalog_encode(keys: torch.Tensor, k_proj: torch.Tensor, codebooks: torch.Tensor, start: int, count: int,
                   k_low: torch.Tensor | None, codes: torch.Tensor | None, n_heads: int | None = None) -> None:
    """Write k_low / codes rows [start, start+count) of every query head.

    keys [Hkv, L, D] (rows contiguous), k_proj [H, D, R] fp32, codebooks [H, S, C, R/S] fp32,
    k_low [H, cap, R] fp32 (contiguous rows), codes [H, cap, S] uint8.
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
    rc = lib.sva_catalog_encode(
        keys.data_ptr(), dtype_code(keys.dtype), keys.stride(0), keys.stride(1), n_heads, n_kv, head_dim, rank,
        k_proj.data_ptr(), codebooks.data_ptr(), subspaces, codewords, int(start), int(count), _ptr(k_low),
        0 if k_low is None else k_low.stride(0), _ptr(codes), 0 if codes is None else codes.stride(0),
        _stream(keys.device))
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
    """
    for name, t in (("q", q), ("codes", codes), ("k_low", k_low), ("keys", keys), ("values", values)):
        _cuda(t, name)
    dev = q.device
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
    sl_out = fin_out = None
    if want_shortlist:
        sl_out = torch.empty(n_heads, n_q, int(shortlist), dtype=torch.int32, device=dev)
        a.shortlist_out = sl_out.data_ptr()
    if want_final:
        fin_out = torch.empty(n_heads, n_q, int(budget), dtype=torch.int32, device=dev)
        a.final_out = fin_out.data_ptr()
    a.stats = _ptr(stats)
    lib = _lib.load()
    ws_bytes = int(lib.sva_decode_workspace_size(ctypes.byref(a)))
    ws = _decode_ws.get(dev, ws_bytes)
    rc = lib.sva_decode(ctypes.byref(a), _ptr(ws), ws_bytes, _stream(dev))
    _lib.check(rc)
    if want_shortlist or want_final:
        return out, sl_out, fin_out
    return out


def sva_scale(logit_scale: torch.Tensor) -> torch.Tensor:
    """clamp(exp(logit_scale), 0.01, 100) computed as the reference does (sva/llama.py:69-73)."""
    return logit_scale.detach().float().exp().clamp(0.01, 100.0)


def sqrt_rank(rank_dim: int) -> float:
    return math.sqrt(rank_dim)
