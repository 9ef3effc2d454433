"""ctypes binding of libsva_b200.so (the C ABI declared in include/sva_b200.h).

The library is loaded from this package directory.  There is no fallback: if the shared
library is missing or cannot be loaded, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsva_b200.so"

SVA_OK = 0
SVA_ERR_SHAPE = 1
SVA_ERR_WORKSPACE = 2
SVA_ERR_TIMEOUT = 3
SVA_ERR_CUDA = 4
SVA_ERR_ALIGN = 5
SVA_ERR_DTYPE = 6

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

STAT_QUERIES = 0
STAT_SUMMONED = 1
STAT_REFILL_POOL = 2
STAT_EXACT_SCORED = 3
STAT_VERIFIED = 4
STAT_CELL_VISITS = 5
STAT_SELECT_FALLBACKS = 6
STAT_COUNT = 8
POSTINGS_NOALLOC_SCRATCH_BYTES = 8 << 20  # SVA_POSTINGS_NOALLOC_SCRATCH_BYTES

# Every symbol include/sva_b200.h declares (checked by the CPU test suite).
EXPORTED = (
    "sva_version",
    "sva_last_error",
    "sva_profile_events",
    "sva_debug_timestamps",
    "sva_host_buffer_device_accessible",
    "sva_catalog_encode",
    "sva_catalog_encode_at",
    "sva_catalog_encode_tc",
    "sva_assign_centroids",
    "sva_pq_scores",
    "sva_decode_workspace_size",
    "sva_decode",
    "sva_decode_batched_workspace_size",
    "sva_decode_batched",
    "sva_shard_workspace_size",
    "sva_shard_summon",
    "sva_shard_rescore",
    "sva_shard_verify",
    "sva_shard_combine",
    "sva_shard_batched_workspace_size",
    "sva_shard_batched_summon",
    "sva_shard_batched_rescore",
    "sva_shard_batched_verify",
    "sva_shard_batched_combine",
    "sva_postings_workspace_size",
    "sva_postings_build",
    "sva_postings_build_noalloc",
    "sva_postings_append",
    "sva_inverted_workspace_size",
    "sva_decode_inverted",
    "sva_inverted_shard_workspace_size",
    "sva_inverted_shard_summon",
    "sva_inverted_shard_verify",
    "sva_inverted_shard_combine",
    "sva_top_unique",
    "sva_adapter_forward",
)

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f32 = ctypes.c_float
c_vp = ctypes.c_void_p
c_sz = ctypes.c_size_t


class DecodeArgs(ctypes.Structure):
    """Mirror of ``sva_decode_args``."""

    _fields_ = [
        ("n_heads", c_i32),
        ("n_kv_heads", c_i32),
        ("n_queries", c_i32),
        ("head_dim", c_i32),
        ("rank_dim", c_i32),
        ("subspaces", c_i32),
        ("codewords", c_i32),
        ("shortlist", c_i32),
        ("budget", c_i32),
        ("qkv_dtype", c_i32),
        ("logits_mode", c_i32),
        ("softmax_scale", c_f32),
        ("key_len", c_i64),
        ("query", c_vp),
        ("q_head_stride", c_i64),
        ("q_row_stride", c_i64),
        ("q_proj", c_vp),
        ("scale", c_vp),
        ("codebooks", c_vp),
        ("lut_override", c_vp),
        ("codes", c_vp),
        ("codes_head_stride", c_i64),
        ("k_low", c_vp),
        ("k_low_head_stride", c_i64),
        ("keys", c_vp),
        ("k_head_stride", c_i64),
        ("k_row_stride", c_i64),
        ("values", c_vp),
        ("v_head_stride", c_i64),
        ("v_row_stride", c_i64),
        ("allowed_len", c_vp),
        ("allowed_mask", c_vp),
        ("mask_row_stride", c_i64),
        ("out", c_vp),
        ("out_head_stride", c_i64),
        ("out_row_stride", c_i64),
        ("shortlist_out", c_vp),
        ("final_out", c_vp),
        ("stats", c_vp),
    ]


class BatchLayout(ctypes.Structure):
    """Mirror of ``sva_batch_layout``."""

    _fields_ = [
        ("n_seqs", c_i32),
        ("page_keys", c_i32),
        ("seq_lens", c_vp),
        ("page_table", c_vp),
        ("page_table_stride", c_i64),
        ("q_seq_stride", c_i64),
        ("out_seq_stride", c_i64),
        ("codes_page_stride", c_i64),
        ("k_low_page_stride", c_i64),
        ("k_page_stride", c_i64),
        ("v_page_stride", c_i64),
    ]


class ShardMap(ctypes.Structure):
    """Mirror of ``sva_shard_map``."""

    _fields_ = [
        ("key_offset", c_i64),
        ("page_world", c_i32),
        ("page_rank", c_i32),
    ]


class InvertedArgs(ctypes.Structure):
    """Mirror of ``sva_inverted_args``."""

    _fields_ = [
        ("n_heads", c_i32),
        ("n_kv_heads", c_i32),
        ("head_dim", c_i32),
        ("rank_dim", c_i32),
        ("subspaces", c_i32),
        ("codewords", c_i32),
        ("budget", c_i32),
        ("cells", c_i32),
        ("refill_factor", c_i32),
        ("dynamic", c_i32),
        ("min_budget", c_i32),
        ("mid_budget", c_i32),
        ("qkv_dtype", c_i32),
        ("low_margin", c_f32),
        ("high_margin", c_f32),
        ("softmax_scale", c_f32),
        ("key_len", c_i64),
        ("postings_len", c_i64),
        ("allowed_len", c_i64),
        ("allowed_mask", c_vp),
        ("query", c_vp),
        ("q_head_stride", c_i64),
        ("q_proj", c_vp),
        ("scale", c_vp),
        ("codebooks", c_vp),
        ("codes", c_vp),
        ("codes_head_stride", c_i64),
        ("post_counts", c_vp),
        ("post_offsets", c_vp),
        ("post_ids", c_vp),
        ("post_ids_sub_stride", c_i64),
        ("max_bucket", c_vp),
        ("k_low", c_vp),
        ("k_low_head_stride", c_i64),
        ("keys", c_vp),
        ("k_head_stride", c_i64),
        ("k_row_stride", c_i64),
        ("values", c_vp),
        ("v_head_stride", c_i64),
        ("v_row_stride", c_i64),
        ("out", c_vp),
        ("out_head_stride", c_i64),
        ("sel_idx_out", c_vp),
        ("sel_valid_out", c_vp),
        ("sel_score_out", c_vp),
        ("budget_out", c_vp),
        ("stats", c_vp),
    ]


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load libsva_b200.so (raises if it is missing)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run `python -m sva_b200.build` (needs nvcc)")
        lib = ctypes.CDLL(os.fspath(LIB_PATH))
        lib.sva_version.restype = ctypes.c_char_p
        lib.sva_last_error.restype = ctypes.c_char_p
        sigs = {
            "sva_profile_events": ([c_vp, c_i32], ctypes.c_int),
            "sva_debug_timestamps": ([c_vp], ctypes.c_int),
            "sva_host_buffer_device_accessible": ([c_vp], ctypes.c_int),
            "sva_catalog_encode": ([c_vp, c_i32, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32, c_i32,
                                    c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp], ctypes.c_int),
            "sva_catalog_encode_at": ([c_vp, c_i32, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32,
                                       c_i32, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp], ctypes.c_int),
            "sva_catalog_encode_tc": ([c_vp, c_i32, c_i64, c_i64, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32,
                                       c_i32, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_vp], ctypes.c_int),
            "sva_assign_centroids": ([c_vp, c_i64, c_i32, c_i64, c_vp, c_i32, c_vp, c_vp], ctypes.c_int),
            "sva_pq_scores": ([c_vp, c_i32, c_i32, c_i32, c_vp, c_i32, c_i32, c_vp, c_i64, c_vp, c_vp], ctypes.c_int),
            "sva_decode_workspace_size": ([ctypes.POINTER(DecodeArgs)], c_sz),
            "sva_decode": ([ctypes.POINTER(DecodeArgs), c_vp, c_sz, c_vp], ctypes.c_int),
            "sva_decode_batched_workspace_size": ([ctypes.POINTER(DecodeArgs), ctypes.POINTER(BatchLayout)], c_sz),
            "sva_decode_batched": ([ctypes.POINTER(DecodeArgs), ctypes.POINTER(BatchLayout), c_vp, c_sz, c_vp],
                                   ctypes.c_int),
            "sva_shard_workspace_size": ([ctypes.POINTER(DecodeArgs)], c_sz),
            "sva_shard_summon": ([ctypes.POINTER(DecodeArgs), c_i64, c_vp, c_vp, c_sz, c_vp], ctypes.c_int),
            "sva_shard_rescore": ([ctypes.POINTER(DecodeArgs), c_i64, c_i32, c_i32, c_vp, c_vp, c_vp, c_sz, c_vp],
                                  ctypes.c_int),
            "sva_shard_verify": ([ctypes.POINTER(DecodeArgs), c_i64, c_i32, c_i32, c_vp, c_vp, c_vp], ctypes.c_int),
            "sva_shard_combine": ([ctypes.POINTER(DecodeArgs), c_i32, c_vp, c_vp], ctypes.c_int),
            "sva_shard_batched_workspace_size": ([ctypes.POINTER(DecodeArgs), c_vp, c_vp, c_i32], c_sz),
            "sva_shard_batched_summon": ([ctypes.POINTER(DecodeArgs), c_vp, c_vp, c_i32, c_vp, c_vp, c_sz, c_vp],
                                         ctypes.c_int),
            "sva_shard_batched_rescore": ([ctypes.POINTER(DecodeArgs), c_vp, c_vp, c_i32, c_i32, c_i32, c_vp, c_vp,
                                           c_vp, c_vp, c_sz, c_vp], ctypes.c_int),
            "sva_shard_batched_verify": ([ctypes.POINTER(DecodeArgs), c_vp, c_vp, c_i32, c_i32, c_i32, c_vp, c_vp,
                                          c_vp], ctypes.c_int),
            "sva_shard_batched_combine": ([ctypes.POINTER(DecodeArgs), c_vp, c_i32, c_vp, c_vp], ctypes.c_int),
            "sva_postings_workspace_size": ([c_i32, c_i32, c_i32, c_i64], c_sz),
            "sva_postings_build": ([c_vp, c_i64, c_i32, c_i32, c_i32, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp,
                                    c_sz, c_vp], ctypes.c_int),
            "sva_postings_build_noalloc": ([c_vp, c_i64, c_i32, c_i32, c_i32, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp,
                                            c_vp], ctypes.c_int),
            "sva_postings_append": ([c_vp, c_i64, c_i32, c_i32, c_i32, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp,
                                     c_vp, c_vp], ctypes.c_int),
            "sva_inverted_workspace_size": ([ctypes.POINTER(InvertedArgs)], c_sz),
            "sva_decode_inverted": ([ctypes.POINTER(InvertedArgs), c_vp, c_sz, c_vp], ctypes.c_int),
            "sva_inverted_shard_workspace_size": ([ctypes.POINTER(InvertedArgs)], c_sz),
            "sva_inverted_shard_summon": ([ctypes.POINTER(InvertedArgs), c_i64, c_i32, c_vp, c_vp, c_sz, c_vp],
                                          ctypes.c_int),
            "sva_inverted_shard_verify": ([ctypes.POINTER(InvertedArgs), c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp,
                                           c_sz, c_vp], ctypes.c_int),
            "sva_inverted_shard_combine": ([ctypes.POINTER(InvertedArgs), c_i32, c_vp, c_vp], ctypes.c_int),
            "sva_top_unique": ([c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp,
                                ctypes.POINTER(ctypes.c_int32), c_vp], ctypes.c_int),
            "sva_adapter_forward": ([c_vp, c_i64, c_vp, c_i64, c_i32, c_vp, c_vp, c_vp, c_vp, c_f32, c_i32, c_i32,
                                     c_i32, c_i32, c_vp, c_i64, c_vp], ctypes.c_int),
        }
        for name, (argtypes, restype) in sigs.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = lib
        return lib


def check(rc: int) -> None:
    """Map an sva_status to a Python exception (no-op for SVA_OK)."""
    if rc == SVA_OK:
        return
    msg = load().sva_last_error().decode("utf-8", "replace")
    if rc in (SVA_ERR_SHAPE, SVA_ERR_WORKSPACE, SVA_ERR_ALIGN):
        raise ValueError(f"sva_b200: {msg}")
    if rc == SVA_ERR_DTYPE:
        raise TypeError(f"sva_b200: {msg}")
    if rc == SVA_ERR_TIMEOUT:
        raise TimeoutError(f"sva_b200: {msg}")
    raise RuntimeError(f"sva_b200 (status {rc}): {msg}")
