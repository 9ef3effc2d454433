"""The C-ABI library loads without a GPU and exports every function include/sva_b200.h declares."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from sva_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "sva_b200.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(sva_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_bound_symbols():
    names = declared_functions()
    assert set(names) == set(_lib.EXPORTED), (set(names) ^ set(_lib.EXPORTED))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.sva_version().startswith(b"sva_b200")


def test_struct_layouts_match_header_field_order():
    text = HEADER.read_text()
    for struct, cls in (("sva_decode_args", _lib.DecodeArgs), ("sva_inverted_args", _lib.InvertedArgs),
                        ("sva_batch_layout", _lib.BatchLayout), ("sva_shard_map", _lib.ShardMap)):
        body = re.search(r"typedef struct " + struct + r" \{(.*?)\} " + struct + ";", text, flags=re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            names = [n.strip().lstrip("*") for n in re.sub(r"^[a-z_ 0-9]*?[a-z_0-9]+\*?\s+", "", decl).split(",")]
            fields.extend(n.split()[-1].lstrip("*") for n in names)
        assert [f[0] for f in cls._fields_] == fields, struct


def test_errors_map_to_exceptions_without_a_gpu():
    lib = _lib.load()
    args = _lib.DecodeArgs()  # all zero: rejected by validation before any CUDA call
    assert lib.sva_decode_workspace_size(ctypes.byref(args)) == 0
    rc = lib.sva_decode(ctypes.byref(args), None, 0, None)
    assert rc == _lib.SVA_ERR_SHAPE
    try:
        _lib.check(rc)
    except ValueError as exc:
        assert "n_heads" in str(exc)
    else:
        raise AssertionError("expected ValueError")


def test_host_buffer_check_rejects_memory_the_gpu_cannot_address():
    """Pageable host memory and NULL are never reported as device-addressable (on a machine
    without a GPU every pointer is rejected), so decode never hands the kernels such a pointer."""
    lib = _lib.load()
    buf = ctypes.create_string_buffer(256)
    assert lib.sva_host_buffer_device_accessible(ctypes.cast(buf, ctypes.c_void_p)) == 0
    assert lib.sva_host_buffer_device_accessible(None) == 0
