"""sva_postings_build_noalloc: the posting lists of sva_postings_build, built from the library's
static per-device scratch instead of a caller workspace.

Collected last on purpose (file name), so it also runs after every other GPU test has used the
library and the caching allocator.  Each case calls the no-alloc entry point twice in a row, on
two different inputs, and compares both results with the workspace entry point.
"""

from __future__ import annotations

import pytest
import torch

from sva_b200 import _lib, kernels

pytestmark = pytest.mark.gpu


def _noalloc(codes: torch.Tensor, codewords: int):
    n_heads, key_len, subspaces = codes.shape
    dev = codes.device
    # filled with a sentinel so that anything the call leaves unwritten shows up
    counts = torch.full((n_heads, subspaces, codewords), -7, dtype=torch.int32, device=dev)
    offsets = torch.full((n_heads, subspaces, codewords + 1), -7, dtype=torch.int32, device=dev)
    ids = torch.full((n_heads, subspaces, key_len), -7, dtype=torch.int32, device=dev)
    max_bucket = torch.full((1,), -7, dtype=torch.int32, device=dev)
    lib = _lib.load()
    rc = lib.sva_postings_build_noalloc(codes.data_ptr(), codes.stride(0), n_heads, subspaces, codewords, key_len,
                                        counts.data_ptr(), offsets.data_ptr(), ids.data_ptr(), ids.shape[-1],
                                        max_bucket.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(rc)
    return counts, offsets, ids, max_bucket


def _codes(seed: int, n_heads: int, key_len: int, subspaces: int, codewords: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, codewords, (n_heads, key_len, subspaces), generator=g, dtype=torch.uint8).cuda()


def _assert_same(got, ref) -> None:
    counts, offsets, ids, max_bucket = got
    assert torch.equal(counts, ref.counts)
    assert torch.equal(offsets, ref.offsets)
    assert torch.equal(ids, ref.ids[..., : ids.shape[-1]])
    assert int(max_bucket.item()) == int(ref.max_bucket.item())


@pytest.mark.parametrize("first,second", [
    ((9, 200_000, 4, 64), (1, 1 << 20, 1, 256)),
    ((1, 1 << 20, 1, 256), (3, 4097, 2, 256)),
    ((9, 3_700_000, 4, 64), (9, 8192, 4, 64)),  # the first input fills nearly the whole scratch
])
def test_noalloc_matches_workspace_entry_point_twice_in_a_row(first, second):
    for seed, (n_heads, key_len, subspaces, codewords) in enumerate((first, second)):
        codes = _codes(seed, n_heads, key_len, subspaces, codewords)
        ref = kernels.postings_build(codes, codewords)
        got = _noalloc(codes, codewords)
        torch.cuda.synchronize()
        _assert_same(got, ref)


def test_noalloc_rejects_a_shape_larger_than_the_scratch():
    lib = _lib.load()
    n_heads, subspaces, codewords, key_len = 9, 4, 64, 4_000_000
    need = int(lib.sva_postings_workspace_size(n_heads, subspaces, codewords, key_len))
    assert need > _lib.POSTINGS_NOALLOC_SCRATCH_BYTES
    # rejected before any pointer is touched, so placeholder pointers are never dereferenced
    rc = lib.sva_postings_build_noalloc(None, key_len * subspaces, n_heads, subspaces, codewords, key_len,
                                        None, None, None, key_len, None, None)
    assert rc == _lib.SVA_ERR_WORKSPACE
    assert b"static scratch" in lib.sva_last_error()
