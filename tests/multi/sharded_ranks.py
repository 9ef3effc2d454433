"""Worker for tests/test_gpu_sharded_nccl.py: one rank of a key-range sharded decode over NCCL.

Every rank builds the same seeded 9-head catalog, keeps its key range, runs ShardedDecoder and
compares the result with the one-GPU decode over all keys (computed on its own GPU).  Exit code
0 when the shortlist-derived output matches; the rank prints one line.
"""

from __future__ import annotations

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))

from sva_b200 import kernels  # noqa: E402
from sva_b200.sharded import ShardedDecoder  # noqa: E402
from tests.golden.inputs import config2  # noqa: E402
from tests.helpers import gpu_catalog, gpu_decode  # noqa: E402


def batched_ranks(rank: int, world: int, dev: torch.device) -> bool:
    """BatchedShardedDecoder over a bf16 batch, eager and captured in a CUDA graph (kernels and
    NCCL all-gathers), must equal the one-GPU batched decode bit for bit."""
    from sva_b200.sharded import BatchedShardedDecoder
    from tests.test_gpu_batched import make_batch
    from tests.test_gpu_sharded_batched import key_range_ranks, one_gpu

    batch = make_batch([60000, 60000, 56000, 64000], seed=41)
    want = one_gpu(batch)
    x = key_range_ranks(batch, world)[rank]
    dec = BatchedShardedDecoder(dist.group.WORLD, 2048, 512, dev)

    def call(saturated=None, out=None):
        return dec.decode(x["q"], x["q_proj"], x["scale"], x["cb"], x["codes"], x["k_low"], x["keys"], x["values"],
                          seq_lens=x["seq_lens"], max_len=x["max_len"], key_offset=x["key_offset"], out=out,
                          logits_mode=1, softmax_scale=0.125, saturated=saturated)

    eager = call()
    torch.cuda.synchronize()
    # captured: the ranks' shares of these shortlists fit the exchange width (no saturation)
    sat = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.empty_like(eager)
    stream = torch.cuda.Stream(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        call(sat, out)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            call(sat, out)
    sat.zero_()
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    flagged = int(sat.item())
    good = torch.equal(eager, want) and (flagged == 1 or torch.equal(out, want))
    print(f"rank {rank}: batched eager_equal={torch.equal(eager, want)} graph_equal={torch.equal(out, want)} "
          f"saturated={flagged}", flush=True)
    del graph
    return good


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        case = config2(key_len=200_000, subspaces=4, codewords=64, n_heads=9)
        k_low, codes = gpu_catalog(case, device=dev)
        ref, _, _ = gpu_decode(case, k_low, codes, device=dev)
        lo = case.key_len * rank // world
        hi = case.key_len * (rank + 1) // world
        dec = ShardedDecoder(dist.group.WORLD, heads=case.n_heads, head_dim=64, shortlist=case.shortlist,
                             budget=case.budget, device=dev)
        out = dec.decode(case.q[0].to(dev), case.q_proj.to(dev), kernels.sva_scale(case.logit_scale).to(dev),
                         case.codebooks.to(dev), codes[:, lo:hi].contiguous(), k_low[:, lo:hi].contiguous(),
                         case.keys[0][:, lo:hi].contiguous().to(dev), case.values[0][:, lo:hi].contiguous().to(dev),
                         key_offset=lo, logits_mode=1, softmax_scale=0.125)
        torch.cuda.synchronize()
        a, b = out[:, 0].float(), ref[:, 0].float()
        close = torch.allclose(a, b, rtol=1e-3, atol=1e-3)
        equal = float((a == b).float().mean())
        print(f"rank {rank}: allclose={close} bit_equal_fraction={equal:.4f}", flush=True)
        ok = close and equal >= 0.99
        ok = batched_ranks(rank, world, dev) and ok
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        return 0 if int(flag.item()) == 1 else 1
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
