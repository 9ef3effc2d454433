"""Generate the golden fixtures under tests/golden by running the reference implementation.

Run in the build container (the reference is importable there, not on the GPU box):

    python tests/golden/make_golden.py --reference /path/to/reference

For every case it records what the reference's own code computes (codes, q_low, LUT, the
shortlist, the final indices, the attention output), using the reference's public ops
(``sva.ops``) and ``SVALlamaAttention``.  The reference's ``torch.topk`` breaks score ties in
an unspecified order, so the scan cases record two versions of every selection:

* ``*_raw``: what ``SVALlamaAttention.sva_attention`` itself selected;
* ``*_canon``: the same reference scores with the canonical tie rule (score descending, key
  index ascending), which is the rule the oracle and the CUDA kernels implement.

The fixtures store only outputs plus the seed; the inputs are regenerated from the seeded
recipes in ``tests/golden/inputs.py``.
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden.inputs import config1, config2  # noqa: E402


def _attention(case, summon_mode: str = "scan", **serving_kw):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaAttention

    from sva import SVALayerArtifacts
    from sva.llama import SVALlamaAttention, SVALlamaServingConfig

    n_heads, n_kv, head_dim = case.n_heads, case.n_kv_heads, int(case.q.shape[-1])
    cfg = LlamaConfig(hidden_size=n_heads * head_dim, num_attention_heads=n_heads, num_key_value_heads=n_kv,
                      head_dim=head_dim, intermediate_size=64, num_hidden_layers=1, vocab_size=16)
    original = LlamaAttention(cfg, 0)
    arts = SVALayerArtifacts(case.q_proj, case.k_proj, case.logit_scale, case.codebooks, 0.0, 0.0, "qk")
    serving = SVALlamaServingConfig(rank_dim=int(case.q_proj.shape[-1]), coarse_shortlist=case.shortlist,
                                    budget=case.budget, summon_mode=summon_mode, **serving_kw)
    attn = SVALlamaAttention(original, arts, serving, None)
    attn.eval()
    return attn


def _stable_desc(scores: torch.Tensor) -> torch.Tensor:
    """Indices sorting a 1-D tensor by (score desc, index asc)."""
    return torch.sort(scores, descending=True, stable=True).indices


def scan_case(case, prefix: str) -> dict:
    from sva.ops import product_quantized_scores

    attn = _attention(case)
    with torch.no_grad():
        out_raw = attn.sva_attention(case.q, case.keys, case.values, None)
    k_low = attn._cached_k_low[0]            # [H, L, R] fp32
    codes = attn._cached_coarse_codes        # [H, L, S] int64
    n_heads, key_len, rank = k_low.shape
    groups = n_heads // case.n_kv_heads
    q_low = torch.einsum("bhtd,hdr->bhtr", case.q.float(), attn.sva_q_proj) * attn.sva_scale[None, :, None, None]
    q_low = q_low[0]                          # [H, 1, R]
    subspaces, codewords, sub = case.codebooks.shape[1:]
    lut = torch.einsum("htsd,hscd->htsc", q_low.reshape(n_heads, 1, subspaces, sub), attn.sva_coarse_codebooks)
    coarse = product_quantized_scores(q_low, attn.sva_coarse_codebooks, codes, rank)  # [H, 1, L]
    sl = min(case.shortlist, key_len)
    bud = min(case.budget, sl)

    # the reference's own selection (same call sequence as sva/llama.py:278 and :295)
    raw_idx = coarse.topk(sl, dim=-1).indices[:, 0]  # [H, SL]
    res = {}
    canon_sl, canon_fin, canon_rs, canon_out, rank_gap, coarse_bound = [], [], [], [], [], []
    above_equal = []
    for h in range(n_heads):
        order = _stable_desc(coarse[h, 0])[:sl]
        boundary = coarse[h, 0, order[-1]]
        # cross-check: the unmodified reference picked the same multiset of scores and the same
        # set of keys strictly above the boundary score.
        raw_scores = torch.sort(coarse[h, 0, raw_idx[h]]).values
        canon_scores = torch.sort(coarse[h, 0, order]).values
        strict_raw = set(raw_idx[h][coarse[h, 0, raw_idx[h]] > boundary].tolist())
        strict_canon = set(order[coarse[h, 0, order] > boundary].tolist())
        above_equal.append(bool(torch.equal(raw_scores, canon_scores)) and strict_raw == strict_canon)
        coarse_bound.append(float(boundary))
        short = torch.sort(order).values     # ascending key index
        low = k_low[h, short]
        rs = (low * q_low[h, 0][None, :]).sum(dim=-1) / math.sqrt(rank)
        keep = _stable_desc(rs)[:bud]
        fin = short[keep]
        srt = torch.sort(rs, descending=True).values
        rank_gap.append(float(srt[bud - 1] - srt[bud]) if bud < srt.shape[0] else float("inf"))
        kv = h // groups
        sel_k = case.keys[0, kv, fin]
        sel_v = case.values[0, kv, fin]
        qq = case.q[0, h, 0]
        logits = (sel_k * qq[None, :]).sum(dim=-1) * attn.scaling
        w = torch.softmax(logits, dim=-1, dtype=torch.float32).to(case.q.dtype)
        canon_out.append((w[:, None] * sel_v).sum(dim=0).float())
        canon_sl.append(short)
        canon_fin.append(fin)
        canon_rs.append(rs[keep])
    sample_rows = torch.cat([torch.arange(0, min(64, key_len)), case.planted.flatten()])
    res[f"{prefix}_codes"] = codes.to(torch.uint8).numpy()
    res[f"{prefix}_k_low_sample_rows"] = sample_rows.numpy()
    res[f"{prefix}_k_low_sample"] = k_low[:, sample_rows].numpy()
    res[f"{prefix}_k_low_headsum"] = k_low.double().sum(dim=(1, 2)).numpy()
    res[f"{prefix}_q_low"] = q_low.numpy()
    res[f"{prefix}_lut"] = lut.numpy()
    res[f"{prefix}_shortlist_raw"] = torch.sort(raw_idx, dim=-1).values.numpy()
    res[f"{prefix}_shortlist_canon"] = torch.stack(canon_sl).numpy()
    res[f"{prefix}_coarse_boundary"] = np.asarray(coarse_bound, dtype=np.float32)
    res[f"{prefix}_raw_vs_canon_consistent"] = np.asarray(above_equal)
    res[f"{prefix}_final_canon"] = torch.stack(canon_fin).numpy()
    res[f"{prefix}_rank_scores_canon"] = torch.stack(canon_rs).numpy()
    res[f"{prefix}_rank_gap"] = np.asarray(rank_gap, dtype=np.float64)
    res[f"{prefix}_out_canon"] = torch.stack(canon_out).numpy()
    res[f"{prefix}_out_raw"] = out_raw[0, :, 0].float().numpy()
    return res


def static_case(case, prefix: str, tail: int, **serving_kw) -> dict:
    """Static inverted decode with ``tail`` keys appended after the postings were built."""
    from sva.llama import SVALlamaAttention

    attn = _attention(case, summon_mode="inverted_static", **serving_kw)
    captured = {}
    original = SVALlamaAttention._top_unique_candidates

    def recording(candidate_idx, candidate_scores, candidate_valid, budget, refill_factor=2):
        out = original(candidate_idx, candidate_scores, candidate_valid, budget, refill_factor)
        captured["sel"] = out
        return out

    key_len = case.key_len
    base = key_len - tail
    with torch.no_grad():
        # prefill-sized first call builds the catalog and the postings
        attn._top_unique_candidates = recording
        attn.sva_attention(case.q, case.keys[:, :, :base], case.values[:, :, :base], None)
        outs = None
        for n in range(base + 1, key_len + 1):
            outs = attn.sva_attention(case.q, case.keys[:, :, :n], case.values[:, :, :n], None)
    sel_idx, sel_scores, sel_valid, refill = captured["sel"]
    res = {
        f"{prefix}_tail": np.asarray(tail),
        f"{prefix}_postings_len": np.asarray(attn._cached_postings_key_len),
        f"{prefix}_sel_idx": sel_idx.numpy(),
        f"{prefix}_sel_valid": sel_valid.numpy(),
        f"{prefix}_sel_scores": sel_scores.numpy(),
        f"{prefix}_refill": np.asarray(refill),
        f"{prefix}_out": outs[0, :, 0].float().numpy(),
        f"{prefix}_counts": attn._cached_posting_counts.numpy(),
    }
    # exact rank-score ties between distinct selected keys would make the raw reference order
    # implementation-defined; the fixture cases are chosen to have none.
    for h in range(sel_idx.shape[0]):
        v = sel_valid[h]
        s = sel_scores[h][v]
        assert torch.unique(s).numel() == s.numel(), "tie among distinct keys in static fixture"
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="path of the reference checkout (contains sva/)")
    ap.add_argument("--out", default=str(HERE / "golden_v1.npz"))
    ap.add_argument("--models", action="store_true", help="write the model-level fixtures instead")
    ap.add_argument("--models-bf16", action="store_true", help="write the bf16 model-level fixtures instead")
    args = ap.parse_args()
    if args.reference:
        sys.path.insert(0, args.reference)
    torch.set_num_threads(8)
    if args.models or args.models_bf16:
        return
    res = {}
    res.update(scan_case(config1(), "cfg1"))
    res.update(scan_case(config2(key_len=1 << 16, subspaces=1, codewords=256), "cfg2s_1x256"))
    res.update(scan_case(config2(key_len=1 << 16, subspaces=4, codewords=64), "cfg2s_4x64"))
    res.update(static_case(config1(key_len=4096), "static_cfg1", tail=3, inverted_cells_per_subspace=8))
    res.update(static_case(config2(key_len=1 << 14, subspaces=4, codewords=64, n_planted=16), "static_4x64", tail=5,
                           inverted_cells_per_subspace=8))
    res.update(static_case(config1(key_len=2048, seed=5), "static_adaptive", tail=2, inverted_cells_per_subspace=4,
                           adaptive_min_budget=64, adaptive_mid_budget=128))
    np.savez_compressed(args.out, **res)
    print("wrote", args.out, {k: v.shape for k, v in res.items()})


if __name__ == "__main__":
    main()


def canonical_topk(self, k, dim=-1, largest=True, sorted=True):
    """torch.topk with the canonical tie rule (score desc, index asc): a stable descending sort."""
    assert largest, "the reference only takes largest-k"
    vals, idx = torch.sort(self, dim=dim, descending=True, stable=True)
    return torch.return_types.topk((vals.narrow(dim, 0, k), idx.narrow(dim, 0, k)))


def model_cases(out_path: str, bf16: bool = False) -> None:
    """Model-level fixtures: the reference's patch_llama_attention on seeded random Llama models,
    with torch.Tensor.topk replaced by canonical_topk for the duration of each run.  ``bf16``
    selects the bf16 SmolLM2-shaped cases (model_cases.BF16_CASES)."""
    from sva import SVAArtifactBundle, SVALayerArtifacts, patch_llama_attention
    from tests.golden import model_cases as mc

    from sva.llama import SVALlamaAttention

    res = {}
    original = torch.Tensor.topk
    original_attention = SVALlamaAttention.sva_attention
    calls: list = []

    def recording_attention(self, query, key, value, attention_mask):
        # the inputs and output of every SVA attention call of layer 1 (bf16 cases): the GPU test
        # feeds the same tensors to the B200 module, so the comparison does not depend on how the
        # rest of the model rounds on each device
        out = original_attention(self, query, key, value, attention_mask)
        if self.layer_idx == 1:
            allowed = None if attention_mask is None else (attention_mask[..., : query.shape[2], : key.shape[2]] > -1e4)
            calls.append((query.detach().clone(), key.detach().clone(), value.detach().clone(),
                          None if allowed is None else allowed.detach().clone(), out.detach().clone()))
        return out

    def bits(t: torch.Tensor) -> np.ndarray:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()

    try:
        torch.Tensor.topk = canonical_topk
        if bf16:
            SVALlamaAttention.sva_attention = recording_attention
        for name in (mc.BF16_CASES if bf16 else mc.CASES):
            calls.clear()
            model, bundle, steps, case = mc.build(name, SVAArtifactBundle, SVALayerArtifacts)
            res[f"{name}_model_checksum"] = np.asarray(sum(float(p.double().sum()) for p in model.parameters()))
            outs, summary, state = mc.run(model, patch_llama_attention, bundle, steps, case)
            if bf16:
                # layer 1's calls: queries and outputs of every step, the final K / V (each step's
                # cache is a prefix of it), and the mask of the calls that had one
                res[f"{name}_l1_calls"] = np.asarray(len(calls))
                res[f"{name}_l1_key"] = bits(calls[-1][1])
                res[f"{name}_l1_value"] = bits(calls[-1][2])
                for i, (q, k, v, allowed, out) in enumerate(calls):
                    res[f"{name}_l1_q_{i}"] = bits(q)
                    res[f"{name}_l1_klen_{i}"] = np.asarray(k.shape[2])
                    res[f"{name}_l1_out_{i}"] = bits(out)
                    if allowed is not None:
                        res[f"{name}_l1_allowed_{i}"] = allowed[0, 0].numpy()
            for i, o in enumerate(outs):
                res[f"{name}_logits_{i}"] = o.numpy()
            for k, v in summary.items():
                res[f"{name}_summary_{k}"] = np.asarray(v)
            for k, v in state.items():
                res[f"{name}_state_{k}"] = np.asarray(v)
    finally:
        torch.Tensor.topk = original
        SVALlamaAttention.sva_attention = original_attention
    np.savez_compressed(out_path, **res)
    print("wrote", out_path, len(res), "arrays")


if __name__ == "__main__" and "--models" in sys.argv:
    model_cases(str(HERE / "golden_models_v1.npz"))
if __name__ == "__main__" and "--models-bf16" in sys.argv:
    model_cases(str(HERE / "golden_models_bf16_v1.npz"), bf16=True)
