"""Batched model decode through the drop-in module, and the fused residual output adapter.

* ``SVALlamaAttention`` with ``allow_batch``: a batch of sequences (prefill, then cached decode
  steps that append to the catalog) gives, for every sequence, exactly the outputs of a batch-1
  module fed that sequence alone; the reference itself only runs batch 1
  (sva/llama.py:182-183), so batch-1 calls are its semantics for a batch.
* ``SVAResidualOutputAdapter``: the fused o_proj + adapter kernel against the reference's
  composition (experiments/sva_late4_logit_distill.py:47-51), restated with torch ops.
* A bf16 SmolLM2-shaped model with a late socket (last layer patched and wrapped in an adapter)
  decoding a batch greedily, against the same sequences decoded one at a time.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F
from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM
from transformers.models.llama.modeling_llama import LlamaAttention

from sva_b200 import SVALayerArtifacts, SVALlamaAttention, SVALlamaServingConfig
from sva_b200.adapter import SVAResidualOutputAdapter

pytestmark = pytest.mark.gpu

H, HKV, D = 9, 3, 64


def make_module(allow_batch: bool, shortlist=96, budget=24, seed=0):
    cfg = LlamaConfig(hidden_size=H * D, num_attention_heads=H, num_key_value_heads=HKV, head_dim=D,
                      intermediate_size=64, num_hidden_layers=1, vocab_size=16)
    gen = torch.Generator().manual_seed(seed)
    arts = SVALayerArtifacts((torch.randn(H, D, 64, generator=gen) * 0.125).to(torch.bfloat16).float(),
                             (torch.randn(H, D, 64, generator=gen) * 0.125).to(torch.bfloat16).float(),
                             torch.randn(H, generator=gen) * 0.1,
                             torch.randn(H, 2, 256, 32, generator=gen).to(torch.bfloat16).float(), 0.0, 0.0, "qk")
    serving = SVALlamaServingConfig(rank_dim=64, coarse_shortlist=shortlist, budget=budget, allow_batch=allow_batch)
    return SVALlamaAttention(LlamaAttention(cfg, 0), arts, serving, None).cuda().eval()


@pytest.mark.parametrize("prefill,shortlist,budget", [(300, 96, 24), (40000, 2048, 512)])
def test_batched_sva_attention_matches_batch_one(prefill, shortlist, budget):
    B, steps = 3, 3
    gen = torch.Generator().manual_seed(prefill)
    total = prefill + steps
    keys = torch.randn(B, HKV, total, D, generator=gen).to(torch.bfloat16).cuda()
    values = torch.randn(B, HKV, total, D, generator=gen).to(torch.bfloat16).cuda()
    q_pre = torch.randn(B, H, min(prefill, 64), D, generator=gen).to(torch.bfloat16).cuda()
    q_dec = torch.randn(B, H, steps, D, generator=gen).to(torch.bfloat16).cuda()
    batched = make_module(True, shortlist, budget)
    singles = [make_module(False, shortlist, budget) for _ in range(B)]
    with torch.no_grad():
        # prefill: the last q_pre.shape[2] tokens of the prompt (causal lengths)
        got = batched.sva_attention(q_pre, keys[:, :, :prefill], values[:, :, :prefill], None)
        for b in range(B):
            want = singles[b].sva_attention(q_pre[b:b + 1], keys[b:b + 1, :, :prefill], values[b:b + 1, :, :prefill],
                                            None)
            assert torch.equal(got[b:b + 1], want), f"prefill, sequence {b}"
        for s in range(steps):
            n = prefill + s + 1
            got = batched.sva_attention(q_dec[:, :, s:s + 1], keys[:, :, :n], values[:, :, :n], None)
            for b in range(B):
                want = singles[b].sva_attention(q_dec[b:b + 1, :, s:s + 1], keys[b:b + 1, :, :n],
                                                values[b:b + 1, :, :n], None)
                assert torch.equal(got[b:b + 1], want), f"decode step {s}, sequence {b}"
    assert batched._bkey_len == total


def test_batch_is_rejected_without_allow_batch():
    m = make_module(False)
    q = torch.zeros(2, H, 1, D, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(2, HKV, 8, D, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="batch size 1"):
        m.sva_attention(q, kv, kv, None)


class _Wrapped(torch.nn.Module):
    def __init__(self, o_proj):
        super().__init__()
        self.o_proj = o_proj


@pytest.mark.parametrize("rows,dtype", [(8, torch.bfloat16), (1, torch.bfloat16), (40, torch.bfloat16),
                                        (5, torch.float32)])
def test_fused_adapter_matches_reference_composition(rows, dtype):
    gen = torch.Generator().manual_seed(rows)
    hidden, rank = 576, 96
    o_proj = torch.nn.Linear(hidden, hidden, bias=False).to(dtype).cuda()
    with torch.no_grad():
        o_proj.weight.copy_((torch.randn(hidden, hidden, generator=gen) * 0.04).to(dtype))
    adapter = SVAResidualOutputAdapter(_Wrapped(o_proj), hidden, rank, scale=0.5).cuda()
    with torch.no_grad():
        adapter.down.weight.copy_(torch.randn(rank, 2 * hidden, generator=gen) * 0.02)
        adapter.up.weight.copy_(torch.randn(hidden, rank, generator=gen) * 0.02)
    h = torch.randn(1, rows, hidden, generator=gen).to(dtype).cuda()
    a = torch.randn(1, rows, hidden, generator=gen).to(dtype).cuda()
    with torch.no_grad():
        got = adapter.fused(h, a, o_proj)
        # the reference adapter around the wrapped layer's output o = o_proj(a)
        o = o_proj(a)
        corr = adapter.up(F.gelu(adapter.down(torch.cat([h.float(), o.float()], dim=-1)))) * adapter.scale
        want = o + corr.to(o.dtype)
    tol = 2e-2 if dtype != torch.float32 else 1e-4
    torch.testing.assert_close(got, want, rtol=tol, atol=tol)


def _socket_model():
    torch.manual_seed(17)
    cfg = LlamaConfig(vocab_size=256, hidden_size=576, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=9, num_key_value_heads=3, head_dim=64, max_position_embeddings=2048,
                      rope_theta=100000.0, rms_norm_eps=1e-5, tie_word_embeddings=True, attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).eval().to(torch.bfloat16).cuda()


def _socket_bundle():
    from sva_b200 import SVAArtifactBundle

    gen = torch.Generator().manual_seed(5)
    layers = {i: SVALayerArtifacts((torch.randn(9, 64, 64, generator=gen) * 0.125).to(torch.bfloat16),
                                   (torch.randn(9, 64, 64, generator=gen) * 0.125).to(torch.bfloat16),
                                   torch.zeros(9), torch.randn(9, 2, 256, 32, generator=gen).to(torch.bfloat16),
                                   0.0, 0.0, "qk") for i in range(2)}
    manifest = {"schema_version": 1, "artifact_type": "summon_verify_attention", "rank_dim": 64,
                "coarse_subspaces": 2, "coarse_codewords": 256, "default_shortlist": 96, "default_budget": 24,
                "layer_count": 2, "layers": [0, 1]}
    return SVAArtifactBundle(manifest=manifest, layers=layers)


def _greedy(model, ids, steps):
    cache = DynamicCache(config=model.config)
    out = model(input_ids=ids, use_cache=True, past_key_values=cache)
    tok = out.logits[:, -1].argmax(-1, keepdim=True)
    toks, logits = [tok], [out.logits[:, -1].float()]
    for _ in range(steps - 1):
        out = model(input_ids=tok, use_cache=True, past_key_values=out.past_key_values)
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        toks.append(tok)
        logits.append(out.logits[:, -1].float())
    return torch.cat(toks, 1), torch.stack(logits, 1)


def test_late_socket_batch_decode_with_adapter():
    from sva_b200 import patch_llama_attention
    from sva_b200.adapter import wrap_socket_layers_with_adapters

    model = _socket_model()
    handle = patch_llama_attention(model, _socket_bundle(), layers=[1], allow_batch=True)
    wrap_socket_layers_with_adapters(model, [1], rank=16, scale=1.0)
    with torch.no_grad():
        torch.nn.init.normal_(model.model.layers[1].self_attn.up.weight, std=0.02)
    ids = torch.randint(0, 256, (4, 200), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.no_grad():
        toks_b, logits_b = _greedy(model, ids, 6)
        for b in range(4):
            handle.reset_catalogs()
            toks_1, logits_1 = _greedy(model, ids[b:b + 1], 6)
            # the unpatched layers run batch GEMMs at batch 4 and 1, which may round differently
            rel = (logits_b[b] - logits_1[0]).norm() / logits_1[0].norm()
            assert rel < 5e-2, f"sequence {b}: relative logit error {float(rel):.3g}"
    assert isinstance(model.model.layers[1].self_attn, SVAResidualOutputAdapter)
    assert handle._unwrap_sva_attention(model.model.layers[1].self_attn) is handle.model.model.layers[1].self_attn.sva_attn
    handle.unpatch()
