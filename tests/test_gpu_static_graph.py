"""The static-cache SVA path and the CUDA-graph decode step (sva_b200.serving).

A model whose attention layers are all SVA-patched must generate exactly the same greedy tokens
(a) eagerly over HF's growing DynamicCache (the reference's way), (b) eagerly over a StaticCache
(SVALlamaAttention.sva_attention_static), and (c) with the per-token step captured in one CUDA
graph and replayed (GraphedGreedyDecoder) -- the SVA layers compute the same selections and
outputs from device-resident positions as from host-side lengths.
"""

from __future__ import annotations

import pytest
import torch
from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM, StaticCache

from sva_b200 import SVAArtifactBundle, SVALayerArtifacts, patch_llama_attention
from sva_b200.serving import GraphedGreedyDecoder

pytestmark = pytest.mark.gpu


def _model(layers=2):
    torch.manual_seed(11)
    cfg = LlamaConfig(vocab_size=512, hidden_size=576, intermediate_size=256, num_hidden_layers=layers,
                      num_attention_heads=9, num_key_value_heads=3, head_dim=64, max_position_embeddings=4096,
                      rope_theta=100000.0, rms_norm_eps=1e-5, tie_word_embeddings=True, attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).eval().to(torch.bfloat16).cuda()


def _bundle(layers=2, shortlist=96, budget=24):
    gen = torch.Generator().manual_seed(9)
    arts = {i: SVALayerArtifacts((torch.randn(9, 64, 64, generator=gen) * 0.125).to(torch.bfloat16),
                                 (torch.randn(9, 64, 64, generator=gen) * 0.125).to(torch.bfloat16),
                                 torch.zeros(9), torch.randn(9, 2, 256, 32, generator=gen).to(torch.bfloat16),
                                 0.0, 0.0, "qk") for i in range(layers)}
    manifest = {"schema_version": 1, "artifact_type": "summon_verify_attention", "rank_dim": 64,
                "coarse_subspaces": 2, "coarse_codewords": 256, "default_shortlist": shortlist,
                "default_budget": budget, "layer_count": layers, "layers": list(range(layers))}
    return SVAArtifactBundle(manifest=manifest, layers=arts)


def _greedy(model, prompt, steps, cache):
    with torch.no_grad():
        out = model(input_ids=prompt, use_cache=True, past_key_values=cache, logits_to_keep=1)
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        toks = [tok]
        for _ in range(steps - 1):
            out = model(input_ids=tok, use_cache=True, past_key_values=cache, logits_to_keep=1)
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            toks.append(tok)
    return torch.cat(toks, 1)


@pytest.mark.parametrize("batch,prompt_len,shortlist,budget", [(1, 300, 96, 24), (3, 200, 96, 24),
                                                               (2, 2500, 2048, 512)])
def test_static_cache_and_graph_decode_match_dynamic_cache(batch, prompt_len, shortlist, budget):
    model = _model()
    handle = patch_llama_attention(model, _bundle(shortlist=shortlist, budget=budget), allow_batch=batch > 1)
    prompt = torch.randint(0, 512, (batch, prompt_len), generator=torch.Generator().manual_seed(batch)).cuda()
    steps = 12
    want = _greedy(model, prompt, steps, DynamicCache(config=model.config))
    handle.reset_catalogs()
    static = _greedy(model, prompt, steps, StaticCache(config=model.config, max_cache_len=prompt_len + steps + 4))
    assert torch.equal(static, want)
    handle.reset_catalogs()
    dec = GraphedGreedyDecoder(model, batch, prompt_len + steps + 4)
    graphed = dec.generate(prompt, steps)
    torch.cuda.synchronize()
    dec.release()
    assert torch.equal(graphed, want)
    handle.unpatch()
