"""Model-level cases shared by the fixture generator (reference run) and the GPU tests.

Each case builds a seeded random-init Llama model and artifact bundle on the CPU, then feeds a
fixed token schedule (a prefill followed by single-token decode steps, sharing the KV cache).
"""

from __future__ import annotations

import torch
from transformers import LlamaConfig, LlamaForCausalLM

from tests.golden.inputs import tiny_bundle_tensors, tiny_manifest

CASES = {
    # the reference unit-test geometry (tests/test_sva_llama_adapter.py:11-54)
    "tiny_scan": dict(model="tiny", mode="scan", kw={}, steps=[[1, 2, 3, 4, 5, 6], [7], [8]]),
    "tiny_inverted": dict(model="tiny", mode="inverted",
                          kw=dict(shortlist=4, budget=2, inverted_cells_per_subspace=2, adaptive_min_budget=1,
                                  adaptive_mid_budget=2), steps=[[1, 2, 3, 4], [5], [6], [7]]),
    "tiny_static": dict(model="tiny", mode="inverted_static",
                        kw=dict(shortlist=4, budget=2, inverted_cells_per_subspace=2, static_tail_rebuild_interval=2),
                        steps=[[1, 2, 3, 4], [5], [6], [7], [8]]),
    # SmolLM2-shaped attention (9 query / 3 KV heads, head_dim 64, rank 64, 2x256), 2 layers
    "small_scan": dict(model="small", mode="scan", kw=dict(shortlist=96, budget=24), steps="small"),
    "small_static": dict(model="small", mode="inverted_static",
                         kw=dict(shortlist=96, budget=24, inverted_cells_per_subspace=8,
                                 static_tail_rebuild_interval=3), steps="small"),
}

# The same SmolLM2-shaped attention in bf16 (model weights, activations and KV cache), with
# artifacts holding bf16 values as real bundles do; the adapter runs with its default write path.
# Their fixtures live in golden_models_bf16_v1.npz and are compared within the bf16 tolerance.
BF16_CASES = {
    "small_bf16_scan": dict(model="small_bf16", mode="scan", kw=dict(shortlist=96, budget=24), steps="small"),
    "small_bf16_static": dict(model="small_bf16", mode="inverted_static",
                              kw=dict(shortlist=96, budget=24, inverted_cells_per_subspace=8,
                                      static_tail_rebuild_interval=3), steps="small"),
}


def tiny_model() -> LlamaForCausalLM:
    torch.manual_seed(1234)
    cfg = LlamaConfig(vocab_size=64, hidden_size=16, intermediate_size=32, num_hidden_layers=2, num_attention_heads=2,
                      num_key_value_heads=2, max_position_embeddings=64, rope_theta=10000.0, tie_word_embeddings=False,
                      attn_implementation="eager")
    return LlamaForCausalLM(cfg).eval()


def small_model() -> LlamaForCausalLM:
    torch.manual_seed(4321)
    cfg = LlamaConfig(vocab_size=256, hidden_size=576, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=9, num_key_value_heads=3, head_dim=64, max_position_embeddings=2048,
                      rope_theta=100000.0, rms_norm_eps=1e-5, tie_word_embeddings=True, attn_implementation="eager")
    return LlamaForCausalLM(cfg).eval()


def small_bundle_tensors(seed: int = 77):
    gen = torch.Generator().manual_seed(seed)
    layers = {}
    for layer_idx in range(2):
        layers[layer_idx] = dict(
            q_proj=torch.randn(9, 64, 64, generator=gen) * 0.125,
            k_proj=torch.randn(9, 64, 64, generator=gen) * 0.125,
            logit_scale=torch.randn(9, generator=gen) * 0.2,
            coarse_codebooks=torch.randn(9, 2, 256, 32, generator=gen),
        )
    manifest = {"schema_version": 1, "artifact_type": "summon_verify_attention", "rank_dim": 64,
                "coarse_subspaces": 2, "coarse_codewords": 256, "default_shortlist": 2048, "default_budget": 512,
                "layer_count": 2, "layers": [0, 1]}
    return layers, manifest


def small_steps():
    gen = torch.Generator().manual_seed(99)
    prefill = torch.randint(0, 256, (300,), generator=gen).tolist()
    decode = [[int(x)] for x in torch.randint(0, 256, (4,), generator=gen)]
    return [prefill] + decode


def build(name: str, bundle_cls, layer_cls):
    """Model, bundle (constructed with the given SVAArtifactBundle / SVALayerArtifacts classes)
    and token steps of a case."""
    case = CASES[name] if name in CASES else BF16_CASES[name]
    if case["model"] == "tiny":
        model = tiny_model()
        tensors, manifest = tiny_bundle_tensors(), tiny_manifest()
    elif case["model"] == "small_bf16":
        model = small_model().to(torch.bfloat16)
        tensors, manifest = small_bundle_tensors()
        tensors = {i: {k: v.to(torch.bfloat16) for k, v in t.items()} for i, t in tensors.items()}
    else:
        model = small_model()
        tensors, manifest = small_bundle_tensors()
    layers = {i: layer_cls(train_loss=0.0, hard_loss=0.0, route_source="qk", **t) for i, t in tensors.items()}
    bundle = bundle_cls(manifest=manifest, layers=layers)
    steps = small_steps() if case["steps"] == "small" else case["steps"]
    return model, bundle, steps, case


def run(model, patch_fn, bundle, steps, case, device="cpu"):
    """Run the token schedule through a patched model; returns logits of the last <= 8 positions of
    every step, the stats summary and catalog state of layer 1."""
    from transformers import DynamicCache

    handle = patch_fn(model, bundle, summon_mode=case["mode"], **case["kw"])
    cache = DynamicCache(config=model.config)
    outs = []
    with torch.no_grad():
        for ids in steps:
            x = torch.tensor([ids], device=device)
            o = model(input_ids=x, use_cache=True, past_key_values=cache)
            cache = o.past_key_values
            outs.append(o.logits[0, -8:].float().cpu())
    summary = handle.stats.summary()
    attn = model.model.layers[1].self_attn
    state = dict(key_len=int(attn._cached_key_len), postings_len=int(attn._cached_postings_key_len),
                 codes_shape=tuple(attn._cached_coarse_codes.shape))
    handle.unpatch()
    return outs, summary, state
