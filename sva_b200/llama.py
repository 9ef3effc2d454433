"""Llama-family drop-in attention for Summon-Verify Attention on B200 (reference sva/llama.py).

``patch_llama_attention`` swaps each selected ``LlamaAttention`` of a Hugging Face model for
``SVALlamaAttention`` with the reference's signature, options, error messages and reversible
handle.  What changes is underneath: the key catalog (rank-64 projected keys and uint8 PQ codes)
lives in preallocated device buffers that grow by doubling and are appended in place, posting
lists are built by a GPU counting sort, every summon / rescore / verify runs in the CUDA kernels
of libsva_b200.so, GQA is handled by index arithmetic instead of ``repeat_kv`` copies, and the
per-step counters stay on the device until ``stats.summary()`` reads them.  There is no CPU
path: the patched layers must run on a CUDA device.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from torch import nn
from transformers.cache_utils import Cache, StaticCache
from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

from . import _lib, kernels
from .artifacts import SVAArtifactBundle, SVALayerArtifacts, load_sva_artifact_bundle
from .stats import SVAStats

# Workspace budget per call of the million-key schedule (candidate buffers are 8 B per key per
# (head, token)); prefill over long caches is split into token chunks that fit it.
_GRID_WORKSPACE_BUDGET = 2 << 30
_FUSED_MAX_KEYS = 32768


def _grid_schedule(k_len: int, shortlist: int, budget: int) -> bool:
    """Whether sva_decode runs the million-key (grid) schedule for this cache: over 32768 keys, or
    when one CTA's shared memory cannot hold every key's ADC key with the shortlist and budget
    arrays (the planner's rule, with a slightly larger fixed part so that this never says no where
    the planner says yes; grid calls are split into token chunks)."""
    sl = min(shortlist, k_len)
    b = min(budget, sl)
    return k_len > _FUSED_MAX_KEYS or 4 * k_len + 8 * (sl + b) + 32 * 1024 > 227 * 1024 or k_len > 4096


@dataclass(frozen=True)
class SVALlamaServingConfig:
    """Serving settings for a patched Llama attention module (reference sva/llama.py:22-38)."""

    rank_dim: int
    coarse_shortlist: int
    budget: int
    assign_chunk_size: int = 8192
    query_chunk_size: int | None = None
    summon_mode: str = "scan"
    inverted_cells_per_subspace: int = 8
    adaptive_min_budget: int | None = None
    adaptive_mid_budget: int | None = None
    adaptive_low_margin: float = 0.35
    adaptive_high_margin: float = 0.70
    profile_components: bool = False
    static_tail_rebuild_interval: int = 64
    # Not in the reference: "exact" (the default) projects keys on CUDA cores in the canonical fp32
    # order, so k_low and the codes are bit-exact; "auto" projects them on the tensor cores
    # (tcgen05) when the keys are bf16 and the key projection holds bf16 values, which changes the
    # fp32 summation order, so k_low may differ by a few ulp and codes may flip at near ties.
    write_path: str = "exact"
    # Not in the reference, which raises on batch != 1 (sva/llama.py:182-183): with allow_batch the
    # scan summon decodes every sequence of a batch in one sva_decode_batched call, each
    # sequence exactly as a batch-1 call would.  Off by default, keeping the reference's error.
    allow_batch: bool = False


class SVALlamaAttention(nn.Module):
    """Drop-in replacement for a Llama attention layer using frozen SVA artifacts."""

    def __init__(self, original: nn.Module, layer_artifacts: SVALayerArtifacts, serving: SVALlamaServingConfig,
                 stats: SVAStats | None = None) -> None:
        super().__init__()
        self.original = original
        self.config = original.config
        self.layer_idx = original.layer_idx
        self.head_dim = original.head_dim
        self.num_key_value_groups = original.num_key_value_groups
        self.scaling = original.scaling
        self.attention_dropout = original.attention_dropout
        self.q_proj = original.q_proj
        self.k_proj = original.k_proj
        self.v_proj = original.v_proj
        self.o_proj = original.o_proj
        self.serving = serving
        self.stats = stats
        self.register_buffer("sva_q_proj", layer_artifacts.q_proj.detach().float().clone(), persistent=False)
        self.register_buffer("sva_k_proj", layer_artifacts.k_proj.detach().float().clone(), persistent=False)
        self.register_buffer("sva_logit_scale", layer_artifacts.logit_scale.detach().float().clone(), persistent=False)
        # computed on the host, where the reference computes it for bundles loaded to the CPU
        scale = layer_artifacts.logit_scale.detach().float().cpu().exp().clamp(0.01, 100.0)
        self.register_buffer("sva_scale", scale.to(layer_artifacts.logit_scale.device), persistent=False)
        self.register_buffer("sva_coarse_codebooks", layer_artifacts.coarse_codebooks.detach().float().clone(),
                             persistent=False)
        self.reset_catalog()

    # ------------------------------------------------------------------------------------
    # catalog state (views keep the reference's attribute names and shapes)
    # ------------------------------------------------------------------------------------
    def reset_catalog(self) -> None:
        self._k_low_buf: torch.Tensor | None = None   # [H, cap, R] fp32
        self._codes_buf: torch.Tensor | None = None   # [H, cap, S] uint8
        self._postings: kernels.Postings | None = None
        self._post_bound = 0
        self._codes_len = 0
        self._cached_postings_key_len = 0
        self._cached_key_len = 0
        self._cached_signature: tuple | None = None
        self._tc_write_key: tuple | None = None
        self._tc_write = False
        self._static_sig = None  # static-cache catalog (sva_attention_static), sized by the cache
        # batched catalog (allow_batch): [B, H, cap, R] fp32 / [B, H, cap, S] uint8
        self._bk_low: torch.Tensor | None = None
        self._bcodes: torch.Tensor | None = None
        self._bkey_len = 0
        self._bsignature: tuple | None = None
        self._brep: tuple | None = None

    @property
    def _cached_k_low(self) -> torch.Tensor | None:
        if self._k_low_buf is None:
            return None
        return self._k_low_buf[:, : self._cached_key_len].unsqueeze(0)

    @property
    def _cached_coarse_codes(self) -> torch.Tensor | None:
        if self._codes_buf is None:
            return None
        return self._codes_buf[:, : self._codes_len]

    @property
    def _cached_postings(self) -> torch.Tensor | None:
        return None if self._postings is None else self._postings.ids

    @property
    def _cached_posting_counts(self) -> torch.Tensor | None:
        return None if self._postings is None else self._postings.counts

    @staticmethod
    def _top_unique_candidates(candidate_idx: torch.Tensor, candidate_scores: torch.Tensor,
                               candidate_valid: torch.Tensor, budget: int, refill_factor: int = 2):
        """Refill-and-dedupe selection (reference sva/llama.py:83-116) on the GPU."""
        return kernels.top_unique(candidate_idx, candidate_scores, candidate_valid, budget, refill_factor)

    # ------------------------------------------------------------------------------------
    def forward(self, hidden_states: torch.Tensor, position_embeddings: tuple[torch.Tensor, torch.Tensor] | None = None,
                attention_mask: torch.Tensor | None = None, past_key_values: Cache | None = None,
                **kwargs: Any) -> tuple[torch.Tensor, None]:
        attn_output, weights = self.forward_attention(hidden_states, position_embeddings, attention_mask,
                                                      past_key_values, **kwargs)
        return self.o_proj(attn_output), weights

    def forward_attention(self, hidden_states: torch.Tensor,
                          position_embeddings: tuple[torch.Tensor, torch.Tensor] | None = None,
                          attention_mask: torch.Tensor | None = None, past_key_values: Cache | None = None,
                          **kwargs: Any) -> tuple[torch.Tensor, None]:
        """forward without the final o_proj: the attention output [B, q, H * D] (the residual
        adapter fuses o_proj into its own kernel)."""
        if self.training:
            raise RuntimeError("SVA Llama adapter is inference-only. Call model.eval() before running it.")
        if kwargs.get("output_attentions"):
            raise RuntimeError("SVA Llama adapter does not materialize dense attention weights.")
        if position_embeddings is None:
            raise ValueError("SVA Llama adapter requires model-provided RoPE position embeddings.")
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, self.head_dim)
        query_states = self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        key_states = self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        value_states = self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
        cos, sin = position_embeddings
        query_states, key_states = apply_rotary_pos_emb(query_states, key_states, cos, sin)
        if past_key_values is not None:
            key_states, value_states = past_key_values.update(key_states, value_states, self.layer_idx)
        position_ids = kwargs.get("position_ids")
        if isinstance(past_key_values, StaticCache) and position_ids is not None:
            attn_output = self.sva_attention_static(query_states, key_states, value_states, position_ids)
        else:
            attn_output = self.sva_attention(query_states, key_states, value_states, attention_mask)
        attn_output = attn_output.transpose(1, 2).contiguous().reshape(*input_shape, -1)
        return attn_output, None

    # ------------------------------------------------------------------------------------
    def sva_attention(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                      attention_mask: torch.Tensor | None) -> torch.Tensor:
        """query [1, H, q, D]; key/value [1, Hkv, L, D] (not repeated) -> [1, H, q, D]."""
        batch, n_heads, q_len, head_dim = query.shape
        k_len = int(key.shape[2])
        if batch != 1:
            if not self.serving.allow_batch:
                raise ValueError("SVA Llama adapter currently expects batch size 1.")
            return self._sva_attention_batched(query, key, value, attention_mask)
        if query.device.type != "cuda":
            raise RuntimeError("The B200 SVA adapter runs on CUDA devices only; move the model to a GPU.")
        mode = self.serving.summon_mode
        if mode not in {"scan", "inverted", "inverted_static"}:
            raise ValueError(f"Unknown SVA summon_mode: {mode!r}")
        dev = query.device
        keys = key[0]
        values = value[0]
        if keys.stride(-1) != 1:
            keys = keys.contiguous()
        if values.stride(-1) != 1:
            values = values.contiguous()
        allowed_mask = None
        if attention_mask is not None:
            allowed_mask = (attention_mask[..., :q_len, :k_len] > -1e4)
            allowed_mask = allowed_mask.reshape(-1, q_len, k_len)[0].to(torch.uint8).contiguous()

        profile = self.serving.profile_components and mode == "inverted_static" and q_len == 1
        ev = _Timer(dev) if profile else None
        if ev:
            ev.mark("start")
        self._key_catalog(keys, q_len)
        if ev:
            ev.mark("catalog")
        counters = None if self.stats is None else self.stats.device_counters(int(self.layer_idx or 0), dev)
        shortlist = min(self.serving.coarse_shortlist, k_len)
        budget = min(self.serving.budget, shortlist)
        k_low = self._k_low_buf[:, :k_len]

        if q_len == 1 and mode in {"inverted", "inverted_static"}:
            max_budget = min(budget, k_len)
            min_budget = min(self.serving.adaptive_min_budget or max_budget, max_budget, k_len)
            mid_budget = min(self.serving.adaptive_mid_budget or max(min_budget, max_budget // 2), max_budget, k_len)
            prof_events = ev.kernel_events(4) if ev else None
            try:
                out = kernels.decode_inverted(
                    query[0, :, 0, :], self.sva_q_proj, self.sva_scale, self.sva_coarse_codebooks, self._codes_buf,
                    self._postings, k_low, keys, values, max_budget, self.serving.inverted_cells_per_subspace,
                    min_budget, mid_budget, low_margin=self.serving.adaptive_low_margin,
                    high_margin=self.serving.adaptive_high_margin, dynamic=(mode == "inverted"),
                    allowed_mask=None if allowed_mask is None else allowed_mask[0], softmax_scale=self.scaling,
                    stats=counters)
            finally:
                if ev:
                    ev.release_kernel_events()
            if ev:
                ev.mark("total")
                self._record_profile(ev, prof_events)
            return out[None, :, None, :]

        out = torch.empty(n_heads, q_len, head_dim, dtype=query.dtype, device=dev)
        q = query[0]
        chunk = q_len
        if _grid_schedule(k_len, self.serving.coarse_shortlist, self.serving.budget):
            chunk = max(1, min(q_len, _GRID_WORKSPACE_BUDGET // max(1, n_heads * k_len * 8), 65535 // n_heads))
        if self.serving.query_chunk_size:
            chunk = min(chunk, int(self.serving.query_chunk_size))
        for t0 in range(0, q_len, chunk):
            t1 = min(q_len, t0 + chunk)
            if allowed_mask is None:
                # no mask: token t may attend to keys [0, k_len - q_len + t + 1) (sva/llama.py:191-198)
                allowed_len = torch.arange(k_len - q_len + t0 + 1, k_len - q_len + t1 + 1, device=dev,
                                           dtype=torch.int64)
            else:
                # with a mask the reference uses the mask alone (sva/llama.py:188-190)
                allowed_len = torch.full((t1 - t0,), k_len, device=dev, dtype=torch.int64)
            kernels.decode(q[:, t0:t1], self.sva_q_proj, self.sva_scale, self.sva_coarse_codebooks,
                           self._codes_buf[:, :k_len], k_low, keys, values, self.serving.coarse_shortlist,
                           self.serving.budget, softmax_scale=self.scaling, logits_mode=1, allowed_len=allowed_len,
                           allowed_mask=None if allowed_mask is None else allowed_mask[t0:t1],
                           out=out[:, t0:t1], stats=counters)
        return out.unsqueeze(0)

    # ------------------------------------------------------------------------------------
    def sva_attention_static(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                             position_ids: torch.Tensor) -> torch.Tensor:
        """The scan summon over a Hugging Face ``StaticCache`` (not in the reference, which runs
        on growing caches).  key / value are the cache's full [B, Hkv, max_len, D] buffers, of
        which the rows before position_ids[0, -1] + 1 are filled; the batch is taken to be
        unpadded, so the attention mask is not consulted.  A single-token step reads its position
        and the valid length from device memory (sva_catalog_encode_at, sva_decode_batched with
        device lengths), so the whole model step can be captured in a CUDA graph and replayed;
        every token gets exactly the result of the growing-cache path."""
        batch, n_heads, q_len, head_dim = query.shape
        max_len = int(key.shape[2])
        if query.device.type != "cuda":
            raise RuntimeError("The B200 SVA adapter runs on CUDA devices only; move the model to a GPU.")
        if self.serving.summon_mode != "scan":
            raise ValueError("The static-cache SVA path supports summon_mode='scan' only.")
        if batch != 1 and not self.serving.allow_batch:
            raise ValueError("SVA Llama adapter currently expects batch size 1.")
        dev = query.device
        rank = self.serving.rank_dim
        subspaces = int(self.sva_coarse_codebooks.shape[1])
        sig = (dev, key.dtype, batch, max_len, key.data_ptr())
        if getattr(self, "_static_sig", None) != sig:
            # buffers sized for the whole cache, allocated before any capture (at the prefill)
            self._sk_low = torch.zeros(batch, n_heads, max_len, rank, dtype=torch.float32, device=dev)
            self._scodes = torch.zeros(batch, n_heads, max_len, subspaces, dtype=torch.uint8, device=dev)
            self._srep = (self.sva_k_proj.to(dev).repeat(batch, 1, 1).contiguous(),
                          self.sva_coarse_codebooks.to(dev).repeat(batch, 1, 1, 1).contiguous())
            self._static_sig = sig
        n_kv = int(key.shape[1])
        flat_keys = key.view(batch * n_kv, max_len, head_dim)
        flat_low = self._sk_low.view(batch * n_heads, max_len, rank)
        flat_codes = self._scodes.view(batch * n_heads, max_len, subspaces)
        counters = None if self.stats is None else self.stats.device_counters(int(self.layer_idx or 0), dev)
        pos = position_ids.reshape(-1, q_len)[0]
        if q_len == 1:
            start = pos.to(torch.int64)
            kernels.catalog_encode_at(flat_keys, self._srep[0], self._srep[1], start, 1, max_len, flat_low, flat_codes,
                                      n_heads=batch * n_heads)
            seq_lens = (start + 1).expand(batch).contiguous()
            return kernels.decode_batched(query, self.sva_q_proj, self.sva_scale, self.sva_coarse_codebooks,
                                          self._scodes, self._sk_low, key, value, self.serving.coarse_shortlist,
                                          self.serving.budget, seq_lens=seq_lens, max_len=max_len,
                                          softmax_scale=self.scaling, logits_mode=1, stats=counters)
        # prefill (not captured): positions and lengths on the host
        first, last = int(pos[0]), int(pos[-1])
        k_len = last + 1
        kernels.catalog_encode(flat_keys, self._srep[0], self._srep[1], first, k_len - first, flat_low, flat_codes,
                               n_heads=batch * n_heads)
        out = torch.empty(batch, n_heads, q_len, head_dim, dtype=query.dtype, device=dev)
        chunk = q_len
        if _grid_schedule(k_len, self.serving.coarse_shortlist, self.serving.budget):
            chunk = max(1, min(q_len, _GRID_WORKSPACE_BUDGET // max(1, batch * n_heads * k_len * 8),
                               65535 // (batch * n_heads)))
        if self.serving.query_chunk_size:
            chunk = min(chunk, int(self.serving.query_chunk_size))
        for t0 in range(0, q_len, chunk):
            t1 = min(q_len, t0 + chunk)
            allowed_len = (pos[t0:t1].to(torch.int64) + 1).expand(batch, t1 - t0).contiguous()
            kernels.decode_batched(query[:, :, t0:t1], self.sva_q_proj, self.sva_scale, self.sva_coarse_codebooks,
                                   self._scodes, self._sk_low, key, value, self.serving.coarse_shortlist,
                                   self.serving.budget, max_len=k_len, softmax_scale=self.scaling, logits_mode=1,
                                   allowed_len=allowed_len, out=out[:, :, t0:t1], stats=counters)
        return out

    # ------------------------------------------------------------------------------------
    def _sva_attention_batched(self, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                               attention_mask: torch.Tensor | None) -> torch.Tensor:
        """query [B, H, q, D]; key/value [B, Hkv, L, D] -> [B, H, q, D]: the scan summon of every
        sequence in one call (allow_batch).  Each sequence gets exactly what a batch-1 call of the
        reference would compute for it (sva/llama.py:171-328)."""
        batch, n_heads, q_len, head_dim = query.shape
        k_len = int(key.shape[2])
        if query.device.type != "cuda":
            raise RuntimeError("The B200 SVA adapter runs on CUDA devices only; move the model to a GPU.")
        mode = self.serving.summon_mode
        if mode not in {"scan", "inverted", "inverted_static"}:
            raise ValueError(f"Unknown SVA summon_mode: {mode!r}")
        if mode != "scan":
            raise ValueError("Batched SVA decode supports summon_mode='scan' only; run inverted modes at batch 1.")
        dev = query.device
        if key.stride(-1) != 1:
            key = key.contiguous()
        if value.stride(-1) != 1:
            value = value.contiguous()
        self._key_catalog_batched(key, q_len)
        allowed_mask = None
        if attention_mask is not None:
            m = attention_mask[..., :q_len, :k_len] > -1e4
            allowed_mask = m.expand(batch, 1, q_len, k_len).reshape(batch * q_len, k_len).to(torch.uint8).contiguous()
        counters = None if self.stats is None else self.stats.device_counters(int(self.layer_idx or 0), dev)
        out = torch.empty(batch, n_heads, q_len, head_dim, dtype=query.dtype, device=dev)
        chunk = q_len
        if _grid_schedule(k_len, self.serving.coarse_shortlist, self.serving.budget):
            chunk = max(1, min(q_len, _GRID_WORKSPACE_BUDGET // max(1, batch * n_heads * k_len * 8),
                               65535 // (batch * n_heads)))
        if self.serving.query_chunk_size:
            chunk = min(chunk, int(self.serving.query_chunk_size))
        for t0 in range(0, q_len, chunk):
            t1 = min(q_len, t0 + chunk)
            if allowed_mask is None:
                lens = torch.arange(k_len - q_len + t0 + 1, k_len - q_len + t1 + 1, device=dev, dtype=torch.int64)
                allowed_len = lens.expand(batch, t1 - t0).contiguous()
                mask = None
            else:
                allowed_len = torch.full((batch, t1 - t0), k_len, device=dev, dtype=torch.int64)
                mask = allowed_mask.view(batch, q_len, k_len)[:, t0:t1].reshape(batch * (t1 - t0), k_len)
            kernels.decode_batched(query[:, :, t0:t1], self.sva_q_proj, self.sva_scale, self.sva_coarse_codebooks,
                                   self._bcodes, self._bk_low, key, value, self.serving.coarse_shortlist,
                                   self.serving.budget, max_len=k_len, softmax_scale=self.scaling, logits_mode=1,
                                   allowed_len=allowed_len, allowed_mask=mask, out=out[:, :, t0:t1], stats=counters)
        return out

    def _key_catalog_batched(self, keys: torch.Tensor, q_len: int) -> None:
        """The batched catalog [B, H, cap, ...]: new keys of every sequence are projected and coded
        in place (one catalog_encode call over the B * H flattened heads)."""
        batch, n_kv, k_len, head_dim = keys.shape
        n_heads = int(self.sva_q_proj.shape[0])
        signature = (keys.device, keys.dtype, batch, n_heads, head_dim)
        can_append = (self._bsignature == signature and self._bk_low is not None and self._bkey_len > 0
                      and k_len > self._bkey_len and k_len - self._bkey_len <= max(q_len, 1) and q_len < k_len)
        start = self._bkey_len if can_append else 0
        cap = 0 if self._bk_low is None else int(self._bk_low.shape[2])
        rank = self.serving.rank_dim
        subspaces = int(self.sva_coarse_codebooks.shape[1])
        if self._bsignature != signature or cap < k_len:
            new_cap = (max(k_len, 2 * cap if self._bsignature == signature else 0, 256) + 255) // 256 * 256
            k_low = torch.empty(batch, n_heads, new_cap, rank, dtype=torch.float32, device=keys.device)
            codes = torch.zeros(batch, n_heads, new_cap, subspaces, dtype=torch.uint8, device=keys.device)
            if can_append:
                k_low[:, :, :start] = self._bk_low[:, :, :start]
                codes[:, :, :start] = self._bcodes[:, :, :start]
            self._bk_low, self._bcodes = k_low, codes
        if self._brep is None or self._brep[0] != batch or self._brep[1].device != keys.device:
            self._brep = (batch, self.sva_k_proj.to(keys.device).repeat(batch, 1, 1).contiguous(),
                          self.sva_coarse_codebooks.to(keys.device).repeat(batch, 1, 1, 1).contiguous())
        flat_keys = keys.reshape(batch * n_kv, k_len, head_dim) if keys.is_contiguous() else keys.contiguous().view(
            batch * n_kv, k_len, head_dim)
        cap = int(self._bk_low.shape[2])
        kernels.catalog_encode(flat_keys, self._brep[1], self._brep[2], start, k_len - start,
                               self._bk_low.view(batch * n_heads, cap, rank),
                               self._bcodes.view(batch * n_heads, cap, subspaces), n_heads=batch * n_heads,
                               tensor_cores=self._tensor_core_write(flat_keys))
        self._bkey_len = k_len
        self._bsignature = signature

    # ------------------------------------------------------------------------------------
    def _ensure_capacity(self, n_heads: int, needed: int, device: torch.device) -> None:
        rank = self.serving.rank_dim
        subspaces = int(self.sva_coarse_codebooks.shape[1])
        cap = 0 if self._k_low_buf is None else int(self._k_low_buf.shape[1])
        if self._k_low_buf is not None and self._k_low_buf.device == device and cap >= needed:
            return
        new_cap = max(needed, 2 * cap, 256)
        new_cap = (new_cap + 255) // 256 * 256
        k_low = torch.empty(n_heads, new_cap, rank, dtype=torch.float32, device=device)
        codes = torch.zeros(n_heads, new_cap, subspaces, dtype=torch.uint8, device=device)
        if self._k_low_buf is not None and self._k_low_buf.device == device and self._cached_key_len > 0:
            k_low[:, : self._cached_key_len] = self._k_low_buf[:, : self._cached_key_len]
            codes[:, : self._cached_key_len] = self._codes_buf[:, : self._cached_key_len]
        self._k_low_buf, self._codes_buf = k_low, codes

    def _rebuild_postings(self, key_len: int) -> None:
        self._postings = kernels.postings_build(self._codes_buf, int(self.sva_coarse_codebooks.shape[2]), key_len=key_len)
        self._cached_postings_key_len = key_len

    def _append_postings(self, start: int, count: int) -> None:
        """Dynamic inverted mode: append the new keys' ids to their cells (reference
        sva/llama.py:659-693) instead of rebuilding every list.  The lists use the padded layout;
        the host keeps an upper bound of the largest list (its size at the last rebuild plus the
        keys appended since), and rebuilds with twice the room when the bound reaches the cell
        size, so appends never overflow and cost O(new keys) between rebuilds."""
        post = self._postings
        if post is None or post.cap is None or self._post_bound + count > post.cap:
            self._postings = kernels.postings_padded(self._codes_buf, int(self.sva_coarse_codebooks.shape[2]),
                                                     start + count)
            self._post_bound = self._postings.largest_at_build  # one host read per rebuild
        else:
            kernels.postings_append(self._codes_buf, post, start, count)
            self._post_bound += count
        self._cached_postings_key_len = start + count

    def _tensor_core_write(self, keys: torch.Tensor) -> bool:
        """Whether new keys go through the tcgen05 projection (serving option ``write_path``)."""
        if self.serving.write_path == "exact":
            return False
        if self.serving.write_path != "auto":
            raise ValueError(f"Unknown write_path {self.serving.write_path!r}; expected 'auto' or 'exact'.")
        key = (keys.device, keys.dtype, keys.data_ptr() % 16, keys.stride(-2), keys.stride(0))
        if self._tc_write_key != key:
            self._tc_write_key = key
            self._tc_write = kernels.tensor_core_write_ok(keys, self.sva_k_proj.to(keys.device))
        return self._tc_write

    def _key_catalog(self, keys: torch.Tensor, q_len: int) -> None:
        """Keep the device catalog in step with the cache (reference sva/llama.py:578-624).

        Keys [Hkv, L, D].  New keys are projected and coded in place; the visible code length and
        the posting-list rebuilds follow the reference's rules per summon mode.
        """
        n_kv, k_len, head_dim = keys.shape
        n_heads = int(self.sva_q_proj.shape[0])
        mode = self.serving.summon_mode
        signature = (keys.device, keys.dtype, n_heads, head_dim, self.serving.rank_dim)
        can_append = (self._cached_signature == signature and self._k_low_buf is not None and self._cached_key_len > 0
                      and k_len > self._cached_key_len and k_len - self._cached_key_len <= max(q_len, 1)
                      and q_len < k_len)
        start = self._cached_key_len if can_append else 0
        self._ensure_capacity(n_heads, k_len, keys.device)
        kernels.catalog_encode(keys, self.sva_k_proj, self.sva_coarse_codebooks, start, k_len - start, self._k_low_buf,
                               self._codes_buf, n_heads=n_heads, tensor_cores=self._tensor_core_write(keys))
        if can_append:
            if mode == "inverted":
                self._codes_len = k_len
                self._append_postings(start, k_len - start)
            elif mode == "inverted_static" and q_len == 1:
                interval = max(1, int(self.serving.static_tail_rebuild_interval))
                if self._postings is None or k_len - self._cached_postings_key_len >= interval:
                    self._codes_len = k_len
                    self._rebuild_postings(k_len)
            else:
                self._codes_len = k_len
        else:
            self._codes_len = k_len
            if mode in {"inverted", "inverted_static"}:
                self._rebuild_postings(k_len)
        self._cached_key_len = k_len
        self._cached_signature = signature

    def _record_profile(self, ev: "_Timer", kernel_events) -> None:
        if self.stats is None:
            return
        t = ev.elapsed()
        k = ev.kernel_elapsed(kernel_events)
        self.stats.add(int(self.layer_idx or 0), {
            "profile_calls": 1.0,
            "profile_outer_calls": 1.0,
            # q_low is computed inside the prep kernel, so the projection stage is part of catalog
            "static_projection_ms": 0.0,
            "static_key_catalog_ms": t["catalog"],
            "static_catalog_ms": k[0] + k[1],
            "static_refill_ms": k[2],
            # budget, gather, exact score and aggregation run fused in the final kernel
            "static_budget_ms": 0.0,
            "static_gather_ms": 0.0,
            "static_exact_score_ms": 0.0,
            "static_aggregate_ms": k[3],
            "static_total_ms": sum(k),
            "static_outer_total_ms": t["catalog"] + t["total"],
        })


class _Timer:
    """CUDA-event stage timing for profile_components (replaces the reference's synchronize +
    perf_counter pairs, sva/llama.py:118-128); reading the times synchronises once."""

    def __init__(self, device: torch.device):
        self.device = device
        self.events: list[tuple[str, torch.cuda.Event]] = []
        self._handles = None

    def mark(self, name: str) -> None:
        e = torch.cuda.Event(enable_timing=True)
        e.record(torch.cuda.current_stream(self.device))
        self.events.append((name, e))

    def kernel_events(self, n: int):
        import ctypes

        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
        for e in evs:
            e.record(torch.cuda.current_stream(self.device))
        self._handles = (ctypes.c_void_p * n)(*[e.cuda_event for e in evs[1:]])
        _lib.load().sva_profile_events(self._handles, n)
        evs[0].record(torch.cuda.current_stream(self.device))
        return evs

    def release_kernel_events(self) -> None:
        _lib.load().sva_profile_events(None, 0)

    def elapsed(self) -> dict[str, float]:
        self.events[-1][1].synchronize()
        out = {}
        for (_, a), (name, b) in zip(self.events, self.events[1:]):
            out[name] = a.elapsed_time(b)
        return out

    @staticmethod
    def kernel_elapsed(evs) -> list[float]:
        evs[-1].synchronize()
        return [evs[i].elapsed_time(evs[i + 1]) for i in range(len(evs) - 1)]


class SVALlamaPatcher:
    """Reversible patch handle for Llama-family Hugging Face models (reference sva/llama.py:696-805)."""

    def __init__(self, model: nn.Module, bundle: SVAArtifactBundle, shortlist: int | None = None,
                 budget: int | None = None, assign_chunk_size: int = 8192, query_chunk_size: int | None = None,
                 summon_mode: str = "scan", inverted_cells_per_subspace: int = 8,
                 adaptive_min_budget: int | None = None, adaptive_mid_budget: int | None = None,
                 adaptive_low_margin: float = 0.35, adaptive_high_margin: float = 0.70,
                 profile_components: bool = False, static_tail_rebuild_interval: int = 64,
                 layers: list[int] | None = None, write_path: str = "exact", allow_batch: bool = False) -> None:
        self.model = model
        self.bundle = bundle
        self.stats = SVAStats()
        self.originals: dict[int, nn.Module] = {}
        self.layers = None if layers is None else list(dict.fromkeys(int(i) for i in layers))
        self.serving = SVALlamaServingConfig(
            rank_dim=bundle.rank_dim,
            coarse_shortlist=bundle.default_shortlist if shortlist is None else int(shortlist),
            budget=bundle.default_budget if budget is None else int(budget),
            assign_chunk_size=assign_chunk_size,
            query_chunk_size=query_chunk_size,
            summon_mode=summon_mode,
            inverted_cells_per_subspace=inverted_cells_per_subspace,
            adaptive_min_budget=adaptive_min_budget,
            adaptive_mid_budget=adaptive_mid_budget,
            adaptive_low_margin=adaptive_low_margin,
            adaptive_high_margin=adaptive_high_margin,
            profile_components=profile_components,
            static_tail_rebuild_interval=static_tail_rebuild_interval,
            write_path=write_path,
            allow_batch=allow_batch,
        )

    def patch(self) -> "SVALlamaPatcher":
        model_layers = getattr(getattr(self.model, "model", None), "layers", None)
        if model_layers is None:
            raise ValueError("Expected a Hugging Face Llama-style model with model.layers.")
        if self.originals:
            return self
        if self.bundle.layer_count != len(model_layers):
            raise ValueError(f"Artifact has {self.bundle.layer_count} layers but model has {len(model_layers)}.")
        model_id = self.bundle.model_id
        model_name = getattr(getattr(self.model, "config", None), "_name_or_path", None)
        if model_id and model_name and str(model_name) not in {"", model_id}:
            raise ValueError(f"Artifact model_id={model_id!r} does not match loaded model {model_name!r}.")
        patch_layers = self.layers if self.layers is not None else list(range(len(model_layers)))
        for layer_idx in patch_layers:
            if layer_idx < 0 or layer_idx >= len(model_layers):
                raise ValueError(f"Patch layer index {layer_idx} is outside model layer range 0..{len(model_layers) - 1}.")
            layer = model_layers[layer_idx]
            artifacts = self.bundle.layers.get(layer_idx)
            if artifacts is None:
                raise ValueError(f"Missing SVA artifacts for layer {layer_idx}.")
            self._validate_layer_shapes(layer_idx, layer.self_attn, artifacts)
            self.originals[layer_idx] = layer.self_attn
            replacement = SVALlamaAttention(layer.self_attn, artifacts, self.serving, self.stats)
            try:
                device = next(layer.self_attn.parameters()).device
            except StopIteration:
                device = artifacts.q_proj.device
            replacement.to(device=device)
            replacement.train(layer.self_attn.training)
            layer.self_attn = replacement
        return self

    def unpatch(self) -> None:
        layers = self.model.model.layers
        for layer_idx, original in self.originals.items():
            layers[layer_idx].self_attn = original
        self.originals.clear()

    def reset_stats(self) -> None:
        self.stats.reset()

    def reset_catalogs(self) -> None:
        for layer in self.model.model.layers:
            attention = self._unwrap_sva_attention(layer.self_attn)
            if isinstance(attention, SVALlamaAttention):
                attention.reset_catalog()

    def _unwrap_sva_attention(self, attention: nn.Module) -> nn.Module:
        while hasattr(attention, "sva_attn"):
            attention = getattr(attention, "sva_attn")
        return attention

    def __enter__(self) -> "SVALlamaPatcher":
        return self.patch()

    def __exit__(self, exc_type: object, exc: object, traceback: object) -> None:
        self.unpatch()

    def _validate_layer_shapes(self, layer_idx: int, attention: nn.Module, artifacts: SVALayerArtifacts) -> None:
        n_heads = int(attention.config.num_attention_heads)
        head_dim = int(attention.head_dim)
        expected = (n_heads, head_dim, self.bundle.rank_dim)
        if tuple(artifacts.q_proj.shape) != expected:
            raise ValueError(f"Layer {layer_idx} artifact q_proj shape {tuple(artifacts.q_proj.shape)} != {expected}.")
        if tuple(artifacts.k_proj.shape) != expected:
            raise ValueError(f"Layer {layer_idx} artifact k_proj shape {tuple(artifacts.k_proj.shape)} != {expected}.")


def patch_llama_attention(model: nn.Module, artifact_dir_or_bundle: str | Path | SVAArtifactBundle,
                          shortlist: int | None = None, budget: int | None = None, assign_chunk_size: int = 8192,
                          query_chunk_size: int | None = None, summon_mode: str = "scan",
                          inverted_cells_per_subspace: int = 8, adaptive_min_budget: int | None = None,
                          adaptive_mid_budget: int | None = None, adaptive_low_margin: float = 0.35,
                          adaptive_high_margin: float = 0.70, profile_components: bool = False,
                          static_tail_rebuild_interval: int = 64, layers: list[int] | None = None,
                          write_path: str = "exact", allow_batch: bool = False) -> SVALlamaPatcher:
    """Patch a Llama-family model with SVA attention and return a reversible handle (reference sva/llama.py:808-848).

    ``write_path`` (not in the reference) selects the key projection: "exact" (default; CUDA cores,
    canonical fp32 order, bit-exact codes) or "auto" (tcgen05 tensor cores when the keys are bf16
    and the projection holds bf16 values; codes may flip at near ties).  ``allow_batch`` (not in the
    reference, which raises on batch != 1) decodes batches of sequences in one call per layer in
    scan mode, each sequence exactly as at batch 1.
    """
    bundle = (artifact_dir_or_bundle if isinstance(artifact_dir_or_bundle, SVAArtifactBundle)
              else load_sva_artifact_bundle(artifact_dir_or_bundle))
    return SVALlamaPatcher(
        model=model, bundle=bundle, shortlist=shortlist, budget=budget, assign_chunk_size=assign_chunk_size,
        query_chunk_size=query_chunk_size, summon_mode=summon_mode,
        inverted_cells_per_subspace=inverted_cells_per_subspace, adaptive_min_budget=adaptive_min_budget,
        adaptive_mid_budget=adaptive_mid_budget, adaptive_low_margin=adaptive_low_margin,
        adaptive_high_margin=adaptive_high_margin, profile_components=profile_components,
        static_tail_rebuild_interval=static_tail_rebuild_interval, layers=layers, write_path=write_path,
        allow_batch=allow_batch,
    ).patch()
