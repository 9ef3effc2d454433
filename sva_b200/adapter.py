"""Residual output adapter for the late-layer SVA socket, with o_proj fused in on the GPU.

Mirrors ``SVAResidualOutputAdapter`` of the reference (experiments/sva_late4_logit_distill.py:37-51)
and its wrapping helper (:164-174): the adapter wraps a patched attention layer and adds a
low-rank correction computed from the layer's input hidden states and the attention output:

    out = o + (up(gelu(down(cat[hidden.float(), o.float()]))) * scale).to(o.dtype)

where o is the wrapped layer's output (its o_proj applied to the attention).  When the wrapped
layer is an ``SVALlamaAttention`` and a step has at most ``fused_max_rows`` token rows (decode),
the o_proj GEMV and the whole adapter run as one clustered CUDA kernel (sva_adapter_forward);
prefill-sized steps use the same composition with torch's GEMMs on the GPU.  The patcher's
``_unwrap_sva_attention`` follows ``.sva_attn`` as the reference's does.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib, kernels


class SVAResidualOutputAdapter(nn.Module):
    fused_max_rows = 64

    def __init__(self, sva_attn: nn.Module, hidden_size: int, rank: int, scale: float) -> None:
        super().__init__()
        self.sva_attn = sva_attn
        self.scale = scale
        self.down = nn.Linear(hidden_size * 2, rank, bias=False, dtype=torch.float32)
        self.up = nn.Linear(rank, hidden_size, bias=False, dtype=torch.float32)
        nn.init.normal_(self.down.weight, mean=0.0, std=0.02)
        nn.init.zeros_(self.up.weight)

    def forward(self, hidden_states: torch.Tensor, *args, **kwargs) -> tuple[torch.Tensor, None]:
        from .llama import SVALlamaAttention

        attn = self.sva_attn
        rows = hidden_states.numel() // hidden_states.shape[-1]
        if isinstance(attn, SVALlamaAttention) and hidden_states.is_cuda and rows <= self.fused_max_rows:
            pre, weights = attn.forward_attention(hidden_states, *args, **kwargs)
            return self.fused(hidden_states, pre, attn.o_proj), weights
        attn_output, attn_weights = attn(hidden_states, *args, **kwargs)
        adapter_input = torch.cat([hidden_states.float(), attn_output.float()], dim=-1)
        correction = self.up(F.gelu(self.down(adapter_input))) * self.scale
        return attn_output + correction.to(dtype=attn_output.dtype), attn_weights

    def fused(self, hidden_states: torch.Tensor, attn_pre: torch.Tensor, o_proj: nn.Linear) -> torch.Tensor:
        """o_proj(attn_pre) and the adapter in one kernel (rows = tokens of the step)."""
        hidden_size = hidden_states.shape[-1]
        h2 = hidden_states.reshape(-1, hidden_size)
        a2 = attn_pre.reshape(-1, attn_pre.shape[-1])
        if h2.stride(-1) != 1:
            h2 = h2.contiguous()
        if a2.stride(-1) != 1:
            a2 = a2.contiguous()
        w = o_proj.weight
        if w.dtype != h2.dtype or a2.dtype != h2.dtype:
            raise TypeError("fused adapter: hidden states, attention output and o_proj must share a dtype")
        bias = o_proj.bias
        out = torch.empty(h2.shape[0], w.shape[0], dtype=h2.dtype, device=h2.device)
        down = self.down.weight.float().contiguous()
        up = self.up.weight.float().contiguous()
        rc = _lib.load().sva_adapter_forward(
            h2.data_ptr(), h2.stride(0), a2.data_ptr(), a2.stride(0), kernels.dtype_code(h2.dtype),
            w.contiguous().data_ptr(), None if bias is None else bias.data_ptr(), down.data_ptr(), up.data_ptr(),
            float(self.scale), h2.shape[0], w.shape[0], w.shape[1], down.shape[0], out.data_ptr(), out.stride(0),
            kernels._stream(h2.device))
        _lib.check(rc)
        return out.view(*hidden_states.shape[:-1], w.shape[0])


def wrap_socket_layers_with_adapters(model: nn.Module, socket_layers: list[int], rank: int, scale: float) -> None:
    """Wrap the attention of each socket layer in a residual adapter (reference
    experiments/sva_late4_logit_distill.py:164-174)."""
    hidden_size = int(model.config.hidden_size)
    for layer_idx in socket_layers:
        layer = model.model.layers[layer_idx]
        device = next(layer.self_attn.parameters()).device
        layer.self_attn = SVAResidualOutputAdapter(layer.self_attn, hidden_size, rank, scale).to(device)
