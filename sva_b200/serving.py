"""Greedy decoding with the per-token model step captured in a CUDA graph.

The reference decodes through Hugging Face's eager loop (experiments/sva_passkey_language_benchmark.py
:165-248), where every step of a patched model pays the Python and launch overhead of every layer;
at small batch that host time, not the GPU, bounds tokens/s.  ``GraphedGreedyDecoder`` runs the
prompt eagerly into a ``StaticCache`` (so every tensor of a step has a fixed address and shape),
then captures one single-token step -- embedding, all layers, the SVA layers' catalog append and
decode with device-resident lengths (``SVALlamaAttention.sva_attention_static``), the head and
the greedy argmax -- in one CUDA graph, and replays it once per token.  The cache and the position
advance on the device inside the graph, so a replay needs no host work besides the launch.
"""

from __future__ import annotations

import torch
from transformers import StaticCache


class GraphedGreedyDecoder:
    """Greedy decoding of a (patched) causal LM with a CUDA-graph step.

    ``model`` is a Hugging Face causal LM on a CUDA device; ``max_len`` bounds prompt + generated
    tokens.  The batch must be unpadded (every sequence has the prompt length).
    """

    def __init__(self, model, batch: int, max_len: int) -> None:
        self.model = model
        self.batch = int(batch)
        self.max_len = int(max_len)
        self.device = next(model.parameters()).device
        self.cache = None
        self.graph = None
        self.tok = None  # [B, 1] the step's input token (static buffer)
        self.next_tok = None

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Runs the prompt [B, T] into a fresh static cache; returns the first generated token."""
        self.cache = StaticCache(config=self.model.config, max_cache_len=self.max_len)
        out = self.model(input_ids=prompt.to(self.device), use_cache=True, past_key_values=self.cache,
                         logits_to_keep=1)
        first = out.logits[:, -1].argmax(-1, keepdim=True)
        self.tok = first.clone()
        self.graph = None
        return first

    @torch.no_grad()
    def _step(self) -> torch.Tensor:
        out = self.model(input_ids=self.tok, use_cache=True, past_key_values=self.cache, logits_to_keep=1)
        return out.logits[:, -1].argmax(-1, keepdim=True)

    @torch.no_grad()
    def capture(self) -> None:
        """Captures one decode step.  The warm-up step it runs first is a real decode step (its
        token is generated and the cache advances), so that every buffer the step uses exists
        before capture; the captured step then continues from there."""
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            nxt = self._step()
            self.tok.copy_(nxt)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        self.warm_token = nxt.clone()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.next_tok = self._step()
            self.tok.copy_(self.next_tok)

    def step(self) -> torch.Tensor:
        """One replay: decodes the token in ``self.tok`` and leaves the next one there."""
        self.graph.replay()
        return self.next_tok

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, steps: int) -> torch.Tensor:
        """Greedy tokens [B, steps] after the prompt (prefill + warm-up step + graph replays)."""
        toks = [self.prefill(prompt)]
        if steps > 1:
            self.capture()
            toks.append(self.warm_token)
            for _ in range(steps - 2):
                toks.append(self.step().clone())
        return torch.cat(toks, 1)[:, :steps]

    def release(self) -> None:
        self.graph = None
        self.cache = None
