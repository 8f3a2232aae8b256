"""Greedy decode step recorded once and replayed per token (drop-in for qwen35_fused/graph.py:13-94).

The reference's interface is kept: ``GreedyDecodeGraph(model, cache, token, position_ids, *,
fused_lm_head=True, steps=1)``, ``set_inputs(token, position_ids)`` and ``replay()``, with the
same ``ValueError`` conditions. The body is organised around a device-side token ring:

* ``_ring[0]`` is the token the next replay consumes; ``_ring[1 + i]`` receives the greedy choice
  of step ``i``. Step ``i`` reads ``_ring[i]``, so the chain of steps needs no copy between them.
* The last action of the recording moves ``_ring[steps]`` into ``_ring[0]`` and advances the
  position tensor by ``steps``: a replay leaves the buffers ready for the next one, and the host
  only reads a token when it wants one (one D2H read per replay in the wrapper).
* The LM head is ``ppu_b200.kernels.lm_head_argmax`` over the last hidden state (the fused top-1
  kernel, ties to the lowest index) or, with ``fused_lm_head=False``, the model's own logits and a
  device argmax.

The recording runs on a side stream (``torch.cuda.graph`` with its own pool), after a device
synchronisation so that the prefill that filled ``cache`` has finished. ``Qwen35Engine.capture``
is the same idea over the fully fused C-ABI decoder (5 kernels per layer).
"""

from __future__ import annotations

import torch

from .kernels import lm_head_argmax


def _greedy_from_model(model, token: torch.Tensor, position_ids: torch.Tensor, cache, fused: bool) -> torch.Tensor:
    """One decode forward of ``model`` at ``position_ids``; returns the greedy token, shaped like
    ``token`` (int64, on device)."""
    if fused:
        state = model.model(input_ids=token, position_ids=position_ids, past_key_values=cache,
                            attention_mask=None, use_cache=True, return_dict=True).last_hidden_state
        return lm_head_argmax(state[:, -1, :].contiguous(), model.lm_head.weight).view_as(token)
    logits = model(input_ids=token, position_ids=position_ids, past_key_values=cache, attention_mask=None,
                   use_cache=True, logits_to_keep=1, return_dict=True).logits
    return logits[:, -1, :].argmax(dim=-1).view_as(token)


class GreedyDecodeGraph:
    """Records ``steps`` greedy decode steps of a fused Qwen3.5 model into one CUDA graph.

    ``cache`` must hold the prefill already and keep static full-attention layers (the graph
    writes K/V at device-side offsets); ``token`` is the first token to feed ([B, 1] int64 on the
    GPU) and ``position_ids`` its position tensor (the multimodal [3 or 4, B, 1] form or [B, 1]).
    """

    def __init__(self, model, cache, token: torch.Tensor, position_ids: torch.Tensor, *,
                 fused_lm_head: bool = True, steps: int = 1) -> None:
        if not (token.is_cuda and token.dtype == torch.long and token.shape[-1] == 1):
            raise ValueError("token must be a CUDA int64 tensor with sequence length 1")
        if not position_ids.is_cuda:
            raise ValueError("position_ids must be on the GPU")
        if steps < 1:
            raise ValueError("steps must be positive")
        self.model, self.cache = model, cache
        self.steps, self.fused_lm_head = steps, fused_lm_head
        self._ring = token.new_empty((steps + 1, *token.shape))
        self._ring[0].copy_(token)
        self.position_ids = position_ids.clone()
        self.graph = torch.cuda.CUDAGraph()
        self._record()

    def _record(self) -> None:
        dev = self._ring.device
        torch.cuda.synchronize(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.cuda.graph(self.graph, stream=side):
            for i in range(self.steps):
                choice = _greedy_from_model(self.model, self._ring[i], self.position_ids, self.cache,
                                            self.fused_lm_head)
                self._ring[i + 1].copy_(choice)
                self.position_ids.add_(1)
            self._ring[0].copy_(self._ring[self.steps])
        torch.cuda.current_stream(dev).wait_stream(side)

    @property
    def token(self) -> torch.Tensor:
        """The token the next replay will consume (the last greedy choice after a replay)."""
        return self._ring[0]

    @property
    def output_tokens(self) -> torch.Tensor | None:
        """The ``steps`` choices of the last replay, ``[steps, B, 1]`` (None for one step)."""
        return self._ring[1:] if self.steps > 1 else None

    def set_inputs(self, token: torch.Tensor, position_ids: torch.Tensor) -> None:
        """Point the next replay at a new first token and position (device copies only)."""
        if token.shape != self._ring[0].shape or position_ids.shape != self.position_ids.shape:
            raise ValueError("graph input shapes do not match the captured buffers")
        self._ring[0].copy_(token)
        self.position_ids.copy_(position_ids)

    def replay(self) -> torch.Tensor:
        """Runs the recorded steps; returns the last token ([B, 1]) for one step, else all
        ``steps`` choices ([steps, B, 1])."""
        self.graph.replay()
        return self._ring[1] if self.steps == 1 else self._ring[1:]
