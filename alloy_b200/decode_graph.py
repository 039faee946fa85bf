"""Decode steps of one Mamba layer replayed from a CUDA graph.

The per-token loop of alloy's ``stream_generate`` (alloy/generate.py:83-92)
runs ``model(token, cache=cache)`` and evaluates the cache arrays each step.
For one Mamba layer that is the in-projection, the cached L=1 step
(conv-cache roll + state update, mamba_block.py:446-448, :160-204), the gate
and inner norm (:495-499) and the out-projection.  On the GPU every piece is
stream-ordered and the cache (``MambaCache``, alloy/models/cache.py:13-25) is
updated in place by ``alloy_ssd_decode_step``, so the whole step is captured
once into a CUDA graph and replayed per token: one launch instead of one per
kernel plus the Python between them.
"""

from __future__ import annotations

import torch

from .mamba_block import MambaBlock, MambaCache

__all__ = ["MambaDecodeGraph"]


class MambaDecodeGraph:
    """A captured decode step of ``block`` over ``cache``.

    ``cache`` must already hold the layer's state (after a prefill); its
    tensors stay the ones the caller owns and advance by one token per
    ``step``.  The block must use the combined projection (the in-place
    decode path).  ``step(x_tok)`` copies ``x_tok`` [batch, 1, d_model] into the
    graph's input and returns the graph's output buffer (overwritten by the
    next step).
    """

    def __init__(self, block: MambaBlock, cache: MambaCache, batch: int,
                 warmup: int = 2):
        if not block.combined_proj:
            raise ValueError("graph capture needs the combined projection (in-place decode)")
        if cache.ssm_state is None or cache.conv_state is None:
            raise ValueError("the cache is empty: prefill the layer first")
        if cache.ssm_state.shape[0] != batch:
            raise ValueError(f"cache batch {cache.ssm_state.shape[0]} != {batch}")
        dev = cache.ssm_state.device
        dtype = block.in_proj.weight.dtype
        self.block, self.cache = block, cache
        self.x = torch.zeros((batch, 1, block.d_model), dtype=dtype, device=dev)
        # warm-up steps (first-use setup outside the capture) advance the cache:
        # keep a copy and restore it afterwards
        saved = (cache.ssm_state.clone(), cache.conv_state.clone())
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):
                block(self.x, cache=cache)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.y = block(self.x, cache=cache)
        cache.ssm_state.copy_(saved[0])
        cache.conv_state.copy_(saved[1])

    def step(self, x_tok: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x_tok)
        self.graph.replay()
        return self.y
