"""MoE-only decoder stack: per layer
``h = h + MoEBlock(RMSNorm(h))`` -- Qwen3_5MoeDecoderLayer with the attention
half omitted (post_attention_layernorm, mlp, residual add:
modeling_qwen3_5_moe.py:795-812, 862-868).

Each layer is one ``pmoe_layer_forward`` call (RMSNorm kernel, router,
expert kernels, combine with the residual folded in), updating the residual
stream in place; with an :class:`~.ep.EPGroup` of several ranks the expert
rows cross NVLink inside the down-projection epilogue and every rank ends
each layer with the full hidden state.  The whole stack can be captured in
one CUDA graph (the exchange uses device-side epochs).
"""
from __future__ import annotations

import torch

from . import _lib
from . import workload as W
from .ep import EPGroup

_BF16 = torch.bfloat16


def make_stack_weights(n_layers: int, shape: W.MoEShape = W.MoEShape(), seed: int = 0,
                       device="cuda"):
    """Seeded random-init weights for ``n_layers`` layers: layer l uses the block
    generator with seed ``seed + l`` and the RMSNorm weights of
    ``workload.make_rmsnorm_weights``.  Returns (norm [L,H] bf16, [MoEWeights])."""
    norms = W.make_rmsnorm_weights(n_layers, shape.H, seed=seed, device=device)
    blocks = [W.make_weights(shape, seed=seed + l, device=device) for l in range(n_layers)]
    return norms, blocks


class MoEStack:
    """``n_layers`` MoE-only decoder layers over a [T, H] bf16 residual stream.

    ``group`` (optional) is an :class:`EPGroup`; without one the stack runs on
    the current GPU.  ``forward(h)`` updates ``h`` in place and returns it."""

    def __init__(self, norms: torch.Tensor, blocks, eps: float = 1e-6,
                 group: EPGroup | None = None):
        if len(blocks) != norms.shape[0]:
            raise ValueError("one RMSNorm weight row per layer")
        self.norms = norms
        self.blocks = blocks
        self.eps = float(eps)
        shape = blocks[0].shape
        self.group = group or EPGroup(shape.E, shape.H, shape.K, mode="fused")
        self._ws = None
        self._graph = None

    def _workspace(self, T: int, device) -> torch.Tensor:
        s = self.blocks[0].shape
        nbytes = _lib.workspace_size(T, s.H, s.E, s.K, s.I, s.Is)
        if self._ws is None or self._ws.numel() < nbytes or self._ws.device != device:
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        return self._ws

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        if h.dtype != _BF16 or not h.is_cuda or not h.is_contiguous():
            raise RuntimeError("MoEStack: h must be a contiguous bf16 CUDA tensor")
        ws = self._workspace(h.shape[0], h.device)
        for l, b in enumerate(self.blocks):
            self.group.layer_forward(h, self.norms[l], self.eps, b.tensors(), out=h,
                                     workspace=ws)
        return h

    # -- CUDA graph of the whole stack at a fixed T ---------------------------
    def capture(self, h_static: torch.Tensor) -> torch.cuda.CUDAGraph:
        """Capture ``forward(h_static)`` (in place) into a CUDA graph; replay with
        ``graph.replay()`` after writing the step's input into ``h_static``."""
        self._workspace(h_static.shape[0], h_static.device)
        s = torch.cuda.Stream(device=h_static.device)
        s.wait_stream(torch.cuda.current_stream(h_static.device))
        with torch.cuda.stream(s):   # warm-up outside the graph (lazy init, tensor maps)
            self.forward(h_static.clone())
        torch.cuda.current_stream(h_static.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.forward(h_static)
        self._graph = g
        return g
