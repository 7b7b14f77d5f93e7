"""Drop-in MoE-block forward and the class-level patch that installs it.

Mirrors the reference's operator boundary:

* ``fused_moe_forward(moe_block, hidden_states)`` has the signature and
  return contract of ``engine/kernels/moe_grouped_mlp.py:166-186``: it reads
  the HF module's own weights (``gate``, ``experts``, ``shared_expert``,
  ``shared_expert_gate``) and returns one ``[B, S, H]`` tensor.
* ``patch_qwen3_5_moe`` / ``unpatch_qwen3_5_moe`` follow
  ``engine/kernels/patch.py:43-101``: class-level reassignment of
  ``Qwen3_5MoeSparseMoeBlock.forward``, the original kept at
  ``_original_forward``, idempotent, the env kill-switch
  ``PARIS_DISABLE_HELION_MOE=1`` runs the original HF forward.

Unlike the reference there is no silent fallback: an exception from the
CUDA op propagates (the reference latches to the HF forward on any
exception, patch.py:68-78).
"""
from __future__ import annotations

import logging
import os

import torch

from . import _lib
from .ops import moe_block as _moe_block_op

log = logging.getLogger(__name__)

_PATCHED = False


def _ep_range(moe_block, num_experts: int):
    """Expert range of this rank when the block was prepared for EP."""
    rng = getattr(moe_block, "_pmoe_expert_range", None)
    return (0, num_experts) if rng is None else rng


def block_weights(moe_block):
    """The seven bf16 weight tensors the op reads, straight from the module
    (no copies; the HF layout is already the kernels' layout)."""
    ex = moe_block.experts
    se = moe_block.shared_expert
    return (moe_block.gate.weight, ex.gate_up_proj, ex.down_proj, se.gate_proj.weight,
            se.up_proj.weight, se.down_proj.weight, moe_block.shared_expert_gate.weight)


def fused_moe_forward(moe_block: torch.nn.Module, hidden_states: torch.Tensor) -> torch.Tensor:
    """Replacement for ``Qwen3_5MoeSparseMoeBlock.forward`` (same return contract)."""
    B, S, H = hidden_states.shape
    x = hidden_states.reshape(-1, H)
    if not x.is_contiguous():
        x = x.contiguous()
    E = moe_block.gate.weight.shape[0]
    lo, hi = _ep_range(moe_block, E)
    flags = _lib.PMOE_F_SHARED | _lib.PMOE_F_ROUTED
    flags |= getattr(moe_block, "_pmoe_extra_flags", 0)
    post = getattr(moe_block, "_pmoe_post", None)
    if post is not None:
        # EP: this rank's routed partial; the post hook reduces across ranks
        # and adds the shared expert (engine/runtime/ep.py:97-143 order).
        return post(moe_block, x).view(B, S, H)
    y = _moe_block_op(x, *block_weights(moe_block), int(moe_block.gate.top_k), lo, hi, flags)
    return y.view(B, S, H)


def _disabled() -> bool:
    return os.environ.get("PARIS_DISABLE_HELION_MOE", "0") == "1"


def patch_qwen3_5_moe() -> bool:
    """Install ``fused_moe_forward`` on ``Qwen3_5MoeSparseMoeBlock`` (idempotent).

    Returns False if the HF class is not importable.  Loads the CUDA library
    eagerly so a missing build fails here, not on the first forward.
    """
    global _PATCHED
    if _PATCHED:
        return True
    try:
        from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    except Exception as e:  # transformers too old
        log.warning("cannot patch Qwen3_5MoeSparseMoeBlock: %s", e)
        return False
    cls = getattr(M, "Qwen3_5MoeSparseMoeBlock", None)
    if cls is None:
        return False
    _lib.load()
    original = cls.forward

    def _patched_forward(self, hidden_states):
        if _disabled():
            return original(self, hidden_states)
        return fused_moe_forward(self, hidden_states)

    cls.forward = _patched_forward
    cls._original_forward = original
    _PATCHED = True
    log.info("patched Qwen3_5MoeSparseMoeBlock.forward -> paris_moe fused_moe_forward")
    return True


def unpatch_qwen3_5_moe() -> bool:
    global _PATCHED
    if not _PATCHED:
        return True
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    cls = M.Qwen3_5MoeSparseMoeBlock
    if not hasattr(cls, "_original_forward"):
        return False
    cls.forward = cls._original_forward
    del cls._original_forward
    _PATCHED = False
    return True
