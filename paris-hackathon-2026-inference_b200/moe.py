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


def _tp_size(linear) -> int:
    """TP degree of a shard made by engine/model/tp_shard.py (ColumnParallelLinear
    / RowParallelLinear carry ``tp_size``, tp_shard.py:37-52, :74-93); 1 for a
    plain nn.Linear."""
    return int(getattr(linear, "tp_size", 1) or 1)


def _gather_tp_shared(se, group=None):
    """Full shared-expert weights from the TP shards of every rank.

    tp_shard._replace_mlp (tp_shard.py:144-159) leaves rank r with rows
    [r*Is/tp, (r+1)*Is/tp) of gate_proj/up_proj (ColumnParallelLinear) and the
    same columns of down_proj (RowParallelLinear); its forward completes the
    sum with an all_reduce over the default group (tp_shard.py:95-100).  The
    block kernels need the whole expert, so the shards are all-gathered once
    (a collective: every rank calls it in lockstep, as every rank runs the
    layer) and cached on the module, keyed by the shards' storage."""
    import torch.distributed as dist
    g, u, d = se.gate_proj, se.up_proj, se.down_proj
    tp = _tp_size(g)
    if _tp_size(u) != tp or _tp_size(d) != tp:
        raise ValueError("shared expert: gate/up/down are sharded to different TP degrees")
    if any(getattr(m, "bias", None) is not None for m in (g, u, d)):
        raise ValueError("shared expert: TP shards with a bias are not supported")
    key = (tp, g.weight.data_ptr(), u.weight.data_ptr(), d.weight.data_ptr(),
           g.weight._version, u.weight._version, d.weight._version)
    cached = getattr(se, "_pmoe_full_shared", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    if not dist.is_initialized() or dist.get_world_size(group) != tp:
        raise RuntimeError(
            f"shared expert is TP-sharded {tp} ways but the process group has "
            f"{dist.get_world_size(group) if dist.is_initialized() else 1} rank(s): "
            "cannot assemble the full expert")
    Is_l, H = g.weight.shape
    if u.weight.shape != (Is_l, H) or d.weight.shape != (H, Is_l):
        raise ValueError(f"shared expert shards disagree: gate {tuple(g.weight.shape)}, "
                         f"up {tuple(u.weight.shape)}, down {tuple(d.weight.shape)}")
    # gloo gathers host tensors; NCCL the device shards themselves
    host = dist.get_backend(group) == "gloo"
    full = []
    for w, dim in ((g.weight, 0), (u.weight, 0), (d.weight, 1)):
        src = w.detach().contiguous()
        src = src.cpu() if host else src
        parts = [torch.empty_like(src) for _ in range(tp)]
        dist.all_gather(parts, src, group=group)
        full.append(torch.cat(parts, dim=dim).to(w.device).contiguous())
    se._pmoe_full_shared = (key, tuple(full))
    return se._pmoe_full_shared[1]


def shared_weights(moe_block, group=None):
    """(gate [Is,H], up [Is,H], down [H,Is]) of the whole shared expert: the
    module's own tensors, or -- under tensor parallelism -- the assembled shards."""
    se = moe_block.shared_expert
    if max(_tp_size(se.gate_proj), _tp_size(se.up_proj), _tp_size(se.down_proj)) > 1:
        return _gather_tp_shared(se, group)
    return se.gate_proj.weight, se.up_proj.weight, se.down_proj.weight


def block_weights(moe_block, group=None):
    """The seven bf16 weight tensors the op reads, straight from the module
    (no copies; the HF layout is already the kernels' layout), with their
    shapes checked against each other: a mismatch raises instead of
    computing."""
    ex = moe_block.experts
    wr, gu, dn = moe_block.gate.weight, ex.gate_up_proj, ex.down_proj
    sg, su, sd = shared_weights(moe_block, group)
    gv = moe_block.shared_expert_gate.weight
    E, H = wr.shape
    I2 = gu.shape[1]
    Is = sg.shape[0]
    want = {"experts.gate_up_proj": (gu, (E, I2, H)), "experts.down_proj": (dn, (E, H, I2 // 2)),
            "shared_expert.gate_proj": (sg, (Is, H)), "shared_expert.up_proj": (su, (Is, H)),
            "shared_expert.down_proj": (sd, (H, Is)), "shared_expert_gate": (gv, (1, H))}
    for name, (t, shape) in want.items():
        if tuple(t.shape) != shape:
            raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {shape}")
    return (wr, gu, dn, sg, su, sd, gv)


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
