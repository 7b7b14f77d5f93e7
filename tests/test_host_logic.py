"""Host-side logic that needs no GPU: the class-level patch, the kill-switch,
and the no-CPU-fallback rule."""
from __future__ import annotations

import pytest
import torch

from conftest import PM


def tiny_block():
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    cfg = Qwen3_5MoeTextConfig(hidden_size=128, num_experts=8, num_experts_per_tok=2,
                               moe_intermediate_size=32, shared_expert_intermediate_size=32)
    torch.manual_seed(0)
    blk = M.Qwen3_5MoeSparseMoeBlock(cfg).to(torch.bfloat16)
    for p in blk.parameters():
        torch.nn.init.normal_(p, std=0.02)
    return M, blk


def test_patch_is_idempotent_and_reversible():
    from paris_moe_b200 import moe
    M, blk = tiny_block()
    orig = M.Qwen3_5MoeSparseMoeBlock.forward
    try:
        assert moe.patch_qwen3_5_moe()
        assert moe.patch_qwen3_5_moe()
        assert M.Qwen3_5MoeSparseMoeBlock._original_forward is orig
        assert M.Qwen3_5MoeSparseMoeBlock.forward is not orig
    finally:
        assert moe.unpatch_qwen3_5_moe()
    assert M.Qwen3_5MoeSparseMoeBlock.forward is orig
    assert not hasattr(M.Qwen3_5MoeSparseMoeBlock, "_original_forward")


def test_kill_switch_runs_the_original(monkeypatch):
    from paris_moe_b200 import moe
    M, blk = tiny_block()
    x = torch.randn(1, 3, 128).to(torch.bfloat16)
    with torch.no_grad():
        want = blk(x)
    try:
        moe.patch_qwen3_5_moe()
        monkeypatch.setenv("PARIS_DISABLE_HELION_MOE", "1")
        with torch.no_grad():
            got = blk(x)
    finally:
        moe.unpatch_qwen3_5_moe()
    assert torch.equal(want, got)


def test_no_cpu_fallback():
    from paris_moe_b200 import moe
    M, blk = tiny_block()
    x = torch.randn(1, 3, 128).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        moe.fused_moe_forward(blk, x)


def test_block_weights_are_the_module_tensors():
    from paris_moe_b200 import moe
    M, blk = tiny_block()
    ws = moe.block_weights(blk)
    assert ws[0] is blk.gate.weight and ws[1] is blk.experts.gate_up_proj
    assert ws[6] is blk.shared_expert_gate.weight
