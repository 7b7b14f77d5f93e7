"""The decoder-layer oracle (config 5) pinned against transformers' own
modules on CPU: ``Qwen3_5MoeRMSNorm`` bit for bit (up to a last-bit flip from
the rsqrt), and ``residual + mlp(post_attention_layernorm(x))`` with the HF
sparse-MoE block."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import moe_oracle as O

hf = pytest.importorskip("transformers.models.qwen3_5_moe.modeling_qwen3_5_moe")


def _bits(t):
    return O.torch_bf16_bits(t)


def test_rmsnorm_matches_hf():
    from paris_moe_b200 import workload as W
    x = W.make_hidden(32, W.MoEShape(), seed=1)
    w = W.make_rmsnorm_weights(1, seed=1)[0]
    mod = hf.Qwen3_5MoeRMSNorm(2048, eps=1e-6)
    with torch.no_grad():
        mod.weight.copy_(w.float())
        ref = _bits(mod(x))
    got = O.rmsnorm(_bits(x), _bits(w), 1e-6)
    diff = got != ref
    assert diff.mean() < 1e-3
    if diff.any():
        assert np.abs(got[diff].astype(np.int32) - ref[diff].astype(np.int32)).max() <= 1


def test_decoder_layer_matches_hf_block():
    """bf16(x + bf16(block(rmsnorm(x)))) with the HF block in eager mode, on a
    small configuration (same code path, 16 experts)."""
    from paris_moe_b200 import workload as W
    shape = W.MoEShape(H=256, E=16, K=4, I=64, Is=64)
    wts = W.make_weights(shape, seed=2)
    x = W.make_hidden(8, shape, seed=2)
    w_norm = W.make_rmsnorm_weights(1, H=shape.H, seed=2)[0]
    cfg = hf.Qwen3_5MoeTextConfig(hidden_size=shape.H, num_experts=shape.E,
                                  num_experts_per_tok=shape.K, moe_intermediate_size=shape.I,
                                  shared_expert_intermediate_size=shape.Is)
    cfg._experts_implementation = "eager"
    blk = hf.Qwen3_5MoeSparseMoeBlock(cfg).to(torch.bfloat16)
    norm = hf.Qwen3_5MoeRMSNorm(shape.H, eps=1e-6)
    with torch.no_grad():
        blk.gate.weight.copy_(wts.w_router)
        blk.experts.gate_up_proj.copy_(wts.w_gate_up)
        blk.experts.down_proj.copy_(wts.w_down)
        blk.shared_expert.gate_proj.weight.copy_(wts.w_sh_gate)
        blk.shared_expert.up_proj.weight.copy_(wts.w_sh_up)
        blk.shared_expert.down_proj.weight.copy_(wts.w_sh_down)
        blk.shared_expert_gate.weight.copy_(wts.w_sh_gvec)
        norm.weight.copy_(w_norm.float())
        xn = norm(x)
        ref = (x + blk(xn[None])[0]).float().numpy()
    got, _ = O.decoder_layer(_bits(x), _bits(w_norm),
                             [_bits(getattr(wts, n)) for n in shape.weight_names()], shape.K)
    # the HF eager block rounds each expert output to bf16; the oracle keeps fp32
    assert O.rel_l2(got, ref) < 6e-3
