"""Seeded synthetic MoE-layer workloads.

The reference quotes no dataset for the MoE block; its configurations are
synthetic by construction (random-init weights of the Qwen3.5-35B-A3B MoE
shape, N(0,1) hidden states).  Every generator here is deterministic for a
given seed and device:

* weights: N(0, 0.02) rounded to bf16, drawn in a fixed order
  (router, gate_up, down, shared gate, shared up, shared down, shared gate
  vector) from one ``torch.Generator``;
* hidden states: N(0, 1) rounded to bf16 from a second generator
  (seed + 1), so the same weights can be reused across token counts;
* skewed ("prefill") routing: a log-Zipf(s) prior over a seeded permutation
  of the experts is folded into the router as a constant input channel
  (``x[:, 0] = 1`` and ``W_r[:, 0] = log p_e``), which keeps the operator
  signature unchanged while producing skewed per-expert counts.

Shapes follow the HF module attributes the reference reads
(``transformers/models/qwen3_5_moe/modeling_qwen3_5_moe.py:698-792``):
``gate.weight [E,H]``, ``experts.gate_up_proj [E,2I,H]``,
``experts.down_proj [E,H,I]``, ``shared_expert.{gate,up}_proj.weight [Is,H]``,
``shared_expert.down_proj.weight [H,Is]``, ``shared_expert_gate.weight [1,H]``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
import torch

# Qwen3.5-35B-A3B MoE constants (configuration_qwen3_5_moe.py:80-102).
HIDDEN = 2048
NUM_EXPERTS = 256
TOP_K = 8
MOE_INTER = 512
SHARED_INTER = 512
RMS_EPS = 1e-6


@dataclass
class MoEShape:
    H: int = HIDDEN
    E: int = NUM_EXPERTS
    K: int = TOP_K
    I: int = MOE_INTER
    Is: int = SHARED_INTER

    def weight_names(self):
        return ("w_router", "w_gate_up", "w_down", "w_sh_gate", "w_sh_up",
                "w_sh_down", "w_sh_gvec")


@dataclass
class MoEWeights:
    """bf16 weights of one MoE block in the HF layout (row-major, K-contiguous)."""
    shape: MoEShape
    w_router: torch.Tensor     # [E, H]
    w_gate_up: torch.Tensor    # [E, 2I, H]  rows [0:I] gate, [I:2I] up
    w_down: torch.Tensor       # [E, H, I]
    w_sh_gate: torch.Tensor    # [Is, H]
    w_sh_up: torch.Tensor      # [Is, H]
    w_sh_down: torch.Tensor    # [H, Is]
    w_sh_gvec: torch.Tensor    # [1, H]
    zipf_s: float | None = None
    meta: dict = field(default_factory=dict)

    def tensors(self):
        return [getattr(self, n) for n in self.shape.weight_names()]

    def to(self, device):
        kw = {n: getattr(self, n).to(device) for n in self.shape.weight_names()}
        return MoEWeights(self.shape, zipf_s=self.zipf_s, meta=dict(self.meta), **kw)

    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in self.tensors())


def _randn_bf16(shape, gen, device, std, chunk_rows=64):
    """N(0, std) in bf16, generated in row chunks to bound fp32 temporaries."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    n0 = shape[0]
    for r in range(0, n0, chunk_rows):
        rr = min(chunk_rows, n0 - r)
        t = torch.randn((rr,) + tuple(shape[1:]), generator=gen, device=device,
                        dtype=torch.float32)
        out[r:r + rr] = (t * std).to(torch.bfloat16)
    return out


def zipf_log_prior(E: int, s: float, seed: int) -> torch.Tensor:
    """log p_e of a Zipf(s) law over a seeded permutation of the E experts (fp32)."""
    ranks = torch.arange(1, E + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p = p / p.sum()
    g = torch.Generator(device="cpu").manual_seed(seed + 7919)
    perm = torch.randperm(E, generator=g)
    logp = torch.empty(E, dtype=torch.float64)
    logp[perm] = p.log()
    return logp.to(torch.float32)


def make_weights(shape: MoEShape = MoEShape(), seed: int = 0, device="cpu",
                 std: float = 0.02, zipf_s: float | None = None) -> MoEWeights:
    """Random-init MoE weights (see module docstring for the draw order)."""
    S = shape
    g = torch.Generator(device=device).manual_seed(seed)
    w_router = _randn_bf16((S.E, S.H), g, device, std)
    w_gate_up = _randn_bf16((S.E, 2 * S.I, S.H), g, device, std, chunk_rows=16)
    w_down = _randn_bf16((S.E, S.H, S.I), g, device, std, chunk_rows=16)
    w_sh_gate = _randn_bf16((S.Is, S.H), g, device, std)
    w_sh_up = _randn_bf16((S.Is, S.H), g, device, std)
    w_sh_down = _randn_bf16((S.H, S.Is), g, device, std)
    w_sh_gvec = _randn_bf16((1, S.H), g, device, std)
    if zipf_s is not None:
        logp = zipf_log_prior(S.E, zipf_s, seed)
        w_router[:, 0] = logp.to(device=device).to(torch.bfloat16)
    return MoEWeights(S, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                      w_sh_down, w_sh_gvec, zipf_s=zipf_s, meta={"seed": seed})


def make_hidden(T: int, shape: MoEShape = MoEShape(), seed: int = 0, device="cpu",
                zipf: bool = False) -> torch.Tensor:
    """Hidden states [T, H] ~ N(0,1) bf16; column 0 is 1 when the Zipf prior is folded in."""
    g = torch.Generator(device=device).manual_seed(seed + 1)
    x = torch.randn((T, shape.H), generator=g, device=device, dtype=torch.float32)
    x = x.to(torch.bfloat16)
    if zipf:
        x[:, 0] = 1.0
    return x


def make_rmsnorm_weights(n_layers: int, H: int = HIDDEN, seed: int = 0, device="cpu"):
    """RMSNorm weights for the MoE-only stack; Qwen3.5 stores (w) and scales by (1 + w)."""
    g = torch.Generator(device=device).manual_seed(seed + 104729)
    return (torch.randn((n_layers, H), generator=g, device=device) * 0.02).to(torch.bfloat16)


# ---- algorithmic work per call (bench roofline numerators) -----------------

def decode_bytes(shape: MoEShape, T: int, experts_hit: int) -> int:
    """Algorithmic HBM bytes of one block call: each hit expert's gate_up+down
    once, router + shared expert + shared gate once, activations in and out."""
    S = shape
    per_expert = (2 * S.I * S.H + S.H * S.I) * 2
    fixed = (S.E * S.H + 3 * S.Is * S.H + S.H) * 2
    return experts_hit * per_expert + fixed + T * S.H * 2 * 2


def block_flops(shape: MoEShape, T: int) -> int:
    """Algorithmic FLOPs of one block call (2 per MAC), independent of skew."""
    S = shape
    routed = S.K * (2 * S.I * S.H + S.H * S.I)
    shared = 3 * S.Is * S.H
    router = S.E * S.H + S.H
    return 2 * T * (routed + shared + router)


def expected_hit(E: int, K: int, T: int) -> float:
    return E * (1.0 - (1.0 - K / E) ** T)

