"""PyTorch custom ops over the C ABI (``torch.ops.paris_moe.*``).

The ops run on the current CUDA stream, allocate their outputs and the
workspace through PyTorch's caching allocator, never synchronise the host,
and have fake (meta) implementations, so they can be captured in CUDA
graphs at fixed T.  A non-CUDA tensor, a missing library or a kernel status
other than 0 raises; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib

_BF16 = torch.bfloat16


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _check_cuda(name: str, *ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError(f"paris_moe.{name}: tensors must be CUDA (no CPU fallback)")
        if t.dtype != _BF16:
            raise RuntimeError(f"paris_moe.{name}: expected bf16, got {t.dtype}")
        if not t.is_contiguous():
            raise RuntimeError(f"paris_moe.{name}: tensors must be contiguous")


def _stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


@torch.library.custom_op("paris_moe::moe_block", mutates_args=())
def moe_block(x: torch.Tensor, w_router: torch.Tensor, w_gate_up: torch.Tensor,
              w_down: torch.Tensor, w_sh_gate: torch.Tensor, w_sh_up: torch.Tensor,
              w_sh_down: torch.Tensor, w_sh_gvec: torch.Tensor, top_k: int, expert_lo: int,
              expert_hi: int, flags: int) -> torch.Tensor:
    """y[T,H] = top_k routed experts in [expert_lo, expert_hi) + gated shared expert.

    ``flags``: bit 0 shared expert, bit 1 routed experts, bits 2/3 force the
    streaming / tensor-core kernels (testing).  See include/paris_moe.h.
    """
    _check_cuda("moe_block", x, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up, w_sh_down,
                w_sh_gvec)
    T, H = x.shape
    E = w_router.shape[0]
    I = w_gate_up.shape[1] // 2
    Is = w_sh_gate.shape[0]
    K = top_k
    with torch.cuda.device(x.device):
        y = torch.empty((T, H), dtype=_BF16, device=x.device)
        if T == 0:
            return y
        nbytes = _lib.workspace_size(T, H, E, K, I, Is)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        st = _lib.load().pmoe_block_forward(
            x.data_ptr(), T, H, E, K, I, Is, w_router.data_ptr(), w_gate_up.data_ptr(),
            w_down.data_ptr(), w_sh_gate.data_ptr(), w_sh_up.data_ptr(), w_sh_down.data_ptr(),
            w_sh_gvec.data_ptr(), expert_lo, expert_hi, flags, y.data_ptr(), ws.data_ptr(),
            nbytes, _stream_ptr(x.device))
    _lib.check("pmoe_block_forward", st)
    return y


@moe_block.register_fake
def _moe_block_fake(x, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up, w_sh_down, w_sh_gvec,
                    top_k, expert_lo, expert_hi, flags):
    return x.new_empty(x.shape)


@torch.library.custom_op("paris_moe::moe_layer", mutates_args=())
def moe_layer(x: torch.Tensor, w_norm: torch.Tensor, eps: float, w_router: torch.Tensor,
              w_gate_up: torch.Tensor, w_down: torch.Tensor, w_sh_gate: torch.Tensor,
              w_sh_up: torch.Tensor, w_sh_down: torch.Tensor, w_sh_gvec: torch.Tensor,
              top_k: int, flags: int) -> torch.Tensor:
    """One MoE-only decoder layer: x + block(RMSNorm(x)) (see pmoe_layer_forward)."""
    _check_cuda("moe_layer", x, w_norm, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                w_sh_down, w_sh_gvec)
    T, H = x.shape
    E = w_router.shape[0]
    I = w_gate_up.shape[1] // 2
    Is = w_sh_gate.shape[0]
    with torch.cuda.device(x.device):
        y = torch.empty((T, H), dtype=_BF16, device=x.device)
        if T == 0:
            return y
        nbytes = _lib.workspace_size(T, H, E, top_k, I, Is)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        st = _lib.load().pmoe_layer_forward(
            x.data_ptr(), T, H, E, top_k, I, Is, w_norm.data_ptr(), float(eps),
            w_router.data_ptr(), w_gate_up.data_ptr(), w_down.data_ptr(), w_sh_gate.data_ptr(),
            w_sh_up.data_ptr(), w_sh_down.data_ptr(), w_sh_gvec.data_ptr(), 0, E, 0, T, flags,
            None, 0, 0, 1, 0, y.data_ptr(), ws.data_ptr(), nbytes, _stream_ptr(x.device))
    _lib.check("pmoe_layer_forward", st)
    return y


@moe_layer.register_fake
def _moe_layer_fake(x, w_norm, eps, w_router, w_gate_up, w_down, w_sh_gate, w_sh_up,
                    w_sh_down, w_sh_gvec, top_k, flags):
    return x.new_empty(x.shape)


@torch.library.custom_op("paris_moe::rmsnorm", mutates_args=())
def rmsnorm(x: torch.Tensor, w_norm: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3_5MoeRMSNorm(x): bf16(x * rsqrt(mean(x^2) + eps) * (1 + w)), fp32 inside."""
    _check_cuda("rmsnorm", x, w_norm)
    T, H = x.shape
    with torch.cuda.device(x.device):
        y = torch.empty((T, H), dtype=_BF16, device=x.device)
        st = _lib.load().pmoe_rmsnorm(x.data_ptr(), T, H, w_norm.data_ptr(), float(eps),
                                      y.data_ptr(), _stream_ptr(x.device))
    _lib.check("pmoe_rmsnorm", st)
    return y


@rmsnorm.register_fake
def _rmsnorm_fake(x, w_norm, eps):
    return x.new_empty(x.shape)


@torch.library.custom_op("paris_moe::moe_route", mutates_args=())
def moe_route(x: torch.Tensor, w_router: torch.Tensor, w_sh_gvec: torch.Tensor,
              k: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                               torch.Tensor, torch.Tensor]:
    """Router + top-k + CSR dispatch.

    Returns (topk_idx int32 [T,k], topk_w fp32 [T,k], offsets int32 [E+1],
    sorted_tok int32 [T*k], sorted_slot int32 [T*k], shared_gate fp32 [T]).
    """
    _check_cuda("moe_route", x, w_router, w_sh_gvec)
    T, H = x.shape
    E = w_router.shape[0]
    dev = x.device
    with torch.cuda.device(dev):
        idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        wts = torch.empty((T, k), dtype=torch.float32, device=dev)
        offs = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        stok = torch.empty(T * k, dtype=torch.int32, device=dev)
        sslot = torch.empty(T * k, dtype=torch.int32, device=dev)
        sg = torch.empty(T, dtype=torch.float32, device=dev)
        if T == 0:
            return idx, wts, offs, stok, sslot, sg
        nbytes = _lib.workspace_size(T, H, E, k, 64, 64)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        st = _lib.load().pmoe_route(
            x.data_ptr(), T, H, E, k, w_router.data_ptr(), w_sh_gvec.data_ptr(), idx.data_ptr(),
            wts.data_ptr(), offs.data_ptr(), stok.data_ptr(), sslot.data_ptr(), sg.data_ptr(),
            ws.data_ptr(), nbytes, _stream_ptr(dev))
    _lib.check("pmoe_route", st)
    return idx, wts, offs, stok, sslot, sg


@moe_route.register_fake
def _moe_route_fake(x, w_router, w_sh_gvec, k):
    T = x.shape[0]
    E = w_router.shape[0]
    i32, f32 = torch.int32, torch.float32
    return (x.new_empty((T, k), dtype=i32), x.new_empty((T, k), dtype=f32),
            x.new_empty((E + 1,), dtype=i32), x.new_empty((T * k,), dtype=i32),
            x.new_empty((T * k,), dtype=i32), x.new_empty((T,), dtype=f32))
