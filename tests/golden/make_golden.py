"""Generate the golden fixtures that pin the CPU oracle (run in a container
that has the reference checked out; the fixtures are committed, the GPU box
never runs this script).

Every fixture is produced by the reference's own code on CPU, from the
seeded workload generators of the package:

* HF ``Qwen3_5MoeSparseMoeBlock`` (transformers 5.5.0, the module the
  reference patches; ``modeling_qwen3_5_moe.py:773-792``) with
  ``_experts_implementation = "grouped_mm"`` (the HF default,
  ``modeling_utils.py:1926-1945``) and ``"eager"``;
* the reference's patched forward ``engine.kernels.moe_grouped_mlp.fused_moe_forward``
  (``engine/kernels/moe_grouped_mlp.py:166-186``, torch dispatch path
  ``engine/kernels/moe_dispatch.py:119-137`` since Helion is absent);
* the reference's ``_torch_dispatch`` for the CSR permutation.

Usage:  python tests/golden/make_golden.py --reference /path/to/reference
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
PKG_DIR = os.path.join(ROOT, "paris-hackathon-2026-inference_b200")


def _load_workload():
    name = "_golden_workload"
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "workload.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


W = _load_workload()


def bits(t):
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def build_hf_block(shape, weights, impl):
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    cfg = Qwen3_5MoeTextConfig(hidden_size=shape.H, num_experts=shape.E,
                               num_experts_per_tok=shape.K,
                               moe_intermediate_size=shape.I,
                               shared_expert_intermediate_size=shape.Is)
    cfg._experts_implementation = impl
    with torch.device("meta"):
        blk = M.Qwen3_5MoeSparseMoeBlock(cfg)
    blk = blk.to_empty(device="cpu").to(torch.bfloat16)
    with torch.no_grad():
        blk.gate.weight.copy_(weights.w_router)
        blk.experts.gate_up_proj.copy_(weights.w_gate_up)
        blk.experts.down_proj.copy_(weights.w_down)
        blk.shared_expert.gate_proj.weight.copy_(weights.w_sh_gate)
        blk.shared_expert.up_proj.weight.copy_(weights.w_sh_up)
        blk.shared_expert.down_proj.weight.copy_(weights.w_sh_down)
        blk.shared_expert_gate.weight.copy_(weights.w_sh_gvec)
    return blk.eval()


def run_case(name, shape, T, seed, zipf_s, full_outputs, ref_mods):
    torch.manual_seed(seed)
    wts = W.make_weights(shape, seed=seed, zipf_s=zipf_s)
    x = W.make_hidden(T, shape, seed=seed, zipf=zipf_s is not None)
    out = {"x": bits(x)} if T <= 1024 else {}
    grouped = build_hf_block(shape, wts, "grouped_mm")
    with torch.inference_mode():
        logits = torch.nn.functional.linear(x, grouped.gate.weight)  # bf16, :764
        _, rw, ri = grouped.gate(x)
        if T <= 1024:
            out["hf_logits"] = bits(logits)
        out["hf_idx"] = ri.to(torch.int32 if shape.E > 256 else torch.uint8).numpy()
        out["hf_w"] = rw.to(torch.float32).numpy()
        tok, slot, offs = ref_mods["dispatch"]._torch_dispatch(ri, shape.E)
        out["ref_offsets"] = offs.to(torch.int32).numpy()
        if T <= 1024:
            out["ref_sorted_tok"] = tok.numpy()
            out["ref_sorted_slot"] = slot.numpy()
        if full_outputs:
            y = grouped(x.view(1, T, shape.H)).view(T, shape.H)
            out["y_hf_grouped"] = bits(y)
            eager = build_hf_block(shape, wts, "eager")
            out["y_hf_eager"] = bits(eager(x.view(1, T, shape.H)).view(T, shape.H))
            y_ref = ref_mods["mlp"].fused_moe_forward(grouped, x.view(1, T, shape.H))
            out["y_ref_fused"] = bits(y_ref.view(T, shape.H))
    # Weights are regenerated from the seed by the tests; a digest of every
    # weight tensor detects a change of torch's CPU generator.
    digests = {n: hashlib.sha256(bits(getattr(wts, n)).tobytes()).hexdigest()[:16]
               for n in shape.weight_names()}
    meta = dict(weights_sha256_16=digests, x_sha256_16=hashlib.sha256(bits(x).tobytes()).hexdigest()[:16],
                name=name, T=T, seed=seed, zipf_s=zipf_s, H=shape.H, E=shape.E, K=shape.K,
                I=shape.I, Is=shape.Is, transformers=__import__("transformers").__version__,
                torch=torch.__version__, generator="tests/golden/make_golden.py")
    out["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path) // 1024} KiB)")


CASES = [
    # name, shape, T, seed, zipf_s, full outputs
    ("tiny_T1", dict(H=256, E=16, K=4, I=64, Is=64), 1, 3, None, True),
    ("tiny_T5", dict(H=256, E=16, K=4, I=64, Is=64), 5, 4, None, True),
    ("tiny_T33", dict(H=256, E=16, K=4, I=64, Is=64), 33, 5, None, True),
    ("tiny_T200_zipf", dict(H=256, E=32, K=8, I=64, Is=128), 200, 6, 1.1, True),
    ("c1_T16", dict(), 16, 0, None, True),
    ("c2_T64", dict(), 64, 0, None, True),          # decode sweep, largest T
    ("c3_T8192_route", dict(), 8192, 0, 1.1, False),  # prefill routing (skewed)
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    import engine.kernels.moe_dispatch as disp      # noqa: E402
    import engine.kernels.moe_grouped_mlp as mlp    # noqa: E402
    torch.set_num_threads(os.cpu_count())
    for name, sh, T, seed, z, full in CASES:
        if a.only and name != a.only:
            continue
        run_case(name, W.MoEShape(**sh), T, seed, z, full, {"dispatch": disp, "mlp": mlp})


if __name__ == "__main__":
    main()
