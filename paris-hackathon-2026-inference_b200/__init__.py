"""B200-native (sm_100a) Qwen3.5-35B-A3B sparse-MoE block.

Importable under the alias ``paris_moe_b200`` (the directory name has
hyphens): ``load_package()`` in ``bench.py`` / ``tests/conftest.py`` /
``__graft_entry__.py`` registers it.

Public surface (mirrors the reference's engine/kernels API):
  fused_moe_forward, patch_qwen3_5_moe, unpatch_qwen3_5_moe   (moe.py)
  torch.ops.paris_moe.moe_block / moe_route / moe_layer / rmsnorm
      (C++ csrc/torch_ops.cpp -> libparis_moe_torch.so, loaded by ops.py)
  EPGroup (NVLink expert parallelism; comm_handle of moe_block)  (ep.py)
  workload generators                                          (workload.py)
"""
from __future__ import annotations

import importlib

__version__ = "0.1.0"

_LAZY = {
    "fused_moe_forward": "moe", "patch_qwen3_5_moe": "moe", "unpatch_qwen3_5_moe": "moe",
    "block_weights": "moe", "moe_block": "ops", "moe_route": "ops",
}


def __getattr__(name):
    if name in _LAZY:
        mod = importlib.import_module(f".{_LAZY[name]}", __name__)
        return getattr(mod, name)
    raise AttributeError(name)
