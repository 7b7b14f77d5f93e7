"""Expert-parallel parity check, one process per GPU (launched by
tests/test_gpu_ep.py through torch.distributed.run).  Every rank compares the
EP output (NVLink exchange and NCCL comparator) with the single-GPU op on the
same seeded inputs and prints one line per check."""
from __future__ import annotations

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from conftest import PM  # noqa: E402,F401  (registers the package)
from oracle import moe_oracle as O  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from paris_moe_b200 import ep, ops, workload as W
    S = W.MoEShape()
    dev = torch.device("cuda", local)
    wts = W.make_weights(S, seed=5, device=dev)
    tensors = wts.tensors()
    fused = ep.EPGroup(S.E, S.H, S.K, mode="fused")
    nccl = ep.EPGroup(S.E, S.H, S.K, mode="nccl")
    ok = True
    for T in (1, 5, 64, 64, 64, 200):
        x = W.make_hidden(T, S, seed=100 + T, device=dev)
        ref = ops.moe_block(x, *tensors, S.K, 0, S.E, 3).float().cpu().numpy()
        for name, g in (("fused", fused), ("nccl", nccl)):
            y = g.forward(x, tensors).float().cpu().numpy()
            r, m = O.rel_l2(y, ref), O.max_abs(y, ref)
            good = r <= 5e-3 and m <= 3e-2
            ok &= good
            print(f"rank{rank} {name} T={T} exchange={g.uses_exchange(T)} rel_l2={r:.2e} "
                  f"max_abs={m:.2e} {'ok' if good else 'FAIL'}", flush=True)
    fused.close()
    dist.barrier()
    print(f"rank{rank} EP_{'OK' if ok else 'FAIL'}", flush=True)
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
