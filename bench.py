"""Benchmark of the B200 MoE block (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--T 64] [--prefill]

A step is one call of the Qwen3.5-35B-A3B MoE layer on T tokens (default
T=64, the decode configuration of BASELINE.json configs[1]).  Weights are
random-init bf16 of the real shape (1.5 GB, larger than the 126 MB L2, so
every step streams them from HBM; no L2 flush is needed) and hidden states
are synthetic N(0,1).

* ``value``: tokens/s with inputs resident in HBM, device-timed with CUDA
  events over exactly K steps between barriers; for N>1 the max over ranks.
* ``e2e``: the same metric through the public op with pinned host buffers:
  every step copies x host->device and y device->host inside the timed region.
* ``roofline``: the dominant kernel (gate_up + SiLU*mul weight stream),
  algorithmic bytes per launch / its event-timed average duration, against
  the measured HBM copy bandwidth in MEASURED_PEAKS.json.
* ``cpu_baseline``: the reference's own path -- HF transformers
  ``Qwen3_5MoeSparseMoeBlock`` (the module the reference serves with) on the
  host cores, on a bounded sample of the same workload.

``--impl reference`` times that CPU path alone, on rank 0 (other ranks exit).
Multi-GPU (N>1): expert parallel, experts split in contiguous ranges by
rank (engine/runtime/ep.py:78-86); strong scaling over the same T tokens.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "paris-hackathon-2026-inference_b200")


def load_package():
    name = "paris_moe_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ------------------------------------------------------------------ clocks --

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.15)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.f is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.f.seek(0)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline --

def cpu_reference(weights_cpu, x_cpu, budget_s: float, max_steps: int | None = None):
    """Time HF's Qwen3_5MoeSparseMoeBlock (grouped_mm, the HF default) on CPU."""
    import torch
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    S = weights_cpu.shape
    torch.set_num_threads(os.cpu_count())
    cfg = Qwen3_5MoeTextConfig(hidden_size=S.H, num_experts=S.E, num_experts_per_tok=S.K,
                               moe_intermediate_size=S.I, shared_expert_intermediate_size=S.Is)
    cfg._experts_implementation = "grouped_mm"
    with torch.device("meta"):
        blk = M.Qwen3_5MoeSparseMoeBlock(cfg)
    blk = blk.to_empty(device="cpu").to(torch.bfloat16).eval()
    with torch.no_grad():
        blk.gate.weight.copy_(weights_cpu.w_router)
        blk.experts.gate_up_proj.copy_(weights_cpu.w_gate_up)
        blk.experts.down_proj.copy_(weights_cpu.w_down)
        blk.shared_expert.gate_proj.weight.copy_(weights_cpu.w_sh_gate)
        blk.shared_expert.up_proj.weight.copy_(weights_cpu.w_sh_up)
        blk.shared_expert.down_proj.weight.copy_(weights_cpu.w_sh_down)
        blk.shared_expert_gate.weight.copy_(weights_cpu.w_sh_gvec)
    T = x_cpu.shape[0]
    x3 = x_cpu.view(1, T, S.H)
    times = []
    with torch.inference_mode():
        for _ in range(2):
            blk(x3)
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end and (max_steps is None or len(times) < max_steps):
            t0 = time.perf_counter()
            blk(x3)
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": T / med, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "reference",
            "sample": f"HF transformers {__import__('transformers').__version__} "
                      f"Qwen3_5MoeSparseMoeBlock grouped_mm on CPU, T={T}, "
                      f"median of {len(times)} calls after 2 warm-ups",
            "ms_per_call": med * 1e3, "calls": len(times)}


# ------------------------------------------------------------------- main ---

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--T", type=int, default=64)
    ap.add_argument("--zipf", type=float, default=None,
                    help="Zipf(s) prior on the router logits (skewed prefill routing)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    PM = load_package()
    from paris_moe_b200 import workload as W

    regime = "decode" if a.T <= 64 else "prefill"
    metric = f"MoE layer tokens/s ({regime} T={a.T})"
    routing = (f"Zipf(s={a.zipf}) skewed routing (BASELINE configs[2])" if a.zipf
               else "near-uniform routing (BASELINE configs[1])")
    config = {"workload": f"Qwen3.5-35B-A3B MoE block, {regime} T={a.T}, {routing}",
              "T": a.T, "hidden": 2048, "experts": 256, "top_k": 8, "moe_ffn": 512,
              "shared_ffn": 512, "parallelism": f"ep{world}" if world > 1 else "single",
              "l2": "weights (1.5 GB) > L2 (126 MB): streamed from HBM every step"}

    if a.impl == "reference":
        if rank != 0:
            return
        wts = W.make_weights(W.MoEShape(), seed=0, zipf_s=a.zipf)
        x = W.make_hidden(a.T, W.MoEShape(), seed=0, zipf=a.zipf is not None)
        ref = cpu_reference(wts, x, budget_s=1e9, max_steps=a.steps + 0)
        line = {"metric": metric, "value": ref["value"], "unit": "tokens/s", "n_gpus": a.gpus,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ref["ms_per_call"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic", "config": config, "impl": "reference",
                "cpu_baseline": {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": ref["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from paris_moe_b200 import _lib, ops
    lib = _lib.load()

    shape = W.MoEShape()
    wts = W.make_weights(shape, seed=0, device=dev, zipf_s=a.zipf)
    x = W.make_hidden(a.T, shape, seed=0, device=dev, zipf=a.zipf is not None)
    E = shape.E
    lo, hi = rank * E // world, (rank + 1) * E // world
    flags = _lib.PMOE_F_ROUTED | (_lib.PMOE_F_SHARED if rank == 0 else 0)
    st = torch.cuda.current_stream(dev)

    nbytes = _lib.workspace_size(a.T, shape.H, E, shape.K, shape.I, shape.Is)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    y = torch.empty((a.T, shape.H), dtype=torch.bfloat16, device=dev)
    wptrs = [t.data_ptr() for t in wts.tensors()]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    for e in ev:          # torch creates the CUDA event lazily, on first record
        e.record(st)
    ev_arr = (_lib._P * 5)(*[e.cuda_event for e in ev])
    phase_ms = [0.0] * 4

    def step(profiled=False):
        args = (x.data_ptr(), a.T, shape.H, E, shape.K, shape.I, shape.Is, *wptrs, lo, hi,
                flags, y.data_ptr(), ws.data_ptr(), nbytes, st.cuda_stream)
        if profiled:
            s = lib.pmoe_block_forward_profiled(*args, ev_arr, 5)
        else:
            s = lib.pmoe_block_forward(*args)
        _lib.check("pmoe_block_forward", s)
        if world > 1:
            dist.all_reduce(y)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()

    # routing statistics of this input (experts hit), for the roofline bytes
    idx = ops.moe_route(x, wts.w_router, wts.w_sh_gvec, shape.K)[0]
    hit = int(torch.unique(idx).numel())
    torch.cuda.synchronize()

    # ---- timed region: exactly K steps, device-timed, max over ranks ----
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0.record(st)
        for _ in range(a.steps):
            step()
        t1.record(st)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = t0.elapsed_time(t1)
    # Per-phase (per-kernel-group) times: a separate pass with phase events,
    # each step synchronised so every event pair can be read.
    n_prof = min(a.steps, 50)
    acc = [0.0] * 4
    for _ in range(n_prof):
        step(profiled=True)
        torch.cuda.synchronize()
        for i in range(4):
            acc[i] += ev[i].elapsed_time(ev[i + 1])
    phase_ms = [v / n_prof for v in acc]
    if world > 1:
        tt = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms = float(tt.item())
    ms_per_step = elapsed_ms / a.steps
    value = a.T * a.steps / (elapsed_ms / 1e3)

    # ---- e2e: public op, pinned host buffers, copies inside the region ----
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((a.T, shape.H), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x)
    tensors = wts.tensors()

    def e2e_step():
        xd.copy_(x_host, non_blocking=True)
        out = ops.moe_block(xd, *tensors, shape.K, lo, hi, flags)
        if world > 1:
            dist.all_reduce(out)
        y_host.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(a.steps):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_value = a.T * a.steps / (e2e_ms / 1e3)

    peaks, peak_kind = measured_peaks()
    # dominant kernel: gate_up + SiLU*mul weight stream (phase 1)
    S = shape
    local_hit = int(((torch.unique(idx) >= lo) & (torch.unique(idx) < hi)).sum().item())
    gu_bytes = (local_hit * 2 * S.I * S.H + (2 * S.Is * S.H if rank == 0 else 0)) * 2 \
        + a.T * S.H * 2 + (a.T * S.K + a.T) * S.I * 2
    gu_ms = phase_ms[1]
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
    layer_bytes = W.decode_bytes(S, a.T, hit)

    line = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init bf16 weights N(0,0.02), hidden N(0,1), seed 0)",
        "config": config,
        "e2e": {"value": e2e_value, "unit": "tokens/s",
                "h2d_bytes_per_step": a.T * S.H * 2, "d2h_bytes_per_step": a.T * S.H * 2},
        "gpu_launches": 6 * a.steps,
        "roofline": {"kernel": "gate_up_stream_kernel", "bound": "hbm",
                     "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                     "peak_source": peak_kind, "algorithmic_bytes": gu_bytes,
                     "avg_launch_ms": gu_ms},
        "layer_roofline": {"bound": "hbm", "algorithmic_bytes": layer_bytes,
                           "experts_hit": hit,
                           "achieved_gbs": layer_bytes / (ms_per_step * 1e-3) / 1e9,
                           "frac": layer_bytes / (ms_per_step * 1e-3) / 1e9 / peaks["hbm_gbs"]},
        "phase_ms": {"route": phase_ms[0], "gate_up": phase_ms[1], "down": phase_ms[2],
                     "combine": phase_ms[3]},
        "clocks": clk.summary(),
    }
    if world == 1 and rank == 0 and not a.no_cpu_baseline:
        ref = cpu_reference(wts.to("cpu"), x.cpu(), budget_s=a.cpu_budget)
        line["cpu_baseline"] = {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
