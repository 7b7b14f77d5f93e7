"""Benchmark of the B200 MoE block (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--T 64] [--prefill-T 8192] [--zipf 1.1] [--no-prefill]
                    [--stack-layers 40] [--stack-T 64] [--no-stack]

A step is one call of the Qwen3.5-35B-A3B MoE layer.  The headline
(``metric``/``value``) is the decode configuration of BASELINE.json
configs[1] at its largest batch, T=64 tokens; the same run also measures the
prefill configuration (configs[2]: T=8192, Zipf(s=1.1)-skewed routing) and
reports it under ``"prefill"``, and the 40-layer MoE-only decoder stack at
batch 64 (configs[4]: RMSNorm + block + residual per layer, attention omitted,
one CUDA graph per step, EP over all ranks) under ``"stack"``.  Weights are random-init bf16 of the real
shape (1.5 GB, larger than the 126 MB L2, so every decode step streams them
from HBM; no L2 flush is needed) and hidden states are synthetic N(0,1).

* ``value``: tokens/s with inputs resident in HBM, device-timed with CUDA
  events over exactly K steps between barriers; for N>1 the max over ranks.
* ``e2e``: the same metric through the public op with pinned host buffers:
  every step copies x host->device and y device->host inside the timed region,
  pipelined as a serving loop would (the next step's upload and the previous
  step's download on their own streams while a step computes).
* ``host_ms_per_step``: host time to enqueue a step (launch-bound if near
  ``ms_per_step``).
* ``roofline``: the dominant kernel (decode: the gate_up + SiLU*mul weight
  stream, HBM-bound; prefill: the gate_up grouped GEMM, tensor-bound),
  algorithmic bytes or FLOPs per launch / its event-timed average duration,
  against MEASURED_PEAKS.json.
* ``cpu_baseline``: the reference's own path -- HF transformers
  ``Qwen3_5MoeSparseMoeBlock`` (the module the reference serves with) on the
  host cores, on a bounded sample of the same workload.

``--impl reference`` times that CPU path alone, on rank 0 (other ranks exit).
Multi-GPU (N>1, one process per GPU under torch.distributed.run): expert
parallel, strong scaling over the same tokens.  Decode: contiguous expert
ranges by rank (engine/runtime/ep.py:78-86), the weighted expert rows cross
NVLink from the down-projection epilogue (no collective kernel).  Prefill:
every rank routes all tokens, computes a cost-balanced run of the dispatched
rows, and its down GEMM stores each row at the rank owning the row's token
over NVLink; each rank combines its token slice and pushes it to every rank
(from 8 ranks on: per-rank partials summed over NVLink, pmoe_rows_allreduce).
``comparators`` (decode and prefill) times the same call with the
reference's NCCL all_reduce exchange and with a token-dispatch
all_to_all_single exchange.
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
        return json.load(open(p)), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ------------------------------------------------------------------ clocks --

class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of this rank's GPU during
    a region, read through NVML -- the counters nvidia-smi reports -- by a
    thread every ~2 ms, plus one reading at each edge of the region, so even
    a region of a few milliseconds has samples.  Falls back to nvidia-smi
    (-lms 20) when NVML is unavailable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.f = None
        self.nvml = None
        self.handle = None
        self.samples = []      # (sm MHz, max sm MHz, set of reasons)
        self.stop = None
        self.thread = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:  # the CUDA device's own GPU (CUDA and NVML orderings can differ)
            uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def _read(self):
        N, h = self.nvml, self.handle
        try:
            sm = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
            smax = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            bits = N.nvmlDeviceGetCurrentClocksEventReasons(h)
        except Exception:
            return
        flags = {"hw_slowdown": N.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": N.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": N.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": N.nvmlClocksEventReasonSwPowerCap}
        self.samples.append((float(sm), float(smax), {n for n, b in flags.items() if bits & b}))

    def __enter__(self):
        import threading
        try:
            self.nvml, self.handle = self._nvml_handle()
        except Exception:
            self.nvml = None
        if self.nvml is not None:
            self._read()
            self.stop = threading.Event()

            def loop():
                while not self.stop.wait(0.002):
                    self._read()
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return self
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
        if self.thread is not None:
            self._read()
            self.stop.set()
            self.thread.join(timeout=5)
            return
        if self.proc is not None:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.thread is not None:
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
            reasons = set().union(*(r for _, _, r in self.samples))
            return {"sm_mhz": statistics.median(x for x, _, _ in self.samples),
                    "sm_max_mhz": max(x for _, x, _ in self.samples),
                    "reasons": sorted(reasons), "samples": len(self.samples), "source": "nvml"}
        if self.proc is None or self.f is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.f.seek(0)
        sm, smax, reasons = [], [], set()
        for line in self.f.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(self.NAMES, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


# ------------------------------------------------------------ CPU baseline --

def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def hf_cpu_block(weights_cpu, impl: str = "grouped_mm"):
    """HF's Qwen3_5MoeSparseMoeBlock on the host, holding ``weights_cpu``."""
    import torch
    from transformers.models.qwen3_5_moe.configuration_qwen3_5_moe import Qwen3_5MoeTextConfig
    from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as M
    S = weights_cpu.shape
    cfg = Qwen3_5MoeTextConfig(hidden_size=S.H, num_experts=S.E, num_experts_per_tok=S.K,
                               moe_intermediate_size=S.I, shared_expert_intermediate_size=S.Is)
    cfg._experts_implementation = impl
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
    return blk


def cpu_reference(weights_cpu, x_cpu, budget_s: float, max_steps: int | None = None,
                  impl: str = "grouped_mm", warmup: int = 2, min_steps: int = 10):
    """Time HF's Qwen3_5MoeSparseMoeBlock (``impl``: grouped_mm, the HF default,
    or eager) on all host cores: ``warmup`` untimed calls, then timed calls
    until ``budget_s`` has passed and at least ``min_steps`` ran (or
    ``max_steps``); the median call time gives tokens/s."""
    import torch
    torch.set_num_threads(os.cpu_count())
    blk = hf_cpu_block(weights_cpu, impl)
    T = x_cpu.shape[0]
    x3 = x_cpu.view(1, T, weights_cpu.shape.H)
    times = []
    with torch.inference_mode():
        for _ in range(warmup):
            blk(x3)
        t_end = time.perf_counter() + budget_s
        while (max_steps is None or len(times) < max_steps) and \
                (time.perf_counter() < t_end or len(times) < min_steps):
            t0 = time.perf_counter()
            blk(x3)
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": T / med, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "reference", "cpu_model": cpu_model(),
            "sample": f"HF transformers {__import__('transformers').__version__} "
                      f"Qwen3_5MoeSparseMoeBlock {impl} on CPU, T={T}, "
                      f"median of {len(times)} calls after {warmup} warm-ups",
            "ms_per_call": med * 1e3, "calls": len(times), "T": T, "impl": impl}


def cpu_baseline_rows(wts_cpu, a):
    """BASELINE's CPU plan: primary T=16 (config 1), extra rows T=64 (the GPU
    headline's batch) and T=16 with HF's eager experts.  Bounded: each row
    about ``a.cpu_budget`` seconds."""
    from paris_moe_b200 import workload as W
    x = W.make_hidden(64, wts_cpu.shape, seed=0)
    prim = cpu_reference(wts_cpu, x[:16].clone(), a.cpu_budget)
    rows = [cpu_reference(wts_cpu, x, a.cpu_budget),
            cpu_reference(wts_cpu, x[:16].clone(), a.cpu_budget / 2, impl="eager", min_steps=5)]
    out = {k: prim[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model")}
    out["rows"] = [{k: r[k] for k in ("T", "impl", "value", "ms_per_call", "calls")}
                   for r in rows]
    return out


# ----------------------------------------------------------- GPU measuring --

class Runner:
    """One configuration (T tokens, router weights) on this rank."""

    def __init__(self, ctx, T, w_router, x):
        import torch
        self.ctx, self.T, self.x = ctx, T, x
        S = ctx.S
        self.tensors = [w_router] + ctx.wts.tensors()[1:]
        self.y = torch.empty((T, S.H), dtype=torch.bfloat16, device=ctx.dev)
        self.nbytes = ctx.lib_.workspace_size(T, S.H, S.E, S.K, S.I, S.Is)
        self.ws = torch.empty(self.nbytes, dtype=torch.uint8, device=ctx.dev)
        self.wp = [t.data_ptr() for t in self.tensors]

    def step(self, profiled=False):
        c = self.ctx
        if c.world > 1:
            c.group.forward(self.x, self.tensors, out=self.y, workspace=self.ws,
                            events=c.ev_arr if profiled else None)
            return
        S = c.S
        args = (self.x.data_ptr(), self.T, S.H, S.E, S.K, S.I, S.Is, *self.wp, 0, S.E, 3,
                self.y.data_ptr(), self.ws.data_ptr(), self.nbytes, c.st.cuda_stream)
        if profiled:
            s = c.lib.pmoe_block_forward_profiled(*args, c.ev_arr, 5)
        else:
            s = c.lib.pmoe_block_forward(*args)
        c.lib_.check("pmoe_block_forward", s)

    def timed(self, steps, warmup):
        """(ms per step max over ranks, clock summary)."""
        import torch
        c = self.ctx
        for _ in range(warmup):
            self.step()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c.barrier()
        torch.cuda.synchronize()
        with ClockSampler(c.local) as clk:
            t0.record(c.st)
            h0 = time.perf_counter()
            for _ in range(steps):
                self.step()
            # host time to enqueue the steps: near the device time means the
            # loop is launch-bound, not GPU-bound
            host = (time.perf_counter() - h0) * 1e3 / steps
            t1.record(c.st)
            torch.cuda.synchronize()
        c.barrier()
        self.host_ms = c.max_over_ranks(host)
        return c.max_over_ranks(t0.elapsed_time(t1)) / steps, clk.summary()

    def phases(self, n):
        """Average per-phase ms (route, expert GEMM 1, expert GEMM 2 + tail,
        combine) from events around the kernels of a synchronised call."""
        import torch
        c = self.ctx
        if c.world > 1 and c.group.uses_exchange(self.T):
            return None      # decode exchange: no phase events across its kernels
        acc = [0.0] * 4
        for _ in range(n):
            self.step(profiled=True)
            torch.cuda.synchronize()
            for i in range(4):
                acc[i] += c.ev[i].elapsed_time(c.ev[i + 1])
        return [v / n for v in acc]

    def e2e(self, steps):
        """The public op end to end: every step copies its input from pinned host
        memory to the GPU, runs the op and copies the result back to pinned host
        memory, all inside the timed region.  The steps are pipelined the way a
        serving loop runs them: three slots, the upload of step i+1 and the
        download of step i-1 on their own streams (the two copy engines) while
        step i computes, ordered by events."""
        import torch
        c = self.ctx
        nslot = 3
        x_host = [self.x.cpu().pin_memory() for _ in range(nslot)]
        y_host = [torch.empty((self.T, c.S.H), dtype=torch.bfloat16).pin_memory()
                  for _ in range(nslot)]
        xd = [torch.empty_like(self.x) for _ in range(nslot)]
        # three non-default streams (the legacy default stream would serialise them)
        s_up, s_comp, s_down = (torch.cuda.Stream(c.dev) for _ in range(3))
        up_done = [torch.cuda.Event() for _ in range(nslot)]
        comp_done = [torch.cuda.Event() for _ in range(nslot)]
        down_done = [torch.cuda.Event() for _ in range(nslot)]
        # each slot keeps its step's output alive until the slot's next step
        # (Tensor.record_stream instead cost ~0.3 ms of host time per step)
        keep = [None] * nslot
        from paris_moe_b200 import ops

        def one(i):
            k = i % nslot
            with torch.cuda.stream(s_up):       # slot k's input is free once step i-3 computed
                if i >= nslot:
                    s_up.wait_event(comp_done[k])
                xd[k].copy_(x_host[k], non_blocking=True)
                up_done[k].record(s_up)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(up_done[k])
                if i >= nslot:                  # step i-3's output has left the GPU, so
                    s_comp.wait_event(down_done[k])  # its memory, freed below, is reusable
                if c.world > 1:
                    out = c.group.forward(xd[k], self.tensors)
                else:
                    out = ops.moe_block(xd[k], *self.tensors, c.S.K, 0, c.S.E, 3)
                comp_done[k].record(s_comp)
            with torch.cuda.stream(s_down):
                s_down.wait_event(comp_done[k])
                y_host[k].copy_(out, non_blocking=True)
                down_done[k].record(s_down)
            keep[k] = out

        for i in range(3):
            one(i)
        torch.cuda.synchronize()
        c.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_up)
        for i in range(steps):
            one(i)
        e1.record(s_down)
        torch.cuda.synchronize()
        ms = c.max_over_ranks(e0.elapsed_time(e1)) / steps
        return {"value": self.T / (ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": self.T * c.S.H * 2,
                "d2h_bytes_per_step": self.T * c.S.H * 2, "ms_per_step": ms,
                "pipeline": "3 slots; upload, op and download on separate streams"}


class Ctx:
    def __init__(self, world, rank, local):
        import torch
        import torch.distributed as dist
        from paris_moe_b200 import _lib, workload as W
        self.world, self.rank, self.local = world, rank, local
        self.dist = dist
        if world > 1:
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        self.dev = torch.device("cuda", local)
        torch.cuda.set_device(self.dev)
        self.lib_ = _lib
        self.lib = _lib.load()
        self.S = W.MoEShape()
        self.wts = W.make_weights(self.S, seed=0, device=self.dev)
        self.st = torch.cuda.current_stream(self.dev)
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        for e in self.ev:      # torch creates the CUDA event lazily, on first record
            e.record(self.st)
        self.ev_arr = (_lib._P * 5)(*[e.cuda_event for e in self.ev])
        self.group = None
        if world > 1:
            from paris_moe_b200 import ep
            self.group = ep.EPGroup(self.S.E, self.S.H, self.S.K, mode="fused")

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v):
        if self.world == 1:
            return v
        import torch
        t = torch.tensor([v], device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def comparators(c, x, tensors, T, steps, warmup):
    """N > 1: the same call through the two comparator exchanges -- contiguous
    expert ranges + NCCL all_reduce (the reference's ep_forward) and token
    dispatch with all_to_all_single -- tokens/s, device-timed, max over ranks."""
    import torch
    from paris_moe_b200 import ep
    out = {}
    runs = [("nccl", "nccl_all_reduce"), ("a2a", "all_to_all")]
    if T > ep.FUSED_MAX_T:
        # the prefill exchange EPGroup does not default to at this world size
        runs.append(("fused", "nvlink_partial_sum" if c.world < 8 else "nvlink_rows_to_owner"))
        runs.append(("fused", "nvlink_rows_route_slices"))  # routing by token slice
    for mode, label in runs:
        g = ep.EPGroup(c.S.E, c.S.H, c.S.K, mode=mode)
        if label == "nvlink_partial_sum":
            g.prefill = "partial"
        elif label == "nvlink_rows_to_owner":
            g.prefill = "rows"
        elif label == "nvlink_rows_route_slices":
            g.prefill = "slice"
        y = torch.empty_like(x)
        for _ in range(warmup):
            g.forward(x, tensors, out=y)
        torch.cuda.synchronize()
        c.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(c.st)
        for _ in range(steps):
            g.forward(x, tensors, out=y)
        t1.record(c.st)
        torch.cuda.synchronize()
        c.barrier()
        ms = c.max_over_ranks(t0.elapsed_time(t1)) / steps
        out[label] = {"value": T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
                      "steps": steps}
        g.close()
    return out


def stack_bench(c, a, peaks, peak_kind):
    """Config 5: the MoE-only decoder stack (RMSNorm + MoE block + residual per
    layer, attention omitted), one decode step of batch ``stack_T`` through all
    layers, replayed as one CUDA graph; EP over all ranks of the job."""
    import torch
    from paris_moe_b200 import stack, workload as W
    S, L, T = c.S, a.stack_layers, a.stack_T
    norms, blocks = stack.make_stack_weights(L, seed=1000, device=c.dev)
    st = stack.MoEStack(norms, blocks, group=c.group)
    h0 = W.make_hidden(T, S, seed=3, device=c.dev)
    hs = h0.clone()
    graph = st.capture(hs)
    steps = max(5, min(a.steps, 50))
    for _ in range(a.warmup):
        hs.copy_(h0)
        graph.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c.barrier()
    torch.cuda.synchronize()
    with ClockSampler(c.local) as clk:
        t0.record(c.st)
        for _ in range(steps):
            hs.copy_(h0)          # the step's input (256 KiB device copy)
            graph.replay()
        t1.record(c.st)
        torch.cuda.synchronize()
    c.barrier()
    ms = c.max_over_ranks(t0.elapsed_time(t1)) / steps
    # HBM roofline per rank: every layer streams the routed experts it hits
    # (in its expert range) plus router, shared expert and activations.
    from paris_moe_b200 import ops
    lo, hi = c.rank * S.E // c.world, (c.rank + 1) * S.E // c.world
    byts = 0
    h = h0.clone()
    for l in range(L):
        xn = ops.rmsnorm(h, norms[l], 1e-6)
        idx = ops.moe_route(xn, blocks[l].w_router, blocks[l].w_sh_gvec, S.K)[0]
        hit = torch.unique(idx)
        byts += W.decode_bytes(S, T, int(((hit >= lo) & (hit < hi)).sum().item()))
        h = ops.moe_layer(h, norms[l], 1e-6, *blocks[l].tensors(), S.K, 3)
    ach = byts / (ms * 1e-3) / 1e9
    per_layer = 6 if c.world > 1 else 5   # rmsnorm, [epoch bump], route, gate_up, down, combine
    out = {"metric": f"MoE-only stack decode step ({L} layers, batch {T}) tokens/s",
           "value": T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
           "ms_per_layer": ms / L, "steps": steps, "layers": L, "batch": T,
           "parallelism": f"ep{c.world}" if c.world > 1 else "single",
           "cuda_graph": True, "gpu_launches": per_layer * L * steps, "clocks": clk.summary(),
           "roofline": {"bound": "hbm", "algorithmic_bytes_per_rank": byts, "unit": "GB/s",
                        "achieved": ach, "peak": peaks["hbm_gbs"],
                        "frac": ach / peaks["hbm_gbs"],
                        "peak_source": f"{peak_kind} (hbm_gbs)"}}
    del graph, st, blocks, norms
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--T", type=int, default=64)
    ap.add_argument("--prefill-T", type=int, default=8192)
    ap.add_argument("--zipf", type=float, default=1.1)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-stack", action="store_true")
    ap.add_argument("--stack-layers", type=int, default=40)
    ap.add_argument("--stack-T", type=int, default=64)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ.setdefault("NCCL_DEBUG", "WARN")   # keep stdout to the one JSON line
    load_package()
    from paris_moe_b200 import workload as W

    metric = f"MoE layer tokens/s (decode T={a.T})"
    config = {"workload": f"Qwen3.5-35B-A3B MoE block, decode T={a.T}, near-uniform routing "
                          "(BASELINE configs[1]); prefill T=8192 Zipf routing (configs[2]) "
                          "reported under 'prefill'",
              "T": a.T, "hidden": 2048, "experts": 256, "top_k": 8, "moe_ffn": 512,
              "shared_ffn": 512, "parallelism": f"ep{world}" if world > 1 else "single",
              "l2": "weights (1.5 GB) > L2 (126 MB): streamed from HBM every step, no flush"}

    if a.impl == "reference":
        if rank != 0:
            return
        wts = W.make_weights(W.MoEShape(), seed=0)
        x = W.make_hidden(a.T, W.MoEShape(), seed=0)
        ref = cpu_reference(wts, x, budget_s=1e9, max_steps=a.steps)
        line = {"metric": metric, "value": ref["value"], "unit": "tokens/s", "n_gpus": a.gpus,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ref["ms_per_call"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic", "config": config, "impl": "reference",
                "cpu_baseline": {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": ref["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    c = Ctx(world, rank, local)
    S = c.S
    peaks, peak_kind = measured_peaks()

    # ------------------------------------------------------------ decode --
    x = W.make_hidden(a.T, S, seed=0, device=c.dev)
    dec = Runner(c, a.T, c.wts.w_router, x)
    ms, clocks = dec.timed(a.steps, a.warmup)
    phase = dec.phases(min(a.steps, 50))
    e2e = dec.e2e(a.steps)
    from paris_moe_b200 import ops
    idx = ops.moe_route(x, c.wts.w_router, c.wts.w_sh_gvec, S.K)[0]
    hit_set = torch.unique(idx)
    hit = int(hit_set.numel())
    lo, hi = rank * S.E // world, (rank + 1) * S.E // world
    local_hit = int(((hit_set >= lo) & (hit_set < hi)).sum().item())
    # dominant kernel: gate_up + SiLU*mul weight stream -- algorithmic bytes:
    # gate/up rows of every hit expert of this rank, its share of the shared
    # expert's gate/up rows, the activations read once and h written once.
    sh_rows = 2 * S.Is * S.H
    gu_bytes = (local_hit * 2 * S.I * S.H) * 2 + sh_rows * 2 + a.T * S.H * 2 \
        + (a.T * S.K + a.T) * S.I * 2
    line = {
        "metric": metric, "value": a.T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "host_ms_per_step": dec.host_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init bf16 weights N(0,0.02), hidden N(0,1), seed 0)",
        "config": config, "e2e": e2e,
        # route (1) + gate_up (1) + down (1) + combine (1) per step
        "gpu_launches": 4 * a.steps,
        "clocks": clocks,
    }
    layer_bytes = W.decode_bytes(S, a.T, hit)
    if c.world > 1:
        line["comparators"] = comparators(c, x, c.wts.tensors(), a.T, steps=20, warmup=3)
    line["layer_roofline"] = {"bound": "hbm", "algorithmic_bytes": layer_bytes,
                              "experts_hit": hit, "unit": "GB/s",
                              "achieved": layer_bytes / (ms * 1e-3) / 1e9,
                              "frac": layer_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"]}
    if phase is not None:
        line["phase_ms"] = dict(zip(("route", "gate_up", "down", "combine"), phase))
        ach = gu_bytes / (phase[1] * 1e-3) / 1e9
        line["roofline"] = {"kernel": "gate_up_tma_kernel", "bound": "hbm", "achieved": ach,
                            "peak": peaks["hbm_gbs"], "unit": "GB/s",
                            "frac": ach / peaks["hbm_gbs"],
                            # DRAM bytes come from ncu, which this run does not use;
                            # the capture of this kernel is summarised in the file named
                            "traffic": None,
                            "traffic_profile": "profiles/gate_up_tma_decode_T64.md",
                            "algorithmic_bytes": gu_bytes, "avg_launch_ms": phase[1],
                            "peak_source": f"{peak_kind} (hbm_gbs)"}
    else:
        lb = W.decode_bytes(S, a.T, local_hit)
        line["roofline"] = {"kernel": "whole layer per rank", "bound": "hbm",
                            "achieved": lb / (ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"],
                            "unit": "GB/s", "frac": lb / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                            "traffic": None, "peak_source": f"{peak_kind} (hbm_gbs)"}

    # ----------------------------------------------------------- prefill --
    if not a.no_prefill:
        wr = c.wts.w_router.clone()
        wr[:, 0] = W.zipf_log_prior(S.E, a.zipf, 0).to(c.dev).to(torch.bfloat16)
        xp = W.make_hidden(a.prefill_T, S, seed=0, device=c.dev, zipf=True)
        pre = Runner(c, a.prefill_T, wr, xp)
        psteps = max(5, min(a.steps, 100))
        pms, pclk = pre.timed(psteps, a.warmup)
        pphase = pre.phases(10)
        flops = W.block_flops(S, a.prefill_T)
        pl = {"metric": f"MoE layer tokens/s (prefill T={a.prefill_T}, Zipf s={a.zipf})",
              "value": a.prefill_T / (pms * 1e-3), "unit": "tokens/s", "steps": psteps,
              "ms_per_step": pms, "host_ms_per_step": pre.host_ms, "algorithmic_flops": flops,
              "layer_tflops": flops / (pms * 1e-3) / 1e12,
              "layer_frac": flops / (pms * 1e-3) / 1e12 / peaks["bf16_tflops"],
              # router_tc, scan, scatter, plan, row copy, gate_up, down, combine per step;
              # N > 1: publish, wait, publish, wait around the slice combine (+ a copy)
              "gpu_launches": (8 if c.world == 1 else 12) * psteps, "clocks": pclk,
              "e2e": pre.e2e(max(5, min(a.steps, 50)))}
        if pphase is not None and c.world > 1:   # rank 0's phases
            pl["phase_ms_rank0"] = dict(zip(("route_plan_copy", "gate_up", "down_peer_stores",
                                             "exchange_combine_gather"), pphase))
        elif pphase is not None:
            pl["phase_ms"] = dict(zip(("route_plan_copy", "gate_up", "down", "combine"), pphase))
            P = a.prefill_T * S.K
            gu_flops = 2 * (P + a.prefill_T) * S.H * 2 * S.I
            ach = gu_flops / (pphase[1] * 1e-3) / 1e12
            pl["roofline"] = {"kernel": "tc_pair_kernel<gate_up>", "bound": "tensor",
                              "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                              "frac": ach / peaks["bf16_tflops"], "traffic": None,
                              "traffic_profile": "profiles/tc_pair_gate_up_prefill_T8192.md",
                              "algorithmic_flops": gu_flops, "avg_launch_ms": pphase[1],
                              "peak_source": f"{peak_kind} (bf16_tflops, burst)"}
        if c.world > 1:
            pl["comparators"] = comparators(c, xp, [wr] + c.wts.tensors()[1:], a.prefill_T,
                                            steps=5, warmup=2)
        line["prefill"] = pl

    # ------------------------------------------------------------- stack --
    if not a.no_stack:
        line["stack"] = stack_bench(c, a, peaks, peak_kind)

    if world == 1 and rank == 0 and not a.no_cpu_baseline:
        wcpu = c.wts.to("cpu")
        line["cpu_baseline"] = cpu_baseline_rows(wcpu, a)
        if "prefill" in line:
            # config 3 on the host: the T=8192 Zipf workload, a bounded sample
            # of calls (each call is the whole layer)
            wz = W.make_weights(S, seed=0, zipf_s=a.zipf)
            xz = W.make_hidden(a.prefill_T, S, seed=0, zipf=True)
            pr = cpu_reference(wz, xz, a.cpu_budget, warmup=1, min_steps=2, max_steps=5)
            line["prefill"]["cpu_baseline"] = {
                k: pr[k] for k in ("value", "unit", "cores", "kind", "sample", "cpu_model",
                                   "ms_per_call")}
    if rank == 0:
        print(json.dumps(line))
    if c.group is not None:
        c.group.close()
    if world > 1:
        c.dist.destroy_process_group()


if __name__ == "__main__":
    main()
