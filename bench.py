"""Benchmark of the B200 quantized MoE layer (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one pass of the MoE layer (route -> permute -> gate/up GEMM -> down GEMM ->
combine) over one batch of the workload's seeded synthetic bf16 activations, with the
seeded random-init layer resident in HBM.  Under torchrun (--gpus N > 1) the layer runs
expert-parallel: the workload's tokens are split over the ranks (strong scaling: the same
total tokens at every N), each rank keeps E/N routed experts, and tokens and partial
outputs cross NCCL.  Timing is CUDA events on the launching stream between barrier +
synchronize fences, max over ranks.  `--workload cfg2_mla_decode` and `cfg3_attn_decode` time
the MLA latent attention kernel and the GQA attention block instead (their own metrics);
`cfg3_engine_decode` times whole-model decode steps through the engine backend.

`value` times K calls of the fused public entry point (ccut_moe_forward), inputs resident in
HBM; `e2e` times the same call with pinned host input and output copies every step; the
roofline kernel (the gate/up GEMM) is timed in a separate pass of K staged steps.

`--impl reference` times the reference algorithm on the host cores instead (the numpy
oracle port of CostCut-Infer's MoE path: per-call dequant of every touched expert, fp32
BLAS matmuls, the reference's combine loop) on the workload's whole batch per call, K calls;
rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

# name -> (config, tokens per GPU, roofline bound of the dominant kernel)
WORKLOADS = {
    "cfg1_prefill": ("cfg1", 2048, "tensor"),
    "cfg1_decode": ("cfg1", 64, "hbm"),
    "cfg1_decode256": ("cfg1", 256, "hbm"),
    "cfg0_decode": ("cfg0", 64, "hbm"),
    "cfg0_decode1": ("cfg0", 1, "hbm"),
    "cfg0_prefill": ("cfg0", 4096, "tensor"),
    "cfg3_decode": ("cfg3", 64, "hbm"),
    "cfg3_prefill": ("cfg3", 4096, "tensor"),
    "cfg4_decode": ("cfg4", 256, "hbm"),
    "cfg4_prefill": ("cfg4", 4096, "tensor"),
}
# Layers generated on the GPU (synthetic.make_layer_device: same shapes and distributions,
# another random stream) because the host generator needs minutes for them; their CPU
# baseline is not run (the oracle would need the same 11 GB of weights in fp32 on the host).
DEVICE_GENERATED = {"cfg4"}
# The default: BASELINE config 3 (Qwen3-30B-A3B-shaped MoE layer, AWQ int4, 128 experts,
# top-8), 4096-token prefill -- the config that names expert parallelism over 2 / 4 / 8 GPUs
# and the token count of the scaling target; the same total tokens at every N.
DEFAULT_WORKLOAD = "cfg3_prefill"
METRIC = "MoE-layer tokens/s"

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the GPU is under load."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons = [], None, set()
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                smax = float(f[1])
            except ValueError:
                continue
            for name, v in zip(self.NAMES, f[3:7]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ algorithmic counts
def gate_up_counts(cfg, offsets: np.ndarray) -> tuple[float, float]:
    """(bytes, flops) of one gate/up launch: weights of experts with rows, rows read once,
    intermediate rows written once."""
    from ccut_b200.synthetic import _matrix_bytes

    ne = cfg.num_experts + (cfg.num_shared * cfg.shared_inter // cfg.inter if cfg.num_shared else 0)
    m = np.diff(offsets[:ne + 1]).astype(np.int64)
    active = int((m > 0).sum())
    rows = int(m.sum())
    wbytes = active * 2 * _matrix_bytes(cfg.fmt, cfg.hidden, cfg.inter)
    byts = wbytes + rows * cfg.hidden * 2 + rows * cfg.inter * 2
    flops = 4.0 * rows * cfg.hidden * cfg.inter
    return float(byts), flops


def layer_flops(cfg, T: int) -> float:
    per_tok = 2 * 3 * cfg.hidden * cfg.inter * cfg.top_k
    shared = 2 * 3 * cfg.hidden * cfg.shared_inter * cfg.num_shared
    return float(T * (per_tok + shared) + 2 * T * cfg.num_experts * cfg.hidden)


# ------------------------------------------------------------------ CPU (oracle) leg
def cpu_sample_run(cfg_name: str, T: int, sample: int, steps: int, budget_s: float) -> dict:
    """Time the oracle port of the reference path on `sample` tokens of the workload (the
    whole batch by default: the reference dequantizes every touched expert once per call, so
    a smaller sample would spread that cost over fewer tokens than the workload has)."""
    from oracle import formats, inputs, moe  # the checker; only this leg runs it

    cores = os.cpu_count() or 1
    try:
        import torch

        torch.set_num_threads(cores)
    except Exception:
        pass
    cfg = inputs.CONFIGS[cfg_name]
    lw = inputs.make_layer(cfg, seed=0)
    xb = lw.make_x(T)[:sample]
    xf = formats.bf16_bits_to_f32(xb)
    times = []
    t_start = time.perf_counter()
    for _ in range(steps):
        lw._cache.clear()  # the reference dequantizes every touched expert on every call
        t0 = time.perf_counter()
        moe.moe_forward(xf, lw.router, cfg.top_k, cfg.routing, lw.w_lookup, shared=lw.shared_cat(),
                        route_kw=cfg.route_kw)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    med = statistics.median(times)
    what = f"the whole {T}-token batch" if sample == T else f"{sample} of the {T} tokens"
    return {
        "value": sample / med, "unit": "tokens/s", "cores": cores, "kind": "port", "steps_run": len(times),
        "ms_per_call": med * 1e3,
        "sample": (f"{what} of {cfg_name} per call; numpy oracle port of the reference path "
                   f"(per-call dequant of every touched expert as the reference does, fp32 BLAS on {cores} "
                   f"threads); median of {len(times)} call(s)"),
    }


def run_reference(args, wl) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg_name, T, _ = WORKLOADS[wl]
    if cfg_name in DEVICE_GENERATED:
        print(json.dumps({"impl": "reference", "unavailable": f"{wl}: the host oracle would need the whole layer "
                          "(11 GB of FP8 weights, 45 GB dequantized) in host memory; the reference arm runs on the "
                          "other workloads"}), flush=True)
        return
    sample = T if args.cpu_sample <= 0 else min(T, args.cpu_sample)
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_sample_run(cfg_name, T, min(sample, 8), 1, 60)
    r = cpu_sample_run(cfg_name, T, sample, args.steps, float("inf"))  # exactly K calls
    # the same config as our arm's line at this N (the same total batch; run here on rank 0's
    # host cores)
    n = max(1, args.gpus)
    cfgd = workload_config(wl, 1, "single" if n == 1 else f"ep{n}")
    if n > 1:
        cfgd["tokens_per_gpu"] = T // n
        cfgd["experts_per_gpu"] = _layer_config(cfg_name).num_experts // n
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": r["steps_run"], "warmup": args.warmup, "ms_per_step": sample / r["value"] * 1000.0,
        "higher_is_better": True, "scaling": "weak" if n == 1 else "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": cfgd, "reference_run": "the whole batch on the host cores of rank 0",
        "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _layer_config(name: str):
    from ccut_b200.synthetic import CONFIGS

    return CONFIGS[name]


def workload_config(wl: str, n: int, parallelism: str) -> dict:
    from ccut_b200.synthetic import CONFIGS

    cfg_name, T, _ = WORKLOADS[wl]
    c = CONFIGS[cfg_name]
    return {
        "workload": wl, "baseline_config": cfg_name, "tokens_per_gpu": T, "global_tokens": T * n,
        "format": c.fmt, "hidden": c.hidden, "inter": c.inter, "experts": c.num_experts, "top_k": c.top_k,
        "shared_experts": c.num_shared, "routing": c.routing, "parallelism": parallelism,
        "l2": "inputs larger than L2: expert weights "
              f"{(c.expert_bytes() * c.num_experts + c.shared_bytes()) / 1e6:.0f} MB > 126 MB L2, no flush",
    }


# DRAM bytes (read + write) of one gate/up launch from an ncu capture of the current kernel on
# the same workload; workloads without such a capture report null.
NCU_TRAFFIC: dict = {"cfg3_prefill": 385_041_920, "cfg0_decode": 202_890_240}

# Dense FP8 (e4m3 x e4m3) peak of this GPU, measured in the run: torch._scaled_mm 8192^3,
# bf16 out, best of 10 (cuBLAS).  MEASURED_PEAKS.json has no FP8 figure.
def fp8_peak_tflops(dev) -> float:
    import torch

    n = 8192
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
    one = torch.tensor(1.0, device=dev)

    def mm():
        return torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)

    for _ in range(3):
        mm()
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        mm()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12

# ------------------------------------------------------------------ end-to-end leg
def e2e_pipelined(forward, x_pin, out_shape, dev, K: int) -> float:
    """K end-to-end steps through the public forward: every step copies its input from
    pinned host memory to the device and its bf16 output back.  The copies run on two copy
    streams, double-buffered, so that step i's input copy and step i-1's output copy
    overlap step i's compute, as a serving loop streams requests.  Returns the milliseconds
    from before the first input copy to after the last output copy."""
    import torch

    comp = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    xin = [torch.empty(tuple(x_pin.shape), dtype=x_pin.dtype, device=dev) for _ in range(2)]
    out_pin = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(K)]
    computed = [torch.cuda.Event() for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(comp)
    h2d.wait_stream(comp)
    d2h.wait_stream(comp)
    for i in range(K):
        b = i % 2
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(computed[i - 2])  # the forward of step i - 2 has read xin[b]
            xin[b].copy_(x_pin, non_blocking=True)
            in_ready[i].record(h2d)
        comp.wait_event(in_ready[i])
        y = forward(xin[b])
        computed[i].record(comp)
        y.record_stream(d2h)
        with torch.cuda.stream(d2h):
            d2h.wait_event(computed[i])
            out_pin[b].copy_(y, non_blocking=True)  # ordered after step i - 2's copy into it
    comp.wait_stream(d2h)
    end.record(comp)
    torch.cuda.synchronize(dev)
    return start.elapsed_time(end)


# ------------------------------------------------------------------ GPU leg
# Kernels of this library per staged single-GPU step: route (logits, top-k), permute
# (count, permute), gate/up (gather or f16 convert, GEMM), down (GEMM), combine.
def ep_launches(cfg) -> int:
    """Kernels of this library per expert-parallel step (NCCL's own kernels not counted):
    route 2, plan 1, count 1, permute 1, routed FFN 3, per-row combine 1, final sum 1, and for
    shared experts permute 1, FFN 3, combine 1."""
    return 10 + (5 if cfg.num_shared else 0)


def run_ep(args, wl, world: int, rank: int, local: int) -> None:
    """Expert-parallel layer over `world` GPUs: the workload's tokens split evenly over the
    ranks (strong scaling), routed experts sharded, routed rows exchanged over NCCL (each token
    row to each rank that owns one of its experts in fixed segments, partial rows back).  No
    step waits on the host, so the K timed steps replay as one CUDA graph, NCCL calls included;
    the graph is released before the communicator is destroyed."""
    import datetime

    import torch
    import torch.distributed as dist

    from ccut_b200 import build
    from ccut_b200.ep import ExpertParallelMoeLayer
    from ccut_b200.synthetic import make_layer, make_layer_device

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    if rank == 0:  # compile (if stale) once, before the other ranks load the library
        build.build()
    dist.barrier()
    build.build()
    cfg_name, T, bound = WORKLOADS[wl]
    if T % world:
        raise SystemExit(f"{T} tokens do not split over {world} ranks")
    Tl = T // world
    lw = make_layer_device(cfg_name, seed=0, device=dev) if cfg_name in DEVICE_GENERATED else make_layer(cfg_name, seed=0)
    c = lw.cfg
    ep = ExpertParallelMoeLayer(c.fmt, c.hidden, c.inter, c.num_experts, c.top_k, c.routing, lw.router, lw.experts,
                                shared=lw.shared, shared_inter=c.shared_inter, n_group=c.n_group,
                                topk_group=c.topk_group, routed_scaling=c.routed_scaling, device=dev, rank=rank,
                                world=world, timeout_s=120.0)
    xb = lw.make_x(T)[rank * Tl:(rank + 1) * Tl]
    x = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
    del lw
    for _ in range(max(args.warmup, 3)):
        ep.forward(x)
    torch.cuda.synchronize()
    K = args.steps
    graph = None
    if args.graph in ("auto", "on"):
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cap):
            ep.forward(x)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=cap):
                for _ in range(K):
                    ep.forward(x)
        torch.cuda.current_stream().wait_stream(cap)
        torch.cuda.synchronize()
        dist.barrier()
        graph.replay()
        torch.cuda.synchronize()
    def timed_steps():
        if graph is not None:
            graph.replay()
        else:
            for _ in range(K):
                ep.forward(x)

    clocks = ClockSampler(local)
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak:
        timed_steps()
        torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    start.record()
    timed_steps()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    ms = start.elapsed_time(end)
    # end to end: pinned host tokens in, host bf16 out, every step
    x_pin = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).pin_memory()
    e2e_pipelined(ep.forward, x_pin, (Tl, c.hidden), dev, 2)
    dist.barrier()
    torch.cuda.synchronize()
    # median of three repetitions: a host-side stall in one (the leg is launched from Python,
    # not replayed as a graph) does not decide the figure; every rank runs all three
    e2e_ms = statistics.median(e2e_pipelined(ep.forward, x_pin, (Tl, c.hidden), dev, K) for _ in range(3))
    dist.barrier()
    clk = clocks.stop()
    status = ep.workspace_status()
    t = torch.tensor([ms, e2e_ms, float(status != 0)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, bad = float(t[0]), float(t[1]), float(t[2])
    if rank == 0:
        if bad:
            raise SystemExit("device status word reports an expired wait")
        pk, src = peaks()
        flops_rank = layer_flops(c, T) / world
        achieved = flops_rank * K / (ms * 1e-3) / 1e12
        peak = pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        roof = {"bound": "tensor" if bound == "tensor" else "hbm", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                "kernel": "ccut_moe_ep_forward (whole layer per rank, collectives included)",
                "algorithmic_flops_per_rank_step": flops_rank,
                "peak_source": f"{src} (MEASURED_PEAKS.json)" if src == "measured" else "fallback"}
        cfgd = workload_config(wl, 1, f"ep{world}")
        cfgd["tokens_per_gpu"] = Tl
        cfgd["global_tokens"] = T
        cfgd["experts_per_gpu"] = c.num_experts // world
        line = {
            "metric": METRIC, "value": T * K / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16" if T * c.top_k / c.num_experts >= 64 else "f16",
            "data": "synthetic", "config": cfgd, "roofline": roof,
            "e2e": {"value": T * K / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": T * c.hidden * 2,
                    "d2h_bytes_per_step": T * c.hidden * 2},
            "gpu_launches": ep_launches(c) * K,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
            "layer_tflops": layer_flops(c, T) * K / (ms * 1e-3) / 1e12,
            "cuda_graph": graph is not None,
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        graph.reset()  # drop the captured NCCL work before the communicator goes
        graph = None
    torch.cuda.synchronize()
    dist.barrier()
    ep.close()
    dist.destroy_process_group()


def run_ours(args, wl) -> None:
    import torch
    import torch.distributed as dist

    from ccut_b200 import MoeLayer, build
    from ccut_b200.synthetic import make_layer, make_layer_device

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world > 1:
        return run_ep(args, wl, world, rank, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    build.build()
    cfg_name, T, bound = WORKLOADS[wl]
    lw = make_layer_device(cfg_name, seed=0, device=dev) if cfg_name in DEVICE_GENERATED else make_layer(cfg_name, seed=0)
    c = lw.cfg
    L = MoeLayer(c.fmt, c.hidden, c.inter, c.num_experts, c.top_k, c.routing, lw.router, lw.experts,
                 shared=lw.shared, shared_inter=c.shared_inter, n_group=c.n_group, topk_group=c.topk_group,
                 routed_scaling=c.routed_scaling, device=dev)
    xb = lw.make_x(T)
    x = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
    del lw
    use_graph = args.graph == "on" or (args.graph == "auto" and T <= 256)
    # the gate/up launch timed between ev0 and ev1: tcgen05 kernel (plus its activation
    # gather) at >= CCUT_TC_MIN_ROWS mean rows per expert, else mma.sync
    tc_path = T * c.top_k / c.num_experts >= 64
    kname = ("tc_gemm_kernel<gate/up> (with its row gather)" if tc_path else "moe_gemm_kernel<gate/up>")

    def fused():  # the public layer call: one ccut_moe_forward
        return L.forward(x)

    def staged(ev0=None, ev1=None):  # the same layer through its stage entry points
        r = L.route(x)
        p = L.permute(r)
        if ev0 is not None:
            ev0.record()
        h = L.gate_up(x, p)
        if ev1 is not None:
            ev1.record()
        y = L.down(h, p, T)
        return L.combine(y, p, T), p

    # warm-up (also sizes every workspace before any capture)
    for _ in range(max(args.warmup, 3)):
        fused()
        staged()
    torch.cuda.synchronize()
    _, perm = staged()
    offsets = perm.offsets.cpu().numpy()
    K = args.steps
    mk = lambda: torch.cuda.Event(enable_timing=True, external=use_graph)  # noqa: E731
    ev0 = [mk() for _ in range(K)]
    ev1 = [mk() for _ in range(K)]
    g_fused = g_staged = None
    if use_graph:
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fused()
            staged()  # warm the side stream
            torch.cuda.synchronize()
            g_fused, g_staged = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_fused, stream=s):
                for _ in range(K):
                    fused()
            with torch.cuda.graph(g_staged, stream=s):
                for i in range(K):
                    staged(ev0[i], ev1[i])
        torch.cuda.current_stream().wait_stream(s)
        g_fused.replay()
        g_staged.replay()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak:  # steady clocks before the timed region
        if g_fused is not None:
            g_fused.replay()
        else:
            fused()
        torch.cuda.synchronize()
    # value: K fused layer calls, inputs resident in HBM
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    if g_fused is not None:
        g_fused.replay()
    else:
        for _ in range(K):
            fused()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    # roofline kernel: its own pass of K staged steps, events around the gate/up call
    if g_staged is not None:
        g_staged.replay()
    else:
        for i in range(K):
            staged(ev0[i], ev1[i])
    torch.cuda.synchronize()
    kern_ms = [a.elapsed_time(b) for a, b in zip(ev0, ev1)]

    # end to end: host bf16 in (pinned) -> public forward -> host bf16 out, every step
    x_pin = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).pin_memory()
    e2e_pipelined(L.forward, x_pin, (T, c.hidden), dev, 2)  # warm the copy streams
    # median of three repetitions: a host-side stall in one (the leg is launched from Python,
    # not replayed as a graph) does not decide the figure
    e2e_ms = statistics.median(e2e_pipelined(L.forward, x_pin, (T, c.hidden), dev, K) for _ in range(3))
    clk = clocks.stop()
    if L.workspace_status() != 0:
        raise SystemExit("device status word reports an expired wait")

    kmean = statistics.mean(kern_ms)
    if rank == 0:
        pk, src = peaks()
        byts, flops = gate_up_counts(c, offsets)
        if bound == "hbm":
            achieved = byts / (kmean * 1e-3) / 1e9
            peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
            roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": NCU_TRAFFIC.get(wl), "kernel": kname, "algorithmic_bytes_per_launch": byts}
        else:
            achieved = flops / (kmean * 1e-3) / 1e12
            peak = pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
            roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": NCU_TRAFFIC.get(wl), "kernel": kname,
                    "algorithmic_flops_per_launch": flops,
                    "mma": "tcgen05 kind::f16, bf16 operands (the exact weight codes), fp32 scale per 128-k block"}
            if c.fmt == "fp8_b128":
                p8 = fp8_peak_tflops(dev)
                roof["peak_fp8"] = p8
                roof["frac_fp8"] = achieved / p8
                roof["peak_fp8_source"] = "measured in this run: torch._scaled_mm e4m3 8192^3, best of 10"
        roof["peak_source"] = f"{src} (MEASURED_PEAKS.json)" if src == "measured" else "fallback"
        roof["kernel_ms"] = kmean
        launches = 7 if tc_path else 6  # route logits, top-k, permute, [row gather], gate/up, down, combine
        line = {
            "metric": METRIC, "value": T * K / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if tc_path else "f16", "data": "synthetic",
            "config": dict(workload_config(wl, 1, "single"),
                           weights={"fp8_b128": "fp8 e4m3, 128x128 fp32 block scales",
                                    "awq_int4_g128": "awq int4, group 128, fp16 scales, packed zero points"}[c.fmt],
                           path="ccut_moe_forward (fused C entry point)"),
            "roofline": roof,
            "e2e": {"value": T * K / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T * c.hidden * 2, "d2h_bytes_per_step": T * c.hidden * 2},
            "gpu_launches": launches * K,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
            "layer_tflops": layer_flops(c, T) * K / (ms * 1e-3) / 1e12,
            "cuda_graph": use_graph,
        }
        if cfg_name in DEVICE_GENERATED:
            line["data"] = "synthetic (generated on the GPU from a seeded torch generator)"
        if not args.no_cpu_baseline and cfg_name not in DEVICE_GENERATED:
            sample = T if args.cpu_sample <= 0 else min(T, args.cpu_sample)
            r = cpu_sample_run(cfg_name, T, sample, 1, args.cpu_budget)
            line["cpu_baseline"] = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    del g_fused, g_staged


# Attention block of the full stacks (not the MoE layer): name -> (batch, heads, kv_heads,
# seq, kv_len, head_dim).  cfg3: Qwen3-30B-A3B GQA (32 query heads, 4 kv heads, head dim
# 128), batch-64 decode over a 4096-position bf16 kv cache.
ATTN_WORKLOADS = {"cfg3_attn_decode": (64, 32, 4, 1, 4096, 128)}
# DeepSeek-V2-Lite MLA decode (config 2's attention): batch, heads, seq, kv_len; latent 512 + rope 64
MLA_WORKLOADS = {"cfg2_mla_decode": (64, 16, 1, 4096)}
# whole-model decode through the engine backend: a Qwen3-30B-A3B-shaped decoder (config 3's MoE
# layer, GQA 32 / 4 heads of 128, 48 layers, vocab 151936), `batch` requests with `prompt`-token
# prompts, one generate_batch call per step
ENGINE_WORKLOADS = {"cfg3_engine_decode": {"moe": "cfg3", "layers": 48, "heads": 32, "kv_heads": 4, "head_dim": 128,
                                           "vocab": 151936, "batch": 8, "prompt": 512, "pool": False}}
# the same with the requests' caches in one pool: one attention launch per layer and step
ENGINE_WORKLOADS["cfg3_engine_decode_pool"] = dict(ENGINE_WORKLOADS["cfg3_engine_decode"], pool=True)
# config 2: the DeepSeek-V2-Lite-shaped stack -- 27 layers, layer 0 a dense FFN of intermediate
# 10944, the others config 0's AWQ MoE layer; MLA attention (16 heads, kv rank 512, nope 128,
# rope 64, v 128); vocab 102400; 2048-token prompts, then decode at batch 32 and batch 1
ENGINE_WORKLOADS["cfg2_engine_decode"] = {"moe": "cfg0", "layers": 27, "attn": "mla", "heads": 16, "d_nope": 128,
                                          "d_rope": 64, "d_v": 128, "dense_layers": 1, "dense_inter": 10944,
                                          "vocab": 102400, "batch": 32, "prompt": 2048, "pool": False}
ENGINE_WORKLOADS["cfg2_engine_decode_b1"] = dict(ENGINE_WORKLOADS["cfg2_engine_decode"], batch=1)
# batch 32 with the latent caches in one pool: one MLA launch per layer and step
ENGINE_WORKLOADS["cfg2_engine_decode_pool"] = dict(ENGINE_WORKLOADS["cfg2_engine_decode"], pool=True)


def run_attn(args, wl) -> None:
    """One GQA attention call per step (ccut_gqa_attention) on device-resident q / k / v;
    roofline: the K and V bytes read (the kv cache exceeds the L2)."""
    import torch

    from ccut_b200 import _lib, build
    from ccut_b200.layer import _ptr, _stream

    if int(os.environ.get("RANK", "0")) != 0:
        return
    build.build()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    b, h, kvh, s, L, d = ATTN_WORKLOADS[wl]
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((b, h, s, d), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((b, kvh, L, d), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((b, kvh, L, d), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty((b, h, s, d), dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    ws = torch.zeros(max(lib.ccut_gqa_attention_workspace_bytes(b, h, kvh, s, L, d), 256), dtype=torch.uint8,
                     device=dev)

    def step():
        _lib.call("ccut_gqa_attention", _ptr(q), _ptr(k), _ptr(v), b, h, kvh, s, L, d, L - s, 0.0, 0.0, _ptr(out),
                  _lib.OUT_BF16, _ptr(ws), ws.numel(), _stream())

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index or 0)
    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(K):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    clk = clocks.stop()
    pk, src = peaks()
    kv_bytes = 2 * b * kvh * L * d * 2
    byts = kv_bytes + 2 * b * h * s * d * 2
    achieved = byts * K / (ms * 1e-3) / 1e9
    peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    print(json.dumps({
        "metric": "GQA attention tokens/s", "value": b * s * K / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1,
        "steps": K, "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 in, f32 accumulate", "data": "synthetic (seeded torch generator)",
        "config": {"workload": wl, "batch": b, "heads": h, "kv_heads": kvh, "seq": s, "kv_len": L, "head_dim": d,
                   "l2": f"kv cache {kv_bytes / 1e6:.0f} MB > 126 MB L2, no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": "gqa_attn_kernel + gqa_combine_kernel",
                     "algorithmic_bytes_per_launch": byts,
                     "peak_source": f"{src} (MEASURED_PEAKS.json)" if src == "measured" else "fallback"},
        "gpu_launches": 2 * K,
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
    }), flush=True)


def run_mla(args, wl) -> None:
    """One MLA latent attention call per step (ccut_mla_attention) on device-resident q and
    latent cache; roofline: the cache bytes read (the cache exceeds the L2)."""
    import torch

    from ccut_b200 import _lib, build
    from ccut_b200.layer import _ptr, _stream

    if int(os.environ.get("RANK", "0")) != 0:
        return
    build.build()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    b, h, s, L = MLA_WORKLOADS[wl]
    width = 512 + 64
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    q = torch.randn((b, s * h, width), generator=g, device=dev)
    kv = torch.randn((b, L, width), generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty((b, s * h, 512), dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = torch.zeros(max(lib.ccut_mla_attention_workspace_bytes(b, h, s, L), 256), dtype=torch.uint8, device=dev)
    scale = 1.0 / (192 ** 0.5)

    def step():
        _lib.call("ccut_mla_attention", _ptr(q), _ptr(kv), b, h, s, L, 512, 64, L - s, scale, _ptr(out),
                  _lib.OUT_F32, _ptr(ws), ws.numel(), _stream())

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index or 0)
    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(K):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    clk = clocks.stop()
    pk, src = peaks()
    kv_bytes = b * L * width * 2
    byts = kv_bytes + b * s * h * (width + 512) * 4
    achieved = byts * K / (ms * 1e-3) / 1e9
    peak = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    split = lib.ccut_mla_attention_workspace_bytes(b, h, s, L) > 256
    print(json.dumps({
        "metric": "MLA attention tokens/s", "value": b * s * K / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1,
        "steps": K, "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 latent cache, f32 accumulate", "data": "synthetic (seeded torch generator)",
        "config": {"workload": wl, "batch": b, "heads": h, "seq": s, "kv_len": L, "latent": 512, "rope": 64,
                   "l2": f"latent cache {kv_bytes / 1e6:.0f} MB > 126 MB L2, no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": "mla_attn_kernel" + (" + gqa_combine_kernel" if split else ""),
                     "algorithmic_bytes_per_launch": byts,
                     "peak_source": f"{src} (MEASURED_PEAKS.json)" if src == "measured" else "fallback"},
        "gpu_launches": (2 if split else 1) * K,
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
    }), flush=True)


def engine_model(w: dict, dev):
    """The seeded synthetic ``MoeDecoder`` of engine workload ``w`` on ``dev``: config
    ``w["moe"]``'s MoE layer (a ``DenseFfn`` in the first ``dense_layers`` layers), GQA or MLA
    attention with bf16 projections, a random embedding and ``lm_head``."""
    import torch

    from ccut_b200.dense import DenseFfn
    from ccut_b200.layer import MoeLayer
    from ccut_b200.model import DecoderLayer, MlaDecoderLayer, MoeDecoder, rope_table
    from ccut_b200.synthetic import CONFIGS, _gen_matrix, make_layer_device

    c = CONFIGS[w["moe"]]
    mla = w.get("attn") == "mla"
    H, nh = c.hidden, w["heads"]
    kvh, d = (1, w["d_rope"]) if mla else (w["kv_heads"], w["head_dim"])
    g = torch.Generator(device=dev)
    g.manual_seed(0)

    def mat(o, i):
        return (torch.randn((o, i), generator=g, device=dev) / i ** 0.5).to(torch.bfloat16)

    def norm_w(n):
        return torch.rand((n,), generator=g, device=dev) + 0.5

    def dense_ffn(i):  # seeded AWQ / FP8 SwiGLU; the down projection drawn over the padded intermediate
        rng = np.random.default_rng(1000 + i)
        inter = w["dense_inter"]
        ip = -(-inter // 128) * 128
        return DenseFfn(c.fmt, H, inter, _gen_matrix(rng, c.fmt, H, inter), _gen_matrix(rng, c.fmt, H, inter),
                        _gen_matrix(rng, c.fmt, ip, H), device=dev, workspaces=ws)

    ws: dict = {}  # one set of FFN workspaces for all layers (they run one after another)
    layers = []
    for i in range(w["layers"]):
        if i < w.get("dense_layers", 0):
            ffn = dense_ffn(i)
        else:
            lw = make_layer_device(c, seed=i, device=dev)
            ffn = MoeLayer(c.fmt, c.hidden, c.inter, c.num_experts, c.top_k, c.routing, lw.router, lw.experts,
                           shared=lw.shared or None, shared_inter=c.shared_inter or None, device=dev, workspaces=ws)
        if mla:
            dn, dr, dv = w["d_nope"], w["d_rope"], w["d_v"]
            layers.append(MlaDecoderLayer(norm_w(H), mat(nh * (dn + dr), H), mat(512 + dr, H), mat(nh * (dn + dv), 512),
                                          mat(H, nh * dv), norm_w(H), ffn, norm_w(512), heads=nh, qk_nope_head_dim=dn,
                                          qk_rope_head_dim=dr, v_head_dim=dv, device=dev))
        else:
            layers.append(DecoderLayer(norm_w(H), mat(nh * d, H), mat(kvh * d, H), mat(kvh * d, H), mat(H, nh * d),
                                       norm_w(H), ffn, norm_w(d), norm_w(d), heads=nh, kv_heads=kvh, head_dim=d,
                                       device=dev))
    inv, af = rope_table(d, 1e4 if mla else 1e6)
    return MoeDecoder(torch.randn((w["vocab"], H), generator=g, device=dev), layers, norm_w(H), mat(w["vocab"], H),
                      inv_freq=inv, attention_factor=af, device=dev)


def run_engine(args, wl) -> None:
    """Decode steps of a whole synthetic model (``engine_model``) through
    ``GenericBackend.generate_batch`` (the call an engine step makes): every step runs one new
    token per request through all layers (bf16 projections on cuBLAS, RMSNorm / RoPE / GQA or
    MLA attention / the MoE layer and the dense FFN on this library's kernels) and samples
    greedily on the device."""
    import torch

    from ccut_b200 import build
    from ccut_b200.backend import GenericBackend

    if int(os.environ.get("RANK", "0")) != 0:
        return
    build.build()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    w = ENGINE_WORKLOADS[wl]
    mla = w.get("attn") == "mla"
    nh = w["heads"]
    kvh, d = (1, w["d_rope"]) if mla else (w["kv_heads"], w["head_dim"])
    dec = engine_model(w, dev)
    B, P = w["batch"], w["prompt"]
    be = GenericBackend(dec, max_seqs=B, max_len=P + args.warmup + args.steps + 8, prefill_chunk=P, pool=w["pool"])
    rng = np.random.default_rng(0)
    seqs = [[int(x) for x in rng.integers(0, w["vocab"], P)] for _ in range(B)]
    greedy = {"temperature": 0.0}

    def step():
        for s, tok in zip(seqs, be.generate_batch([(s, greedy) for s in seqs])):
            s.append(tok)

    step()  # the prompts (prefill), untimed
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index or 0)
    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record()
    for _ in range(K):
        step()
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = start.elapsed_time(end)
    clk = clocks.stop()
    print(json.dumps({
        "metric": "engine decode tokens/s", "value": B * K / (ms * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 activations, AWQ int4 experts, f32 accumulate", "data": "synthetic (seeded torch generator)",
        "config": {"workload": wl, "layers": w["layers"], "batch": B, "prompt": P, "moe": w["moe"], "pool": w["pool"],
                   "attention": "mla (rank 512, nope / rope / v = %d / %d / %d)" % (w["d_nope"], d, w["d_v"]) if mla
                   else "gqa", "heads": nh, "kv_heads": kvh, "head_dim": d, "vocab": w["vocab"],
                   "dense_layers": w.get("dense_layers", 0),
                   "l2": "expert weights of every layer exceed the 126 MB L2, no flush"},
        "e2e": {"value": B * K / wall, "unit": "tokens/s", "h2d_bytes_per_step": B * 8 * 2,
                "d2h_bytes_per_step": B * 8},
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
    }), flush=True)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(ATTN_WORKLOADS) + sorted(MLA_WORKLOADS)
                    + sorted(ENGINE_WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--graph", choices=("auto", "on", "off"), default="auto")
    ap.add_argument("--soak", type=float, default=1.0, help="untimed seconds of load before timing")
    ap.add_argument("--cpu-sample", type=int, default=0,
                    help="tokens per CPU-baseline call (0: the whole batch of the workload)")
    ap.add_argument("--cpu-budget", type=float, default=120.0, help="seconds cap of the cpu_baseline leg")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.workload in ATTN_WORKLOADS or args.workload in MLA_WORKLOADS or args.workload in ENGINE_WORKLOADS:
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the MoE layer; the "
                              "attention and engine workloads have no reference timing"}), flush=True)
        elif args.workload in ENGINE_WORKLOADS:
            run_engine(args, args.workload)
        elif args.workload in MLA_WORKLOADS:
            run_mla(args, args.workload)
        else:
            run_attn(args, args.workload)
    elif args.impl == "reference":
        run_reference(args, args.workload)
    else:
        run_ours(args, args.workload)
    return 0


if __name__ == "__main__":
    sys.exit(main())
