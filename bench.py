#!/usr/bin/env python
"""MSDA forward + backward benchmark on B200 (BEVFormer-base spatial cross-attention).

One *step* is the reference benchmark's ``forward-backward`` scope
(``benchmarks/msda/benchmark_msda.py:85-119`` in the muSPACE tree): the forward
launch, the zero fill of the fp32 ``grad_value`` accumulator and the backward
launch, through the C-ABI (``ms_deform_attn_forward`` / ``ms_deform_attn_backward``)
on device-resident inputs. The workload is BASELINE config 4: the c2 shapes
(6 cameras x 4 levels [(116,200),(58,100),(29,50),(15,25)], Lq=10000, 8 heads x
32 channels, 8 points) at batch 8 x 6 cameras = 48 images, bf16 storage with fp32
accumulation, 10% of the locations out of bounds. Inputs are seeded synthetic
tensors (no dataset) and total 1.7 GB, far beyond the 126 MB L2, so no flush is
needed between steps.

``value`` is effective GB/s: the algorithmic (compulsory) bytes of the step
(fwd: value + locations + weights + output; bwd: the same reads plus fp32
writes of the three gradients) over the device time, whole job. With N GPUs the
48 images of config 4 are split across the ranks, 48 / N each (strong scaling,
config 4 as stated: one batch sharded by batch x camera, no collective on the
data path), and the time is the slowest rank's; ``--scaling weak`` gives every
rank its own 48-image shard instead. ``--variant query`` runs the bs=1 form: one
6-camera sample, queries split across ranks, value replicated, fp32
``grad_value`` reduce-scattered with NCCL; its ``kernels_ms`` separate the
kernels from the reduce-scatter. At N = 1 the line also carries
``other_workloads``: 10-step device times of the other configs (c0-c3, the
reference's ``bevformer-1l``) and of the ops built next to MSDA.
``--protocol reference`` times the reference's
published-case protocol instead (20 warm-ups, 5 repeats x 100 launches, median;
``benchmarks/_harness.py:226-260``) for both the reference's timed closure and
this build's step, next to the published figures.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from muspace_b200 import cases  # noqa: E402

METRIC = "MSDA fwd+bwd µs & effective HBM GB/s (BEVFormer-base SCA), 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 2**20


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--config", default=None, choices=sorted(cases.CONFIGS),
                   help="default: c4 (bevformer-1l with --protocol reference)")
    p.add_argument("--dtype", choices=("bfloat16", "float32"), default=None)
    p.add_argument("--scaling", choices=("weak", "strong"), default="strong",
                   help="strong (default): the workload's images split across the ranks; weak: a whole workload per rank")
    p.add_argument("--variant", choices=("batch", "query"), default="batch")
    p.add_argument("--per-image", action="store_true",
                   help="--variant query: backward and grad_value reduce-scatter per camera image, overlapped")
    p.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    p.add_argument("--e2e-streams", type=int, default=1,
                   help="copy streams per direction in the end-to-end leg (a tensor always on the same one)")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    p.add_argument("--no-other-workloads", action="store_true",
                   help="skip the short device-time runs of the other configs and ops (N = 1 only)")
    p.add_argument("--quiet", action="store_true", help="print only the JSON line")
    p.add_argument("--protocol", choices=("contract", "reference"), default="contract",
                   help="reference: the reference's published-case timing protocol (p50 of 5 x 100 launches)")
    p.add_argument("--op", choices=("msda", "deformable_aggregation", "flash_sca", "sca_scatter"), default="msda",
                   help="msda (default: the headline workload) or one of the ops built next to it")
    return p.parse_args()


# --------------------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------------------


def _dtype(args, cfg) -> torch.dtype:
    name = args.dtype or cfg.dtypes[0]
    return {"bfloat16": torch.bfloat16, "float32": torch.float32}[name]


def _dtype_tag(dtype) -> str:
    return {torch.bfloat16: "bf16", torch.float32: "f32"}[dtype]


def _peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs: STREAM-style copy)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (6.65 TB/s, earlier measurement on this pool)"


# Payload rate of red.global.add.v4.f32 into an L2-resident region with 128 B
# per 8-lane group (whole lines), measured on this pool's B200s (6.34-6.39
# TB/s over 296-1184 CTAs); bulk reductions from shared memory reached less.
RED_PEAK_GBS = 6390.0
RED_PEAK_SOURCE = ("measured: red.global.add.v4.f32, 128-byte lines into an L2-resident region (B200; method and "
                   "results in profiles/red_path_microbenchmarks.md)")


def _red_bytes(kernel: str, launch_units: float):
    """RED payload bytes per launch from the committed ncu summary, scaled by units."""
    try:
        entry = json.loads((ROOT / "profiles" / "dram_traffic.json").read_text())[kernel]
        return entry["red_bytes"] / entry["units"] * launch_units
    except Exception:
        return None


def _traffic(kernel: str, workload: str, launch_units: float):
    """DRAM bytes per launch from the committed ncu summary, scaled by units."""
    path = ROOT / "profiles" / "dram_traffic.json"
    try:
        entry = json.loads(path.read_text())[kernel]
    except Exception:
        return None, None
    per_unit = entry["dram_bytes"] / entry["units"]
    return per_unit * launch_units, entry.get("source")


class Clocks:
    """Samples nvidia-smi during the timed region (5 Hz)."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        if self.proc is None or not getattr(self, "out", ""):
            return None
        rows = [r.split(",") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        power = [float(r[3]) for r in rows if r[3].strip().replace(".", "").isdigit()]
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(rows),
            "power_w_max": max(power) if power else None,
        }


# --------------------------------------------------------------------------------------
# CPU legs (the oracle port of the reference's PyTorch path)
# --------------------------------------------------------------------------------------


def _cpu_sample_cfg(cfg):
    """One camera image of the workload: about 1 s of fwd+bwd on 8 host threads."""
    return cfg.with_(batch=1)


def cpu_time_per_call(cfg, dtype, reps: int, warmup: int = 1):
    from oracle.msda_torch import msda_grid_sample_fwd_bwd

    torch.set_num_threads(os.cpu_count() or 1)
    sample = _cpu_sample_cfg(cfg)
    inp = cases.make_inputs(sample, dtype=dtype, seed=2333)
    # the reference's PyTorch path runs in the storage dtype's fp32 form on CPU
    args = [inp[k].float() if inp[k].dtype.is_floating_point else inp[k] for k in
            ("value", "spatial_shapes", "sampling_locations", "attention_weights", "grad_output")]
    for _ in range(warmup):
        msda_grid_sample_fwd_bwd(*args)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        msda_grid_sample_fwd_bwd(*args)
        times.append(time.perf_counter() - t0)
    nbytes = cases.compulsory_bytes(sample, dtype)["total"]
    return times, nbytes, sample, torch.get_num_threads()


def cpu_baseline(cfg, dtype):
    times, nbytes, sample, cores = cpu_time_per_call(cfg, dtype, reps=3)
    t = statistics.median(times)
    return {
        "value": round(nbytes / t / 1e9, 4),
        "unit": "GB/s",
        "cores": cores,
        "kind": "port",
        "sample": (
            f"{sample.name} shapes at batch 1 (one camera image of the workload), fwd+bwd of the reference's "
            f"PyTorch grid_sample formulation (oracle/msda_torch.py) on CPU tensors, median of 3 after 1 warm-up; "
            f"{t * 1e3:.1f} ms per call, {nbytes / 1e6:.1f} MB compulsory"
        ),
        "ms_per_call": round(t * 1e3, 3),
    }


def run_reference(args, cfg, dtype, rank: int):
    if rank != 0:
        return
    times, nbytes, sample, cores = cpu_time_per_call(cfg, dtype, reps=args.steps, warmup=args.warmup)
    total = sum(times)
    value = nbytes * len(times) / total / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total / len(times) * 1e3, 3),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": _dtype_tag(dtype),
        "data": "synthetic",
        "config": {"workload": _workload_name(cfg, dtype, args), "sample": f"{sample.name} at batch 1"},
        "cpu_baseline": {
            "value": round(value, 4),
            "unit": "GB/s",
            "cores": cores,
            "kind": "port",
            "sample": "one camera image per step (batch 1 of the workload), reference PyTorch grid_sample path "
                      "restated in oracle/msda_torch.py, fwd+bwd on CPU tensors",
        },
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _workload_name(cfg, dtype, args) -> str:
    if args.variant == "query":
        return f"config 4 bs=1 variant: {cfg.name} shapes at batch 6, queries split across ranks, grad_value reduce-scatter"
    label = "config 4: BEVFormer-base SCA MSDA fwd+bwd" if cfg.name == "c4" else f"{cfg.name}: {cfg.description}"
    return (
        f"{label}, {cfg.batch} images per {'rank' if args.scaling == 'weak' else 'job'}, "
        f"{_dtype_tag(dtype)} storage, fp32 accumulate"
    )


# --------------------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------------------


class Step:
    """Device buffers and the two C-ABI calls of one forward-backward step."""

    def __init__(self, inp: dict, dtype, device):
        from muspace_b200.runtime.native import native_function

        self.fwd = native_function("ms_deform_attn_forward")
        self.bwd = native_function("ms_deform_attn_backward")
        self.inp = inp
        self.names = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")
        self.out = torch.empty(inp["grad_output"].shape, dtype=dtype, device=device)
        self.gv = torch.zeros(inp["value"].shape, dtype=torch.float32, device=device)
        self.gl = torch.empty(inp["sampling_locations"].shape, dtype=torch.float32, device=device)
        self.gw = torch.empty(inp["attention_weights"].shape, dtype=torch.float32, device=device)

    def __call__(self, events=None):
        a = [self.inp[n] for n in self.names]
        if events:
            events[0].record()
        self.fwd(*a, self.out, 64)
        if events:
            events[1].record()
        self.gv.zero_()
        if events:
            events[2].record()
        # the reference's forward-backward scope makes grad_output contiguous
        # inside the timed region (benchmarks/msda/benchmark_msda.py:110-117)
        self.bwd(*a, self.inp["grad_output"].contiguous(), self.gv, self.gl, self.gw, 64)
        if events:
            events[3].record()


def run_b200(args, cfg, dtype, rank, world, device):
    import torch.distributed as dist

    distributed = world > 1
    if args.variant == "query":
        return run_query_variant(args, cfg, dtype, rank, world, device)
    if args.scaling == "strong":
        from muspace_b200.sharding import shard_range

        b0, b1 = shard_range(cfg.batch, world, rank)
        if b1 == b0:
            raise SystemExit(f"strong scaling: {world} ranks for {cfg.batch} images leaves rank {rank} without work")
        local = cfg.with_(batch=b1 - b0)
        job_total = cases.compulsory_bytes(cfg, dtype)["total"]
    else:
        local = cfg
        job_total = cases.compulsory_bytes(cfg, dtype)["total"] * world
    inp = cases.make_inputs(local, dtype=dtype, seed=2333 + 7919 * rank, device=device)
    step = Step(inp, dtype, device)
    units = cases.compulsory_bytes(local, dtype)
    fwd_bytes, bwd_bytes = units["fwd"], units["bwd"]
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # per-kernel durations: a separate pass with events between the launches
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    for e in ev:
        step(e)
    torch.cuda.synchronize()
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    fill_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    bwd_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in ev)

    # the timed region: K steps bracketed by a barrier and a synchronize
    if distributed:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(device.index) as clocks:
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
    if distributed:
        dist.barrier()
    elapsed_ms = start.elapsed_time(end)
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
    if distributed:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = job_total * args.steps / (elapsed_ms / 1e3) / 1e9

    e2e = None if args.no_e2e else run_e2e(args, local, dtype, inp, device, job_total, distributed)

    if rank != 0:
        return None
    peak, peak_src = _peaks()
    dominant, dom_ms, dom_bytes = ("ms_deformable_backward", bwd_ms, bwd_bytes) if bwd_ms >= fwd_ms else (
        "ms_deformable_forward", fwd_ms, fwd_bytes)
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    traffic, traffic_src = _traffic(dominant, local.name, local.batch)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "us_per_call": round(ms_per_step * 1e3, 1),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": _dtype_tag(dtype),
        "data": "synthetic",
        "config": {
            "workload": _workload_name(cfg, dtype, args),
            "batch_per_rank": local.batch,
            "global_batch": cfg.batch if args.scaling == "strong" else cfg.batch * world,
            "queries": local.queries,
            "levels": [list(s) for s in local.shapes],
            "points": local.points,
            "heads": local.heads,
            "channels": local.channels,
            "parallelism": (f"batch x camera sharded over {world} ranks (no collective)" if world > 1
                            else "one GPU"),
            "l2": f"inputs {sum(t.numel() * t.element_size() for t in inp.values()) / 1e9:.2f} GB per rank > 126 MB L2; no flush",
            "scope": "forward launch + grad_value zero fill + backward launch through the C-ABI (reference forward-backward scope)",
            "compulsory_bytes_per_step_per_rank": fwd_bytes + bwd_bytes,
        },
        "kernels_ms": {"forward": round(fwd_ms, 4), "grad_value_fill": round(fill_ms, 4), "backward": round(bwd_ms, 4)},
        "roofline": {
            "bound": "hbm",
            "kernel": dominant,
            "achieved": round(achieved, 1),
            "peak": peak,
            "peak_source": peak_src,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": None if traffic is None else int(traffic),
            "traffic_source": traffic_src,
            "algorithmic_bytes": dom_bytes,
        },
        "gpu_launches": 2 * args.steps * world,
        "gpu_launches_per_rank": 2 * args.steps,
        "clocks": clocks.summary(),
        "e2e": e2e,
    }
    red = _red_bytes("ms_deformable_backward", local.batch)
    if red is not None:
        # the limit that binds the backward: its grad_value RED payload (ncu)
        # against the rate L2 reductions reach at best
        red_gbs = red / (bwd_ms / 1e3) / 1e9
        line["reduction_roofline"] = {
            "bound": "L2 reductions", "kernel": "ms_deformable_backward", "achieved": round(red_gbs, 1),
            "peak": RED_PEAK_GBS, "unit": "GB/s", "frac": round(red_gbs / RED_PEAK_GBS, 4),
            "payload_bytes": int(red), "peak_source": RED_PEAK_SOURCE}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, dtype)
    if world == 1 and not args.no_other_workloads:
        line["other_workloads"] = other_workloads(device)
    return line


# The other BASELINE configs and the reference's published case, each as the
# headline's step (forward, grad_value fill, backward) on device-resident inputs.
OTHER_CONFIGS = (("c0", torch.float32), ("c1", torch.float32), ("c1", torch.bfloat16), ("c2", torch.bfloat16),
                 ("c3", torch.bfloat16), ("bevformer-1l", torch.float32), ("bevformer-1l", torch.bfloat16))
OTHER_OPS = ("deformable_aggregation", "flash_sca", "sca_scatter")


def _time_steps(step, steps=10, warmup=3, phases=None):
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def other_workloads(device):
    """Device time per step of every other config (c0-c3, bevformer-1l) and of
    the ops built next to MSDA, 10 timed steps after 3 warm-ups each (inputs
    resident on the device, so their own bench lines' e2e and CPU legs are
    left out): the configs as the headline's step, the ops as their own
    ``--op`` step."""
    out = {}
    for name, dtype in OTHER_CONFIGS:
        cfg = cases.CONFIGS[name]
        inp = cases.make_inputs(cfg, dtype=dtype, device=device)
        step = Step(inp, dtype, device)
        ms = _time_steps(step)
        nbytes = cases.compulsory_bytes(cfg, dtype)["total"]
        out[f"{name}/{_dtype_tag(dtype)}"] = {"ms_per_step": round(ms, 4),
                                              "gbs": round(nbytes / (ms / 1e3) / 1e9, 1)}
        del inp, step
        torch.cuda.empty_cache()
    for op in OTHER_OPS:
        w = OpWorkload(op, device)
        ms = _time_steps(w.step)
        out[op] = {"ms_per_step": round(ms, 4), "gbs": round(w.bytes / (ms / 1e3) / 1e9, 1)}
        del w
        torch.cuda.empty_cache()
    return out


class E2ESlot:
    """One set of device buffers of the end-to-end leg: ``inputs`` receive the
    host copies, ``step()`` runs the op through the C-ABI, ``outputs`` go back."""

    def __init__(self, inputs, outputs, step):
        self.inputs, self.outputs, self.step = inputs, outputs, step


def _spread(tensors, n: int) -> list[int]:
    """Stream index of each tensor: largest first onto the least-loaded of n."""
    load = [0] * n
    where = [0] * len(tensors)
    for k in sorted(range(len(tensors)), key=lambda k: -tensors[k].numel() * tensors[k].element_size()):
        w = min(range(n), key=lambda x: load[x])
        where[k] = w
        load[w] += tensors[k].numel() * tensors[k].element_size()
    return where


def pipelined_e2e(slots, host_in, steps: int, distributed: bool, device, copy_streams: int = 1) -> float:
    """Device time per step of ``steps`` end-to-end steps, each with the H2D
    copy of its inputs from pinned host memory and the D2H copy of all its
    outputs, double-buffered over ``slots`` (two sets of device buffers): the
    H2D of step i + 1 and the D2H of step i - 1 overlap the compute of step i,
    and the two copy directions run concurrently (PCIe is full duplex). Each
    direction's copies are spread over ``copy_streams`` streams (a tensor
    always on the same one). A slot's inputs are rewritten only after its
    previous compute, and its outputs only after their previous D2H. Max over
    ranks."""
    import torch.distributed as dist

    s_comp = torch.cuda.Stream(device)
    s_in = [torch.cuda.Stream(device) for _ in range(copy_streams)]
    s_out = [torch.cuda.Stream(device) for _ in range(copy_streams)]
    # one pinned output set: a tensor's D2H copies of the slots run one after
    # another on its stream, so they never write it at the same time (and a
    # rank pins its inputs and outputs once, not twice, which matters with 8
    # ranks a node)
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in slots[0].outputs]
    in_where, out_where = _spread(host_in, copy_streams), _spread(host_out, copy_streams)
    in_done = [[torch.cuda.Event() for _ in s_in] for _ in slots]
    comp_done = [torch.cuda.Event() for _ in slots]
    out_done = [[torch.cuda.Event() for _ in s_out] for _ in slots]

    def one(i):
        j = i % len(slots)
        slot = slots[j]
        for k, s in enumerate(s_in):
            s.wait_event(comp_done[j])
            with torch.cuda.stream(s):
                for dst, src, w in zip(slot.inputs, host_in, in_where):
                    if w == k:
                        dst.copy_(src, non_blocking=True)
            in_done[j][k].record(s)
        for e in in_done[j] + out_done[j]:
            s_comp.wait_event(e)
        with torch.cuda.stream(s_comp):
            slot.step()
        comp_done[j].record(s_comp)
        for k, s in enumerate(s_out):
            s.wait_event(comp_done[j])
            with torch.cuda.stream(s):
                for dst, src, w in zip(host_out, slot.outputs, out_where):
                    if w == k:
                        dst.copy_(src, non_blocking=True)
            out_done[j][k].record(s)

    for i in range(len(slots)):  # warm-up: every slot once
        one(i)
    torch.cuda.synchronize(device)
    if distributed:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in[0])
    for s in s_in[1:] + [s_comp] + s_out:
        s.wait_event(start)
    for i in range(steps):
        one(i)
    main = torch.cuda.current_stream(device)
    for s in s_in + [s_comp] + s_out:
        main.wait_stream(s)
    end.record(main)
    torch.cuda.synchronize(device)
    t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
    if distributed:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()) / steps


E2E_PATH = ("pinned host buffers -> cudaMemcpyAsync H2D -> {calls} (C-ABI) -> cudaMemcpyAsync D2H -> pinned host; "
            "two device buffer sets, compute on one stream, H2D and D2H on {streams} stream(s) each")


def run_e2e(args, local, dtype, inp, device, job_total, distributed):
    """The same step through the C-ABI with host buffers: pinned H2D of the
    inputs and D2H of the output and the three gradients, every step."""
    keys = [k for k in inp if k not in ("spatial_shapes", "level_start_index")]
    host_in = [inp[k].cpu().pin_memory() for k in keys]
    slots = []
    for _ in range(2):
        dev_in = {k: (v if k in ("spatial_shapes", "level_start_index") else v.clone()) for k, v in inp.items()}
        step = Step(dev_in, dtype, device)
        slots.append(E2ESlot([dev_in[k] for k in keys], [step.out, step.gv, step.gl, step.gw], step))
    steps = max(3, min(args.steps, 10))
    ms = pipelined_e2e(slots, host_in, steps, distributed, device, args.e2e_streams)
    return {
        "value": round(job_total / (ms / 1e3) / 1e9, 3),
        "unit": "GB/s",
        "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host_in),
        "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in slots[0].outputs),
        "ms_per_step": round(ms, 3),
        "steps": steps,
        "path": E2E_PATH.format(calls="ms_deform_attn_forward/backward", streams=args.e2e_streams),
    }


def run_query_variant(args, cfg, dtype, rank, world, device):
    from muspace_b200.sharding import QueryShardedStep

    sample = cases.CONFIGS["c2"].with_(locations=cfg.locations)
    inp = cases.make_inputs(sample, dtype=dtype, seed=2333, device=device)
    step = QueryShardedStep(inp, dtype, rank, world, per_image=args.per_image)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(device.index) as clocks:
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    nbytes = cases.compulsory_bytes(sample, dtype)["total"]
    # per-phase device time (whole-batch exchange): events between the
    # launches on the current stream, a separate pass after the timed one
    kernels_ms = None
    if not args.per_image:
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
        for e in ev:
            step(e)
        torch.cuda.synchronize()
        phases = torch.tensor([statistics.mean(e[i].elapsed_time(e[i + 1]) for e in ev) for i in range(4)],
                              dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(phases, op=dist.ReduceOp.MAX)
        kernels_ms = {k: round(float(v), 4) for k, v in
                      zip(("forward", "grad_value_fill", "backward", "reduce_scatter"), phases.tolist())}
    if rank != 0:
        return None
    return {
        "metric": METRIC,
        "value": round(nbytes / (ms / 1e3) / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "us_per_call": round(ms * 1e3, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": _dtype_tag(dtype),
        "data": "synthetic",
        "config": {"workload": _workload_name(sample, dtype, args),
                   "parallelism": (f"query-sharded x{world} + per-image NCCL reduce_scatter(grad_value) overlapped "
                                   "with the next image's backward") if args.per_image and world > 1 else
                                  f"query-sharded x{world} + NCCL reduce_scatter(grad_value)"},
        "kernels_ms": kernels_ms,
        "gpu_launches": (1 + sample.batch if args.per_image and world > 1 else 2) * args.steps * world,
        "clocks": clocks.summary(),
    }


# --------------------------------------------------------------------------------------
# the ops next to MSDA (--op): one JSON line each, same contract as the headline
# --------------------------------------------------------------------------------------


def _nbytes(*tensors) -> int:
    return sum(t.numel() * t.element_size() for t in tensors)


class OpWorkload:
    """One op's step on device buffers, as a list of phases (name, call,
    algorithmic bytes, our kernel launches; the fills that the reference's
    autograd performs count no bytes and no launches). ``inputs`` / ``outputs``
    are the tensors e2e copies in / out, ``bytes`` the compulsory HBM bytes of
    a step, ``dominant`` the phase the roofline is quoted on with its
    ``profiles/dram_traffic.json`` key and units (launch_units)."""

    def __init__(self, op: str, device):
        from muspace_b200.runtime.native import native_function

        self.op = op
        if op == "deformable_aggregation":
            (mc, sp, st, loc, w), grad = cases.deformable_aggregation_inputs(device)
            out = torch.empty(mc.shape[0], loc.shape[1], mc.shape[2], device=device)
            gmc, gl, gw = torch.empty_like(mc), torch.empty_like(loc), torch.empty_like(w)
            fwd = native_function("deformable_aggregation_forward_opt")
            bwd = native_function("deformable_aggregation_backward_opt")
            self.phases = [
                ("forward", lambda: fwd(mc, sp, st, loc, w, out), _nbytes(mc, loc, w, out), 1),
                # accumulated into, as the reference's autograd zero-fills it
                ("grad_fill", gmc.zero_, 0, 0),
                ("backward", lambda: bwd(mc, sp, st, loc, w, grad, gmc, gl, gw),
                 _nbytes(mc, loc, w, grad, gmc, gl, gw), 1),
            ]
            self.dominant = ("backward", "deformable_aggregation_backward", 1)
            self.calls = "deformable_aggregation_forward_opt/backward_opt"
            self.inputs, self.outputs = [mc, loc, w, grad], [out, gmc, gl, gw]
            self.workload = ("SparseDrive deformable aggregation fwd+bwd, reference production shapes: mc_ms_feat "
                             "[8, 89760, 256] fp32, 6 cams x 4 scales, 900 anchors x 13 pts, 8 groups, 40% in image")
            self.dtype = "f32"
        elif op == "flash_sca":
            t, kw = cases.flash_sca_inputs(device)
            value, proj, shapes, starts, image, offsets, weights = t
            gx, gy, gz = kw["grid_size"]
            (sx, sy, sz), (x0, y0, z0) = kw["voxel_size"], kw["voxel_min"]
            out = torch.empty(value.shape[0], gy, gx, value.shape[3], device=device)
            grad = torch.randn(out.shape, generator=torch.Generator().manual_seed(3)).to(device)
            roi = torch.tensor([x0, x0 + gx * sx, y0, y0 + gy * sy, z0, z0 + gz * sz], device=device)
            gv, go, gwt = torch.empty_like(value), torch.empty_like(offsets), torch.empty_like(weights)
            heads, points = offsets.shape[3], offsets.shape[5]
            fwd = native_function("flash_bevpool_sca_forward")
            bwd = native_function("flash_bevpool_sca_backward")

            def fill():  # accumulated into (the reference's autograd zero-fills them)
                for buf in (gv, go, gwt):
                    buf.zero_()

            self.phases = [
                ("forward", lambda: fwd(value, proj, shapes, starts, image, offsets, weights, out, heads, points, gx,
                                        gy, gz, sx, sy, sz, x0, y0, z0, value.shape[2], 1e-5),
                 _nbytes(value, proj, offsets, weights, out), 1),
                ("grad_fill", fill, 0, 0),
                ("backward", lambda: bwd(grad, value, proj, shapes, starts, image, roi, offsets, weights, gv, go, gwt,
                                         heads, points, gx, gy, gz, value.shape[2], 1e-5),
                 _nbytes(value, proj, offsets, weights, grad, gv, go, gwt), 1),
            ]
            self.dominant = ("backward", "flash_sca_backward", 1)
            self.calls = "flash_bevpool_sca_forward/backward"
            self.inputs, self.outputs = [value, proj, offsets, weights, grad], [out, gv, go, gwt]
            self.workload = ("FlashSCA fwd+bwd, BEVFormer-base: 200x200x4 BEV grid, 6 cams, 4 levels of a 480x800 "
                             "image, 8 heads x 32 channels, 2 points per height, fp32")
            self.dtype = "f32"
        else:
            inp, indexes, count, slots = cases.sca_scatter_inputs(device)
            names = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")
            args = [inp[k] for k in names]
            scatter = native_function("ms_deform_attn_scatter_div_forward")

            def cameras():
                for cam, index in enumerate(indexes):
                    scatter(*args, index, count, slots, cam)

            valid = sum(int(i.numel()) for i in indexes)
            loc, w = inp["sampling_locations"], inp["attention_weights"]
            per_row = (loc[0, 0].numel() + w[0, 0].numel()) * loc.element_size()  # one rebatched query, all heads
            scatter_bytes = (_nbytes(inp["value"], count) + valid * per_row + valid * 8
                             + 2 * valid * slots.shape[2] * slots.element_size())
            self.phases = [("slots_fill", slots.zero_, 0, 0),
                           ("scatter", cameras, scatter_bytes, len(indexes))]
            # traffic is recorded per valid rebatched query of a camera launch
            self.dominant = ("scatter", "sca_scatter", valid)
            self.calls = "ms_deform_attn_scatter_div_forward x 6 cameras"
            self.inputs, self.outputs = [inp["value"], loc, w, count], [slots]
            self.workload = ("BEVFormer-base SCA forward + rebatch scatter + count normalisation, 6 cameras x 10000 "
                             "rebatched queries (6000-10000 valid), 40000 BEV queries, 8 heads x 32 channels, bf16")
            self.dtype = "bf16"
        self.bytes = sum(p[2] for p in self.phases)
        self.launches = sum(p[3] for p in self.phases)

    def step(self):
        for _, call, _, _ in self.phases:
            call()


def _op_cpu_baseline(op: str, step_bytes: int):
    """The op's CPU restatement (oracle/) on a bounded sample of the workload,
    all host threads. The value is in the GPU line's units: the full step's
    compulsory bytes over the sample's time scaled to the full step's work
    (anchor rows, BEV cells or valid rebatched queries)."""
    torch.set_num_threads(os.cpu_count() or 1)
    if op == "deformable_aggregation":
        from oracle.deformable_aggregation import deformable_aggregation_forward_backward

        (mc, sp, st, loc, w), grad = cases.deformable_aggregation_inputs("cpu", batch=1, anchors=64)
        run = lambda: deformable_aggregation_forward_backward(mc, sp, st, loc, w, grad)  # noqa: E731
        scale, sample = 8 * 900 / 64, "64 anchor rows of the 8 x 900 (batch 1)"
    elif op == "flash_sca":
        from oracle.flash_sca import flash_sca_forward_backward

        t, kw = cases.flash_sca_inputs("cpu", grid=(20, 20, 4))
        grad = torch.randn(1, 20, 20, t[0].shape[3])
        run = lambda: flash_sca_forward_backward(*t, kw["grid_size"], kw["voxel_size"], kw["voxel_min"], grad)  # noqa: E731
        scale, sample = 200 * 200 / (20 * 20), "a 20x20x4 BEV patch of the 200x200x4 grid, all cameras"
    else:
        from oracle import oracle_scatter_div

        inp, indexes, count, slots = cases.sca_scatter_inputs("cpu", dtype=torch.float32, cams=1, max_len=1000,
                                                              num_query=4000, lens=(1000,))
        names = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")
        arrays = [inp[k].numpy() for k in names]
        run = lambda: oracle_scatter_div(*arrays, indexes[0].numpy(), count.numpy(), slots.numpy(), 0)  # noqa: E731
        scale, sample = 50000 / 1000, "1000 of the 50000 valid rebatched queries, one camera (C oracle, fp32)"
    run()
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(step_bytes / (t * scale) / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{sample}; median of 3 after 1 warm-up, {t * 1e3:.1f} ms per sample, x{scale:g} to a step",
            "ms_per_step": round(t * scale * 1e3, 1)}


def run_op(args, rank, world, device):
    """--op: K timed steps of one op on device-resident inputs (each rank an
    independent replica, weak scaling), then K steps with CUDA events around
    every phase (kernels_ms and the dominant kernel's roofline), the e2e leg
    with pinned host buffers and the CPU baseline on rank 0."""
    import torch.distributed as dist

    w = OpWorkload(args.op, device)
    for _ in range(args.warmup):
        w.step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(device.index) as clocks:
        start.record()
        for _ in range(args.steps):
            w.step()
        end.record()
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps

    # per-phase device time: events on the launching (current) stream around every phase
    events = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in w.phases]
              for _ in range(args.steps)]
    for step_events in events:
        for (a, b), (_, call, _, _) in zip(step_events, w.phases):
            a.record()
            call()
            b.record()
    torch.cuda.synchronize()
    phase_ms = torch.tensor([sum(step_events[i][0].elapsed_time(step_events[i][1]) for step_events in events)
                             / args.steps for i in range(len(w.phases))], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(phase_ms, op=dist.ReduceOp.MAX)
    kernels_ms = {p[0]: round(float(v), 4) for p, v in zip(w.phases, phase_ms.tolist())}

    e2e = None
    if not args.no_e2e:
        host_in = [x.cpu().pin_memory() for x in w.inputs]
        second = OpWorkload(args.op, device)  # the second device buffer set of the pipeline
        slots = [E2ESlot(x.inputs, x.outputs, x.step) for x in (w, second)]
        steps = max(3, min(args.steps, 10))
        e2e_ms = pipelined_e2e(slots, host_in, steps, world > 1, device, args.e2e_streams)
        e2e = {"value": round(w.bytes * world / (e2e_ms / 1e3) / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": _nbytes(*host_in), "d2h_bytes_per_step": _nbytes(*w.outputs),
               "ms_per_step": round(e2e_ms, 3), "steps": steps,
               "path": E2E_PATH.format(calls=w.calls, streams=args.e2e_streams)}
        del second, slots
    if rank != 0:
        return None
    peak, peak_src = _peaks()
    achieved = w.bytes / (ms / 1e3) / 1e9
    dom_name, dom_key, dom_units = w.dominant
    dom = next(p for p in w.phases if p[0] == dom_name)
    dom_ms = kernels_ms[dom_name]
    dom_achieved = dom[2] / (dom_ms / 1e3) / 1e9
    traffic, traffic_src = _traffic(dom_key, args.op, dom_units)
    line = {
        "metric": f"{args.op} step us & effective HBM GB/s (compulsory bytes / device time)",
        "value": round(achieved * world, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "us_per_call": round(ms * 1e3, 1),
        "kernels_ms": kernels_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": w.dtype,
        "data": "synthetic",
        "config": {"workload": w.workload, "parallelism": f"{world} independent replicas",
                   "compulsory_bytes_per_step": w.bytes, "l2": "inputs > 126 MB L2; no flush"},
        "roofline": {"bound": "hbm", "kernel": dom_key, "achieved": round(dom_achieved, 1), "peak": peak,
                     "peak_source": peak_src, "unit": "GB/s", "frac": round(dom_achieved / peak, 4),
                     "traffic": None if traffic is None else int(traffic),
                     "algorithmic_bytes": dom[2], "launches_per_step": dom[3]},
        "gpu_launches": w.launches * args.steps * world,
        "clocks": clocks.summary(),
        "e2e": e2e,
    }
    if traffic_src:
        line["roofline"]["traffic_source"] = traffic_src
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = _op_cpu_baseline(args.op, w.bytes)
    return line


# The reference's only published numbers for this path: the bevformer-1l
# case, forward-backward scope, p50 of 5 repeats x 100 launches after 20
# warm-ups (benchmarks/msda/README.md:72-73 in the muSPACE tree).
PUBLISHED = {
    ("bevformer-1l", torch.float32): {
        "S5000_p50_ms": 4.2387, "S5000_normalised_to_A100_bandwidth_ms": 3.5049, "mmcv_A100_p50_ms": 4.0895,
        "source": "benchmarks/msda/README.md:72 (MTT S5000; mmcv CUDA MSDA on A100 80GB PCIe)"},
    ("bevformer-1l", torch.bfloat16): {
        "S5000_p50_ms": 3.9933, "source": "benchmarks/msda/README.md:73 (MTT S5000; no mmcv bf16 path to time)"},
}


def protocol_measure(launch, warmup=20, iterations=100, repeats=5):
    """The reference harness's timing (benchmarks/_harness.py:226-260): warm-up
    launches, then `repeats` samples, each the mean of `iterations` launches
    between two device events; the published figure is the median sample."""
    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    samples = []
    for _ in range(repeats):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iterations):
            launch()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) / iterations)
    return samples


def run_protocol(args, cfg, dtype, device):
    """--protocol reference: the published case timed the reference's way,
    through the same C-ABI entry points its harness calls, in two scopes:
    the reference's timed closure (benchmarks/msda/benchmark_msda.py:98-119:
    output allocation, forward launch, three zero-filled accumulators,
    grad_output.contiguous(), backward launch) and this build's step (forward,
    zero fill of grad_value only -- grad_loc / grad_w are written everywhere
    -- backward)."""
    from muspace_b200.runtime.native import native_function

    fwd, bwd = native_function("ms_deform_attn_forward"), native_function("ms_deform_attn_backward")
    # drawn on the CPU from the reference's seeds (2333 forward, 2334 backward), then moved
    inp = {k: v.to(device) for k, v in cases.make_inputs(cfg, dtype=dtype, seed=2333, device="cpu").items()}
    grad = inp["grad_output"]
    names = ("value", "spatial_shapes", "level_start_index", "sampling_locations", "attention_weights")
    a = [inp[n] for n in names]
    value, loc, weight = a[0], a[3], a[4]

    def reference_closure():
        output = value.new_empty((value.size(0), loc.size(1), value.size(2) * value.size(3)))
        fwd(*a, output, 64)
        gv = torch.zeros(value.shape, dtype=torch.float32, device=device)
        gl = torch.zeros(loc.shape, dtype=torch.float32, device=device)
        gw = torch.zeros(weight.shape, dtype=torch.float32, device=device)
        bwd(*a, grad.contiguous(), gv, gl, gw, 64)

    step = Step(inp, dtype, device)
    with Clocks(device.index) as clocks:
        ref_samples = protocol_measure(reference_closure)
        own_samples = protocol_measure(step)
    ref_p50, own_p50 = statistics.median(ref_samples), statistics.median(own_samples)
    nbytes = cases.compulsory_bytes(cfg, dtype)["total"]
    peak, peak_src = _peaks()
    published = PUBLISHED.get((cfg.name, dtype))
    line = {
        "metric": "MSDA fwd+bwd p50 ms, reference published-case protocol",
        "value": round(ref_p50, 4),
        "unit": "ms",
        "n_gpus": 1,
        "higher_is_better": False,
        "dtype": _dtype_tag(dtype),
        "data": "synthetic",
        "config": {"workload": f"{cfg.name}: {cfg.description}", "protocol":
                   "20 warm-up launches, 5 repeats x 100 launches between device events, median repeat "
                   "(benchmarks/_harness.py:226-260)",
                   "scope": "the reference's timed closure: output allocation, forward, three torch.zeros "
                            "accumulators, grad_output.contiguous(), backward (benchmarks/msda/benchmark_msda.py:98-119)",
                   "compulsory_bytes": nbytes},
        "reference_closure": {"p50_ms": round(ref_p50, 4), "samples_ms": [round(x, 4) for x in ref_samples],
                              "effective_gbs": round(nbytes / (ref_p50 / 1e3) / 1e9, 1),
                              "roofline_frac": round(nbytes / (ref_p50 / 1e3) / 1e9 / peak, 4)},
        "own_step": {"p50_ms": round(own_p50, 4), "samples_ms": [round(x, 4) for x in own_samples],
                     "effective_gbs": round(nbytes / (own_p50 / 1e3) / 1e9, 1),
                     "roofline_frac": round(nbytes / (own_p50 / 1e3) / 1e9 / peak, 4),
                     "scope": "forward, grad_value zero fill, backward (grad_loc / grad_w written, not zeroed)"},
        "peak": {"hbm_gbs": peak, "source": peak_src},
        "published": published,
        "clocks": clocks.summary(),
    }
    if published:
        line["speedup_vs_published"] = {k: round(v / ref_p50, 2) for k, v in published.items() if k.endswith("_ms")}
    return line


def main():
    args = parse_args()
    if args.config is None:
        args.config = "bevformer-1l" if args.protocol == "reference" else "c4"
    cfg = cases.CONFIGS[args.config]
    dtype = _dtype(args, cfg)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, dtype, rank)
        return
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs CUDA devices for the b200 arm")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    if args.protocol == "reference":
        if world != 1 or args.op != "msda":
            raise SystemExit("--protocol reference times the MSDA published case on one GPU")
        print(json.dumps(run_protocol(args, cfg, dtype, device)), flush=True)
        return
    try:
        line = run_op(args, rank, world, device) if args.op != "msda" else run_b200(args, cfg, dtype, rank, world, device)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
