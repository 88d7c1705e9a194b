"""Benchmark of the MSAT all-modality control step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl b200|reference]
                    [--workload c2|production|production_addons]

One step = one control step of the action head for B observations per GPU: state encoder,
physics history encoder and 4 flow-matching Euler steps of [action + physics encoders, 16
ExpandedDoubleStreamBlocks over [VL 512 | SA 18 | P 32] at width 1536 (24 x 64 heads), output
projections, decoders, Euler updates], replayed as one CUDA graph.  Weights are seeded random
init with the reference module layout (no checkpoint ships); inputs are seeded synthetic tensors
with the config-2 shapes and distributions.

Multi-GPU (torchrun, one process per GPU): every GPU serves its own observations with a full
weight copy ("replicas", weak scaling); no collective runs on the step path — torch.distributed
only supplies the barrier and the max-over-ranks of the timed region.

--workload production / production_addons measures the reference's released head without /
with add-ons instead (4 double + 8 single blocks, VL width 4096; the shapes of the reference's
own published action-head benchmark, rldx/inference/action_model/README.md:9-37); the default
line is config 2.

Printed JSON (rank 0): value = control steps/s of the whole job with inputs resident in HBM;
e2e = the same through the C ABI with pinned host buffers (host->device inputs and device->host
actions inside the timed region); roofline of the dominant kernel (the grouped tcgen05 GEMM)
from a per-launch event-timed pass; cpu_baseline = the CPU restatement of the reference path
(oracle/, fp32, all host threads) on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=300)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch", type=int, default=1, help="observations per GPU per control step")
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--workload", choices=["c2", "production", "production_addons"], default="c2")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-sample-s", type=float, default=20.0, help="CPU baseline time budget")
    p.add_argument("--profile-step", action="store_true",
                   help="bracket one extra step with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    return p.parse_args()


def dist_setup(n):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    if n != world and world > 1:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE {world}")
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM traffic of the dominant kernel from a committed ncu capture summary."""
    p = ROOT / "profiles" / "gemm_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return None
    return None


# ----------------------------------------------------------------------------------------------
# CPU baseline: the oracle restatement of the reference path (fp32, all host threads)
# ----------------------------------------------------------------------------------------------
WORKLOADS = {
    "c2": ("BASELINE config 2: all-modality MSAT control step (4 Euler steps, one CUDA graph)",
           "MSAT 16 x ExpandedDoubleStreamBlock [VL 512 | SA 18 | P 32], hidden 1536, 24x64"),
    "production": ("reference's released head, no add-ons (4 Euler steps, one CUDA graph)",
                   "MSAT 4 x DoubleStreamBlock [VL 64 x 4096 | SA 18 x 1536] + 8 x SingleStreamBlock, "
                   "24x64, 1244.6M parameters"),
    "production_addons": ("reference's released head, all add-ons (4 Euler steps, one CUDA graph)",
                          "MSAT 4 x ExpandedDoubleStreamBlock [VL 80 x 4096 | SA 18 | P 32] + 8 x "
                          "ExpandedSingleStreamBlock, 24x64, 1842.6M parameters"),
}


def oracle_config(workload: str):
    """The oracle's MsatHeadConfig of a bench workload."""
    from oracle import msat_oracle as om

    if workload == "c2":
        return om.MsatHeadConfig()
    base = dict(n_vl=64 if workload == "production" else 80, depth=4, depth_single=8, vl_dim=4096,
                action_dim=64, max_seq_len=512)
    if workload == "production":
        base.update(use_physics=False, physics_hist=0, physics_fut=0)
    return om.MsatHeadConfig(**base)


def cpu_baseline(budget_s: float, steps: int = 8, warmup: int = 1, workload: str = "c2"):
    from oracle import msat_oracle as om

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = oracle_config(workload)
    head = om.init_weights(om.ActionHead(cfg), seed=0)
    inp = om.make_inputs(cfg, batch=1, seed=42)
    msat = head.model
    with torch.no_grad():
        sf = head.state_encoder(inp["state"], inp["embodiment_id"])
        t0 = torch.zeros(1)
        af = head.action_encoder(inp["init_noise"], t0, inp["embodiment_id"])
        sa = torch.cat([sf, af], 1)
        if cfg.use_physics:
            pe = torch.cat([head.physics.physics_cond_encoder(inp["physics_hist"]),
                            head.physics.physics_fut_encoder(inp["physics_noise"], t0)], dim=1)
            fwd = lambda: msat(sa, inp["vl"], t0, pe)  # noqa: E731
        else:
            fwd = lambda: msat(sa, inp["vl"], t0)  # noqa: E731
        for _ in range(max(1, min(warmup, 2))):
            fwd()
        times = []
        start = time.perf_counter()
        while True:
            t = time.perf_counter()
            fwd()
            times.append(time.perf_counter() - t)
            if time.perf_counter() - start > budget_s or len(times) >= max(1, steps):
                break
    per_forward = statistics.median(times)
    # one control step = num_steps MSAT forwards (+ encoders/decoders, < 5 % of the work)
    per_step = per_forward * cfg.num_steps
    return {"value": 1.0 / per_step, "unit": "control steps/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} MSAT forwards ({workload}, fp32, batch 1) timed on the host; "
                      f"p50 {per_forward * 1e3:.0f} ms x {cfg.num_steps} Euler steps = one control step"}


def run_reference(args):
    cb = cpu_baseline(args.cpu_sample_s, steps=args.steps, warmup=args.warmup, workload=args.workload)
    desc, model = WORKLOADS[args.workload]
    line = {"metric": "control_steps_per_s", "value": cb["value"], "unit": "control steps/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": desc + ", batch 1", "model": model,
                       "global_batch": 1, "seq_len": oracle_config(args.workload).n_vl + 18 +
                       (32 if oracle_config(args.workload).use_physics else 0), "parallelism": "cpu"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "control steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------
# B200 arm
# ----------------------------------------------------------------------------------------------
def run_b200(args, rank, world, local):
    import rldx_b200  # noqa: F401
    from rldx_b200.chain import B200ActionHeadChain, B200ExpandedActionHeadChain
    from rldx_b200.synthetic import PRESETS, random_action_head, random_inputs

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dims = PRESETS[args.workload]()
    B = args.batch
    head = random_action_head(dims, seed=0, device=dev)
    chain = (B200ExpandedActionHeadChain if dims.use_physics else B200ActionHeadChain)(head, dev)
    inp = random_inputs(dims, B, seed=42 + rank, device=dev)
    host = random_inputs(dims, B, seed=42 + rank, device="cpu", pin=True)
    out_host = torch.empty(B, dims.horizon, dims.action_dim, dtype=torch.bfloat16).pin_memory()

    def step():
        if dims.use_physics:
            return chain(inp["vl"], inp["state"], inp["embodiment_id"], inp["init_noise"],
                         inp["physics_hist"], inp["physics_noise"])
        return chain(inp["vl"], inp["state"], inp["embodiment_id"], inp["init_noise"])

    step()  # binds: weight arena, tables, graph capture
    torch.cuda.synchronize()
    del head  # the runtime holds its own copy of every weight
    torch.cuda.empty_cache()
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.int32, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region: device-resident inputs ----
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            flush.fill_(i)  # evict L2 between iterations (outside the event pair)
            starts[i].record()
            step()
            ends[i].record()
        torch.cuda.synchronize()
    barrier(world)
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(sum(ms), world, dev)
    p50 = statistics.median(ms)

    # ---- e2e: C ABI with pinned host buffers, copies inside the timed region ----
    chain.forward_host(host, out_host)
    e_ms = []
    barrier(world)
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.fill_(i)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        chain.forward_host(host, out_host)
        e.record()
        e.synchronize()
        e_ms.append(s.elapsed_time(e))
    barrier(world)
    e_total = max_over_ranks(sum(e_ms), world, dev)
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = out_host.numel() * out_host.element_size()

    if args.profile_step:
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()

    # ---- per-launch pass for the roofline of the dominant kernel ----
    prof = chain.profile(inp)
    gem = [p for p in prof if p[0] == "gemm"]
    g_ms = sum(p[2] for p in gem)
    g_bytes = sum(p[3] for p in gem)
    g_flops = sum(p[4] for p in gem)
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    achieved = (g_bytes / len(gem)) / (g_ms / len(gem) * 1e-3) / 1e9
    tflops = g_flops / (g_ms * 1e-3) / 1e12
    by_kind = {}
    for p in prof:
        d = by_kind.setdefault(p[0], [0, 0.0])
        d[0] += 1
        d[1] += p[2]
    traffic = ncu_traffic()

    if rank != 0:
        return
    n_obs = world * args.steps * B
    line = {
        "metric": "control_steps_per_s",
        "value": n_obs / (total_ms * 1e-3),
        "unit": "control steps/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "p50_ms_per_control_step": p50,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random weights with the reference layout; shaped inputs)",
        "config": {"workload": WORKLOADS[args.workload][0] + ", batch %d per GPU" % B,
                   "model": WORKLOADS[args.workload][1],
                   "global_batch": world * B, "seq_len": dims.tokens,
                   "parallelism": f"replicas x{world} (data parallel, no collective)",
                   "l2": "flushed between timed steps (256 MB write); weights streamed per step > L2"},
        "e2e": {"value": n_obs / (e_total * 1e-3), "unit": "control steps/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "p50_ms": statistics.median(e_ms)},
        "gpu_launches": chain.launches_per_step * args.steps,
        "roofline": {"bound": "hbm", "kernel": "gemm_bf16_kernel (grouped tcgen05 GEMM, all launches of a step)",
                     "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                     "peak_source": peak_kind,
                     # ncu DRAM bytes of a captured launch, scaled by its ratio to the algorithmic
                     # bytes onto the average launch of the step (one capture, not every launch)
                     "traffic": (traffic["dram_bytes"] / traffic["algorithmic_bytes"] * g_bytes / len(gem))
                                if traffic else None,
                     "traffic_source": traffic.get("capture") if traffic else None,
                     "bytes_per_launch": g_bytes / len(gem), "avg_launch_us": g_ms / len(gem) * 1e3,
                     "tensor_tflops": tflops, "tensor_frac": tflops / tc_peak},
        "breakdown_ms": {k: {"launches": v[0], "ms": round(v[1], 4)} for k, v in by_kind.items()},
    }
    line["clocks"] = clocks.summary()
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_sample_s, workload=args.workload)
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        # rank 0 alone times the CPU restatement; the other ranks exit without work
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        run_b200(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
