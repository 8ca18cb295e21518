"""Benchmark of the B200 batched-inference hot path (samples/s).

Default workload: cfg4, the residual MLP 16->128, 4 x [LayerNorm(128) ->
Dense128 -> GELU -> Dense128 + skip], ->8 (fp32), the largest configuration
by work (268,288 FLOP per sample), batch 33,554,432 columns per GPU,
synthetic inputs N(0,1) generated on each device by a counter-based RNG
keyed by the global column.  A step is one forward_batch_parallel over the
whole batch; the 2 GB input exceeds the 126 MB L2, so no flush is needed
between steps (workloads smaller than L2 are timed step by step with an
L2-flushing write before each step, outside the timed events).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfgX] [--scaling weak|strong]
                  [--impl ours|reference]

Weak scaling: rank r owns columns [r*B, (r+1)*B).  Strong scaling: the
config's batch B is split into N contiguous column ranges.  Under torchrun
(N>1) every rank runs its shard with no collective on the data path; timing
is CUDA events on each rank's stream, max over ranks.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# The CPUs this process may use before any NUMA binding of a GPU rank: the
# CPU baseline runs on all of them.
ALL_CPUS = os.sched_getaffinity(0)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--config", default="cfg4")
    p.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                   help="weak: the config's batch on every GPU; strong: the config's batch split across GPUs")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--batch", type=int, default=0, help="override per-GPU batch (default: the config's)")
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--arith", default="", choices=["", "auto", "reference", "tensor"],
                   help="kernel selection (ponni_b200_model_set_arithmetic); default: the config's")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "sm_max_mhz": 1965.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None
        sm = [v for v in (num(s[1]) for s in self.samples) if v is not None]
        mx = [v for v in (num(s[2]) for s in self.samples) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def host_cpu():
    """(physical cores available to this process, CPU model) from lscpu."""
    model, cores = "unknown", os.cpu_count() or 1
    try:
        allowed = ALL_CPUS
        out = subprocess.run(["lscpu", "-p=CPU,CORE,SOCKET"], capture_output=True, text=True, timeout=10).stdout
        phys = {(f[2], f[1]) for f in (ln.split(",") for ln in out.splitlines() if ln and ln[0] != "#")
                if int(f[0]) in allowed}
        cores = max(1, len(phys))
        info = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for ln in info.splitlines():
            if ln.startswith("Model name:"):
                model = ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return cores, model


def cpu_reference(cfg_name, seconds=10.0, max_cols=1 << 20):
    """Time the reference's path on the host cores (oracle/cpu_bench.py, a
    child process): the reference's own template code compiled against the
    host Kokkos shim (oracle/_ref, kind "reference") where it was built, else
    the C port (kind "port"), with one OpenMP thread per physical core,
    OMP_PROC_BIND=spread, OMP_PLACES=cores: median samples/s over passes that
    total at least one second.  Returns (samples/s, cores, description, kind)."""
    cores, model = host_cpu()
    env = dict(os.environ, OMP_NUM_THREADS=str(cores), OMP_PROC_BIND="spread", OMP_PLACES="cores")
    out = subprocess.run([sys.executable, "-m", "oracle.cpu_bench", "--config", cfg_name, "--seconds", str(seconds),
                          "--max-cols", str(max_cols)], cwd=ROOT, env=env, capture_output=True, text=True,
                         check=True, preexec_fn=lambda: os.sched_setaffinity(0, ALL_CPUS)).stdout
    r = json.loads(out.strip().splitlines()[-1])
    desc = (f"{r['kind']}: {r['columns']} columns of {cfg_name} per pass, median of {r['passes']} passes "
            f"({r['seconds']:.1f} s), {cores} OpenMP threads (OMP_PROC_BIND=spread, OMP_PLACES=cores) on "
            f"{cores} physical cores, {model}")
    return r["samples_per_s"], cores, desc, r["kind"]


def run_reference(args, cfg, rank, metric, unit, dtype_name):
    """CPU reference arm: the oracle port of the reference's path on the host cores."""
    if rank != 0:
        return
    steps, info = [], None
    per_step = min(10.0, 120.0 / max(1, args.warmup + args.steps))
    for i in range(args.warmup + args.steps):
        v, cores, sample, kind = cpu_reference(args.config, seconds=per_step)
        if i >= args.warmup:
            steps.append(v)
        info = (cores, sample, kind)
    value = statistics.median(steps)
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": dtype_name, "data": "synthetic",
        "config": {"workload": cfg.name, "batch_per_gpu": cfg.batch, "sample": info[1]},
        "cpu_baseline": {"value": value, "unit": unit, "cores": info[0], "kind": info[2], "sample": info[1]},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


L2_FLUSH_BYTES = 256 << 20


def param_update_latency(model, reps=20):
    """Wall-clock latency of one parameter update of the planned model
    (synchronized, measured after the timed region): from device memory,
    from host memory (pinned staging + device scatter), and through a full
    re-plan (PONNI_B200_PARAM_SCATTER=0: re-pack and re-upload every image)."""
    import numpy as np
    import torch

    n = model.get_num_trainable_parameters()
    if n == 0:
        return None
    saved = model.get_trainable_parameters()
    hv = np.random.default_rng(1).normal(0, 0.1, n)
    dv = torch.from_numpy(hv).to(model.torch_dtype()).cuda(model.device)

    def wall_us(fn, k):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(k):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / k * 1e6

    out = {"params": n, "device_update_us": wall_us(lambda: model.set_trainable_parameters_device(dv), reps),
           "host_update_us": wall_us(lambda: model.set_trainable_parameters(hv), reps)}
    os.environ["PONNI_B200_PARAM_SCATTER"] = "0"
    try:
        out["replan_update_us"] = wall_us(lambda: (model.set_trainable_parameters(hv), model.kernel()), 3)
    finally:
        del os.environ["PONNI_B200_PARAM_SCATTER"]
    model.set_trainable_parameters(saved)
    out["timing"] = "wall clock per update incl. host work, synchronized, after the timed region"
    return out


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    from ponni_b200 import configs

    cfg = configs.ALL[args.config](batch=args.batch) if args.batch else configs.ALL[args.config]()
    metric, unit = "samples/sec", "samples/s"
    dtype_name = {0: "f32", 1: "f64", 2: "f16", 3: "bf16"}[cfg.dtype]
    if args.impl == "reference":
        run_reference(args, cfg, rank, metric, unit, dtype_name)
        return

    import torch
    import torch.distributed as dist
    import ponni_b200 as pb
    from ponni_b200.sharding import bind_numa, job_time, shard_range, split_range

    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if args.scaling == "strong":
        col0, B = split_range(rank, world, cfg.batch)
    else:
        B = cfg.batch
        col0, _ = shard_range(rank, world, B)
    numa = bind_numa(local)
    nin, nout = cfg.layers[0].num_inputs, cfg.layers[-1].num_outputs
    arith_name = args.arith or cfg.arith
    arith = {"auto": pb._abi.ARITH_AUTO, "reference": pb._abi.ARITH_REFERENCE,
             "tensor": pb._abi.ARITH_TENSOR}[arith_name]
    model = pb.Inference(cfg.layers, dtype=cfg.dtype, device=local, arithmetic=arith)
    try:
        model.kernel()
    except pb.PonniError as e:  # the config's kernel is unavailable for this model: say so, use the default
        print(f"note: {arith_name} arithmetic unavailable ({e.message}); using the default", file=sys.stderr)
        arith_name = "auto"
        model.set_arithmetic(pb._abi.ARITH_AUTO)
    kernel_name = {1: "tile_forward_kernel (SIMT)", 2: "tc_forward_kernel (tcgen05)",
                   3: "narrow_forward_kernel (streaming)",
                   4: "ponni_narrow_jit (streaming, model-specialised)",
                   5: "ts_forward_kernel (tcgen05, streamed weights)",
                   6: "tr_forward_kernel (tcgen05, LayerNorm/residual epilogue)"}[model.kernel()]
    tdt = model.torch_dtype()
    x = torch.empty((nin, B), dtype=tdt, device=dev)
    y = torch.empty((nout, B), dtype=tdt, device=dev)
    pb.fill_synthetic(x, configs.INPUT_SEED, col0=col0, dist=cfg.input_dist, lo=cfg.lo, hi=cfg.hi)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        model.forward_batch_parallel(x, y)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    # Workloads smaller than L2 (126 MB) are timed step by step with a 256 MB
    # L2-flushing write between steps, outside the events; larger ones back
    # to back (their inputs already exceed L2).
    work_bytes = (nin + nout) * B * x.element_size()
    flush = work_bytes < L2_FLUSH_BYTES
    torch.cuda.synchronize(dev)
    if flush:
        scrub = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in evs:
            scrub.fill_(1)
            # a short device-side spin (bounded, ~0.1 ms) keeps the host's
            # enqueue of the forward ahead of the GPU, so the events time the
            # kernel and not the Python call that launches it
            torch.cuda._sleep(200_000)
            a.record(stream)
            model.forward_batch_parallel(x, y)
            b.record(stream)
        torch.cuda.synchronize(dev)
        ms = sum(a.elapsed_time(b) for a, b in evs)
        del scrub
    else:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            model.forward_batch_parallel(x, y)
        end.record(stream)
        torch.cuda.synchronize(dev)
        ms = start.elapsed_time(end)
    clk = clocks.stop()
    ms_step = job_time(ms, world, dev) / args.steps
    total_cols = cfg.batch if args.scaling == "strong" else world * B
    value = total_cols / (ms_step / 1e3)

    # Roofline of the fused kernel (one launch per step), algorithmic FLOPs or bytes.
    pk, pk_src = peaks()
    launch_s = (ms / args.steps) / 1e3
    sm_mhz = clk.get("sm_mhz") or pk.get("sm_max_mhz", 1965.0)
    kernel = model.kernel()
    if cfg.bound == "hbm":
        roof = {"bound": "hbm", "achieved": cfg.bytes_per_sample * B / launch_s / 1e9, "peak": pk["hbm_gbs"],
                "unit": "GB/s", "peak_source": f"hbm_gbs ({pk_src})"}
    elif kernel in (pb._abi.KERNEL_TENSOR, pb._abi.KERNEL_TENSOR_STREAM, pb._abi.KERNEL_TENSOR_RESID):
        # fp32 models run six bf16 MMAs per multiply-add (exact 3-way operand
        # split), so their tensor roofline is a sixth of the bf16 peak.
        passes = 6 if cfg.dtype == pb.F32 else 1
        roof = {"bound": "tensor", "achieved": cfg.flops_per_sample * B / launch_s / 1e12,
                "peak": pk["bf16_tflops"] / passes, "unit": "TFLOP/s",
                "peak_source": f"bf16_tflops ({pk_src})" + (" / 6 (six bf16 MMAs per fp32 multiply-add)"
                                                             if passes == 6 else "")}
    else:
        lanes = 128 if cfg.dtype == pb.F32 else 64
        roof = {"bound": "compute", "achieved": cfg.flops_per_sample * B / launch_s / 1e12,
                "peak": 148 * lanes * 2 * sm_mhz * 1e6 / 1e12, "unit": "TFLOP/s",
                "peak_source": f"SIMT FMA peak (148 SMs x {lanes} lanes x 2) at the sampled median SM clock "
                               f"{sm_mhz:.0f} MHz; no measured fp32 peak exists"}
    roof["hbm_gbs_achieved"] = cfg.bytes_per_sample * B / launch_s / 1e9
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["traffic"] = None
    tpath = os.path.join(ROOT, "profiles", f"traffic_{cfg.name}.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            tr = json.load(f)
        roof["traffic"] = tr.get("bytes_per_full_launch")
        roof["traffic_note"] = tr.get("note")

    # End to end through the host-buffer C-ABI entry point (pinned host memory).
    e2e = None
    if args.e2e_steps > 0:
        xh = torch.empty((nin, B), dtype=tdt, pin_memory=True)
        yh = torch.empty((nout, B), dtype=tdt, pin_memory=True)
        xh.copy_(x)
        model.forward_batch_parallel(xh, yh)  # warm-up (allocates staging)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            model.forward_batch_parallel(xh, yh)
        e2e_s = (time.perf_counter() - t0) / args.e2e_steps
        e2e_s = job_time(e2e_s, world, dev)
        esz = x.element_size()
        e2e = {"value": total_cols / e2e_s, "unit": unit, "h2d_bytes_per_step": total_cols * nin * esz,
               "d2h_bytes_per_step": total_cols * nout * esz,
               "host_link_gbs": {"h2d": nin * B * esz / e2e_s / 1e9, "d2h": nout * B * esz / e2e_s / 1e9,
                                 "note": "per GPU; the copies of one step overlap its kernel chunk by chunk"},
               "path": "ponni_b200_forward_host (C ABI), pinned host buffers, chunked copy/compute overlap"}
        del xh, yh

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample, kind = cpu_reference(args.config)
        cpu = {"value": v, "unit": unit, "cores": cores, "kind": kind, "sample": sample}

    upd = param_update_latency(model) if rank == 0 else None

    if world > 1:
        dist.barrier()
    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": dtype_name, "data": "synthetic",
            "config": {"workload": cfg.name, "batch_per_gpu": B, "global_batch": total_cols, "nin": nin,
                       "nout": nout, "parallelism": f"column shards x{world} ({args.scaling} scaling), no collective",
                       "host_numa_node_rank0": numa,
                       "l2": ("L2 flushed (256 MB write) before each step, outside the timed events "
                              "(then a 0.1 ms device spin so that the launch is queued before the start event)" if flush
                              else "inputs larger than L2 (no flush)")},
            "kernel": kernel_name, "arithmetic": arith_name, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clk,
            "param_update": upd,
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
