"""Benchmark of the chess-engine-4 forward on B200: positions/s at d512 x 12, batch 4096.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward of one batch of synthetic positions (lc0 InputPlane records,
seeded Bernoulli(0.08) planes) through the dense d512 x 12 SwiGLU tower (hidden 1536,
BF16, weights N(0, 0.02)). Each rank of a multi-GPU run is an independent replica
processing its own batch (weak scaling, no collective on the data path). Rank 0 prints
one JSON line.

* ``value``: device-timed throughput (CUDA events per step, L2 flushed between steps,
  inputs resident in HBM), all ranks' positions / the slowest rank's time.
* ``e2e``: the same metric through the engine-facing C ABI call
  (``ce4b_model_evaluate_async``) with pinned host buffers: H2D of the planes, the
  forward (CUDA graph) and D2H of policy / WDL / moves-left inside every timed step.
* ``roofline``: the dominant kernel (gate_up GEMM with the fused SwiGLU epilogue), timed
  live with CUDA events recorded by the library around it during the timed steps.
* ``cpu_baseline``: the CPU restatement of the reference's portable PyTorch forward
  (oracle/dense.py, mode fp32 = PortableChessNet) on the host cores, bounded sample.
* ``--impl reference``: rank 0 times that CPU implementation as the reference arm.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "chess-engine-4_b200"))
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402
import torch  # noqa: E402

D_MODEL, DEPTH, RATIO, BATCH = 512, 12, 3.0, 4096
HIDDEN = int(D_MODEL * RATIO)
IN_DIM = 112 * 64
POLICY = 1858
# Algorithmic GEMM FLOPs per position: input projection, 3 projections per layer, heads
# (policy 1858 + wdl 3 + moves-left 1).
FLOP_PER_POS = 2 * (IN_DIM * D_MODEL + DEPTH * 3 * D_MODEL * HIDDEN + 1862 * D_MODEL)
GATE_UP_FLOP_PER_POS = 2 * 2 * HIDDEN * D_MODEL
METRIC = "positions/sec (dense d512x12 forward, batch 4096 per GPU)"
WORKLOAD = "dense-d512-L12-h1536-bf16-b4096"


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=BATCH)
    p.add_argument("--quick", action="store_true", help="skip e2e, latency, clocks and CPU baseline (profiling)")
    return p.parse_args()


def peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return {
            "hbm_gbs": data["hbm_gbs"],
            "bf16_tflops": data["bf16_tflops"],
            "bf16_tflops_sustained": data["bf16_tflops_sustained"],
            "source": "measured",
        }
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------- distributed plumbing
def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group(
            "nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local)
        )
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_teardown(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons every 200 ms while running."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, device: int) -> None:
        # nvidia-smi numbering can differ from CUDA's under CUDA_VISIBLE_DEVICES: use the UUID.
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        self.device = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc: subprocess.Popen | None = None

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for name, flag in zip(names, r[5:9]):
                if flag.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {
            "sm_mhz": statistics.median(sm),
            "sm_max_mhz": max(mx),
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ---------------------------------------------------------------- CPU implementation
def cpu_forward_rate(batch: int, sample: int, repeats: int, seed: int = 0) -> dict:
    """Times the FP32 CPU restatement of PortableChessNet on a bounded sample."""

    from ce4b200 import synthetic
    from oracle import dense as oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    weights = synthetic.make_dense_weights(d_model=D_MODEL, depth=DEPTH, hidden_dim=HIDDEN, seed=seed)
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(sample, 1))
    with torch.no_grad():
        oracle.forward(weights, planes[: min(64, sample)], depth=DEPTH, mode="fp32")
        times = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            oracle.forward(weights, planes, depth=DEPTH, mode="fp32")
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {
        "value": sample / med,
        "unit": "positions/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{sample} of the {batch} positions of one step, fp32 PortableChessNet restatement "
        f"(oracle/dense.py), median of {repeats} runs",
    }


def run_reference(args: argparse.Namespace) -> None:
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return
    from ce4b200 import synthetic
    from oracle import dense as oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample = min(args.batch, 512)
    weights = synthetic.make_dense_weights(d_model=D_MODEL, depth=DEPTH, hidden_dim=HIDDEN, seed=0)
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(sample, 1))
    steps, warmup = max(1, min(args.steps, 20)), max(1, min(args.warmup, 3))
    with torch.no_grad():
        for _ in range(warmup):
            oracle.forward(weights, planes, depth=DEPTH, mode="fp32")
        t0 = time.perf_counter()
        for _ in range(steps):
            oracle.forward(weights, planes, depth=DEPTH, mode="fp32")
        elapsed = time.perf_counter() - t0
    value = sample * steps / elapsed
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "positions/s",
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": 1000.0 * elapsed / steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_positions_per_step": sample, "l2": "n/a (CPU)"},
        "cpu_baseline": {
            "value": value,
            "unit": "positions/s",
            "cores": threads,
            "kind": "port",
            "sample": f"{sample} positions per step (of {args.batch}); fp32 restatement of "
            "PortableChessNet (oracle/dense.py); the reference itself does not travel to the box",
        },
        "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU implementation
def make_model(device: int, batch: int):
    from ce4b200 import _lib, synthetic

    lib = _lib.library()
    cfg = _lib.ModelConfigStruct(
        arch=_lib.ARCH_DENSE, d_model=D_MODEL, depth=DEPTH, history_length=8,
        expansion_ratio=RATIO, rms_norm_eps=1e-6, policy_size=POLICY, policy_storage_size=1888,
        precision=_lib.PRECISION_BF16,
    )
    handle = ctypes.c_void_p()
    _lib.check(lib.ce4b_model_create(ctypes.byref(cfg), device, batch, ctypes.byref(handle)))
    weights = synthetic.make_dense_weights(
        d_model=D_MODEL, depth=DEPTH, hidden_dim=HIDDEN, seed=0, norm_std=0.0,
        device=f"cuda:{device}",
    )
    torch.cuda.synchronize()
    for name, t in weights.items():
        t = t.contiguous()
        dtype = _lib.DTYPE_F32 if t.dtype == torch.float32 else _lib.DTYPE_BF16
        shape = (ctypes.c_int64 * t.ndim)(*t.shape)
        _lib.check(lib.ce4b_model_set_tensor(handle, name.encode(), t.data_ptr(), dtype, t.ndim, shape, 1))
    _lib.check(lib.ce4b_model_finalize(handle))
    del weights
    return lib, handle


def run_ours(args: argparse.Namespace) -> None:
    from ce4b200 import _lib, synthetic

    world, rank, local = dist_setup(args.gpus)
    device = local
    torch.cuda.set_device(device)
    batch = args.batch
    lib, handle = make_model(device, batch)
    stream = torch.cuda.Stream(device)
    sptr = stream.cuda_stream

    lc0 = synthetic.make_lc0_planes(batch, 1 + rank)
    planes_host = synthetic.lc0_planes_tensor(lc0).pin_memory()
    planes_dev = planes_host.to(f"cuda:{device}")
    policy = torch.empty(batch, POLICY, dtype=torch.float32, device=device)
    wdl = torch.empty(batch, 3, dtype=torch.float32, device=device)
    ml = torch.empty(batch, dtype=torch.float32, device=device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)  # > 126 MB L2

    def forward() -> None:
        _lib.check(lib.ce4b_model_forward(
            handle, _lib.INPUT_LC0, planes_dev.data_ptr(), None, batch, policy.data_ptr(),
            wdl.data_ptr(), ml.data_ptr(), 0, 0, None, sptr))

    # Trace events: one per kernel of the forward, per timed step (steps are enqueued
    # back to back; the host never waits inside the timed loop).
    n_kernels = 2 * DEPTH + 3
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            forward()
            flush.zero_()
        stream.synchronize()
        barrier(world)
        torch.cuda.synchronize()

        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        traces = [[torch.cuda.Event(enable_timing=True) for _ in range(n_kernels)] for _ in range(args.steps)]
        for tr in traces:  # torch creates the CUDA event on first record
            for e in tr:
                e.record(stream)
        stream.synchronize()
        arrays = [(ctypes.c_void_p * n_kernels)(*[e.cuda_event for e in tr]) for tr in traces]
        sampler = ClockSampler(device) if not args.quick else None
        if sampler:
            sampler.__enter__()
        try:
            for step in range(args.steps):
                starts[step].record(stream)
                _lib.check(lib.ce4b_model_set_trace(handle, arrays[step], n_kernels))
                forward()
                flush.zero_()
            _lib.check(lib.ce4b_model_set_trace(handle, None, 0))
            stream.synchronize()
        finally:
            if sampler:
                sampler.__exit__(None, None, None)
    step_ms, gate_ms = [], []
    for step in range(args.steps):
        tr = traces[step]
        step_ms.append(starts[step].elapsed_time(tr[-1]))
        for i in range(2, n_kernels - 1, 2):  # gate_up kernel of layer l sits at 2 + 2l
            gate_ms.append(tr[i - 1].elapsed_time(tr[i]))
    labels = []
    buf = ctypes.create_string_buffer(64)
    for i in range(n_kernels):
        _lib.check(lib.ce4b_model_trace_label(handle, i, buf, 64))
        labels.append(buf.value.decode())
    assert all(labels[i] == "gate_up_swiglu" for i in range(2, n_kernels - 1, 2)), labels
    barrier(world)
    total_ms = sum(step_ms)
    slowest_ms = max_over_ranks(total_ms, world)
    value = world * batch * args.steps / (slowest_ms / 1000.0)
    clocks = sampler.summary() if sampler else None

    # ---- end to end through the C ABI with pinned host buffers
    e2e = None
    latency = None
    if not args.quick:
        pol_h = torch.empty(batch, POLICY, dtype=torch.float32).pin_memory()
        wdl_h = torch.empty(batch, 3, dtype=torch.float32).pin_memory()
        ml_h = torch.empty(batch, dtype=torch.float32).pin_memory()

        def evaluate(b: int) -> None:
            _lib.check(lib.ce4b_model_evaluate_async(
                handle, planes_host.data_ptr(), b, pol_h.data_ptr(), wdl_h.data_ptr(), ml_h.data_ptr(), sptr))

        e2e_steps = max(1, min(args.steps, 300))
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                evaluate(batch)
            stream.synchronize()
            barrier(world)
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            e2e_ms = 0.0
            for _ in range(e2e_steps):
                ev0.record(stream)
                evaluate(batch)
                ev1.record(stream)
                stream.synchronize()
                e2e_ms += ev0.elapsed_time(ev1)
                flush.zero_()
            stream.synchronize()
        e2e_slowest = max_over_ranks(e2e_ms, world)
        e2e = {
            "value": world * batch * e2e_steps / (e2e_slowest / 1000.0),
            "unit": "positions/s",
            "h2d_bytes_per_step": batch * 112 * 16,
            "d2h_bytes_per_step": batch * (POLICY + 3 + 1) * 4,
            "steps": e2e_steps,
            "api": "ce4b_model_evaluate_async (pinned host buffers, CUDA graph per batch size)",
        }
        # ---- p50 latency at batch 64 (blocking engine call, host buffers)
        lat = []
        for i in range(220):
            t0 = time.perf_counter()
            _lib.check(lib.ce4b_model_evaluate(handle, planes_host.data_ptr(), 64, pol_h.data_ptr(),
                                               wdl_h.data_ptr(), ml_h.data_ptr()))
            if i >= 20:
                lat.append((time.perf_counter() - t0) * 1000.0)
        lat.sort()
        latency = {"batch": 64, "p50_ms": lat[len(lat) // 2], "p90_ms": lat[int(len(lat) * 0.9)],
                   "api": "ce4b_model_evaluate (blocking, host buffers, wall clock)"}

    code = _lib.check_device_error(device)
    if code != 0:
        raise RuntimeError(f"device error word set: {code}")
    lib.ce4b_model_destroy(handle)

    if rank == 0:
        pk = peaks()
        gate_avg_ms = statistics.mean(gate_ms)
        achieved = GATE_UP_FLOP_PER_POS * batch / (gate_avg_ms / 1000.0) / 1e12
        peak = pk["bf16_tflops_sustained"]
        traffic = None
        traffic_file = REPO / "profiles" / "gate_up_swiglu_traffic.json"
        if traffic_file.is_file():
            traffic = json.loads(traffic_file.read_text()).get("bytes_per_launch")
        cpu = None if args.quick else cpu_forward_rate(batch, 512, 3)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "positions/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": WORKLOAD,
                "global_batch": batch * world,
                "per_gpu_batch": batch,
                "parallelism": f"replicas x{world} (no collective)",
                "l2": "flushed between timed steps (256 MiB write, untimed)",
                "input_layout": "lc0 InputPlane records resident in HBM",
            },
            "roofline": {
                "kernel": "gate_up GEMM + fused SwiGLU (gemm_tc_kernel<256,4,2,2,...,EpiSwiGLU<128>>)",
                "bound": "tensor",
                "achieved": achieved,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": achieved / peak,
                "frac_of_burst": achieved / pk["bf16_tflops"],
                "peak_source": f"{pk['source']} bf16 sustained",
                "traffic": traffic,
                "avg_launch_ms": gate_avg_ms,
                "flop_per_launch": GATE_UP_FLOP_PER_POS * batch,
            },
            "forward_tflops": FLOP_PER_POS * batch / (total_ms / args.steps / 1000.0) / 1e12,
            "gpu_launches": n_kernels * args.steps,
            "clocks": clocks,
            "e2e": e2e,
            "latency_b64": latency,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    dist_teardown(world)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
