"""Benchmark driver: one JSON line for the headline workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload norm|attn_small|attn_long|gemm]

Default workload: fused residual-add + RMSNorm,
forward + backward, x/residual bf16 [8192, 4096] ~ N(0,1), weight f32
1 + 0.1 N(0,1), eps 1e-6, upstream grads bf16 ~ N(0,1).  One step =
``add_rmsnorm_fwd`` on one buffer set + ``rmsnorm_bwd`` (dh and the
deterministic dw reduction) on the other set's saved h; two buffer sets
alternate so that every kernel streams operands that are not L2-resident
(each set is 448 MiB, the L2 is 126 MB).  The metric is algorithmic HBM bytes
(read x, r; write h, y; read h, dy, dh_direct; write dh; plus w and dw) per
second, summed over ranks.

Multi-GPU (torchrun, one rank per GPU, NCCL): weak scaling.  Every rank
normalises its own 8192-token shard; the only exchange is the real one of the
backward, the all-reduce of the f32 dw partial (16 KiB) per step.  Timing is
CUDA events on the launching stream between barriers + synchronize, max over
ranks.

``--impl reference`` times the CPU restatement of the reference's path (the
``oracle`` package, numpy, all host threads) on a bounded sample of the same
workload; under torchrun only rank 0 runs it.
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
sys.path.insert(0, os.path.join(ROOT, "ferrite-tpu_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

ROWS, DIM, EPS = 8192, 4096, 1e-6
FWD_BYTES = 4 * ROWS * DIM * 2 + 4 * DIM  # read x, r; write h, y (bf16); read w (f32)
BWD_BYTES = 4 * ROWS * DIM * 2 + 4 * DIM + 4 * DIM  # read h, dy, dh_direct; write dh; read w; write dw
STEP_BYTES = FWD_BYTES + BWD_BYTES


# ----------------------------------------------------------------------------- helpers


def _dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons in the background during the
    timed region (the profiling recipe's query), for the GPU this rank drives."""

    FIELDS = (
        "index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, device: torch.device):
        self.bus = None
        try:
            props = torch.cuda.get_device_properties(device)
            self.bus = int(getattr(props, "pci_bus_id"))
        except Exception:  # noqa: BLE001
            pass
        self.proc = None
        self.lines: list[str] = []
        self.err = ""
        self._t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
            )
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError as e:
            self.proc, self.err = None, str(e)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                _, err = self.proc.communicate(timeout=5)
                self.err = (err or "")[:200]
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)

    def _mine(self, parts) -> bool:
        if self.bus is None:
            return True
        try:
            return int(parts[1].split(":")[1], 16) == self.bus
        except (IndexError, ValueError):
            return True

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10 or not self._mine(parts):
                continue
            try:
                sm.append(float(parts[2]))
                mx = float(parts[3])
            except ValueError:
                continue
            for name, val in zip(names, parts[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}
        if not sm:
            out["error"] = self.err or "no parsable samples"
            out["raw"] = self.lines[:2]
        return out


def _load_traffic(kernel: str):
    """Per-launch DRAM bytes of ``kernel`` from the committed ncu summary (profiles/ncu_traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(kernel, {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


# ----------------------------------------------------------------------------- norm workload (ours)


class NormWorkload:
    name = "add_rmsnorm_fwd_bwd_bf16_8192x4096"
    metric = "add+RMSNorm fwd+bwd HBM GB/s"
    unit = "GB/s"

    def __init__(self, device: torch.device):
        from ferrite import _native as nat

        self.nat = nat
        self.lib = nat.lib()
        self.dev = device
        g = torch.Generator(device=device)
        g.manual_seed(1234 + device.index if device.index is not None else 1234)

        def rn(*shape, dtype=torch.bfloat16):
            return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)

        self.sets = []
        for _ in range(2):
            s = {
                "x": rn(ROWS, DIM), "r": rn(ROWS, DIM), "dy": rn(ROWS, DIM), "dhd": rn(ROWS, DIM),
                "h": torch.empty(ROWS, DIM, dtype=torch.bfloat16, device=device),
                "y": torch.empty(ROWS, DIM, dtype=torch.bfloat16, device=device),
                "dh": torch.empty(ROWS, DIM, dtype=torch.bfloat16, device=device),
            }
            self.sets.append(s)
        self.w = (1.0 + 0.1 * torch.randn(DIM, generator=g, device=device)).float()
        self.dw = torch.empty(DIM, dtype=torch.float32, device=device)
        ws = int(self.lib.ferrite_rmsnorm_bwd_workspace_size(ROWS, DIM))
        self.ws = torch.empty(ws, dtype=torch.uint8, device=device)
        # make every h valid before the first backward reads it
        for s in self.sets:
            self.fwd(s)
        torch.cuda.synchronize(device)

    def fwd(self, s):
        nat = self.nat
        nat.check(self.lib.ferrite_add_rmsnorm_fwd(
            nat.stream_ptr(self.dev), s["x"].data_ptr(), s["r"].data_ptr(), self.w.data_ptr(), s["h"].data_ptr(), s["y"].data_ptr(),
            ROWS, DIM, EPS, nat.BF16, nat.F32))

    def bwd(self, s):
        nat = self.nat
        nat.check(self.lib.ferrite_rmsnorm_bwd(
            nat.stream_ptr(self.dev), s["h"].data_ptr(), self.w.data_ptr(), s["dy"].data_ptr(), s["dhd"].data_ptr(), s["dh"].data_ptr(),
            self.dw.data_ptr(), self.ws.data_ptr(), self.ws.numel(), ROWS, DIM, EPS, nat.BF16, nat.F32))

    launches_per_step = 3  # add_rmsnorm_fwd, rmsnorm_bwd, dw_reduce

    def step(self, i: int, events=None):
        a, b = self.sets[i % 2], self.sets[(i + 1) % 2]
        if events is not None:
            events[0].record()
        self.fwd(a)
        if events is not None:
            events[1].record()
        self.bwd(b)
        if events is not None:
            events[2].record()

    # ---- end to end through the public API, host buffers in and out
    def e2e_setup(self):
        pin = lambda t: t.cpu().pin_memory()  # noqa: E731
        s = self.sets[0]
        self.host = {k: pin(s[k]) for k in ("x", "r", "dy", "dhd")}
        self.host_w = pin(self.w)
        self.out_host = {k: torch.empty(ROWS, DIM, dtype=torch.bfloat16).pin_memory() for k in ("h", "y", "dx")}
        self.out_dw = torch.empty(DIM, dtype=torch.float32).pin_memory()
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host.values()) + self.host_w.numel() * 4
        self.d2h_bytes = sum(t.numel() * t.element_size() for t in self.out_host.values()) + DIM * 4

    def e2e_step(self):
        from ferrite.kernels.rmsnorm import rmsnorm

        d = self.dev
        x = self.host["x"].to(d, non_blocking=True).requires_grad_(True)
        r = self.host["r"].to(d, non_blocking=True).requires_grad_(True)
        w = self.host_w.to(d, non_blocking=True).requires_grad_(True)
        dy = self.host["dy"].to(d, non_blocking=True)
        dhd = self.host["dhd"].to(d, non_blocking=True)
        h, y = rmsnorm(x, w, residual=r, eps=EPS)
        torch.autograd.backward([h, y], [dhd, dy])
        self.out_host["h"].copy_(h.detach(), non_blocking=True)
        self.out_host["y"].copy_(y.detach(), non_blocking=True)
        self.out_host["dx"].copy_(x.grad, non_blocking=True)
        self.out_dw.copy_(w.grad, non_blocking=True)


# ----------------------------------------------------------------------------- CPU baseline / reference arm


def cpu_norm_baseline(sample_rows: int = 8192, repeats: int = 5, threads: int | None = None) -> dict:
    """Time the oracle restatement (numpy, f32 statistics) of add+RMSNorm fwd+bwd on
    ``sample_rows`` x 4096 bf16 rows, split over ``threads`` host threads."""
    import concurrent.futures as cf

    import ml_dtypes

    sys.path.insert(0, ROOT)
    from oracle import rmsnorm as on

    threads = threads or _host_cores()
    rng = np.random.default_rng(0)
    bf = ml_dtypes.bfloat16
    x = rng.standard_normal((sample_rows, DIM), dtype=np.float32).astype(bf)
    r = rng.standard_normal((sample_rows, DIM), dtype=np.float32).astype(bf)
    dy = rng.standard_normal((sample_rows, DIM), dtype=np.float32).astype(bf)
    dhd = rng.standard_normal((sample_rows, DIM), dtype=np.float32).astype(bf)
    w = (1 + 0.1 * rng.standard_normal(DIM)).astype(np.float32)
    chunks = np.array_split(np.arange(sample_rows), threads)

    def work(idx):
        h, y = on.add_rmsnorm_fwd(x[idx], r[idx], w, EPS)
        dh, dw = on.rmsnorm_bwd(h, w, dy[idx], dhd[idx], EPS)
        return dw

    times = []
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(work, chunks))  # warm-up
        for _ in range(repeats):
            t0 = time.perf_counter()
            parts = list(ex.map(work, chunks))
            np.sum(parts, axis=0)  # the dw exchange across chunks
            times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    bytes_sample = STEP_BYTES * sample_rows / ROWS
    return {
        "value": bytes_sample / t / 1e9,
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{sample_rows} of {ROWS} rows x {DIM} (fwd+bwd), median of {repeats}, numpy oracle over {threads} threads",
        "seconds_per_sample": t,
    }


# ----------------------------------------------------------------------------- main


def run_ours(args, ws, rank, local):
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    wl = NormWorkload(dev)
    dw_sum = torch.empty_like(wl.dw)

    def one_step(i, ev=None):
        wl.step(i, ev)
        if ws > 1:
            dw_sum.copy_(wl.dw)
            dist.all_reduce(dw_sum)

    for i in range(args.warmup):
        one_step(i)
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)

    # untimed pre-roll length (same on every rank): about 0.6 s of steps
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    for i in range(4):
        wl.step(i)
    p1.record()
    torch.cuda.synchronize(dev)
    n_pre = torch.tensor([max(1, int(600.0 / max(p0.elapsed_time(p1) / 4, 1e-3)))], device=dev)
    if ws > 1:
        dist.all_reduce(n_pre, op=dist.ReduceOp.MAX)
    n_pre = int(min(n_pre.item(), 20000))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        # nvidia-smi samples every 100 ms; keep the GPU under the same load (untimed
        # steps) until the sampler is producing samples, so the clock record covers
        # the loaded window that ends with the timed region.
        for i in range(n_pre):
            one_step(i)
        torch.cuda.synchronize(dev)
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        start.record()
        for i in range(args.steps):
            one_step(i, evs[i])
        stop.record()
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(stop)
    fwd_ms = [e[0].elapsed_time(e[1]) for e in evs]
    bwd_ms = [e[1].elapsed_time(e[2]) for e in evs]
    t = torch.tensor([ms, statistics.mean(fwd_ms), statistics.mean(bwd_ms)], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, fwd_avg, bwd_avg = (float(v) for v in t.tolist())
    value = STEP_BYTES * ws * args.steps / (ms / 1e3) / 1e9

    # end-to-end through the public API with host buffers
    wl.e2e_setup()
    for _ in range(max(1, args.warmup)):
        wl.e2e_step()
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        wl.e2e_step()
    e1.record()
    torch.cuda.synchronize(dev)
    e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_value = STEP_BYTES * ws * args.steps / (float(e_ms.item()) / 1e3) / 1e9

    from ferrite import platform

    pk = platform.peaks()
    dominant = ("add_rmsnorm_fwd", fwd_avg, FWD_BYTES) if fwd_avg >= bwd_avg else ("rmsnorm_bwd", bwd_avg, BWD_BYTES)
    achieved = dominant[2] / (dominant[1] / 1e3) / 1e9
    peak = pk.hbm_bytes_per_s / 1e9
    out = {
        "metric": wl.metric,
        "value": round(value, 1),
        "unit": wl.unit,
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {
            "workload": wl.name,
            "rows_per_gpu": ROWS,
            "dim": DIM,
            "eps": EPS,
            "algorithmic_bytes_per_step_per_gpu": STEP_BYTES,
            "l2": "inputs larger than L2 (two 448 MiB buffer sets alternate)",
            "parallelism": f"tokens sharded, {ws} rank(s), dw all-reduce" if ws > 1 else "single GPU",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": dominant[0],
            "achieved": round(achieved, 1),
            "peak": round(peak, 1),
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_source": f"{pk.source} (MEASURED_PEAKS.json hbm_gbs)" if pk.source == "measured" else "fallback 6.65 TB/s",
            "traffic": _load_traffic(dominant[0]),
            "kernels_ms": {"add_rmsnorm_fwd": round(fwd_avg, 5), "rmsnorm_bwd+dw_reduce": round(bwd_avg, 5)},
            "kernels_gbs": {
                "add_rmsnorm_fwd": round(FWD_BYTES / (fwd_avg / 1e3) / 1e9, 1),
                "rmsnorm_bwd+dw_reduce": round(BWD_BYTES / (bwd_avg / 1e3) / 1e9, 1),
            },
        },
        "e2e": {
            "value": round(e2e_value, 2),
            "unit": wl.unit,
            "h2d_bytes_per_step": wl.h2d_bytes,
            "d2h_bytes_per_step": wl.d2h_bytes,
            "api": "ferrite.kernels.rmsnorm.rmsnorm(x, w, residual=r) + autograd backward, pinned host buffers",
        },
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_norm_baseline(sample_rows=args.cpu_rows)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_reference(args, ws, rank):
    if rank != 0:
        return
    steps = []
    for _ in range(args.warmup):
        cpu_norm_baseline(sample_rows=args.cpu_rows, repeats=1)
    for _ in range(args.steps):
        steps.append(cpu_norm_baseline(sample_rows=args.cpu_rows, repeats=1))
    v = statistics.median(s["value"] for s in steps)
    base = steps[0]
    out = {
        "metric": NormWorkload.metric,
        "value": round(v, 3),
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(statistics.median(s["seconds_per_sample"] for s in steps) * 1e3 * ROWS / args.cpu_rows, 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "impl": "reference",
        "config": {"workload": NormWorkload.name, "rows_per_gpu": ROWS, "dim": DIM, "eps": EPS},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": base["cores"], "kind": "port", "sample": base["sample"]},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "JAX (the reference's runtime) is not installable here; the reference's CPU path is timed as the numpy restatement in oracle/",
    }
    print(json.dumps(out), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["norm"], default="norm")
    ap.add_argument("--cpu-rows", type=int, default=8192, help="rows in the bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)  # timing rule: at least 3 untimed warm-up steps
    ws, rank, local = _dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
