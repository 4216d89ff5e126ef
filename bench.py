"""Benchmark driver: one JSON line for one workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload norm|attn|gemm|gpt|prefill|decode]

Workloads (the benchmark configs; synthetic inputs, seeded):

* ``attn`` (default, configs[3]) -- causal flash attention fwd + bwd, b8 h32 s8192
  d128 bf16 (the north star's primary target), the 256 (batch, head) slices
  sharded over ranks (strong scaling, no communication).  One step = forward,
  delta prep, dK/dV (which stores dS) and dQ from dS.  Metric: algorithmic
  TFLOP/s (fwd + bwd = 3.5 x fwd, flash_attention.py:383-390).
* ``norm`` -- fused residual-add + RMSNorm forward +
  backward, x/residual bf16 [8192, 4096] ~ N(0,1), weight f32 1 + 0.1 N(0,1),
  eps 1e-6, upstream grads bf16 ~ N(0,1).  One step = ``add_rmsnorm_fwd`` on one
  buffer set + ``rmsnorm_bwd`` (dh and the deterministic dw reduction) on the
  other set's saved h; the two 448 MiB sets alternate, so no kernel reads
  L2-resident operands (L2 is 126 MB).  Metric: algorithmic HBM bytes / s.
  Multi-GPU: weak scaling, every rank normalises its own 8192-token shard; the
  only exchange is the backward's all-reduce of the f32 dw partial (16 KiB).
* ``gemm`` -- bf16 8192^3 forward + the two backward GEMMs of the
  VJP; replicas at N > 1.  Metric: TFLOP/s.
* ``gpt`` -- GPT training step (d1024 L24 H16 ff4096 V32000 s1024,
  global batch 64, data-parallel over ranks with one NCCL gradient all-reduce,
  AdamW), all kernels on the B200 path.  Metric: tokens/s.
* ``prefill`` -- bucketed prefill of 8 prompts x 512 into the
  static [24, 8, 16, 512, 64] KV cache through a captured CUDA graph.  Metric:
  prefill tokens/s.
* ``decode`` (configs[4], decode) -- the attention of one greedy-decode step in all
  24 layers: new K/V rows written into the static [24, 8, 16, 1024, 64] bf16 cache
  and softmax(q K^T) V over positions 0..1023 (the last step of a 1024-token
  context), one fused kernel per layer, the 24 launches replayed as one CUDA graph.
  Metric: algorithmic HBM bytes / s (the cached K and V rows dominate).

Timing: W untimed warm-up steps, an untimed pre-roll (~0.6 s) while nvidia-smi
starts sampling clocks, then exactly K steps between a barrier + synchronize on
both sides, CUDA events on the launching stream around the region only, max over
ranks.  The per-kernel times behind ``roofline`` come from a second pass of the same
K steps with events recorded between the kernels (those events serialise the
kernels, so they stay out of the headline region).  ``e2e``
repeats the measurement through the public API with pinned host inputs copied
in and results copied out every step.

``--impl reference`` times the CPU restatement of the reference's path (the
``oracle`` package: JAX, the reference's runtime, cannot be installed here) on
the host cores; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import ctypes
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
            self.bus = int(getattr(torch.cuda.get_device_properties(device), "pci_bus_id"))
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
        return out


def _load_traffic(kernel: str):
    """Per-launch DRAM bytes of ``kernel`` from the committed ncu summary (profiles/ncu_traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(kernel, {}).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


def _events(n):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def _fp32_line(kernel: str, flops: float, seconds: float) -> dict:
    """Roofline object for the exact-f32 CUDA-core GEMM: against the nominal FP32 FMA rate
    (SMs x 128 lanes x 2 FLOP x the maximum SM clock), there being no measured figure."""
    from ferrite import platform

    sms = platform.sm_count()
    mhz = 1965.0
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mhz = float(json.load(f).get("sm_max_mhz", mhz))
    except (OSError, ValueError):
        pass
    peak = sms * 128 * 2 * mhz * 1e6 / 1e12
    achieved = flops / seconds / 1e12
    return {"bound": "fp32", "kernel": kernel, "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "peak_source": f"nominal FP32 FMA rate ({sms} SMs x 128 lanes x 2 x {mhz:.0f} MHz)",
            "traffic": None}


def _oracle_pool(workers: int):
    """A process pool for the CPU oracle: spawned (never forked from a process that
    holds a CUDA context) with single-threaded BLAS in every worker, so ``workers``
    processes use ``workers`` cores."""
    import concurrent.futures as cf
    import multiprocessing as mp

    keys = ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")
    saved = {k: os.environ.get(k) for k in keys}
    os.environ.update({k: "1" for k in keys})
    try:
        ex = cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn"))
        list(ex.map(abs, range(workers)))  # start every worker while the variables are set
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return ex


def _attn_oracle_slice(args):
    """One causal (b, h) slice through the oracle's blockwise forward and backward."""
    seed, s, d = args
    import ml_dtypes

    sys.path.insert(0, ROOT)
    from oracle import attention as oa

    rng = np.random.default_rng(seed)
    q, k, v, do = (rng.standard_normal((1, 1, s, d), dtype=np.float32).astype(ml_dtypes.bfloat16) for _ in range(4))
    o, lse = oa.flash_fwd(q, k, v, causal=True)
    oa.flash_bwd(q, k, v, o, lse, do, causal=True)
    return s


# ----------------------------------------------------------------------------- workloads


class NormWorkload:
    """fused add + RMSNorm fwd + bwd, 8192 x 4096 bf16 per rank."""

    name = "add_rmsnorm_fwd_bwd_bf16_8192x4096"
    metric = "add+RMSNorm fwd+bwd HBM GB/s"
    unit = "GB/s"
    dtype = "bf16"
    scaling = "weak"
    bound = "hbm"
    ROWS, DIM, EPS = 8192, 4096, 1e-6
    FWD_BYTES = 4 * ROWS * DIM * 2 + 4 * DIM  # read x, r; write h, y (bf16); read w (f32)
    BWD_BYTES = 4 * ROWS * DIM * 2 + 4 * DIM + 4 * DIM  # read h, dy, dh_direct; write dh; read w; write dw
    kernels = ("add_rmsnorm_fwd", "rmsnorm_bwd+dw_reduce")
    kernel_work = {"add_rmsnorm_fwd": FWD_BYTES, "rmsnorm_bwd+dw_reduce": BWD_BYTES}
    launches_per_step = 3  # add_rmsnorm_fwd, rmsnorm_bwd, dw_reduce
    n_events = 3

    def __init__(self, dev, ws, rank, shape=None):
        from ferrite import _native as nat

        if shape:  # smaller cases for profiling captures: "rows,dim"
            self.ROWS, self.DIM = shape
            self.FWD_BYTES = 4 * self.ROWS * self.DIM * 2 + 4 * self.DIM
            self.BWD_BYTES = 4 * self.ROWS * self.DIM * 2 + 8 * self.DIM
            self.kernel_work = {"add_rmsnorm_fwd": self.FWD_BYTES, "rmsnorm_bwd+dw_reduce": self.BWD_BYTES}
        self.nat, self.lib, self.dev, self.ws = nat, nat.lib(), dev, ws
        R, D = self.ROWS, self.DIM
        g = torch.Generator(device=dev)
        g.manual_seed(1234 + rank)

        def rn(*shape):
            return torch.randn(*shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)

        self.sets = []
        for _ in range(2):
            self.sets.append({
                "x": rn(R, D), "r": rn(R, D), "dy": rn(R, D), "dhd": rn(R, D),
                "h": torch.empty(R, D, dtype=torch.bfloat16, device=dev),
                "y": torch.empty(R, D, dtype=torch.bfloat16, device=dev),
                "dh": torch.empty(R, D, dtype=torch.bfloat16, device=dev),
            })
        self.w = (1.0 + 0.1 * torch.randn(D, generator=g, device=dev)).float()
        # the sharded backward's one exchange (ferrite.sharding.DwExchange): dw of step i
        # is summed over ranks on NCCL's stream (one-CTA communicator) while the next
        # step's kernels run; its buffer is rewritten two steps later, after a wait
        from ferrite.sharding import DwExchange, one_cta_nccl_group

        self.exchange = DwExchange(D, dev, group=one_cta_nccl_group() if ws > 1 else None)
        self.ws_buf = torch.empty(int(self.lib.ferrite_rmsnorm_bwd_workspace_size(R, D)), dtype=torch.uint8, device=dev)
        for s in self.sets:
            self._fwd(s)
        torch.cuda.synchronize(dev)

    @property
    def units_per_step(self):
        return self.FWD_BYTES + self.BWD_BYTES

    def _fwd(self, s):
        nat = self.nat
        nat.check(self.lib.ferrite_add_rmsnorm_fwd(
            nat.stream_ptr(self.dev), s["x"].data_ptr(), s["r"].data_ptr(), self.w.data_ptr(), s["h"].data_ptr(), s["y"].data_ptr(),
            self.ROWS, self.DIM, self.EPS, nat.BF16, nat.F32))

    def _bwd(self, s, dw):
        nat = self.nat
        nat.check(self.lib.ferrite_rmsnorm_bwd(
            nat.stream_ptr(self.dev), s["h"].data_ptr(), self.w.data_ptr(), s["dy"].data_ptr(), s["dhd"].data_ptr(), s["dh"].data_ptr(),
            dw.data_ptr(), self.ws_buf.data_ptr(), self.ws_buf.numel(), self.ROWS, self.DIM, self.EPS, nat.BF16, nat.F32))

    def step(self, i, ev=None):
        a, b = self.sets[i % 2], self.sets[(i + 1) % 2]
        if ev:
            ev[0].record()
        self._fwd(a)
        if ev:
            ev[1].record()
        self._bwd(b, self.exchange.buffer(i))  # the stream first waits for step i - 2's all-reduce
        if ev:
            ev[2].record()
        self.exchange.start(i)

    def breakdown(self, evs):
        fwd = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
        bwd = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
        return {"add_rmsnorm_fwd": fwd, "rmsnorm_bwd+dw_reduce": bwd}

    @classmethod
    def static_config(cls, ws):
        """The config keys, from the class (the reference arm prints the same ones)."""
        return {
            "workload": cls.name, "rows_per_gpu": cls.ROWS, "dim": cls.DIM, "eps": cls.EPS,
            "algorithmic_bytes_per_step_per_gpu": cls.FWD_BYTES + cls.BWD_BYTES,
            "l2": "inputs larger than L2 (two 448 MiB buffer sets alternate)",
            "parallelism": f"tokens sharded, {ws} rank(s), dw all-reduce" if ws > 1 else "single GPU",
        }

    def config(self):
        return {**self.static_config(self.ws), "rows_per_gpu": self.ROWS, "dim": self.DIM,
                "algorithmic_bytes_per_step_per_gpu": self.units_per_step}

    def e2e_setup(self):
        s = self.sets[0]
        self.host = {k: s[k].cpu().pin_memory() for k in ("x", "r", "dy", "dhd")}
        self.host_w = self.w.cpu().pin_memory()
        self.out_host = {k: torch.empty(self.ROWS, self.DIM, dtype=torch.bfloat16).pin_memory() for k in ("h", "y", "dx")}
        self.out_dw = torch.empty(self.DIM, dtype=torch.float32).pin_memory()
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host.values()) + self.host_w.numel() * 4
        self.d2h_bytes = sum(t.numel() * t.element_size() for t in self.out_host.values()) + self.DIM * 4
        self.e2e_api = "ferrite.kernels.rmsnorm.rmsnorm(x, w, residual=r) + autograd backward, pinned host buffers"

    def e2e_step(self):
        from ferrite.kernels.rmsnorm import rmsnorm

        d = self.dev
        x = self.host["x"].to(d, non_blocking=True).requires_grad_(True)
        r = self.host["r"].to(d, non_blocking=True).requires_grad_(True)
        w = self.host_w.to(d, non_blocking=True).requires_grad_(True)
        dy = self.host["dy"].to(d, non_blocking=True)
        dhd = self.host["dhd"].to(d, non_blocking=True)
        h, y = rmsnorm(x, w, residual=r, eps=self.EPS)
        torch.autograd.backward([h, y], [dhd, dy])
        self.out_host["h"].copy_(h.detach(), non_blocking=True)
        self.out_host["y"].copy_(y.detach(), non_blocking=True)
        self.out_host["dx"].copy_(x.grad, non_blocking=True)
        self.out_dw.copy_(w.grad, non_blocking=True)

    @classmethod
    def cpu_baseline(cls, sample_rows=8192, repeats=5, threads=None):
        """The oracle restatement (numpy, f32 statistics) of add+RMSNorm fwd+bwd on
        ``sample_rows`` x 4096 bf16 rows, split over ``threads`` host threads."""
        import concurrent.futures as cf

        import ml_dtypes

        sys.path.insert(0, ROOT)
        from oracle import rmsnorm as on

        threads = threads or _host_cores()
        rng = np.random.default_rng(0)
        bf = ml_dtypes.bfloat16
        D, E = cls.DIM, cls.EPS
        x, r, dy, dhd = (rng.standard_normal((sample_rows, D), dtype=np.float32).astype(bf) for _ in range(4))
        w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
        chunks = np.array_split(np.arange(sample_rows), threads)

        def work(idx):
            h, _ = on.add_rmsnorm_fwd(x[idx], r[idx], w, E)
            _, dw = on.rmsnorm_bwd(h, w, dy[idx], dhd[idx], E)
            return dw

        times = []
        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(work, chunks))
            for _ in range(repeats):
                t0 = time.perf_counter()
                parts = list(ex.map(work, chunks))
                np.sum(parts, axis=0)  # the dw exchange across chunks
                times.append(time.perf_counter() - t0)
        t = statistics.median(times)
        work_bytes = (cls.FWD_BYTES + cls.BWD_BYTES) * sample_rows / cls.ROWS
        return {"value": work_bytes / t / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                "sample": f"{sample_rows} of {cls.ROWS} rows x {D} (fwd+bwd), median of {repeats}, numpy oracle over {threads} threads",
                "seconds_per_sample": t, "sample_fraction": sample_rows / cls.ROWS}


class AttnWorkload:
    """causal flash attention fwd + bwd, b8 h32 s8192 d128 bf16, heads sharded."""

    name = "flash_attention_causal_fwd_bwd_b8_h32_s8192_d128_bf16"
    metric = "causal flash-attn fwd+bwd TFLOP/s"
    unit = "TFLOP/s"
    dtype = "bf16"
    scaling = "strong"
    bound = "tensor"
    B, H, S, D = 8, 32, 8192, 128
    L2_NOTE = "inputs larger than L2 (q, k, v, dO 512 MiB each at 1 GPU)"
    kernels = ("attn_fwd", "attn_bwd_prep", "attn_bwd")
    launches_per_step = 3
    n_events = 4

    def __init__(self, dev, ws, rank, shape=None):
        from ferrite.kernels.flash_attention import DS_WORKSPACE_BUDGET, attention_flops

        if shape:  # smaller cases for profiling captures: "b,h,s,d"
            self.B, self.H, self.S, self.D = shape
        self.dev, self.ws = dev, ws
        bh = self.B * self.H
        if bh % ws:
            raise ValueError("batch*heads must divide over ranks")
        from ferrite.sharding import attention_slices

        b0, b1 = attention_slices(self.B, self.H, ws, rank)  # this rank's (batch, head) slices
        self.bh_local = b1 - b0
        g = torch.Generator(device=dev)
        g.manual_seed(rank)
        shape = (1, self.bh_local, self.S, self.D)  # this rank's (b, h) slices as one batch row
        self.q, self.k, self.v, self.do = (torch.randn(*shape, generator=g, device=dev).to(torch.bfloat16) for _ in range(4))
        self.fwd_flops_local = attention_flops(1, self.bh_local, self.S, self.S, self.D, causal=True)
        # tensor-core work each kernel issues, in units of one causal S*S*D/2 product:
        # fwd 2 (S, PV); the fused backward 5 (dK/dV units: S, dP, dV, dK; dQ units: dS K)
        unit = self.fwd_flops_local / 2
        self.kernel_work = {"attn_fwd": 2 * unit, "attn_bwd_prep": 0, "attn_bwd": 5 * unit}
        self.o = torch.empty_like(self.q)
        self.lse = torch.empty(1, self.bh_local, self.S, device=dev)
        self.delta = torch.empty_like(self.lse)
        self.dq, self.dk, self.dv = (torch.empty_like(self.q) for _ in range(3))
        from ferrite import _native as nat

        # dS scratch + scheduler state, sized like the Python API's (flash_attention.DS_WORKSPACE_BUDGET)
        full = nat.lib().ferrite_attn_bwd_ds_workspace_size(1, self.bh_local, self.S, self.S, self.D, nat.BF16)
        per = full // self.bh_local
        self.ds = torch.empty(max(per, min(full, DS_WORKSPACE_BUDGET // per * per)), dtype=torch.uint8, device=dev)
        self.strides = nat.attn_strides(q=self.q, k=self.k, v=self.v, o=self.o, dout=self.do, dq=self.dq, dk=self.dk, dv=self.dv)

    @property
    def units_per_step(self):
        return 3.5 * self.fwd_flops_local  # per rank (bench_kernels.py:119)

    def step(self, i, ev=None):
        from ferrite import _native as nat

        lib = nat.lib()
        s = nat.stream_ptr(self.dev)
        bh, S, D = self.bh_local, self.S, self.D
        sc = 1.0 / np.sqrt(D)
        if ev:
            ev[0].record()
        nat.check(lib.ferrite_attn_fwd(s, self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.o.data_ptr(), self.lse.data_ptr(), 1, bh, S, S, D, sc, 1, 128, 128, nat.BF16))
        if ev:
            ev[1].record()
        nat.check(lib.ferrite_attn_bwd_prep(s, self.do.data_ptr(), self.o.data_ptr(), self.delta.data_ptr(), 1, bh, S, D, nat.BF16))
        if ev:
            ev[2].record()
        st = ctypes.byref(self.strides)
        nat.check(lib.ferrite_attn_bwd_ds(s, self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self.do.data_ptr(), self.lse.data_ptr(),
                                          self.delta.data_ptr(), self.dq.data_ptr(), self.dk.data_ptr(), self.dv.data_ptr(), st, self.ds.data_ptr(),
                                          self.ds.numel(), 1, bh, S, S, D, sc, 1, 128, 128, nat.BF16))
        if ev:
            ev[3].record()

    def breakdown(self, evs):
        return {k: statistics.mean(e[j].elapsed_time(e[j + 1]) for e in evs) for j, k in enumerate(self.kernels)}

    @classmethod
    def static_config(cls, ws):
        """The config keys, from the class (the reference arm prints the same ones)."""
        return {"workload": cls.name, "batch": cls.B, "heads": cls.H, "seq_len": cls.S, "head_dim": cls.D, "causal": True,
                "block_q": 128, "block_k": 128, "heads_per_gpu": cls.B * cls.H // ws, "parallelism": f"batch*heads sharded over {ws} rank(s)",
                "l2": cls.L2_NOTE}

    def config(self):
        return {**self.static_config(self.ws), "batch": self.B, "heads": self.H, "seq_len": self.S, "head_dim": self.D,
                "heads_per_gpu": self.bh_local}

    def e2e_setup(self):
        self.host = {k: getattr(self, k).cpu().pin_memory() for k in ("q", "k", "v", "do")}
        self.out_host = {k: torch.empty_like(self.host["q"]).pin_memory() for k in ("o", "dq", "dk", "dv")}
        self.h2d_bytes = sum(t.numel() * 2 for t in self.host.values())
        self.d2h_bytes = sum(t.numel() * 2 for t in self.out_host.values())
        self.e2e_api = "ferrite.kernels.flash_attention.flash_attention(q, k, v, causal=True) + autograd backward, pinned host buffers"

    def e2e_step(self):
        from ferrite.kernels.flash_attention import flash_attention

        d = self.dev
        q, k, v = (self.host[n].to(d, non_blocking=True).requires_grad_(True) for n in ("q", "k", "v"))
        do = self.host["do"].to(d, non_blocking=True)
        o = flash_attention(q, k, v, causal=True)
        o.backward(do)
        for name, t in (("o", o.detach()), ("dq", q.grad), ("dk", k.grad), ("dv", v.grad)):
            self.out_host[name].copy_(t, non_blocking=True)

    @classmethod
    def cpu_baseline(cls, slices=None, threads=None):
        """The oracle's blockwise fwd + bwd (numpy) on ``slices`` of the 256 independent
        (b, h) slices (default: one per host core), one slice per process of a spawned
        pool with single-threaded BLAS in each, extrapolated linearly to the whole
        config (the slices are independent, so the work is linear in their number)."""
        threads = threads or _host_cores()
        slices = slices or threads
        with _oracle_pool(threads) as ex:
            list(ex.map(_attn_oracle_slice, [(i, 512, cls.D) for i in range(threads)]))  # warm-up: imports, BLAS
            t0 = time.perf_counter()
            list(ex.map(_attn_oracle_slice, [(i, cls.S, cls.D) for i in range(slices)]))
            t = time.perf_counter() - t0
        sys.path.insert(0, ROOT)
        from oracle import attention as oa

        flops = 3.5 * oa.attention_flops(1, slices, cls.S, cls.S, cls.D, causal=True)
        return {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"{slices} of {cls.B * cls.H} (b,h) slices of {cls.S} x {cls.D}, numpy blockwise oracle fwd+bwd, "
                          f"{threads} spawned processes (one slice each, single-threaded BLAS); extrapolated linearly in slices",
                "seconds_per_sample": t, "sample_fraction": slices / (cls.B * cls.H)}


class AttnSmallWorkload(AttnWorkload):
    """the reference's CPU-runnable attention case, causal fwd + bwd at
    b2 h4 s512 d64 bf16 (blocks 128)."""

    name = "flash_attention_causal_fwd_bwd_b2_h4_s512_d64_bf16"
    metric = "causal flash-attn fwd+bwd TFLOP/s (b2 h4 s512 d64)"
    B, H, S, D = 2, 4, 512, 64
    L2_NOTE = "inputs 256 KiB each (L2-resident; launch-latency bound)"

    @classmethod
    def cpu_baseline(cls, slices=None, threads=None):
        return super().cpu_baseline(slices=cls.B * cls.H, threads=min(threads or _host_cores(), cls.B * cls.H))


class GemmWorkload:
    """bf16 8192^3 forward + the two backward GEMMs (replicas at N > 1)."""

    name = "matmul_bf16_8192cubed_fwd_and_vjp"
    metric = "matmul bf16 8192^3 fwd+2bwd TFLOP/s"
    unit = "TFLOP/s"
    dtype = "bf16"
    scaling = "weak"
    bound = "tensor"
    M = N = K = 8192
    TORCH_DTYPE = torch.bfloat16
    L2_NOTE = "operands 128 MiB each (larger than L2)"
    kernels = ("gemm_fwd", "gemm_dA", "gemm_dB")
    launches_per_step = 3
    n_events = 4

    def __init__(self, dev, ws, rank, shape=None):
        if shape:  # "m,n,k"
            self.M, self.N, self.K = shape
        self.dev, self.ws = dev, ws
        g = torch.Generator(device=dev)
        g.manual_seed(rank)
        sk = 1 / np.sqrt(self.K)
        dt = self.TORCH_DTYPE
        self.a = (torch.randn(self.M, self.K, generator=g, device=dev) * sk).to(dt)
        self.b = (torch.randn(self.K, self.N, generator=g, device=dev) * sk).to(dt)
        self.gout = torch.randn(self.M, self.N, generator=g, device=dev).to(dt)
        self.c = torch.empty(self.M, self.N, dtype=dt, device=dev)
        self.da = torch.empty_like(self.a)
        self.db = torch.empty_like(self.b)
        f = 2 * self.M * self.N * self.K
        self.kernel_work = {"gemm_fwd": f, "gemm_dA": f, "gemm_dB": f}

    @property
    def units_per_step(self):
        return 3 * 2 * self.M * self.N * self.K

    def step(self, i, ev=None):
        from ferrite.kernels.matmul import gemm

        if ev:
            ev[0].record()
        gemm(self.a, self.b, out=self.c)
        if ev:
            ev[1].record()
        gemm(self.gout, self.b, trans_b=True, out=self.da)
        if ev:
            ev[2].record()
        gemm(self.a, self.gout, trans_a=True, out=self.db)
        if ev:
            ev[3].record()

    def breakdown(self, evs):
        return {k: statistics.mean(e[j].elapsed_time(e[j + 1]) for e in evs) for j, k in enumerate(self.kernels)}

    def config(self):
        return {"workload": self.name, "m": self.M, "n": self.N, "k": self.K, "parallelism": "independent replicas" if self.ws > 1 else "single GPU",
                "l2": self.L2_NOTE}

    def e2e_setup(self):
        self.host = {"a": self.a.cpu().pin_memory(), "b": self.b.cpu().pin_memory(), "g": self.gout.cpu().pin_memory()}
        self.out_host = {"c": torch.empty(self.M, self.N, dtype=self.TORCH_DTYPE).pin_memory(),
                         "da": torch.empty(self.M, self.K, dtype=self.TORCH_DTYPE).pin_memory(),
                         "db": torch.empty(self.K, self.N, dtype=self.TORCH_DTYPE).pin_memory()}
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host.values())
        self.d2h_bytes = sum(t.numel() * t.element_size() for t in self.out_host.values())
        self.e2e_api = "ferrite.kernels.matmul.matmul(x, y) + autograd backward, pinned host buffers"

    def e2e_step(self):
        from ferrite.kernels.matmul import matmul

        d = self.dev
        x = self.host["a"].to(d, non_blocking=True).requires_grad_(True)
        y = self.host["b"].to(d, non_blocking=True).requires_grad_(True)
        g = self.host["g"].to(d, non_blocking=True)
        c = matmul(x, y)
        c.backward(g)
        self.out_host["c"].copy_(c.detach(), non_blocking=True)
        self.out_host["da"].copy_(x.grad, non_blocking=True)
        self.out_host["db"].copy_(y.grad, non_blocking=True)

    @classmethod
    def cpu_baseline(cls, rows=256, threads=None):
        """numpy f32 (BLAS, all threads) on a ``rows``-row sample of A and G (the three
        products scale linearly in the sampled rows)."""
        rng = np.random.default_rng(0)
        a = rng.standard_normal((rows, cls.K), dtype=np.float32)
        b = rng.standard_normal((cls.K, cls.N), dtype=np.float32)
        g = rng.standard_normal((rows, cls.N), dtype=np.float32)
        a @ b  # warm-up
        t0 = time.perf_counter()
        a @ b
        g @ b.T
        a.T @ g
        t = time.perf_counter() - t0
        flops = 3 * 2 * rows * cls.N * cls.K
        return {"value": flops / t / 1e12, "unit": "TFLOP/s", "cores": threads or _host_cores(), "kind": "port",
                "sample": f"{rows} of {cls.M} rows, numpy f32 BLAS (oracle matmul_reference / matmul_vjp arithmetic)",
                "seconds_per_sample": t, "sample_fraction": rows / cls.M}


class GemmRaggedWorkload(GemmWorkload):
    """configs[2], ragged case: bf16 M=4000, N=3000, K=5000 forward + both VJP products
    (no dimension a multiple of the 128 / 256 tiles: TMA zero-fills the edges)."""

    name = "matmul_bf16_ragged_4000x3000x5000_fwd_and_vjp"
    metric = "matmul bf16 4000x3000x5000 fwd+2bwd TFLOP/s"
    M, N, K = 4000, 3000, 5000
    L2_NOTE = "operands 30-40 MB each (inside L2; the shapes' edge tiles dominate)"


class GemmF32Workload(GemmWorkload):
    """configs[2], f32 case: 2048^3 at Precision.HIGHEST (exact f32 products on the CUDA
    cores, _compat.py:17-26), forward + both VJP products."""

    name = "matmul_f32_2048cubed_highest_fwd_and_vjp"
    metric = "matmul f32 2048^3 HIGHEST fwd+2bwd TFLOP/s"
    dtype = "f32"
    bound = "fp32"  # CUDA-core FMA rate, not the tensor cores
    M = N = K = 2048
    TORCH_DTYPE = torch.float32
    L2_NOTE = "operands 16 MiB each (inside L2)"


GPT_CFG = dict(vocab_size=32000, seq_len=1024, d_model=1024, n_head=16, n_layer=24, d_ff=4096)


class GptWorkload:
    """one data-parallel GPT training step, global batch 64 x 1024 tokens."""

    name = "gpt_train_step_d1024_L24_H16_ff4096_V32000_s1024_b64"
    metric = "GPT train tokens/s"
    unit = "tokens/s"
    dtype = "bf16"
    scaling = "strong"
    bound = "tensor"
    GLOBAL_BATCH = 64
    n_events = 2
    kernels = ("train_step",)

    def __init__(self, dev, ws, rank, shape=None):
        from ferrite import _native as nat
        from ferrite.model.gpt import GPTConfig, flops_per_token, init_params, param_count, param_leaves
        from ferrite.model.train import TrainConfig, build_train_step, make_optimizer

        self.dev, self.ws, self.rank = dev, ws, rank
        if shape:  # "global_batch": e.g. one GPU at the per-rank batch of a dp run
            self.GLOBAL_BATCH = int(shape[0])
        self.cfg = GPTConfig(**GPT_CFG, attention="pallas", norm="pallas", linear="pallas", dtype=torch.bfloat16)
        self.tcfg = TrainConfig(steps=1000, batch=self.GLOBAL_BATCH, lr=6e-4, warmup=20)
        if self.GLOBAL_BATCH % ws:
            raise ValueError("global batch must divide over ranks")
        self.local_batch = self.GLOBAL_BATCH // ws
        self.params = init_params(0, self.cfg, device=dev)
        leaves = param_leaves(self.params)
        for p in leaves:
            p.requires_grad_(True)
        n = param_count(self.params)
        nonembed = n - self.params["tok_emb"].numel() - self.params["pos_emb"].numel()
        self.flops_per_step_global = 3 * flops_per_token(self.cfg, nonembed)["total"] * self.GLOBAL_BATCH * self.cfg.seq_len
        # native fused AdamW over flat buffers; at N > 1 the gradient all-reduce runs in
        # buckets during backward (tied embedding and position table reduced last)
        self.opt, self.flat = make_optimizer(leaves, self.tcfg, late=(self.params["tok_emb"], self.params["pos_emb"]))
        self._step = build_train_step(self.cfg, self.tcfg, leaves, self.opt, self.flat, self.params)
        rng = np.random.default_rng(rank)
        ids = rng.integers(0, self.cfg.vocab_size, size=(self.local_batch, self.cfg.seq_len + 1))
        self.x = torch.from_numpy(ids[:, :-1]).to(dev)
        self.y = torch.from_numpy(ids[:, 1:]).to(dev)
        self.kernel_work = {"train_step": self.flops_per_step_global / ws}
        self._count_launches(nat)

    def _count_launches(self, nat):
        """Count native kernel launches of one step by wrapping every launching entry
        point of the C ABI (kernels per call: rmsnorm_bwd 2, adamw 2, a split-K gemm 2,
        the dS attention backward 2 per chunk of slices, everything else 1)."""
        lib = nat.lib()
        counts, kernels = {}, {}

        def per_call(name, a):
            if name in ("ferrite_rmsnorm_bwd", "ferrite_rmsnorm_bwd_noalloc", "ferrite_adamw_step"):
                return 2
            if name == "ferrite_gemm_ws":
                return 2 if a[-1] else 1
            if name == "ferrite_attn_bwd_ds":
                ws_bytes, b, h, sq, sk = a[12], a[13], a[14], a[15], a[16]
                per = ws_bytes // (((sq + 63) // 64) * 64 * sk * 2) if ws_bytes else 0
                return 2 * -(-(b * h) // per) if per else 2
            return 1

        originals = {}
        skip = ("ferrite_last_error", "ferrite_version", "ferrite_device_status")
        for name in nat.SIGNATURES:
            if name in skip or name.endswith("_workspace_size"):
                continue
            fn = getattr(lib, name)
            originals[name] = fn

            def wrap(*a, _fn=fn, _n=name):
                counts[_n] = counts.get(_n, 0) + 1
                kernels[_n] = kernels.get(_n, 0) + per_call(_n, a)
                return _fn(*a)

            setattr(lib, name, wrap)
        try:
            self._step(self.x, self.y)
            torch.cuda.synchronize(self.dev)
        finally:
            for name, fn in originals.items():
                setattr(lib, name, fn)
        self.launches_per_step = sum(kernels.values())
        self.launch_counts = counts

    @property
    def units_per_step(self):
        return self.local_batch * self.cfg.seq_len  # tokens this rank processes

    def step(self, i, ev=None):
        if ev:
            ev[0].record()
        self.loss, _ = self._step(self.x, self.y)
        if ev:
            ev[1].record()

    def breakdown(self, evs):
        return {"train_step": statistics.mean(e[0].elapsed_time(e[1]) for e in evs)}

    def config(self):
        return {"workload": self.name, "model": "ferrite GPT (pre-norm decoder)", **GPT_CFG, "global_batch": self.GLOBAL_BATCH,
                "per_gpu_batch": self.local_batch, "parallelism": f"dp{self.ws}", "optimizer": "AdamW (reference formula), clip 1.0",
                "init": "normal(0, 0.02), GPT-2 residual scaling", "data": "token ids uniform in [0, 32000)",
                "train_flops_per_step": self.flops_per_step_global, "native_launch_counts": self.launch_counts}

    def e2e_setup(self):
        self.host_x = self.x.cpu().pin_memory()
        self.host_y = self.y.cpu().pin_memory()
        self.loss_host = torch.empty((), dtype=torch.float32).pin_memory()
        self.h2d_bytes = 2 * self.host_x.numel() * 8
        self.d2h_bytes = 4
        self.e2e_api = "ferrite.model.train step (forward, backward, NCCL all-reduce, AdamW) with host token batches in, loss out"

    def e2e_step(self):
        x = self.host_x.to(self.dev, non_blocking=True)
        y = self.host_y.to(self.dev, non_blocking=True)
        loss, _ = self._step(x, y)
        self.loss_host.copy_(loss, non_blocking=True)

    @classmethod
    def cpu_baseline(cls, tokens=1024, threads=None):
        """The reference's plain path restated in torch f32 on the CPU (oracle/gpt.py),
        forward + backward of one 1024-token sequence of the full model."""
        sys.path.insert(0, ROOT)
        from oracle import gpt as og

        threads = threads or _host_cores()
        torch.set_num_threads(threads)
        cfg = dict(GPT_CFG)
        params = og.init(cfg)
        rng = np.random.default_rng(0)
        ids = torch.from_numpy(rng.integers(0, cfg["vocab_size"], size=(1, tokens + 1)))
        t0 = time.perf_counter()
        og.loss(params, ids[:, :-1], ids[:, 1:], cfg).backward()
        t = time.perf_counter() - t0
        return {"value": tokens / t, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": f"1 sequence x {tokens} tokens fwd+bwd (no optimizer), torch f32 CPU restatement (oracle/gpt.py)",
                "seconds_per_sample": t, "sample_fraction": tokens / (cls.GLOBAL_BATCH * cfg["seq_len"])}


class PrefillWorkload:
    """configs[4] serving half: bucketed prefill of 8 prompts x 512 into [24, 8, 16, 512, 64]."""

    name = "gpt_bucketed_prefill_8x512_into_kv_24x8x16x512x64"
    metric = "GPT prefill tokens/s"
    unit = "tokens/s"
    dtype = "bf16"
    scaling = "weak"
    bound = "tensor"
    n_events = 2
    kernels = ("prefill_graph",)
    PROMPTS, LEN = 8, 512

    def __init__(self, dev, ws, rank, shape=None):
        from ferrite.model.gpt import GPTConfig, flops_per_token, init_params, param_count
        from ferrite.serving.engine import Engine, ServeConfig

        self.dev, self.ws = dev, ws
        cfg = GPTConfig(**GPT_CFG, attention="pallas", norm="pallas", linear="pallas", dtype=torch.bfloat16)
        self.params = init_params(0, cfg, device=dev)
        self.engine = Engine(self.params, cfg, ServeConfig(batch=self.PROMPTS, max_len=512, buckets=(512,)))
        rng = np.random.default_rng(rank)
        self.prompts = [list(rng.integers(0, cfg.vocab_size, size=self.LEN)) for _ in range(self.PROMPTS)]
        n = param_count(self.params)
        nonembed = n - self.params["tok_emb"].numel() - self.params["pos_emb"].numel()
        self.kernel_work = {"prefill_graph": flops_per_token(cfg, nonembed)["total"] * self.PROMPTS * self.LEN}
        # one C call per kernel: per layer 2 norms, 4 GEMMs, 1 attention; final norm; LM head
        self.launches_per_step = cfg.n_layer * 7 + 2
        self.cfg = cfg

    @property
    def units_per_step(self):
        return self.PROMPTS * self.LEN

    def step(self, i, ev=None):
        if ev:
            ev[0].record()
        self.tok, _, _, _ = self.engine.prefill(self.prompts)
        if ev:
            ev[1].record()

    def breakdown(self, evs):
        return {"prefill_graph": statistics.mean(e[0].elapsed_time(e[1]) for e in evs)}

    def config(self):
        return {"workload": self.name, "model": "ferrite GPT (pre-norm decoder)", **GPT_CFG, "prompts": self.PROMPTS, "prompt_len": self.LEN,
                "bucket": 512, "kv_cache": [24, self.PROMPTS, 16, 512, 64], "parallelism": "replicas" if self.ws > 1 else "single GPU"}

    def e2e_setup(self):
        self.h2d_bytes = self.PROMPTS * self.LEN * 8 + self.PROMPTS * 8
        self.d2h_bytes = self.PROMPTS * 8
        self.e2e_api = "ferrite.serving.Engine.prefill(prompts) (host token lists in, first tokens out)"

    def e2e_step(self):
        tok, _, _, _ = self.engine.prefill(self.prompts)
        tok.cpu()

    @classmethod
    def cpu_baseline(cls, threads=None):
        """oracle/gpt.py forward on one 512-token prompt (torch f32, CPU)."""
        sys.path.insert(0, ROOT)
        from oracle import gpt as og

        threads = threads or _host_cores()
        torch.set_num_threads(threads)
        cfg = dict(GPT_CFG)
        params = og.init(cfg)
        ids = torch.from_numpy(np.random.default_rng(0).integers(0, cfg["vocab_size"], size=(1, cls.LEN + 1)))
        with torch.no_grad():
            t0 = time.perf_counter()
            og.loss(params, ids[:, :-1], ids[:, 1:], cfg)
            t = time.perf_counter() - t0
        return {"value": cls.LEN / t, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": f"1 prompt x {cls.LEN} tokens forward, torch f32 CPU restatement (oracle/gpt.py)", "seconds_per_sample": t,
                "sample_fraction": 1 / cls.PROMPTS}


class DecodeWorkload:
    """configs[4] serving half, decode: the attention of one greedy-decode step (cache
    write + softmax(q K^T) V over the static cache) in all 24 layers, for 8 sequences at
    the last position of a 1024-token context."""

    name = "gpt_decode_attention_kv_24x8x16x1024x64_pos1023_bf16"
    metric = "decode attention HBM GB/s"
    unit = "GB/s"
    dtype = "bf16"
    scaling = "weak"
    bound = "hbm"
    n_events = 2
    kernels = ("attn_decode",)
    L, B, H, T, D = 24, 8, 16, 1024, 64

    @classmethod
    def step_bytes(cls, layers, b, h, pos, d, esz=2):
        """Algorithmic bytes of one step: per (layer, b, h) the pos cached K and V rows,
        q / k_new / v_new read, o written, the new K and V rows written."""
        return layers * b * h * d * esz * (2 * pos + 3 + 1 + 2)

    def __init__(self, dev, ws, rank, shape=None):
        if shape:  # smaller cases: "layers,b,h,max_len,d"
            self.L, self.B, self.H, self.T, self.D = shape
        self.dev, self.ws = dev, ws
        g = torch.Generator(device=dev)
        g.manual_seed(77 + rank)
        L, B, H, T, D = self.L, self.B, self.H, self.T, self.D
        self.kc = torch.randn(L, B, H, T, D, generator=g, device=dev).to(torch.bfloat16)
        self.vc = torch.randn(L, B, H, T, D, generator=g, device=dev).to(torch.bfloat16)
        self.qkv = torch.randn(L, B, 3, H, D, generator=g, device=dev).to(torch.bfloat16)  # each layer's projection
        self.pos = torch.full((B,), T - 1, dtype=torch.int64, device=dev)
        self.o = torch.empty(L, B, H, D, dtype=torch.bfloat16, device=dev)
        self.kernel_work = {"attn_decode": self.step_bytes(L, B, H, T - 1, D)}
        self.launches_per_step = L
        self._launch()  # first call: module load and per-device set-up, before the capture
        torch.cuda.synchronize(dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self._launch()
        torch.cuda.current_stream(dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._launch()

    def _launch(self):
        from ferrite import _native as nat

        lib = nat.lib()
        st = nat.stream_ptr(self.dev)
        B, H, T, D = self.B, self.H, self.T, self.D
        ld = 3 * H * D
        for i in range(self.L):
            base = self.qkv[i].data_ptr()
            nat.check(lib.ferrite_attn_decode(st, base, base + H * D * 2, base + 2 * H * D * 2, self.kc[i].data_ptr(), self.vc[i].data_ptr(),
                                              self.pos.data_ptr(), self.o[i].data_ptr(), B, H, T, D, ld, 1.0 / np.sqrt(D), nat.BF16))

    @property
    def units_per_step(self):
        return self.kernel_work["attn_decode"]

    def step(self, i, ev=None):
        if ev:
            ev[0].record()
        self.graph.replay()
        if ev:
            ev[1].record()

    def breakdown(self, evs):
        return {"attn_decode": statistics.mean(e[0].elapsed_time(e[1]) for e in evs)}

    def config(self):
        return {"workload": self.name, "kv_cache": [self.L, self.B, self.H, self.T, self.D], "pos": self.T - 1, "layers": self.L,
                "launches": "one ferrite_attn_decode per layer, the 24 captured in one CUDA graph",
                "l2": f"caches {2 * self.kc.numel() * 2 / 2**20:.0f} MiB, larger than L2",
                "parallelism": "replicas" if self.ws > 1 else "single GPU"}

    def e2e_setup(self):
        self.host_qkv = self.qkv.cpu().pin_memory()
        self.host_pos = self.pos.cpu().pin_memory()
        self.host_o = torch.empty(self.o.shape, dtype=self.o.dtype).pin_memory()
        self.h2d_bytes = self.host_qkv.numel() * 2 + self.host_pos.numel() * 8
        self.d2h_bytes = self.host_o.numel() * 2
        self.e2e_api = ("ferrite.kernels.decode_attention.decode_attention(q, k_cache[l], v_cache[l], pos, k_new, v_new) per layer, "
                        "eager; the new rows and positions copied in from pinned host memory and the outputs copied out every step, "
                        "the caches resident in HBM as in a decode server")

    def e2e_step(self):
        from ferrite.kernels.decode_attention import decode_attention

        qkv = self.host_qkv.to(self.dev, non_blocking=True)
        pos = self.host_pos.to(self.dev, non_blocking=True)
        for i in range(self.L):
            o = decode_attention(qkv[i, :, 0], self.kc[i], self.vc[i], pos, k_new=qkv[i, :, 1], v_new=qkv[i, :, 2])
            self.host_o[i].copy_(o, non_blocking=True)

    @classmethod
    def cpu_baseline(cls, layers=1, threads=None):
        """The oracle's decode step (numpy, the reference's masked full-cache attention)
        on ``layers`` of the 24 layers, extrapolated linearly."""
        import ml_dtypes

        sys.path.insert(0, ROOT)
        from oracle import attention as oa

        rng = np.random.default_rng(0)
        bf = ml_dtypes.bfloat16
        kc, vc = (rng.standard_normal((cls.B, cls.H, cls.T, cls.D), dtype=np.float32).astype(bf) for _ in range(2))
        q, kn, vn = (rng.standard_normal((cls.B, cls.H, cls.D), dtype=np.float32).astype(bf) for _ in range(3))
        pos = np.full(cls.B, cls.T - 1)
        t0 = time.perf_counter()
        for _ in range(layers):
            oa.decode_reference(q, kc, vc, pos, 1.0 / np.sqrt(cls.D), kn, vn)
        t = time.perf_counter() - t0
        nbytes = cls.step_bytes(layers, cls.B, cls.H, cls.T - 1, cls.D)
        return {"value": nbytes / t / 1e9, "unit": "GB/s", "cores": threads or _host_cores(), "kind": "port",
                "sample": f"{layers} of {cls.L} layers, numpy oracle (BLAS threads)", "seconds_per_sample": t,
                "sample_fraction": layers / cls.L}


WORKLOADS = {"norm": NormWorkload, "attn": AttnWorkload, "attn_small": AttnSmallWorkload, "gemm": GemmWorkload,
             "gemm_ragged": GemmRaggedWorkload, "gemm_f32": GemmF32Workload, "gpt": GptWorkload, "prefill": PrefillWorkload,
             "decode": DecodeWorkload}
DEFAULT_WORKLOAD = "attn"
# the other benchmark configs, measured after the default workload at N = 1 and reported
# as compact lines inside its JSON line (so one driver run covers every config)
OTHER_CONFIGS = ("attn_small", "norm", "gemm", "gemm_ragged", "gemm_f32", "gpt", "prefill", "decode")


# ----------------------------------------------------------------------------- runners


def run_ours(args, ws, rank, local):
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    W = WORKLOADS[args.workload]
    shape = tuple(int(v) for v in args.shape.split(",")) if args.shape else None
    out = measure(W, args, ws, rank, dev, shape, cpu_baseline=rank == 0 and ws == 1 and not args.no_cpu_baseline)
    if ws == 1 and shape is None and args.workload == DEFAULT_WORKLOAD and not args.no_other_configs:
        # every other benchmark config on the same GPU, each with its own roofline,
        # e2e and CPU baseline, reported inside this line
        import gc

        others = []
        for name in OTHER_CONFIGS:
            gc.collect()
            torch.cuda.empty_cache()
            sub = argparse.Namespace(**{**vars(args), "steps": min(args.steps, 10), "warmup": 3})
            others.append(measure(WORKLOADS[name], sub, 1, rank, dev, None, cpu_baseline=not args.no_cpu_baseline))
        out["other_configs"] = others
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def measure(W, args, ws, rank, dev, shape, cpu_baseline):
    """One workload: warm-up, the timed K steps, the per-kernel pass, the end-to-end
    pass through the public API and (optionally) the CPU baseline; returns its line."""
    import torch.distributed as dist

    wl = W(dev, ws, rank, shape)

    def sync_all():
        torch.cuda.synchronize(dev)
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for i in range(args.warmup):
        wl.step(i)
    sync_all()

    # untimed pre-roll length (same on every rank): about 0.6 s of steps
    p0, p1 = _events(2)
    p0.record()
    wl.step(0)
    p1.record()
    torch.cuda.synchronize(dev)
    n_pre = torch.tensor([max(1, int(600.0 / max(p0.elapsed_time(p1), 1e-3)))], device=dev)
    if ws > 1:
        dist.all_reduce(n_pre, op=dist.ReduceOp.MAX)
    n_pre = int(min(n_pre.item(), 20000))

    evs = [_events(wl.n_events) for _ in range(args.steps)]
    start, stop = _events(2)
    with ClockSampler(dev) as clk:
        for i in range(n_pre):
            wl.step(i)
        sync_all()
        # value: the K steps back to back, with events only around the whole region
        # (an event recorded between two kernels serialises them and costs ~5 us)
        start.record()
        for i in range(args.steps):
            wl.step(i)
        stop.record()
        torch.cuda.synchronize(dev)
        sync_all()
        # per-kernel breakdown (roofline): a second pass of the same K steps with
        # events between the kernels
        for i in range(args.steps):
            wl.step(i, evs[i])
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(stop)
    bd = wl.breakdown(evs)
    names = list(bd)
    t = torch.tensor([ms] + [bd[k] for k in names], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    bd = {k: float(v) for k, v in zip(names, t[1:].tolist())}
    scale = 1e9 if wl.unit == "GB/s" else (1e12 if wl.unit == "TFLOP/s" else 1.0)
    value = wl.units_per_step * ws * args.steps / (ms / 1e3) / scale

    # end to end through the public API with host buffers
    wl.e2e_setup()
    for _ in range(max(1, min(args.warmup, 3))):
        wl.e2e_step()
    sync_all()
    e0, e1 = _events(2)
    e0.record()
    for _ in range(args.steps):
        wl.e2e_step()
    e1.record()
    torch.cuda.synchronize(dev)
    e_ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_value = wl.units_per_step * ws * args.steps / (float(e_ms.item()) / 1e3) / scale

    from ferrite.profiling import roofline as rl

    dom = rl.dominant(bd, wl.kernel_work)
    # burst tensor peak for a sub-second timed region, sustained for a longer one
    sustained = rl.Ceilings.from_platform().for_region(ms / 1e3)
    work = wl.kernel_work[dom]
    point = rl.analyze(dom, flops=work if wl.bound != "hbm" else 0.0, bytes_=work if wl.bound == "hbm" else 0.0,
                       seconds=bd[dom] / 1e3, sustained=sustained)
    out = {
        "metric": wl.metric,
        "value": round(value, 3),
        "unit": wl.unit,
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": wl.scaling,
        "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic",
        "config": wl.config(),
        "roofline": {
            **(point.line(traffic=_load_traffic(dom)) if wl.bound != "fp32" else _fp32_line(dom, work, bd[dom] / 1e3)),
            "timing": "kernel times from a second pass of the same K steps with CUDA events between kernels",
            "kernels_ms": {k: round(v, 5) for k, v in bd.items()},
        },
        "e2e": {"value": round(e2e_value, 3), "unit": wl.unit, "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": wl.d2h_bytes, "api": wl.e2e_api},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if wl.bound == "hbm":
        out["roofline"]["kernels_gbs"] = {k: round(wl.kernel_work[k] / (v / 1e3) / 1e9, 1) for k, v in bd.items() if wl.kernel_work.get(k)}
    else:
        out["roofline"]["kernels_tflops"] = {k: round(wl.kernel_work[k] / (v / 1e3) / 1e12, 1) for k, v in bd.items() if wl.kernel_work.get(k)}
    if cpu_baseline:
        cb = W.cpu_baseline()
        out["cpu_baseline"] = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in cb.items()}
    if getattr(wl, "exchange", None) is not None:
        wl.exchange.finish()
    del wl
    return out


def run_reference(args, ws, rank):
    if rank != 0:
        return
    W = WORKLOADS[args.workload]
    heavy = args.workload in ("gpt", "attn", "attn_small", "prefill", "decode")
    for _ in range(1 if heavy else min(args.warmup, 3)):
        W.cpu_baseline()
    runs = [W.cpu_baseline() for _ in range(min(args.steps, 3) if heavy else args.steps)]
    v = statistics.median(r["value"] for r in runs)
    base = runs[0]
    per_step_s = statistics.median(r["seconds_per_sample"] for r in runs) / (base.get("sample_fraction") or 1.0)
    out = {
        "metric": W.metric,
        "value": round(v, 4),
        "unit": W.unit,
        "n_gpus": ws,
        "steps": len(runs),
        "warmup": args.warmup,
        "ms_per_step": round(per_step_s * 1e3, 3),
        "higher_is_better": True,
        "scaling": W.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "impl": "reference",
        "config": W.static_config(ws) if hasattr(W, "static_config") else {"workload": W.name},
        "cpu_baseline": {"value": round(v, 4), "unit": W.unit, "cores": base["cores"], "kind": base["kind"], "sample": base["sample"]},
        "e2e": {"value": round(v, 4), "unit": W.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "JAX (the reference's runtime) is not installable here; the reference's CPU path is timed as its restatement in oracle/",
    }
    print(json.dumps(out), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true", help="default workload only (no sub-lines for the other configs)")
    ap.add_argument("--shape", default=None, help="smaller case for profiling captures: norm rows,dim | attn b,h,s,d | gemm m,n,k | gpt global_batch | decode layers,b,h,max_len,d")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)  # timing rule: at least 3 untimed warm-up steps
    ws, rank, local = _dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
