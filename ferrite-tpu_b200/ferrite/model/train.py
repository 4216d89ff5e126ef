"""Data-parallel training of the GPT with the reference's hand-written AdamW.

Restates src/ferrite/model/train.py: ``TrainConfig`` (:29-41), ``adamw_init``
(:47-49), ``lr_at`` (:52-56, linear warm-up then cosine to 10%), ``adamw_update``
(:59-74: global-norm clip, bias-corrected Adam, decoupled weight decay on 2-D
parameters only), ``train`` (:102-177: results dict with tokens/s, MFU, loss
curve) and ``load_params`` (:188-198).

B200 layout: one process per GPU (``torchrun``); parameters are replicated (same
seed on every rank), the global batch is split over ranks like the reference's
``NamedSharding(P('data'))``, and the gradients -- accumulated by autograd into
one flat f32 buffer -- are averaged with a single NCCL all-reduce per step (the
collective XLA inserts for the reference).  Attention, norms and (with
``linear="pallas"``) every matmul run on the B200 kernels.
"""

from __future__ import annotations

import dataclasses
import json
import math
import os
import time
from typing import Any

import numpy as np
import torch

from ferrite import platform
from ferrite.model import data as data_lib
from ferrite.model.gpt import GPTConfig, flops_per_token, init_params, loss_fn, param_count, param_leaves


@dataclasses.dataclass(frozen=True)
class TrainConfig:
    steps: int = 200
    batch: int = 64
    lr: float = 6e-4
    warmup: int = 20
    weight_decay: float = 0.1
    clip: float = 1.0
    seed: int = 0
    log_every: int = 10
    data: str = "synthetic"  # "synthetic" (Markov bytes) | "uniform" (ids uniform in [0, vocab))
    out: str | None = None
    save_params: str | None = None


# ---------------------------------------------------------------- optimiser


def lr_at(step: int, cfg: TrainConfig) -> float:
    warm = cfg.lr * (step + 1) / max(1, cfg.warmup)
    progress = min(max((step - cfg.warmup) / max(1, cfg.steps - cfg.warmup), 0.0), 1.0)
    cosine = 0.1 * cfg.lr + 0.9 * cfg.lr * 0.5 * (1 + math.cos(math.pi * progress))
    return warm if step < cfg.warmup else cosine


class AdamW:
    """adamw_update (train.py:59-74) over a list of f32 parameter tensors."""

    def __init__(self, params: list[torch.Tensor], cfg: TrainConfig, b1=0.9, b2=0.95, eps=1e-8):
        self.params = params
        self.m = [torch.zeros_like(p) for p in params]
        self.v = [torch.zeros_like(p) for p in params]
        self.step = 0
        self.cfg, self.b1, self.b2, self.eps = cfg, b1, b2, eps
        self.decay = [cfg.weight_decay if p.ndim >= 2 else 0.0 for p in params]

    @torch.no_grad()
    def update(self, grads: list[torch.Tensor]) -> torch.Tensor:
        self.step += 1
        step, cfg, b1, b2 = self.step, self.cfg, self.b1, self.b2
        lr = lr_at(step, cfg)
        gnorm = torch.linalg.vector_norm(torch.stack([torch.linalg.vector_norm(g.float()) for g in grads]))
        scale = torch.clamp(cfg.clip / (gnorm + 1e-6), max=1.0)
        g = torch._foreach_mul(grads, scale)
        torch._foreach_mul_(self.m, b1)
        torch._foreach_add_(self.m, g, alpha=1 - b1)
        torch._foreach_mul_(self.v, b2)
        torch._foreach_addcmul_(self.v, g, g, value=1 - b2)
        bc1, bc2 = 1 - b1**step, 1 - b2**step
        denom = torch._foreach_div(self.v, bc2)
        torch._foreach_sqrt_(denom)
        torch._foreach_add_(denom, self.eps)
        upd = torch._foreach_div(self.m, bc1)
        torch._foreach_div_(upd, denom)
        for p, u, dcy in zip(self.params, upd, self.decay):
            if dcy:
                u.add_(p, alpha=dcy)
            p.sub_(u, alpha=lr)
        return gnorm


# ---------------------------------------------------------------- distributed helpers


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class FlatGrads:
    """Points every parameter's ``.grad`` at a view of one flat f32 buffer, so the
    data-parallel gradient exchange is one buffer's worth of all-reduce.

    With ``overlap=True`` (and a process group of more than one rank) the buffer
    is cut into buckets of about ``bucket_mb`` MiB taken from its end -- the last
    layers' gradients, which backward produces first -- and each bucket's
    all-reduce (a sum) is launched on NCCL's stream from a post-accumulate hook as
    soon as all of its gradients are final, so the exchange overlaps the rest of
    the backward.  ``late`` parameters (e.g. a tied embedding, accumulated twice)
    go in a final bucket reduced after backward.  :meth:`finish` waits for all
    buckets; the caller divides by the world size (the fused AdamW does it in its
    gradient pre-scale)."""

    def __init__(self, params: list[torch.Tensor], *, overlap: bool = False, bucket_mb: float = 64.0, late=(), group=None):
        n = sum(p.numel() for p in params)
        self.flat = torch.zeros(n, dtype=torch.float32, device=params[0].device)
        self.views = []
        self.offsets = []
        off = 0
        for p in params:
            v = self.flat[off : off + p.numel()].view_as(p)
            p.grad = v
            self.views.append(v)
            self.offsets.append(off)
            off += p.numel()
        self.params = params
        self.group = group
        self.works = []
        self.buckets = []
        self.overlap = overlap and self._world() > 1
        if self.overlap:
            self._build_buckets(bucket_mb, {id(p) for p in late})

    @staticmethod
    def _dist():
        import torch.distributed as dist

        return dist

    def _world(self) -> int:
        dist = self._dist()
        return dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1

    def _build_buckets(self, bucket_mb, late_ids):
        limit = int(bucket_mb * (1 << 20) / 4)
        order = [i for i in range(len(self.params)) if id(self.params[i]) not in late_ids][::-1]
        cur, cur_n = [], 0
        runs = []
        for i in order:  # contiguous runs of the flat buffer, from its end
            if cur and (cur_n >= limit or self.offsets[i] + self.params[i].numel() != self.offsets[cur[-1]]):
                runs.append(cur)
                cur, cur_n = [], 0
            cur.append(i)
            cur_n += self.params[i].numel()
        if cur:
            runs.append(cur)
        for idx in runs:
            lo = self.offsets[idx[-1]]
            hi = self.offsets[idx[0]] + self.params[idx[0]].numel()
            self.buckets.append({"lo": lo, "hi": hi, "members": set(idx), "expected": len(idx)})
        for i in range(len(self.params)):
            if id(self.params[i]) in late_ids:  # reduced after backward, not by a hook
                self.buckets.append({"lo": self.offsets[i], "hi": self.offsets[i] + self.params[i].numel(), "members": {i}, "expected": None})
        self.bucket_of = {i: b for b in self.buckets for i in b["members"]}
        self._reset_buckets()
        for i, p in enumerate(self.params):
            if id(p) not in late_ids:
                p.register_post_accumulate_grad_hook(self._hook(i))

    def _reset_buckets(self):
        for b in self.buckets:
            b["left"] = b["expected"]
            b["launched"] = False

    def _hook(self, i):
        def fire(_p):
            b = self.bucket_of[i]
            if b["expected"] is None or b["launched"]:
                return
            b["left"] -= 1
            if b["left"] == 0:
                self._launch(b)

        return fire

    def _launch(self, b):
        b["launched"] = True
        self.works.append(self._dist().all_reduce(self.flat[b["lo"] : b["hi"]], group=self.group, async_op=True))

    def zero(self):
        self.flat.zero_()
        for p, v in zip(self.params, self.views):
            p.grad = v
        self._reset_buckets()

    def finish(self):
        """Overlap mode: launch the buckets still pending, then make the current
        stream wait for every bucket's all-reduce (sums; divide by the world size)."""
        for b in self.buckets:
            if not b["launched"]:
                self._launch(b)
        for w in self.works:
            w.wait()
        self.works = []

    def all_reduce_mean(self, group=None):
        dist = self._dist()
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, group=group)
            self.flat.div_(dist.get_world_size(group))


class FusedAdamW:
    """adamw_update (train.py:59-74) as one native pass over flat f32 buffers
    (``ferrite_adamw_step``: grad-norm clipping, bias-corrected Adam, decoupled
    weight decay on ndim >= 2 parameters).

    The parameters are moved into one flat buffer, decayed (ndim >= 2) ones first;
    ``self.grads`` is a :class:`FlatGrads` with the same layout, and the moments
    are flat.  ``grad_scale`` multiplies the gradients first (1 / world size after
    a summed all-reduce)."""

    def __init__(self, params: list[torch.Tensor], cfg: TrainConfig, b1=0.9, b2=0.95, eps=1e-8, *, overlap=False, late=(), bucket_mb=64.0):
        from ferrite import _native as nat

        self.nat, self.lib = nat, nat.lib()
        decayed = [p for p in params if p.ndim >= 2]
        self.order = decayed + [p for p in params if p.ndim < 2]
        self.n_decay = sum(p.numel() for p in decayed)
        self.n = sum(p.numel() for p in self.order)
        dev = params[0].device
        nat.require_cuda(params[0])
        self.flat = torch.empty(self.n, dtype=torch.float32, device=dev)
        off = 0
        with torch.no_grad():
            for p in self.order:
                k = p.numel()
                self.flat[off : off + k].copy_(p.reshape(-1))
                p.data = self.flat[off : off + k].view_as(p)
                off += k
        self.grads = FlatGrads(self.order, overlap=overlap, late=late, bucket_mb=bucket_mb)
        self.m = torch.zeros_like(self.flat)
        self.v = torch.zeros_like(self.flat)
        self.ws = torch.empty(int(self.lib.ferrite_adamw_workspace_size(self.n)), dtype=torch.uint8, device=dev)
        self.gnorm = torch.zeros((), dtype=torch.float32, device=dev)
        self.step = 0
        self.cfg, self.b1, self.b2, self.eps = cfg, b1, b2, eps
        self.params = self.order

    @torch.no_grad()
    def update(self, grads=None, grad_scale: float = 1.0) -> torch.Tensor:
        self.step += 1
        cfg, nat = self.cfg, self.nat
        with torch.cuda.device(self.flat.device):
            nat.check(
                self.lib.ferrite_adamw_step(
                    nat.stream_ptr(self.flat.device), self.flat.data_ptr(), self.grads.flat.data_ptr(), self.m.data_ptr(),
                    self.v.data_ptr(), self.n, self.n_decay, lr_at(self.step, cfg), self.b1, self.b2, self.eps,
                    cfg.weight_decay, self.step, cfg.clip, grad_scale, self.gnorm.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                )
            )
        return self.gnorm.clone()


def make_optimizer(params: list[torch.Tensor], cfg: TrainConfig, *, fused: bool | None = None, late=()):
    """(optimizer, FlatGrads): the native fused AdamW over flat buffers on CUDA
    (with bucketed, backward-overlapped gradient all-reduce at more than one rank),
    else the per-tensor reference AdamW."""
    if fused is None:
        fused = params[0].is_cuda
    if fused:
        opt = FusedAdamW(params, cfg, overlap=True, late=late)
        return opt, opt.grads
    return AdamW(params, cfg), FlatGrads(params)


def build_train_step(model_cfg: GPTConfig, train_cfg: TrainConfig, params_list, opt, flat: FlatGrads, params):
    """One DP step: forward + backward on the local shard, gradient all-reduce, AdamW."""

    def step(x, y):
        flat.zero()
        loss = loss_fn(params, x, y, model_cfg)
        loss.backward()
        if isinstance(opt, FusedAdamW):
            world = flat._world()
            if flat.overlap:
                flat.finish()  # bucket sums, launched during backward
            elif world > 1:
                flat._dist().all_reduce(flat.flat, group=flat.group)
            gnorm = opt.update(grad_scale=1.0 / world)
        else:
            flat.all_reduce_mean()
            gnorm = opt.update(flat.views)
        return loss.detach(), gnorm

    return step


def train(model_cfg: GPTConfig, train_cfg: TrainConfig, *, verbose: bool = True) -> dict[str, Any]:
    ws, rank, local = dist_env()
    if train_cfg.batch % ws:
        raise ValueError(f"batch {train_cfg.batch} must be divisible by {ws} devices")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1 and not torch.distributed.is_initialized():
        from datetime import timedelta

        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    local_batch = train_cfg.batch // ws
    rng = np.random.default_rng(train_cfg.seed + 1000 * rank)
    corpus = data_lib.synthetic(200_000, seed=train_cfg.seed) if train_cfg.data == "synthetic" else None

    params = init_params(train_cfg.seed, model_cfg, device=device)
    leaves = param_leaves(params)
    for p in leaves:
        p.requires_grad_(True)
    n_params = param_count(params)
    n_nonembed = n_params - params["tok_emb"].numel() - params["pos_emb"].numel()
    opt, flat = make_optimizer(leaves, train_cfg, late=(params["tok_emb"], params["pos_emb"]))
    step_fn = build_train_step(model_cfg, train_cfg, leaves, opt, flat, params)

    def batch():
        if corpus is not None:
            x, y = data_lib.get_batch(rng, corpus, local_batch, model_cfg.seq_len)
        else:
            x, y = data_lib.uniform_batch(rng, local_batch, model_cfg.seq_len, model_cfg.vocab_size)
        return torch.from_numpy(x).to(device, non_blocking=True), torch.from_numpy(y).to(device, non_blocking=True)

    tokens_per_step = train_cfg.batch * model_cfg.seq_len
    fpt = flops_per_token(model_cfg, n_nonembed)
    train_flops_per_step = 3 * fpt["total"] * tokens_per_step
    peak = platform.peaks()
    peak_flops = peak.bf16_flops * ws

    losses, step_times, gnorms = [], [], []
    warm = min(5, train_cfg.steps // 4)
    for i in range(train_cfg.steps):
        x, y = batch()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        loss, gnorm = step_fn(x, y)
        t1.record()
        loss_v = float(loss.item())
        dt = t0.elapsed_time(t1) / 1e3
        losses.append(loss_v)
        gnorms.append(float(gnorm))
        if i >= warm:
            step_times.append(dt)
        if verbose and rank == 0 and (i % train_cfg.log_every == 0 or i == train_cfg.steps - 1):
            print(f"step {i:5d} loss {loss_v:.4f} gnorm {float(gnorm):.3f} step {dt * 1e3:.1f} ms")

    med = float(np.median(step_times)) if step_times else float("nan")
    result = {
        "platform": platform.describe(),
        "model": {**{k: (str(v) if k == "dtype" else v) for k, v in dataclasses.asdict(model_cfg).items()}, "params": n_params, "params_nonembed": n_nonembed},
        "train": dataclasses.asdict(train_cfg),
        "world_size": ws,
        "step_ms_median": med * 1e3,
        "step_ms_min": float(np.min(step_times)) * 1e3 if step_times else float("nan"),
        "tokens_per_second": tokens_per_step / med if step_times else float("nan"),
        "train_flops_per_step_analytic": train_flops_per_step,
        "achieved_tflops": train_flops_per_step / med / 1e12 if step_times else float("nan"),
        "mfu": (train_flops_per_step / med / peak_flops) if step_times else None,
        "loss_first": losses[0],
        "loss_last": float(np.mean(losses[-10:])),
        "loss_curve": losses[:: max(1, len(losses) // 50)],
    }
    if rank == 0 and train_cfg.out:
        os.makedirs(os.path.dirname(train_cfg.out) or ".", exist_ok=True)
        with open(train_cfg.out, "w") as f:
            json.dump(result, f, indent=2)
    if rank == 0 and train_cfg.save_params:
        os.makedirs(os.path.dirname(train_cfg.save_params) or ".", exist_ok=True)
        np.savez(train_cfg.save_params, **{k: v.detach().cpu().numpy() for k, v in _flatten(params)})
    return result


def _flatten(params):
    out = [("tok_emb", params["tok_emb"]), ("pos_emb", params["pos_emb"]), ("ln_f", params["ln_f"])]
    for i, layer in enumerate(params["layers"]):
        out += [(f"layers/{i}/{k}", v) for k, v in layer.items()]
    return out


def load_params(path: str, cfg: GPTConfig, device="cuda") -> dict:
    """Inverse of the ``save_params`` layout (train.py:188-198)."""
    raw = np.load(path)
    params = {"layers": [dict() for _ in range(cfg.n_layer)]}
    for k in raw.files:
        parts = k.split("/")
        t = torch.from_numpy(raw[k]).to(device)
        if parts[0] == "layers":
            params["layers"][int(parts[1])][parts[2]] = t
        else:
            params[parts[0]] = t
    return params


def main(argv=None):
    import argparse

    ap = argparse.ArgumentParser(description="Train the small transformer on the B200 kernels or plain torch.")
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seq", type=int, default=256)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--d-model", type=int, default=512)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--d-ff", type=int, default=2048)
    ap.add_argument("--vocab", type=int, default=256)
    ap.add_argument("--attention", choices=["pallas", "xla"], default="pallas")
    ap.add_argument("--norm", choices=["pallas", "xla"], default="pallas")
    ap.add_argument("--linear", choices=["pallas", "xla"], default="xla")
    ap.add_argument("--dtype", choices=["bfloat16", "float32"], default="bfloat16")
    ap.add_argument("--lr", type=float, default=6e-4)
    ap.add_argument("--data", choices=["synthetic", "uniform"], default="synthetic")
    ap.add_argument("--out", default=None)
    ap.add_argument("--save-params", default=None)
    a = ap.parse_args(argv)
    mcfg = GPTConfig(
        vocab_size=a.vocab, seq_len=a.seq, d_model=a.d_model, n_head=a.heads, n_layer=a.layers, d_ff=a.d_ff,
        attention=a.attention, norm=a.norm, linear=a.linear, dtype=getattr(torch, a.dtype),
    )
    tcfg = TrainConfig(steps=a.steps, batch=a.batch, lr=a.lr, data=a.data, out=a.out, save_params=a.save_params)
    res = train(mcfg, tcfg)
    if dist_env()[1] == 0:
        print(json.dumps({k: v for k, v in res.items() if k != "loss_curve"}, indent=2, default=str))


if __name__ == "__main__":
    main()
