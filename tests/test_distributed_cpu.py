"""Multi-rank host logic on CPU with ``gloo`` (world size 2): the data-parallel
gradient all-reduce of the training step, the token-sharded RMSNorm backward's dw
exchange (the only collective of the sharded bench), and failure detection when a
rank leaves (a short process-group timeout turns the missing rank into an error
on the survivor)."""

import os
import socket
import sys
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, ws, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path[:0] = [ROOT, os.path.join(ROOT, "ferrite-tpu_b200")]
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=timeout_s))


def _dp_worker(rank, ws, port, out):
    _init(rank, ws, port)
    from ferrite.model.train import FlatGrads

    torch.manual_seed(0)
    params = [torch.zeros(3, 4, requires_grad=True), torch.zeros(5, requires_grad=True)]
    flat = FlatGrads(params)
    flat.zero()
    loss = (params[0] * (rank + 1)).sum() + (params[1] * (2.0 * rank)).sum()
    loss.backward()
    flat.all_reduce_mean()
    torch.save([p.grad.clone() for p in params], os.path.join(out, f"g{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _bucket_worker(rank, ws, port, out):
    """Bucketed gradient exchange launched from post-accumulate hooks during
    backward (tiny buckets so every layer is its own bucket; a 'late' tied
    parameter used twice, reduced after backward)."""
    _init(rank, ws, port)
    from ferrite.model.train import FlatGrads

    torch.manual_seed(0)
    emb = torch.randn(6, 4, requires_grad=True)  # used twice (input and tied output)
    layers = [torch.randn(4, 4, requires_grad=True) for _ in range(3)]
    gain = torch.ones(4, requires_grad=True)
    params = [emb] + layers + [gain]
    flat = FlatGrads(params, overlap=True, bucket_mb=1e-5, late=(emb,))
    assert flat.overlap and len(flat.buckets) >= 4
    for step in range(2):  # buckets reset between steps
        flat.zero()
        x = emb[torch.tensor([1, 3, 5])] * (rank + 1)
        for w in layers:
            x = torch.tanh(x @ w)
        loss = ((x * gain) @ emb.t()).sum() * (step + 1)
        loss.backward()
        flat.finish()
    torch.save([p.grad.clone() for p in params], os.path.join(out, f"g{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _norm_worker(rank, ws, port, out):
    """The token-sharded RMSNorm backward as the benchmark runs it: each rank takes
    its row range (ferrite.sharding.norm_rows), writes its dw partial into the
    exchange's buffer for the step and starts the overlapped all-reduce
    (ferrite.sharding.DwExchange, two alternating buffers); four steps with
    different upstream gradients, results read after later steps were started."""
    _init(rank, ws, port)
    from ferrite.sharding import DwExchange, norm_rows
    from oracle import rmsnorm as on

    rng = np.random.default_rng(7)
    rows, dim = 66, 48  # 33 rows a rank
    h = rng.standard_normal((rows, dim)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    dys = [rng.standard_normal((rows, dim)).astype(np.float32) for _ in range(4)]
    r0, r1 = norm_rows(rows, ws, rank)
    ex = DwExchange(dim, "cpu")
    dws = {}
    for step, dy in enumerate(dys):
        dh, dw = on.rmsnorm_bwd(h[r0:r1], w, dy[r0:r1])
        ex.buffer(step).copy_(torch.from_numpy(dw))  # waits for step - 2's all-reduce first
        ex.start(step)
        if step >= 1:  # read the previous step's sum while this one is in flight
            dws[step - 1] = ex.result(step - 1).clone()
        np.save(os.path.join(out, f"dh{rank}_{step}.npy"), dh)
    dws[3] = ex.result(3).clone()
    ex.finish()
    for step, t in dws.items():
        np.save(os.path.join(out, f"dw{rank}_{step}.npy"), t.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _leaver_worker(rank, ws, port, out):
    _init(rank, ws, port, timeout_s=3)
    if rank == 1:
        return  # leaves between steps, never joins the next collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        status = "no-error"
    except Exception as e:  # noqa: BLE001
        status = "error:" + type(e).__name__
    with open(os.path.join(out, "status.txt"), "w") as f:
        f.write(status)


def _run(fn, ws=2):
    out = tempfile.mkdtemp()
    mp.start_processes(fn, args=(ws, _free_port(), out), nprocs=ws, join=True, start_method="spawn")
    return out


def test_dp_gradient_all_reduce_is_the_mean():
    out = _run(_dp_worker)
    g0 = torch.load(os.path.join(out, "g0.pt"))
    g1 = torch.load(os.path.join(out, "g1.pt"))
    for a, b in zip(g0, g1):
        assert torch.equal(a, b)
    assert torch.allclose(g0[0], torch.full((3, 4), 1.5)) and torch.allclose(g0[1], torch.full((5,), 1.0))


def test_token_sharded_rmsnorm_backward_exchange():
    out = _run(_norm_worker)
    sys.path.insert(0, ROOT)
    from oracle import rmsnorm as on

    rng = np.random.default_rng(7)
    h = rng.standard_normal((66, 48)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(48)).astype(np.float32)
    dys = [rng.standard_normal((66, 48)).astype(np.float32) for _ in range(4)]
    for step, dy in enumerate(dys):
        dh_full, dw_full = on.rmsnorm_bwd(h, w, dy)
        for r in range(2):
            np.testing.assert_allclose(np.load(os.path.join(out, f"dw{r}_{step}.npy")), dw_full, rtol=1e-5, atol=1e-5)
        dh = np.concatenate([np.load(os.path.join(out, f"dh{r}_{step}.npy")) for r in range(2)])
        np.testing.assert_array_equal(dh, dh_full)  # row-local: sharding changes nothing


def test_shard_ranges_cover_every_unit_once():
    sys.path[:0] = [os.path.join(ROOT, "ferrite-tpu_b200")]
    from ferrite.sharding import attention_slices, norm_rows, shard_range

    for n in (0, 1, 7, 256, 8192):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [e - b for b, e in ranges]
            assert max(sizes) - min(sizes) <= 1
    assert attention_slices(8, 32, 8, 3) == (96, 128)  # the long config at 8 GPUs: 32 slices a rank
    assert norm_rows(8192, 4, 1) == (2048, 4096)
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


@pytest.mark.timeout(120)
def test_missing_rank_surfaces_as_an_error():
    out = _run(_leaver_worker)
    status = open(os.path.join(out, "status.txt")).read()
    assert status.startswith("error:"), status


def test_bucketed_overlapped_gradient_sum_matches_full_all_reduce():
    out = _run(_bucket_worker)
    g = [torch.load(os.path.join(out, f"g{r}.pt")) for r in range(2)]
    # reference: the same step computed for both ranks in one process, summed
    torch.manual_seed(0)
    emb = torch.randn(6, 4, requires_grad=True)
    layers = [torch.randn(4, 4, requires_grad=True) for _ in range(3)]
    gain = torch.ones(4, requires_grad=True)
    params = [emb] + layers + [gain]
    for rank in range(2):
        x = emb[torch.tensor([1, 3, 5])] * (rank + 1)
        for w in layers:
            x = torch.tanh(x @ w)
        (((x * gain) @ emb.t()).sum() * 2).backward()
    for a, b, p in zip(g[0], g[1], params):
        assert torch.equal(a, b)
        torch.testing.assert_close(a, p.grad, rtol=1e-5, atol=1e-6)
