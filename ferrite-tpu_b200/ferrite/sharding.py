"""How the hot path shards over the GPUs of one box, and its one exchange.

The reference runs its sharded configs under ``jax.shard_map`` with
``P('data')`` specs (model/train.py:80-99 for the data-parallel step; the
benchmarks shard attention over batch x heads and the norm over tokens): every
device sees only its shard and XLA inserts no gathers.  Here one process drives
one GPU and these helpers say which shard it owns:

* attention: the ``b * h`` (batch, head) slices are independent, so rank r takes
  a contiguous range of them -- no communication;
* fused add + RMSNorm: rows (tokens) are independent in the forward and in dh,
  so rank r takes a contiguous row range; the backward's weight gradient
  ``dw = sum_rows dy * xhat`` is the one exchange: each rank's partial sum
  (f32 ``[dim]``) is summed over ranks.

:class:`DwExchange` is that exchange as the benchmark and a training step run it:
an asynchronous all-reduce per step that overlaps the next step's kernels, with
two buffers that alternate so a buffer is rewritten only after its previous
all-reduce has finished.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous ``[begin, end)`` of ``n`` units owned by ``rank`` of ``world``
    (units split as evenly as possible, the first ``n % world`` ranks one more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def attention_slices(b: int, h: int, world: int, rank: int) -> tuple[int, int]:
    """The (batch, head) slice range ``[begin, end)`` of the flattened ``b * h`` this rank computes."""
    return shard_range(b * h, world, rank)


def norm_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """The token (row) range ``[begin, end)`` of the norm's input this rank normalises."""
    return shard_range(rows, world, rank)


def one_cta_nccl_group():
    """A NCCL communicator limited to one CTA, for a small all-reduce that must
    overlap kernels on the same GPU: a default-width NCCL kernel spinning on late
    peers holds SMs that the CTAs of a persistent kernel wait for (measured at 4
    GPUs on the norm step: 3.6x one GPU with one CTA, 2.3-2.9x with NCCL's
    default).  Returns None (the default group) when the options are unavailable."""
    try:
        opts = dist.ProcessGroupNCCL.Options()
        opts.config.min_ctas = 1
        opts.config.max_ctas = 1
        return dist.new_group(backend="nccl", pg_options=opts)
    except (AttributeError, RuntimeError, TypeError):
        return None


class DwExchange:
    """Sum of the per-rank dw partials of a token-sharded RMSNorm backward.

    Step i writes its partial into ``buffer(i)`` (a GPU stream write, or any
    writer) and calls ``start(i)``: the all-reduce (sum) runs asynchronously --
    on NCCL's stream for GPU buffers -- while the next steps proceed.  Buffers
    alternate over ``slots`` (default 2): ``buffer(i)`` first makes the caller wait
    (the current CUDA stream for NCCL, the host for gloo) for the all-reduce of
    step ``i - slots``, which used the same buffer, so no partial is overwritten
    while it is being reduced.  ``result(i)`` waits for step i's sum and returns
    it.  Every rank calls start() for the same steps in the same order, as a
    collective requires.
    """

    def __init__(self, dim: int, device: torch.device | str, *, group=None, slots: int = 2, dtype=torch.float32):
        if slots < 1:
            raise ValueError("slots must be >= 1")
        self.bufs = [torch.zeros(dim, dtype=dtype, device=device) for _ in range(slots)]
        self.pending = [None] * slots
        self.group = group
        self.slots = slots

    def _slot(self, step: int) -> int:
        return step % self.slots

    def buffer(self, step: int) -> torch.Tensor:
        """The buffer step ``step`` writes its partial into, once it is free."""
        s = self._slot(step)
        if self.pending[s] is not None:
            self.pending[s].wait()
            self.pending[s] = None
        return self.bufs[s]

    def start(self, step: int) -> None:
        """Begin summing step ``step``'s partial over the ranks (asynchronous)."""
        s = self._slot(step)
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            self.pending[s] = dist.all_reduce(self.bufs[s], group=self.group, async_op=True)

    def result(self, step: int) -> torch.Tensor:
        """Step ``step``'s summed dw (valid until step ``step + slots`` reuses the buffer)."""
        s = self._slot(step)
        if self.pending[s] is not None:
            self.pending[s].wait()
            self.pending[s] = None
        return self.bufs[s]

    def finish(self) -> None:
        """Wait for every all-reduce in flight."""
        for s in range(self.slots):
            if self.pending[s] is not None:
                self.pending[s].wait()
                self.pending[s] = None
