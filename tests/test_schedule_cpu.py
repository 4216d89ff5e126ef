"""Work-unit order of the persistent dQ-from-dS kernel (attn_dq_ds_kernel in
csrc/attention.cu): CTA c of G takes, in round r, unit r * G + c for even r and
r * G + (G - 1 - c) for odd r, until the unit index passes the end.  Every unit
must be taken exactly once, and the order must even out heavy and light query
tiles across CTAs (the plain stride c, c + G, ... did not)."""

import numpy as np


def units_of(c, G, units):
    out, r = [], 0
    while True:
        u = r * G + ((G - 1 - c) if (r & 1) else c)
        if u >= units:
            return out
        out.append(u)
        r += 1


def test_every_unit_taken_once():
    rng = np.random.default_rng(0)
    cases = [(148, 2048), (148, 16384), (148, 100), (1, 7), (5, 5), (7, 50), (148, 148), (148, 149), (148, 295), (148, 296)]
    cases += [(int(g), int(u)) for g, u in zip(rng.integers(1, 200, 40), rng.integers(1, 5000, 40))]
    for G, units in cases:
        G = min(G, units)  # the host launches min(units, SMs) CTAs
        seen = []
        for c in range(G):
            seen += units_of(c, G, units)
        assert sorted(seen) == list(range(units)), (G, units)


def test_boustrophedon_balances_causal_tiles():
    # unit u -> query tile n_q - 1 - u % n_q; its dS work is proportional to the tile index + 1
    for n_q, slices in ((8, 256), (8, 1024), (64, 256)):
        G, units = 148, n_q * slices
        cost = lambda u: n_q - u % n_q  # (n_q - 1 - u % n_q) + 1
        snake = [sum(cost(u) for u in units_of(c, G, units)) for c in range(G)]
        stride = [sum(cost(u) for u in range(c, units, G)) for c in range(G)]
        assert max(snake) / np.mean(snake) < 1.03
        assert max(snake) / np.mean(snake) <= max(stride) / np.mean(stride)


def batched_order(lin, ntiles, nslices, batch=8):
    """CPU restatement of batched_order() in csrc/attention.cu for grids of at least
    16 tiles a slice: linear CTA index -> (tile, slice), tile slowest inside a batch
    of `batch` slices."""
    per_batch = batch * ntiles
    b = lin // per_batch
    s0 = b * batch
    nb = min(batch, nslices - s0)
    idx = lin - b * per_batch
    return idx // nb, s0 + idx % nb


def test_batched_order_is_a_bijection_heaviest_first():
    for ntiles, nslices in ((16, 1), (16, 7), (32, 256), (64, 32), (64, 33), (17, 9)):
        pairs = [batched_order(lin, ntiles, nslices) for lin in range(ntiles * nslices)]
        assert sorted(pairs) == [(t, s) for t in range(ntiles) for s in range(nslices)]
        # inside each batch the tile index never decreases: heavy (low index) tiles first
        for b0 in range(0, nslices, 8):
            nb = min(8, nslices - b0)
            lo = b0 * ntiles
            tiles = [pairs[lin][0] for lin in range(lo, lo + nb * ntiles)]
            assert tiles == sorted(tiles)
