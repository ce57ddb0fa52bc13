"""Model check of the stage-ring protocol of dw_stream_kernel (CPU).

A Python model of the kernel's producer warp and consumer warps -- the same
stage order, slot/parity bookkeeping and mbarrier semantics (a phase with
parity P is complete when the barrier's phase count has the other parity) --
run under random interleavings over many plan geometries: tile heights, row
blockings, row splits, ring depths down to the minimum (tile_h stages),
multi-tile persistent walks and image heights smaller than the kernel.  Every
run must finish (no deadlock) and every consumer must find, at every step,
its input rows and its weight row in the slots it reads.
"""
from __future__ import annotations

import random

import pytest


class Bar:
    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):
        return (self.phase & 1) != parity


def _tiles(H, K, tile_h, ntiles):
    """(s_lo, nsteps, nrows) of the tiles a persistent CTA walks (decode_tile's row bounds)."""
    pad, out = K // 2, []
    for t in range(ntiles):
        th = t % ((H + tile_h - 1) // tile_h)
        h0 = th * tile_h
        rows_in = min(tile_h, H - h0)
        s_lo = max(0, pad - (h0 + rows_in - 1))
        s_hi = min(K, H + pad - h0)
        out.append((s_lo, s_hi - s_lo, s_hi - s_lo + tile_h - 1))
    return out


def _run(H, K, tile_h, M, NS, nsplit, ntiles, seed):
    rnd = random.Random(seed)
    tiles = _tiles(H, K, tile_h, ntiles)
    slots = tile_h // M
    CW = nsplit * slots
    full = [Bar(1) for _ in range(NS)]
    empty = [Bar(CW) for _ in range(NS)]
    content = [None] * NS

    def producer():
        slot, phase, fills = 0, 0, 0
        for ti, (_, _, nrows) in enumerate(tiles):
            for q in range(nrows):
                if fills >= NS:
                    while not empty[slot].done(phase ^ 1):
                        yield
                content[slot] = (ti, q)  # input row q; weight row q - (tile_h - 1) when q >= tile_h - 1
                full[slot].arrive()
                slot += 1
                if slot == NS:
                    slot, phase = 0, phase ^ 1
                fills += 1
                yield

    def consumer(w):
        trow0 = (w % slots) * M
        ws, wp, rs = 0, 0, 0
        for ti, (_, nsteps, nrows) in enumerate(tiles):
            my = (rs + trow0) % NS
            for _ in range(tile_h - 1):
                while not full[ws].done(wp):
                    yield
                ws += 1
                if ws == NS:
                    ws, wp = 0, wp ^ 1
            for st in range(nsteps):
                while not full[ws].done(wp):
                    yield
                assert content[ws] == (ti, st + tile_h - 1)  # this step's weight row
                ws += 1
                if ws == NS:
                    ws, wp = 0, wp ^ 1
                for m in range(M):
                    assert content[(my + m) % NS] == (ti, st + trow0 + m)  # this step's input rows
                yield
                empty[rs].arrive()
                rs = (rs + 1) % NS
                my = (my + 1) % NS
            for _ in range(nsteps, nrows):
                empty[rs].arrive()
                rs = (rs + 1) % NS

    agents = [producer()] + [consumer(w) for w in range(CW)]
    alive, steps = list(range(len(agents))), 0
    while alive:
        i = rnd.choice(alive)
        try:
            next(agents[i])
        except StopIteration:
            alive.remove(i)
        steps += 1
        assert steps < 2_000_000, "deadlock"


@pytest.mark.parametrize("seed", range(0, 300, 3))
def test_stage_ring_never_deadlocks_and_serves_the_right_rows(seed):
    r = random.Random(seed)
    K = r.choice([1, 3, 7, 9, 13, 27, 31])
    M = r.choice([1, 2])
    tile_h = M * r.choice([1, 2, 3])
    H = r.choice([1, 2, 5, 7, 14, 32])
    nsplit = r.choice([1, 2, 3, 4])
    NS = r.randint(tile_h, tile_h + K + 2)  # the launcher accepts any depth >= tile_h
    _run(H, K, tile_h, M, NS, nsplit, r.randint(1, 6), seed)
