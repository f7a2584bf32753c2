"""bench.py's chunk preparation and row shards, on the CPU (no GPU needed).

The driver runs `bench.py --steps 20 --warmup 5` at 1, 2, 4 and 8 GPUs, so
every rank must pack 25 chunks that the budget closed (none of them a
stream's partial last chunk) from its own token-balanced row slice.
"""

import numpy as np
import pytest
import torch

import bench
from quail_b200.arena import KVArena
from quail_b200.model import QWEN3_4B
from quail_b200.workload import config1, shard, token_shard

BUDGET = QWEN3_4B.max_chunk_tokens


def _pack(wl, world, rank, n_chunks):
    lo, hi = token_shard(wl.row_tokens(), rank, world)
    arena = KVArena(QWEN3_4B.n_layers, 16384, 16, 8, 128, device=None)
    chunks, n_rows = bench.prepack(torch, arena, wl, lo, hi, BUDGET, n_chunks, "cpu")
    return chunks, n_rows, (lo, hi)


@pytest.mark.parametrize("world,rank", [(1, 0), (8, 0), (8, 7)])
def test_prepack_driver_steps(world, rank):
    """warmup 5 + steps 20 = 25 chunks, each filled to within one row of
    the budget, from the rank's own rows."""
    wl = config1()
    chunks, n_rows, (lo, hi) = _pack(wl, world, rank, 25)
    assert len(chunks) == 25
    assert n_rows <= hi - lo
    longest = int(wl.fresh_row_tokens(lo, hi).max())
    for c in chunks:
        assert BUDGET - longest <= c.tokens <= BUDGET


def test_prepack_too_few_rows_raises():
    """A slice that cannot fill the asked chunk count is an error, not a
    short timed region."""
    wl = config1(rows=300)
    arena = KVArena(QWEN3_4B.n_layers, 16384, 16, 8, 128, device=None)
    with pytest.raises(RuntimeError, match="pack only"):
        bench.prepack(torch, arena, wl, 0, 300, BUDGET, 25, "cpu")


def test_rows_needed_counts_fresh_tokens():
    """The estimate counts suffix + tail per row (the 64 prefix tokens are
    borrowed), so it asks for at least as many rows as the budget needs."""
    wl = config1()
    n = bench.rows_needed(wl, 0, wl.rows, 25, BUDGET)
    fresh = wl.fresh_row_tokens(0, n).sum()
    assert fresh >= 25 * BUDGET
    assert n < 1.2 * 25 * BUDGET / wl.fresh_row_tokens(0, 20000).mean()


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_token_shard_partition(world):
    """Token-balanced slices tile the rows in order, and every rank's
    tokens are within one row of the even share."""
    wl = config1()
    tok = wl.row_tokens()
    bounds = [token_shard(tok, r, world) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == len(tok)
    for (a, b), (c, _) in zip(bounds, bounds[1:]):
        assert b == c and a <= b
    even = tok.sum() / world
    for a, b in bounds:
        assert abs(tok[a:b].sum() - even) <= tok.max()


def test_token_shard_edges():
    assert token_shard([], 0, 2) == (0, 0)
    assert token_shard([5], 0, 1) == (0, 1)
    assert [token_shard([5], r, 3) for r in range(3)] in (
        [(0, 0), (0, 1), (1, 1)], [(0, 1), (1, 1), (1, 1)], [(0, 0), (0, 0), (0, 1)])
    # equal lengths: the same cuts as equal row counts
    tok = np.full(100, 7)
    for r in range(4):
        assert token_shard(tok, r, 4) == shard(100, r, 4)
