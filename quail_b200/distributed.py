"""Data parallelism over rows: one process per GPU, contiguous row slices.

The reference runs one spawned child per GPU and merges pickled results on
the host (quail/backends/quail/worker.py:646-711, coordinator.py:45-83).
Here every rank is a torch.distributed process (NCCL over NVLink on GPUs,
gloo on CPU for the host-logic tests): rank r filters one contiguous slice
of the input rows (equal row counts, or balanced by tokens when the
caller gives per-row token counts) on its own model replica with its own
prefix tree, and the per-row results (bit, margin) are all-gathered so
every rank ends with the answers of all rows in input order. There is no
other cross-GPU traffic: rows are independent.

Failure handling (the reference re-raises a child's exception as
"GPU child failed", worker.py:382-384, 665-667): every rank reports
success or failure in one all-reduce before the result gather, so an
exception on any rank raises RankFailed on all of them instead of leaving
the others waiting; a rank that dies outright ends the others' next
collective with the process group's timeout error.
"""

import numpy as np

from quail_b200.workload import shard, token_shard


class RankFailed(RuntimeError):
    """Another rank (or this one) failed during the sharded filter."""


def gather_rows(torch, dist, values, device, dtype=np.float32):
    """All-gather a variable-length 1-D array from every rank, in rank order.

    dtype is the element type on the wire: float32 for margins and bits,
    int64 for row ids and lengths (float32 is exact only up to 2^24)."""
    world = dist.get_world_size()
    n = torch.tensor([len(values)], dtype=torch.int64, device=device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n)
    width = int(max(int(s) for s in sizes))
    host = np.asarray(values, dtype=dtype)
    buf = torch.zeros(max(width, 1), dtype=torch.from_numpy(host[:0]).dtype, device=device)
    buf[:len(host)] = torch.as_tensor(host, device=device)
    parts = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    return np.concatenate([p[:int(s)].cpu().numpy() for p, s in zip(parts, sizes)])


def run_sharded(torch, dist, n_rows, run_slice, device="cpu", row_tokens=None):
    """Run run_slice(lo, hi) -> (bits, margins) on this rank's rows; gather all.

    Slices are contiguous; with row_tokens (tokens per row) they are
    balanced by tokens (workload.token_shard), else by row count.
    Returns (bits uint8 [n_rows], margins float32 [n_rows]) in row order on
    every rank. Raises RankFailed on every rank when any rank raised.
    """
    rank, world = dist.get_rank(), dist.get_world_size()
    if row_tokens is not None:
        if len(row_tokens) != n_rows:
            raise ValueError("row_tokens must give one count per row")
        lo, hi = token_shard(row_tokens, rank, world)
    else:
        lo, hi = shard(n_rows, rank, world)
    error = None
    bits = margins = np.zeros(0, dtype=np.float32)
    try:
        bits, margins = run_slice(lo, hi)
    except Exception as exc:  # reported to every rank below
        error = exc
    ok = torch.tensor([0 if error is not None else 1], dtype=torch.int32, device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok) == 0:
        raise RankFailed(f"rank {rank}: a rank failed during the sharded filter") from error
    all_bits = gather_rows(torch, dist, np.asarray(bits, dtype=np.float32), device)
    all_margins = gather_rows(torch, dist, np.asarray(margins, dtype=np.float32), device)
    if len(all_bits) != n_rows:
        raise RankFailed(f"gathered {len(all_bits)} rows, expected {n_rows}")
    return all_bits.astype(np.uint8), all_margins


def run_sharded_join(torch, dist, n_anchors, n_stages, run_slice, device="cpu"):
    """A join sharded by anchor (config 2 shards by left row, coordinator.py:
    125-207): run_slice(lo, hi) runs this rank's anchors [lo, hi) and returns
    answers[stage][local anchor] -> row; every rank gets the rows of all
    anchors, keyed by global anchor index. Raises RankFailed on every rank
    when any rank raised."""
    rank, world = dist.get_rank(), dist.get_world_size()
    lo, hi = shard(n_anchors, rank, world)
    error = None
    answers = [dict() for _ in range(n_stages)]
    try:
        answers = run_slice(lo, hi)
    except Exception as exc:  # reported to every rank below
        error = exc
    ok = torch.tensor([0 if error is not None else 1], dtype=torch.int32, device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok) == 0:
        raise RankFailed(f"rank {rank}: a rank failed during the sharded join") from error
    out = []
    for j in range(n_stages):
        stage = answers[j] if j < len(answers) else {}
        local = sorted(stage)
        ids = np.asarray([lo + a for a in local], dtype=np.int64)
        lens = np.asarray([len(stage[a]) for a in local], dtype=np.int64)
        vals = (np.concatenate([np.asarray(stage[a], dtype=np.float32) for a in local])
                if local else np.zeros(0, dtype=np.float32))
        g_ids = gather_rows(torch, dist, ids, device, np.int64)
        g_lens = gather_rows(torch, dist, lens, device, np.int64)
        g_vals = gather_rows(torch, dist, vals, device)
        rows, at = {}, 0
        for a, n in zip(g_ids, g_lens):
            rows[int(a)] = g_vals[at:at + n]
            at += n
        out.append(rows)
    return out
