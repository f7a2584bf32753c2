"""Row sharding and result gathering across ranks, on CPU with gloo.

Two ranks run the real host loop (packer, arena, admission) over their
contiguous row slices with a deterministic CPU answer model, gather
(bit, margin) per row, and must reproduce the single-process answers in
row order. Failure injection happens on the host: a rank that raises makes
every rank raise RankFailed; a rank that exits makes the other's next
collective fail with the process group's timeout instead of hanging.
"""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from quail_b200 import loop
from quail_b200.arena import KVArena
from quail_b200.distributed import RankFailed, gather_rows, run_sharded, run_sharded_join
from quail_b200.pipeline import ModelPipeline
from quail_b200.tokens import prefix_tree
from quail_b200.workload import token_shard

N_ROWS = 37


def make_docs():
    rng = np.random.default_rng(9)
    prefix = rng.integers(100, 900, 64).tolist()
    return [prefix + rng.integers(100, 900, int(n)).tolist() for n in rng.integers(4, 80, N_ROWS)]


def cpu_filter(docs):
    """Single-stage filter on the CPU: bit = (last token + position) % 2,
    margin = a deterministic function of the answer row's position."""
    arena = KVArena(1, 256, 16, 1, 8, device=None)

    class Rec(ModelPipeline):
        def forward_chunk(self, chunk):
            return chunk.host

    class Ans:
        def submit(self, host):
            fin = host.final_indices
            return list(((host.input_ids[fin] + host.positions[fin]) % 2).astype(int))

        def result(self, h):
            return h

    answers, _, _ = loop.run_filter(torch, arena, Rec(), Ans(), docs, [[5]], 400,
                                    arena_writes=True, attention_mode="tree",
                                    prefix_tree=prefix_tree(docs, 16), device="cpu")
    bits = np.array([answers[i][-1] for i in range(len(docs))], dtype=np.float32)
    margins = np.array([len(d) * 0.01 - 0.3 for d in docs], dtype=np.float32)
    return bits, margins


def make_join():
    rng = np.random.default_rng(12)
    instr = rng.integers(100, 900, 32).tolist()
    anchors = [instr + rng.integers(100, 900, int(n)).tolist() for n in rng.integers(8, 60, 11)]
    stages = [[rng.integers(100, 900, int(n)).tolist() for n in rng.integers(4, 20, k)]
              for k in (7, 5)]
    frames = [[3, 4], [5]]
    return anchors, stages, frames


def cpu_join(anchors, stages, frames):
    """A two-stage join on the CPU with the same deterministic answer model."""
    arena = KVArena(1, 256, 16, 1, 8, device=None)

    class Rec(ModelPipeline):
        def forward_chunk(self, chunk):
            return chunk.host

    class Ans:
        dtype = None

        def submit(self, host):
            fin = host.final_indices
            return list(((host.input_ids[fin] + host.positions[fin]) % 2).astype(int))

        def result(self, h):
            return h

    answers, _, _ = loop.run_join(torch, arena, Rec(), Ans(), anchors, stages, 300,
                                  stage_frames=frames, attention_mode="tree",
                                  prefix_tree=prefix_tree(anchors, 16), device="cpu")
    return answers


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    docs = make_docs()
    try:
        def run_slice(lo, hi):
            if mode == "raise" and rank == 1:
                raise ValueError("injected host failure")
            return cpu_filter(docs[lo:hi])

        if mode == "exit" and rank == 1:
            os._exit(0)    # leaves between steps; nothing in flight
        if mode.startswith("join"):
            anchors, stages, frames = make_join()

            def run_join_slice(lo, hi):
                if mode == "join_raise" and rank == 0:
                    raise ValueError("injected host failure")
                return cpu_join(anchors[lo:hi], stages, frames)

            rows = run_sharded_join(torch, dist, len(anchors), len(stages), run_join_slice)
            out.put((rank, "ok", [{a: r.tolist() for a, r in st.items()} for st in rows], None))
            return
        if mode == "int64":
            # ids past 2^24 survive the gather unchanged
            mine = np.arange(3 + rank, dtype=np.int64) + (1 << 40) + (rank << 33) + 1
            got = gather_rows(torch, dist, mine, "cpu", np.int64)
            out.put((rank, "ok", [int(x) for x in got], str(got.dtype)))
            return
        row_tokens = [len(d) + 1 for d in docs] if mode == "tokens" else None
        bits, margins = run_sharded(torch, dist, len(docs), run_slice, row_tokens=row_tokens)
        out.put((rank, "ok", bits.tolist(), margins.tolist()))
    except RankFailed as exc:
        out.put((rank, "RankFailed", str(exc), None))
    except Exception as exc:
        out.put((rank, type(exc).__name__, str(exc), None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def run_ranks(mode, world=2):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    expected = world - (1 if mode == "exit" else 0)
    for _ in range(expected):
        rank, kind, a, b = out.get(timeout=120)
        results[rank] = (kind, a, b)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_two_ranks_reproduce_single_process_answers():
    docs = make_docs()
    want_bits, want_margins = (np.concatenate(x) for x in zip(
        cpu_filter(docs[:19]), cpu_filter(docs[19:])))
    results = run_ranks("ok")
    for rank in (0, 1):
        kind, bits, margins = results[rank]
        assert kind == "ok"
        assert np.array_equal(np.asarray(bits), want_bits.astype(np.uint8))
        assert np.allclose(margins, want_margins)


def test_token_balanced_ranks_reproduce_single_process_answers():
    """Slices balanced by tokens: the same per-row answers in row order."""
    docs = make_docs()
    tok = [len(d) + 1 for d in docs]
    cuts = [token_shard(tok, r, 2) for r in range(2)]
    assert cuts[0][1] == cuts[1][0]
    want_bits, want_margins = (np.concatenate(x) for x in zip(
        *(cpu_filter(docs[a:b]) for a, b in cuts)))
    results = run_ranks("tokens")
    for rank in (0, 1):
        kind, bits, margins = results[rank]
        assert kind == "ok"
        assert np.array_equal(np.asarray(bits), want_bits.astype(np.uint8))
        assert np.allclose(margins, want_margins)


def test_int64_gather_keeps_large_ids():
    results = run_ranks("int64")
    want = [int(x) for r in range(2)
            for x in np.arange(3 + r, dtype=np.int64) + (1 << 40) + (r << 33) + 1]
    for rank in (0, 1):
        kind, got, dtype = results[rank]
        assert kind == "ok" and dtype == "int64"
        assert got == want


def test_a_raising_rank_fails_every_rank():
    results = run_ranks("raise")
    assert results[0][0] == "RankFailed"
    assert results[1][0] == "RankFailed"


@pytest.mark.timeout(120)
def test_an_exiting_rank_ends_the_others_collective_with_an_error():
    results = run_ranks("exit")
    kind, msg, _ = results[0]
    assert kind != "ok"


def test_two_ranks_reproduce_single_process_join():
    """A two-stage join sharded by anchor over two gloo ranks: every rank
    ends with the rows the single-process join gives, keyed by anchor."""
    anchors, stages, frames = make_join()
    want = cpu_join(anchors, stages, frames)
    want = [{a: [float(x) for x in row] for a, row in st.items()} for st in want]
    results = run_ranks("join")
    for rank in (0, 1):
        kind, rows, _ = results[rank]
        assert kind == "ok"
        assert rows == want


def test_a_raising_rank_fails_every_rank_of_a_join():
    results = run_ranks("join_raise")
    assert {k for k, _, _ in results.values()} == {"RankFailed"}

