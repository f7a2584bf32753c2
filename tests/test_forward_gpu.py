"""End-to-end parity: the filter loop on the GPU against the CPU oracle.

quail_b200.loop.run_filter drives the sm_100a pipeline over seeded rows
that share an instruction prefix (the BASELINE config-1 row layout:
prefix | suffix, one-token question tail); every packed chunk is replayed
through the oracle's forward pass on the CPU in the same order, over a CPU
copy of the arena.

The north-star bar is |margin difference| <= 0.05 and equal decisions
where the oracle's |margin| > 0.1. These tests hold the stronger bar the
exact oracle allows: margins equal bit for bit. (With random-init weights
the bar needs it: one rounding tie that moves a single FP8 group scale
changes a 36-layer model's margins by up to about 0.3, the oracle against
itself with fp32 instead of exact GEMM partial sums included.)
"""

import numpy as np
import pytest
import torch

from oracle import forward as of
from oracle import numerics as nx
from quail_b200 import _native as nat
from quail_b200 import loop
from quail_b200.arena import KVArena
from quail_b200.model import QWEN3_4B, TINY, random_weights
from quail_b200.pipeline import Qwen3Pipeline
from quail_b200.readout import AnswerRows, AsyncAnswers, AsyncScores
from quail_b200.tokens import prefix_tree

pytestmark = pytest.mark.gpu

MARGIN_TOL = 0.05
DECISION_MARGIN = 0.1


def rows_with_prefix(seed, n, prefix_len, lo, hi, vocab_lo, vocab_hi):
    rng = np.random.default_rng(seed)
    prefix = rng.integers(vocab_lo, vocab_hi, prefix_len).tolist()
    lens = rng.integers(lo, hi + 1, n)
    docs = [prefix + rng.integers(vocab_lo, vocab_hi, int(s)).tolist() for s in lens]
    question = [int(np.random.default_rng(3).integers(vocab_lo, vocab_hi))]
    return docs, [question]


def run_and_compare(cfg, weights, docs, questions, budget, n_pages, mode):
    dev = torch.device("cuda")
    arena = KVArena(cfg.n_layers, n_pages, 16, cfg.n_kv, cfg.head_dim, device=dev)
    arena.pools.zero_()
    pipe = Qwen3Pipeline(torch, weights, arena)
    ans = AsyncAnswers(torch, AnswerRows(torch, weights), keep_margins=True)
    hosts = []
    answers, _, _ = loop.run_filter(
        torch, arena, pipe, ans, docs, questions, budget, arena_writes=True,
        attention_mode=mode, prefix_tree=prefix_tree(docs, 16), device=dev,
        on_chunk=lambda host, groups: hosts.append((host, list(groups))))
    torch.cuda.synchronize()
    assert nat.kernel_status(torch.cuda.current_device()) == 0
    assert len(ans.margins) == len(hosts)
    cpu_w = weights.to("cpu")
    cpu_arena = of.CpuArena(cfg.n_layers, arena.pool_rows, cfg.n_kv, cfg.head_dim)
    allowed, ans_w, tc, fc = cpu_w.answer_rows()
    worst = 0.0
    compared = 0
    for (host, groups), got in zip(hosts, ans.margins):
        normed = of.forward_chunk(cpu_w, host, cpu_arena)
        want, _ = nx.answer_margin(normed, ans_w, tc, fc)
        want = want.numpy()
        diff = np.abs(got - want)
        worst = max(worst, float(diff.max()))
        assert diff.max() <= MARGIN_TOL, (diff.max(), got, want)
        sure = np.abs(want) > DECISION_MARGIN
        assert np.array_equal(got[sure] > 0, want[sure] > 0)
        assert np.array_equal(got.view(np.int32), want.astype(np.float32).view(np.int32)), \
            (got, want)
        compared += len(want)
    assert compared == sum(len(h.final_indices) for h, _ in hosts)
    return answers, worst


@pytest.mark.parametrize("mode", ["tree", "unified"])
def test_tiny_filter_matches_oracle(mode):
    cfg = TINY
    weights = random_weights(cfg, seed=0, device="cuda")
    docs, questions = rows_with_prefix(1, 48, 64, 16, 200, 16, cfg.vocab)
    answers, worst = run_and_compare(cfg, weights, docs, questions, budget=1500,
                                     n_pages=400, mode=mode)
    assert len(answers) == len(docs)


def test_staged_uploads_give_the_same_answers():
    """Chunk uploads through one reused InputStaging (pinned host and device
    buffers per array, reused across chunks and calls) give the margins of
    fresh per-chunk copies, over several chunks and two calls."""
    from quail_b200.loop import InputStaging
    cfg = TINY
    dev = torch.device("cuda")
    weights = random_weights(cfg, seed=5, device=dev)
    docs, questions = rows_with_prefix(6, 40, 64, 16, 160, 16, cfg.vocab)

    def run(staging):
        arena = KVArena(cfg.n_layers, 400, 16, cfg.n_kv, cfg.head_dim, device=dev)
        arena.pools.zero_()
        pipe = Qwen3Pipeline(torch, weights, arena)
        ans = AsyncAnswers(torch, AnswerRows(torch, weights), keep_margins=True)
        stats = {}
        loop.run_filter(torch, arena, pipe, ans, docs, questions, 900, arena_writes=True,
                        attention_mode="tree", prefix_tree=prefix_tree(docs, 16), device=dev,
                        stats=stats, staging=staging)
        torch.cuda.synchronize()
        return np.concatenate(ans.margins), stats

    want, base = run(None)
    staging = InputStaging(torch, dev)
    for _ in range(2):
        got, stats = run(staging)
        assert stats["chunks"] == base["chunks"] > 3
        assert stats["h2d_bytes"] == base["h2d_bytes"]
        assert np.array_equal(got.view(np.int32), want.view(np.int32))
    assert len(staging.buffers) <= 16
    assert nat.kernel_status(torch.cuda.current_device()) == 0


def test_tiny_multistage_filter_matches_oracle():
    cfg = TINY
    weights = random_weights(cfg, seed=4, device="cuda")
    docs, _ = rows_with_prefix(2, 20, 48, 8, 100, 16, cfg.vocab)
    questions = [[30, 31, 32], [30, 31, 40, 41], [30, 50]]
    run_and_compare(cfg, weights, docs, questions, budget=800, n_pages=300, mode="tree")


def test_qwen3_4b_shaped_rows_match_oracle():
    """Full-width 36-layer model on a handful of config-1-shaped rows."""
    cfg = QWEN3_4B
    weights = random_weights(cfg, seed=0, device="cuda")
    docs, questions = rows_with_prefix(0, 3, 64, 16, 48, 1000, 150000)
    run_and_compare(cfg, weights, docs, questions, budget=4096, n_pages=200, mode="tree")


def test_full_budget_config1_chunk_rows_match_oracle():
    """A full config-1 chunk (the 110,376-token budget, about 450 rows with
    suffixes lognormal(5.3, 0.6) clipped to [32, 2048], one of them past
    1,500 tokens) through a 2-layer model of Qwen3-4B's width: the
    persistent GEMMs' multi-wave tile walk at M near 110k, many-tile causal
    segments and the shared prefix read by every row. A row's margin
    depends only on its own tokens and the shared prefix (every kernel is
    per row or per segment), so the oracle replays two rows of the chunk -
    the prefix-tree root that computes the shared 64 tokens and the longest
    row, which borrows them - as a chunk of their own, and their margins must
    equal the GPU's bit for bit. (About two minutes of exact-mode oracle
    time on 16 host cores for the two replayed rows.)"""
    import dataclasses
    from quail_b200.workload import config1
    cfg = dataclasses.replace(QWEN3_4B, name="qwen3-4b-2l", n_layers=2)
    wl = config1()
    lengths = wl.docs.lengths
    long_row = int(np.flatnonzero(lengths >= 1500)[0])
    picked = list(range(470)) + [long_row]
    docs = [wl.docs[i] for i in picked]
    budget = QWEN3_4B.max_chunk_tokens
    dev = torch.device("cuda")
    weights = random_weights(cfg, seed=0, device=dev)
    arena = KVArena(cfg.n_layers, 8192, 16, cfg.n_kv, cfg.head_dim, device=dev)
    arena.pools.zero_()
    pipe = Qwen3Pipeline(torch, weights, arena)
    ans = AsyncAnswers(torch, AnswerRows(torch, weights), keep_margins=True)
    hosts = []
    loop.run_filter(torch, arena, pipe, ans, docs, wl.questions, budget, arena_writes=True,
                    attention_mode="tree", prefix_tree=prefix_tree(docs, 16), device=dev,
                    on_chunk=lambda host, groups: hosts.append(host))
    torch.cuda.synchronize()
    assert nat.kernel_status(torch.cuda.current_device()) == 0
    first = hosts[0]
    assert first.tokens > 100_000
    got = {}
    for host, margins in zip(hosts, ans.margins):
        for (doc, _), m in zip(host.layout, margins):
            got[doc] = m
    tree = prefix_tree(docs, 16)
    root = int(tree.order[0])
    first_docs = [doc for doc, _ in first.layout]
    assert root in first_docs and len(picked) - 1 in first_docs, "the long row is in chunk 1"
    check = [root, len(picked) - 1]
    sub = [docs[d] for d in check]
    sub_tree = prefix_tree(sub, 16)
    assert int(sub_tree.order[0]) == 0, "the same row computes the shared prefix"
    cpu_w = weights.to("cpu")
    cpu_arena = of.CpuArena(cfg.n_layers, 64 * 16 * 16, cfg.n_kv, cfg.head_dim)
    sub_arena = KVArena(1, 1024, 16, 1, 8, device=None)
    _, ans_w, tc, fc = cpu_w.answer_rows()
    want = {}

    class Oracle:
        tree_attention = True

        def forward_chunk(self, chunk):
            return chunk.host

    class Answers:
        def submit(self, host):
            normed = of.forward_chunk(cpu_w, host, cpu_arena)
            margin, _ = nx.answer_margin(normed, ans_w, tc, fc)
            for (doc, _), m in zip(host.layout, margin.numpy()):
                want[check[doc]] = m
            return [1] * len(host.layout)

        def result(self, h):
            return h

    loop.run_filter(torch, sub_arena, Oracle(), Answers(), sub, wl.questions, budget,
                    arena_writes=True, attention_mode="tree", prefix_tree=sub_tree,
                    device="cpu")
    for d in check:
        assert np.float32(got[d]).view(np.int32) == np.float32(want[d]).view(np.int32), \
            (d, got[d], want[d])


def test_qwen3_32b_width_rows_match_oracle():
    """Qwen3-32B's layer shapes (hidden 5120, 64 query / 8 KV heads, inter
    25600), two layers, on a few config-3-shaped rows."""
    import dataclasses
    from quail_b200.model import QWEN3_32B
    cfg = dataclasses.replace(QWEN3_32B, name="qwen3-32b-2l", n_layers=2)
    weights = random_weights(cfg, seed=2, device="cuda")
    docs, questions = rows_with_prefix(3, 2, 96, 16, 48, 1000, 150000)
    run_and_compare(cfg, weights, docs, questions, budget=4096, n_pages=100, mode="tree")


def join_rows(seed, cfg, n_anchors, n_partners, n_stages):
    """Config 2's shape, small: a shared instruction + left document per
    anchor, right documents as partners, a frame per stage."""
    rng = np.random.default_rng(seed)
    instr = rng.integers(16, cfg.vocab, 48).tolist()
    anchors = [instr + rng.integers(16, cfg.vocab, int(rng.integers(20, 120))).tolist()
               for _ in range(n_anchors)]
    stages = [[rng.integers(16, cfg.vocab, int(rng.integers(8, 48))).tolist()
               for _ in range(n_partners)] for _ in range(n_stages)]
    frames = [rng.integers(16, cfg.vocab, 3).tolist() for _ in range(n_stages)]
    return anchors, stages, frames


class RecordingScores(AsyncScores):
    """AsyncScores that keeps each chunk's scores for the comparison."""

    def __init__(self, torch_, rows):
        super().__init__(torch_, rows)
        self.kept = []

    def result(self, handle):
        out = super().result(handle)
        self.kept.append(out.copy())
        return out


def run_join_and_compare(cfg, weights, anchors, stages, frames, budget, n_pages, mode,
                         score=False, partners=None):
    dev = torch.device("cuda")
    arena = KVArena(cfg.n_layers, n_pages, 16, cfg.n_kv, cfg.head_dim, device=dev)
    arena.pools.zero_()
    pipe = Qwen3Pipeline(torch, weights, arena)
    rows = AnswerRows(torch, weights)
    ans = RecordingScores(torch, rows) if score else AsyncAnswers(torch, rows, keep_margins=True)
    hosts = []
    answers, _, _ = loop.run_join(
        torch, arena, pipe, ans, anchors, stages, budget, stage_frames=frames,
        attention_mode=mode, prefix_tree=prefix_tree(anchors, 16), device=dev,
        anchor_partners=None if partners is None else (lambda key: [partners[key]]),
        on_chunk=lambda host, groups: hosts.append(host))
    torch.cuda.synchronize()
    assert nat.kernel_status(torch.cuda.current_device()) == 0
    got_rows = ans.kept if score else ans.margins
    assert len(got_rows) == len(hosts)
    cpu_w = weights.to("cpu")
    cpu_arena = of.CpuArena(cfg.n_layers, arena.pool_rows, cfg.n_kv, cfg.head_dim)
    _, ans_w, tc, fc = cpu_w.answer_rows()
    for host, got in zip(hosts, got_rows):
        normed = of.forward_chunk(cpu_w, host, cpu_arena)
        if score:
            want = nx.answer_score(normed, ans_w, tc, fc).numpy()
        else:
            want = nx.answer_margin(normed, ans_w, tc, fc)[0].numpy()
        assert np.array_equal(got.view(np.int32), want.astype(np.float32).view(np.int32)), \
            (got, want)
    assert not arena.accounting.owned  # every anchor settled and freed
    return answers


@pytest.mark.parametrize("mode", ["tree", "unified"])
def test_tiny_join_matches_oracle(mode):
    """AI join (run_join): two stages with frames, prefix-sharing anchors."""
    cfg = TINY
    weights = random_weights(cfg, seed=5, device="cuda")
    anchors, stages, frames = join_rows(6, cfg, 8, 10, 2)
    answers = run_join_and_compare(cfg, weights, anchors, stages, frames, budget=700,
                                   n_pages=300, mode=mode)
    assert len(answers) == 2 and answers[0]


def test_tiny_score_matches_oracle():
    """AI.SCORE (run_join with AsyncScores): float32 scores per partner."""
    cfg = TINY
    weights = random_weights(cfg, seed=6, device="cuda")
    anchors, stages, _ = join_rows(7, cfg, 8, 10, 1)
    rng = np.random.default_rng(8)
    partners = [sorted(int(i) for i in rng.choice(10, size=int(rng.integers(1, 10)),
                                                   replace=False)) for _ in anchors]
    answers = run_join_and_compare(cfg, weights, anchors, stages, None, budget=600,
                                   n_pages=300, mode="tree", score=True, partners=partners)
    assert sorted(answers[0]) == list(range(len(anchors)))
    for a, row in answers[0].items():
        assert row.dtype == np.float32 and len(row) == len(partners[a])


def test_executor_join_and_score_api():
    """B200Executor.join / .score (the public calls) on the tiny model: rows
    per anchor over its partners, every page back on the free list."""
    from quail_b200.api import B200Executor
    cfg = TINY
    ex = B200Executor(torch, cfg, 300, seed=5)
    anchors, stages, frames = join_rows(9, cfg, 5, 7, 2)
    res = ex.join(anchors, stages, stage_frames=frames, budget=700)
    assert len(res.answers) == 2
    assert all(len(row) == 7 for row in res.answers[0].values())
    assert res.fresh_tokens > 0 and res.gpu_s > 0
    assert ex.arena.free_pages == 300
    partners = [[0, 2, 4], [1], [0, 1, 2, 3, 4, 5, 6], [6], [3, 5]]
    scores = ex.score(anchors, stages[0], budget=700, partners=partners)
    for a, row in scores.answers[0].items():
        assert row.dtype == np.float32 and len(row) == len(partners[a])
        assert np.all((row >= 0) & (row <= 1))
    assert ex.arena.free_pages == 300


def test_tiny_filter_feeding_join_matches_oracle():
    """A filter whose survivors stream into a join as resident anchors
    (FilterStream hold_survivors as run_join's anchor_source): every chunk of
    both loops, in launch order, bit-exact against the oracle."""
    cfg = TINY
    weights = random_weights(cfg, seed=7, device="cuda")
    dev = torch.device("cuda")
    rng = np.random.default_rng(15)
    instr = rng.integers(16, cfg.vocab, 32).tolist()
    docs = [instr + rng.integers(16, cfg.vocab, int(rng.integers(10, 90))).tolist()
            for _ in range(14)]
    question = [int(rng.integers(16, cfg.vocab)), 5]
    frame = rng.integers(16, cfg.vocab, 3).tolist()
    partners = [rng.integers(16, cfg.vocab, int(rng.integers(6, 30))).tolist() for _ in range(7)]
    arena = KVArena(cfg.n_layers, 200, 16, cfg.n_kv, cfg.head_dim, device=dev)
    arena.pools.zero_()
    pipe = Qwen3Pipeline(torch, weights, arena)
    rows = AnswerRows(torch, weights)
    readouts = {"filter": AsyncAnswers(torch, rows, keep_margins=True),
                "join": AsyncAnswers(torch, rows, keep_margins=True)}
    launched = []
    source = loop.FilterStream(
        torch, arena, pipe, readouts["filter"], docs, [question], 350, arena_writes=True,
        arena_keys=[("d", i) for i in range(len(docs))], hold_survivors=True,
        hold_extra_tokens=len(frame), prefix_tree=prefix_tree(docs, 16), attention_mode="tree",
        device=dev, on_chunk=lambda host, groups: launched.append(("filter", host)))
    keys = []
    answers, _, _ = loop.run_join(
        torch, arena, pipe, readouts["join"], [], [partners], 350, stage_frames=[frame],
        anchor_keys=keys, anchor_source=source, attention_mode="tree", device=dev,
        on_chunk=lambda host, groups: launched.append(("join", host)))
    torch.cuda.synchronize()
    assert nat.kernel_status(torch.cuda.current_device()) == 0
    assert keys and len(answers[0]) == len(keys)
    cpu_w = weights.to("cpu")
    cpu_arena = of.CpuArena(cfg.n_layers, arena.pool_rows, cfg.n_kv, cfg.head_dim)
    _, ans_w, tc, fc = cpu_w.answer_rows()
    got = {kind: iter(r.margins) for kind, r in readouts.items()}
    for kind, host in launched:
        normed = of.forward_chunk(cpu_w, host, cpu_arena)
        want = nx.answer_margin(normed, ans_w, tc, fc)[0].numpy()
        g = next(got[kind])
        assert np.array_equal(g.view(np.int32), want.astype(np.float32).view(np.int32)), kind
    assert not arena.accounting.owned


def test_retained_survivors_feed_a_join_like_fresh_anchors():
    """Retention between operators on the GPU: a filter keeps its survivors'
    KV (retain_survivors), and a join over them reads that resident KV
    instead of recomputing the prefixes. The join's answers equal a join
    whose anchors are computed fresh, with fewer fresh tokens."""
    from quail_b200.api import B200Executor
    from quail_b200.retention import apply_retention

    cfg = TINY
    docs, questions = rows_with_prefix(9, 24, 48, 16, 120, 16, cfg.vocab)
    partners = [list(np.random.default_rng(4).integers(16, cfg.vocab, n)) for n in (9, 17, 12)]
    ex = B200Executor(torch, cfg, 600, seed=1)
    keys = [("d", i) for i in range(len(docs))]
    res = ex.filter(docs, questions, keys=keys, retain_survivors=True, budget=1200)
    survivors = [d for d in range(len(docs)) if res.bits[d]]
    assert survivors and set(k[1] for k in ex.arena.retained_keys()) <= set(survivors)
    config = {"linear_seconds": 1e-6, "pair_seconds": 1e-9, "cap_pages": ex.arena.n_pages}
    apply_retention(ex.arena, config, {"d": (1.0, 1)}, survivors={"d": survivors})
    resident = [d for d in survivors if ex.arena.is_resident(keys[d])]
    assert resident
    anchors = [docs[d] for d in survivors]
    warm = ex.join(anchors, [partners], budget=1200, anchor_keys=[keys[d] for d in survivors],
                   share_prefixes=False)
    ex.reset_arena()
    cold = ex.join(anchors, [partners], budget=1200, share_prefixes=False)
    assert warm.answers == cold.answers
    assert warm.fresh_tokens < cold.fresh_tokens
    assert nat.kernel_status(torch.cuda.current_device()) == 0
