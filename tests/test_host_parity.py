"""quail_b200's host loop against the reference's own, chunk by chunk.

The fixtures (tests/golden/host_*.npz/.json) were produced by running the
reference's run_filter and run_join with a recording pipeline (tests/golden/
make_golden.py). The same documents (anchors and partners for the joins)
go through quail_b200.loop.run_filter / run_join here; every packed array
must match bit for bit: token ids, positions,
answer rows, KV scatter rows, segment bounds, reader rows, block tables,
the merge source map, unified tables, chunk layouts and final answers.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from quail_b200 import loop
from quail_b200.arena import KVArena
from quail_b200.pipeline import ModelPipeline
from quail_b200.tokens import prefix_tree
from tests.golden import make_golden as mg

GOLDEN = Path(__file__).resolve().parent / "golden"


def run_ours(name):
    docs, questions, budget, pages, attention, use_tree, writes = mg.scenario_docs(name)
    arena = KVArena(1, pages, 16, 1, 8, device=None)
    arrays, entries = {}, []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(mg.chunk_record(chunk.host, arrays, len(entries)))
            return chunk.host

    class Answers:
        def submit(self, host):
            return mg.answer_bits(host.input_ids, host.positions, host.final_indices)

        def result(self, handle):
            return handle

    tree = prefix_tree(docs, 16) if use_tree else None
    stats = {}
    answers, _, tokens = loop.run_filter(
        torch, arena, Recorder(), Answers(), docs, questions, budget, arena_writes=writes,
        attention_mode=attention, prefix_tree=tree, stats=stats, device="cpu")
    return dict(entries=entries, arrays=arrays, tokens=tokens, answers=answers, stats=stats,
                arena=arena, tree=tree)


@pytest.mark.parametrize("name", mg.SCENARIOS)
def test_packed_chunks_match_reference(name):
    want = json.loads((GOLDEN / f"host_{name}.json").read_text())
    want_arrays = np.load(GOLDEN / f"host_{name}.npz")
    got = run_ours(name)
    assert len(got["entries"]) == len(want["chunks"])
    for i, (g, w) in enumerate(zip(got["entries"], want["chunks"])):
        assert g == w, f"chunk {i} metadata differs"
    assert sorted(got["arrays"]) == sorted(want_arrays.files)
    for key in want_arrays.files:
        a, b = got["arrays"][key], want_arrays[key]
        assert a.shape == b.shape, key
        assert np.array_equal(a.astype(np.int64), b.astype(np.int64)), key
    assert got["tokens"] == want["tokens"]
    assert got["stats"]["borrowed_tokens"] == want["borrowed_tokens"]
    assert {str(k): v for k, v in sorted(got["answers"].items())} == want["answers"]
    assert got["arena"].free_pages == want["free_pages_after"]
    if want["tree"] is not None:
        assert list(got["tree"].order) == want["tree"]["order"]
        assert got["tree"].parent == want["tree"]["parent"]
        assert list(got["tree"].shared) == want["tree"]["shared"]


def run_ours_join(name):
    anchors, stage_suffixes, frames, partners, budget, pages, attention, resident = \
        mg.join_inputs(name)
    arena = KVArena(1, pages, 16, 1, 8, device=None)
    frame_max = max(len(f) for f in frames) if frames else 0
    for a in resident:
        assert arena.activate(("a", a), len(anchors[a]),
                              capacity_tokens=len(anchors[a]) + frame_max) is not None
    arrays, entries = {}, []
    score = name.startswith("score")

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(mg.chunk_record(chunk.host, arrays, len(entries)))
            return chunk.host

    class Answers:
        dtype = np.float32 if score else None

        def submit(self, host):
            f = mg.score_values if score else mg.answer_bits
            return f(host.input_ids, host.positions, host.final_indices)

        def result(self, handle):
            return handle

    keys = [("a", i) for i in range(len(anchors))]
    stats = {}
    answers, _, tokens = loop.run_join(
        torch, arena, Recorder(), Answers(), anchors, stage_suffixes, budget,
        stage_frames=frames, anchor_keys=keys, attention_mode=attention,
        anchor_partners=None if partners is None else (lambda key: partners[key[1]]),
        prefix_tree=prefix_tree(anchors, 16), stats=stats, device="cpu")
    return dict(entries=entries, arrays=arrays, tokens=tokens, answers=answers, stats=stats,
                arena=arena)


@pytest.mark.parametrize("name", mg.JOIN_SCENARIOS)
def test_join_chunks_match_reference(name):
    """run_join (AI joins and AI.SCORE) against the reference's, chunk by chunk."""
    want = json.loads((GOLDEN / f"host_{name}.json").read_text())
    want_arrays = np.load(GOLDEN / f"host_{name}.npz")
    got = run_ours_join(name)
    assert len(got["entries"]) == len(want["chunks"])
    for i, (g, w) in enumerate(zip(got["entries"], want["chunks"])):
        assert g == w, f"chunk {i} metadata differs"
    assert sorted(got["arrays"]) == sorted(want_arrays.files)
    for key in want_arrays.files:
        a, b = got["arrays"][key], want_arrays[key]
        assert a.shape == b.shape, key
        assert np.array_equal(a.astype(np.int64), b.astype(np.int64)), key
    assert got["tokens"] == want["tokens"]
    assert got["stats"]["borrowed_tokens"] == want["borrowed_tokens"]
    answers = [{str(a): [float(x) for x in row] for a, row in sorted(st.items())}
               for st in got["answers"]]
    assert answers == want["answers"]
    assert got["arena"].free_pages == want["free_pages_after"]


def test_prefix_tree_shapes():
    """The reference's own prefix-tree cases (tests/test_tokens.py:74-108)."""
    docs = [list(range(40)), list(range(50)), list(range(32)) + [99] * 20, [7] * 20, [7] * 10]
    tree = prefix_tree(docs, 16)
    assert tree.order == [0, 1, 2, 4, 3]
    assert tree.parent == [None, 0, 0, None, None]
    assert tree.shared == [0, 32, 32, 0, 0]
    assert tree.shared_tokens == 64
    assert prefix_tree([], 16).shared_tokens == 0
    tree = prefix_tree([[], [], [5] * 16 + [6]], 16)
    assert tree.parent == [None, None, None]
    header = list(range(64))
    docs = [header + [1] * 8, header + [2] * 8, header + [3] * 8,
            header + [3] * 8 + [4] * 40, header + [5] * 8]
    tree = prefix_tree(docs, 16)
    assert tree.parent == [None, 0, 0, 0, 0]
    assert tree.shared == [0, 64, 64, 64, 64]
    docs = [header + [1] * 32, header + [1] * 32 + [2] * 8, header + [1] * 32 + [3] * 8]
    tree = prefix_tree(docs, 16)
    assert tree.parent == [None, 0, 0]
    assert tree.shared == [0, 96, 96]


def test_attention_tiles_cover_every_row_once():
    cu = [0, 5, 5, 200, 264, 265]
    tiles = loop.attention_tiles(cu)
    covered = []
    for seg, row0 in tiles:
        end = min(row0 + loop.ATTN_TILE, cu[seg + 1])
        assert cu[seg] <= row0 < cu[seg + 1]
        covered.extend(range(row0, end))
    assert sorted(covered) == list(range(265))
    # most work first: offsets within a segment never increase
    offsets = [row0 - cu[seg] for seg, row0 in tiles]
    assert offsets == sorted(offsets, reverse=True)


def test_arena_free_stack_and_borrow_holds():
    arena = KVArena(1, 8, 16, 1, 8, device=None)
    assert arena.alloc("a", 40) == [0, 1, 2]
    assert arena.alloc("b", 48, borrow=("a", 32)) == [3]
    assert arena.owned_pages("b") == [0, 1, 3]
    assert list(arena.capacity_rows("b")[:3]) == [0, 1, 2]
    arena.hold("a", 1)
    assert arena.free_key("a") == 0          # deferred: a borrower is queued
    arena.release("a")                       # the last borrower admitted
    assert not arena.is_resident("a")
    assert arena.free_pages == 8 - 3         # pages 0, 1 still held by b
    arena.free_key("b")
    assert arena.free_pages == 8
    # LIFO: freed pages come back in release order
    assert arena.alloc("c", 16) == [3]


def test_join_survivors_semi_and_anti():
    """EXISTS / NOT EXISTS over a join's last-stage rows (backend.py:231-240)."""
    from quail_b200.api import JoinResult
    res = JoinResult(answers=[{0: [1, 0], 1: [0, 0], 3: [0, 1]}, {0: [0, 1], 3: [0, 0]}],
                     fresh_tokens=0, borrowed_tokens=0, chunks=0, h2d_bytes=0, d2h_bytes=0,
                     gpu_s=0.0, wall_s=0.0, n_anchors=5)
    assert res.survivors("semi") == [0]
    assert res.survivors("anti") == [1, 2, 3, 4]


def test_exists_workload_scores_each_candidate_once():
    """Config 4's EXISTS variant through run_join's per-anchor partner lists:
    every outer row answers exactly its own candidates, each candidate is
    packed once, the outer rows once with their shared 64-token prefix
    computed by the first and borrowed by the others, and no chunk exceeds
    the budget."""
    from quail_b200.workload import config4_exists
    wl = config4_exists(outer=6)
    outer = [1, 2, 3]
    anchors = [wl.anchors[a] for a in outer]
    sufs, partners = [], []
    for a in outer:
        first = len(sufs)
        sufs.extend(wl.candidates(a))
        partners.append([list(range(first, len(sufs)))])
    assert all(len(x) == 576 for x in anchors)
    assert all(4096 + 1 <= len(x) <= 16384 + 1 for x in sufs)
    arena = KVArena(1, 16384, 16, 1, 8, device=None)
    budget = 110376
    sizes = []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            sizes.append(chunk.host.tokens)
            return len(chunk.host.final_indices)

    class Answers:
        dtype = None  # 0/1 answer rows, as AsyncAnswers

        def submit(self, n):
            return [1] * n

        def result(self, handle):
            return handle

    stats = {}
    answers, _, tokens = loop.run_join(
        torch, arena, Recorder(), Answers(), anchors, [sufs], budget, attention_mode="tree",
        prefix_tree=prefix_tree(anchors, 16), anchor_partners=lambda k: partners[k],
        stats=stats, device="cpu")
    assert {a: len(row) for a, row in answers[0].items()} == {0: 8, 1: 8, 2: 8}
    assert stats["borrowed_tokens"] == 64 * (len(anchors) - 1)
    assert tokens == sum(map(len, anchors)) + sum(map(len, sufs)) - stats["borrowed_tokens"]
    assert max(sizes) <= budget


def _exists_join(anchors, sufs, partners, budget, stop, true_rate, step=None):
    """Single-stage join on the CPU; a partner answers TRUE when a hash of
    its final row's token and position falls under true_rate."""
    arena = KVArena(1, 4096, 16, 1, 8, device=None)
    packed = []

    class Rec(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            packed.append(chunk.host.tokens)
            return chunk.host

    class Ans:
        dtype = None

        def submit(self, host):
            fin = host.final_indices
            h = (host.input_ids[fin] * 2654435761 + host.positions[fin] * 40503) % 1000
            return list((h < true_rate * 1000).astype(int))

        def result(self, h):
            return h

    stats = {}
    answers, _, tokens = loop.run_join(
        torch, arena, Rec(), Ans(), anchors, [sufs], budget, attention_mode="tree",
        prefix_tree=prefix_tree(anchors, 16), anchor_partners=lambda k: partners[k],
        stats=stats, device="cpu", stop_at_true=stop, stream_step=step)
    assert arena.free_pages == arena.n_pages, "every page returns to the free stack"
    return answers[0], stats["skipped_partners"], tokens


def _exists_case(true_rate, step):
    """Full join vs early-stopped join of 9 outer rows x 16 candidates;
    returns the candidates the stop skipped."""
    from quail_b200.api import JoinResult
    rng = np.random.default_rng(31)
    prefix = rng.integers(100, 900, 64).tolist()
    anchors = [prefix + rng.integers(100, 900, 96).tolist() for _ in range(9)]
    sufs, partners = [], []
    for _ in anchors:
        first = len(sufs)
        sufs.extend(rng.integers(100, 900, int(n)).tolist() + [7]
                    for n in rng.integers(20, 100, 16))
        partners.append([list(range(first, len(sufs)))])
    full, skipped_full, tok_full = _exists_join(anchors, sufs, partners, 400, False, true_rate)
    stop, skipped, tok_stop = _exists_join(anchors, sufs, partners, 400, True, true_rate, step)
    assert skipped_full == 0
    kw = dict(fresh_tokens=0, borrowed_tokens=0, chunks=0, h2d_bytes=0, d2h_bytes=0,
              gpu_s=0.0, wall_s=0.0, n_anchors=len(anchors))
    for sem in ("semi", "anti"):
        assert (JoinResult(answers=[stop], **kw).survivors(sem)
                == JoinResult(answers=[full], **kw).survivors(sem))
    cut = 0
    for a, row in full.items():
        got = stop[a]
        assert list(got) == list(row[:len(got)])
        if len(got) < len(row):
            assert any(got)
            cut += len(row) - len(got)
    assert cut == skipped
    skipped_tokens = sum(len(sufs[i]) for a, row in full.items()
                         for i in partners[a][0][len(stop[a]):])
    assert tok_stop == tok_full - skipped_tokens
    return skipped


@pytest.mark.parametrize("step", [None, 1, 3])
@pytest.mark.parametrize("true_rate", [0.05, 0.3, 0.9])
def test_exists_early_stop_keeps_survivors(true_rate, step):
    """EXISTS early stop: an outer row's candidates not yet launched when one
    of its candidates answers TRUE are skipped. The EXISTS and NOT EXISTS
    survivors equal those of the full join (the reference's any(row) gate,
    backend.py:231-240), every stopped row is a prefix of the full row that
    holds a TRUE, and the skipped candidates are never packed."""
    skipped = _exists_case(true_rate, step)
    if true_rate >= 0.3:
        assert skipped > 0


def test_interleaved_streams_skip_more():
    """One candidate per outer row per chunk lets a TRUE stop its stream
    before most of it is packed."""
    assert _exists_case(0.3, 1) > _exists_case(0.3, None)


def test_exists_stop_rejects_scores():
    from quail_b200.pack import JoinAdmission
    with pytest.raises(ValueError, match="0/1 answers"):
        JoinAdmission([10], [[5]], 100, 64, 16, answer_dtype=np.float32, stop_at_true=True)


def test_token_store_reads_reference_file():
    """The host input format: a token store file written by the reference's
    TokenStore opens here with the same documents and lengths, and (checked
    when the fixture was made) one written here opens in the reference."""
    from quail_b200.token_store import TokenStore
    want = json.loads((GOLDEN / "token_store.json").read_text())
    store = TokenStore(GOLDEN / "token_store.arrow")
    assert len(store) == len(want["documents"])
    for i, doc in enumerate(want["documents"]):
        assert store[i].tolist() == doc
        assert store.lengths[i] == len(doc)
    assert want["reads_ours"]
    store.close()


def test_filter_over_token_store_matches_reference(tmp_path):
    """run_filter over documents served from a memory-mapped token store
    packs the same chunks as over lists (the cfg1_tree golden)."""
    from quail_b200.token_store import write_token_store
    name = "cfg1_tree"
    docs, questions, budget, pages, attention, use_tree, writes = mg.scenario_docs(name)
    store = write_token_store(tmp_path / "docs.arrow", docs, batch_rows=16)
    want = json.loads((GOLDEN / f"host_{name}.json").read_text())
    want_arrays = np.load(GOLDEN / f"host_{name}.npz")
    arena = KVArena(1, pages, 16, 1, 8, device=None)
    arrays, entries = {}, []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(mg.chunk_record(chunk.host, arrays, len(entries)))
            return chunk.host

    class Answers:
        def submit(self, host):
            return mg.answer_bits(host.input_ids, host.positions, host.final_indices)

        def result(self, handle):
            return handle

    answers, _, tokens = loop.run_filter(
        torch, arena, Recorder(), Answers(), store, questions, budget, arena_writes=writes,
        attention_mode=attention, prefix_tree=prefix_tree(store, 16), device="cpu")
    assert entries == want["chunks"]
    for key in want_arrays.files:
        assert np.array_equal(arrays[key].astype(np.int64), want_arrays[key].astype(np.int64)), key
    assert {str(k): v for k, v in sorted(answers.items())} == want["answers"]
    assert tokens == want["tokens"]
    store.close()


@pytest.mark.parametrize("name", mg.FEED_SCENARIOS)
def test_filter_feeding_join_matches_reference(name):
    """A filter whose survivors stream into a join as resident anchors
    (FilterStream hold_survivors as run_join's anchor_source): both loops'
    chunks in launch order, the filter's answers, the anchors admitted and
    the join's answers."""
    docs, question, frame, partners, budget, pages, attention = mg.feed_inputs(name)
    want = json.loads((GOLDEN / f"host_{name}.json").read_text())
    want_arrays = np.load(GOLDEN / f"host_{name}.npz")
    arena = KVArena(1, pages, 16, 1, 8, device=None)
    arrays, entries = {}, []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(mg.chunk_record(chunk.host, arrays, len(entries)))
            return chunk.host

    class Answers:
        dtype = None

        def submit(self, host):
            return mg.answer_bits(host.input_ids, host.positions, host.final_indices)

        def result(self, handle):
            return handle

    source = loop.FilterStream(
        torch, arena, Recorder(), Answers(), docs, [question], budget, arena_writes=True,
        arena_keys=[("d", i) for i in range(len(docs))], hold_survivors=True,
        hold_extra_tokens=len(frame), prefix_tree=prefix_tree(docs, 16),
        attention_mode=attention, device="cpu")
    keys = []
    answers, _, tokens = loop.run_join(
        torch, arena, Recorder(), Answers(), [], [partners], budget, stage_frames=[frame],
        anchor_keys=keys, anchor_source=source, attention_mode=attention, device="cpu")
    assert entries == want["chunks"]
    assert sorted(arrays) == sorted(want_arrays.files)
    for key in want_arrays.files:
        assert np.array_equal(arrays[key].astype(np.int64), want_arrays[key].astype(np.int64)), key
    assert {str(k): v for k, v in sorted(source.answers.items())} == want["filter_answers"]
    assert [key[1] for key in keys] == want["keys"]
    assert [{str(a): [float(x) for x in row] for a, row in sorted(st.items())}
            for st in answers] == want["answers"]
    assert tokens == want["tokens"] and source.tokens == want["source_tokens"]
    assert arena.free_pages == want["free_pages_after"]



@pytest.mark.parametrize("name", mg.RETAIN_SCENARIOS)
def test_retention_between_operators_matches_reference(name):
    """KV retention across operators (arena retention, FilterStream
    retain_survivors, quail_b200.retention): a filter whose survivors stay
    resident (evicted past the cap in priority order), a boundary that frees
    the survivors no later operator reads and re-prioritises the rest, and a
    join over every survivor (the retained ones resident, so their prefixes
    are not recomputed; admission evicting retained KV when short of pages)
    whose matching anchors are retained again. Chunks of both loops, the
    answers and the arena's retained keys, free pages and eviction counters
    after each phase equal the reference's."""
    from quail_b200.retention import apply_retention, retain_after_join

    (docs, question, frame, partners, budget, pages, attention, config, uses,
     after) = mg.retention_inputs(name)
    want = json.loads((GOLDEN / f"host_{name}.json").read_text())
    want_arrays = np.load(GOLDEN / f"host_{name}.npz")
    arena = KVArena(1, pages, 16, 1, 8, device=None)
    arrays, entries = {}, []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(mg.chunk_record(chunk.host, arrays, len(entries)))
            return chunk.host

    class Answers:
        dtype = None

        def submit(self, host):
            return mg.answer_bits(host.input_ids, host.positions, host.final_indices)

        def result(self, handle):
            return handle

    keys = [("d", i) for i in range(len(docs))]
    f_answers, _, f_tokens = loop.run_filter(
        torch, arena, Recorder(), Answers(), docs, [question], budget, arena_writes=True,
        arena_keys=keys, retain_survivors=True, attention_mode=attention,
        prefix_tree=prefix_tree(docs, 16), device="cpu")
    assert len(entries) == want["n_filter_chunks"]
    assert mg.arena_state(arena) == want["after_filter"]
    survivors = sorted(d for d, row in f_answers.items() if row and row[-1])
    assert survivors == want["survivors"]
    apply_retention(arena, config, uses, survivors={"d": survivors[:-2]})
    assert mg.arena_state(arena) == want["after_boundary"]
    anchors = [docs[d] for d in survivors]
    akeys = [keys[d] for d in survivors]

    def anchor_done(a, row):
        if any(row):
            retain_after_join(arena, akeys[a], len(anchors[a]), config, after)
        else:
            arena.free_key(akeys[a])

    j_answers, _, j_tokens = loop.run_join(
        torch, arena, Recorder(), Answers(), anchors, [partners], budget,
        stage_frames=[frame], anchor_keys=akeys, anchor_done=anchor_done,
        attention_mode=attention, device="cpu")
    assert entries == want["chunks"]
    assert sorted(arrays) == sorted(want_arrays.files)
    for key in want_arrays.files:
        assert np.array_equal(arrays[key].astype(np.int64), want_arrays[key].astype(np.int64)), key
    assert {str(k): v for k, v in sorted(f_answers.items())} == want["filter_answers"]
    assert [{str(a): [float(x) for x in row] for a, row in sorted(st.items())}
            for st in j_answers] == want["join_answers"]
    assert (f_tokens, j_tokens) == (want["filter_tokens"], want["join_tokens"])
    assert mg.arena_state(arena) == want["after_join"]


def test_retention_priority_and_rewind():
    """Unit checks of the retention rules on the accounting alone: a
    retained key rewinds to its prefix, eviction takes the lowest priority
    first, a held key is passed over, pinning withdraws a key and the cap
    evicts on retain."""
    from quail_b200.retention import RetentionPolicy, causal_pairs

    assert causal_pairs(4) == 10 and causal_pairs(10, 4) == 4 * 10 - 6
    arena = KVArena(1, 20, 16, 1, 8, device=None)
    for i, n in enumerate((40, 64, 20)):
        assert arena.activate(("d", i), n, capacity_tokens=n + 30) is not None
    free0 = arena.free_pages
    assert arena.retain(("d", 0), 40) == 2  # 70 capacity tokens: 5 pages; 40 tokens: 3
    arena.retain(("d", 1), 64)
    arena.retain(("d", 2), 20)
    assert arena.free_pages > free0
    assert sorted(arena.retained_keys()) == [("d", 0), ("d", 1), ("d", 2)]
    # tokens per page: d0 40/3, d1 64/4, d2 20/2 -> d2 goes first, then d0
    arena.hold(("d", 2), 1)
    assert arena.evict_retained(1) == (("d", 0),)
    arena.drop_holds([("d", 2)])
    arena.pin(("d", 1))
    assert arena.retained_keys() == [("d", 2)]
    arena.configure_retention(RetentionPolicy(1e-6, 1e-9, {"d": (1.0, 1)}), 0)
    assert arena.evict_retained(arena.retained_pages) == (("d", 2),)
    assert arena.evicted_keys == 2 and arena.retained_pages == 0
    with pytest.raises(TypeError):
        arena.retain(7, 10)
