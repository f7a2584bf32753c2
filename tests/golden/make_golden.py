"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the reference checkout (not on the GPU box):

    python tests/golden/make_golden.py /path/to/quail [scenario ...]

Two kinds of fixtures:

- host_<scenario>.npz + .json: the reference's own run_filter
  (quail/backends/quail/executor/loop.py:1535) driven over seeded
  documents with a CPU KVArena and a recording pipeline; every packed
  chunk's arrays (ids, positions, finals, KV scatter, reads, source map,
  unified tables) and the final answers. quail_b200's packer must match
  them bit for bit. host_join_* / host_score_*: the same record of the
  reference's run_join (loop.py:609) over config-2-shaped anchors and
  partners, with 0/1 answers (AI joins) or float32 scores (AI.SCORE).
- host_feed_*: a filter whose survivors feed a join (FilterStream
  hold_survivors as run_join's anchor_source): both streams' chunks in
  launch order, the filter's answers, the admitted anchors and the join's.
- token_store.arrow + .json: a token store file written by the
  reference's TokenStore (the host input format) and its documents.
- kernels.npz: seeded inputs and outputs of the reference's fused Triton
  kernels (add_rms_norm_quant, qk_norm_rope, silu_mul_quant,
  merge_attn_quant, kv_row_scatter; attention.py:293-642) run on CPU
  tensors under TRITON_INTERPRET=1, the quantisers in both scale modes
  (UE8M0=False and True). The oracle must reproduce them.
- requant_ue8m0.npz: block-scaled fp8 weights and their re-quantisation to
  power-of-two scales by vLLM's requant_weight_ue8m0_inplace (the installed
  vllm package, on CPU tensors), the load-time step of the UE8M0 mode.

The reference imports sqlglot at package import; only the SQL frontend
uses it, so an empty stand-in module is installed for the import.
"""

import json
import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def _install_reference(path):
    class _Anything(types.ModuleType):
        def __getattr__(self, name):
            if name.startswith("__"):
                raise AttributeError(name)
            return type(name, (), {})

    stub = _Anything("sqlglot")
    stub.exp = _Anything("sqlglot.exp")
    stub.errors = types.SimpleNamespace(SqlglotError=Exception)
    sys.modules.setdefault("sqlglot", stub)
    sys.modules.setdefault("sqlglot.exp", stub.exp)
    sys.path.insert(0, str(path))


class _Torch:
    """The real torch with CPU-only stand-ins for the CUDA events."""

    def __getattr__(self, name):
        return getattr(torch, name)

    cuda = types.SimpleNamespace(
        Event=lambda **kw: types.SimpleNamespace(record=lambda: None,
                                                 synchronize=lambda: None,
                                                 elapsed_time=lambda other: 0.0),
        synchronize=lambda: None)


def answer_bits(input_ids, positions, finals):
    """The recording pipeline's answers: (token + position) % 2 at each final row."""
    ids = np.asarray(input_ids)
    pos = np.asarray(positions)
    fin = np.asarray(finals)
    return [int(b) for b in (ids[fin] + pos[fin]) % 2]


# ---- host scenarios (shared with tests/test_host_parity.py) ------------------

def scenario_docs(name):
    """(documents, question_ids, budget, n_pages, attention, tree, arena_writes)."""
    rng = np.random.default_rng({"cfg1_tree": 0, "cfg1_unified": 0, "stages_tree": 1,
                                 "stages_unified": 1, "tight_tree": 2, "headers_tree": 3,
                                 "headers_unified": 3, "plain_tree": 4}[name])
    if name.startswith("cfg1") or name.startswith("tight"):
        prefix = rng.integers(1000, 150000, 64).tolist()
        lens = np.clip(rng.lognormal(5.3, 0.6, 40).astype(int), 32, 2048)
        docs = [prefix + rng.integers(1000, 150000, int(n)).tolist() for n in lens]
        questions = [[int(rng.integers(1000, 150000))]]
        budget, pages = 2048 + 64 + 8, 600
        if name.startswith("tight"):
            pages = 130
    elif name.startswith("stages"):
        prefix = rng.integers(1000, 150000, 48).tolist()
        lens = rng.integers(20, 200, 30)
        docs = [prefix + rng.integers(1000, 150000, int(n)).tolist() for n in lens]
        pre = rng.integers(1000, 150000, 3).tolist()
        questions = [pre + [5, 6], pre + [7], pre + [8, 9, 10]]
        budget, pages = 700, 300
    elif name.startswith("headers"):
        headers = [rng.integers(1000, 150000, int(n)).tolist() for n in (16, 40, 70)]
        docs = []
        for _ in range(36):
            h = headers[int(rng.integers(0, 3))]
            body = rng.integers(1000, 150000, int(rng.integers(1, 90))).tolist()
            docs.append(h + body)
        docs.append(list(docs[3]))      # a duplicate document
        questions = [[int(rng.integers(1000, 150000)), 4]]
        budget, pages = 400, 200
    else:  # plain: no prefix tree, no arena writes
        docs = [rng.integers(1000, 150000, int(rng.integers(5, 120))).tolist()
                for _ in range(25)]
        questions = [[17]]
        budget, pages = 300, 64
    attention = "unified" if name.endswith("unified") else "tree"
    tree = name != "plain_tree"
    writes = name != "plain_tree"
    return docs, questions, budget, pages, attention, tree, writes


SCENARIOS = ("cfg1_tree", "cfg1_unified", "stages_tree", "stages_unified", "tight_tree",
             "headers_tree", "headers_unified", "plain_tree")

CHUNK_FIELDS = ("input_ids", "positions", "final_indices", "kv_src", "kv_dst", "cu_a")
READ_FIELDS = ("rows", "cu_q", "used", "table", "source")
UNIFIED_FIELDS = ("src", "dst", "tail_src", "tail_dst", "used", "table", "cu_q")


def _np(x):
    if x is None:
        return None
    if torch.is_tensor(x):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def chunk_record(chunk, arrays, index):
    """Flatten a chunk (reference or quail_b200) into arrays + a JSON entry."""
    meta = chunk.meta
    entry = dict(tokens=int(chunk.tokens), mode=chunk.attention_mode,
                 max_a=int(meta["max_a"]),
                 layout=[[k if isinstance(k, int) else str(k), int(n)]
                         for k, n in chunk.layout])
    for f in CHUNK_FIELDS:
        src = getattr(chunk, f, None) if f in ("input_ids", "positions", "final_indices") \
            else meta[f]
        val = _np(src)
        if val is not None:
            arrays[f"c{index}_{f}"] = val
    reads = meta["reads"]
    entry["reads"] = None
    if reads is not None:
        entry["reads"] = dict(max_q=int(reads["max_q"]), max_used=int(reads["max_used"]))
        for f in READ_FIELDS:
            arrays[f"c{index}_reads_{f}"] = _np(reads[f])
    uni = meta["unified"]
    entry["unified"] = None
    if uni is not None:
        entry["unified"] = dict(max_q=int(uni["max_q"]), max_used=int(uni["max_used"]))
        for f in UNIFIED_FIELDS:
            val = _np(uni[f])
            if val is not None:
                arrays[f"c{index}_unified_{f}"] = val
    return entry


def _cpu_staging(loop):
    """The reference loop's pinned-memory uploads, as plain CPU tensors."""
    def staged(torch_, data, dtype, pinned=True):
        if isinstance(data, np.ndarray) or torch.is_tensor(data):
            return torch.as_tensor(data, dtype=dtype)
        return torch.tensor(data, dtype=dtype)

    def token_parts(torch_, sequences, total, pinned=True, staging=None):
        ids = [int(t) for seq in sequences for part in loop._token_parts(seq) for t in part]
        assert len(ids) == total
        return torch.tensor(ids, dtype=torch.int64)

    loop._staged = staged
    loop._staged_token_parts = token_parts


def run_reference_scenario(name):
    from quail.backends.quail.executor import loop
    from quail.backends.quail.executor.arena import KVArena
    from quail.backends.quail.executor.models.base import ModelPipeline
    from quail.execution.tokens import prefix_tree

    _cpu_staging(loop)
    docs, questions, budget, pages, attention, use_tree, writes = scenario_docs(name)
    arena = KVArena(1, pages, 16, 1, 8, dtype=torch.bfloat16, device="cpu")
    chunks, arrays, entries = [], {}, []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(chunk_record(chunk, arrays, len(entries)))
            return chunk

    class Answers:
        dtype = None

        def submit(self, chunk):
            return answer_bits(chunk.input_ids, chunk.positions, chunk.final_indices)

        def result(self, handle):
            return handle

    tree = prefix_tree(docs, 16) if use_tree else None
    stats = {}
    answers, _, tokens = loop.run_filter(
        _Torch(), arena, Recorder(), Answers(), docs, questions, budget, pinned=False,
        arena_writes=writes, attention_mode=attention, prefix_tree=tree, stats=stats)
    del chunks
    summary = dict(name=name, chunks=entries, tokens=int(tokens),
                   borrowed_tokens=int(stats.get("borrowed_tokens", 0)),
                   answers={str(k): v for k, v in sorted(answers.items())},
                   free_pages_after=int(arena.free_pages),
                   tree=None if tree is None else dict(order=list(map(int, tree.order)),
                                                       parent=tree.parent,
                                                       shared=list(map(int, tree.shared))))
    np.savez_compressed(HERE / f"host_{name}.npz", **arrays)
    (HERE / f"host_{name}.json").write_text(json.dumps(summary, separators=(",", ":")))
    return summary


# ---- join scenarios (run_join, loop.py:609-978) ------------------------------

JOIN_SCENARIOS = ("join_tree", "join_unified", "join_stages_tree", "join_stages_unified",
                  "join_tight_unified", "score_tree", "score_unified", "join_edges_tree",
                  "join_resident_unified")


def join_inputs(name):
    """(anchors, stage_suffixes, frames, partners, budget, n_pages, attention).

    Config 2's shape scaled down: every anchor is a 48-token shared
    instruction + a left document (two-level prefix sharing through the
    prefix tree), partners are right documents; joins frame each stage,
    AI.SCORE streams a per-anchor subset of the partners."""
    seed = {"join_tree": 10, "join_unified": 10, "join_stages_tree": 11,
            "join_stages_unified": 11, "join_tight_unified": 12, "score_tree": 13,
            "score_unified": 13, "join_edges_tree": 16, "join_resident_unified": 17}[name]
    rng = np.random.default_rng(seed)
    instr = rng.integers(1000, 150000, 48).tolist()
    anchors = [instr + rng.integers(1000, 150000, int(rng.integers(20, 100))).tolist()
               for _ in range(10)]
    n_stages = 2 if ("stages" in name or "edges" in name) else 1
    stage_suffixes = [[rng.integers(1000, 150000, int(rng.integers(8, 40))).tolist()
                       for _ in range(12 - 3 * j)] for j in range(n_stages)]
    score = name.startswith("score")
    frames = None if score else [rng.integers(1000, 150000, 3 - j).tolist()
                                 for j in range(n_stages)]
    partners = None
    if score:
        partners = [[sorted(int(i) for i in rng.choice(12, size=int(rng.integers(1, 12)),
                                                        replace=False))]
                    for _ in anchors]
    if "edges" in name:
        # per-anchor partner lists with empty ones: anchor 1 has none at the
        # first stage (settles without a chunk, dropped), anchor 2 none at
        # the last (an empty row once it passes), anchor 3 one partner each
        partners = [[None, None] for _ in anchors]
        partners[1] = [[], None]
        partners[2] = [None, []]
        partners[3] = [[4], [0]]
    budget, pages = 400, 300
    if "tight" in name:
        budget, pages = 500, 40
    # anchors already resident (their prefix KV in the arena): 0, 3, 7
    resident = (0, 3, 7) if "resident" in name else ()
    attention = "unified" if name.endswith("unified") else "tree"
    return anchors, stage_suffixes, frames, partners, budget, pages, attention, resident


def score_values(input_ids, positions, finals):
    """The recording readout's AI.SCORE values: a float32 per final row."""
    ids = np.asarray(input_ids)
    pos = np.asarray(positions)
    fin = np.asarray(finals)
    return ((ids[fin] * 7 + pos[fin]) % 1000).astype(np.float32) / np.float32(1000.0)


def run_reference_join(name):
    from quail.backends.quail.executor import loop
    from quail.backends.quail.executor.arena import KVArena
    from quail.backends.quail.executor.models.base import ModelPipeline
    from quail.execution.tokens import prefix_tree

    _cpu_staging(loop)
    anchors, stage_suffixes, frames, partners, budget, pages, attention, resident = \
        join_inputs(name)
    arena = KVArena(1, pages, 16, 1, 8, dtype=torch.bfloat16, device="cpu")
    frame_max = max(len(f) for f in frames) if frames else 0
    for a in resident:
        assert arena.activate(("a", a), len(anchors[a]),
                              capacity_tokens=len(anchors[a]) + frame_max) is not None
    arrays, entries = {}, []
    score = name.startswith("score")

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(chunk_record(chunk, arrays, len(entries)))
            return chunk

    class Answers:
        dtype = np.float32 if score else None

        def submit(self, chunk):
            f = score_values if score else answer_bits
            return f(chunk.input_ids, chunk.positions, chunk.final_indices)

        def result(self, handle):
            return handle

    keys = [("a", i) for i in range(len(anchors))]
    stats = {}
    answers, _, tokens = loop.run_join(
        _Torch(), arena, Recorder(), Answers(), anchors, stage_suffixes, budget,
        stage_frames=frames, anchor_keys=keys, attention_mode=attention,
        anchor_partners=None if partners is None else (lambda key: partners[key[1]]),
        prefix_tree=prefix_tree(anchors, 16), stats=stats)
    summary = dict(name=name, chunks=entries, tokens=int(tokens),
                   borrowed_tokens=int(stats.get("borrowed_tokens", 0)),
                   answers=[{str(a): [float(x) for x in row] for a, row in sorted(st.items())}
                            for st in answers],
                   free_pages_after=int(arena.free_pages))
    np.savez_compressed(HERE / f"host_{name}.npz", **arrays)
    (HERE / f"host_{name}.json").write_text(json.dumps(summary, separators=(",", ":")))
    return summary


# ---- a filter feeding a join (FilterStream hold_survivors + anchor_source) ----

FEED_SCENARIOS = ("feed_tree", "feed_unified")


def feed_inputs(name):
    """(docs, question, frame, partners, budget, n_pages, attention)."""
    rng = np.random.default_rng(14)
    instr = rng.integers(1000, 150000, 32).tolist()
    docs = [instr + rng.integers(1000, 150000, int(rng.integers(10, 90))).tolist()
            for _ in range(16)]
    question = [int(rng.integers(1000, 150000)), 5]
    frame = rng.integers(1000, 150000, 3).tolist()
    partners = [rng.integers(1000, 150000, int(rng.integers(6, 30))).tolist()
                for _ in range(9)]
    attention = "unified" if name.endswith("unified") else "tree"
    return docs, question, frame, partners, 350, 200, attention


def run_reference_feed(name):
    from quail.backends.quail.executor import loop
    from quail.backends.quail.executor.arena import KVArena
    from quail.backends.quail.executor.models.base import ModelPipeline
    from quail.execution.tokens import prefix_tree

    _cpu_staging(loop)
    docs, question, frame, partners, budget, pages, attention = feed_inputs(name)
    arena = KVArena(1, pages, 16, 1, 8, dtype=torch.bfloat16, device="cpu")
    arrays, entries = {}, []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(chunk_record(chunk, arrays, len(entries)))
            return chunk

    class Answers:
        dtype = None

        def submit(self, chunk):
            return answer_bits(chunk.input_ids, chunk.positions, chunk.final_indices)

        def result(self, handle):
            return handle

    source = loop.FilterStream(
        _Torch(), arena, Recorder(), Answers(), docs, [question], budget, pinned=False,
        arena_writes=True, arena_keys=[("d", i) for i in range(len(docs))],
        hold_survivors=True, hold_extra_tokens=len(frame), prefix_tree=prefix_tree(docs, 16),
        attention_mode=attention)
    keys = []
    answers, _, tokens = loop.run_join(
        _Torch(), arena, Recorder(), Answers(), [], [partners], budget, stage_frames=[frame],
        anchor_keys=keys, anchor_source=source, attention_mode=attention)
    summary = dict(name=name, chunks=entries, tokens=int(tokens),
                   source_tokens=int(source.tokens),
                   filter_answers={str(k): v for k, v in sorted(source.answers.items())},
                   keys=[int(key[1]) for key in keys],
                   answers=[{str(a): [float(x) for x in row] for a, row in sorted(st.items())}
                            for st in answers],
                   free_pages_after=int(arena.free_pages))
    np.savez_compressed(HERE / f"host_{name}.npz", **arrays)
    (HERE / f"host_{name}.json").write_text(json.dumps(summary, separators=(",", ":")))
    return summary


# ---- retention between operators (arena.py:153-226, 541-620; retention.py) ----

RETAIN_SCENARIOS = ("retain_tree", "retain_unified")


def retention_inputs(name):
    """(docs, question, frame, partners, budget, n_pages, attention, config,
    uses, after): a filter whose survivors stay resident, a boundary that
    frees and evicts some, and a join over every survivor whose finished
    matching anchors are retained again."""
    rng = np.random.default_rng(21)
    instr = rng.integers(1000, 150000, 48).tolist()
    docs = [instr + rng.integers(1000, 150000, int(rng.integers(20, 120))).tolist()
            for _ in range(18)]
    question = [int(rng.integers(1000, 150000)), 7]
    frame = rng.integers(1000, 150000, 4).tolist()
    partners = [rng.integers(1000, 150000, int(rng.integers(6, 30))).tolist()
                for _ in range(7)]
    attention = "unified" if name.endswith("unified") else "tree"
    config = {"linear_seconds": 1e-6, "pair_seconds": 3e-9, "cap_pages": 24}
    return (docs, question, frame, partners, 400, 64, attention, config,
            {"d": (0.75, 2)}, {"d": (0.5, 3)})


def arena_state(arena):
    return dict(retained=sorted([list(k) for k in arena.retained_keys()]),
                resident=sorted([list(k) for k in arena.resident_keys()
                                 if isinstance(k, tuple)]),
                retained_pages=int(arena.retained_pages), free_pages=int(arena.free_pages),
                evicted_keys=int(arena.evicted_keys), evicted_pages=int(arena.evicted_pages),
                evicted_prefix_tokens=int(arena.evicted_prefix_tokens))


def run_reference_retention(name):
    from quail.backends.quail.executor import loop
    from quail.backends.quail.executor.arena import KVArena
    from quail.backends.quail.executor.models.base import ModelPipeline
    from quail.backends.quail.retention import apply_retention, retain_after_join
    from quail.execution.tokens import prefix_tree

    _cpu_staging(loop)
    (docs, question, frame, partners, budget, pages, attention, config, uses,
     after) = retention_inputs(name)
    arena = KVArena(1, pages, 16, 1, 8, dtype=torch.bfloat16, device="cpu")
    arena.reset_stats()
    arrays, entries = {}, []

    class Recorder(ModelPipeline):
        tree_attention = True

        def forward_chunk(self, chunk):
            entries.append(chunk_record(chunk, arrays, len(entries)))
            return chunk

    class Answers:
        dtype = None

        def submit(self, chunk):
            return answer_bits(chunk.input_ids, chunk.positions, chunk.final_indices)

        def result(self, handle):
            return handle

    keys = [("d", i) for i in range(len(docs))]
    f_answers, _, f_tokens = loop.run_filter(
        _Torch(), arena, Recorder(), Answers(), docs, [question], budget, pinned=False,
        arena_writes=True, arena_keys=keys, retain_survivors=True, attention_mode=attention,
        prefix_tree=prefix_tree(docs, 16))
    n_filter_chunks = len(entries)
    after_filter = arena_state(arena)
    survivors = sorted(d for d, row in f_answers.items() if row and row[-1])
    apply_retention(arena, config, uses, survivors={"d": survivors[:-2]})
    after_boundary = arena_state(arena)
    anchors = [docs[d] for d in survivors]
    akeys = [keys[d] for d in survivors]

    def anchor_done(a, row):
        if any(row):
            retain_after_join(arena, akeys[a], len(anchors[a]), config, after)
        else:
            arena.free_key(akeys[a])

    j_answers, _, j_tokens = loop.run_join(
        _Torch(), arena, Recorder(), Answers(), anchors, [partners], budget,
        stage_frames=[frame], anchor_keys=akeys, anchor_done=anchor_done,
        attention_mode=attention)
    summary = dict(name=name, chunks=entries, n_filter_chunks=n_filter_chunks,
                   filter_tokens=int(f_tokens), join_tokens=int(j_tokens),
                   filter_answers={str(k): v for k, v in sorted(f_answers.items())},
                   survivors=survivors,
                   join_answers=[{str(a): [float(x) for x in row] for a, row in sorted(st.items())}
                                 for st in j_answers],
                   after_filter=after_filter, after_boundary=after_boundary,
                   after_join=arena_state(arena))
    np.savez_compressed(HERE / f"host_{name}.npz", **arrays)
    (HERE / f"host_{name}.json").write_text(json.dumps(summary, separators=(",", ":")))
    return summary


# ---- token store (quail/execution/tokens.py:180-359) ---------------------------

def make_token_store():
    """token_store.arrow: a store written by the reference's TokenStore.write
    (tokenizer: a fixed text -> ids map), and token_store.json: its
    documents as lists. Also checks that a store written by
    quail_b200.token_store opens in the reference's TokenStore with the
    same documents (recorded as reads_ours)."""
    import tempfile

    import pyarrow as pa
    from quail.execution.tokens import TokenStore as RefStore

    sys.path.insert(0, str(HERE.parent.parent))
    from quail_b200.token_store import write_token_store

    rng = np.random.default_rng(21)
    texts = [" ".join(str(int(x)) for x in rng.integers(1000, 150000, int(n)))
             for n in rng.integers(1, 60, 23)]

    def tokenizer(text):
        return [int(t) for t in text.split()]

    batches = [pa.RecordBatch.from_arrays([pa.array(texts[i:i + 8])], names=["doc"])
               for i in range(0, len(texts), 8)]
    path = HERE / "token_store.arrow"
    store = RefStore.write(str(path), batches, document_column="doc", tokenizer=tokenizer,
                           token_type=pa.int32())
    def as_ints(view):
        return [int(t.as_py()) if hasattr(t, "as_py") else int(t) for t in view]

    docs = [as_ints(store[i]) for i in range(len(store))]
    assert docs == [tokenizer(t) for t in texts]
    with tempfile.TemporaryDirectory() as tmp:
        write_token_store(f"{tmp}/ours.arrow", docs, batch_rows=5)
        ref = RefStore(f"{tmp}/ours.arrow")
        back = [as_ints(ref[i]) for i in range(len(ref))]
        reads_ours = back == docs and list(ref.lengths) == [len(d) for d in docs]
        ref.close()
    store.close()
    (HERE / "token_store.json").write_text(json.dumps(dict(documents=docs,
                                                           reads_ours=reads_ours)))


# ---- kernel vectors ---------------------------------------------------------------

def make_kernel_vectors():
    from quail.backends.quail.executor.attention import Engine

    eng = Engine.__new__(Engine)
    eng.torch = torch
    eng.use_ue8m0 = False
    eng.fp8 = torch.float8_e4m3fn
    eng.is_fp8 = True
    k = eng._triton_kernels()
    g = torch.Generator().manual_seed(7)
    out = {}

    # add_rms_norm_quant: rows x 512, residual updated in place
    n, h = 6, 512
    x = (torch.randn(n, h, generator=g) * 2).to(torch.bfloat16)
    r = torch.randn(n, h, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(h, generator=g)).to(torch.bfloat16)
    out.update(norm_x=x, norm_r_in=r.clone(), norm_w=w)
    r8 = r.clone()
    q = torch.empty(n, h, dtype=torch.float8_e4m3fn)
    s = torch.empty(h // 128, n, dtype=torch.float32).t()
    k["norm"][(n,)](x, r, w, q, s, x.stride(0), r.stride(0), q.stride(0), s.stride(1),
                    s.stride(0), 1e-6, H=h, BLOCK=512, GROUP_C=128, NG=h // 128, UE8M0=False)
    out.update(norm_r_out=r, norm_q=q.view(torch.uint8), norm_s=s.t().contiguous())
    # the same inputs in the UE8M0 scale mode
    q = torch.empty(n, h, dtype=torch.float8_e4m3fn)
    s = torch.empty(h // 128, n, dtype=torch.float32).t()
    k["norm"][(n,)](x, r8, w, q, s, x.stride(0), r8.stride(0), q.stride(0), s.stride(1),
                    s.stride(0), 1e-6, H=h, BLOCK=512, GROUP_C=128, NG=h // 128, UE8M0=True)
    out.update(norm_q_ue8m0=q.view(torch.uint8), norm_s_ue8m0=s.t().contiguous())

    # qk_norm_rope: 4 q heads, 2 kv heads, head 128
    n, qh, kh, d = 5, 4, 2, 128
    qkv = torch.randn(n, (qh + 2 * kh) * d, generator=g).to(torch.bfloat16)
    pos = torch.tensor([0, 3, 17, 100, 127], dtype=torch.int64)
    t = torch.arange(128, dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, dtype=torch.float32) / d))
    f = torch.einsum("i,j->ij", t, inv)
    cs = torch.cat((f.cos(), f.sin()), dim=-1).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    qo = torch.empty(n, qh * d, dtype=torch.bfloat16)
    ko = torch.empty(n, kh * d, dtype=torch.bfloat16)
    k["qk"][(n,)](qkv, qo, ko, cs, pos, qw, kw, qkv.stride(0), qo.stride(0), ko.stride(0),
                  1e-6, QH=qh, KH=kh, HD=d, HALF=d // 2)
    out.update(rope_qkv=qkv, rope_pos=pos, rope_cs=cs, rope_qw=qw, rope_kw=kw, rope_q=qo,
               rope_k=ko)

    # silu_mul_quant: rows x (2 x 1024)
    n, half = 4, 1024
    gu = (torch.randn(n, 2 * half, generator=g) * 3).to(torch.bfloat16)
    q = torch.empty(n, half, dtype=torch.float8_e4m3fn)
    s = torch.empty(half // 128, n, dtype=torch.float32).t()
    k["silu"][(n, half // 512)](gu, q, s, gu.stride(0), q.stride(0), s.stride(1), s.stride(0),
                                HALF=half, GROUP_C=128, GPB=4, UE8M0=False)
    out.update(silu_gu=gu, silu_q=q.view(torch.uint8), silu_s=s.t().contiguous())
    q = torch.empty(n, half, dtype=torch.float8_e4m3fn)
    s = torch.empty(half // 128, n, dtype=torch.float32).t()
    k["silu"][(n, half // 512)](gu, q, s, gu.stride(0), q.stride(0), s.stride(1), s.stride(0),
                                HALF=half, GROUP_C=128, GPB=4, UE8M0=True)
    out.update(silu_q_ue8m0=q.view(torch.uint8), silu_s_ue8m0=s.t().contiguous())

    # merge_attn_quant: 6 rows, 4 heads x 128; rows 1 and 4 read nothing
    n, heads, d = 6, 4, 128
    a = torch.randn(n, heads, d, generator=g).to(torch.bfloat16)
    b = torch.randn(4, heads, d, generator=g).to(torch.bfloat16)
    la = torch.randn(heads, n, generator=g).t()
    lb = torch.randn(heads, 4, generator=g).t()
    src = torch.tensor([0, -1, 1, 2, -1, 3], dtype=torch.int32)
    q = torch.empty(n, heads * d, dtype=torch.float8_e4m3fn)
    s = torch.empty(heads, n, dtype=torch.float32).t()
    k["merge_quant"][(n, heads // 4)](
        a, b, la, lb, src, q, s, a.stride(0), a.stride(1), b.stride(0), b.stride(1),
        la.stride(0), la.stride(1), lb.stride(0), lb.stride(1), q.stride(0), s.stride(1),
        s.stride(0), D=d, GPB=4, UE8M0=False)
    out.update(merge_a=a, merge_b=b, merge_la=la.contiguous(), merge_lb=lb.contiguous(),
               merge_src=src, merge_q=q.view(torch.uint8), merge_s=s.t().contiguous())
    q = torch.empty(n, heads * d, dtype=torch.float8_e4m3fn)
    s = torch.empty(heads, n, dtype=torch.float32).t()
    k["merge_quant"][(n, heads // 4)](
        a, b, la, lb, src, q, s, a.stride(0), a.stride(1), b.stride(0), b.stride(1),
        la.stride(0), la.stride(1), lb.stride(0), lb.stride(1), q.stride(0), s.stride(1),
        s.stride(0), D=d, GPB=4, UE8M0=True)
    out.update(merge_q_ue8m0=q.view(torch.uint8), merge_s_ue8m0=s.t().contiguous())

    # kv_row_scatter: 3 rows into a 10-row pool of 2 x 128
    kk = torch.randn(4, 2, 128, generator=g).to(torch.bfloat16)
    vv = torch.randn(4, 2, 128, generator=g).to(torch.bfloat16)
    kpool = torch.zeros(10, 2, 128, dtype=torch.bfloat16)
    vpool = torch.zeros(10, 2, 128, dtype=torch.bfloat16)
    ssrc = torch.tensor([0, 2, 3], dtype=torch.int64)
    sdst = torch.tensor([9, 0, 5], dtype=torch.int64)
    k["kv_scatter"][(3,)](kk, vv, kpool, vpool, ssrc, sdst, ROW=256, ROW_POW2=256)
    out.update(scat_k=kk, scat_v=vv, scat_src=ssrc, scat_dst=sdst, scat_kpool=kpool,
               scat_vpool=vpool)

    arrays = {}
    for name, val in out.items():
        if val.dtype == torch.bfloat16:
            arrays[name + "__bf16"] = val.contiguous().view(torch.int16).numpy()
        else:
            arrays[name] = val.contiguous().numpy()
    np.savez_compressed(HERE / "kernels.npz", **arrays)


def make_requant_vectors():
    os.environ["TORCHDYNAMO_DISABLE"] = "1"
    from vllm.model_executor.layers.quantization.utils.fp8_utils import (
        requant_weight_ue8m0_inplace,
    )

    g = torch.Generator().manual_seed(11)
    out = {}
    n, k = 384, 512
    # config-1 weights: e4m3(N(0, 1)) codes, lognormal(ln 0.02, 0.3) scales;
    # block (0, 1) all zeros (amax clamped to 1e-4), block (1, 2) holding a
    # +-448 code, block (2, 3) tiny codes only
    w = torch.randn(n, k, generator=g).to(torch.float8_e4m3fn)
    w[0:128, 128:256] = 0
    w[128, 300] = 448.0
    w[256:384, 384:512] = (torch.randn(128, 128, generator=g) * 0.01).to(torch.float8_e4m3fn)
    s = torch.exp(np.log(0.02) + 0.3 * torch.randn(n // 128, k // 128, generator=g))
    s[2, 0] = 2.0 ** -20
    w2, s2 = w.clone(), s.clone()
    requant_weight_ue8m0_inplace(w2, s2, (128, 128))
    out.update(w=w.view(torch.uint8), s=s, w_ue8m0=w2.view(torch.uint8), s_ue8m0=s2)
    np.savez_compressed(HERE / "requant_ue8m0.npz",
                        **{name: val.contiguous().numpy() for name, val in out.items()})


def main():
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QUAIL_REFERENCE", ""))
    if not (ref / "quail").is_dir():
        sys.exit("usage: make_golden.py <reference checkout>")
    _install_reference(ref)
    only = sys.argv[2:]
    for name in SCENARIOS:
        if only and name not in only:
            continue
        summary = run_reference_scenario(name)
        print(name, "chunks", len(summary["chunks"]), "tokens", summary["tokens"])
    for name in JOIN_SCENARIOS:
        if only and name not in only:
            continue
        summary = run_reference_join(name)
        print(name, "chunks", len(summary["chunks"]), "tokens", summary["tokens"])
    for name in FEED_SCENARIOS:
        if only and name not in only:
            continue
        summary = run_reference_feed(name)
        print(name, "chunks", len(summary["chunks"]), "anchors", len(summary["keys"]))
    for name in RETAIN_SCENARIOS:
        if only and name not in only:
            continue
        summary = run_reference_retention(name)
        print(name, "chunks", len(summary["chunks"]), "after join", summary["after_join"])
    if not only or "token_store" in only:
        make_token_store()
        print("token_store.arrow written")
    if not only or "requant" in only:
        make_requant_vectors()
        print("requant_ue8m0.npz written")
    if only and "kernels" not in only:
        return
    make_kernel_vectors()
    print("kernels.npz written")


if __name__ == "__main__":
    main()
