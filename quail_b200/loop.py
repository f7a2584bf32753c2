"""The overlapped filter loop: admit, pack on the CPU, run the GPU, gate.

Same contracts as Quail's chunk loop (quail/backends/quail/executor/
loop.py): ``pack_chunk`` lays out one forward pass's rows and attention
bookkeeping (loop.py:219-577), ``FilterStream`` runs one chunk per
``next()`` and reads the previous chunk's answers while the new one runs
(loop.py:1195-1532), and ``run_filter`` drives it to the end
(loop.py:1535-1559); ``run_join`` streams partner lists against anchors
for AI joins and AI.SCORE (loop.py:609-978). Page indices, scatter maps, block tables, reader
rows, the merge source map and the answer rows are bit-identical to the
reference's for the same inputs.

Packing happens on the host in numpy (``HostChunk``); ``HostChunk.upload``
copies it to the device in one pinned transfer per array. Not built here:
diffusion canvas rows, sliding-window pools and survivor retention
(outside the AI.IF prefill path).
"""

import time
from dataclasses import dataclass, field

import numpy as np

from quail_b200.pack import FilterAdmission, JoinAdmission, partner_pages

ATTENTION_PATHS = ("unified", "tree")
ATTN_TILE = 64   # query rows per attention block


class ArenaFullError(RuntimeError):
    """A chunk's suffix pages do not fit the free KV arena."""


def _tick(timing, key, t0):
    if timing is not None:
        timing[key] = timing.get(key, 0.0) + time.perf_counter() - t0
    return time.perf_counter()


def _cat(parts, dtype=np.int64):
    if not parts:
        return np.empty(0, dtype=dtype)
    return np.concatenate([np.asarray(p, dtype=dtype) for p in parts])


def attention_tiles(cu) -> np.ndarray:
    """int32 [n, 2] (segment, first row) of 64-row query tiles, most work first.

    Work of a tile grows with the keys before it in its segment, so tiles
    sort by descending offset within the segment, then segment order.
    """
    cu = np.asarray(cu, dtype=np.int64)
    starts, ends = cu[:-1], cu[1:]
    counts = np.maximum(0, (ends - starts + ATTN_TILE - 1) // ATTN_TILE)
    seg = np.repeat(np.arange(len(starts)), counts)
    first = np.repeat(np.cumsum(counts) - counts, counts)
    offset = (np.arange(int(counts.sum())) - first) * ATTN_TILE
    rows = starts[seg] + offset
    order = np.lexsort((seg, -offset))
    return np.stack([seg[order], rows[order]], axis=1).astype(np.int32)


class InputStaging:
    """Reused pinned host and device buffers for chunk uploads, one pair per
    array name (Quail's InputStaging, quail/backends/quail/executor/loop.py:
    66-133).

    A chunk's arrays are copied into the pinned host buffer of their name
    (grown when too small) and sent with one asynchronous copy on the
    current stream into the device buffer of that name. The host buffer is
    reused once the event recorded after its last copy has passed, so the
    CPU never overwrites data a transfer still reads; the device buffer is
    reused in stream order, after the kernels of the chunk before. The
    device tensors of an upload are therefore valid until the next upload
    of the same name has run: callers that keep several chunks' inputs
    resident at once (bench.py's prepacked chunks) upload without staging.
    """

    def __init__(self, torch, device="cuda"):
        self.torch = torch
        self.device = device
        self.buffers = {}   # name -> (pinned host, device, event)
        self.h2d_bytes = 0

    def copy(self, name, array, dtype):
        torch = self.torch
        src = torch.from_numpy(np.ascontiguousarray(array).reshape(-1))
        n = src.numel()
        held = self.buffers.get(name)
        if held is not None:
            held[2].synchronize()   # the last transfer from this host buffer is done
        if held is None or held[0].numel() < n or held[0].dtype != dtype:
            size = max(n, 1)
            if held is not None:
                size = max(size, 2 * held[0].numel())
            held = (torch.empty(size, dtype=dtype, pin_memory=True),
                    torch.empty(size, dtype=dtype, device=self.device),
                    torch.cuda.Event())
            self.buffers[name] = held
        host, dev, event = held
        host[:n].copy_(src)
        dev[:n].copy_(host[:n], non_blocking=True)
        event.record()
        self.h2d_bytes += n * host.element_size()
        shape = np.shape(array)
        return dev[:n].view(shape) if len(shape) > 1 else dev[:n]


@dataclass
class Chunk:
    """One packed forward pass (device tensors), Quail's Chunk contract."""

    input_ids: object
    positions: object
    final_indices: object
    meta: dict
    attention_mode: str
    tokens: int
    layout: list
    temporary_keys: tuple = ()
    fresh_keys: tuple = ()
    host: object = None


@dataclass
class HostChunk:
    """A packed chunk as host arrays; the parity tests compare these."""

    input_ids: np.ndarray
    positions: np.ndarray
    final_indices: np.ndarray
    meta: dict
    attention_mode: str
    tokens: int
    layout: list
    temporary_keys: tuple = ()
    fresh_keys: tuple = ()
    h2d_bytes: int = field(default=0)

    def upload(self, torch, device="cuda", staging=None) -> Chunk:
        """Copy every array to the device (non-blocking): through the reused
        pinned buffers of an InputStaging, or, without one, through fresh
        pinned copies that the chunk owns."""
        nbytes = [0]

        def dev(name, a, dtype):
            if a is None:
                return None
            if staging is not None and str(device) != "cpu":
                before = staging.h2d_bytes
                out = staging.copy(name, np.asarray(a), dtype)
                nbytes[0] += staging.h2d_bytes - before
                return out
            t = torch.from_numpy(np.ascontiguousarray(a))
            if t.dtype != dtype:
                t = t.to(dtype)
            nbytes[0] += t.numel() * t.element_size()
            if str(device) == "cpu":
                return t
            return t.pin_memory().to(device, non_blocking=True)

        m = self.meta
        i64, i32 = torch.int64, torch.int32
        meta = dict(layer=0, kv_src=dev("kv_src", m["kv_src"], i64),
                    kv_dst=dev("kv_dst", m["kv_dst"], i64), reads=None, unified=None,
                    canvas=None, cu_a=dev("cu_a", m["cu_a"], i32), max_a=m["max_a"])
        if self.attention_mode == "tree":
            meta["tiles"] = dev("tiles", attention_tiles(m["cu_a"]), i32)
        if m["reads"] is not None:
            r = m["reads"]
            meta["reads"] = dict(
                rows=dev("reads.rows", r["rows"], i64), cu_q=dev("reads.cu_q", r["cu_q"], i32),
                max_q=r["max_q"], used=dev("reads.used", r["used"], i32),
                max_used=r["max_used"], table=dev("reads.table", r["table"], i32),
                source=dev("reads.source", r["source"], i32))
        if m["unified"] is not None:
            u = m["unified"]
            meta["unified"] = dict(
                src=dev("unified.src", u["src"], i64), dst=dev("unified.dst", u["dst"], i64),
                tail_src=dev("unified.tail_src", u["tail_src"], i64),
                tail_dst=dev("unified.tail_dst", u["tail_dst"], i64),
                used=dev("unified.used", u["used"], i32),
                table=dev("unified.table", u["table"], i32),
                max_used=u["max_used"], cu_q=dev("unified.cu_q", u["cu_q"], i32),
                max_q=u["max_q"], tiles=dev("unified.tiles", attention_tiles(u["cu_q"]), i32))
        chunk = Chunk(
            input_ids=dev("input_ids", self.input_ids, i64),
            positions=dev("positions", self.positions, i64),
            final_indices=dev("final_indices", self.final_indices, i64),
            meta=meta, attention_mode=self.attention_mode, tokens=self.tokens,
            layout=self.layout, temporary_keys=self.temporary_keys,
            fresh_keys=self.fresh_keys, host=self)
        self.h2d_bytes = nbytes[0]
        return chunk


class _Pool:
    """Scatter map, block table rows and lengths of the unified paged call."""

    def __init__(self):
        self.page_rows, self.lengths = [], []
        self.src, self.dst, self.tail_src, self.tail_dst = [], [], [], []

    def sequence(self, pages, kv_tokens):
        self.page_rows.append(list(pages))
        self.lengths.append(kv_tokens)

    def direct(self, rows, r0, r1, logical_start):
        if r0 >= r1:
            return
        self.src.append(np.arange(r0, r1, dtype=np.int64))
        self.dst.append(rows[logical_start:logical_start + (r1 - r0)])

    def suffix(self, pages, temp_rows, s0, s1, f, remainder, page_tokens):
        self.src.append(np.arange(s0, s1, dtype=np.int64))
        self.dst.append(temp_rows[remainder:remainder + (s1 - s0)])
        if remainder:
            base = pages[f // page_tokens] * page_tokens
            self.tail_src.append(np.arange(base, base + remainder, dtype=np.int64))
            self.tail_dst.append(temp_rows[:remainder])

    def build(self, arena):
        return dict(src=_cat(self.src), dst=_cat(self.dst),
                    tail_src=_cat(self.tail_src) if self.tail_src else None,
                    tail_dst=_cat(self.tail_dst) if self.tail_dst else None,
                    used=np.asarray(self.lengths, dtype=np.int32),
                    table=arena.block_table_rows(self.page_rows),
                    max_used=max(self.lengths))


def pack_chunk(arena, groups, *, attention_mode, timing=None) -> HostChunk:
    """Lay out one chunk from groups in chunk order (see Quail's pack_chunk).

    Each group: key, prefix (fresh token ids or None when the KV is
    resident), start (borrowed positions before the prefix), read_key (the
    parent a single-suffix borrower reads under tree attention), f (where
    suffix positions start), suffixes, write_suffix_tokens.
    """
    if attention_mode not in ATTENTION_PATHS:
        raise ValueError(f"attention_mode must be one of {ATTENTION_PATHS}, "
                         f"got {attention_mode!r}")
    t = time.perf_counter() if timing is not None else 0.0
    tree = attention_mode == "tree"
    ids, pos = [], []
    count = 0
    cu_a, finals = [0], []
    reader_spans = []            # (first row, end row) of rows reading resident KV
    kv_writes, layout, fresh_keys = [], [], []
    read_keys, read_used, cu_q = [], [], [0]
    max_q = 0
    unified_groups = []
    for g in groups:
        prefix = g.get("prefix")
        fresh = prefix is not None
        f, key = g["f"], g["key"]
        start = g.get("start", 0)
        suffixes = g["suffixes"]
        paged = arena.is_resident(key)
        row0 = count
        borrowing = bool(fresh and start and tree)
        stacked = borrowing and len(suffixes) == 1 and g.get("read_key") is not None
        if fresh:
            if not paged and len(suffixes) > 1:
                raise ValueError(f"group {key!r}: an unpaged fresh group packs "
                                 f"[prefix | suffix] as one causal segment")
            if start and not paged:
                raise ValueError(f"group {key!r}: a borrowed prefix needs arena pages")
            ids.append(prefix)
            count += len(prefix)
            pos.append(np.arange(start, start + len(prefix), dtype=np.int64))
            if (paged or not suffixes) and not stacked:
                cu_a.append(count)
            if borrowing and not stacked:
                reader_spans.append((row0, count))
                cu_q.append(cu_q[-1] + count - row0)
                read_keys.append(key)
                read_used.append(start)
                max_q = max(max_q, count - row0)
            if paged and tree:
                kv_writes.append((key, row0, row0 + len(prefix), start))
                fresh_keys.append(key)
        prefix_end = count
        s_row0 = count
        spans = []
        for si, suf in enumerate(suffixes):
            srow = count
            ids.append(suf)
            count += len(suf)
            pos.append(np.arange(f, f + len(suf), dtype=np.int64))
            finals.append(count - 1)
            spans.append((srow, count))
            cu_a.append(count)
            wst = g.get("write_suffix_tokens", 0)
            if si == 0 and wst and paged and tree:
                dest = start + len(prefix) if fresh else f
                kv_writes.append((key, srow, srow + wst, dest))
        s_count = count - s_row0
        layout.append((key, len(suffixes)))
        if stacked:
            n = count - row0
            reader_spans.append((row0, count))
            read_key = g["read_key"]
            if read_keys and read_keys[-1] == read_key and read_used[-1] == start:
                cu_q[-1] += n
                max_q = max(max_q, cu_q[-1] - cu_q[-2])
            else:
                cu_q.append(cu_q[-1] + n)
                read_keys.append(read_key)
                read_used.append(start)
                max_q = max(max_q, n)
        elif s_count and f and paged and tree:
            reader_spans.append((s_row0, count))
            cu_q.append(cu_q[-1] + s_count)
            read_keys.append(key)
            read_used.append(f)
            max_q = max(max_q, s_count)
        if attention_mode == "unified":
            if paged:
                unified_groups.append(dict(key=key, fresh=fresh, f=f, row0=row0, start=start,
                                           prefix_end=prefix_end, row1=count, spans=spans))
            elif not fresh:
                raise ValueError("unified attention requires pages for a kept group")
    t = _tick(timing, "pack_py", t)

    reads = None
    if read_keys:
        table, _ = arena.block_table(read_keys)
        rows = _cat([np.arange(a, b, dtype=np.int64) for a, b in reader_spans])
        source = np.full(count, -1, dtype=np.int32)
        source[rows] = np.arange(len(rows), dtype=np.int32)
        reads = dict(rows=rows, cu_q=np.asarray(cu_q, dtype=np.int32), max_q=max_q,
                     used=np.asarray(read_used, dtype=np.int32), max_used=max(read_used),
                     table=table, source=source)
    t = _tick(timing, "pack_reads", t)

    unified = None
    temporary_keys = []
    if attention_mode == "unified" and unified_groups:
        if len(unified_groups) != len(layout):
            raise ValueError("a unified chunk cannot mix paged and unpaged groups")
        pool = _Pool()
        ucu = [0]
        pt = arena.page_tokens
        try:
            for spec in unified_groups:
                key, f = spec["key"], spec["f"]
                r0, r1, spans = spec["row0"], spec["row1"], spec["spans"]
                logical_start = spec["start"] if spec["fresh"] else f
                if spec["fresh"]:
                    fresh_keys.append(key)
                rows = arena.capacity_rows(key)
                pages = arena.owned_pages(key)
                n = r1 - r0
                if len(spans) == 1 and logical_start + n <= len(rows):
                    pool.direct(rows, r0, r1, logical_start)
                    pool.sequence(pages, f + sum(e - s for s, e in spans))
                    ucu.append(ucu[-1] + n)
                    continue
                prefix_count = spec["prefix_end"] - r0
                if prefix_count:
                    pool.direct(rows, r0, spec["prefix_end"], spec["start"])
                    pool.sequence(pages[:arena.pages_needed(f)], f)
                    ucu.append(ucu[-1] + prefix_count)
                for s0, s1 in spans:
                    remainder = f % pt
                    got = arena.alloc_temporary(remainder + (s1 - s0))
                    if got is None:
                        raise ArenaFullError(
                            f"unified suffix pages exceed the free KV arena (asked "
                            f"{remainder + s1 - s0} rows; free pages {arena.free_pages})")
                    temp_key = got[0]
                    temporary_keys.append(temp_key)
                    pool.suffix(pages, arena.capacity_rows(temp_key), s0, s1, f, remainder, pt)
                    pool.sequence(pages[:f // pt] + arena.owned_pages(temp_key),
                                  f + (s1 - s0))
                    ucu.append(ucu[-1] + (s1 - s0))
            built = pool.build(arena)
            unified = dict(built, cu_q=np.asarray(ucu, dtype=np.int32),
                           max_q=int(np.diff(ucu).max()))
        except Exception:
            for key in temporary_keys:
                arena.free_key(key)
            raise

    kv_src = kv_dst = None
    if kv_writes:
        src, dst = [], []
        for key, r0, r1, dest in kv_writes:
            src.append(np.arange(r0, r1, dtype=np.int64))
            rows = arena.capacity_rows(key)[dest:dest + (r1 - r0)]
            if len(rows) != r1 - r0:
                raise AssertionError("KV write exceeds reserved rows")
            dst.append(rows)
        kv_src, kv_dst = _cat(src), _cat(dst)
    t = _tick(timing, "pack_kv", t)

    cu = np.asarray(cu_a, dtype=np.int32)
    meta = dict(layer=0, kv_src=kv_src, kv_dst=kv_dst, reads=reads, unified=unified,
                canvas=None, cu_a=cu, max_a=int(np.diff(cu).max()))
    out = HostChunk(input_ids=_cat(ids), positions=_cat(pos),
                    final_indices=np.asarray(finals, dtype=np.int64), meta=meta,
                    attention_mode=attention_mode, tokens=count, layout=layout,
                    temporary_keys=tuple(temporary_keys), fresh_keys=tuple(fresh_keys))
    _tick(timing, "pack_arrays", t)
    return out


def attention_path(pipeline, requested, default="unified") -> str:
    """The plan's attention path where the model has it (loop.py:580-590)."""
    if requested is None:
        requested = default
    if requested == "tree" and pipeline.tree_attention:
        return "tree"
    return "unified"


def _forward(pipeline, arena, chunk):
    try:
        return pipeline.forward_chunk(chunk)
    finally:
        keys, chunk.temporary_keys = chunk.temporary_keys, ()
        for key in keys:
            arena.free_key(key)


def _shared_preamble_tokens(question_ids):
    if len(question_ids) < 2:
        return 0
    p = 0
    while all(len(q) > p and q[p] == question_ids[0][p] for q in question_ids):
        p += 1
    return p


def borrow_check(arena, keys, borrowing):
    """can_borrow for Borrowing: the arena still holds the parent's pages."""
    def can_borrow(doc, parent, same_chunk):
        shared = borrowing.tree_shared[doc]
        if not same_chunk or arena.is_resident(keys[parent]):
            return arena.can_borrow(keys[parent], shared)
        return True
    return can_borrow


def lowest_borrows(borrowing):
    lowest = {}
    for doc, parent in enumerate(borrowing.tree_parent):
        if parent is not None:
            shared = borrowing.tree_shared[doc]
            lowest[parent] = min(lowest.get(parent, shared), shared)
    return lowest


class FilterStream:
    """The filter chain, one chunk per next() call (Quail's FilterStream).

    Args:
        torch: the torch module.
        arena: KVArena of the documents' KV pages.
        pipeline: the model pipeline; forward_chunk(chunk) -> normed rows.
        async_ans: readout with submit(normed) -> handle and result(handle).
        doc_ids: per-document token sequences.
        question_ids: per-stage question token lists.
        budget: chunk token budget.
        arena_writes: whether document KV is written to the arena.
        arena_keys: stable arena key per document (positions by default).
        attention_mode: "tree" or "unified".
        prefix_tree: PrefixTree over doc_ids, or None.
        limit: stop admitting after this many survivors.
        device: where chunks are uploaded ("cuda" or "cpu" for host tests).
        staging: an InputStaging whose pinned buffers the uploads reuse, or
            None for fresh pinned copies per chunk (needed when the caller
            keeps several chunks' device inputs at once).
    """

    def __init__(self, torch, arena, pipeline, async_ans, doc_ids, question_ids, budget,
                 timing=None, limit=None, *, arena_writes, arena_keys=None,
                 retain_survivors=(), hold_survivors=False, hold_extra_tokens=0,
                 attention_mode=None, document_done=None, prefix_tree=None,
                 device="cuda", on_chunk=None, staging=None):
        p = _shared_preamble_tokens(question_ids)
        keys = range(len(doc_ids)) if arena_keys is None else arena_keys
        if len(keys) != len(doc_ids):
            raise ValueError("arena_keys must match doc_ids")
        # retain_survivors: True, or the document positions whose KV stays
        # resident (rewound to the document) after a last-stage TRUE
        retain_all = retain_survivors is True
        retain = set() if retain_all else set(retain_survivors)
        if hold_survivors and (retain_all or retain):
            raise ValueError("held survivors are pinned, not retained")
        stage_tokens = [len(question_ids[0])] + [len(q) - p for q in question_ids[1:]]
        tails = [list(question_ids[0])] + [list(q[p:]) for q in question_ids[1:]]
        for i, tail in enumerate(tails):
            if not tail:
                raise ValueError(f"stage {i} question has no tokens beyond the shared "
                                 f"preamble ({p} tokens)")
        if not arena_writes and (len(question_ids) > 1 or retain_all or retain
                                 or hold_survivors):
            raise ValueError("arena_writes=False needs a single stage")
        self.attention_mode = attention_path(pipeline, attention_mode)
        unified = self.attention_mode == "unified"
        if prefix_tree is not None and prefix_tree.shared_tokens:
            if not arena_writes:
                raise ValueError("a prefix tree needs arena writes")
        else:
            prefix_tree = None
        temp_tail = max(0, *(len(q) - p for q in question_ids)) if unified and arena_writes \
            else 0
        capacity_extra = p + temp_tail
        if hold_survivors:
            # a held document's pages cover the consumer's largest frame
            capacity_extra = max(capacity_extra, hold_extra_tokens)
        if arena.retention_cap_pages is None:
            arena.retention_cap_pages = max(0, arena.n_pages - arena.pages_needed(2 * budget))
        self.sched = FilterAdmission(
            [len(d) for d in doc_ids], stage_tokens, budget,
            arena_pages=arena.n_pages if arena_writes else None,
            page_tokens=arena.page_tokens, kept_extra_tokens=capacity_extra, limit=limit,
            page_cost=arena.page_cost, tree=prefix_tree)
        borrowing = self.sched.borrowing
        borrowing.can_borrow = borrow_check(arena, keys, borrowing)
        self.tree = prefix_tree
        self.tree_position = ({doc: i for i, doc in enumerate(prefix_tree.order)}
                              if prefix_tree is not None else {})
        self.borrowers = borrowing.borrowers()
        self.lowest_borrow = lowest_borrows(borrowing)
        self.torch = torch
        self.arena = arena
        self.pipeline = pipeline
        self.async_ans = async_ans
        self.doc_ids = doc_ids
        self.keys = keys
        self.timing = timing
        self.arena_writes = arena_writes
        self.hold = hold_survivors
        self.retain_all = retain_all
        self.retain = retain
        self.reserve_pages = 0  # pages a join consumer needs free for its partners
        self.preamble = p
        self.capacity_extra = capacity_extra
        self.tails = tails
        self.device = device
        self.staging = staging
        self.on_chunk = on_chunk
        self.spans = []
        self.tokens = 0
        self.chunks = 0
        self.h2d_bytes = 0
        self.done = False
        self.outstanding = []
        self.document_done = document_done

    @property
    def answers(self):
        return self.sched.answers

    def _spec(self, doc, stage, fresh):
        if fresh:
            borrowing = self.sched.borrowing
            shared = borrowing.shared(doc)
            prefix = self.doc_ids[doc]
            read_key = None
            if shared:
                prefix = prefix[shared:]
                read_key = self.keys[borrowing.parent(doc)]
            return dict(key=self.keys[doc], prefix=prefix, start=shared, read_key=read_key,
                        f=len(self.doc_ids[doc]), suffixes=[self.tails[0]],
                        write_suffix_tokens=self.preamble)
        return dict(key=self.keys[doc], prefix=None, f=len(self.doc_ids[doc]) + self.preamble,
                    suffixes=[self.tails[stage]])

    def set_reserve(self, pages):
        """Leave pages free for a join consumer's partner rows."""
        for doc, ids in enumerate(self.doc_ids):
            if self.arena.page_cost(len(ids) + self.capacity_extra) + pages > self.arena.n_pages:
                raise ValueError(f"document {doc} needs more pages than the arena holds "
                                 f"beside the join's {pages} pages of partner rows")
        self.reserve_pages = pages

    def _activate(self, doc):
        borrowing = self.sched.borrowing
        key = self.keys[doc]
        shared = borrowing.shared(doc)
        n = len(self.doc_ids[doc])
        got = self.arena.activate(
            key, n + self.preamble, capacity_tokens=n + self.capacity_extra, base_tokens=n,
            borrow=((self.keys[borrowing.parent(doc)], shared) if shared else None))
        assert got is not None, "scheduler admitted a doc the arena cannot hold"
        if self.borrowers[doc]:
            self.arena.hold(key, self.borrowers[doc])
            self.arena.keep_window(key, self.lowest_borrow[doc])

    def _report(self, entry, items):
        t = time.perf_counter() if self.timing is not None else 0.0
        groups, handle = entry
        bits = self.async_ans.result(handle)
        t = _tick(self.timing, "report_wait", t)
        last_stage = len(self.tails) - 1
        finished = []
        for (doc, stage, _fresh), bit in zip(groups, bits):
            passed = bool(bit)
            last = stage == last_stage
            # a retained survivor stays resident for a later operator; a
            # held one keeps its pages for the join consumer, which frees them
            keep = passed and last and (self.retain_all or doc in self.retain)
            hold = passed and last and self.hold
            for d in self.sched.report(doc, stage, passed, release=not (keep or hold)):
                self.arena.free_key(self.keys[d])
            if keep:
                self.arena.retain(self.keys[doc], len(self.doc_ids[doc]))
            if hold:
                items.append((self.keys[doc], self.doc_ids[doc]))
            if not passed or stage == last_stage:
                finished.append((doc, stage, passed))
        if finished and self.document_done is not None:
            self.document_done(finished)
        _tick(self.timing, "report_rest", t)

    def _finish(self, items):
        while self.outstanding:
            self._report(self.outstanding.pop(0), items)
        for doc in self.sched.drain_ready():
            self.arena.free_key(self.keys[doc])
        self.arena.drop_holds([self.keys[doc] for doc, n in enumerate(self.borrowers) if n])
        self.done = True

    def next(self, evict_retained=False):
        """Run one chunk; reads the previous chunk's answers while it runs.

        Returns (held, blocked) as Quail's FilterStream.next (loop.py:
        1438-1532): the (key, prefix) pairs of survivors handed over with
        their KV (hold_survivors), and whether fresh admission is short of
        pages that only the join consumer can free."""
        items = []
        if self.done:
            return items, False
        sched, arena, timing = self.sched, self.arena, self.timing
        while True:
            if sched.done():
                self._finish(items)
                return items, False
            free = (max(0, arena.free_pages - self.reserve_pages) if self.arena_writes
                    else None)
            t = time.perf_counter() if timing is not None else 0.0
            groups = sched.next_chunk(free)
            t = _tick(timing, "next_chunk", t)
            if groups:
                break
            if self.outstanding:
                self._report(self.outstanding.pop(0), items)
                continue
            if sched.blocked_pages and (evict_retained or not self.hold):
                if arena.evict_retained(sched.blocked_pages):
                    continue
            if self.hold and sched.blocked_pages and not evict_retained:
                return items, True  # the consumer frees pages first
            if arena.drop_holds([self.keys[doc] for doc, n in enumerate(self.borrowers) if n]):
                continue
            if self.hold and sched.blocked_pages:
                return items, True
            raise AssertionError("nothing buildable and nothing in flight")
        if self.tree is not None and self.attention_mode != "unified":
            def borrow_order(group):
                doc, _, fresh = group
                if not fresh:
                    return (False, -1, 0)
                parent = sched.borrowing.parent(doc)
                return (True, self.tree_position[doc if parent is None else parent],
                        sched.borrowing.shared(doc))
            groups.sort(key=borrow_order)
        fresh_docs = [doc for doc, _, fresh in groups if fresh]
        if self.arena_writes:
            for doc in fresh_docs:
                self._activate(doc)
        t = _tick(timing, "alloc", t)
        host = pack_chunk(arena, [self._spec(*g) for g in groups],
                          attention_mode=self.attention_mode, timing=timing)
        for doc in fresh_docs:
            parent = sched.borrowing.tree_parent[doc]
            if parent is not None:
                arena.release(self.keys[parent])
        chunk = host.upload(self.torch, self.device, self.staging)
        self.h2d_bytes += host.h2d_bytes
        if self.on_chunk is not None:
            self.on_chunk(host, groups)
        t = _tick(timing, "pack", t)
        self.tokens += chunk.tokens
        e0 = e1 = None
        if self.device != "cpu":
            e0 = self.torch.cuda.Event(enable_timing=True)
            e1 = self.torch.cuda.Event(enable_timing=True)
            e0.record()
        normed = _forward(self.pipeline, arena, chunk)
        if e1 is not None:
            e1.record()
        if self.arena_writes:
            for doc in fresh_docs:
                arena.trim_window(self.keys[doc])
        t = _tick(timing, "forward_launch", t)
        self.spans.append((0, e0, e1))
        self.outstanding.append((groups, self.async_ans.submit(normed)))
        self.chunks += 1
        _tick(timing, "submit", t)
        while len(self.outstanding) > 1:
            self._report(self.outstanding.pop(0), items)
        return items, bool(self.hold and sched.blocked_pages)


def run_filter(torch, arena, pipeline, async_ans, doc_ids, question_ids, budget, timing=None,
               limit=None, *, arena_writes, arena_keys=None, retain_survivors=(),
               attention_mode=None, document_done=None, prefix_tree=None, stats=None,
               device="cuda", on_chunk=None, staging=None):
    """The filter chain run to the end; see FilterStream for the arguments.

    Returns:
        (answers, spans, tokens): answers[d] is the 0/1 list up to the first
        FALSE; spans the per-chunk CUDA event pairs; tokens the fresh tokens.
    """
    stream = FilterStream(torch, arena, pipeline, async_ans, doc_ids, question_ids, budget,
                          timing=timing, limit=limit, arena_writes=arena_writes,
                          arena_keys=arena_keys, retain_survivors=retain_survivors,
                          attention_mode=attention_mode, document_done=document_done,
                          prefix_tree=prefix_tree, device=device, on_chunk=on_chunk,
                          staging=staging)
    while not stream.done:
        stream.next()
    if stats is not None:
        stats["borrowed_tokens"] = stream.sched.borrowing.borrowed_tokens
        stats["h2d_bytes"] = stream.h2d_bytes
        stats["chunks"] = stream.chunks
    return stream.answers, stream.spans, stream.tokens


def run_join(torch, arena, pipeline, async_ans, anchor_prefixes, stage_suffixes, budget,
             stage_frames=None, anchor_keys=None, anchor_done=None, anchor_source=None,
             anchor_partners=None, anchor_batch=None, attention_mode=None, prefix_tree=None,
             stats=None, device="cuda", on_chunk=None, stop_at_true=False, stream_step=None,
             staging=None):
    """Stream partner lists against anchors, gating survivors between stages
    (Quail's run_join, loop.py:609-978; arguments as there).

    Each chunk packs anchors' prefixes (fresh anchors; a tree borrower only
    past its shared tokens), the stage frame written after the anchor's
    document rows (a frame entry, whose answer is skipped) and runs of
    partner suffixes read against the anchor's kept KV. The readout's dtype
    picks the answer rows: None for 0/1 lists (AI joins), float32 arrays for
    AI.SCORE. With anchor_source (a FilterStream with hold_survivors), the
    filter's survivors stream in as resident anchors between join chunks.
    With stop_at_true (an EXISTS join; the reference has no such stop and
    scores every partner), an anchor's last-stage partners that are not yet
    launched when one of its partners answers TRUE are skipped: its row
    then ends after the launched ones, and which anchors have a TRUE is
    unchanged. stream_step caps the partners one anchor launches per chunk,
    so with a small step the anchors' streams interleave and a TRUE arrives
    before most of its anchor's stream is packed.

    Returns:
        (answers, spans, tokens): answers[j][a] is anchor a's row over the
        stage-j partners it streams; spans (stage, start, end) CUDA events
        per forward; tokens the fresh tokens packed.
    """
    if tuple(getattr(pipeline, "canvas_ids", ()) or ()):
        raise NotImplementedError("run_join: diffusion canvas rows are not built here")
    k = len(stage_suffixes)
    if anchor_source is not None:
        # the source hands over resident anchors; the join appends them
        if anchor_prefixes or anchor_keys:
            raise ValueError("anchor_source fills anchor_prefixes and anchor_keys")
        prefixes, keys = anchor_prefixes, anchor_keys
    else:
        prefixes = list(anchor_prefixes)
        keys = list(range(len(prefixes))) if anchor_keys is None else list(anchor_keys)
    if len(keys) != len(prefixes):
        raise ValueError("anchor_keys must match anchor_prefixes")
    frames = stage_frames or [[] for _ in range(k)]
    mode = attention_path(pipeline, attention_mode, default="tree")
    if k == 0:
        return [], [], 0
    frame_max = max(len(f) for f in frames)
    if anchor_source is not None and mode == "unified":
        # the source leaves room for one partner's temporary rows, or held
        # anchors could fill the arena before the join can run
        longest = [max((len(x) for x in sufs), default=0) for sufs in stage_suffixes]
        anchor_source.set_reserve(max(
            (partner_pages(arena.page_cost, arena.page_tokens, len(doc), len(frame), rows)
             for doc in anchor_source.doc_ids for frame, rows in zip(frames, longest)),
            default=0))

    def entry_rows(a, j, start, end, carried):
        rows = (len(prefixes[a]) if carried else 0) + sum(
            len(stage_suffixes[j][i]) for i in sched.partner_indices(a, j, start, end))
        if frames[j] and start == 0:
            rows += len(frames[j])
        return rows

    def held_pages(key, prefix_tokens):
        capacity = prefix_tokens + frame_max
        return arena.page_cost(capacity) - arena.growth_cost(key, capacity)

    resident = {a: held_pages(keys[a], len(prefixes[a]))
                for a in range(len(keys)) if arena.is_resident(keys[a])}
    for a in resident:
        arena.pin(keys[a])
    if prefix_tree is not None and not prefix_tree.shared_tokens:
        prefix_tree = None
    partners_of = (lambda key: None) if anchor_partners is None else anchor_partners
    sched = JoinAdmission(
        [len(p) for p in prefixes], [[len(s) for s in sufs] for sufs in stage_suffixes],
        budget, arena.n_pages, arena.page_tokens, frame_tokens=[len(f) for f in frames],
        resident=resident, anchor_partners={a: partners_of(keys[a]) for a in range(len(keys))},
        temporary_suffix_pages=mode == "unified", answer_dtype=async_ans.dtype,
        page_cost=arena.page_cost, tree=prefix_tree, stop_at_true=stop_at_true,
        stream_step=stream_step)
    borrowing = sched.borrowing
    borrowing.can_borrow = borrow_check(arena, keys, borrowing)
    borrowers = borrowing.borrowers()
    lowest_borrow = lowest_borrows(borrowing)
    held = [keys[a] for a, n in enumerate(borrowers) if n]
    spans, outstanding = [], []
    tokens = 0
    h2d = [0, 0]  # bytes, chunks

    def admit(items):
        if anchor_batch is not None and items:
            kept = set(anchor_batch([key for key, _ in items]))
            for key, _ in items:
                if key not in kept and arena.is_resident(key):
                    arena.free_key(key)
            items = [(key, prefix) for key, prefix in items if key in kept]
        for key, prefix in items:
            if not arena.is_resident(key):
                raise ValueError(f"streamed anchor {key!r} has no KV in the arena")
            arena.pin(key)
            keys.append(key)
            prefixes.append(prefix)
            sched.admit(len(prefix), held_pages(key, len(prefix)), partners=partners_of(key))

    def pull(evict_retained=False, force=False):
        """Source chunks until a join chunk can fill or the source blocks;
        whether the source ran a chunk or handed an anchor over."""
        moved = False
        while not anchor_source.done and (force or sched.buildable_tokens() < budget):
            force = False
            before = anchor_source.chunks
            items, blocked = anchor_source.next(evict_retained=evict_retained)
            admit(items)
            moved = moved or bool(items) or anchor_source.chunks > before
            if blocked:
                break
        return moved

    def build(part):
        specs = []
        for a, j, start, end, carried in part:
            key, f, frame = keys[a], len(prefixes[a]), frames[j]
            parent, shared = ((borrowing.parent(a), borrowing.shared(a)) if carried
                              else (None, 0))
            fresh = not arena.is_resident(key)
            got = arena.activate(key, f, capacity_tokens=f + frame_max, base_tokens=f,
                                 borrow=(keys[parent], shared) if shared else None)
            assert got is not None, "scheduler admitted an anchor the arena cannot hold"
            if fresh and a < len(borrowers) and borrowers[a]:
                arena.hold(key, borrowers[a])
                arena.keep_window(key, lowest_borrow[a])
            prefix = None
            if carried:
                prefix = prefixes[a][shared:] if shared else prefixes[a]
            sufs = [stage_suffixes[j][i] for i in sched.partner_indices(a, j, start, end)]
            if frame and start == 0:
                # the frame goes into the anchor's KV after its document rows
                # (this entry's answer means nothing); the partners read both
                specs.append(dict(key=key, prefix=prefix, start=shared, f=f, suffixes=[frame],
                                  write_suffix_tokens=len(frame)))
                specs.append(dict(key=key, prefix=None, f=f + len(frame), suffixes=sufs))
            else:
                specs.append(dict(key=key, prefix=prefix, start=shared, f=f + len(frame),
                                  suffixes=sufs))
        return pack_chunk(arena, specs, attention_mode=mode)

    def settle(anchor):
        if anchor_done is None:
            if arena.is_resident(keys[anchor]):
                arena.free_key(keys[anchor])
        else:
            anchor_done(anchor, sched.answers[k - 1].get(anchor, []))

    def event(kind, anchor):
        if kind == "finished":
            settle(anchor)
        elif arena.is_resident(keys[anchor]):
            arena.free_key(keys[anchor])

    def report(entry):
        part, handle = entry
        bits = async_ans.result(handle)
        pos = 0
        for a, j, start, end, _ in part:
            if frames[j] and start == 0:
                pos += 1
            for kind, anchor in sched.report(a, j, start, end, bits[pos:pos + end - start]):
                event(kind, anchor)
            pos += end - start

    def run_one(part):
        nonlocal tokens
        host = build(part)
        chunk = host.upload(torch, device, staging)
        h2d[0] += host.h2d_bytes
        h2d[1] += 1
        if on_chunk is not None:
            on_chunk(host, part)
        tokens += chunk.tokens
        e0 = e1 = None
        if device != "cpu":
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
        normed = _forward(pipeline, arena, chunk)
        if e1 is not None:
            e1.record()
        for key in chunk.fresh_keys:
            arena.trim_window(key)
        spans.append((part[0][1], e0, e1))
        outstanding.append((part, async_ans.submit(normed)))
        while len(outstanding) > 1:
            report(outstanding.pop(0))

    def run_part(part):
        # a chunk whose temporary suffix pages do not fit (the packer takes
        # them a page at a time) is retried after evicting retained KV, or
        # halved
        try:
            run_one(part)
        except ArenaFullError:
            need = arena.page_cost(sum(entry_rows(*e) for e in part))
            if arena.evict_retained(need):
                run_part(part)
                return
            if len(part) < 2:
                raise
            half = len(part) // 2
            run_part(part[:half])
            run_part(part[half:])

    while True:
        if anchor_source is not None and not anchor_source.done:
            pull()
        for kind, anchor in sched.take_settled():
            event(kind, anchor)
        if sched.done() and (anchor_source is None or anchor_source.done):
            break
        if sched.blocked_pages:
            arena.evict_retained(sched.blocked_pages)
        groups = sched.next_chunk(arena.free_pages)
        if not groups:
            if outstanding:
                report(outstanding.pop(0))
                continue
            if anchor_source is not None and not anchor_source.done:
                # the source has to move; it may evict retained KV to admit
                if pull(evict_retained=True, force=True):
                    continue
            if sched.blocked_pages and arena.evict_retained(sched.blocked_pages):
                continue
            if arena.drop_holds(held):
                continue
            raise AssertionError("nothing buildable and nothing in flight")
        run_part(groups)
        # the packed children hold their parents' pages now
        for a, _, start, _, carried in groups:
            parent = borrowing.tree_parent[a] if a < len(borrowing.tree_parent) else None
            if carried and start == 0 and parent is not None:
                arena.release(keys[parent])
    while outstanding:
        report(outstanding.pop(0))
    arena.drop_holds(held)
    if stats is not None:
        stats["borrowed_tokens"] = borrowing.borrowed_tokens
        stats["h2d_bytes"] = h2d[0]
        stats["chunks"] = h2d[1]
        stats["skipped_partners"] = sched.skipped_partners
    return sched.answers, spans, tokens
