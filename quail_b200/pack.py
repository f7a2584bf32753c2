"""Admission for filter chains and joins: which rows and stages form each chunk.

Same policy as Quail's FilterAdmission and Borrowing
(quail/backends/quail/executor/pack.py:131-209, 647-836):

- survivor suffixes (documents that answered TRUE and have a later stage)
  pack first, oldest first, while they fit the chunk's token room;
- then fresh documents in queue order (prefix-tree order when there is a
  tree): pages are granted strictly in queue order (the first that does
  not fit the free pages stops admission), while chunk room may be skipped
  (a document that does not fit the room waits for the next chunk, ahead
  of the rest of the queue);
- a document whose tree parent is still queued waits; one whose parent
  has run borrows the parent's shared pages if the arena can serve them,
  and otherwise packs whole.
"""

from bisect import bisect_right
from collections import deque

import numpy as np


def pages_for(tokens: int, page_tokens: int) -> int:
    return -(-tokens // page_tokens)


def partner_pages(page_cost, page_tokens, prefix_tokens, frame_tokens, suffix_rows):
    """Temporary pages one partner's rows take on the unified path: they
    follow the anchor's last partial page, whose rows are copied in first
    (pack.py:120-128)."""
    return page_cost((prefix_tokens + frame_tokens) % page_tokens + suffix_rows, 0)


class DocumentQueue:
    """FIFO of document positions with cheap bulk prepends."""

    def __init__(self, values=()):
        self._parts = deque()
        self._size = 0
        self.prepend(values)

    def __bool__(self):
        return self._size > 0

    def __len__(self):
        return self._size

    def prepend(self, values) -> None:
        values = list(values)
        if values:
            self._parts.appendleft(deque(values))
            self._size += len(values)

    def appendleft(self, value) -> None:
        self.prepend([value])

    def popleft(self):
        if not self._size:
            raise IndexError("pop from an empty document queue")
        head = self._parts[0]
        value = head.popleft()
        if not head:
            self._parts.popleft()
        self._size -= 1
        return value


class Borrowing:
    """Per document: which parent it borrows its prefix pages from, if any."""

    WAIT = "wait"

    def __init__(self, n, tree=None, can_borrow=None):
        self.tree_parent = [None] * n if tree is None else list(tree.parent)
        self.tree_shared = [0] * n if tree is None else list(tree.shared)
        self.can_borrow = can_borrow
        self.admitted = set()
        self.skipped = set()
        self.chosen = {}
        self.borrowed_tokens = 0

    def add(self):
        """A document admitted after construction: it borrows nothing."""
        self.tree_parent.append(None)
        self.tree_shared.append(0)
        return len(self.tree_parent) - 1

    def detach(self, doc):
        """The document's KV is resident already: it borrows nothing."""
        self.tree_parent[doc] = None
        self.tree_shared[doc] = 0

    def skip(self, doc):
        """The document never runs a chunk: its borrowers pack whole."""
        self.skipped.add(doc)

    def borrowers(self):
        counts = [0] * len(self.tree_parent)
        for p in self.tree_parent:
            if p is not None:
                counts[p] += 1
        return counts

    def decide(self, doc, chunk):
        """WAIT, None (pack whole) or (parent, shared tokens)."""
        parent = self.tree_parent[doc]
        if parent is None or parent in self.skipped:
            return None
        if parent not in self.admitted:
            return self.WAIT
        if self.can_borrow is not None and not self.can_borrow(doc, parent, parent in chunk):
            return None
        return parent, self.tree_shared[doc]

    def record(self, doc, choice):
        self.admitted.add(doc)
        if choice is not None:
            self.chosen[doc] = choice
            self.borrowed_tokens += choice[1]

    def parent(self, doc):
        return self.chosen.get(doc, (None, 0))[0]

    def shared(self, doc):
        return self.chosen.get(doc, (None, 0))[1]


class FilterAdmission:
    """Builds the (doc, stage, fresh) groups of each chunk; gates answers."""

    def __init__(self, doc_tokens, stage_tokens, chunk_budget, arena_pages, page_tokens,
                 kept_extra_tokens=0, limit=None, page_cost=None, tree=None,
                 can_borrow=None):
        self.page_cost = page_cost or (lambda tokens, base=None: pages_for(tokens, page_tokens))
        self.doc_tokens = list(doc_tokens)
        n = len(self.doc_tokens)
        self.borrowing = Borrowing(n, tree, can_borrow)
        self.stage_tokens = list(stage_tokens)
        self.chunk_budget = chunk_budget
        self.page_tokens = page_tokens
        self.pages = arena_pages is not None
        self.blocked_pages = 0
        self.limit = limit
        self._survivors = 0
        self.kept_extra = kept_extra_tokens
        if tree is not None and arena_pages is None:
            raise ValueError("a prefix tree needs page accounting")
        longest_stage = max(self.stage_tokens)
        for d, t in enumerate(self.doc_tokens):
            if t + longest_stage > chunk_budget:
                raise ValueError(f"document {d} + question needs {t + longest_stage} "
                                 f"tokens > chunk budget {chunk_budget}")
            if arena_pages is not None and self.page_cost(t + kept_extra_tokens) > arena_pages:
                raise ValueError(f"document {d} needs more pages than the arena holds")
        order = range(n) if tree is None else tree.order
        self.pending = DocumentQueue(order)
        self.ready = deque()
        self.in_flight = set()
        self.resident = set()
        self.answers = {}

    def next_chunk(self, free_pages=None):
        """[(doc, stage, fresh)] for the next chunk; [] when nothing fits."""
        if self._limit_reached():
            return []
        self.blocked_pages = 0
        room = self.chunk_budget
        groups = []
        admitted = set()
        while self.ready:
            doc, stage = self.ready[0]
            cost = self.stage_tokens[stage]
            if cost > room:
                break
            self.ready.popleft()
            groups.append((doc, stage, False))
            self.in_flight.add(doc)
            room -= cost
        waiting = []
        while self.pending:
            doc = self.pending.popleft()
            choice = self.borrowing.decide(doc, admitted)
            if choice == Borrowing.WAIT:
                waiting.append(doc)
                continue
            own = self.doc_tokens[doc] - (choice[1] if choice else 0)
            need = 0
            if free_pages is not None:
                need = self.page_cost(own + self.kept_extra)
                if need > free_pages:
                    self.pending.appendleft(doc)
                    self.blocked_pages = need - free_pages
                    break
            cost = self.stage_tokens[0] + own
            if cost > room:
                waiting.append(doc)
                continue
            if free_pages is not None:
                free_pages -= need
            self.borrowing.record(doc, choice)
            self.resident.add(doc)
            groups.append((doc, 0, True))
            self.in_flight.add(doc)
            admitted.add(doc)
            room -= cost
        self.pending.prepend(waiting)
        return groups

    def report(self, doc, stage, passed, release=True):
        """Record one answer; returns the documents whose pages may be freed."""
        self.in_flight.discard(doc)
        self.answers.setdefault(doc, []).append(1 if passed else 0)
        last = stage == len(self.stage_tokens) - 1
        if passed and last:
            self._survivors += 1
        if passed and not last:
            self.ready.append((doc, stage + 1))
            return ()
        self.resident.discard(doc)
        if not self.pages or not release:
            return ()
        return (doc,)

    def _limit_reached(self):
        return self.limit is not None and self._survivors >= self.limit

    def done(self):
        if self._limit_reached():
            return not self.in_flight
        return not self.pending and not self.ready and not self.in_flight

    def drain_ready(self):
        out = []
        while self.ready:
            doc, _ = self.ready.popleft()
            self.resident.discard(doc)
            if self.pages:
                out.append(doc)
        return out

    def survivors(self):
        n = len(self.stage_tokens)
        return sorted(d for d, row in self.answers.items() if len(row) == n and all(row))


_DONE = -2  # the anchor answered its last stage, or failed a gate


class JoinAdmission:
    """Join scheduler: anchors stream partner lists, stages mix in one chunk.

    The same policy as Quail's JoinAdmission (pack.py:212-458), whose chunk
    composition the page tables depend on:

    - each chunk fills, in order, the streams the previous chunk cut and
      the anchors starting their next stage (ready queue, FIFO), then fresh
      anchors (pending queue, tree order when there is a tree: resident
      anchors first);
    - a partner run is atomic per partner and ends where the chunk's token
      room (and, on the unified path, the temporary suffix pages) runs out;
    - fresh anchors take pages strictly in queue order (the first that
      does not fit stops admission unless zero-cost anchors remain), while
      chunk room may be skipped;
    - an anchor moves to its next stage once its whole stream at the
      current one is launched and one partner answered TRUE; it drops out
      when every partner answered FALSE; one with no partner at a stage
      settles without a chunk.

    Args mirror the reference: prefix_tokens per anchor; stage_suffixes
    per stage, the partner suffix token counts; chunk_budget; arena_pages;
    page_tokens; frame_tokens per stage; resident {anchor: pages held};
    anchor_partners {anchor: per-stage index lists or None};
    temporary_suffix_pages (unified path); answer_dtype (None: 0/1 lists);
    canvas_tokens; page_cost; tree; can_borrow.
    """

    def __init__(self, prefix_tokens, stage_suffixes, chunk_budget, arena_pages, page_tokens,
                 frame_tokens=None, resident=None, anchor_partners=None,
                 temporary_suffix_pages=False, answer_dtype=None, canvas_tokens=0,
                 page_cost=None, tree=None, can_borrow=None, stop_at_true=False,
                 stream_step=None):
        if stop_at_true and answer_dtype is not None:
            raise ValueError("stop_at_true needs 0/1 answers (an EXISTS join), not scores")
        if stream_step is not None and stream_step < 1:
            raise ValueError("stream_step must be at least 1")
        # at most this many partners of one anchor per chunk (None: as many
        # as fit); with stop_at_true, a small step interleaves the anchors'
        # streams so a TRUE answer arrives before most of a stream launches
        self.stream_step = stream_step
        self.answer_dtype = answer_dtype
        # EXISTS early stop (not in the reference, which scores every partner
        # and gates afterwards, backend.py:231-240): once a last-stage
        # partner of an anchor answers TRUE, its partners not launched yet
        # are skipped; _cut[a] is the count its last-stage row stops at
        self.stop_at_true = stop_at_true
        self._cut = {}
        self.skipped_partners = 0
        self.borrowing = Borrowing(len(prefix_tokens), tree, can_borrow)
        self.page_cost = page_cost or (lambda tokens, base=None: pages_for(tokens, page_tokens))
        self.chunk_budget = chunk_budget
        self.arena_pages = arena_pages
        self.page_tokens = page_tokens
        self.temporary_suffix_pages = temporary_suffix_pages
        self.stages = [[t + canvas_tokens for t in lens] for lens in stage_suffixes]
        if not self.stages:
            raise ValueError("a join needs at least one stage")
        self.frames = list(frame_tokens) if frame_tokens else [0] * len(self.stages)
        if len(self.frames) != len(self.stages):
            raise ValueError("frame_tokens must match stage_suffixes")
        # rows a frame entry packs (canvas included) vs keeps in the KV
        self.frame_rows = [f + canvas_tokens if f else 0 for f in self.frames]
        self._stage_cum = []
        for j, (lens, frame) in enumerate(zip(self.stages, self.frame_rows)):
            cum = [0]
            for t in lens:
                cum.append(cum[-1] + t)
            self._stage_cum.append(cum)
            if lens and frame + max(lens) > chunk_budget:
                raise ValueError(f"stage {j}: a {frame + max(lens)}-token partner exceeds the "
                                 f"{chunk_budget}-token chunk budget (suffixes are atomic)")
        self._extra = max(self.frame_rows)
        # per anchor
        self.prefix = []
        self._lists = []        # per stage: partner indices, or None (all)
        self._cums = []         # per stage: cumulative costs of its own list
        self._page_need = []    # pages a fresh admission takes
        self._carried = []      # prefix tokens a fresh admission packs
        self._first = []        # tokens of its first partner (and frame)
        self._stage = []        # current stage, -1 before admission, or _DONE
        self._next = []         # next partner position at the stage
        self._true = []         # per stage: one partner answered TRUE
        self._min_fresh = float("inf")
        self._zero_cost = 0
        self._page_reserve = 0
        self._page_cums = {}
        self._counts = [{} for _ in self.stages]
        self._settled = []
        self.pending = deque()
        self.ready = deque()
        self.in_flight = 0
        self.blocked_pages = 0
        self.answers = [dict() for _ in self.stages]
        resident = dict(resident or {})
        partners = dict(anchor_partners or {})
        for a, prefix in enumerate(prefix_tokens):
            self._register(prefix, resident.get(a), partners.get(a))
        n = len(self.prefix)
        order = range(n) if tree is None else tree.order
        self.pending.extend(a for a in range(n) if a in resident and self._stage[a] == -1)
        self.pending.extend(a for a in order if a not in resident and self._stage[a] == -1)
        for a in resident:
            self.borrowing.detach(a)

    # ---- per-anchor costs ---------------------------------------------------

    def _count(self, a, j):
        if j == len(self.stages) - 1 and a in self._cut:
            return self._cut[a]
        lst = self._lists[a][j]
        return len(self.stages[j]) if lst is None else len(lst)

    def _cum_of(self, a, j):
        return self._stage_cum[j] if self._lists[a][j] is None else self._cums[a][j]

    def _suffix(self, a, j, i):
        lst = self._lists[a][j]
        return self.stages[j][i if lst is None else lst[i]]

    def partner_indices(self, a, j, start, end):
        """Stage j's partner list indices of one launched group."""
        lst = self._lists[a][j]
        return list(range(start, end)) if lst is None else list(lst[start:end])

    def _suffix_page_cost(self, a, j, i):
        return partner_pages(self.page_cost, self.page_tokens, self.prefix[a], self.frames[j],
                             self._suffix(a, j, i))

    def _register(self, prefix, resident_pages, partners):
        a = len(self.prefix)
        k = len(self.stages)
        if partners is None:
            lists, cums = [None] * k, [None] * k
        else:
            lists = [None if lst is None else list(lst) for lst in partners]
            if len(lists) != k:
                raise ValueError(f"anchor {a}: partner lists for {len(lists)} stages, "
                                 f"the join has {k}")
            cums = []
            for j, lst in enumerate(lists):
                if lst is None:
                    cums.append(None)
                    continue
                cum = [0]
                for i in lst:
                    if not 0 <= i < len(self.stages[j]):
                        raise ValueError(f"anchor {a} stage {j}: partner {i} is out of range")
                    cum.append(cum[-1] + self.stages[j][i])
                cums.append(cum)
        need = self.page_cost(prefix + self._extra)
        if resident_pages is not None:
            need = max(0, need - resident_pages)
        elif need > self.arena_pages:
            raise ValueError(f"anchor {a} needs {need} KV pages; the arena holds "
                             f"{self.arena_pages}")
        carried = 0 if resident_pages is not None else prefix
        self.prefix.append(prefix)
        self._lists.append(lists)
        self._cums.append(cums)
        self._page_need.append(need)
        self._carried.append(carried)
        self._stage.append(-1)
        self._next.append(0)
        self._true.append([False] * k)
        if self._count(a, 0) == 0:
            # nothing to evaluate: settles without a chunk
            self._first.append(0)
            self._stage[a] = _DONE
            self._settled.append(("finished" if k == 1 else "dropped", a))
            self.borrowing.skip(a)
            return a
        first = self.frame_rows[0] + self._suffix(a, 0, 0)
        if resident_pages is None and prefix + first > self.chunk_budget:
            raise ValueError(f"anchor {a}: prefix {prefix} tokens leaves no room for a partner "
                             f"in a {self.chunk_budget}-token chunk")
        if self.temporary_suffix_pages:
            largest = max((self._suffix_page_cost(a, j, i)
                           for j in range(k) for i in range(self._count(a, j))), default=0)
            if self.page_cost(prefix + self._extra) + largest > self.arena_pages:
                raise ValueError("anchor and one suffix exceed the KV arena")
            self._page_reserve = max(self._page_reserve, largest)
        self._first.append(first)
        shared = self.borrowing.tree_shared
        own_shared = shared[a] if a < len(shared) else 0
        self._min_fresh = min(self._min_fresh, max(0, carried - own_shared) + first)
        if not need:
            self._zero_cost += 1
        return a

    def admit(self, prefix_tokens, resident_pages=None, partners=None):
        """Queue one more anchor behind the pending ones; returns its index."""
        a = self._register(prefix_tokens, resident_pages, partners)
        self.borrowing.add()
        if self._stage[a] == -1:
            self.pending.append(a)
        return a

    def take_settled(self):
        """("finished" | "dropped", anchor) events of anchors that never ran."""
        events, self._settled = self._settled, []
        return events

    def buildable_tokens(self):
        """Tokens the next chunk could pack (chunk room only), capped at the budget."""
        total = 0
        for a in self.ready:
            j, i = self._stage[a], self._next[a]
            cum = self._cum_of(a, j)
            total += (self.frame_rows[j] if i == 0 else 0) + cum[-1] - cum[i]
            if total >= self.chunk_budget:
                return self.chunk_budget
        for a in self.pending:
            total += self._carried[a] + self.frame_rows[0] + self._cum_of(a, 0)[-1]
            if total >= self.chunk_budget:
                return self.chunk_budget
        return total

    # ---- chunk building -------------------------------------------------------

    def _first_cost(self, a, j, i):
        return self._suffix(a, j, i) + (self.frame_rows[j] if i == 0 else 0)

    def _take(self, a, j, i, room, page_room):
        """(end, tokens, pages): the partner run from i that fits the token
        room and, on the unified path, the temporary page room."""
        cum = self._cum_of(a, j)
        frame = self.frame_rows[j] if i == 0 else 0
        end = bisect_right(cum, cum[i] + room - frame) - 1
        if self.stream_step is not None:
            end = min(end, i + self.stream_step)
        pages = 0
        if self.temporary_suffix_pages:
            costs = self._page_cums.get((a, j))
            if costs is None:
                costs = [0]
                for x in range(self._count(a, j)):
                    costs.append(costs[-1] + self._suffix_page_cost(a, j, x))
                self._page_cums[(a, j)] = costs
            end = min(end, bisect_right(costs, costs[i] + page_room) - 1)
            pages = costs[end] - costs[i]
        return end, frame + cum[end] - cum[i], pages

    def _launch(self, a, j, end):
        """Record a launched group; True while the stream continues."""
        self._next[a] = end
        self.in_flight += 1
        return end < self._count(a, j)

    def next_chunk(self, free_pages):
        """[(anchor, stage, start, end, carried)] for the next chunk, [] when
        nothing is buildable. carried: the anchor's prefix is packed."""
        self.blocked_pages = 0
        room = self.chunk_budget
        groups, continued = [], []
        temporary_pages = 0
        # placed anchors: cut streams first, then next-stage starts (FIFO)
        for _ in range(len(self.ready)):
            a = self.ready.popleft()
            j, i = self._stage[a], self._next[a]
            if self._first_cost(a, j, i) > room:
                self.ready.appendleft(a)
                break
            end, tokens, pages = self._take(a, j, i, room, free_pages)
            if end == i:  # the temporary pages of one partner do not fit
                self.blocked_pages = self._suffix_page_cost(a, j, i) - free_pages
                self.ready.appendleft(a)
                break
            free_pages -= pages
            temporary_pages += pages
            groups.append((a, j, i, end, False))
            room -= tokens
            if self._launch(a, j, end):
                continued.append(a)
        # fresh anchors: pages strictly in queue order, chunk room may skip
        held, admitted = [], set()
        blocked = False
        while self.pending and room >= self._min_fresh:
            a = self.pending.popleft()
            borrow = self.borrowing.decide(a, admitted)
            if borrow == Borrowing.WAIT:
                held.append(a)
                continue
            need = (self._page_need[a] if borrow is None
                    else self.page_cost(self.prefix[a] - borrow[1] + self._extra))
            if blocked and need:
                held.append(a)
                if not self._zero_cost:
                    break
                continue
            required = need + max(0, self._page_reserve - temporary_pages)
            if required > free_pages:
                blocked = True
                self.blocked_pages = required - free_pages
                held.append(a)
                if not self._zero_cost:
                    break
                continue
            carried = self._carried[a] if borrow is None else self.prefix[a] - borrow[1]
            if carried + self._first[a] > room:
                held.append(a)
                continue
            end, tokens, pages = self._take(a, 0, 0, room - carried, free_pages - need)
            if end == 0:
                held.append(a)
                self.blocked_pages = need + self._suffix_page_cost(a, 0, 0) - free_pages
                break
            temporary_pages += pages
            groups.append((a, 0, 0, end, carried > 0))
            room -= carried + tokens
            free_pages -= need + pages
            if not self._page_need[a]:
                self._zero_cost -= 1
            self._stage[a] = 0
            admitted.add(a)
            self.borrowing.record(a, borrow)
            if self._launch(a, 0, end):
                continued.append(a)
        self.pending.extendleft(reversed(held))
        self.ready.extendleft(reversed(continued))
        return groups

    # ---- gating -----------------------------------------------------------------

    def report(self, a, j, start, end, bits):
        """Record one group's answers; returns ("dropped" | "finished", a)
        events (the anchor's pages may go)."""
        if self.answer_dtype is None:
            row = self.answers[j].setdefault(a, [])
            received = len(row)
        else:
            if a not in self.answers[j]:
                self.answers[j][a] = np.empty(self._count(a, j), dtype=self.answer_dtype)
            row = self.answers[j][a]
            received = self._counts[j].get(a, 0)
        if received != start or len(bits) != end - start:
            raise AssertionError(f"anchor {a} stage {j}: answers for partners {start}:{end} "
                                 f"arrived with {received} recorded")
        if self.answer_dtype is None:
            row.extend(bits)
        else:
            row[start:end] = bits
            self._counts[j][a] = end
        self.in_flight -= 1
        if any(bits) if self.answer_dtype is None else np.any(bits):
            self._true[a][j] = True
        k = len(self.stages)
        if (self.stop_at_true and j == k - 1 and self._true[a][j] and a not in self._cut
                and self._next[a] < self._count(a, j)):
            # the rest of the stream is decided: stop it where it was launched
            self.skipped_partners += self._count(a, j) - self._next[a]
            self._cut[a] = self._next[a]
            if a in self.ready:
                self.ready.remove(a)
        n_j = self._count(a, j)
        complete = end == n_j
        events = []
        if j == self._stage[a] and j + 1 < k:
            if self._true[a][j] and self._next[a] == n_j:
                # the whole stream is launched: later chunks are behind it, so
                # the next stage's frame write cannot race this stage's reads
                self._stage[a] = j + 1
                self._next[a] = 0
                if self._count(a, j + 1):
                    self.ready.append(a)
                else:
                    self._stage[a] = _DONE
                    events.append(("finished" if j + 2 == k else "dropped", a))
            elif complete and not self._true[a][j]:
                self._stage[a] = _DONE
                events.append(("dropped", a))
        if j == k - 1 and complete:
            self._stage[a] = _DONE
            events.append(("finished", a))
        return events

    def done(self):
        return not self.pending and not self.ready and not self.in_flight and not self._settled
