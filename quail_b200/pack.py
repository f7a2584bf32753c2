"""Admission for filter chains: which documents and stages form each chunk.

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

from collections import deque


def pages_for(tokens: int, page_tokens: int) -> int:
    return -(-tokens // page_tokens)


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
