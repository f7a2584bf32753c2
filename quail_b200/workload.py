"""Seeded synthetic AI.IF rows with the BASELINE configurations' shapes.

The reference's benchmark data (QUAIL-B) is not available here; these
seeded rows stand in for it with the configurations' lengths and token-id
ranges. Each row is one document ``prefix | suffix`` (the shared
instruction prefix is the first tokens of every document, as Quail's
DocumentPrefixes lays it out, quail/execution/tokens.py:412-429) and the
stage question is a one-token tail drawn with seed 3.

Rows are generated on access (row i's suffix from its own seeded
generator), so a rank materialises only the rows of its slice.
"""

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np


class DocRows(Sequence):
    """Lazy documents: row i = prefix | suffix_i, suffix_i from rng(seed, i)."""

    def __init__(self, prefix, lengths, lo, hi, seed, start=0, stop=None):
        self.prefix = np.asarray(prefix, dtype=np.int32)
        self.lengths = np.asarray(lengths, dtype=np.int64)
        self.lo, self.hi, self.seed = lo, hi, seed
        self.start = start
        self.stop = len(self.lengths) if stop is None else stop
        self._cache = {}

    def __len__(self):
        return self.stop - self.start

    def __getitem__(self, i):
        if isinstance(i, slice):
            a, b, step = i.indices(len(self))
            if step != 1:
                return [self[j] for j in range(a, b, step)]
            return DocRows(self.prefix, self.lengths, self.lo, self.hi, self.seed,
                           self.start + a, self.start + b)
        if i < 0:
            i += len(self)
        if not 0 <= i < len(self):
            raise IndexError(i)
        row = self.start + i
        got = self._cache.get(row)
        if got is None:
            rng = np.random.default_rng([self.seed, row])
            body = rng.integers(self.lo, self.hi, int(self.lengths[row]), dtype=np.int32)
            got = np.concatenate([self.prefix, body])
            self._cache[row] = got
        return got


@dataclass
class Workload:
    name: str
    model: str
    docs: Sequence
    questions: list
    prefix_tokens: int

    @property
    def rows(self) -> int:
        return len(self.docs)

    def logical_tokens(self, lo=0, hi=None) -> int:
        """prefix + suffix + question tail per row, over rows [lo, hi)."""
        hi = len(self.docs) if hi is None else hi
        lengths = self.docs.lengths[self.docs.start + lo:self.docs.start + hi]
        n = hi - lo
        return int(lengths.sum() + n * (self.prefix_tokens + len(self.questions[0])))

    def row_tokens(self) -> np.ndarray:
        """Logical tokens (prefix + suffix + tail) of every row, in row order."""
        lengths = self.docs.lengths[self.docs.start:self.docs.start + len(self.docs)]
        return lengths + self.prefix_tokens + len(self.questions[0])

    def fresh_row_tokens(self, lo=0, hi=None) -> np.ndarray:
        """Tokens each row of [lo, hi) puts into a chunk when its first
        prefix_tokens are borrowed from a resident parent: suffix + tail."""
        hi = len(self.docs) if hi is None else hi
        lengths = self.docs.lengths[self.docs.start + lo:self.docs.start + hi]
        return lengths + len(self.questions[0])


def _question():
    return [int(np.random.default_rng(3).integers(1000, 150000))]


def config1(rows=100_000, seed=0) -> Workload:
    """Qwen3-4B FP8 AI.IF filter: a 64-token shared prefix, suffixes
    lognormal(5.3, 0.6) clipped to [32, 2048], ids uniform in [1000, 150000)."""
    rng = np.random.default_rng(seed)
    prefix = rng.integers(1000, 150000, 64)
    lens = np.clip(rng.lognormal(5.3, 0.6, rows).astype(np.int64), 32, 2048)
    return Workload("config1", "qwen3-4b-fp8", DocRows(prefix, lens, 1000, 150000, seed),
                    [_question()], 64)


def config3(rows=50_000, seed=0) -> Workload:
    """Qwen3-32B FP8 filter: 96-token prefix, lognormal(5.5, 0.5) in [64, 2048]."""
    rng = np.random.default_rng(seed)
    prefix = rng.integers(1000, 150000, 96)
    lens = np.clip(rng.lognormal(5.5, 0.5, rows).astype(np.int64), 64, 2048)
    return Workload("config3", "qwen3-32b-fp8", DocRows(prefix, lens, 1000, 150000, seed),
                    [_question()], 96)


def config4(rows=4_000, seed=0) -> Workload:
    """Qwen3-4B FP8 long-document filter: a 64-token shared prefix and
    suffixes uniform in [4096, 16384] tokens, ids uniform in [1000, 150000)."""
    rng = np.random.default_rng(seed)
    prefix = rng.integers(1000, 150000, 64)
    lens = rng.integers(4096, 16385, rows).astype(np.int64)
    return Workload("config4", "qwen3-4b-fp8", DocRows(prefix, lens, 1000, 150000, seed),
                    [_question()], 64)


@dataclass
class JoinWorkload:
    """An AI join: anchors (left rows) stream every partner (right row)."""
    name: str
    model: str
    anchors: Sequence           # instruction | left document, per left row
    partners: list              # right document | question tail, per right row
    instruction_tokens: int

    @property
    def pairs(self) -> int:
        return len(self.anchors) * len(self.partners)

    def logical_tokens(self, lo=0, hi=None) -> int:
        """Prompt tokens of every pair whose anchor is in [lo, hi)."""
        hi = len(self.anchors) if hi is None else hi
        anchor = sum(len(self.anchors[a]) for a in range(lo, hi))
        partner = sum(len(p) for p in self.partners)
        return (hi - lo) * partner + anchor * len(self.partners)


def config2(left=200, right=500, seed=0) -> JoinWorkload:
    """Qwen3-4B FP8 AI join: a 48-token shared instruction, left documents
    uniform in [128, 512] tokens (one anchor each), right documents uniform
    in [64, 256] (each followed by the one-token question tail), ids uniform
    in [1000, 150000); shard by left row."""
    rng = np.random.default_rng(seed)
    instruction = rng.integers(1000, 150000, 48)
    left_lens = rng.integers(128, 513, left)
    right_lens = rng.integers(64, 257, right)
    anchors = DocRows(instruction, left_lens, 1000, 150000, seed + 1)
    tail = _question()
    prng = np.random.default_rng(seed + 2)
    partners = [prng.integers(1000, 150000, int(n)).tolist() + tail for n in right_lens]
    return JoinWorkload("config2", "qwen3-4b-fp8", anchors, partners, 48)


@dataclass
class ExistsWorkload:
    """Config 4's EXISTS variant: outer rows (anchors) each scored against
    their own correlated candidate rows, not a cross product.

    anchors[a] = the 64-token shared prefix | outer row a's 512-token
    context (the second-level prefix its candidates share);
    candidates(a) = its candidate documents, each followed by the question
    tail. An outer row survives EXISTS when any candidate answers TRUE.
    """
    name: str
    model: str
    anchors: Sequence
    n_candidates: int
    candidate_lengths: np.ndarray   # [outer rows, n_candidates]
    tail: list
    seed: int

    def candidates(self, a: int) -> list:
        """Outer row a's candidate token lists (generated on access)."""
        out = []
        for j, n in enumerate(self.candidate_lengths[a]):
            rng = np.random.default_rng([self.seed, a, j])
            out.append(rng.integers(1000, 150000, int(n)).tolist() + self.tail)
        return out


def config4_exists(outer=4_000, candidates=8, seed=0) -> ExistsWorkload:
    """Qwen3-4B FP8 EXISTS probe: a 64-token shared prefix and a 512-token
    context per outer row (the second-level prefix), then 8 candidate
    documents per outer row with config 4's lengths (uniform in [4096,
    16384] tokens), ids uniform in [1000, 150000)."""
    rng = np.random.default_rng(seed)
    prefix = rng.integers(1000, 150000, 64)
    context = np.full(outer, 512, dtype=np.int64)
    lens = rng.integers(4096, 16385, (outer, candidates)).astype(np.int64)
    return ExistsWorkload("config4-exists", "qwen3-4b-fp8",
                          DocRows(prefix, context, 1000, 150000, seed + 1), candidates, lens,
                          _question(), seed + 2)


def shard(n_rows: int, rank: int, world: int) -> tuple:
    """Contiguous row slice [lo, hi) of one rank (equal row counts)."""
    per = -(-n_rows // world)
    lo = min(n_rows, rank * per)
    return lo, min(n_rows, lo + per)


def token_shard(row_tokens, rank: int, world: int) -> tuple:
    """Contiguous row slice [lo, hi) of one rank, balanced by tokens.

    Rank k's slice ends at the row boundary nearest to k/world of the total
    token count (running sums over row_tokens), so every rank gets about
    the same prefill work whatever the length distribution. Quail's filter
    planner splits ordered documents into token-balanced contiguous ranges
    the same way (quail/planner/decide.py:308-338, contiguous_shards);
    results are per row, so where the cut falls changes no answer.
    """
    c = np.cumsum(np.asarray(row_tokens, dtype=np.int64))
    n = len(c)
    total = int(c[-1]) if n else 0

    def cut(k):
        if k <= 0 or n == 0:
            return 0
        if k >= world:
            return n
        target = total * k / world
        i = min(int(np.searchsorted(c, target)), n - 1)   # first row reaching target
        before = int(c[i - 1]) if i else 0
        return i + 1 if int(c[i]) - target <= target - before else i

    return cut(rank), cut(rank + 1)
