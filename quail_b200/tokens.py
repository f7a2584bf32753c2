"""Prefix tree over documents: which document borrows whose KV pages.

Same contract as Quail's ``prefix_tree`` (quail/execution/tokens.py:514-591):

- documents are visited in sorted order of their big-endian int32 token
  bytes (ties keep input order);
- a document shares with its predecessor the longest common token prefix,
  capped one short of its own length (it always computes its last token)
  and rounded down to a whole page;
- its parent is the predecessor, or the highest ancestor of the
  predecessor that itself borrowed at least as many tokens, so siblings of
  one prefix all read the same parent's pages.
"""

import numpy as np


class PrefixTree:
    """order, parent and shared per document (see module docstring)."""

    def __init__(self, order, parent, shared):
        self.order = order
        self.parent = parent
        self.shared = shared

    @property
    def shared_tokens(self) -> int:
        return int(sum(self.shared))


def _as_array(doc):
    if isinstance(doc, np.ndarray):
        return doc.astype(np.int32, copy=False)
    return np.asarray(list(doc), dtype=np.int32)


def _lcp(a, b) -> int:
    n = min(len(a), len(b))
    if n == 0:
        return 0
    diff = np.flatnonzero(a[:n] != b[:n])
    return int(diff[0]) if diff.size else n


def prefix_tree(documents, page_tokens: int) -> PrefixTree:
    """Build the prefix tree of a sequence of token documents."""
    n = len(documents)
    arrays = [_as_array(documents[i]) for i in range(n)]
    keys = [a.astype(">i4").tobytes() for a in arrays]
    order = sorted(range(n), key=keys.__getitem__)
    parent = [None] * n
    shared = [0] * n
    prev = None
    for doc in order:
        if prev is not None:
            common = min(_lcp(arrays[prev], arrays[doc]), max(len(arrays[doc]) - 1, 0))
            pages = (common // page_tokens) * page_tokens
            if pages:
                owner = prev
                while parent[owner] is not None and shared[owner] >= pages:
                    owner = parent[owner]
                parent[doc] = owner
                shared[doc] = pages
        prev = doc
    return PrefixTree(order, parent, shared)
