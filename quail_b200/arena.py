"""Paged KV arena: per-layer bf16 K and V pools reached through page tables.

The page-table contract is Quail's (quail/backends/quail/executor/arena.py):

- pages come from a LIFO free stack initialised to [n-1, ..., 0], so a
  fresh arena hands out pages 0, 1, 2, ...;
- a key owns the pages it writes and may borrow the leading whole pages of
  a resident parent's prefix; its block table lists borrowed pages first;
- page p holds pool rows p * page_tokens .. p * page_tokens + page_tokens;
- a page returns to the free stack when its last holder frees it;
- a key held for queued borrowers is freed only when the last one releases.

HBM layout: one allocation of shape (n_layers, 2, n_pages * page_tokens,
n_kv, head_dim) bf16; ``layer_kv(l)`` views its K and V halves as the flat
(rows, n_kv, head_dim) pools the kernels index by row.

Cross-operator retention (arena.py:153-226, 556-620): a filter survivor
or a finished join anchor can stay resident for a later operator, rewound
to its prefix; retained keys are evicted lowest planned-reuse priority
first (a heap of (priority, version, key, pages, tokens), stale entries
skipped by version) when admission is short of pages or the retained
pages pass the cap. Not built here (Gemma only): sliding-window pools;
the methods the filter loop calls for them are no-ops.
"""

import heapq

import numpy as np


class PageArena:
    """Page accounting only: a free stack, page lists and hold counts."""

    def __init__(self, n_pages: int, page_tokens: int):
        self.n_pages = n_pages
        self.page_tokens = page_tokens
        self.free = list(range(n_pages - 1, -1, -1))
        self.owned = {}
        self.borrowed = {}
        self.holds = [0] * n_pages
        self.tokens = {}
        self.pinned = set()
        # retention: key -> prefix tokens kept, key -> pages its eviction
        # frees (when retained), the priority heap and entry versions
        self.retained = {}
        self.retained_sizes = {}
        self.retained_pages = 0
        self.retention_heap = []
        self.retention_versions = {}
        self.retention_counter = 0
        self.retention_policy = None
        self.retention_cap_pages = None

    def pages_needed(self, tokens: int) -> int:
        return -(-tokens // self.page_tokens)

    @property
    def retained_prefix_tokens(self) -> int:
        return sum(self.tokens[key] for key in self.retained)

    @property
    def free_pages(self) -> int:
        return len(self.free)

    def alloc(self, key, tokens, capacity_tokens=None, borrowed=()):
        """Own pages for a new key (borrowed pages count toward its tokens).

        Returns the new page ids, or None when the free stack is short.
        """
        if key in self.owned:
            raise KeyError(f"{key!r} already resident")
        capacity = tokens if capacity_tokens is None else capacity_tokens
        if capacity < tokens:
            raise ValueError("capacity_tokens must cover logical tokens")
        borrowed = list(borrowed)
        if len(borrowed) * self.page_tokens > tokens:
            raise ValueError("a key cannot borrow past its own tokens")
        need = self.pages_needed(capacity) - len(borrowed)
        if need > len(self.free):
            return None
        mine = [self.free.pop() for _ in range(need)]
        self.owned[key] = mine
        self.borrowed[key] = borrowed
        self.tokens[key] = tokens
        for page in borrowed:
            self.holds[page] += 1
        for page in mine:
            self.holds[page] += 1
        return mine

    def shared_pages(self, parent, shared: int, start: int = 0) -> list:
        """The parent's pages covering its tokens [start, shared)."""
        pt = self.page_tokens
        if (shared - start) % pt or start % pt:
            raise ValueError("a borrowed prefix is a whole number of pages")
        if parent not in self.owned:
            raise KeyError(f"borrow parent {parent!r} is not resident")
        if shared > self.tokens[parent]:
            raise ValueError(f"{parent!r} holds fewer tokens than borrowed")
        return self.table_pages(parent)[start // pt:shared // pt]

    def table_pages(self, key) -> list:
        return self.borrowed[key] + self.owned[key]

    def release_pages(self, pages) -> int:
        freed = 0
        for page in pages:
            self.holds[page] -= 1
            if self.holds[page] == 0:
                self.free.append(page)
                freed += 1
        return freed

    def free_key(self, key) -> int:
        pages = self.owned.pop(key)
        borrowed = self.borrowed.pop(key)
        self.tokens.pop(key)
        self.pinned.discard(key)
        self._unretain(key)
        return self.release_pages(borrowed + pages)

    def pin(self, key) -> None:
        if key not in self.owned:
            raise KeyError(key)
        self._unretain(key)
        self.pinned.add(key)

    # ---- retention --------------------------------------------------------

    def _unretain(self, key) -> None:
        # a heap entry stays behind; its version no longer matches
        self.retained_pages -= self.retained_sizes.pop(key, 0)
        self.retained.pop(key, None)
        self.retention_versions.pop(key, None)

    def retain(self, key, priority=None) -> None:
        """Make a resident key evictable once its current use ends.

        The pages counted are the ones evicting it would free now (those it
        alone holds); priority defaults to the policy's, else tokens per
        page."""
        if key not in self.owned:
            raise KeyError(key)
        self.pinned.discard(key)
        tokens = self.tokens[key]
        self._unretain(key)
        pages = sum(1 for page in self.table_pages(key) if self.holds[page] == 1)
        self.retained[key] = tokens
        self.retained_sizes[key] = pages
        self.retained_pages += pages
        self.retention_counter += 1
        version = self.retention_counter
        self.retention_versions[key] = version
        if priority is None:
            if self.retention_policy is not None:
                priority = self.retention_policy.priority(key, tokens, max(1, pages))
            else:
                priority = (tokens / max(1, pages),)
        heapq.heappush(self.retention_heap, (priority, version, key, pages, tokens))

    def configure_retention(self, policy, cap_pages: int) -> None:
        """A new priority rule and retained-page cap: every retained key is
        re-entered under it (active keys stay unevictable)."""
        if not 0 <= cap_pages <= self.n_pages:
            raise ValueError("retention capacity must fit inside the arena")
        self.retention_policy = policy
        self.retention_cap_pages = cap_pages
        self.retention_heap = []
        for key in list(self.retained):
            self.retain(key)

    def pop_retained_victim(self, keep=frozenset()):
        """(key, pages, tokens) of the lowest-priority retained key, no longer
        retained; keys in keep are passed over. None when there is none."""
        passed, victim = [], None
        while self.retention_heap:
            entry = heapq.heappop(self.retention_heap)
            _, version, key, pages, tokens = entry
            if self.retention_versions.get(key) != version:
                continue
            if key in keep:
                passed.append(entry)
                continue
            self._unretain(key)
            victim = (key, pages, tokens)
            break
        for entry in passed:
            heapq.heappush(self.retention_heap, entry)
        return victim

    def borrowed_tokens(self, key) -> int:
        return len(self.borrowed[key]) * self.page_tokens

    def rewind(self, key, tokens: int) -> int:
        """Keep the key's first tokens; its trailing unused pages go back."""
        if key not in self.owned:
            raise KeyError(key)
        borrowed = self.borrowed_tokens(key)
        capacity = borrowed + len(self.owned[key]) * self.page_tokens
        if tokens < borrowed or tokens > capacity:
            raise ValueError("rewind tokens leave the resident capacity")
        keep = self.pages_needed(tokens) - len(self.borrowed[key])
        released = self.owned[key][keep:]
        self.owned[key] = self.owned[key][:keep]
        self.tokens[key] = tokens
        freed = self.release_pages(released)
        if key in self.retained:
            self.retain(key)
        return freed

    def grow(self, key, capacity_tokens: int):
        if key not in self.owned:
            raise KeyError(key)
        need = (self.pages_needed(capacity_tokens) - len(self.borrowed[key])
                - len(self.owned[key]))
        if need <= 0:
            return 0
        if need > len(self.free):
            return None
        added = [self.free.pop() for _ in range(need)]
        self.owned[key].extend(added)
        for page in added:
            self.holds[page] += 1
        return need


class KVArena:
    """Tensor pools plus the accounting above; the surface the loop uses.

    Args:
        n_layers, n_pages, page_tokens, n_kv, d_head: pool geometry.
        device: torch device of the pools; None builds the accounting only
            (host-side tests of the packer).
    """

    def __init__(self, n_layers: int, n_pages: int, page_tokens: int, n_kv: int,
                 d_head: int, device="cuda"):
        self.n_layers = n_layers
        self.n_kv = n_kv
        self.d_head = d_head
        self.device = device
        self.accounting = PageArena(n_pages, page_tokens)
        self.pools = None
        if device is not None:
            import torch
            self.pools = torch.empty(
                (n_layers, 2, n_pages * page_tokens, n_kv, d_head),
                dtype=torch.bfloat16, device=device)
        self._capacity_rows = {}
        self._holds = {}
        self._deferred = set()
        self.reset_stats()

    def reset(self) -> None:
        """Forget every key, hold and retention (the pools stay allocated)."""
        self.accounting = PageArena(self.accounting.n_pages, self.accounting.page_tokens)
        self._capacity_rows = {}
        self._holds = {}
        self._deferred = set()
        self.reset_stats()

    def reset_stats(self) -> None:
        """Zero the eviction counters."""
        self.evicted_keys = 0
        self.evicted_pages = 0
        self.evicted_prefix_tokens = 0

    # ---- geometry ---------------------------------------------------------

    @property
    def page_tokens(self) -> int:
        return self.accounting.page_tokens

    @property
    def n_pages(self) -> int:
        return self.accounting.n_pages

    @property
    def pool_rows(self) -> int:
        return self.n_pages * self.page_tokens

    @property
    def free_pages(self) -> int:
        return self.accounting.free_pages

    @property
    def has_sliding(self) -> bool:
        return False

    @property
    def retained_pages(self) -> int:
        return self.accounting.retained_pages

    @property
    def retained_prefix_tokens(self) -> int:
        return self.accounting.retained_prefix_tokens

    @property
    def retention_cap_pages(self):
        return self.accounting.retention_cap_pages

    @retention_cap_pages.setter
    def retention_cap_pages(self, pages) -> None:
        self.accounting.retention_cap_pages = pages

    def configure_retention(self, policy, cap_pages: int) -> None:
        """Set the eviction priority rule and the retained-page cap."""
        self.accounting.configure_retention(policy, cap_pages)

    def retained_keys(self) -> list:
        """Every key whose KV is kept for a later operator."""
        return list(self.accounting.retained)

    def pages_needed(self, tokens: int) -> int:
        return self.accounting.pages_needed(tokens)

    def page_cost(self, tokens: int, base_tokens=None) -> int:
        return self.accounting.pages_needed(tokens)

    # ---- allocation ---------------------------------------------------------

    def _set_rows(self, key):
        pages = np.asarray(self.accounting.table_pages(key), dtype=np.int64)
        pt = self.page_tokens
        self._capacity_rows[key] = (pages[:, None] * pt
                                    + np.arange(pt, dtype=np.int64)).reshape(-1)

    def alloc(self, key, tokens, capacity_tokens=None, base_tokens=None,
              sliding_tokens=None, borrow=None):
        borrowed = ()
        if borrow is not None:
            borrowed = self.accounting.shared_pages(*borrow)
        pages = self.accounting.alloc(key, tokens, capacity_tokens, borrowed=borrowed)
        if pages is None:
            return None
        self._set_rows(key)
        return pages

    def pin(self, key) -> None:
        """Mark a resident key active (a join's anchor): eviction skips it."""
        self.accounting.pin(key)

    def growth_cost(self, key, capacity_tokens: int) -> int:
        """Pages a resident key needs to grow to capacity (arena.py:772-786,
        without the sliding pool)."""
        return max(0, self.accounting.pages_needed(capacity_tokens)
                   - len(self.accounting.table_pages(key)))

    def can_borrow(self, parent, shared: int) -> bool:
        return (parent in self.accounting.owned
                and shared <= self.accounting.tokens[parent])

    def activate(self, key, tokens, capacity_tokens=None, base_tokens=None, borrow=None):
        """Make a key's prefix active: grow a resident key, or allocate a fresh one."""
        capacity = tokens if capacity_tokens is None else capacity_tokens
        acct = self.accounting
        if key in acct.owned:
            acct.pin(key)
            need = max(0, acct.pages_needed(capacity) - len(acct.table_pages(key)))
            if need > acct.free_pages:
                return None
            acct.grow(key, capacity)
            acct.tokens[key] = tokens
            self._set_rows(key)
            return acct.owned[key]
        pages = self.alloc(key, tokens, capacity, base_tokens, borrow=borrow)
        if pages is not None:
            acct.pin(key)
        return pages

    def alloc_temporary(self, tokens: int, sliding_tokens=None):
        key = object()
        pages = self.alloc(key, tokens, base_tokens=0)
        return None if pages is None else (key, pages)

    def hold(self, key, borrowers: int) -> None:
        if borrowers:
            self._holds[key] = self._holds.get(key, 0) + borrowers

    def release(self, key) -> None:
        if key not in self._holds:
            return
        self._holds[key] -= 1
        if not self._holds[key]:
            del self._holds[key]
            if key in self._deferred:
                self._deferred.discard(key)
                self.free_key(key)

    def drop_holds(self, keys=None) -> bool:
        keys = list(self._holds) if keys is None else [k for k in keys if k in self._holds]
        for key in keys:
            del self._holds[key]
            if key in self._deferred:
                self._deferred.discard(key)
                self.free_key(key)
        return bool(keys)

    def free_key(self, key) -> int:
        if key in self._holds:
            self._deferred.add(key)
            return 0
        self._capacity_rows.pop(key)
        return self.accounting.free_key(key)

    # ---- retention (arena.py:541-620) ------------------------------------------

    def retain(self, key, tokens: int, priority=None) -> int:
        """Rewind a key to its first tokens and keep it for a later
        operator; returns the pages that came free (the rewind's, and any
        eviction the cap forces). Keys are (alias, document) pairs."""
        if not (isinstance(key, tuple) and len(key) == 2):
            raise TypeError(f"retained keys are (alias, document) pairs, got {key!r}")
        acct = self.accounting
        before = self.free_pages
        acct.rewind(key, tokens)
        self._set_rows(key)
        acct.retain(key, priority)
        if acct.retention_cap_pages is not None:
            self.evict_retained(max(0, acct.retained_pages - acct.retention_cap_pages))
        return self.free_pages - before

    def evict_retained(self, pages_needed: int) -> tuple:
        """Evict retained keys, lowest priority first, until pages_needed
        pages have come free; keys held for queued borrowers stay. Returns
        the evicted keys."""
        start = self.free_pages
        evicted = []
        while self.free_pages - start < pages_needed:
            victim = self.accounting.pop_retained_victim(keep=self._holds)
            if victim is None:
                break
            evicted.append(victim[0])
            self.evict_key(victim[0])
        return tuple(evicted)

    def evict_key(self, key) -> int:
        """Free one retained key and count the KV lost."""
        tokens = self.accounting.tokens[key]
        pages = self.free_key(key)
        self.evicted_keys += 1
        self.evicted_pages += pages
        self.evicted_prefix_tokens += tokens
        return pages

    # the sliding window is outside this path
    def keep_window(self, key, shared: int) -> None:
        return None

    def trim_window(self, key) -> int:
        return 0

    # ---- residency ----------------------------------------------------------

    def is_resident(self, key) -> bool:
        return key in self.accounting.owned

    def resident_keys(self) -> list:
        return list(self.accounting.owned)

    def owned_pages(self, key) -> list:
        return self.accounting.table_pages(key)

    def capacity_rows(self, key):
        """Pool rows (int64 numpy) of every row in the key's pages."""
        return self._capacity_rows[key]

    def tokens(self, key) -> int:
        return self.accounting.tokens[key]

    # ---- tensors --------------------------------------------------------------

    def layer_kv(self, layer: int):
        """Flat K and V pools of one layer, (rows, n_kv, d_head)."""
        return self.pools[layer, 0], self.pools[layer, 1]

    def paged_kv(self, layer: int):
        k, v = self.layer_kv(layer)
        shape = (-1, self.page_tokens, self.n_kv, self.d_head)
        return k.view(shape), v.view(shape)

    def block_table_rows(self, pages, pad_to=None) -> np.ndarray:
        """A zero-padded int32 block table from explicit page lists."""
        width = max(len(p) for p in pages)
        if pad_to:
            width = max(width, pad_to)
        table = np.zeros((len(pages), width), dtype=np.int32)
        for i, p in enumerate(pages):
            table[i, :len(p)] = p
        return table

    def block_table(self, keys, pad_to=None):
        """(block table int32 [n, width], used tokens int32 [n]) on the host."""
        pages = [self.accounting.table_pages(k) for k in keys]
        used = np.asarray([self.accounting.tokens[k] for k in keys], dtype=np.int32)
        return self.block_table_rows(pages, pad_to), used
