"""KV retention between operators: which document prefixes stay resident.

The decisions Quail's planner saves for an execution boundary
(quail/backends/quail/retention.py, quail/cost/retention.py) applied to a
quail_b200 KVArena:

- ``RetentionPolicy.priority``: the recompute seconds a retained prefix
  saves per page it holds, weighted by the probability of its next planned
  use; ties go to the later next use, then the higher document index.
  Lower priorities are evicted first.
- ``apply_retention``: at a boundary, free retained prefixes no later
  operator reads (their alias has no planned use, or the document is not a
  survivor), re-prioritise the rest under the boundary's policy and cap,
  and evict down to the cap.
- ``retain_after_join``: a finished join anchor offered for reuse at its
  next planned priority.

config carries the planner's numbers: linear_seconds (per token),
pair_seconds (per causal attention pair), optionally sliding_pair_seconds
and sliding_window, and cap_pages; uses maps an alias to (probability,
next use).
"""

from dataclasses import dataclass, field


def causal_pairs(n: float, window: int = 0) -> float:
    """Causal attention pairs of n tokens, each token's own key included
    (within a sliding window when window > 0) (quail/cost/work.py:51-55)."""
    if window and n > window:
        return window * n - window * (window - 1) / 2
    return n * (n + 1) / 2


@dataclass(frozen=True)
class RetentionPolicy:
    """Prices the next planned reuse of each (alias, document) prefix."""

    linear_seconds: float
    pair_seconds: float
    uses: dict = field(default_factory=dict)
    sliding_pair_seconds: float = 0.0
    sliding_window: int = 0

    def priority(self, key, tokens: int, pages: int) -> tuple:
        alias, document = key
        probability, next_use = self.uses.get(alias, (0.0, 0))
        seconds = (self.linear_seconds * tokens + self.pair_seconds * causal_pairs(tokens)
                   + self.sliding_pair_seconds * causal_pairs(tokens, self.sliding_window))
        return (probability * seconds / pages, -next_use, -document)


def policy(config, uses) -> RetentionPolicy:
    """The priority rule of one planned execution boundary."""
    return RetentionPolicy(config["linear_seconds"], config["pair_seconds"], uses,
                           sliding_pair_seconds=config.get("sliding_pair_seconds", 0.0),
                           sliding_window=config.get("sliding_window", 0))


def apply_retention(arena, config, uses, survivors=None) -> None:
    """Free the retained prefixes no later operator reads, re-prioritise the
    rest and evict down to the cap. survivors: alias -> documents still
    alive (a document of a listed alias that is not among them is freed)."""
    if not config:
        return
    alive = {alias: set(documents) for alias, documents in (survivors or {}).items()}
    for key in arena.retained_keys():
        alias, document = key
        if alias not in uses or (alias in alive and document not in alive[alias]):
            arena.free_key(key)
    arena.configure_retention(policy(config, uses), min(config["cap_pages"], arena.n_pages))
    arena.evict_retained(max(0, arena.retained_pages - arena.retention_cap_pages))


def retain_after_join(arena, key, tokens, config, uses) -> int:
    """Keep a finished anchor's prefix for reuse at its next planned priority;
    returns the pages that came free."""
    priority = None
    if config:
        priority = policy(config, uses).priority(key, tokens, arena.pages_needed(tokens))
    return arena.retain(key, tokens, priority=priority)
