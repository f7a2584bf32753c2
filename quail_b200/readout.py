"""Answer readouts over the retained TRUE/FALSE rows of the output head.

Same seam as Quail's readout.py (quail/backends/quail/executor/readout.py:
17-117): ``AnswerRows`` holds the retained head rows, ``AsyncAnswers``
(AI_FILTER / AI_JOIN bits) and ``AsyncScores`` (AI.SCORE sigmoids) score
the forward pass's normed rows without stalling the stream - submit()
launches the readout kernel and a non-blocking copy into pinned memory and
records an event; result() waits on that event.
"""

import numpy as np

from quail_b200 import _native as nat


class AnswerRows:
    """The retained output rows for one query's two answer classes."""

    def __init__(self, torch, weights, true_ids=None, false_ids=None):
        cfg = weights.config
        true_ids = tuple(cfg.true_ids if true_ids is None else true_ids)
        false_ids = tuple(cfg.false_ids if false_ids is None else false_ids)
        self.allowed = sorted(set(true_ids) | set(false_ids))
        if len(self.allowed) > 16:
            raise ValueError("at most 16 answer token ids")
        idx = torch.tensor(self.allowed, device=weights.device)
        self.weights = weights.embed.index_select(0, idx).contiguous()
        true_set, false_set = set(true_ids), set(false_ids)
        self.true_cols = torch.tensor([i for i, t in enumerate(self.allowed) if t in true_set],
                                      dtype=torch.int32, device=weights.device)
        self.false_cols = torch.tensor([i for i, t in enumerate(self.allowed) if t in false_set],
                                       dtype=torch.int32, device=weights.device)
        self.torch = torch

    def scores(self, normed):
        """sigmoid(yes - no) f32 device tensor (fp32 logits) for each row."""
        t = self.torch
        n, h = normed.shape
        score = t.empty(n, dtype=t.float32, device=normed.device)
        nat.call("qb_answer_score", nat.ptr(normed), n, h, nat.ptr(self.weights),
                 len(self.allowed), nat.ptr(self.true_cols), self.true_cols.shape[0],
                 nat.ptr(self.false_cols), self.false_cols.shape[0], nat.ptr(score),
                 nat.stream_handle(t))
        return score

    def margins(self, normed):
        """(margin f32, bit u8) device tensors for each normed row."""
        t = self.torch
        n, h = normed.shape
        margin = t.empty(n, dtype=t.float32, device=normed.device)
        bits = t.empty(n, dtype=t.uint8, device=normed.device)
        nat.call("qb_answer_margin", nat.ptr(normed), n, h, nat.ptr(self.weights),
                 len(self.allowed), nat.ptr(self.true_cols), self.true_cols.shape[0],
                 nat.ptr(self.false_cols), self.false_cols.shape[0], nat.ptr(margin),
                 nat.ptr(bits), nat.stream_handle(t))
        return margin, bits


class AsyncAnswers:
    """Non-blocking TRUE/FALSE readout; keeps each row's margin too."""

    dtype = None

    def __init__(self, torch, rows: AnswerRows, keep_margins=False):
        self.torch = torch
        self.rows = rows
        self.keep_margins = keep_margins
        self.margins = []
        self.d2h_bytes = 0

    def submit(self, normed):
        t = self.torch
        margin, bits = self.rows.margins(normed)
        n = bits.shape[0]
        host_bits = t.empty(n, dtype=t.uint8, pin_memory=True)
        host_bits.copy_(bits, non_blocking=True)
        host_margin = None
        if self.keep_margins:
            host_margin = t.empty(n, dtype=t.float32, pin_memory=True)
            host_margin.copy_(margin, non_blocking=True)
        self.d2h_bytes += n * (5 if self.keep_margins else 1)
        event = t.cuda.Event()
        event.record()
        return event, host_bits, host_margin

    def result(self, handle):
        event, host_bits, host_margin = handle
        event.synchronize()
        if host_margin is not None:
            self.margins.append(host_margin.numpy().copy())
        return [int(b) for b in host_bits.tolist()]


class AsyncScores:
    """Non-blocking yes-against-no sigmoid readout for AI.SCORE
    (readout.py:88-117): result() returns float32 scores."""

    dtype = np.float32

    def __init__(self, torch, rows: AnswerRows):
        self.torch = torch
        self.rows = rows
        self.available = []
        self.d2h_bytes = 0

    def submit(self, normed):
        t = self.torch
        scores = self.rows.scores(normed)
        n = scores.shape[0]
        host = self.available.pop() if self.available else None
        if host is None or host.numel() < n:
            host = t.empty(n, dtype=t.float32, pin_memory=True)
        host[:n].copy_(scores, non_blocking=True)
        self.d2h_bytes += 4 * n
        event = t.cuda.Event()
        event.record()
        return event, host, n

    def result(self, handle):
        event, host, count = handle
        event.synchronize()
        self.available.append(host)
        return host[:count].numpy().copy()
