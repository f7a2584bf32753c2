"""The public entry point of the B200 AI.IF path: one loaded GPU.

``B200Executor`` is what Quail's per-GPU state holds after boot
(quail/backends/quail/worker.py:46-148: model, KVArena, pipeline).
``filter`` is the AiFilter branch of QuailModelExecution._execute_quail_node
(quail/backends/quail/backend.py:107-162): build the prefix tree when the
plan shares prefixes, run the filter loop to the end, return per-document
answers. Margins (yes - no logits) come back too, for parity checks.
``join`` is its AI join branch (backend.py:166-214: run_join over anchors
and per-stage partner lists) and ``score`` the AI.SCORE reranker
(quail/backends/quail/executor/score.py:46-66: run_join with the sigmoid
readout).
"""

import time
from dataclasses import dataclass, field

import numpy as np

from quail_b200 import loop
from quail_b200.arena import KVArena
from quail_b200.loop import InputStaging
from quail_b200.model import random_weights, requant_ue8m0, scales_are_ue8m0
from quail_b200.pipeline import build_pipeline
from quail_b200.readout import AnswerRows, AsyncAnswers, AsyncScores
from quail_b200.tokens import prefix_tree


@dataclass
class FilterResult:
    answers: dict                      # doc -> [0/1 per answered stage]
    bits: np.ndarray                   # last answered stage's bit per doc
    margins: np.ndarray                # last answered stage's margin per doc
    fresh_tokens: int
    borrowed_tokens: int
    chunks: int
    h2d_bytes: int
    d2h_bytes: int
    gpu_s: float
    wall_s: float
    timing: dict = field(default_factory=dict)


@dataclass
class JoinResult:
    answers: list                      # per stage: anchor -> row over its partners
    fresh_tokens: int
    borrowed_tokens: int
    chunks: int
    h2d_bytes: int
    d2h_bytes: int
    gpu_s: float
    wall_s: float
    n_anchors: int = 0
    skipped_pairs: int = 0             # EXISTS early stop: partners never computed

    def survivors(self, semantics="semi"):
        """Anchors the join keeps (backend.py:231-240): with "semi" (EXISTS)
        those with a TRUE partner at the last stage, with "anti" (NOT EXISTS)
        the rest, in anchor order."""
        if semantics not in ("semi", "anti"):
            raise ValueError(f"join semantics {semantics!r}: semi or anti")
        last = self.answers[-1] if self.answers else {}
        matched = {a for a, row in last.items() if any(row)}
        keep = (lambda a: a in matched) if semantics == "semi" else (lambda a: a not in matched)
        return [a for a in range(self.n_anchors) if keep(a)]


class B200Executor:
    """A model replica, its KV arena and pipeline on one GPU.

    Args:
        torch: the torch module.
        cfg: ModelConfig (FP8 Qwen3 shapes).
        n_pages: KV arena pages (16 tokens each).
        weights: loaded Weights, or None for seeded random-init weights.
        device: the CUDA device.
        scales: "fp32" (block scales as loaded) or "ue8m0" (the reference's
            UE8M0 mode, DeepGEMM's on sm_100: power-of-two scales, the
            block-scaled MMA; weights whose scales are not all powers of two
            are re-quantised in place first, as vLLM does at load).
    """

    def __init__(self, torch, cfg, n_pages, weights=None, device="cuda", seed=0,
                 scales="fp32"):
        if scales not in ("fp32", "ue8m0"):
            raise ValueError(f"scales {scales!r}: fp32 or ue8m0")
        self.torch = torch
        self.cfg = cfg
        self.device = torch.device(device)
        self.scales = scales
        self.weights = weights or random_weights(cfg, seed=seed, device=self.device)
        if scales == "ue8m0" and not scales_are_ue8m0(self.weights):
            with torch.cuda.device(self.device):
                requant_ue8m0(self.weights)
        self.arena = KVArena(cfg.n_layers, n_pages, 16, cfg.n_kv, cfg.head_dim,
                             device=self.device)
        self.pipeline = build_pipeline(torch, self.weights, self.arena,
                                       ue8m0=scales == "ue8m0")
        self.answer_rows = AnswerRows(torch, self.weights)
        self.budget = cfg.max_chunk_tokens
        # pinned host / device input buffers reused by every chunk upload
        self.staging = InputStaging(torch, self.device)

    def reset_arena(self):
        """Free every page (the pools stay allocated)."""
        self.arena.reset()

    def filter(self, documents, question_ids, *, budget=None, attention="tree",
               share_prefixes=True, arena_writes=True, limit=None, keys=None,
               retain_survivors=()) -> FilterResult:
        """Run one AI.IF filter over documents; returns answers and margins.

        keys: the documents' arena keys ((alias, document) pairs to retain
        them); retain_survivors: True or document positions whose KV stays
        resident after a TRUE for a later operator (quail_b200.retention
        manages it between operators)."""
        torch = self.torch
        t0 = time.perf_counter()
        tree = prefix_tree(documents, self.arena.page_tokens) if share_prefixes else None
        ans = AsyncAnswers(torch, self.answer_rows, keep_margins=True)
        last_margin = {}

        def done(finished):
            pass

        stats, timing = {}, {}
        order = []

        def on_chunk(host, groups):
            order.append([(doc, stage) for doc, stage, _ in groups])

        answers, spans, tokens = loop.run_filter(
            torch, self.arena, self.pipeline, ans, documents,
            [list(q) for q in question_ids], budget or self.budget, timing=timing,
            limit=limit, arena_writes=arena_writes, arena_keys=keys,
            retain_survivors=retain_survivors, attention_mode=attention,
            document_done=done, prefix_tree=tree, stats=stats, device=self.device,
            on_chunk=on_chunk, staging=self.staging)
        for groups, margins in zip(order, ans.margins):
            for (doc, _stage), m in zip(groups, margins):
                last_margin[doc] = float(m)
        torch.cuda.synchronize(self.device)
        wall = time.perf_counter() - t0
        n = len(documents)
        bits = np.array([answers.get(d, [0])[-1] for d in range(n)], dtype=np.uint8)
        margins = np.array([last_margin.get(d, np.nan) for d in range(n)], dtype=np.float32)
        gpu_s = sum(a.elapsed_time(b) for _, a, b in spans if a is not None) / 1000.0
        return FilterResult(answers=answers, bits=bits, margins=margins, fresh_tokens=tokens,
                            borrowed_tokens=stats.get("borrowed_tokens", 0),
                            chunks=stats.get("chunks", 0), h2d_bytes=stats.get("h2d_bytes", 0),
                            d2h_bytes=ans.d2h_bytes, gpu_s=gpu_s, wall_s=wall, timing=timing)

    def _join(self, readout, anchors, stage_suffixes, stage_frames, budget, attention,
              share_prefixes, partners, stop_at_true=False, stream_step=None,
              anchor_keys=None, anchor_done=None):
        torch = self.torch
        t0 = time.perf_counter()
        tree = prefix_tree(anchors, self.arena.page_tokens) if share_prefixes else None
        stats = {}
        answers, spans, tokens = loop.run_join(
            torch, self.arena, self.pipeline, readout, anchors,
            [[list(s) for s in sufs] for sufs in stage_suffixes], budget or self.budget,
            stage_frames=stage_frames, attention_mode=attention, prefix_tree=tree,
            anchor_partners=None if partners is None else (lambda key: partners[key]),
            stats=stats, device=self.device, stop_at_true=stop_at_true,
            stream_step=stream_step, staging=self.staging, anchor_keys=anchor_keys,
            anchor_done=anchor_done)
        torch.cuda.synchronize(self.device)
        wall = time.perf_counter() - t0
        gpu_s = sum(a.elapsed_time(b) for _, a, b in spans if a is not None) / 1000.0
        return JoinResult(answers=answers, fresh_tokens=tokens,
                          borrowed_tokens=stats.get("borrowed_tokens", 0),
                          chunks=stats.get("chunks", 0), h2d_bytes=stats.get("h2d_bytes", 0),
                          d2h_bytes=readout.d2h_bytes, gpu_s=gpu_s, wall_s=wall,
                          n_anchors=len(anchors),
                          skipped_pairs=stats.get("skipped_partners", 0))

    def join(self, anchors, stage_suffixes, *, stage_frames=None, budget=None,
             attention="tree", share_prefixes=True, partners=None,
             exists_stop=False, anchor_keys=None, anchor_done=None) -> JoinResult:
        """Run one AI join: every anchor against its partners, stage by stage
        (an anchor continues to stage j + 1 once a stage-j partner answered
        TRUE). partners: per anchor, per stage, partner indices or None.
        exists_stop: for an EXISTS (semi) or NOT EXISTS (anti) join, stop an
        anchor's last-stage stream at its first TRUE answer (partners not yet
        launched are skipped; survivors are unchanged), with the anchors'
        streams interleaved one partner per anchor per chunk. anchor_keys:
        the anchors' arena keys (a retained key's KV is reused as a resident
        anchor); anchor_done(a, row): the finished anchor's free or retain
        decision (retention.retain_after_join), else it is freed."""
        ans = AsyncAnswers(self.torch, self.answer_rows)
        return self._join(ans, anchors, stage_suffixes, stage_frames, budget, attention,
                          share_prefixes, partners, stop_at_true=exists_stop,
                          stream_step=1 if exists_stop else None, anchor_keys=anchor_keys,
                          anchor_done=anchor_done)

    def score(self, anchors, suffixes, *, budget=None, attention="tree",
              share_prefixes=True, partners=None) -> JoinResult:
        """AI.SCORE: sigmoid(yes - no) per (anchor, partner) as float32 rows;
        partners: per anchor, the partner indices it scores, or None for all."""
        ans = AsyncScores(self.torch, self.answer_rows)
        per = None if partners is None else [[p] for p in partners]
        return self._join(ans, anchors, [suffixes], None, budget, attention, share_prefixes,
                          per)
