"""The drop-in seam: chunks packed by the reference's own pack_chunk, run
through quail_b200's Qwen3Pipeline.forward_chunk.

tests/golden/host_<scenario>.npz holds every array Quail's loop handed its
model pipeline (input ids, positions, final rows, the KV scatter lists,
cu_a, the read groups with their block tables and merge source map, the
unified scatter/tail/tables), recorded from the reference itself by
tests/golden/make_golden.py. Here those arrays - not this repository's
packer - become loop.Chunk objects, in the order the reference launched
them, as Quail's loop would pass them to a B200 pipeline that replaced
Qwen3Pipeline (quail/backends/quail/executor/models/base.py:11-47,
qwen3.py:46-77). The GPU's answer margins must equal the oracle's replay of
the same arrays bit for bit: what the boundary promises is that Quail's
loop, unchanged, can drive the B200 path.

The model is the tiny test shape with Qwen3's vocabulary (the recorded
token ids run up to 150,000) so that the oracle replays the chunks in
seconds.
"""

import dataclasses
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import forward as of
from oracle import numerics as nx
from quail_b200 import _native as nat
from quail_b200.arena import KVArena
from quail_b200.loop import HostChunk
from quail_b200.model import TINY, random_weights
from quail_b200.pipeline import Qwen3Pipeline
from quail_b200.readout import AnswerRows

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
CFG = dataclasses.replace(TINY, name="tiny-qwen3-vocab", vocab=151936)
PAGES = {"cfg1_tree": 600, "cfg1_unified": 600, "stages_tree": 300, "stages_unified": 300}


def reference_chunks(name):
    """The recorded chunks of one scenario as HostChunk objects."""
    meta_json = json.loads((GOLDEN / f"host_{name}.json").read_text())
    arr = np.load(GOLDEN / f"host_{name}.npz")

    def get(key):
        return arr[key] if key in arr.files else None

    out = []
    for c, entry in enumerate(meta_json["chunks"]):
        p = f"c{c}_"
        reads = None
        if entry["reads"] is not None:
            reads = dict(rows=get(p + "reads_rows"), cu_q=get(p + "reads_cu_q"),
                         used=get(p + "reads_used"), table=get(p + "reads_table"),
                         source=get(p + "reads_source"), max_q=entry["reads"]["max_q"],
                         max_used=entry["reads"]["max_used"])
        unified = None
        if entry["unified"] is not None:
            unified = dict(src=get(p + "unified_src"), dst=get(p + "unified_dst"),
                           tail_src=get(p + "unified_tail_src"),
                           tail_dst=get(p + "unified_tail_dst"), used=get(p + "unified_used"),
                           table=get(p + "unified_table"), cu_q=get(p + "unified_cu_q"),
                           max_used=entry["unified"]["max_used"],
                           max_q=entry["unified"]["max_q"])
        meta = dict(layer=0, kv_src=get(p + "kv_src"), kv_dst=get(p + "kv_dst"), reads=reads,
                    unified=unified, canvas=None, cu_a=get(p + "cu_a"), max_a=entry["max_a"])
        out.append(HostChunk(input_ids=get(p + "input_ids"), positions=get(p + "positions"),
                             final_indices=get(p + "final_indices"), meta=meta,
                             attention_mode=entry["mode"], tokens=entry["tokens"],
                             layout=[tuple(x) for x in entry["layout"]]))
    return out


@pytest.mark.parametrize("name", sorted(PAGES))
def test_reference_packed_chunks_run_bit_exact(name):
    dev = torch.device("cuda")
    weights = random_weights(CFG, seed=7, device=dev)
    arena = KVArena(CFG.n_layers, PAGES[name], 16, CFG.n_kv, CFG.head_dim, device=dev)
    arena.pools.zero_()
    pipe = Qwen3Pipeline(torch, weights, arena)
    rows = AnswerRows(torch, weights)
    cpu_w = weights.to("cpu")
    cpu_arena = of.CpuArena(CFG.n_layers, arena.pool_rows, CFG.n_kv, CFG.head_dim)
    _, ans_w, tc, fc = cpu_w.answer_rows()
    hosts = reference_chunks(name)
    assert len(hosts) >= 2
    for i, host in enumerate(hosts):
        chunk = host.upload(torch, dev)
        got, _ = rows.margins(pipe.forward_chunk(chunk))
        torch.cuda.synchronize()
        assert nat.kernel_status(torch.cuda.current_device()) == 0
        want, _ = nx.answer_margin(of.forward_chunk(cpu_w, host, cpu_arena), ans_w, tc, fc)
        got = got.cpu().numpy()
        want = want.numpy().astype(np.float32)
        assert got.shape == want.shape == (len(host.final_indices),)
        assert np.array_equal(got.view(np.int32), want.view(np.int32)), (name, i, got, want)
