"""The give-up path of the tcgen05 kernels' bounded waits, without a fault.

Every wait a GEMM block makes on another of its roles (the TMA producer,
the MMA issuer, the scale loader, the epilogue) is bounded: when one runs
out it sets a status bit, raises the block's abort flag so the other roles
stop at their next wait, drains the copies and MMAs already issued and frees
TMEM before the block exits. qb_set_wait_limit shortens that limit to 1 ns,
so the waits of a real GEMM give up while the GEMM runs normally; the test
then checks that the status word reports it, that reading the word clears
it, and that the next GEMM on the same device (which allocates TMEM on
every SM again) runs and gives the same bits as before. Nothing here makes
a GPU fault or hang: the copies and MMAs in flight end on their own, and
the drains that wait for them keep their one-second limit.
"""

import pytest
import torch

from oracle import numerics as nx
from quail_b200 import _native as nat
from quail_b200.engine import Engine, QuantRows
from quail_b200.model import TINY

pytestmark = pytest.mark.gpu

GEMM_BITS = 0xF  # STATUS_GEMM_PRODUCER | _MMA | _EPILOGUE | _DRAIN


class _Arena:
    pool_rows = 64


def _operands(m, n, k, dev):
    g = torch.Generator().manual_seed(17)
    aq, as_ = nx.quant_groups(torch.randn(m, k, generator=g))
    wq = torch.randn(n, k, generator=g).to(torch.float8_e4m3fn)
    ws = torch.exp(-4.0 + 0.3 * torch.randn(n // 128, k // 128, generator=g))
    return QuantRows(aq.to(dev), as_.to(dev).contiguous(), m), wq.to(dev), ws.to(dev)


def test_gemm_waits_give_up_and_the_device_recovers():
    dev = torch.device("cuda")
    d = torch.cuda.current_device()
    eng = Engine(torch, _Arena(), TINY)
    # a down-projection shape: 76 K blocks, two waves of tiles
    x, w, s = _operands(16384, 2560, 9728, dev)
    assert nat.kernel_status(d) == 0
    want = eng.gemm(x, w, s)
    torch.cuda.synchronize()
    assert nat.kernel_status(d) == 0

    nat.set_wait_limit(d, 1)
    try:
        eng.gemm(x, w, s)
        torch.cuda.synchronize()
        seen = nat.kernel_status(d)
    finally:
        nat.set_wait_limit(d, 0)
    assert seen & GEMM_BITS, f"no wait gave up (status {seen:#x})"
    assert nat.kernel_status(d) == 0, "reading the status word clears it"

    # TMEM was freed on every SM: the next GEMM allocates it again and
    # computes the same bits
    again = eng.gemm(x, w, s)
    torch.cuda.synchronize()
    assert nat.kernel_status(d) == 0
    assert torch.equal(again.view(torch.int16), want.view(torch.int16))
