"""The failure path every waiting kernel shares, exercised without a fault, a trap or an endless loop:
sa_wait_selftest waits, with the library's bounded mbarrier wait, for a barrier phase that nothing
completes.  The wait gives up after its limit, SA_DEV_WAIT_TEST lands in the device status word, and
the context stays usable for the next kernel."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda')


@pytest.mark.parametrize('limit_ms', [2, 20])
def test_expired_wait_sets_status_and_context_survives(limit_ms):
    from sm120_attn import _native as N
    from sm120_attn import ops
    ops.read_status(DEV)                                 # start from a clear word
    st = ops.status_word(DEV)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    N.call('sa_wait_selftest', ops._p(st), limit_ms * 1_000_000, ops._stream(DEV))
    b.record()
    torch.cuda.synchronize()
    assert a.elapsed_time(b) >= 0.9 * limit_ms           # the wait ran to its limit
    assert a.elapsed_time(b) < 2000                      # and no further
    assert ops.read_status(DEV) == N.SA_DEV_WAIT_TEST
    # a kernel of the library runs on the same context and leaves the word clear
    x = torch.randn(256, 4, 128, device=DEV).to(torch.bfloat16)
    m = ops.absmax(x, per_head=False)
    torch.cuda.synchronize()
    assert float(m.reshape(-1)[0]) == float(x.float().abs().max())
    ops.check_status(DEV)
