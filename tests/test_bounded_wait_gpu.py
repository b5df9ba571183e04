"""Failure detection on the device without a GPU fault: every wait inside a
kernel is bounded, and a wait that runs out records a status code and lets
the kernel return, so the context stays usable.

The test makes a wait run out on purpose -- an mbarrier phase nobody arrives
on, and a global flag nobody sets -- with a 1 ms limit passed at run time,
then checks the status word, the time actually waited, and that the next
kernels still run. Would fail if a wait were unbounded (the test would hang
until its timeout), ignored its limit, recorded no status, or left the
context broken.
"""

import pytest
import torch

from elysium_wan_b200 import ops

pytestmark = pytest.mark.gpu

TIMEOUT_SMEM_FULL = 1  # status codes of csrc/common.cuh
TIMEOUT_PEER = 5


@pytest.mark.timeout(60)
@pytest.mark.parametrize("mode,code", [(0, TIMEOUT_SMEM_FULL), (1, TIMEOUT_PEER)])
def test_wait_that_nobody_releases_gives_up_and_reports(cuda, mode, code):
    ext = ops.ext()
    assert ext.status_read_clear() == 0
    limit_ns = 1_000_000  # 1 ms
    done, waited = ext.wait_probe(mode, False, limit_ns)
    assert done == 0
    assert limit_ns <= waited < 200 * limit_ns, waited
    assert ext.status_read_clear() == code
    assert ext.status_read_clear() == 0  # read-and-clear
    # the context is intact: the same wait, released, completes at once, and
    # a kernel of the model runs and is right
    done, waited = ext.wait_probe(mode, True, limit_ns)
    assert done == 1 and waited < limit_ns
    assert ext.status_read_clear() == 0
    x = torch.randn(256, 512, device=cuda).to(torch.bfloat16)
    w = torch.randn(384, 512, device=cuda).to(torch.bfloat16)
    y = torch.empty(256, 384, dtype=torch.bfloat16, device=cuda)
    ops.gemm(x, w, y, ops.EPI_BF16)
    ref = (x.float() @ w.float().t())
    torch.cuda.synchronize()
    assert torch.allclose(y.float(), ref, rtol=2e-2, atol=2e-1)
    assert ext.status_read_clear() == 0
