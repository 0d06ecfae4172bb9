"""Device-side waits are bounded: a wait nothing satisfies runs out, the
kernel returns, the status word says so, and the context stays usable.

No GPU is faulted: the probe waits on an mbarrier that nobody arrives on,
with a 50 ms limit, and returns normally."""

import pytest
import torch

from rdna3_fastmm import _native

pytestmark = pytest.mark.gpu


def test_unsatisfied_wait_times_out_and_reports():
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    _native.device_status(0, reset=True)
    _native.test_bounded_wait(50_000_000, device)  # 50 ms
    status, site = _native.device_status(0, reset=True)
    assert status & _native.FMM_STATUS_TIMEOUT
    assert site >> 16 == 7  # the probe's wait site
    # the context is still healthy: ordinary work runs and the status is clear
    x = torch.ones(1024, device=device)
    assert float(x.sum()) == 1024.0
    assert _native.device_status(0)[0] == 0
