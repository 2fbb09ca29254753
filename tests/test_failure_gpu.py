"""A cross-GPU wait that runs out returns an error status instead of hanging (GPU).

The GEMM -> all-reduce consumer (the fused RMSNorm) waits on a counter that
the producing GEMMs on every rank bump. Here nothing bumps it: the wait gives
up after its limit (about 2 s), records the timeout and the site in the
library's status word, and the kernel finishes, so the context stays usable.
"""
import time

import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.api.driver import DeviceStatusError

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_with_status():
    ops.require()
    ops.status(clear=True)
    n = 512
    x = torch.zeros(2, n, dtype=torch.float32, device="cuda")
    w = torch.ones(n, dtype=torch.bfloat16, device="cuda")
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")   # a counter nobody signals
    state = torch.zeros(2, dtype=torch.int64, device="cuda")
    t0 = time.monotonic()
    y = ops.rmsnorm(x, w, 1e-6, sync=(flag, state, 1))
    torch.cuda.synchronize()
    dt = time.monotonic() - t0
    st = ops.status(clear=True)
    assert st & 0xFF == 2 and (st >> 8) == 201, hex(st)
    assert "peer wait timed out" in str(DeviceStatusError(st))
    assert 1.0 < dt < 30.0
    assert torch.isfinite(y.float()).all()
    # the context is still usable
    z = ops.rmsnorm(torch.ones(2, n, dtype=torch.bfloat16, device="cuda"), w, 1e-6)
    torch.cuda.synchronize()
    assert ops.status() == 0 and torch.allclose(z.float(), torch.ones_like(z.float()), atol=1e-2)
