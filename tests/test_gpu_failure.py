"""Failure detection without a GPU fault: every wait inside the kernels is
bounded, and a wait that gives up sets a bit of the device status word that
the host reads with ovb_device_status.  The self-test kernel waits on an
mbarrier that nothing arrives on; its wait runs out (~1 s), the kernel ends
normally and the context keeps working."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from ovnative_b200 import _lib as L

pytestmark = pytest.mark.gpu


def test_bounded_wait_timeout_sets_status_and_context_survives(cuda):
    assert ovb.device_status() == 0
    L.check(L.lib().ovb_selftest_wait_timeout(torch.cuda.current_stream().cuda_stream))
    assert ovb.device_status() == 64
    assert ovb.device_status() == 0  # reading clears it
    # The context still runs GEMMs, bit-exactly.
    rng = np.random.default_rng(5)
    M, N, K = 64, 256, 512
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (np.abs(rng.standard_normal(N)) * 0.02 / 127).astype(np.float32)
    w = ovb.Weight.from_nk(W, s)
    C = ovb.linear_s8_nk_packed(torch.from_numpy(A).to(cuda), w)
    aq, asc = O.quantize(A)
    assert C.cpu().numpy().tobytes() == O.linear_q(aq, asc, W, s, K).tobytes()
    assert ovb.device_status() == 0
    w.close()
