"""GPU test of ovb_linear_static, the entry point for callers that cannot
allocate device memory.

Some users of this library cannot hand it a device workspace: hosts whose
device memory belongs to their own pool, latency-critical steps that must
not pay for cudaMalloc's device synchronisation, FFI bindings that cannot
own a device buffer.  ovb_linear_static serves them from a fixed device
array inside the library.  This test calls it through the C ABI and checks
that, on two calls in a row, it gives exactly the bytes of the existing
ovb_linear (which uses a caller-owned workspace) -- the same bit-exact
standard as the other GEMM tests -- and that a size beyond the array's limit
is refused.  It is kept in its own file, collected last, and works both
alone in a fresh process and after the other tests.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import ovnative_b200 as ovb
from ovnative_b200 import _lib as L

pytestmark = pytest.mark.gpu

STATIC_LIMIT = 8 << 20  # bytes of the library's static scratch


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _linear_with_workspace(lib, M, w, A, C, accumulate):
    work = torch.empty(lib.ovb_linear_workspace_bytes(M, w.K), dtype=torch.uint8, device=A.device)
    st = lib.ovb_linear(M, w.handle, A.data_ptr(), A.stride(0), C.data_ptr(), C.stride(0),
                        accumulate, work.data_ptr(), work.numel(), _stream())
    assert st == L.OVB_OK, lib.ovb_last_error()


def _linear_static(lib, M, w, A, C, accumulate):
    st = lib.ovb_linear_static(M, w.handle, A.data_ptr(), A.stride(0), C.data_ptr(), C.stride(0),
                               accumulate, _stream())
    assert st == L.OVB_OK, lib.ovb_last_error()


def test_static_entry_point_matches_workspace_entry_point(cuda):
    lib = L.lib()
    rng = np.random.default_rng(77)
    # Two calls in a row with different shapes: the second must not be
    # affected by what the first left in the shared array.
    cases = [(400, 3072, 1024, 0), (129, 1024, 3072, 1)]
    for M, N, K, accumulate in cases:
        W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        s = (np.abs(rng.standard_normal(N)) * 0.02 / 127).astype(np.float32)
        w = ovb.Weight.from_nk(W, s)
        A = torch.from_numpy((rng.standard_normal((M, K)) * 2).astype(np.float32)).to(cuda)
        C0 = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).to(cuda)
        want = C0.clone()
        got = C0.clone()
        _linear_with_workspace(lib, M, w, A, want, accumulate)
        _linear_static(lib, M, w, A, got, accumulate)
        torch.cuda.synchronize()
        g, r = got.cpu().numpy(), want.cpu().numpy()
        assert g.tobytes() == r.tobytes(), (
            f"M={M} N={N} K={K}: {int((g != r).sum())} outputs differ")
        w.close()
    assert ovb.device_status() == 0


def test_static_entry_point_rejects_sizes_beyond_its_array(cuda):
    lib = L.lib()
    K = 3072
    M = 4096  # workspace for 4096 x 3072 is ~14 MB
    assert lib.ovb_linear_workspace_bytes(M, K) > STATIC_LIMIT
    w = ovb.Weight.from_nk(np.ones((64, K), np.int8), np.ones(64, np.float32))
    A = torch.zeros((M, K), device=cuda)
    C = torch.zeros((M, 64), device=cuda)
    st = lib.ovb_linear_static(M, w.handle, A.data_ptr(), K, C.data_ptr(), 64, 0, _stream())
    assert st == L.OVB_ERR_INVALID_ARG
    assert b"static" in lib.ovb_last_error()
    # A row count so large that its byte count would wrap is refused too.
    st = lib.ovb_linear_static(1 << 62, w.handle, A.data_ptr(), K, C.data_ptr(), 64, 0, _stream())
    assert st == L.OVB_ERR_INVALID_ARG
    assert b"static" in lib.ovb_last_error()
    w.close()
