"""GPU parity of the activation quantisers against the reference.

Bit-exact (byte equality of aq and of the fp32 asc) with the golden vectors
from the reference's own code and with the oracle port on seeded inputs,
including every tail the reference tests (K % 32, K % 8, single rows),
strided and misaligned inputs, and special values.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from tests.golden.make_golden import NORM_CASES, QUANT_CASES, SILU_CASES

pytestmark = pytest.mark.gpu


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def assert_same(got, want):
    got, want = np.ascontiguousarray(got), np.ascontiguousarray(want)
    assert got.shape == want.shape
    if got.tobytes() != want.tobytes():
        bad = np.argwhere(got.view(np.uint8).reshape(-1) != want.view(np.uint8).reshape(-1))
        raise AssertionError(f"{len(bad)} bytes differ, first at {bad[:5].ravel()}")


@pytest.mark.parametrize("i", range(len(QUANT_CASES)))
def test_quantize_golden(cuda, golden, i):
    A = dev(golden[f"quant{i}_A"], cuda)
    aq, asc = ovb.s8_nk_quantize(A, u8=True)
    assert_same(host(aq), golden[f"quant{i}_aq"])
    assert_same(host(asc), golden[f"quant{i}_asc"])
    # the int8 form the GEMM consumes is the same numbers minus the zero point
    aq8, asc8 = ovb.s8_nk_quantize(A)
    q8 = host(aq8).astype(np.int16)
    ref = golden[f"quant{i}_aq"].astype(np.int16)
    K = A.shape[1]
    assert np.array_equal(q8[:, :K], ref[:, :K] - 128) and not q8[:, K:].any()
    assert_same(host(asc8), golden[f"quant{i}_asc"])


@pytest.mark.parametrize("i", range(len(NORM_CASES)))
def test_rmsnorm_quantize_golden(cuda, golden, i):
    x, w = dev(golden[f"norm{i}_x"], cuda), dev(golden[f"norm{i}_w"], cuda)
    aq, asc = ovb.rmsnorm_quantize_f32(x, w, 1e-6, u8=True)
    assert_same(host(aq), golden[f"norm{i}_aq"])
    assert_same(host(asc), golden[f"norm{i}_asc"])


@pytest.mark.parametrize("i", range(len(SILU_CASES)))
def test_silu_mul_quantize_golden(cuda, golden, i):
    g, u = dev(golden[f"silu{i}_g"], cuda), dev(golden[f"silu{i}_u"], cuda)
    aq, asc = ovb.silu_mul_quantize_f32(g, u, u8=True)
    assert_same(host(aq), golden[f"silu{i}_aq"])
    assert_same(host(asc), golden[f"silu{i}_asc"])


@pytest.mark.parametrize("M,K", [(400, 1024), (400, 2048), (1400, 1024), (129, 3072), (1, 1),
                                 (64, 1000), (7, 96), (3, 4), (5, 1020), (2, 1028)])
def test_quantizers_lm_shapes_vs_port(cuda, M, K):
    rng = np.random.default_rng(M * 7 + K)
    A = (rng.standard_normal((M, K)) * 4).astype(np.float32)
    w = rng.uniform(0.5, 1.5, K).astype(np.float32)
    g = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    for got, want in [
        (ovb.s8_nk_quantize(dev(A, cuda), u8=True), O.quantize(A)),
        (ovb.rmsnorm_quantize_f32(dev(A, cuda), dev(w, cuda), 1e-6, u8=True),
         O.rmsnorm_quantize(A, w, 1e-6)),
        (ovb.silu_mul_quantize_f32(dev(g, cuda), dev(A, cuda), u8=True),
         O.silu_mul_quantize(g, A)),
    ]:
        assert_same(host(got[0]), want[0])
        assert_same(host(got[1]), want[1])


@pytest.mark.parametrize("M", [1185, 15408])
def test_rmsnorm_quantize_many_rows(cuda, M):
    """Beyond 8 rows per SM the warp-per-row kernel runs: the same bytes as
    the reference restatement, in the int8 / u8 forms and the fp16 form
    fp16(q * asc)."""
    rng = np.random.default_rng(M)
    K = 1024
    A = (rng.standard_normal((M, K)) * 4).astype(np.float32)
    w = rng.uniform(0.5, 1.5, K).astype(np.float32)
    want_q, want_s = O.rmsnorm_quantize(A, w, 1e-6)
    got = ovb.rmsnorm_quantize_f32(dev(A, cuda), dev(w, cuda), 1e-6, u8=True)
    assert_same(host(got[0]), want_q)
    assert_same(host(got[1]), want_s)
    a16, s16 = ovb.rmsnorm_quantize_f32(dev(A, cuda), dev(w, cuda), 1e-6, f16=True)
    q = want_q.astype(np.int32) - 128
    deq = (q.reshape(M, -1, 32).astype(np.float32) * want_s[:, :, None]).reshape(M, -1)
    assert_same(host(a16), deq.astype(np.float16))
    assert_same(host(s16), want_s)


def test_rmsnorm_quantize_many_rows_all_forms_and_special_values(cuda):
    """The row-batched kernel (beyond 8 rows per SM) in every output form:
    int8 q, the fp16 form and fp16 of the normalised values themselves
    (OVB_AQ_F16_RAW), with blocks holding zeros, denormals, huge values, an
    infinity and a NaN (the x86-conversion path) among ordinary rows."""
    rng = np.random.default_rng(9)
    M, K = 2000, 1024
    A = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    A[3, :32] = 0.0
    A[5, 100:140] = 1e-40
    A[7, 64:96] = 3e37
    A[11, 200] = np.inf
    A[13, 300] = np.nan
    A[17] = 0.0
    w = rng.uniform(0.5, 1.5, K).astype(np.float32)
    want_q, want_s = O.rmsnorm_quantize(A, w, 1e-6)
    q8, s8 = ovb.rmsnorm_quantize_f32(dev(A, cuda), dev(w, cuda), 1e-6)
    assert_same(host(q8).view(np.uint8), (want_q.astype(np.int32) - 128).astype(np.int8).view(np.uint8))
    assert_same(host(s8), want_s)
    raw = ovb.rmsnorm_f16(dev(A, cuda), dev(w, cuda), 1e-6)
    want_raw = O.rmsnorm_into(A, w, 1e-6).astype(np.float16)
    np.testing.assert_array_equal(host(raw), want_raw)  # NaN payloads aside, the same values
    assert ovb.device_status() in (0, 16)  # the huge row leaves the fp16 range


def test_strided_and_misaligned_inputs(cuda):
    rng = np.random.default_rng(5)
    M, K = 33, 200
    big = rng.standard_normal((M, K + 13)).astype(np.float32)
    t = dev(big, cuda)[:, 1:K + 1]  # row stride K+13, start not 16-byte aligned
    aq, asc = ovb.s8_nk_quantize(t, u8=True)
    want = O.quantize(big[:, 1:K + 1])
    assert_same(host(aq), want[0])
    assert_same(host(asc), want[1])
    g = dev(big, cuda)[:, 5:5 + K]
    u = dev(big[::-1].copy(), cuda)[:, 2:2 + K]
    aq, asc = ovb.silu_mul_quantize_f32(g, u, u8=True)
    want = O.silu_mul_quantize(big[:, 5:5 + K], big[::-1][:, 2:2 + K])
    assert_same(host(aq), want[0])
    assert_same(host(asc), want[1])


def test_special_values(cuda):
    A = np.zeros((3, 70), np.float32)
    A[1, 3] = np.inf
    A[1, 5] = 2.0
    A[1, 35] = -1e-40          # denormal: must not be flushed
    A[2, :] = 1e-42
    A[2, 64:] = -3e38
    aq, asc = ovb.s8_nk_quantize(dev(A, cuda), u8=True)
    want = O.quantize(A)
    assert_same(host(aq), want[0])
    assert_same(host(asc), want[1])


def test_empty_is_noop(cuda):
    A = torch.zeros((0, 64), device=cuda)
    aq, asc = ovb.s8_nk_quantize(A)
    assert aq.shape[0] == 0 and asc.shape[0] == 0
