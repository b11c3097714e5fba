"""CPU tests: pin the oracle port (oracle/ovb_oracle.c) to the reference.

The port is the checker for the GPU tests, so it is held to byte equality
with (a) the golden vectors made by the reference's own code
(tests/golden/make_golden.py) and (b) the reference library itself when it is
built and the host has AVX-VNNI.  Mirrors the reference's test strategy in
cpp/tests/test_gemm.cpp (double-precision oracle with lossless activations,
plus fused-equals-composed byte identities).
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

import oracle as O
from tests.golden.make_golden import (EXACT_CASES, GEMM_CASES, NORM_CASES, QUANT_CASES,
                                      SILU_CASES, cfg0_inputs)


def same(a, b) -> bool:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.dtype == b.dtype and a.shape == b.shape and a.tobytes() == b.tobytes()


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("i", range(len(QUANT_CASES)))
def test_port_quantize_golden(golden, i):
    aq, asc = O.quantize(golden[f"quant{i}_A"])
    assert same(aq, golden[f"quant{i}_aq"]) and same(asc, golden[f"quant{i}_asc"])


@pytest.mark.parametrize("i", range(len(NORM_CASES)))
def test_port_rmsnorm_quantize_golden(golden, i):
    aq, asc = O.rmsnorm_quantize(golden[f"norm{i}_x"], golden[f"norm{i}_w"], 1e-6)
    assert same(aq, golden[f"norm{i}_aq"]) and same(asc, golden[f"norm{i}_asc"])


@pytest.mark.parametrize("i", range(len(SILU_CASES)))
def test_port_silu_mul_quantize_golden(golden, i):
    aq, asc = O.silu_mul_quantize(golden[f"silu{i}_g"], golden[f"silu{i}_u"])
    assert same(aq, golden[f"silu{i}_aq"]) and same(asc, golden[f"silu{i}_asc"])


@pytest.mark.parametrize("i", range(len(GEMM_CASES)))
def test_port_gemm_golden(golden, i):
    M, N, K = GEMM_CASES[i]
    W, s = golden[f"gemm{i}_W"], golden[f"gemm{i}_s"]
    aq, asc = O.quantize(golden[f"gemm{i}_A"])
    assert same(O.linear_q(aq, asc, W, s, K), golden[f"gemm{i}_C"])
    assert same(O.linear_q(aq, asc, W, s, K, golden[f"gemm{i}_C0"]), golden[f"gemm{i}_Cadd"])
    # linear_s8_nk_packed quantises inside: same bytes as the hoisted path
    # (test_gemm.cpp:151-179).
    assert same(golden[f"gemm{i}_Cpk"], golden[f"gemm{i}_C"])
    assert same(golden[f"gemm{i}_Cpkadd"], golden[f"gemm{i}_Cadd"])


@pytest.mark.parametrize("i", range(len(EXACT_CASES)))
def test_port_exact_quantisation_against_double(golden, i):
    """test_gemm.cpp:114-146: with lossless activations the int8 path equals a
    double-precision product to 1e-5 relative."""
    M, N, K = EXACT_CASES[i]
    A, W, s = golden[f"exact{i}_A"], golden[f"exact{i}_W"], golden[f"exact{i}_s"]
    aq, asc = O.quantize(A)
    C = O.linear_q(aq, asc, W, s, K)
    assert same(C, golden[f"exact{i}_C"])
    R = (A.astype(np.float64) @ W.T.astype(np.float64)) * s.astype(np.float64)
    rel = np.abs(C - R).max() / (np.abs(R).max() + 1e-12)
    assert rel <= 1e-5


@pytest.mark.parametrize("i", range(3))
def test_port_sliced_golden(golden, i):
    A = golden[f"sliced{i}_A"]
    K = A.shape[1]
    aq, asc = O.quantize(A)
    for j in range(len(golden[f"sliced{i}_Ns"])):
        C = O.linear_q(aq, asc, golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"], K)
        assert same(C, golden[f"sliced{i}_C{j}"])


def test_port_block_products_exact():
    rng = np.random.default_rng(7)
    M, N, K = 5, 9, 77
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    aq, _ = O.quantize(A)
    P = O.block_products(aq, W, K)
    q = aq[:, :K].astype(np.int64) - 128
    for b in range((K + 31) // 32):
        sl = slice(32 * b, min(K, 32 * b + 32))
        assert np.array_equal(P[:, :, b], q[:, sl] @ W[:, sl].T.astype(np.int64))


def test_port_fused_equals_composed():
    """test_gemm.cpp:182-201 and :331-351 on the port."""
    rng = np.random.default_rng(3)
    for M, K in [(7, 69), (8, 1024)]:
        g = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        u = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        a1 = O.quantize(O.silu_mul(g, u))
        a2 = O.silu_mul_quantize(g, u)
        assert same(a1[0], a2[0]) and same(a1[1], a2[1])
    for M, K in [(7, 33), (8, 1024)]:
        x = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        w = rng.uniform(0.1, 1.1, K).astype(np.float32)
        a1 = O.quantize(O.rmsnorm_into(x, w, 1e-6))
        a2 = O.rmsnorm_quantize(x, w, 1e-6)
        assert same(a1[0], a2[0]) and same(a1[1], a2[1])


def test_port_special_values_match_reference_semantics():
    """Zero blocks give scale 0 and q = 0 (u8 128); an inf makes the block
    scale inf and every other element 0, the inf itself -127 (cvtps_epi32 of
    NaN is INT32_MIN, clamped)."""
    A = np.zeros((2, 40), np.float32)
    A[1, 3] = np.inf
    A[1, 5] = 2.0
    A[1, 35] = -1e-40  # denormal, alone in its block
    aq, asc = O.quantize(A)
    assert asc[0, 0] == 0 and np.all(aq[0, :40] == 128) and np.all(aq[0, 40:] == 0)
    assert np.isinf(asc[1, 0]) and aq[1, 3] == 1 and aq[1, 5] == 128
    assert asc[1, 1] == np.float32(1e-40) / np.float32(127) and aq[1, 35] == 1
    if O.ref_vnni():
        r = O.ref_quantize(A)
        assert same(aq, r[0]) and same(asc, r[1])


@pytest.mark.skipif(not O.ref_vnni(), reason="reference library not built or no AVX-VNNI")
def test_port_nan_blocks_match_reference():
    """Blocks holding NaNs: the reference folds each of its eight lanes with
    MAXPS (a NaN yields the other operand) and the lanes with std::max (which
    drops a NaN), so a NaN after a lane's maximum erases it.  The restatement
    reproduces that in every position: mid-lane, last vector, tail, all-NaN,
    for the three quantisers."""
    rng = np.random.default_rng(23)
    K = 70  # two whole blocks and a 6-element tail block
    A = (rng.standard_normal((8, K)) * 3).astype(np.float32)
    A[0, 1] = 50.0
    A[0, 9] = np.nan            # lane 1: 50 then NaN -> 50 lost
    A[1, 24 + 3] = np.nan       # lane 3, last vector of block 0
    A[2, 33] = np.nan           # block 1, first vector
    A[3, 66] = np.nan           # the tail block
    A[4, :32] = np.nan          # an all-NaN block
    A[5, 5] = np.nan
    A[5, 13] = 80.0             # lane 5: NaN then 80 -> 80 kept
    a1, a2 = O.quantize(A), O.ref_quantize(A)
    assert same(a1[0], a2[0]) and same(a1[1], a2[1])
    w = rng.uniform(0.5, 1.5, K).astype(np.float32)
    b1, b2 = O.rmsnorm_quantize(A, w, 1e-6), O.ref_rmsnorm_quantize(A, w, 1e-6)
    assert same(b1[0], b2[0]) and same(b1[1], b2[1])
    g = (rng.standard_normal((8, K)) * 3).astype(np.float32)
    c1, c2 = O.silu_mul_quantize(g, A), O.ref_silu_mul_quantize(g, A)
    assert same(c1[0], c2[0]) and same(c1[1], c2[1])


def test_port_cfg0_digests(cfg0_digests):
    """BASELINE config 0 at full size: the port reproduces the reference's
    outputs byte for byte (digests recorded by make_golden.py)."""
    A, W_kn, scale = cfg0_inputs()
    assert sha(A) == cfg0_digests["inputs_A"]
    assert sha(W_kn) == cfg0_digests["inputs_W_kn"]
    assert sha(scale) == cfg0_digests["inputs_scale"]
    aq, asc = O.quantize(A)
    assert sha(aq) == cfg0_digests["aq_u8"] and sha(asc) == cfg0_digests["asc"]
    C = O.linear_q(aq, asc, np.ascontiguousarray(W_kn.T), scale, 1024)
    assert sha(C) == cfg0_digests["C"]


@pytest.mark.skipif(not O.ref_vnni(), reason="reference library not built or no AVX-VNNI")
def test_port_matches_reference_live():
    rng = np.random.default_rng(11)
    for M, N, K in [(3, 64, 3072), (17, 40, 2048), (6, 130, 1000)]:
        A = (rng.standard_normal((M, K)) * 5).astype(np.float32)
        W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        s = (np.abs(rng.standard_normal(N)) * 0.02 / 127).astype(np.float32)
        aq, asc = O.quantize(A)
        r = O.ref_quantize(A)
        assert same(aq, r[0]) and same(asc, r[1])
        C0 = rng.standard_normal((M, N)).astype(np.float32)
        rp = O.RefPacked(W, s)
        assert same(O.linear_q(aq, asc, W, s, K), rp.linear_q(aq, asc))
        assert same(O.linear_q(aq, asc, W, s, K, C0), rp.linear_q(aq, asc, C0))
        w = rng.uniform(0.5, 1.5, K).astype(np.float32)
        a1, a2 = O.rmsnorm_quantize(A, w, 1e-6), O.ref_rmsnorm_quantize(A, w, 1e-6)
        assert same(a1[0], a2[0]) and same(a1[1], a2[1])
        g = (rng.standard_normal((M, K)) * 3).astype(np.float32)
        b1, b2 = O.silu_mul_quantize(g, A), O.ref_silu_mul_quantize(g, A)
        assert same(b1[0], b2[0]) and same(b1[1], b2[1])
