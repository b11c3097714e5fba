"""GPU parity of the tcgen05 int8 GEMM against the reference.

* per-32-k block int32 products: bit-exact against exact integer arithmetic;
* fp32 outputs: bit-exact against the reference's outputs (golden vectors
  from its own code, and the oracle port) -- stricter than the stated
  tolerance rel-L2 <= 1e-3 and max-abs <= 1e-2 * rms, which is also checked
  so a failure says how far off a result is;
* every entry point of the contract: plain, residual-add, quantise-inside,
  sliced, [K,N] and [N,K] weight layouts; M / N / K tails; argument errors.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from tests.golden.make_golden import EXACT_CASES, GEMM_CASES, cfg0_inputs

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3       # north-star tolerance on fp32 outputs
MAX_ABS_RMS = 1e-2  # max |delta| <= 1e-2 * rms(reference)


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def check_close_and_exact(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    d = got.astype(np.float64) - want.astype(np.float64)
    rms = np.sqrt(np.mean(want.astype(np.float64) ** 2)) + 1e-30
    rel = np.linalg.norm(d) / (np.linalg.norm(want.astype(np.float64)) + 1e-30)
    assert rel <= REL_L2, f"rel-L2 {rel:.3e}"
    assert np.abs(d).max() <= MAX_ABS_RMS * rms, f"max-abs {np.abs(d).max():.3e}"
    nbad = int((got.view(np.uint32) != want.view(np.uint32)).sum())
    assert nbad == 0, f"{nbad} of {got.size} outputs not bit-identical (rel-L2 {rel:.2e})"


@pytest.mark.parametrize("i", range(len(GEMM_CASES)))
def test_gemm_golden(cuda, golden, i):
    M, N, K = GEMM_CASES[i]
    w = ovb.Weight.from_nk(golden[f"gemm{i}_W"], golden[f"gemm{i}_s"])
    A = dev(golden[f"gemm{i}_A"], cuda)
    aq, asc = ovb.s8_nk_quantize(A)
    check_close_and_exact(host(ovb.linear_s8_nk_packed_q(aq, asc, w)), golden[f"gemm{i}_C"])
    C = dev(golden[f"gemm{i}_C0"], cuda)
    ovb.linear_s8_nk_packed_q_add(aq, asc, w, C)
    check_close_and_exact(host(C), golden[f"gemm{i}_Cadd"])
    check_close_and_exact(host(ovb.linear_s8_nk_packed(A, w)), golden[f"gemm{i}_Cpk"])
    C = dev(golden[f"gemm{i}_C0"], cuda)
    ovb.linear_s8_nk_packed_add(A, w, C)
    check_close_and_exact(host(C), golden[f"gemm{i}_Cpkadd"])
    assert ovb.device_status() == 0


@pytest.mark.parametrize("i", range(len(EXACT_CASES)))
def test_gemm_exact_quantisation(cuda, golden, i):
    """test_gemm.cpp:114-146 on the GPU: lossless activations, so the result
    equals a double-precision product to 1e-5 (and the reference bit for bit)."""
    M, N, K = EXACT_CASES[i]
    A, W, s = golden[f"exact{i}_A"], golden[f"exact{i}_W"], golden[f"exact{i}_s"]
    w = ovb.Weight.from_nk(W, s)
    C = host(ovb.linear_s8_nk_packed(dev(A, cuda), w))
    check_close_and_exact(C, golden[f"exact{i}_C"])
    R = (A.astype(np.float64) @ W.T.astype(np.float64)) * s.astype(np.float64)
    assert np.abs(C - R).max() / (np.abs(R).max() + 1e-12) <= 1e-5


@pytest.mark.parametrize("i", range(3))
def test_gemm_sliced_golden(cuda, golden, i):
    Ns = [int(n) for n in golden[f"sliced{i}_Ns"]]
    parts = [ovb.Weight.from_nk(golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"])
             for j in range(len(Ns))]
    wc = ovb.Weight.concat(parts)
    A = dev(golden[f"sliced{i}_A"], cuda)
    aq, asc = ovb.s8_nk_quantize(A)
    Cs = [torch.full((A.shape[0], n), float("nan"), device=cuda) for n in Ns]
    ovb.linear_s8_nk_packed_q_sliced(aq, asc, wc, Cs)
    for j, c in enumerate(Cs):
        check_close_and_exact(host(c), golden[f"sliced{i}_C{j}"])
        # sliced == per-slice GEMM, byte for byte (test_gemm.cpp:240-297)
        check_close_and_exact(host(ovb.linear_s8_nk_packed_q(aq, asc, parts[j])), host(c))


@pytest.mark.parametrize("M,N,K", [(1, 8, 32), (127, 130, 64), (128, 128, 1024), (129, 257, 96),
                                   (300, 64, 3072), (40, 1000, 33)])
def test_block_products_bit_exact(cuda, M, N, K):
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    w = ovb.Weight.from_nk(W, np.ones(N, np.float32))
    aq, _ = ovb.s8_nk_quantize(dev(A, cuda))
    P = host(ovb.block_products(aq, w))
    aq_u8, _ = O.quantize(A)
    assert np.array_equal(P, O.block_products(aq_u8, W, K))


def test_kn_and_nk_layouts_agree(cuda):
    rng = np.random.default_rng(9)
    N, K, M = 3072, 1024, 64
    W_kn = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    s = (np.abs(rng.standard_normal(N)) * 0.02 / 127).astype(np.float32)
    w1 = ovb.Weight.from_kn(W_kn, s)
    w2 = ovb.Weight.from_nk(np.ascontiguousarray(W_kn.T), s)
    We, se = w1.export()
    assert np.array_equal(We, W_kn.T) and np.array_equal(se, s)
    # device-resident source, ragged K
    Wd = rng.integers(-127, 128, size=(100, 45), dtype=np.int8)
    w3 = ovb.Weight.from_kn(dev(Wd, cuda), dev(np.ones(45, np.float32), cuda))
    assert np.array_equal(w3.export()[0], Wd.T)
    A = dev(rng.standard_normal((M, K)).astype(np.float32), cuda)
    aq, asc = ovb.s8_nk_quantize(A)
    c1 = host(ovb.linear_s8_nk_packed_q(aq, asc, w1))
    c2 = host(ovb.linear_s8_nk_packed_q(aq, asc, w2))
    assert c1.tobytes() == c2.tobytes()


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_cfg0_full_size_matches_reference_digest(cuda, cfg0_digests):
    """BASELINE config 0 (M=256, K=1024, N=3072, [K,N] weights): the GPU's aq,
    asc and fp32 C have the same SHA-256 as the reference's."""
    A, W_kn, scale = cfg0_inputs()
    assert sha(A) == cfg0_digests["inputs_A"]
    w = ovb.Weight.from_kn(W_kn, scale)
    Ad = dev(A, cuda)
    aq_u8, asc = ovb.s8_nk_quantize(Ad, u8=True)
    assert sha(host(aq_u8)) == cfg0_digests["aq_u8"]
    assert sha(host(asc)) == cfg0_digests["asc"]
    C = host(ovb.linear_s8_nk_packed(Ad, w))
    assert sha(C) == cfg0_digests["C"]


# LM projection shapes (N, K) and M values of the M-sweep; rows are
# independent, so a row subset is checked against the port.
LM_SHAPES = [(2048, 1024), (1024, 1024), (1024, 2048), (4096, 1024), (6144, 1024),
             (1024, 3072), (8200, 1024)]


@pytest.mark.parametrize("M", [16, 64, 256, 1024])
@pytest.mark.parametrize("N,K", LM_SHAPES)
def test_lm_shapes_rows_vs_port(cuda, M, N, K):
    rng = np.random.default_rng(N * 3 + K + M)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (np.abs(rng.standard_normal(N)) * 0.02 / 127).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = ovb.Weight.from_nk(W, s)
    C = dev(C0, cuda)
    ovb.linear_s8_nk_packed_add(dev(A, cuda), w, C)
    got = host(C)
    rows = np.unique(np.concatenate([[0, M - 1], rng.integers(0, M, 3)]))
    aq, asc = O.quantize(A[rows])
    want = O.linear_q(aq, asc, W, s, K, C0[rows])
    check_close_and_exact(got[rows], want)


def test_argument_errors(cuda):
    rng = np.random.default_rng(1)
    w = ovb.Weight.from_nk(rng.integers(-127, 128, (192, 64), dtype=np.int8),
                           np.ones(192, np.float32))
    aq, asc = ovb.s8_nk_quantize(torch.randn(4, 64, device=cuda))
    with pytest.raises(ValueError, match="multiple of 64"):
        ovb.linear_s8_nk_packed_q_sliced(aq, asc, w, [torch.empty(4, 100, device=cuda),
                                                      torch.empty(4, 92, device=cuda)])
    with pytest.raises(ValueError, match="add up"):
        ovb.linear_s8_nk_packed_q_sliced(aq, asc, w, [torch.empty(4, 128, device=cuda)])
    with pytest.raises(ValueError, match="ldc"):
        ovb.linear_s8_nk_packed_q(aq, asc, w, torch.empty(4, 64, device=cuda))
    raw = torch.empty(4 * 64 + 16, dtype=torch.int8, device=cuda)
    with pytest.raises(ValueError, match="aligned"):
        ovb.linear_s8_nk_packed_q(raw[1:1 + 256].view(4, 64), asc, w)
    # M = 0 is a silent no-op, as in the reference
    out = ovb.linear_s8_nk_packed_q(aq[:0], asc[:0], w)
    assert out.shape == (0, 192)
    assert ovb.device_status() == 0


# K = 33, 96, 160, 1056: 2, 3, 5, 33 quantisation blocks, so the last TMEM
# slot of a tile holds fewer blocks than the slot size (1, 2 or 4 by width).
WIDTH_CASES = [(1, 8, 33), (127, 130, 96), (129, 257, 160), (300, 1000, 1056), (400, 1024, 2048)]


@pytest.mark.parametrize("tile_n", [128, 64, 32])
@pytest.mark.parametrize("M,N,K", WIDTH_CASES)
def test_every_tile_width_bit_exact(cuda, monkeypatch, tile_n, M, N, K):
    """The GEMM is built for output tiles 128, 64 and 32 columns wide; the
    host picks one by shape.  Force each and check the plain, residual-add
    and products outputs against the port."""
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    rng = np.random.default_rng(M * 7 + N + K)
    A = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (np.abs(rng.standard_normal(N)) * 0.02 / 127 + 1e-6).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = ovb.Weight.from_nk(W, s)
    aq, asc = ovb.s8_nk_quantize(dev(A, cuda))
    aq_h, asc_h = O.quantize(A)
    check_close_and_exact(host(ovb.linear_s8_nk_packed_q(aq, asc, w)),
                          O.linear_q(aq_h, asc_h, W, s, K))
    C = dev(C0, cuda)
    ovb.linear_s8_nk_packed_q_add(aq, asc, w, C)
    check_close_and_exact(host(C), O.linear_q(aq_h, asc_h, W, s, K, C_in=C0))
    if M * N * ((K + 31) // 32) <= 4_000_000:
        assert np.array_equal(host(ovb.block_products(aq, w)), O.block_products(aq_h, W, K))
    assert ovb.device_status() == 0


@pytest.mark.parametrize("tile_n", [64, 32])
def test_narrow_tiles_sliced(cuda, golden, monkeypatch, tile_n):
    """Sliced output (qkv / gate|up) with narrow tiles: slices are multiples
    of 64 columns, so a warp's columns never straddle two slices."""
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    for i in range(3):
        Ns = [int(n) for n in golden[f"sliced{i}_Ns"]]
        parts = [ovb.Weight.from_nk(golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"])
                 for j in range(len(Ns))]
        wc = ovb.Weight.concat(parts)
        A = dev(golden[f"sliced{i}_A"], cuda)
        aq, asc = ovb.s8_nk_quantize(A)
        Cs = [torch.full((A.shape[0], n), float("nan"), device=cuda) for n in Ns]
        ovb.linear_s8_nk_packed_q_sliced(aq, asc, wc, Cs)
        for j, c in enumerate(Cs):
            check_close_and_exact(host(c), golden[f"sliced{i}_C{j}"])
