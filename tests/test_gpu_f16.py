"""GPU parity of the fp16 tensor-core mainloop (weights created with
OVB_WEIGHT_F16) against the reference's numerics.

The mainloop dequantises the reference's quantised activations to
fp16(q * asc) and accumulates in fp32, so it is held to the contract's
tolerance -- relative L2 <= 1e-3 and max |delta| <= 1e-2 * rms(reference) --
not to bit equality.  The expected error is ~3e-4 relative L2 (one fp16
rounding of each activation); the tests also assert a tighter 6e-4 so a
regression that still fits the contract (a lost scale correction, a wrong
fold) shows up.  Every tile width is forced once, with K tails (odd block
counts), ragged M/N, residual accumulation and sliced outputs.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3       # north-star tolerance on fp32 outputs
MAX_ABS_RMS = 1e-2  # max |delta| <= 1e-2 * rms(reference)
REL_L2_EXPECTED = 6e-4


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def check_tolerance(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    d = got - want
    rms = np.sqrt(np.mean(want ** 2)) + 1e-30
    rel = np.linalg.norm(d) / (np.linalg.norm(want) + 1e-30)
    assert rel <= REL_L2, f"rel-L2 {rel:.3e}"
    assert np.abs(d).max() <= MAX_ABS_RMS * rms, f"max-abs {np.abs(d).max():.3e} rms {rms:.3e}"
    assert rel <= REL_L2_EXPECTED, f"rel-L2 {rel:.3e} above the expected fp16 error"
    return rel


def case(rng, M, N, K, scale=3.0):
    A = (rng.standard_normal((M, K)) * scale).astype(np.float32)
    W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (np.abs(rng.standard_normal(N)) * 0.02 / 127 + 1e-6).astype(np.float32)
    return A, W, s


SHAPES = [(1, 8, 32), (127, 130, 96), (129, 257, 160), (300, 1000, 1056), (400, 1024, 2048),
          (400, 6144, 1024), (256, 3072, 1024), (1030, 4096, 1024)]


@pytest.mark.parametrize("tile_n", [256, 128, 64, 32])
@pytest.mark.parametrize("M,N,K", SHAPES[:5])
def test_f16_every_tile_width(cuda, monkeypatch, tile_n, M, N, K):
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    rng = np.random.default_rng(M * 13 + N + K)
    A, W, s = case(rng, M, N, K)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = ovb.Weight.from_nk(W, s, f16=True)
    aq, asc = ovb.s8_nk_quantize(dev(A, cuda))
    aq_h, asc_h = O.quantize(A)
    check_tolerance(host(ovb.linear_s8_nk_packed_q(aq, asc, w)), O.linear_q(aq_h, asc_h, W, s, K))
    C = dev(C0, cuda)
    ovb.linear_s8_nk_packed_q_add(aq, asc, w, C)
    check_tolerance(host(C), O.linear_q(aq_h, asc_h, W, s, K, C_in=C0))
    assert ovb.device_status() == 0
    w.close()


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_f16_default_tile_choice(cuda, M, N, K):
    rng = np.random.default_rng(M + 7 * N + K)
    A, W, s = case(rng, M, N, K, scale=1.0)
    w = ovb.Weight.from_nk(W, s, f16=True)
    got = host(ovb.linear_s8_nk_packed(dev(A, cuda), w))
    aq_h, asc_h = O.quantize(A)
    check_tolerance(got, O.linear_q(aq_h, asc_h, W, s, K))
    assert ovb.device_status() == 0
    w.close()


def test_f16_sliced_and_concat(cuda, golden):
    for i in range(3):
        Ns = [int(n) for n in golden[f"sliced{i}_Ns"]]
        parts = [ovb.Weight.from_nk(golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"], f16=True)
                 for j in range(len(Ns))]
        wc = ovb.Weight.concat(parts)
        assert wc.f16
        A = dev(golden[f"sliced{i}_A"], cuda)
        aq, asc = ovb.s8_nk_quantize(A)
        Cs = [torch.full((A.shape[0], n), float("nan"), device=cuda) for n in Ns]
        ovb.linear_s8_nk_packed_q_sliced(aq, asc, wc, Cs)
        for j, c in enumerate(Cs):
            check_tolerance(host(c), golden[f"sliced{i}_C{j}"])


def test_f16_and_exact_paths_on_one_layer(cuda):
    """The same weights through both mainloops: the exact one is bit-identical
    to the port, the fp16 one within tolerance of it."""
    rng = np.random.default_rng(5)
    M, N, K = 400, 3072, 1024
    A, W, s = case(rng, M, N, K, scale=1.0)
    we = ovb.Weight.from_nk(W, s)
    wf = ovb.Weight.from_nk(W, s, f16=True)
    aq, asc = ovb.s8_nk_quantize(dev(A, cuda))
    exact = host(ovb.linear_s8_nk_packed_q(aq, asc, we))
    fast = host(ovb.linear_s8_nk_packed_q(aq, asc, wf))
    aq_h, asc_h = O.quantize(A)
    ref = O.linear_q(aq_h, asc_h, W, s, K)
    assert exact.tobytes() == ref.tobytes()
    rel = check_tolerance(fast, ref)
    assert rel > 0  # the fp16 path is genuinely a different computation
    # block products stay on the int8 path for an f16 handle, bit-exact
    P = host(ovb.block_products(aq[:64], wf))
    assert np.array_equal(P, O.block_products(aq_h[:64], W, K))


def test_f16_range_flag(cuda):
    """Activations beyond fp16's range set status bit 16 instead of passing
    silently (the exact path has no such limit)."""
    rng = np.random.default_rng(11)
    M, N, K = 64, 128, 64
    A, W, s = case(rng, M, N, K, scale=1.0)
    A[3, 5] = 1.0e5
    w = ovb.Weight.from_nk(W, s, f16=True)
    aq, asc = ovb.s8_nk_quantize(dev(A, cuda))
    ovb.linear_s8_nk_packed_q(aq, asc, w)
    assert ovb.device_status() == 16
    assert ovb.device_status() == 0  # reading clears it


# ------------------------------------------------- OVB_AQ_F16 + ovb_linear_h
def test_quantisers_f16_form_is_dequantised_q(cuda):
    """The fp16 output form of each quantiser is fp16(q * asc) of the same q
    and asc the int8 form gives (which match the reference byte for byte)."""
    rng = np.random.default_rng(21)
    M, K = 67, 1000
    A = dev((rng.standard_normal((M, K)) * 2).astype(np.float32), cuda)
    G = dev(rng.standard_normal((M, K)).astype(np.float32), cuda)
    U = dev(rng.standard_normal((M, K)).astype(np.float32), cuda)
    gain = dev((1 + 0.1 * rng.standard_normal(K)).astype(np.float32), cuda)
    pairs = [
        (ovb.s8_nk_quantize(A), ovb.s8_nk_quantize(A, f16=True)),
        (ovb.rmsnorm_quantize_f32(A, gain, 1e-6), ovb.rmsnorm_quantize_f32(A, gain, 1e-6, f16=True)),
        (ovb.silu_mul_quantize_f32(G, U), ovb.silu_mul_quantize_f32(G, U, f16=True)),
    ]
    for (aq, asc), (a16, asc16) in pairs:
        assert torch.equal(asc, asc16)
        q = host(aq).astype(np.float32)
        s = np.repeat(host(asc), 32, axis=1)
        want = (q * s).astype(np.float16)
        assert a16.dtype == torch.float16
        assert np.array_equal(host(a16).view(np.uint16), want.view(np.uint16))
    assert ovb.device_status() == 0


@pytest.mark.parametrize("tile_n", [256, 128, 64, 32])
@pytest.mark.parametrize("M,N,K", SHAPES[:5])
def test_linear_h_every_tile_width(cuda, monkeypatch, tile_n, M, N, K):
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    rng = np.random.default_rng(M * 17 + N + K)
    A, W, s = case(rng, M, N, K)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = ovb.Weight.from_nk(W, s, f16=True)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    aq_h, asc_h = O.quantize(A)
    check_tolerance(host(ovb.linear_h(a16, w)), O.linear_q(aq_h, asc_h, W, s, K))
    C = dev(C0, cuda)
    ovb.linear_h(a16, w, C, accumulate=True)
    check_tolerance(host(C), O.linear_q(aq_h, asc_h, W, s, K, C_in=C0))
    assert ovb.device_status() == 0
    w.close()


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_h_default_tile_choice(cuda, M, N, K):
    rng = np.random.default_rng(3 * M + N + K)
    A, W, s = case(rng, M, N, K, scale=1.0)
    w = ovb.Weight.from_nk(W, s, f16=True)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    aq_h, asc_h = O.quantize(A)
    check_tolerance(host(ovb.linear_h(a16, w)), O.linear_q(aq_h, asc_h, W, s, K))
    assert ovb.device_status() == 0
    w.close()


def test_linear_h_sliced(cuda, golden):
    for i in range(3):
        Ns = [int(n) for n in golden[f"sliced{i}_Ns"]]
        parts = [ovb.Weight.from_nk(golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"], f16=True)
                 for j in range(len(Ns))]
        wc = ovb.Weight.concat(parts)
        a16, _ = ovb.s8_nk_quantize(dev(golden[f"sliced{i}_A"], cuda), f16=True)
        Cs = [torch.full((a16.shape[0], n), float("nan"), device=cuda) for n in Ns]
        ovb.linear_h_sliced(a16, wc, Cs)
        for j, c in enumerate(Cs):
            check_tolerance(host(c), golden[f"sliced{i}_C{j}"])


def test_linear_h_argument_errors(cuda):
    w8 = ovb.Weight.from_nk(np.ones((64, 64), np.int8), np.ones(64, np.float32))
    a16 = torch.zeros((4, 64), dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError, match="OVB_WEIGHT_F16"):
        ovb.linear_h(a16, w8)
    w16 = ovb.Weight.from_nk(np.ones((64, 64), np.int8), np.ones(64, np.float32), f16=True)
    with pytest.raises(ValueError, match="16-byte aligned"):
        ovb.linear_h(a16.view(-1)[1:129].view(2, 64), w16)
    with pytest.raises(ValueError, match="exclusive"):
        ovb.s8_nk_quantize(torch.zeros((4, 64), device=cuda), u8=True, f16=True)


def test_quantiser_f16_range_flag(cuda):
    A = torch.zeros((4, 64), device=cuda)
    A[1, 3] = 1.0e5
    ovb.s8_nk_quantize(A, f16=True)
    assert ovb.device_status() == 16
    assert ovb.device_status() == 0


# ------------------------------------------- split-K clusters (fp16 mainloop)
SPLIT_SHAPES = [(400, 1024, 3072), (129, 320, 1056), (300, 1000, 256), (1, 128, 512),
                (400, 1024, 2048)]


@pytest.mark.parametrize("tile_n,split", [(64, 2), (128, 2), (128, 4)])
@pytest.mark.parametrize("M,N,K", SPLIT_SHAPES)
def test_linear_h_split_k(cuda, monkeypatch, tile_n, split, M, N, K):
    """K split over a cluster of `split` CTAs per output tile; each rank sums
    its partners' partials in rank order.  1056 gives 17 k-stages (uneven
    per rank), 256 gives 4 (one per rank at split 4)."""
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    monkeypatch.setenv("OVB_GEMM_SPLIT_K", str(split))
    rng = np.random.default_rng(M * 5 + N + K + split)
    A, W, s = case(rng, M, N, K)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = ovb.Weight.from_nk(W, s, f16=True)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    aq_h, asc_h = O.quantize(A)
    got = host(ovb.linear_h(a16, w))
    check_tolerance(got, O.linear_q(aq_h, asc_h, W, s, K))
    # deterministic: the partial sums are added in a fixed order
    assert host(ovb.linear_h(a16, w)).tobytes() == got.tobytes()
    C = dev(C0, cuda)
    ovb.linear_h(a16, w, C, accumulate=True)
    check_tolerance(host(C), O.linear_q(aq_h, asc_h, W, s, K, C_in=C0))
    assert ovb.device_status() == 0
    w.close()


@pytest.mark.parametrize("split", [2, 4])
def test_linear_h_split_k_sliced(cuda, golden, monkeypatch, split):
    monkeypatch.setenv("OVB_GEMM_TILE_N", "128")
    monkeypatch.setenv("OVB_GEMM_SPLIT_K", str(split))
    for i in range(3):
        Ns = [int(n) for n in golden[f"sliced{i}_Ns"]]
        parts = [ovb.Weight.from_nk(golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"], f16=True)
                 for j in range(len(Ns))]
        wc = ovb.Weight.concat(parts)
        a16, _ = ovb.s8_nk_quantize(dev(golden[f"sliced{i}_A"], cuda), f16=True)
        Cs = [torch.full((a16.shape[0], n), float("nan"), device=cuda) for n in Ns]
        ovb.linear_h_sliced(a16, wc, Cs)
        for j, c in enumerate(Cs):
            check_tolerance(host(c), golden[f"sliced{i}_C{j}"])
    assert ovb.device_status() == 0


# C rows that are not 16-byte aligned take the epilogue's scalar store path
# (the float4 path needs C and ldc multiples of 4 floats).
@pytest.mark.parametrize("offset,pad", [(1, 0), (0, 3), (2, 5)])
@pytest.mark.parametrize("tile_n,split", [(128, 1), (32, 1), (64, 2), (128, 4)])
def test_linear_h_unaligned_c(cuda, monkeypatch, offset, pad, tile_n, split):
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    monkeypatch.setenv("OVB_GEMM_SPLIT_K", str(split))
    M, N, K = 150, 256, 1024
    rng = np.random.default_rng(offset * 7 + pad + tile_n + split)
    A, W, s = case(rng, M, N, K)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = ovb.Weight.from_nk(W, s, f16=True)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    aq_h, asc_h = O.quantize(A)
    buf = torch.full((M, N + offset + pad), float("nan"), device=cuda)
    C = buf[:, offset:offset + N]
    ovb.linear_h(a16, w, C)
    check_tolerance(host(C), O.linear_q(aq_h, asc_h, W, s, K))
    # the columns around the view are untouched
    assert torch.isnan(buf[:, :offset]).all() and torch.isnan(buf[:, offset + N:]).all()
    C.copy_(dev(C0, cuda))
    ovb.linear_h(a16, w, C, accumulate=True)
    check_tolerance(host(C), O.linear_q(aq_h, asc_h, W, s, K, C_in=C0))
    assert ovb.device_status() == 0
    w.close()


# ------------------------------------ CTA pairs (tcgen05 cta_group::2, M = 256)
PAIR_SHAPES = [(400, 1024, 1024), (129, 320, 1056), (300, 4096, 1024), (1, 256, 64),
               (1400, 6144, 1024), (600, 1000, 256), (3000, 4096, 1024), (2600, 1000, 512)]


@pytest.mark.parametrize("tile_n", [256, 128])
@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
def test_linear_h_pair(cuda, monkeypatch, tile_n, M, N, K):
    """A 2-CTA cluster computes 256-row tiles with cta_group::2 MMAs, each
    CTA loading half of the W tile.  300 rows leave the second pair's peer
    CTA without rows; 1400 x 6144 and the two larger shapes give each
    cluster of the persistent grid several tiles (both accumulators and
    the peer's release of them in use)."""
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    monkeypatch.setenv("OVB_GEMM_PAIR", "1")
    rng = np.random.default_rng(M * 3 + N + K + tile_n)
    A, W, s = case(rng, M, N, K)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    w = ovb.Weight.from_nk(W, s, f16=True)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    aq_h, asc_h = O.quantize(A)
    got = host(ovb.linear_h(a16, w))
    check_tolerance(got, O.linear_q(aq_h, asc_h, W, s, K))
    assert host(ovb.linear_h(a16, w)).tobytes() == got.tobytes()  # deterministic
    C = dev(C0, cuda)
    ovb.linear_h(a16, w, C, accumulate=True)
    check_tolerance(host(C), O.linear_q(aq_h, asc_h, W, s, K, C_in=C0))
    # unaligned C rows take the epilogue's scalar path
    buf = torch.full((M, N + 3), float("nan"), device=cuda)
    ovb.linear_h(a16, w, buf[:, 1:N + 1])
    check_tolerance(host(buf[:, 1:N + 1]), O.linear_q(aq_h, asc_h, W, s, K))
    assert torch.isnan(buf[:, 0]).all() and torch.isnan(buf[:, N + 1:]).all()
    assert ovb.device_status() == 0
    w.close()


# The plain epilogue writes C through TMA boxes (stores; element-wise adds
# at L2 when accumulating) whenever every output slice's rows are 16-byte
# aligned; OVB_GEMM_TMA_OUT=0 keeps the register stores and residual loads.
# Both forms compute fl(fl(acc * wscale) + C) and must agree bit for bit.
@pytest.mark.parametrize("tile_n,pair", [(256, 0), (128, 0), (64, 0), (32, 0), (256, 1),
                                         (128, 1)])
@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (300, 1000, 256), (2600, 1024, 1024),
                                   (777, 4096, 512)])
def test_tma_output_equals_register_stores(cuda, monkeypatch, tile_n, pair, M, N, K):
    monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
    monkeypatch.setenv("OVB_GEMM_PAIR", str(pair))
    rng = np.random.default_rng(M + N + K + tile_n + pair)
    A, W, s = case(rng, M, N, K)
    w = ovb.Weight.from_nk(W, s, f16=True)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    C0 = dev(rng.standard_normal((M, N)).astype(np.float32), cuda)
    outs = {}
    for tma in ("1", "0"):
        monkeypatch.setenv("OVB_GEMM_TMA_OUT", tma)
        plain = torch.full((M, N), float("nan"), device=cuda)
        ovb.linear_h(a16, w, plain)
        acc = C0.clone()
        ovb.linear_h(a16, w, acc, accumulate=True)
        # a row stride with padding (ldc = N + 4 keeps 16-byte rows)
        wide = torch.full((M, N + 4), float("nan"), device=cuda)
        ovb.linear_h(a16, w, wide[:, :N])
        outs[tma] = (host(plain), host(acc), host(wide))
    for a, b in zip(outs["1"], outs["0"]):
        assert a.tobytes() == b.tobytes()
    assert np.isnan(outs["1"][2][:, N:]).all()  # the padding is untouched
    assert ovb.device_status() == 0
    w.close()


def test_tma_output_sliced(cuda, golden, monkeypatch):
    """Three output slices (q|k|v-like): one TMA map per slice."""
    monkeypatch.setenv("OVB_GEMM_TILE_N", "256")
    for pair in ("0", "1"):
        monkeypatch.setenv("OVB_GEMM_PAIR", pair)
        for i in range(3):
            Ns = [int(n) for n in golden[f"sliced{i}_Ns"]]
            parts = [ovb.Weight.from_nk(golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"],
                                        f16=True) for j in range(len(Ns))]
            wc = ovb.Weight.concat(parts)
            a16, _ = ovb.s8_nk_quantize(dev(golden[f"sliced{i}_A"], cuda), f16=True)
            got = {}
            for tma in ("1", "0"):
                monkeypatch.setenv("OVB_GEMM_TMA_OUT", tma)
                Cs = [torch.ones((a16.shape[0], n), device=cuda) for n in Ns]
                ovb.linear_h_sliced(a16, wc, Cs)
                got[tma] = [host(c) for c in Cs]
            for a, b in zip(got["1"], got["0"]):
                assert a.tobytes() == b.tobytes()
    assert ovb.device_status() == 0


def test_linear_h_pair_sliced(cuda, golden, monkeypatch):
    monkeypatch.setenv("OVB_GEMM_TILE_N", "128")
    monkeypatch.setenv("OVB_GEMM_PAIR", "1")
    for i in range(3):
        Ns = [int(n) for n in golden[f"sliced{i}_Ns"]]
        parts = [ovb.Weight.from_nk(golden[f"sliced{i}_W{j}"], golden[f"sliced{i}_s{j}"], f16=True)
                 for j in range(len(Ns))]
        wc = ovb.Weight.concat(parts)
        a16, _ = ovb.s8_nk_quantize(dev(golden[f"sliced{i}_A"], cuda), f16=True)
        Cs = [torch.full((a16.shape[0], n), float("nan"), device=cuda) for n in Ns]
        ovb.linear_h_sliced(a16, wc, Cs)
        for j, c in enumerate(Cs):
            check_tolerance(host(c), golden[f"sliced{i}_C{j}"])
    assert ovb.device_status() == 0


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("M,N,K", [(1, 64, 32), (77, 8200, 1024), (300, 1024, 1000)])
def test_fp32_weight_linear_matches_fp64(cuda, layout, M, N, K):
    """ovb_weight_create_f32 + OVB_AQ_F16_RAW + ovb_linear_h against the
    reference's fp32 linear_f32 (C = A W, mat.cpp:11-13), computed here in
    float64: fp16 operands and fp32 accumulation hold rel-L2 <= 1e-3 and
    max-abs <= 1e-2 * rms (the path's tolerance)."""
    rng = np.random.default_rng(M + N + K + layout)
    Wnk = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    Wnk[N // 3] *= 1e-3  # a quiet channel keeps its precision (own scale)
    A = rng.standard_normal((M, K)).astype(np.float32)
    w = ovb.Weight.from_f32(Wnk if layout == 0 else np.ascontiguousarray(Wnk.T), layout=layout)
    assert (w.N, w.K) == (N, K)
    got = ovb.linear_f32(torch.from_numpy(A).to(cuda), w).cpu().numpy()
    want = A.astype(np.float64) @ Wnk.astype(np.float64).T
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    rms = np.sqrt((want ** 2).mean())
    assert err <= 1e-3, err
    assert np.abs(got - want).max() <= 1e-2 * rms
    q = want[:, N // 3]
    assert np.linalg.norm(got[:, N // 3] - q) <= 1e-3 * np.linalg.norm(q)
    # accumulate (linear_f32_ld with accumulate, Mat::mul_add, mat.cpp:39-43)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    Ct = torch.from_numpy(C0).to(cuda)
    ovb.linear_f32(torch.from_numpy(A).to(cuda), w, Ct, accumulate=True)
    got2 = Ct.cpu().numpy()
    assert np.linalg.norm(got2 - (C0 + want)) <= 1e-3 * np.linalg.norm(C0 + want)
    assert ovb.device_status() == 0
    w.close()


def test_raw_f16_forms(cuda):
    """OVB_AQ_F16_RAW writes fp16 of the values themselves (zero K tail) from
    ovb_quantize and of rmsnorm_into_f32's values from ovb_rmsnorm_quantize,
    and the int8 entry points refuse an fp32-created weight."""
    rng = np.random.default_rng(3)
    A = (rng.standard_normal((37, 70)) * 3).astype(np.float32)
    a16 = ovb.to_f16(torch.from_numpy(A).to(cuda)).cpu().numpy()
    assert a16.shape == (37, 96)
    np.testing.assert_array_equal(a16[:, :70], A.astype(np.float16))
    assert not a16[:, 70:].any()
    x = rng.standard_normal((20, 1024)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    h = ovb.rmsnorm_f16(torch.from_numpy(x).to(cuda), torch.from_numpy(g).to(cuda), 1e-6)
    want = O.rmsnorm_into(x, g, 1e-6).astype(np.float16)
    np.testing.assert_array_equal(h.cpu().numpy(), want)
    w = ovb.Weight.from_f32(np.ones((64, 32), np.float32), layout=0)
    aq, asc = ovb.s8_nk_quantize(torch.from_numpy(A[:, :32].copy()).to(cuda))
    with pytest.raises(ValueError, match="no int8 image"):
        ovb.linear_s8_nk_packed_q(aq, asc, w)
    w.close()
