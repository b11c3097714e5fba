"""GPU parity of the gate|up GEMM fused with SiLU*up + quantise
(ovb_linear_q_silu / ovb_linear_h_silu on an ovb_weight_gate_up handle).

* int8 mainloop: the quantised output and its scales are byte-identical to
  the reference's two calls -- linear_s8_nk_packed_q_sliced on gate|up, then
  silu_mul_quantize_f32 (lm.cpp:295-311) -- restated by the oracle;
* fp16 mainloop: agrees with the unfused fp16 sequence (linear_h_sliced then
  the fp16-form silu_mul_quantize) -- the same accumulators and scales, silu
  with the hardware's fast exp/division instead of the reference polynomial,
  so an int8 step differs only where a value sits on a rounding boundary --
  and is within the contract's tolerance of the reference;
* every output form (int8, u8, fp16), ragged M, forced tile widths, errors.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from ovnative_b200 import layer as LY

pytestmark = pytest.mark.gpu


def dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def weights(rng, inter, K, f16):
    Wg = rng.integers(-127, 128, size=(inter, K), dtype=np.int8)
    Wu = rng.integers(-127, 128, size=(inter, K), dtype=np.int8)
    sg = (np.abs(rng.standard_normal(inter)) * 0.02 / 127 + 1e-6).astype(np.float32)
    su = (np.abs(rng.standard_normal(inter)) * 0.02 / 127 + 1e-6).astype(np.float32)
    g = ovb.Weight.from_nk(Wg, sg, f16=f16)
    u = ovb.Weight.from_nk(Wu, su, f16=f16)
    return (Wg, sg, Wu, su), g, u


@pytest.mark.parametrize("M,inter,K", [(1, 64, 64), (129, 256, 96), (400, 3072, 1024), (257, 640, 160)])
def test_q_silu_bit_exact_vs_reference(cuda, M, inter, K):
    rng = np.random.default_rng(M + inter + K)
    (Wg, sg, Wu, su), g, u = weights(rng, inter, K, False)
    gu = ovb.Weight.gate_up(g, u)
    A = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    aq, asc = ovb.s8_nk_quantize(dev(A, cuda))
    q, sc = ovb.linear_q_silu(aq, asc, gu, u8=True)
    aq_h, asc_h = O.quantize(A)
    gate = O.linear_q(aq_h, asc_h, Wg, sg, K)
    up = O.linear_q(aq_h, asc_h, Wu, su, K)
    want_q, want_s = O.silu_mul_quantize(gate, up)
    assert host(q).tobytes() == want_q.tobytes()
    assert host(sc).tobytes() == want_s.tobytes()
    # int8 form: the same q, signed
    q8, sc8 = ovb.linear_q_silu(aq, asc, gu)
    assert np.array_equal(host(q8).astype(np.int16), want_q.astype(np.int16) - 128)
    assert ovb.device_status() == 0


# (tile width, CTA pair): the single-CTA widths and the cta_group::2 pairs.
@pytest.mark.parametrize("tile_n,pair", [(256, 0), (128, 0), (64, 0), (256, 1), (128, 1)])
@pytest.mark.parametrize("M,inter,K", [(1, 64, 64), (129, 256, 96), (400, 3072, 1024),
                                       (300, 640, 1056), (2000, 3072, 1024)])
def test_h_silu_agrees_with_unfused_fp16_sequence(cuda, monkeypatch, tile_n, pair, M, inter, K):
    rng = np.random.default_rng(3 * M + inter + K)
    (Wg, sg, Wu, su), g, u = weights(rng, inter, K, True)
    gu = ovb.Weight.gate_up(g, u)
    cat = ovb.Weight.concat([g, u])
    A = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    gate = torch.empty((M, inter), device=cuda)
    up = torch.empty((M, inter), device=cuda)
    ovb.linear_h_sliced(a16, cat, [gate, up])
    for f16_out in (True, False):
        want_q, want_s = ovb.silu_mul_quantize_f32(gate, up, f16=f16_out)
        monkeypatch.setenv("OVB_GEMM_TILE_N", str(tile_n))
        monkeypatch.setenv("OVB_GEMM_PAIR", str(pair))
        q, sc = ovb.linear_h_silu(a16, gu, f16=f16_out)
        monkeypatch.delenv("OVB_GEMM_TILE_N")
        monkeypatch.delenv("OVB_GEMM_PAIR")
        got_s, ref_s = host(sc).astype(np.float64), host(want_s).astype(np.float64)
        assert np.all(np.abs(got_s - ref_s) <= 1e-5 * np.abs(ref_s) + 1e-30)
        if f16_out:
            a, b = host(q).astype(np.float64), host(want_q).astype(np.float64)
            assert np.linalg.norm(a - b) <= 1e-3 * np.linalg.norm(b)
        else:
            dq = np.abs(host(q).astype(np.int16) - host(want_q).astype(np.int16))
            assert dq.max() <= 1 and (dq != 0).mean() <= 1e-3
    assert ovb.device_status() == 0


def test_h_silu_within_tolerance_of_reference(cuda):
    rng = np.random.default_rng(99)
    M, inter, K = 400, 3072, 1024
    (Wg, sg, Wu, su), g, u = weights(rng, inter, K, True)
    gu = ovb.Weight.gate_up(g, u)
    A = rng.standard_normal((M, K)).astype(np.float32)
    a16, _ = ovb.s8_nk_quantize(dev(A, cuda), f16=True)
    q16, _ = ovb.linear_h_silu(a16, gu, f16=True)
    aq_h, asc_h = O.quantize(A)
    want_q, want_s = O.silu_mul_quantize(O.linear_q(aq_h, asc_h, Wg, sg, K),
                                         O.linear_q(aq_h, asc_h, Wu, su, K))
    want = (want_q.astype(np.float64) - 128) * np.repeat(want_s, 32, axis=1)
    got = host(q16).astype(np.float64)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    # requantisation of slightly different inputs flips a few int8 steps:
    # bounded by the step size, well inside 1e-2 relative
    assert rel <= 1e-2, rel


def test_silu_argument_errors(cuda):
    w = ovb.Weight.from_nk(np.ones((64, 64), np.int8), np.ones(64, np.float32))
    aq, asc = ovb.s8_nk_quantize(torch.zeros((4, 64), device=cuda))
    with pytest.raises(ValueError, match="gate\\|up weight"):
        ovb.linear_q_silu(aq, asc, w, out=(torch.empty((4, 32), dtype=torch.int8, device=cuda),
                                            torch.empty((4, 1), device=cuda)))
    g = ovb.Weight.from_nk(np.ones((64, 64), np.int8), np.ones(64, np.float32))
    u = ovb.Weight.from_nk(np.ones((32, 64), np.int8), np.ones(32, np.float32))
    with pytest.raises(ValueError, match="differ in shape"):
        ovb.Weight.gate_up(g, u)


@pytest.mark.parametrize("f16", [False, True])
def test_fused_layer_matches_unfused_layer(cuda, f16):
    """The layer with the fused gate|up+SiLU*up GEMM gives the same bytes as
    the reference's unfused sequence on the int8 mainloop, and agrees within
    1e-4 relative on the fp16 mainloop (fast silu in the fused epilogue)."""
    rng = np.random.default_rng(31)
    M = 400
    w = LY.random_layer_host(rng)
    x0 = torch.from_numpy(rng.standard_normal((M, LY.HIDDEN)).astype(np.float32)).to(cuda)
    lw_f = LY.LayerWeights.from_host(w, cuda, f16=f16)
    lw_u = LY.LayerWeights.from_host(w, cuda, f16=f16, fused=False)
    xa, xb = x0.clone(), x0.clone()
    LY.run(xa, lw_f, LY.LayerBuffers(M, cuda, f16=f16))
    LY.run_unfused(xb, lw_u, LY.LayerBuffers(M, cuda, f16=f16))
    a, b = host(xa), host(xb)
    if f16:
        d = (a - x0.cpu().numpy()).astype(np.float64)
        e = (b - x0.cpu().numpy()).astype(np.float64)
        assert np.linalg.norm(d - e) <= 1e-3 * np.linalg.norm(e)
    else:
        assert a.tobytes() == b.tobytes()
