"""Device weights straight from an OVW1 file (ovb_ovw1_weight): both stored
orientations ([N, K] layout 0, [K, N] layout 1) give the same device image
as ovb_weight_create on the arrays, and GEMMs with them are bit-identical to
the reference's arithmetic (oracle port of linear_s8_nk_packed_q)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from ovnative_b200 import ovw1

pytestmark = pytest.mark.gpu


def make_file(path, rng, shapes):
    ts, want = [], {}
    for name, (N, K, layout) in shapes.items():
        W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        s = (np.abs(rng.standard_normal(N)) * 0.02 / 127).astype(np.float32)
        ts.append((name, W if layout == 0 else np.ascontiguousarray(W.T), layout, s))
        want[name] = (W, s)
    ovw1.write(str(path), ts)
    return want


SHAPES = {"q_nk": (192, 1024, 0), "o_kn": (256, 2048, 1), "odd_nk": (100, 70, 0),
          "odd_kn": (72, 33, 1)}


@pytest.mark.parametrize("f16", [False, True])
def test_weights_match_arrays(cuda, repo_tmp, f16):
    rng = np.random.default_rng(3)
    want = make_file(repo_tmp / "w.ovw", rng, SHAPES)
    with ovw1.OVW1File(str(repo_tmp / "w.ovw")) as f:
        for name, (W, s) in want.items():
            w = f.weight(name, f16=f16)
            assert (w.N, w.K) == W.shape
            gW, gs = w.export()
            np.testing.assert_array_equal(gW, W)
            np.testing.assert_array_equal(gs, s)
            w.close()
    assert ovb.device_status() == 0


def test_gemm_bit_exact_from_file(cuda, repo_tmp):
    rng = np.random.default_rng(4)
    want = make_file(repo_tmp / "w.ovw", rng, SHAPES)
    with ovw1.OVW1File(str(repo_tmp / "w.ovw")) as f:
        for name, (W, s) in want.items():
            N, K = W.shape
            A = rng.standard_normal((37, K)).astype(np.float32)
            w = f.weight(name)
            aq, asc = ovb.s8_nk_quantize(torch.from_numpy(A).to(cuda))
            C = ovb.linear_s8_nk_packed_q(aq, asc, w).cpu().numpy()
            qa, qs = O.quantize(A)
            np.testing.assert_array_equal(C, O.linear_q(qa, qs, W, s, K))
            w.close()
    assert ovb.device_status() == 0


def test_concat_from_file(cuda, repo_tmp):
    """q | k | v loaded from the file and concatenated (combine_packed)."""
    rng = np.random.default_rng(5)
    shapes = {"q": (256, 128, 0), "k": (128, 128, 1), "v": (128, 128, 0)}
    want = make_file(repo_tmp / "qkv.ovw", rng, shapes)
    with ovw1.OVW1File(str(repo_tmp / "qkv.ovw")) as f:
        parts = [f.weight(n) for n in shapes]
        qkv = ovb.Weight.concat(parts)
        gW, gs = qkv.export()
        np.testing.assert_array_equal(gW, np.concatenate([want[n][0] for n in shapes]))
        np.testing.assert_array_equal(gs, np.concatenate([want[n][1] for n in shapes]))
        for p in parts + [qkv]:
            p.close()


@pytest.mark.parametrize("f16", [False, True])
def test_batch_load_matches_arrays(cuda, repo_tmp, f16):
    """ovb_ovw1_weights (one device allocation): the same device
    images as one-by-one creation, and the handles free independently."""
    rng = np.random.default_rng(6)
    want = make_file(repo_tmp / "w.ovw", rng, SHAPES)
    names = list(want)
    with ovw1.OVW1File(str(repo_tmp / "w.ovw")) as f:
        ws = f.weights(names, f16=f16)
    for name, w in zip(names, ws):
        W, s = want[name]
        assert (w.N, w.K) == W.shape
        gW, gs = w.export()
        np.testing.assert_array_equal(gW, W)
        np.testing.assert_array_equal(gs, s)
    # free out of order; the survivors stay usable (the arena lives on)
    ws[0].close()
    ws[2].close()
    W, s = want[names[1]]
    A = rng.standard_normal((5, W.shape[1])).astype(np.float32)
    aq, asc = ovb.s8_nk_quantize(torch.from_numpy(A).to(cuda))
    C = ovb.linear_s8_nk_packed_q(aq, asc, ws[1]).cpu().numpy()
    qa, qs = O.quantize(A)
    want_C = O.linear_q(qa, qs, W, s, W.shape[1])
    if f16:  # an OVB_WEIGHT_F16 handle runs the fp16 mainloop: the tolerance contract
        d = C.astype(np.float64) - want_C
        rms = np.sqrt(np.mean(want_C.astype(np.float64) ** 2))
        assert np.linalg.norm(d) / np.linalg.norm(want_C) <= 1e-3
        assert np.abs(d).max() <= 1e-2 * rms
    else:
        np.testing.assert_array_equal(C, want_C)
    ws[1].close()
    ws[3].close()
    assert ovb.device_status() == 0


def test_batch_from_device_sources(cuda):
    """ovb_weight_create_batch with OVB_SRC_DEVICE sources of both layouts."""
    import ctypes as C

    from ovnative_b200 import _lib as L
    rng = np.random.default_rng(7)
    shapes = [(64, 96, 0), (40, 33, 1), (128, 1024, 1)]
    keep, srcs, want = [], (L.WeightSrc * len(shapes))(), []
    for i, (N, K, layout) in enumerate(shapes):
        W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        s = rng.random(N).astype(np.float32)
        dW = torch.from_numpy(W if layout == 0 else np.ascontiguousarray(W.T)).to(cuda)
        ds = torch.from_numpy(s).to(cuda)
        keep += [dW, ds]
        srcs[i] = L.WeightSrc(dW.data_ptr(), layout, N, K, ds.data_ptr())
        want.append((W, s))
    out = (C.c_void_p * len(shapes))()
    L.check(L.lib().ovb_weight_create_batch(srcs, len(shapes), L.OVB_SRC_DEVICE, None, out))
    for i, (W, s) in enumerate(want):
        w = ovb.Weight(out[i], W.shape[0], W.shape[1], False)
        gW, gs = w.export()
        np.testing.assert_array_equal(gW, W)
        np.testing.assert_array_equal(gs, s)
        w.close()
