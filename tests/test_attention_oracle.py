"""The attention checker (oracle.attention) and the host-side argument
checks of ovb_attention, on the CPU.

oracle.attention runs the reference's own ov::attention_head_f32
(cpp/src/backend/cpu/ops_cpu.cpp:907-943, built into oracle/_ref) over the
segment/head loop of LM::run_layer (cpp/src/model/lm.cpp:256-274); its
float64 numpy restatement must agree with it, including the fully masked
rows (all scores below -1e29 -> zeros) that the reference's -1e30 padding
bias (lm.cpp:365, :431-434) produces."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import oracle as O

D = 128


def make_case(rng, seg_rows, n_heads, n_kv, masked_rows=(), pad_keys=0, scale_qk=1.0):
    T = sum(seg_rows)
    q = (rng.standard_normal((T, n_heads * D)) * scale_qk).astype(np.float32)
    k = (rng.standard_normal((T, n_kv * D)) * scale_qk).astype(np.float32)
    v = rng.standard_normal((T, n_kv * D)).astype(np.float32)
    segs, r0 = [], 0
    for rows in seg_rows:
        allow = np.ones((rows, rows), dtype=bool)
        allow[:, :min(pad_keys, rows - 1)] = False  # left padding: keys masked
        for r in masked_rows:
            if r < rows:
                allow[r, :] = False  # a padding row sees nothing
        bias = np.where(allow, 0.0, -1e30).astype(np.float32)
        segs.append((bias, rows, r0 * n_heads * D, r0 * n_kv * D))
        r0 += rows
    return q, k, v, segs


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("seg_rows,n_heads,n_kv", [((37,), 4, 2), ((130, 61), 4, 4), ((5, 9, 3), 2, 1)])
def test_reference_matches_restatement(seg_rows, n_heads, n_kv):
    rng = np.random.default_rng(11)
    q, k, v, segs = make_case(rng, seg_rows, n_heads, n_kv, masked_rows=(2,), pad_keys=3)
    scale = 1.0 / np.sqrt(D)
    a = O.attention(q, k, v, segs, n_heads, n_kv, D, scale, use_ref=True)
    b = O.attention(q, k, v, segs, n_heads, n_kv, D, scale, use_ref=False)
    np.testing.assert_allclose(a, b, rtol=2e-5, atol=2e-6)
    # the padding row of every segment is exactly zero on both sides
    r0 = 0
    for rows in seg_rows:
        assert not a[r0 + 2].any() and not b[r0 + 2].any()
        r0 += rows


def test_restatement_without_bias_is_softmax():
    rng = np.random.default_rng(5)
    q, k, v, _ = make_case(rng, (7,), 2, 1)
    out = O.attention(q, k, v, [(None, 7, 0, 0)], 2, 1, D, 0.1, use_ref=False)
    for h in range(2):
        Q, K, V = q[:, h * D:(h + 1) * D], k[:, :D], v[:, :D]
        s = (Q.astype(np.float64) @ K.T.astype(np.float64)) * 0.1
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        np.testing.assert_allclose(out[:, h * D:(h + 1) * D], p @ V, rtol=1e-5, atol=1e-6)


def _call(**kw):
    import ovnative_b200._lib as L
    a = dict(q=16, k=16, v=16, out=16, q_stride=256, kv_stride=128, n_heads=2, n_kv=1,
             head_dim=128, scale=1.0, segs=None, n_segs=1)
    a.update(kw)
    seg = (L.AttnSegment * 1)(L.AttnSegment(None, 4, 0, 0))
    segs = C.cast(seg, C.POINTER(L.AttnSegment)) if a["segs"] is None else a["segs"]
    return L.lib().ovb_attention(a["q"], a["k"], a["v"], a["out"], a["q_stride"],
                                 a["kv_stride"], a["n_heads"], a["n_kv"], a["head_dim"],
                                 a["scale"], segs, a["n_segs"], None)


@pytest.mark.parametrize("kw", [dict(head_dim=64), dict(n_heads=3, n_kv=2), dict(n_kv=0),
                                dict(q_stride=128), dict(kv_stride=130), dict(q=8),
                                dict(n_segs=65), dict(n_segs=-1), dict(v=0)])
def test_abi_rejects_bad_arguments(kw):
    import ovnative_b200._lib as L
    assert _call(**kw) == L.OVB_ERR_INVALID_ARG
    assert L.lib().ovb_last_error()


def test_abi_rejects_bad_segments():
    import ovnative_b200._lib as L
    for seg in (L.AttnSegment(None, -1, 0, 0), L.AttnSegment(None, 4, 2, 0),
                L.AttnSegment(None, 4, 0, -4),
                L.AttnSegment(None, 4, 4, 0),     # head 1 would wrap into the next row
                L.AttnSegment(None, 4, 0, 132)):
        arr = (L.AttnSegment * 1)(seg)
        assert _call(segs=C.cast(arr, C.POINTER(L.AttnSegment))) == L.OVB_ERR_INVALID_ARG


def test_abi_no_work_is_ok():
    import ovnative_b200._lib as L
    assert _call(n_segs=0, q=0) == L.OVB_OK
    arr = (L.AttnSegment * 2)(L.AttnSegment(None, 0, 0, 0), L.AttnSegment(None, 0, 256, 128))
    assert _call(segs=C.cast(arr, C.POINTER(L.AttnSegment)), n_segs=2) == L.OVB_OK


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")
def test_reference_layer_loop_equals_per_head_calls():
    """oracle.attention_layer (the OpenMP loop of LM::run_layer over the
    reference's attention_head_f32, the bench's CPU baseline) gives the same
    bytes as calling attention_head_f32 head by head."""
    rng = np.random.default_rng(9)
    q, k, v, segs = make_case(rng, (130, 61, 7), 8, 2, masked_rows=(2,), pad_keys=3)
    segs[1] = (None,) + segs[1][1:]
    a = O.attention(q, k, v, segs, 8, 2, D, 0.07, use_ref=True)
    b = O.attention_layer(q, k, v, segs, 8, 2, D, 0.07)
    assert a.tobytes() == b.tobytes()
