"""The tensor-core attention (ovb_attention) against the reference's own
ov::attention_head_f32 (oracle.attention; cpp/src/backend/cpu/ops_cpu.cpp:
907-943 over the loop of LM::run_layer, cpp/src/model/lm.cpp:256-274).

Contract (fp16 operands, fp32 accumulation and softmax): per case
rel-L2 <= 2e-3 and max-abs <= 2e-2 * rms(reference); fully masked rows
(every score below -1e29) exactly zero; rows outside every segment
untouched; device status 0."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from tests.test_attention_oracle import D, make_case

pytestmark = pytest.mark.gpu

REL_L2 = 2e-3
MAX_ABS = 2e-2


def run(q, k, v, segs, n_heads, n_kv, scale, cuda, out=None):
    tq, tk, tv = (torch.from_numpy(x).to(cuda) for x in (q, k, v))
    tsegs = [(None if b is None else torch.from_numpy(b).to(cuda), r, qo, ko)
             for b, r, qo, ko in segs]
    o = None if out is None else torch.from_numpy(out).to(cuda)
    got = ovb.attention(tq, tk, tv, tsegs, n_heads, n_kv, scale, out=o)
    torch.cuda.synchronize()
    assert ovb.device_status() == 0
    return got.cpu().numpy()


def compare(got, want):
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2))) or 1.0
    err = got.astype(np.float64) - want
    rel = float(np.linalg.norm(err) / (np.linalg.norm(want) or 1.0))
    mx = float(np.abs(err).max())
    assert rel <= REL_L2, rel
    assert mx <= MAX_ABS * rms, (mx, rms)
    return rel, mx


@pytest.mark.parametrize("rows", [1, 2, 31, 128, 129, 200, 256, 385])
def test_single_segment(rows, cuda):
    rng = np.random.default_rng(rows)
    q, k, v, segs = make_case(rng, (rows,), 16, 8, masked_rows=(1,), pad_keys=2)
    scale = 1.0 / np.sqrt(D)
    got = run(q, k, v, segs, 16, 8, scale, cuda)
    want = O.attention(q, k, v, segs, 16, 8, D, scale)
    compare(got, want)
    if rows > 1:
        assert not got[1].any()


@pytest.mark.parametrize("n_heads,n_kv", [(16, 16), (16, 4), (8, 1)])
def test_gqa_groups(n_heads, n_kv, cuda):
    rng = np.random.default_rng(n_heads * 10 + n_kv)
    q, k, v, segs = make_case(rng, (150,), n_heads, n_kv)
    scale = 1.0 / np.sqrt(D)
    compare(run(q, k, v, segs, n_heads, n_kv, scale, cuda),
            O.attention(q, k, v, segs, n_heads, n_kv, D, scale))


def test_cfg_pair_segments(cuda):
    """The CFG layout of LM::forward_cfg (lm.cpp:441-443): cond rows then
    uncond rows packed back-to-back, each with its own padding bias."""
    rng = np.random.default_rng(7)
    q, k, v, segs = make_case(rng, (300, 97), 16, 8, masked_rows=(0, 3), pad_keys=5)
    scale = 1.0 / np.sqrt(D)
    got = run(q, k, v, segs, 16, 8, scale, cuda)
    compare(got, O.attention(q, k, v, segs, 16, 8, D, scale))
    for r in (0, 3, 300, 303):
        assert not got[r].any()


def test_batch_segments_no_bias(cuda):
    """The batch layout of LM::forward (lm.cpp:371-375) with no bias."""
    rng = np.random.default_rng(9)
    q, k, v, segs = make_case(rng, (100, 100, 100, 100), 16, 8)
    segs = [(None, r, qo, ko) for _, r, qo, ko in segs]
    scale = 1.0 / np.sqrt(D)
    compare(run(q, k, v, segs, 16, 8, scale, cuda), O.attention(q, k, v, segs, 16, 8, D, scale))


def test_peaked_scores(cuda):
    """Large logits (|score| up to ~40): the softmax max-subtraction keeps
    the fp16 probabilities in range."""
    rng = np.random.default_rng(3)
    q, k, v, segs = make_case(rng, (180,), 16, 8, scale_qk=2.5)
    scale = 1.0 / np.sqrt(D)
    compare(run(q, k, v, segs, 16, 8, scale, cuda), O.attention(q, k, v, segs, 16, 8, D, scale))


def test_uncovered_rows_untouched(cuda):
    rng = np.random.default_rng(4)
    q, k, v, segs = make_case(rng, (64, 40, 64), 16, 8)
    segs = [segs[0], segs[2]]  # the middle 40 rows belong to no segment
    out = np.full_like(q, 7.0)
    scale = 1.0 / np.sqrt(D)
    got = run(q, k, v, segs, 16, 8, scale, cuda, out=out)
    assert (got[64:104] == 7.0).all()
    want = O.attention(q, k, v, segs, 16, 8, D, scale)
    compare(got[np.r_[0:64, 104:168]], want[np.r_[0:64, 104:168]])


def test_many_segments(cuda):
    rng = np.random.default_rng(12)
    rows = tuple(int(x) for x in rng.integers(1, 40, size=64))
    q, k, v, segs = make_case(rng, rows, 4, 2, masked_rows=(0,))
    scale = 0.09
    compare(run(q, k, v, segs, 4, 2, scale, cuda), O.attention(q, k, v, segs, 4, 2, D, scale))


def test_strided_views_with_column_offset(cuda):
    """q / k / v as column windows of wider row-major buffers (row stride
    larger than the heads, segment offsets not at column 0), through the C
    ABI directly."""
    import ctypes as C
    import ovnative_b200._lib as L
    rng = np.random.default_rng(21)
    seg_rows = (140, 70)
    q, k, v, segs = make_case(rng, seg_rows, 8, 2, masked_rows=(4,), pad_keys=3)
    T, QD, KVD = q.shape[0], q.shape[1], k.shape[1]
    qpad, kvpad = 256, 132
    qb = np.zeros((T, QD + qpad), np.float32)
    kb = np.zeros((T, KVD + kvpad), np.float32)
    vb = np.zeros((T, KVD + kvpad), np.float32)
    qb[:, qpad:] = q
    kb[:, kvpad:] = k
    vb[:, kvpad:] = v
    tq, tk, tv = (torch.from_numpy(x).to(cuda) for x in (qb, kb, vb))
    out = torch.zeros_like(tq)
    biases = [torch.from_numpy(b).to(cuda) for b, _, _, _ in segs]
    arr = (L.AttnSegment * len(segs))()
    r0 = 0
    for i, (_, rows, _, _) in enumerate(segs):
        arr[i] = L.AttnSegment(biases[i].data_ptr(), rows, r0 * (QD + qpad) + qpad,
                               r0 * (KVD + kvpad) + kvpad)
        r0 += rows
    L.check(L.lib().ovb_attention(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), out.data_ptr(),
                                  QD + qpad, KVD + kvpad, 8, 2, D, 0.07,
                                  C.cast(arr, C.POINTER(L.AttnSegment)), len(segs),
                                  torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert ovb.device_status() == 0
    got = out.cpu().numpy()
    assert not got[:, :qpad].any()
    compare(got[:, qpad:], O.attention(q, k, v, segs, 8, 2, D, 0.07))


def test_fp16_range_flag(cuda):
    """A value beyond the fp16 range sets status bit 16 (and is cleared by
    the read)."""
    rng = np.random.default_rng(8)
    q, k, v, segs = make_case(rng, (40,), 2, 1)
    k[3, 5] = 1e5
    tq, tk, tv = (torch.from_numpy(x).to(cuda) for x in (q, k, v))
    ovb.attention(tq, tk, tv, [(None, 40, 0, 0)], 2, 1, 0.05)
    torch.cuda.synchronize()
    assert ovb.device_status() == 16
    assert ovb.device_status() == 0


@pytest.mark.parametrize("slope", [0.1, -0.1, 0.03])
def test_rescale_paths(cuda, slope):
    """A bias rising along the keys by 12.8 per 128-key tile moves the softmax
    reference point (and rescales O in TMEM) on every tile; a falling one
    keeps the first tile's maximum; 3.8 per tile stays under the rescale
    threshold for several tiles."""
    rng = np.random.default_rng(int(abs(slope) * 1000) + (slope > 0))
    S = 700
    q, k, v, _ = make_case(rng, (S,), 4, 2)
    bias = np.broadcast_to((slope * np.arange(S)).astype(np.float32), (S, S)).copy()
    bias[:, 5] = -1e30
    segs = [(bias, S, 0, 0)]
    scale = 1.0 / np.sqrt(D)
    compare(run(q, k, v, segs, 4, 2, scale, cuda), O.attention(q, k, v, segs, 4, 2, D, scale))


def test_long_segment(cuda):
    """1500 rows: 12 key tiles and 12 query blocks per head."""
    rng = np.random.default_rng(15)
    q, k, v, segs = make_case(rng, (1500,), 4, 1, masked_rows=(7,), pad_keys=11)
    scale = 1.0 / np.sqrt(D)
    got = run(q, k, v, segs, 4, 1, scale, cuda)
    compare(got, O.attention(q, k, v, segs, 4, 1, D, scale))
    assert not got[7].any()
