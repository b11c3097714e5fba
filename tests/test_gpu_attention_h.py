"""The fp16-operand attention (ovb_attention_h; warp-specialised, two query
heads per CTA, S / P / O in tensor memory, V read as an MN-major operand)
against the reference's own ov::attention_head_f32 (oracle.attention;
cpp/src/backend/cpu/ops_cpu.cpp:907-943 over the loop of LM::run_layer,
cpp/src/model/lm.cpp:256-274), with the reference's fp32 q / k / v and the
device's fp16 copies of them.

Each case runs twice: with the segments' fp32 biases read per element, and
with the tile table built from the u8 masks the biases encode
(ovb_attention_tiles: whole tiles attended, mixed, or skipped).  Contract as
for ovb_attention: rel-L2 <= 2e-3 and max-abs <= 2e-2 * rms of the
reference; fully masked rows exactly zero; rows outside every segment
untouched; device status 0."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from tests.test_attention_oracle import D, make_case
from tests.test_gpu_attention import compare

pytestmark = pytest.mark.gpu


def run_h(q, k, v, segs, n_heads, n_kv, scale, cuda, mode, out=None):
    tq, tk, tv = (torch.from_numpy(x.astype(np.float16)).to(cuda) for x in (q, k, v))
    o = None if out is None else torch.from_numpy(out).to(cuda)
    if mode == "bias":
        tsegs = [(None if b is None else torch.from_numpy(b).to(cuda), r, qo, ko)
                 for b, r, qo, ko in segs]
        got = ovb.attention_h(tq, tk, tv, tsegs, n_heads, n_kv, scale, out=o)
    else:
        rows = [r for _, r, _, _ in segs]
        masks = np.concatenate([(np.ones((r, r), np.uint8) if b is None else
                                 (b > -1e29).astype(np.uint8)).reshape(-1)
                                for b, r, _, _ in segs] + [np.zeros(1, np.uint8)])
        tiles = ovb.attention_tiles(rows, torch.from_numpy(masks).to(cuda))
        got = ovb.attention_h(tq, tk, tv, [(None, r, qo, ko) for _, r, qo, ko in segs],
                              n_heads, n_kv, scale, out=o, tiles=tiles)
    torch.cuda.synchronize()
    assert ovb.device_status() == 0
    return got.cpu().numpy()


MODES = ["bias", "table"]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("rows", [1, 2, 31, 128, 129, 200, 256, 385])
def test_single_segment(rows, mode, cuda):
    rng = np.random.default_rng(rows)
    q, k, v, segs = make_case(rng, (rows,), 16, 8, masked_rows=(1,), pad_keys=2)
    scale = 1.0 / np.sqrt(D)
    got = run_h(q, k, v, segs, 16, 8, scale, cuda, mode)
    compare(got, O.attention(q, k, v, segs, 16, 8, D, scale))
    if rows > 1:
        assert not got[1].any()


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("n_heads,n_kv", [(16, 16), (16, 8), (16, 4), (8, 1), (6, 2)])
def test_gqa_groups(n_heads, n_kv, mode, cuda):
    """Groups of 1 (one head per CTA), 2 (one pair), 4 and 8 (several pairs
    per kv head) and 3 (a pair and a single head)."""
    rng = np.random.default_rng(n_heads * 10 + n_kv)
    q, k, v, segs = make_case(rng, (150,), n_heads, n_kv, masked_rows=(3,), pad_keys=1)
    scale = 1.0 / np.sqrt(D)
    compare(run_h(q, k, v, segs, n_heads, n_kv, scale, cuda, mode),
            O.attention(q, k, v, segs, n_heads, n_kv, D, scale))


@pytest.mark.parametrize("mode", MODES)
def test_cfg_pair_segments(mode, cuda):
    rng = np.random.default_rng(7)
    q, k, v, segs = make_case(rng, (300, 97), 16, 8, masked_rows=(0, 3), pad_keys=5)
    scale = 1.0 / np.sqrt(D)
    got = run_h(q, k, v, segs, 16, 8, scale, cuda, mode)
    compare(got, O.attention(q, k, v, segs, 16, 8, D, scale))
    for r in (0, 3, 300, 303):
        assert not got[r].any()


@pytest.mark.parametrize("mode", MODES)
def test_batch_segments_no_bias(mode, cuda):
    rng = np.random.default_rng(9)
    q, k, v, segs = make_case(rng, (100, 100, 100, 100), 16, 8)
    segs = [(None, r, qo, ko) for _, r, qo, ko in segs]
    scale = 1.0 / np.sqrt(D)
    compare(run_h(q, k, v, segs, 16, 8, scale, cuda, mode),
            O.attention(q, k, v, segs, 16, 8, D, scale))


@pytest.mark.parametrize("mode", MODES)
def test_peaked_scores(mode, cuda):
    rng = np.random.default_rng(3)
    q, k, v, segs = make_case(rng, (180,), 16, 8, scale_qk=2.5)
    scale = 1.0 / np.sqrt(D)
    compare(run_h(q, k, v, segs, 16, 8, scale, cuda, mode),
            O.attention(q, k, v, segs, 16, 8, D, scale))


@pytest.mark.parametrize("mode", MODES)
def test_uncovered_rows_untouched(mode, cuda):
    rng = np.random.default_rng(4)
    q, k, v, segs = make_case(rng, (64, 40, 64), 16, 8)
    segs = [segs[0], segs[2]]  # the middle 40 rows belong to no segment
    out = np.full_like(q, 7.0)
    scale = 1.0 / np.sqrt(D)
    got = run_h(q, k, v, segs, 16, 8, scale, cuda, mode, out=out)
    assert (got[64:104] == 7.0).all()
    want = O.attention(q, k, v, segs, 16, 8, D, scale)
    compare(got[np.r_[0:64, 104:168]], want[np.r_[0:64, 104:168]])


@pytest.mark.parametrize("mode", MODES)
def test_many_segments(mode, cuda):
    rng = np.random.default_rng(12)
    rows = tuple(int(x) for x in rng.integers(1, 300, size=64))
    q, k, v, segs = make_case(rng, rows, 4, 2, masked_rows=(0,))
    scale = 0.09
    compare(run_h(q, k, v, segs, 4, 2, scale, cuda, mode),
            O.attention(q, k, v, segs, 4, 2, D, scale))


@pytest.mark.parametrize("slope", [0.1, -0.1, 0.03])
def test_rescale_paths(cuda, slope):
    """Biases rising along the keys move the softmax reference point on every
    tile (O rescaled in TMEM), falling ones never after the first."""
    rng = np.random.default_rng(int(abs(slope) * 1000) + (slope > 0))
    S = 700
    q, k, v, _ = make_case(rng, (S,), 4, 2)
    bias = np.broadcast_to((slope * np.arange(S)).astype(np.float32), (S, S)).copy()
    bias[:, 5] = -1e30
    segs = [(bias, S, 0, 0)]
    scale = 1.0 / np.sqrt(D)
    compare(run_h(q, k, v, segs, 4, 2, scale, cuda, "bias"),
            O.attention(q, k, v, segs, 4, 2, D, scale))


@pytest.mark.parametrize("mode", MODES)
def test_long_segment(mode, cuda):
    rng = np.random.default_rng(15)
    q, k, v, segs = make_case(rng, (1500,), 4, 1, masked_rows=(7,), pad_keys=11)
    scale = 1.0 / np.sqrt(D)
    got = run_h(q, k, v, segs, 4, 1, scale, cuda, mode)
    compare(got, O.attention(q, k, v, segs, 4, 1, D, scale))
    assert not got[7].any()


def test_table_skips_masked_tiles_like_the_bias(cuda):
    """The reference CUDA path's unconditional row (tts.cpp:186-198): keys past
    the target slice masked for the slice's queries, the tail rows seeing only
    themselves -- so whole key tiles are skipped for the first query blocks,
    others are mixed -- plus a query block whose rows see nothing at all."""
    rng = np.random.default_rng(31)
    S, T = 700, 260
    q, k, v, _ = make_case(rng, (S,), 16, 8)
    allow = np.zeros((S, S), bool)
    allow[:T, :T] = True
    allow[np.arange(T, S), np.arange(T, S)] = True
    allow[512:640] = False           # a whole query block fully masked
    bias = np.where(allow, 0.0, -1e30).astype(np.float32)
    segs = [(bias, S, 0, 0)]
    scale = 1.0 / np.sqrt(D)
    want = O.attention(q, k, v, segs, 16, 8, D, scale)
    for mode in MODES:
        got = run_h(q, k, v, segs, 16, 8, scale, cuda, mode)
        compare(got, want)
        assert not got[512:640].any()
    masks = torch.from_numpy(allow.astype(np.uint8).reshape(-1)).to(cuda)
    tiles = ovb.attention_tiles([S], masks).cpu().numpy()
    cls = tiles[:36].reshape(6, 6)   # 6 query blocks x 6 key tiles
    assert cls[0, 0] == 0 and cls[0, 3] == 3 and cls[0, 2] == 1 and (cls[4] == 3).all()


def test_matches_fp32_entry_point(cuda):
    """ovb_attention_h equals the fp32-operand ovb_attention to the
    precision both share (fp16 operands)."""
    rng = np.random.default_rng(5)
    q, k, v, segs = make_case(rng, (300, 300), 16, 8, pad_keys=8)
    scale = 1.0 / np.sqrt(D)
    tq, tk, tv = (torch.from_numpy(x).to(cuda) for x in (q, k, v))
    tsegs = [(torch.from_numpy(b).to(cuda), r, qo, ko) for b, r, qo, ko in segs]
    a = ovb.attention(tq, tk, tv, tsegs, 16, 8, scale).cpu().numpy()
    b = run_h(q, k, v, segs, 16, 8, scale, cuda, "table")
    assert np.linalg.norm(a - b) <= 1e-3 * np.linalg.norm(a)


@pytest.mark.parametrize("form", ["int8", "u8", "fp16"])
@pytest.mark.parametrize("mode", MODES)
def test_fused_quantised_output_equals_quantise_of_output(form, mode, cuda):
    """ovb_attention_h_q writes exactly ovb_quantize(ovb_attention_h(...)):
    the same fp32 values, quantised per 32-k block in the epilogue."""
    rng = np.random.default_rng(41)
    q, k, v, segs = make_case(rng, (300, 97, 150), 16, 8, masked_rows=(2,), pad_keys=4)
    scale = 1.0 / np.sqrt(D)
    tq, tk, tv = (torch.from_numpy(x.astype(np.float16)).to(cuda) for x in (q, k, v))
    if mode == "bias":
        tsegs = [(torch.from_numpy(b).to(cuda), r, qo, ko) for b, r, qo, ko in segs]
        tiles = None
    else:
        tsegs = [(None, r, qo, ko) for _, r, qo, ko in segs]
        masks = np.concatenate([(b > -1e29).astype(np.uint8).reshape(-1) for b, _, _, _ in segs])
        tiles = ovb.attention_tiles([r for _, r, _, _ in segs], torch.from_numpy(masks).to(cuda))
    kw = {"u8": form == "u8", "f16": form == "fp16"}
    out = ovb.attention_h(tq, tk, tv, tsegs, 16, 8, scale, tiles=tiles)
    want_q, want_s = ovb.s8_nk_quantize(out, **kw)
    got_q, got_s = ovb.attention_h_q(tq, tk, tv, tsegs, 16, 8, scale, tiles=tiles, **kw)
    torch.cuda.synchronize()
    assert ovb.device_status() == 0
    assert torch.equal(got_q.view(torch.uint8), want_q.view(torch.uint8))
    assert torch.equal(got_s, want_s)
