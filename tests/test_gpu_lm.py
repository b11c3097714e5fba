"""The whole LM forward on the device (ovb_lm_*, from an OVW1 checkpoint)
against the reference's own LM forward (cpp/src/model/lm.cpp, oracle/_ref)
on the same random checkpoint and inputs -- the end-to-end pin, judged as the
reference's own LM test judges an int8 forward (cpp/tests/test_lm.cpp:
198-231: cosine, mean |delta| and argmax agreement over every (row,
codebook) position), with tighter bounds: both sides run the same int8
arithmetic, and only the attention (fp16 operands), RoPE (CUDA's cos/sin)
and the fp16 mainloop (when selected) differ."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from ovnative_b200 import lm as LM
from ovnative_b200 import ovw1
from tests.test_lm_oracle import C, V, cfg_inputs

pytestmark = pytest.mark.gpu

LAYERS, VOCAB = 2, 512


@pytest.fixture(scope="module")
def model_path():
    import os
    import shutil

    from tests.conftest import ROOT
    d = os.path.join(ROOT, ".test_tmp", "gpu_lm")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, "lm2.ovw")
    ovw1.random_lm(p, n_layers=LAYERS, vocab=VOCAB, seed=7)
    yield p
    shutil.rmtree(d, ignore_errors=True)


def metrics(got, want):
    g = got.reshape(-1, V).astype(np.float64)
    w = want.reshape(-1, V).astype(np.float64)
    cos = float((g * w).sum() / (np.linalg.norm(g) * np.linalg.norm(w)))
    mean = float(np.abs(g - w).mean())
    agree = float((g.argmax(1) == w.argmax(1)).mean())
    return cos, mean, agree


@pytest.mark.parametrize("f16", [False, True])
def test_forward_cfg_matches_reference(cuda, model_path, f16):
    rng = np.random.default_rng(11)
    ids, amask, cond, unc, pos = cfg_inputs(rng, 150, 97, VOCAB)
    want = O.RefLM(model_path, LAYERS).forward_cfg(ids, amask, cond, unc, pos)
    m = LM.LM(model_path, f16=f16)
    assert m.config["n_layers"] == LAYERS and m.config["vocab"] == VOCAB
    got = m.forward_cfg(ids, amask, cond, unc, pos)
    cos, mean, agree = metrics(got, want)
    print(f"f16={f16} cos={cos:.8f} mean={mean:.3e} agree={agree:.4f}")
    assert np.isfinite(got).all()
    assert cos > (0.9999 if f16 else 0.99999)
    assert mean < 0.02 * float(np.abs(want).mean())
    assert agree >= (0.97 if f16 else 0.99)
    assert ovb.device_status() == 0
    m.close()


def test_forward_batched_matches_reference(cuda, model_path):
    rng = np.random.default_rng(12)
    B, S = 2, 90
    ids = rng.integers(0, V, size=(B, C, S)).astype(np.int64)
    amask = np.ones((B, S), np.uint8)
    amask[:, :10] = 0
    ids[:, 0, :10] = rng.integers(0, VOCAB, size=(B, 10))
    attn = np.ones((B, S, S), np.uint8)
    attn[1, :, :4] = 0
    pos = np.tile(np.arange(S, dtype=np.int64), (B, 1))
    want = O.RefLM(model_path, LAYERS).forward(ids, amask, attn, pos)
    m = LM.LM(model_path)
    got = m.forward(ids, amask, attn, pos)
    assert got.shape == (B, C, S, V)
    cos, mean, agree = metrics(got, want)
    print(f"batched cos={cos:.8f} mean={mean:.3e} agree={agree:.4f}")
    assert cos > 0.99999 and agree >= 0.99
    assert ovb.device_status() == 0
    m.close()


def test_device_forward_equals_host_forward(cuda, model_path):
    rng = np.random.default_rng(13)
    ids, amask, cond, unc, pos = cfg_inputs(rng, 64, 40, VOCAB)
    m = LM.LM(model_path)
    host = m.forward_cfg(ids, amask, cond, unc, pos)
    t = [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (ids, amask, cond, unc, pos)]
    dev = m.forward_cfg_device(*t)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dev.cpu().numpy(), host)
    m.close()


def test_bad_ids_flagged_not_faulted(cuda, model_path):
    """A token id outside the table leaves its row zero and sets status bit
    128 instead of reading out of bounds."""
    rng = np.random.default_rng(14)
    ids, amask, cond, unc, pos = cfg_inputs(rng, 30, 20, VOCAB)
    ids[0, 3] = VOCAB + 5  # a text row (amask 0)
    m = LM.LM(model_path)
    with pytest.raises(Exception, match="status 128"):
        m.forward_cfg(ids, amask, cond, unc, pos)
    assert ovb.device_status() == 0
    m.close()


@pytest.fixture(scope="module")
def model_path_f32_heads():
    import os
    import shutil

    from tests.conftest import ROOT
    d = os.path.join(ROOT, ".test_tmp", "gpu_lm_f32h")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, "lm2f.ovw")
    ovw1.random_lm(p, n_layers=LAYERS, vocab=VOCAB, seed=9, heads_f32=True)
    yield p
    shutil.rmtree(d, ignore_errors=True)


@pytest.mark.parametrize("f16", [False, True])
def test_fp32_audio_heads_match_reference(cuda, model_path_f32_heads, f16):
    """The reference's default checkpoint keeps the audio heads fp32
    (tools/convert_weights.py:326-327); its LM runs them through linear_f32
    (lm.cpp:449-451).  The device LM takes them on the fp16 tensor cores:
    fp16 of the normalised rows times fp16 heads (power-of-two channel
    scales), fp32 accumulation -- judged like the int8 heads above."""
    rng = np.random.default_rng(21)
    ids, amask, cond, unc, pos = cfg_inputs(rng, 120, 80, VOCAB)
    want = O.RefLM(model_path_f32_heads, LAYERS).forward_cfg(ids, amask, cond, unc, pos)
    m = LM.LM(model_path_f32_heads, f16=f16)
    got = m.forward_cfg(ids, amask, cond, unc, pos)
    cos, mean, agree = metrics(got, want)
    print(f"fp32 heads f16={f16} cos={cos:.8f} mean={mean:.3e} agree={agree:.4f}")
    assert np.isfinite(got).all()
    assert cos > (0.9999 if f16 else 0.99999)
    assert mean < 0.02 * float(np.abs(want).mean())
    assert agree >= (0.97 if f16 else 0.99)
    assert ovb.device_status() == 0
    m.close()


def _pack_pairs(pairs):
    """Concatenate per-pair forward_cfg inputs into one segment-packed batch."""
    ids = np.concatenate([p[0] for p in pairs], axis=1)
    amask = np.concatenate([p[1] for p in pairs])
    masks = np.concatenate([m.reshape(-1) for p in pairs for m in (p[2], p[3])])
    pos = np.concatenate([p[4] for p in pairs])
    seg_rows = [r for p in pairs for r in (p[2].shape[0], p[3].shape[0])]
    return seg_rows, ids, amask, masks, pos


@pytest.mark.parametrize("f16", [False, True])
def test_segment_packed_forward_equals_one_pair_at_a_time(cuda, model_path, f16):
    """Several utterances' CFG pairs in one forward (ovb_lm_forward_segments_
    device) give each pair the logits of its own forward_cfg: every step but
    attention works row by row and attention stays inside each segment.  The
    int8 mainloop's per-row results do not depend on M, so they are equal
    bit for bit; the fp16 mainloop may pick another split-K for the larger
    M, so its results agree to the fp16 path's tolerance."""
    rng = np.random.default_rng(31)
    pairs = [cfg_inputs(rng, cs, us, VOCAB) for cs, us in ((70, 70), (33, 20), (129, 97))]
    m = LM.LM(model_path, f16=f16)
    seg_rows, ids, amask, masks, pos = _pack_pairs(pairs)
    t = [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (ids, amask, masks, pos)]
    m.reserve(sum(seg_rows), int(sum(r * r for r in seg_rows)))
    packed = m.forward_segments_device(seg_rows, *t).cpu().numpy()
    r0 = 0
    for p in pairs:
        single = m.forward_cfg(*p)
        got = packed[r0:r0 + single.shape[0]]
        if f16:
            err = np.linalg.norm(got - single) / np.linalg.norm(single)
            assert err < 1e-3, err
        else:
            np.testing.assert_array_equal(got, single)
        r0 += single.shape[0]
    assert ovb.device_status() == 0
    m.close()
