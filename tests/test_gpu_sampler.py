"""The device guided-argmax pass (ovb_guided_sample) against the CPU
checker (oracle.guided_sample, the log-probabilities that
cpp/src/model/tts.cpp:291-326 computes -- and the reference's CUDA kernel,
cpp/src/backend/cuda/cuda_lm.cu:679-758).

Contract: scores within 2e-5 * (1 + |score|) (both sides sum exp values in a
different order); pred identical wherever the best and second-best mixed
log-probabilities differ by more than 1e-4 (below that, rounding can flip
the winner on either side)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb

pytestmark = pytest.mark.gpu


def make(rng, C, V, cond_seq, uncond_seq, scale=3.0):
    cond = (rng.standard_normal((cond_seq, C * V)) * scale).astype(np.float32)
    unc = (rng.standard_normal((uncond_seq, C * V)) * scale).astype(np.float32)
    return cond, unc


def second_gap(cond, unc, C, V, T, g, mask_id):
    """Best minus second-best mixed log-probability per row (float64)."""
    S = cond.shape[0]
    gap = np.zeros((C, T))
    for c in range(C):
        for t in range(T):
            a = cond[S - T + t, c * V:(c + 1) * V].astype(np.float64)
            b = unc[t, c * V:(c + 1) * V].astype(np.float64)
            a = a - (np.log(np.exp(a - a.max()).sum()) + a.max())
            b = b - (np.log(np.exp(b - b.max()).sum()) + b.max())
            mix = a + g * (a - b) if g != 0 else a
            if 0 <= mask_id < V:
                mix[mask_id] = -np.inf
            top = np.sort(mix)[-2:]
            gap[c, t] = top[1] - top[0]
    return gap


def check(cond, unc, C, V, T, g, pen, mask_id, cuda):
    pred, scores = ovb.guided_sample(torch.from_numpy(cond).to(cuda),
                                     torch.from_numpy(unc).to(cuda), T, C, g, pen, mask_id)
    torch.cuda.synchronize()
    want_p, want_s = O.guided_sample(cond, unc, T, C, g, pen, mask_id)
    got_p, got_s = pred.cpu().numpy(), scores.cpu().numpy()
    assert got_p.shape == (C, T) and got_s.shape == (C, T)
    np.testing.assert_allclose(got_s, want_s, rtol=2e-5, atol=2e-5)
    clear = second_gap(cond, unc, C, V, T, g, mask_id) > 1e-4
    assert (got_p[clear] == want_p[clear]).all()
    if 0 <= mask_id < V:
        assert (got_p != mask_id).all()
    assert ovb.device_status() == 0
    return got_p, got_s


# V = 1025 is the LM's audio vocabulary (8 codebooks x 1025 = the 8200-wide
# heads); 1500 takes the 64-per-lane register kernel, 3000 the generic one.
@pytest.mark.parametrize("C,V,T,cond_seq,uncond_seq", [
    (8, 1025, 37, 45, 37), (8, 1025, 1, 1, 1), (8, 1025, 64, 300, 300), (2, 1500, 9, 12, 9),
    (3, 3000, 5, 5, 8), (4, 7, 6, 6, 6), (1, 33, 40, 41, 40)])
@pytest.mark.parametrize("g", [3.0, 0.0, -0.75])
def test_guided_sample_matches_oracle(cuda, C, V, T, cond_seq, uncond_seq, g):
    rng = np.random.default_rng(C * 7919 + V * 31 + T + int(g * 4))
    cond, unc = make(rng, C, V, cond_seq, uncond_seq)
    check(cond, unc, C, V, T, g, 5.0, 1024, cuda)


@pytest.mark.parametrize("mask_id", [-1, 0, 1024, 5000])
def test_guided_sample_mask(cuda, mask_id):
    rng = np.random.default_rng(11 + mask_id)
    C, V, T = 8, 1025, 12
    cond, unc = make(rng, C, V, 20, 12)
    if 0 <= mask_id < V:  # make the mask token the clear winner before masking
        cond[:, mask_id::V] += 50.0
    check(cond, unc, C, V, T, 2.0, 5.0, mask_id, cuda)


def test_guided_sample_ties_and_extremes(cuda):
    C, V, T = 3, 1025, 4
    cond = np.zeros((T, C * V), np.float32)
    unc = np.zeros((T, C * V), np.float32)
    pred, scores = ovb.guided_sample(torch.from_numpy(cond).to(cuda),
                                     torch.from_numpy(unc).to(cuda), T, C, 3.0, 1.0, 0)
    assert (pred.cpu().numpy() == 1).all()  # all equal, token 0 masked: the first of the rest
    # large logits (exp range) and a one-hot row
    rng = np.random.default_rng(5)
    cond, unc = make(rng, C, V, T, T, scale=60.0)
    cond[0, 5] = 1e4
    check(cond, unc, C, V, T, 3.0, 5.0, 1024, cuda)


def test_guided_sample_full_step_shape(cuda):
    """Config 3's target: 8 codebooks x 585 frames, cond plane of 700 tokens."""
    rng = np.random.default_rng(2024)
    C, V, T = 8, 1025, 585
    cond, unc = make(rng, C, V, 700, 585)
    check(cond, unc, C, V, T, 3.0, 5.0, 1024, cuda)


def test_guided_sample_arguments(cuda):
    C, V = 2, 16
    cond = torch.zeros((3, C * V), device=cuda)
    unc = torch.zeros((3, C * V), device=cuda)
    with pytest.raises(ValueError):
        ovb.guided_sample(cond, unc, 4, C, 1.0, 1.0)  # cond_seq < target_len
    pred, scores = ovb.guided_sample(cond, unc, 0, C, 1.0, 1.0)  # no work
    assert pred.shape == (C, 0)
    assert ovb.device_status() == 0


@pytest.mark.parametrize("V", [1025, 300])
def test_guided_sample_batch_equals_one_call_per_pair(cuda, V):
    """ovb_guided_sample_batch over ragged pairs (one launch for V = 1025, a
    loop for other V) writes exactly what one ovb_guided_sample per pair
    writes, pair after pair."""
    rng = np.random.default_rng(V)
    C, g, pen = 8, 2.0, 5.0
    planes, want_p, want_s = [], [], []
    for S, T in ((60, 20), (300, 260), (45, 0), (129, 89), (7, 7)):
        cond = torch.from_numpy((rng.standard_normal((S, C * V)) * 3).astype(np.float32)).to(cuda)
        unc = torch.from_numpy((rng.standard_normal((S, C * V)) * 3).astype(np.float32)).to(cuda)
        planes.append((cond, unc, T))
        p, s = ovb.guided_sample(cond, unc, T, C, g, pen)
        want_p.append(p.reshape(-1))
        want_s.append(s.reshape(-1))
    n = sum(C * T for _, _, T in planes)
    pred = torch.full((n + 5,), -1, dtype=torch.int32, device=cuda)
    scores = torch.full((n + 5,), float("nan"), device=cuda)
    ovb.guided_sample_batch(planes, C, g, pen, pred, scores)
    assert torch.equal(pred[:n], torch.cat(want_p))
    assert torch.equal(scores[:n], torch.cat(want_s))
    assert (pred[n:] == -1).all() and torch.isnan(scores[n:]).all()  # nothing past the outputs
    with pytest.raises(ValueError):
        ovb.guided_sample_batch(planes, C, g, pen, pred[: n - 1], scores)
