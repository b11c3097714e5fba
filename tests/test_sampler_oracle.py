"""The sampler's CPU checker (oracle.guided_sample, a restatement of
cpp/src/model/tts.cpp:91-101 and :291-326) against an independent float64
evaluation of the same formulas, and the reference's in-place log_softmax
quirk (tts.cpp:313) it can reproduce.  CPU only."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O


def log_softmax64(x):
    m = x.max()
    return x - (np.log(np.exp(x - m).sum()) + m)


def planes(rng, C, V, T, cond_seq, uncond_seq, scale=3.0):
    cond = (rng.standard_normal((cond_seq, C * V)) * scale).astype(np.float32)
    unc = (rng.standard_normal((uncond_seq, C * V)) * scale).astype(np.float32)
    return cond, unc


def expected64(cond, unc, C, V, T, g, pen, mask_id):
    S = cond.shape[0]
    pred = np.zeros((C, T), np.int64)
    score = np.zeros((C, T))
    gap = np.zeros((C, T))
    for c in range(C):
        for t in range(T):
            a = log_softmax64(cond[S - T + t, c * V:(c + 1) * V].astype(np.float64))
            b = log_softmax64(unc[t, c * V:(c + 1) * V].astype(np.float64))
            mix = log_softmax64(a + g * (a - b)) if g != 0 else a
            if 0 <= mask_id < V:
                mix[mask_id] = -np.inf
            order = np.argsort(-mix, kind="stable")
            pred[c, t] = order[0]
            score[c, t] = mix[order[0]] - c * pen
            gap[c, t] = mix[order[0]] - mix[order[1]]
    return pred, score, gap


@pytest.mark.parametrize("C,V,T,cond_seq,uncond_seq,g,mask_id", [
    (8, 1025, 6, 10, 6, 3.0, 1024),
    (8, 1025, 4, 4, 9, 0.0, 1024),
    (2, 37, 5, 7, 5, 1.5, 0),
    (3, 300, 3, 3, 3, -0.5, -1),
])
def test_oracle_sampler_matches_float64(C, V, T, cond_seq, uncond_seq, g, mask_id):
    rng = np.random.default_rng(C * 1000 + V + T)
    cond, unc = planes(rng, C, V, T, cond_seq, uncond_seq)
    pred, scores = O.guided_sample(cond, unc, T, C, g, 5.0, mask_id)
    want_p, want_s, gap = expected64(cond, unc, C, V, T, g, 5.0, mask_id)
    clear = gap > 1e-4
    assert (pred[clear] == want_p[clear]).all()
    np.testing.assert_allclose(scores, want_s, rtol=1e-5, atol=1e-4)
    if 0 <= mask_id < V:
        assert (pred != mask_id).all()


def test_oracle_sampler_in_place_quirk():
    """tts.cpp:313 calls log_softmax(lp_mix, V, lp_mix): its second loop
    overwrites the input with exp(x - m), so the third returns
    exp(mix - max) - lse instead of mix - lse.  The argmax is unchanged (the
    map is monotonic); the scores are not."""
    rng = np.random.default_rng(7)
    C, V, T = 4, 1025, 3
    cond, unc = planes(rng, C, V, T, 5, 3)
    p1, s1 = O.guided_sample(cond, unc, T, C, 3.0, 5.0, in_place=False)
    p2, s2 = O.guided_sample(cond, unc, T, C, 3.0, 5.0, in_place=True)
    assert (p1 == p2).all()
    assert np.abs(s1 - s2).max() > 1.0
    for c in range(C):
        for t in range(T):
            a = log_softmax64(cond[5 - T + t, c * V:(c + 1) * V].astype(np.float64))
            b = log_softmax64(unc[t, c * V:(c + 1) * V].astype(np.float64))
            mix = a + 3.0 * (a - b)
            m = mix.max()
            lse = np.log(np.exp(mix - m).sum()) + m
            masked = mix.copy()
            masked[1024] = -np.inf
            quirk = np.exp(masked.max() - m) - lse - 5.0 * c
            assert abs(s2[c, t] - quirk) < 1e-3 * (1 + abs(quirk))


def test_oracle_sampler_ties_pick_first():
    C, V, T = 2, 64, 2
    cond = np.zeros((T, C * V), np.float32)
    unc = np.zeros((T, C * V), np.float32)
    pred, scores = O.guided_sample(cond, unc, T, C, 2.0, 1.0, mask_id=0)
    assert (pred == 1).all()  # token 0 is masked; 1 is the first of the equal rest
    np.testing.assert_allclose(scores[1], -np.log(64.0) - 1.0, rtol=1e-5)
