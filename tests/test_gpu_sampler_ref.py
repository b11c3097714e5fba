"""The device guided sampler (ovb_guided_sample) and the oracle's C
restatement, both against the reference's OWN CUDA sampler: its
guided_sample_kernel (cpp/src/backend/cuda/cuda_lm.cu:679-758), compiled
unchanged from the reference's source for sm_100a into oracle/_ref and
launched as its LmRunnerSampleThunk launches it (cuda_lm.cu:1227-1252).

Contract (the same as against the restatement): scores within
2e-5 * (1 + |score|) -- the two kernels sum exponentials in different orders
and both use the hardware's approximate exp and log -- and predictions equal
wherever the two best mixed log-probabilities differ by more than 1e-4."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from tests.test_gpu_sampler import make, second_gap

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_cuda_available(),
                                 reason="oracle/_ref/libovref_cuda.so not built")]


def _compare(cond, unc, C, V, T, g, pen, mask_id, cuda):
    tc, tu = torch.from_numpy(cond).to(cuda), torch.from_numpy(unc).to(cuda)
    ref_p, ref_s = O.ref_cuda_guided_sample(tc, tu, T, C, g, pen, mask_id)
    got_p, got_s = ovb.guided_sample(tc, tu, T, C, g, pen, mask_id)
    torch.cuda.synchronize()
    ref_p, ref_s = ref_p.cpu().numpy(), ref_s.cpu().numpy()
    got_p, got_s = got_p.cpu().numpy(), got_s.cpu().numpy()
    port_p, port_s = O.guided_sample(cond, unc, T, C, g, pen, mask_id)
    clear = second_gap(cond, unc, C, V, T, g, mask_id) > 1e-4
    for name, p, s in (("ovb_guided_sample", got_p, got_s), ("restatement", port_p, port_s)):
        np.testing.assert_allclose(s, ref_s, rtol=2e-5, atol=2e-5, err_msg=name)
        assert (p[clear] == ref_p[clear]).all(), name
    assert clear.mean() > 0.9
    assert ovb.device_status() == 0


@pytest.mark.parametrize("C,V,T,cs,us,g,pen", [
    (8, 1025, 585, 700, 585, 2.0, 5.0),   # config 3's step, the defaults of TtsOptions
    (8, 1025, 260, 300, 300, 3.0, 5.0),   # config 2, B = 2 planes of equal length
    (8, 1025, 37, 40, 37, 0.0, 1.0),      # no guidance
    (2, 1025, 5, 9, 5, -0.5, 0.0),        # negative guidance
])
def test_matches_reference_cuda_kernel(cuda, C, V, T, cs, us, g, pen):
    rng = np.random.default_rng(C * 1000 + T)
    cond, unc = make(rng, C, V, cs, us)
    _compare(cond, unc, C, V, T, g, pen, 1024, cuda)


@pytest.mark.parametrize("mask_id", [0, 1024, -1])
def test_mask_token_like_reference(cuda, mask_id):
    """The mask token is excluded from the argmax (not from the normaliser),
    and a mask id outside the vocabulary excludes nothing."""
    rng = np.random.default_rng(7)
    C, V, T = 4, 1025, 50
    cond, unc = make(rng, C, V, 60, 50)
    if 0 <= mask_id < V:  # make the mask token the row maximum
        cond[:, np.arange(C) * V + mask_id] += 50.0
    _compare(cond, unc, C, V, T, 2.0, 5.0, mask_id, cuda)


def test_peaked_rows_like_reference(cuda):
    """Rows with one dominant token (as trained heads give) and rows with
    large logits (|x| ~ 30) agree as well."""
    rng = np.random.default_rng(11)
    C, V, T = 8, 1025, 64
    cond, unc = make(rng, C, V, 64, 64, scale=30.0)
    cond[np.arange(T), rng.integers(0, C * V, size=T)] += 40.0
    _compare(cond, unc, C, V, T, 2.0, 5.0, 1024, cuda)
