"""The reference-side binding (include/ovb200_ov_hooks.hpp), compiled into a
program on the reference's own LM, Mat and WeightFile (oracle/
ov_hooks_test.cpp -> oracle/_ref/ov_hooks_test) and run on the GPU:

* LM::forward through LM::set_cuda_backend (the B200 path behind the
  reference's own hook) against the same LM on its CPU path, on the B = 2
  CFG batch the reference's CUDA path builds;
* LM::sample_guided through LM::set_cuda_sampler with device sampling (the
  forward leaves its logits on the device) against the guided-sampling
  checker on those device planes;
* ovb_hooks::Mat (the Mat dispatch on the device) against Mat::mul /
  Mat::mul_add for int8 [N, K] (bit-identical on an AVX-VNNI host: both run
  the reference's quantised int8 arithmetic), int8 [K, N] (the reference's
  AVX2 path multiplies unquantised activations, this build quantises them
  as its VNNI path does: agreement to the quantisation's ~3e-3) and fp32
  (fp16 tensor cores against fp32: rel-L2 <= 1e-3)."""
from __future__ import annotations

import json
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle as O
from ovnative_b200 import ovw1
from tests.conftest import ROOT
from tests.test_gpu_sampler import second_gap

BIN = os.path.join(ROOT, "oracle", "_ref", "ov_hooks_test")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.exists(BIN), reason="oracle/_ref/ov_hooks_test not built")]

LAYERS = 2


@pytest.fixture(scope="module")
def files():
    d = os.path.join(ROOT, ".test_tmp", "ov_hooks")
    os.makedirs(d, exist_ok=True)
    lm = os.path.join(d, "lm2.ovw")
    ovw1.random_lm(lm, n_layers=LAYERS, vocab=2048, seed=33)
    rng = np.random.default_rng(34)
    nk = rng.integers(-127, 128, size=(256, 1024), dtype=np.int8)
    kn = rng.integers(-127, 128, size=(512, 320), dtype=np.int8)
    f32 = (rng.standard_normal((768, 1000)) * 0.02).astype(np.float32)
    mats = os.path.join(d, "mats.ovw")
    ovw1.write(mats, [
        ("mat.int8_nk.weight", nk, 0, (np.abs(rng.standard_normal(256)) * 0.02 / 127)
         .astype(np.float32)),
        ("mat.int8_kn.weight", kn, 1, (np.abs(rng.standard_normal(320)) * 0.02 / 127)
         .astype(np.float32)),
        ("mat.fp32.weight", f32, 1, None),
    ])
    yield lm, mats, d
    shutil.rmtree(d, ignore_errors=True)


@pytest.mark.parametrize("flags", [0, 2])
def test_reference_lm_runs_through_the_hooks(cuda, files, flags):
    lm, mats, d = files
    out = os.path.join(d, f"out{flags}")
    os.makedirs(out, exist_ok=True)
    r = subprocess.run([BIN, lm, str(LAYERS), mats, str(flags), out], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    print("\n".join(json.dumps(x) for x in lines))
    by = {}
    for x in lines:
        by.setdefault(x["check"], []).append(x)
    assert "done" in by
    # 1. LM::forward through CudaForwardFn against the CPU path
    f = by["forward_hook"][0]
    assert f["cos"] > (0.99999 if flags == 0 else 0.9999)
    assert f["agree"] >= (0.99 if flags == 0 else 0.97)
    # 2. LM::sample_guided through CudaSampleFn on the device planes
    s = by["sample_hook"][0]
    S, T, C, V = s["S"], s["T"], s["C"], s["V"]
    assert s["host_logits_untouched"]
    planes = np.fromfile(os.path.join(out, "planes_dev.f32"), np.float32).reshape(2 * S, C * V)
    logits = np.fromfile(os.path.join(out, "logits_dev.f32"), np.float32).reshape(2, C, S, V)
    np.testing.assert_array_equal(planes.reshape(2, S, C, V).transpose(0, 2, 1, 3), logits)
    pred = np.fromfile(os.path.join(out, "pred.i32"), np.int32).reshape(C, T)
    scores = np.fromfile(os.path.join(out, "scores.f32"), np.float32).reshape(C, T)
    want_p, want_s = O.guided_sample(planes[:S], planes[S:], T, C, 2.0, 5.0, 1024)
    np.testing.assert_allclose(scores, want_s, rtol=2e-5, atol=2e-5)
    clear = second_gap(planes[:S], planes[S:], C, V, T, 2.0, 1024) > 1e-4
    assert (pred[clear] == want_p[clear]).all() and clear.mean() > 0.9
    # 3. the Mat shim against the reference's Mat
    mats_ = {x["kind"]: x for x in by["mat"]}
    assert set(mats_) == {"int8_nk", "int8_kn", "fp32"}
    nk = mats_["int8_nk"]
    if nk["packed"] and flags == 0:  # AVX-VNNI host: the same quantised arithmetic
        assert nk["mul_identical"] and nk["add_identical"]
    assert nk["mul_rel_l2"] <= 1e-3 and nk["add_rel_l2"] <= 1e-3
    assert mats_["int8_kn"]["mul_rel_l2"] <= 1e-2
    assert mats_["fp32"]["mul_rel_l2"] <= 1e-3 and mats_["fp32"]["add_rel_l2"] <= 1e-3
