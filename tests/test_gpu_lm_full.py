"""The full 28-layer LM forward at BASELINE configs 2 and 3 against the
reference's own LM (cpp/src/model/lm.cpp, oracle/_ref) on the same random
checkpoint of the real shape (151,676-token vocabulary) and inputs, judged
by the reference's own int8 LM gate (cpp/tests/test_lm.cpp:228-230:
cosine > 0.99999, mean |delta| < 0.15, argmax agreement >= 80 % over every
(row, codebook) position).  The two small-model tests in test_gpu_lm.py hold
tighter bounds; these show that the per-layer differences (fp16 attention
operands everywhere, fp16 GEMM operands on the fp16 path) do not compound
over 28 layers."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
import ovnative_b200 as ovb
from ovnative_b200 import lm as LM
from ovnative_b200 import ovw1
from tests.test_gpu_lm import metrics

pytestmark = pytest.mark.gpu

LAYERS, VOCAB = 28, 151676
C, V = 8, 1025


@pytest.fixture(scope="module")
def full_model():
    import os
    import shutil

    from tests.conftest import ROOT
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    d = os.path.join(ROOT, ".test_tmp", "gpu_lm_full")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, "lm28.ovw")
    ovw1.random_lm(p, n_layers=LAYERS, vocab=VOCAB, seed=21)
    ref = O.RefLM(p, LAYERS)
    yield p, ref
    ref.close()
    shutil.rmtree(d, ignore_errors=True)


def config_inputs(rng, S, n_text=40):
    """BASELINE configs 2/3: a CFG pair of S + S rows, 40 text ids uniform in
    [0, 151000) at the start of the conditional half, audio ids elsewhere."""
    rows = 2 * S
    ids = rng.integers(0, V, size=(C, rows)).astype(np.int64)
    amask = np.ones(rows, np.uint8)
    amask[:n_text] = 0
    ids[0, :n_text] = rng.integers(0, 151000, size=n_text)
    cond = np.ones((S, S), np.uint8)
    unc = np.ones((S, S), np.uint8)
    pos = np.concatenate([np.arange(S), np.arange(S)]).astype(np.int64)
    return ids, amask, cond, unc, pos


@pytest.mark.parametrize("S,f16", [(300, False), (300, True), (700, False), (700, True)])
def test_28_layers_within_reference_int8_gate(cuda, full_model, S, f16):
    path, ref = full_model
    rng = np.random.default_rng(S)
    inp = config_inputs(rng, S)
    want = ref.forward_cfg(*inp)
    m = LM.LM(path, f16=f16)
    got = m.forward_cfg(*inp)
    m.close()
    cos, mean, agree = metrics(got, want)
    print(f"config S={S} f16={f16}: cos={cos:.8f} mean|d|={mean:.3e} agree={agree:.4f} "
          f"(|logit| mean {np.abs(want).mean():.3f})")
    assert np.isfinite(got).all()
    assert cos > 0.99999 and mean < 0.15 and agree >= 0.80
    assert ovb.device_status() == 0
