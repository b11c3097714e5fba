"""The full 28-layer LM forward at BASELINE configs 2 and 3 against the
reference's own LM on its CPU path (cpp/src/model/lm.cpp, AVX-VNNI int8,
oracle/_ref), on the same random checkpoint of the real shape (151,676-token
vocabulary) and inputs: a CFG pair as the B = 2 batch of the reference's
CUDA path (LM::forward, tts.cpp:172-204, 260-266).

Judged by the reference's own int8 LM gate (cpp/tests/test_lm.cpp:198-230:
cosine, mean |delta| < 0.15, argmax agreement >= 80 % over every (row,
codebook) position) and, for the cosine, against the reference's OWN GPU
path: its CUDA runner (cpp/src/backend/cuda/cuda_lm.cu:790-1221, built from
its source into oracle/_ref: fp16 cuBLAS GEMMs on dequantised weights, TF32
attention) run on the same integer weights in its [K, N] encoding.  The
device forward must sit as close to the CPU path as the reference's own CUDA
forward does, within 15 % of that distance.  (On random weights the logits are small, |x| ~ 0.24,
so the cosine is far more sensitive than on the trained checkpoint the gate
was written for; the fp16 attention operands -- the precision of the
reference's TF32 attention -- account for most of the difference, and the
int8 and fp16 GEMM mainloops give the same figures.)"""
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
    nk = os.path.join(d, "lm28_nk.ovw")
    kn = os.path.join(d, "lm28_kn.ovw")
    ovw1.random_lm(nk, n_layers=LAYERS, vocab=VOCAB, seed=21)
    ovw1.random_lm(kn, n_layers=LAYERS, vocab=VOCAB, seed=21, layout="kn")
    ref = O.RefLM(nk, LAYERS)
    yield nk, kn, ref
    ref.close()
    shutil.rmtree(d, ignore_errors=True)


def b2_inputs(rng, S, n_text=40):
    """BASELINE configs 2/3 as LM::forward's B = 2 CFG batch: 40 text ids
    uniform in [0, 151000) then audio ids in the conditional row; the
    unconditional row holds the target slice (S - 40 audio rows) followed by
    mask-id text rows that attend only to themselves (tts.cpp:186-198)."""
    T = S - n_text
    ids = np.full((2, C, S), 1024, np.int64)
    ids[0] = rng.integers(0, V - 1, size=(C, S))
    ids[0, :, :n_text] = rng.integers(0, 151000, size=n_text)
    ids[1, :, :T] = ids[0, :, S - T:]
    amask = np.zeros((2, S), np.uint8)
    amask[0, n_text:] = 1
    amask[1, :T] = 1
    attn = np.zeros((2, S, S), np.uint8)
    attn[0] = 1
    attn[1, :T, :T] = 1
    attn[1, np.arange(T, S), np.arange(T, S)] = 1
    pos = np.tile(np.arange(S, dtype=np.int64), (2, 1))
    return ids, amask, attn, pos


@pytest.fixture(scope="module")
def ref_gpu(full_model):
    if not O.ref_cuda_available():
        pytest.skip("oracle/_ref/libovref_cuda.so not built")
    r = O.RefCudaLM(full_model[1], LAYERS)
    yield r
    r.close()


@pytest.mark.parametrize("S", [300, 700])
def test_28_layers_against_reference_cpu_and_gpu(cuda, full_model, ref_gpu, S):
    nk, _, ref = full_model
    rng = np.random.default_rng(S)
    inp = b2_inputs(rng, S)
    want = ref.forward(*inp)
    rg = metrics(ref_gpu.forward(*inp), want)
    print(f"S={S} reference CUDA runner vs CPU: cos={rg[0]:.8f} mean|d|={rg[1]:.3e} "
          f"agree={rg[2]:.4f} (|logit| mean {np.abs(want).mean():.3f})")
    for f16 in (False, True):
        m = LM.LM(nk, f16=f16)
        got = m.forward(*inp)
        m.close()
        cos, mean, agree = metrics(got, want)
        print(f"S={S} f16={f16} vs CPU: cos={cos:.8f} mean|d|={mean:.3e} agree={agree:.4f}")
        assert np.isfinite(got).all()
        assert mean < 0.15 and agree >= 0.80          # the reference's int8 gate
        # as close to the CPU path as the reference's own GPU forward, within
        # 15 % of its distance (measured at S = 300: 1.03x on the int8
        # mainloop, 1.10x on the fp16 one, whose fp16 activations add their
        # rounding to the fp16 attention operands)
        assert 1 - cos <= 1.15 * (1 - rg[0])
    assert ovb.device_status() == 0
