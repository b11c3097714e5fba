"""Batched TTS steps on the GPU (ovnative_b200.tts_batch.Stepper): several
utterances' CFG pairs packed into each forward, the guided sampler per pair,
one CUDA graph per batch -- against the reference.

For every utterance the predictions and scores are compared with the
reference's own LM::forward over the B = 2 CFG batch its CUDA path builds
(cpp/src/model/tts.cpp:172-204, 260-266; oracle/_ref) followed by the
guidance + argmax loop (tts.cpp:291-326, the oracle restatement): scores to
the sampler's tolerance plus the forward's, predictions equal wherever the
two best mixed log-probabilities are clearly apart.  The int8 mainloop's
results do not depend on how rows are packed, so the packed step also equals
a one-utterance-at-a-time step bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import ovnative_b200 as ovb
from ovnative_b200 import lm as LM
from ovnative_b200 import ovw1
from ovnative_b200 import tts_batch as TB
from tests.test_gpu_sampler import second_gap

pytestmark = pytest.mark.gpu

LAYERS, VOCAB = 2, 2048  # > the mask id 1024, which the uncond tail rows embed as a token
LENGTHS = {0: 50, 1: 75, 2: 41, 3: 120, 4: 64}


@pytest.fixture(scope="module")
def model_path():
    import os
    import shutil

    from tests.conftest import ROOT
    d = os.path.join(ROOT, ".test_tmp", "gpu_tts")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, "lm2.ovw")
    ovw1.random_lm(p, n_layers=LAYERS, vocab=VOCAB, seed=17)
    yield p
    shutil.rmtree(d, ignore_errors=True)


def _inputs_b2(batch, p):
    """The packed pair of utterance p as LM::forward's B = 2 arguments."""
    C = batch.lm.C
    S = p.S
    ids = batch.ids[:, p.row0:p.row0 + 2 * S].cpu().numpy().reshape(C, 2, S).transpose(1, 0, 2)
    amask = batch.amask[p.row0:p.row0 + 2 * S].cpu().numpy().reshape(2, S)
    r = [x for q in batch.pairs for x in (q.S, q.S)]
    k = batch.pairs.index(p)
    off = sum(x * x for x in r[:2 * k])
    m = batch.masks.cpu().numpy()
    attn = np.stack([m[off:off + S * S].reshape(S, S), m[off + S * S:off + 2 * S * S].reshape(S, S)])
    pos = batch.pos[p.row0:p.row0 + 2 * S].cpu().numpy().reshape(2, S)
    return np.ascontiguousarray(ids), amask, attn, pos


@pytest.mark.parametrize("f16", [False, True])
def test_batched_steps_match_reference(cuda, model_path, f16):
    m = LM.LM(model_path, f16=f16)
    st = torch.cuda.Stream()
    # max_rows 300 -> several batches of several pairs
    sp = TB.Stepper(m, LENGTHS, list(LENGTHS), cuda, st, max_rows=300, seed=3)
    assert len(sp.batches) >= 2 and any(len(b.pairs) >= 2 for b in sp.batches)
    sp.warm_and_capture()
    sp.step()
    torch.cuda.synchronize()
    got = sp.results()
    ref = O.RefLM(model_path, LAYERS)
    C, V = m.C, m.V
    gs, ws, agree, n_clear, n_rows = [], [], 0, 0, 0
    for b in sp.batches:
        for p in b.pairs:
            ids, amask, attn, pos = _inputs_b2(b, p)
            lg = ref.forward(ids, amask, attn, pos)          # [2, C, S, V]
            cond = lg[0].transpose(1, 0, 2).reshape(p.S, C * V)
            unc = lg[1].transpose(1, 0, 2).reshape(p.S, C * V)
            want_p, want_s = O.guided_sample(cond, unc, p.T, C, TB.GUIDANCE, TB.LAYER_PENALTY,
                                             TB.MASK_ID)
            got_p, got_s = got[p.uid]
            assert got_p.shape == (C, p.T) and np.isfinite(got_s).all()
            gs.append(got_s.ravel())
            ws.append(want_s.ravel())
            clear = second_gap(cond, unc, C, V, p.T, TB.GUIDANCE, TB.MASK_ID) > 0.05
            agree += int((got_p[clear] == want_p[clear]).sum())
            n_clear += int(clear.sum())
            n_rows += clear.size
    ref.close()
    g, w = np.concatenate(gs).astype(np.float64), np.concatenate(ws).astype(np.float64)
    err = np.abs(g - w)
    print(f"f16={f16} scores mean|d|={err.mean():.2e} max|d|={err.max():.2e} "
          f"pred agree (clear rows) {agree / n_clear:.4f} of {n_clear}/{n_rows}")
    # the scores are log-probabilities of the guided mix: the forward's error
    # (fp16 attention operands; fp16 GEMM operands on the fp16 path) passes
    # through three log-softmaxes and the guidance factor
    assert err.mean() <= (0.02 if f16 else 0.01) * np.abs(w).mean()
    assert (err <= 0.1 + 0.02 * np.abs(w)).all()
    assert n_clear > 0.5 * n_rows
    assert agree / n_clear >= (0.98 if f16 else 0.995)
    # the end-to-end step (ids in from pinned memory, predictions out) gives
    # the same predictions
    sp.step_e2e()
    for b in sp.batches:
        for p in b.pairs:
            n = C * p.T
            np.testing.assert_array_equal(b.h_pred.numpy()[p.out0:p.out0 + n].reshape(C, p.T),
                                          got[p.uid][0])
    assert ovb.device_status() == 0
    sp.release()
    m.close()


def test_packed_step_equals_one_utterance_at_a_time(cuda, model_path):
    """Bit-identical on the int8 mainloop: packing changes nothing per row."""
    m = LM.LM(model_path, f16=False)
    st = torch.cuda.Stream()
    packed = TB.Stepper(m, LENGTHS, list(LENGTHS), cuda, st, max_rows=1 << 14, seed=5)
    assert len(packed.batches) == 1
    packed.warm_and_capture()
    packed.step()
    torch.cuda.synchronize()
    a = packed.results()
    packed.release()
    for u in LENGTHS:
        one = TB.Stepper(m, LENGTHS, [u], cuda, st, max_rows=1 << 14, seed=5)
        # the same inputs as in the packed run: copy them over
        pb = next(b for b in packed.batches if any(p.uid == u for p in b.pairs))
        pp = next(p for p in pb.pairs if p.uid == u)
        ob = one.batches[0]
        ob.ids.copy_(pb.ids[:, pp.row0:pp.row0 + 2 * pp.S])
        with torch.cuda.stream(st):
            ob.run()
        torch.cuda.synchronize()
        b_p, b_s = one.results()[u]
        np.testing.assert_array_equal(b_p, a[u][0])
        np.testing.assert_array_equal(b_s, a[u][1])
    assert ovb.device_status() == 0
    m.close()


@pytest.mark.parametrize("f16", [False, True])
def test_two_lanes_equal_one(cuda, model_path, f16):
    """Batches dealt to two LM instances on two streams give the same
    predictions and scores as one lane, bit for bit (the forwards are
    independent; only their timing overlaps)."""
    st = torch.cuda.Stream()
    out = []
    for lanes in (1, 2):
        ms = [LM.LM(model_path, f16=f16) for _ in range(lanes)]
        sp = TB.Stepper(ms[0], LENGTHS, list(LENGTHS), cuda, st, max_rows=256, seed=7,
                        extra_lms=ms[1:])
        assert len(sp.batches) >= 3
        sp.warm_and_capture()
        for _ in range(2):
            sp.step()
        sp.step_e2e()
        torch.cuda.synchronize()
        out.append(sp.results())
        sp.release()
        for m in ms:
            m.close()
    for u in LENGTHS:
        np.testing.assert_array_equal(out[0][u][0], out[1][u][0])
        np.testing.assert_array_equal(out[0][u][1], out[1][u][1])
    assert ovb.device_status() == 0
