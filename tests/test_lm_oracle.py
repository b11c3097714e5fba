"""The reference's own LM (cpp/src/model/lm.cpp, built into oracle/_ref) on a
random checkpoint written by ovnative_b200.ovw1.random_lm: the reference
loads the file (so the writer produces what its LM expects) and its two
forwards agree with each other where the reference says they must (the
ragged CFG forward equals the batched one on the conditional rows,
lm.h:71-76)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from ovnative_b200 import ovw1

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")

C, V = 8, 1025


def cfg_inputs(rng, cs, us, vocab, n_text=12, pad=2):
    rows = cs + us
    ids = rng.integers(0, V, size=(C, rows)).astype(np.int64)
    amask = np.ones(rows, np.uint8)
    amask[:n_text] = 0
    ids[0, :n_text] = rng.integers(0, vocab, size=n_text)
    cond = np.ones((cs, cs), np.uint8)
    cond[:, :pad] = 0          # padded keys
    unc = np.ones((us, us), np.uint8)
    pos = np.concatenate([np.arange(cs), np.arange(us)]).astype(np.int64)
    return ids, amask, cond, unc, pos


def test_reference_lm_runs_on_written_checkpoint(repo_tmp):
    p = str(repo_tmp / "lm2.ovw")
    ovw1.random_lm(p, n_layers=2, vocab=512, seed=1)
    ref = O.RefLM(p, 2)
    rng = np.random.default_rng(2)
    ids, amask, cond, unc, pos = cfg_inputs(rng, 40, 24, 512)
    logits = ref.forward_cfg(ids, amask, cond, unc, pos)
    assert logits.shape == (64, C * V) and np.isfinite(logits).all()
    assert logits.std() > 0.05
    # forward(B=1) over the conditional rows alone gives the same cond logits
    ids_b = ids[:, :40][None]
    lb = ref.forward(ids_b, amask[None, :40], cond[None], pos[None, :40])
    np.testing.assert_allclose(lb[0].transpose(1, 0, 2).reshape(40, C * V), logits[:40],
                               rtol=1e-4, atol=1e-4)
    ref.close()


def test_reference_lm_rejects_missing_layers(repo_tmp):
    p = str(repo_tmp / "lm1.ovw")
    ovw1.random_lm(p, n_layers=1, vocab=64, seed=3)
    with pytest.raises(RuntimeError, match="tensor not found"):
        O.RefLM(p, 2)


def _create(path):
    import ctypes as Cc

    from ovnative_b200 import _lib as L
    h = Cc.c_void_p()
    rc = L.lib().ovb_lm_create(path.encode(), 0, None, Cc.byref(h))
    return rc, L.lib().ovb_last_error().decode()


def test_lm_create_rejects_bad_checkpoints(repo_tmp):
    """ovb_lm_create's checks run before any device call (so on the CPU):
    a missing file, a file without layers, and fp16 audio heads (neither the
    int8 nor the fp32 encoding of a linear weight) are invalid arguments with
    a message."""
    from ovnative_b200 import _lib as L
    rc, msg = _create(str(repo_tmp / "absent.ovw"))
    assert rc == L.OVB_ERR_INVALID_ARG and "cannot open" in msg
    p = str(repo_tmp / "norm_only.ovw")
    ovw1.write(p, [("llm.norm.weight", np.ones(1024, np.float32), 0, None)])
    rc, msg = _create(p)
    assert rc == L.OVB_ERR_INVALID_ARG and "llm.layers.0" in msg
    # a one-layer checkpoint whose audio heads are fp16 [K, N]
    full = str(repo_tmp / "lm1.ovw")
    ovw1.random_lm(full, n_layers=1, vocab=64, seed=5)
    with ovw1.OVW1File(full) as f:
        ts = []
        for name in f.names():
            a = np.array(f.array(name))
            sc = f.scales(name)
            if name == "audio_heads.weight":
                ts.append((name, np.zeros((1024, 8200), np.float16), 1, None))
            else:
                ts.append((name, a, f.info(name).layout, None if sc is None else np.array(sc)))
    p = str(repo_tmp / "fp16_heads.ovw")
    ovw1.write(p, ts)
    rc, msg = _create(p)
    assert rc == L.OVB_ERR_INVALID_ARG and "audio_heads.weight" in msg
    assert "int8 or fp32" in msg


def test_reference_lm_runs_fp32_heads(repo_tmp):
    """The reference's default conversion keeps the audio heads fp32 [K, N]
    (tools/convert_weights.py:326-327); its LM loads such a file written by
    random_lm(heads_f32=True) and runs them through linear_f32."""
    p = str(repo_tmp / "lm1f.ovw")
    ovw1.random_lm(p, n_layers=1, vocab=256, seed=4, heads_f32=True)
    with ovw1.OVW1File(p) as f:
        t = f.info("audio_heads.weight")
        assert t.dtype == 0 and t.layout == 1 and t.dims[0] == 1024 and t.dims[1] == C * V
    ref = O.RefLM(p, 1)
    rng = np.random.default_rng(6)
    ids, amask, cond, unc, pos = cfg_inputs(rng, 20, 12, 256)
    logits = ref.forward_cfg(ids, amask, cond, unc, pos)
    assert logits.shape == (32, C * V) and np.isfinite(logits).all() and logits.std() > 0.01
    ref.close()


def test_lm_entry_points_reject_null_model():
    from ovnative_b200 import _lib as L
    lib = L.lib()
    assert lib.ovb_lm_forward_cfg(None, 4, 4, None, None, None, None, None, None, None) == \
        L.OVB_ERR_INVALID_ARG
    assert lib.ovb_lm_forward(None, 1, 4, None, None, None, None, None, None) == \
        L.OVB_ERR_INVALID_ARG
    assert lib.ovb_lm_reserve(None, 4, 16) == L.OVB_ERR_INVALID_ARG
    assert lib.ovb_lm_forward_segments_device(None, 1, None, None, None, None, None, None) == \
        L.OVB_ERR_INVALID_ARG
    assert lib.ovb_lm_destroy(None) == L.OVB_OK
    assert lib.ovb_lm_logits(None) is None


def test_kn_encoding_of_the_same_weights(repo_tmp):
    """random_lm(layout="kn") writes the same integer weights in the
    converter's default [K, N] encoding (layout 1, column scales), which the
    reference's LM reads too (Mat::mul -> linear_s8, mat.cpp:11-24)."""
    a, b = str(repo_tmp / "nk.ovw"), str(repo_tmp / "kn.ovw")
    ovw1.random_lm(a, n_layers=1, vocab=1100, seed=8)
    ovw1.random_lm(b, n_layers=1, vocab=1100, seed=8, layout="kn")
    name = "llm.layers.0.self_attn.q_proj.weight"
    with ovw1.OVW1File(a) as fa, ovw1.OVW1File(b) as fb:
        assert fa.info(name).layout == 0 and fb.info(name).layout == 1
        np.testing.assert_array_equal(fa.array(name), fb.array(name).T)
        np.testing.assert_array_equal(fa.scales(name), fb.scales(name))
    ref = O.RefLM(b, 1)
    rng = np.random.default_rng(9)
    ids, amask, cond, unc, pos = cfg_inputs(rng, 20, 12, 1100)
    out = ref.forward_cfg(ids, amask, cond, unc, pos)
    assert np.isfinite(out).all() and out.std() > 0.01
    ref.close()
