"""GPU parity of one decoder layer's linear set against
the reference's own sequence (LM::run_layer, lm.cpp:217-322), composed from
the oracle: bit-exact residual stream after the layer, at full size
(M = 2 x 200 tokens, hidden 1024)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from ovnative_b200 import layer as LY

pytestmark = pytest.mark.gpu


def oracle_layer(x, w, attn=None):
    """The same eight steps on the CPU with the oracle (port)."""
    x = x.copy()
    aq, asc = O.rmsnorm_quantize(x, w["input_ln"], LY.RMS_EPS)
    q = O.linear_q(aq, asc, *w["q"], LY.HIDDEN)
    a = q if attn is None else attn
    aq, asc = O.quantize(a)
    x = O.linear_q(aq, asc, *w["o"], LY.QD, x)
    aq, asc = O.rmsnorm_quantize(x, w["post_ln"], LY.RMS_EPS)
    gate = O.linear_q(aq, asc, *w["gate"], LY.HIDDEN)
    up = O.linear_q(aq, asc, *w["up"], LY.HIDDEN)
    aq, asc = O.silu_mul_quantize(gate, up)
    x = O.linear_q(aq, asc, *w["down"], LY.INTER, x)
    return x, q


def test_layer_cfg1_bit_exact(cuda):
    rng = np.random.default_rng(2024)
    M = 400
    w = LY.random_layer_host(rng)
    x = rng.standard_normal((M, LY.HIDDEN)).astype(np.float32)
    lw = LY.LayerWeights.from_host(w, cuda)
    buf = LY.LayerBuffers(M, cuda)
    xd = torch.from_numpy(x).to(cuda)
    LY.run(xd, lw, buf)
    torch.cuda.synchronize()
    want, q = oracle_layer(x, w)
    got_q = buf.q.cpu().numpy()
    assert got_q.tobytes() == q.tobytes()
    got = xd.cpu().numpy()
    bad = int((got.view(np.uint32) != want.view(np.uint32)).sum())
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert bad == 0, f"{bad} outputs differ, rel-L2 {rel:.2e}"


def test_layer_graph_replay_matches_eager(cuda):
    """The layer captured in a CUDA graph gives the same bytes as eager runs."""
    rng = np.random.default_rng(7)
    M = 200
    lw = LY.LayerWeights.from_host(LY.random_layer_host(rng), cuda)
    buf = LY.LayerBuffers(M, cuda)
    x0 = torch.from_numpy(rng.standard_normal((M, LY.HIDDEN)).astype(np.float32)).to(cuda)
    xe = x0.clone()
    LY.run(xe, lw, buf)
    LY.run(xe, lw, buf)
    xg = x0.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        LY.run(xg.clone(), lw, buf)  # warm-up outside capture (sets kernel attributes)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        LY.run(xg, lw, buf)
    xg.copy_(x0)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert xg.cpu().numpy().tobytes() == xe.cpu().numpy().tobytes()


def test_layer_cfg1_f16_path_within_tolerance(cuda):
    """The same layer on the fp16 mainloop (fp16 weight copies, quantisers in
    the OVB_AQ_F16 form, ovb_linear_h): each GEMM output within the contract's
    rel-L2 1e-3 of the reference, the residual stream too; the layer's own
    contribution (x_out - x_in) within 1e-2 (two GEMMs deep, requantised)."""
    rng = np.random.default_rng(2024)
    M = 400
    w = LY.random_layer_host(rng)
    x = rng.standard_normal((M, LY.HIDDEN)).astype(np.float32)
    lw = LY.LayerWeights.from_host(w, cuda, f16=True)
    buf = LY.LayerBuffers(M, cuda, f16=True)
    xd = torch.from_numpy(x).to(cuda)
    LY.run(xd, lw, buf)
    torch.cuda.synchronize()
    want, q = oracle_layer(x, w)

    def rel(a, b):
        return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))

    got_q = buf.q.cpu().numpy()
    assert rel(got_q, q) <= 1e-3
    got = xd.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel(got, want) <= 1e-3
    assert rel(got - x, want - x) <= 1e-2


@pytest.mark.parametrize("f16", [True, False])
def test_step_pipeline_matches_direct_steps(cuda, f16):
    """StepPipeline (the serving loop bench.py's e2e line uses: copies of the
    next input and the previous result inside each step's graph, three device
    buffers in rotation) returns exactly what running each step directly
    returns, for distinct inputs and layers per step."""
    rng = np.random.default_rng(31 + f16)
    M, n_layers, steps = 200, 2, 7
    layers = [LY.LayerWeights.from_host(LY.random_layer_host(rng), cuda, f16=f16)
              for _ in range(n_layers)]
    buf = LY.LayerBuffers(M, cuda, f16=f16)
    xs = [rng.standard_normal((M, LY.HIDDEN)).astype(np.float32) for _ in range(steps)]
    want = []
    for i, xi in enumerate(xs):
        x = torch.from_numpy(xi).to(cuda)
        LY.run(x, layers[i % n_layers], buf)
        want.append(x.cpu().numpy())
    stream = torch.cuda.Stream(device=cuda)
    pipe = LY.StepPipeline(layers, buf, M, cuda, stream)
    got = []
    pipe.host_in[0].copy_(torch.from_numpy(xs[0]))
    pipe.start()
    for i in range(steps):
        # step i+1's input must be in place before step i starts
        if i + 1 < steps:
            stream.synchronize()
            pipe.host_in[(i + 1) % 3].copy_(torch.from_numpy(xs[i + 1]))
        pipe.step(i, i % n_layers)
        if i >= 1:  # step i-1's result is out once step i has completed
            stream.synchronize()
            got.append(pipe.host_out[(i - 1) % 3].numpy().copy())
    pipe.finish(steps - 1)
    stream.synchronize()
    got.append(pipe.host_out[(steps - 1) % 3].numpy().copy())
    for i in range(steps):
        assert np.array_equal(got[i], want[i]), f"step {i}"
    pipe.release()
