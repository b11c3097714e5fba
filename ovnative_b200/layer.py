"""The linear sequence of one OVNative LM decoder layer on the B200 path.

Mirrors the int8 branch of LM::run_layer (cpp/src/model/lm.cpp:217-322):

    1. rmsnorm_quantize_f32(x, input_ln)              lm.cpp:232
    2. qkv sliced GEMM -> q [M,2048], k, v [M,1024]     lm.cpp:233-237
    3. (q/k norm, RoPE, attention -> attn [M,2048])    lm.cpp:252-277  -- out of scope
    4. o_proj.mul_add(attn, x): quantise + GEMM, += x   lm.cpp:281
    5. rmsnorm_quantize_f32(x, post_ln)               lm.cpp:292
    6. gate|up sliced GEMM -> gate, up [M,3072]         lm.cpp:293-297
    7. silu_mul_quantize_f32(gate, up)                lm.cpp:310
    8. down.mul_q_add -> x += ...                       lm.cpp:311

Attention is not part of this path.  ``run`` takes the attention output as an
argument; when it is omitted the q projection itself is fed to o_proj (an
identity stand-in that keeps the data flow of a real layer without adding
work).  All buffers are allocated once, so ``run`` can be captured in a CUDA
graph.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import gemm as G

HIDDEN = 1024
N_HEADS, N_KV, HEAD_DIM = 16, 8, 128
QD = N_HEADS * HEAD_DIM   # 2048
KVD = N_KV * HEAD_DIM     # 1024
INTER = 3072
RMS_EPS = 1e-6

# (name, N, K) of the seven projections of one layer
SHAPES = [("q", QD, HIDDEN), ("k", KVD, HIDDEN), ("v", KVD, HIDDEN), ("o", HIDDEN, QD),
          ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]


def ops_per_token() -> int:
    """2 * sum(N*K) over the seven projections: 31.46 M int8 ops per token."""
    return 2 * sum(n * k for _, n, k in SHAPES)


def random_layer_host(rng: np.random.Generator):
    """Random int8 weights ([N, K], uniform in [-127, 127]) and per-channel
    scales |N(0, 0.02)|/127 for the seven projections, RMSNorm gains 1."""
    w = {}
    for name, n, k in SHAPES:
        W = rng.integers(-127, 128, size=(n, k), dtype=np.int8)
        s = (np.abs(rng.standard_normal(n)) * 0.02 / 127.0).astype(np.float32)
        w[name] = (W, s)
    w["input_ln"] = np.ones(HIDDEN, np.float32)
    w["post_ln"] = np.ones(HIDDEN, np.float32)
    return w


@dataclass
class LayerWeights:
    qkv: G.Weight
    o: G.Weight
    gate_up: G.Weight
    down: G.Weight
    input_ln: torch.Tensor
    post_ln: torch.Tensor

    @classmethod
    def from_host(cls, w: dict, device, f16: bool = False, fused: bool = True) -> "LayerWeights":
        """``f16`` selects the fp16 tensor-core mainloop (OVB_WEIGHT_F16) for
        all four GEMMs; otherwise they reproduce the reference bit for bit.
        ``fused`` builds gate|up for the fused SiLU*up GEMM (run); otherwise a
        plain concatenation (run_unfused)."""
        parts = {name: G.Weight.from_nk(*w[name], f16=f16) for name, _, _ in SHAPES}
        qkv = G.Weight.concat([parts["q"], parts["k"], parts["v"]])
        if fused:
            gu = G.Weight.gate_up(parts["gate"], parts["up"])
        else:
            gu = G.Weight.concat([parts["gate"], parts["up"]])
        for name in ("q", "k", "v", "gate", "up"):
            parts[name].close()
        return cls(qkv=qkv, o=parts["o"], gate_up=gu, down=parts["down"],
                   input_ln=torch.from_numpy(w["input_ln"]).to(device),
                   post_ln=torch.from_numpy(w["post_ln"]).to(device))

    def close(self):
        for m in (self.qkv, self.o, self.gate_up, self.down):
            m.close()


class LayerBuffers:
    """Activation buffers for M rows (allocated once).  ``f16`` holds the
    quantisers' outputs in the dequantised fp16 form (OVB_AQ_F16) that the
    fp16 mainloop (linear_h) reads."""

    def __init__(self, M: int, device, f16: bool = False):
        f32 = dict(dtype=torch.float32, device=device)
        self.M = M
        self.f16 = f16
        self.q = torch.empty((M, QD), **f32)
        self.k = torch.empty((M, KVD), **f32)
        self.v = torch.empty((M, KVD), **f32)
        self.gate = torch.empty((M, INTER), **f32)
        self.up = torch.empty((M, INTER), **f32)
        alloc = G.empty_quant_f16 if f16 else G.empty_quant
        self.qh = alloc(M, HIDDEN, device)   # norm+quant of x
        self.qo = alloc(M, QD, device)       # quant of attn
        self.qi = alloc(M, INTER, device)    # silu*up quant


def run(x: torch.Tensor, lw: LayerWeights, buf: LayerBuffers, attn: torch.Tensor | None = None):
    """One layer's linear set on x [M, 1024] (updated in place, residual stream),
    LM::run_layer's order (lm.cpp:217-322).  With fp16 buffers the quantisers
    write fp16(q * asc) and the GEMMs run the plain fp16 mainloop; otherwise
    int8 q + scales and the exact int8 mainloop."""
    a = buf.q if attn is None else attn
    if buf.f16:
        G.rmsnorm_quantize_f32(x, lw.input_ln, RMS_EPS, out=buf.qh, f16=True)
        G.linear_h_sliced(buf.qh[0], lw.qkv, [buf.q, buf.k, buf.v])
        G.s8_nk_quantize(a, out=buf.qo, f16=True)
        G.linear_h(buf.qo[0], lw.o, x, accumulate=True)
        G.rmsnorm_quantize_f32(x, lw.post_ln, RMS_EPS, out=buf.qh, f16=True)
        G.linear_h_silu(buf.qh[0], lw.gate_up, out=buf.qi, f16=True)  # gate|up + SiLU*up quant
        G.linear_h(buf.qi[0], lw.down, x, accumulate=True)
        return x
    G.rmsnorm_quantize_f32(x, lw.input_ln, RMS_EPS, out=buf.qh)
    G.linear_s8_nk_packed_q_sliced(*buf.qh, lw.qkv, [buf.q, buf.k, buf.v])
    G.s8_nk_quantize(a, out=buf.qo)
    G.linear_s8_nk_packed_q_add(*buf.qo, lw.o, x)
    G.rmsnorm_quantize_f32(x, lw.post_ln, RMS_EPS, out=buf.qh)
    G.linear_q_silu(*buf.qh, lw.gate_up, out=buf.qi)  # gate|up + SiLU*up quant, bit-exact
    G.linear_s8_nk_packed_q_add(*buf.qi, lw.down, x)
    return x


def run_unfused(x: torch.Tensor, lw_cat, buf: LayerBuffers, attn: torch.Tensor | None = None):
    """The same layer with the reference's separate gate|up GEMM and
    silu_mul_quantize call (lw_cat.gate_up a plain concatenation): used by the
    tests to check the fused epilogue against the unfused sequence."""
    a = buf.q if attn is None else attn
    kw = dict(f16=True) if buf.f16 else {}
    G.rmsnorm_quantize_f32(x, lw_cat.input_ln, RMS_EPS, out=buf.qh, **kw)
    if buf.f16:
        G.linear_h_sliced(buf.qh[0], lw_cat.qkv, [buf.q, buf.k, buf.v])
    else:
        G.linear_s8_nk_packed_q_sliced(*buf.qh, lw_cat.qkv, [buf.q, buf.k, buf.v])
    G.s8_nk_quantize(a, out=buf.qo, **kw)
    if buf.f16:
        G.linear_h(buf.qo[0], lw_cat.o, x, accumulate=True)
    else:
        G.linear_s8_nk_packed_q_add(*buf.qo, lw_cat.o, x)
    G.rmsnorm_quantize_f32(x, lw_cat.post_ln, RMS_EPS, out=buf.qh, **kw)
    if buf.f16:
        G.linear_h_sliced(buf.qh[0], lw_cat.gate_up, [buf.gate, buf.up])
    else:
        G.linear_s8_nk_packed_q_sliced(*buf.qh, lw_cat.gate_up, [buf.gate, buf.up])
    G.silu_mul_quantize_f32(buf.gate, buf.up, out=buf.qi, **kw)
    if buf.f16:
        G.linear_h(buf.qi[0], lw_cat.down, x, accumulate=True)
    else:
        G.linear_s8_nk_packed_q_add(*buf.qi, lw_cat.down, x)
    return x


KERNELS_PER_LAYER = 7  # 3 quantisers + 4 GEMMs (gate|up fused with SiLU*up quantise)


class StepPipeline:
    """Drives layer steps over inputs in pinned host memory with the copies
    overlapping the compute, as a serving loop does.

    Three device buffers rotate: step i runs in place on buffer i % 3, and the
    CUDA graph of step i (one per (layer, rotation)) also copies step i+1's
    input from ``host_in[(i+1) % 3]`` into its buffer and step i-1's result
    from its buffer into ``host_out[(i-1) % 3]``, on two copy streams.  So
    every step is one graph launch; step i's input must be in
    ``host_in[i % 3]`` when step i-1 starts (step 0's when ``start`` is
    called), and its result is in ``host_out[i % 3]`` once step i+1 (or
    ``finish``) has completed on the stream.
    """

    def __init__(self, layers: list[LayerWeights], buf: LayerBuffers, M: int, device,
                 stream: torch.cuda.Stream):
        self.stream = stream
        self.host_in = [torch.empty((M, HIDDEN), dtype=torch.float32).pin_memory()
                        for _ in range(3)]
        self.host_out = [torch.empty((M, HIDDEN), dtype=torch.float32).pin_memory()
                         for _ in range(3)]
        self.dev = [torch.empty((M, HIDDEN), dtype=torch.float32, device=device)
                    for _ in range(3)]
        s_in = torch.cuda.Stream(device=device)
        s_out = torch.cuda.Stream(device=device)
        self.graphs = {}
        with torch.cuda.stream(stream):
            for lid, lw in enumerate(layers):
                for r in range(3):
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=stream):
                        s_in.wait_stream(stream)
                        s_out.wait_stream(stream)
                        with torch.cuda.stream(s_in):  # step i+1's input
                            self.dev[(r + 1) % 3].copy_(self.host_in[(r + 1) % 3],
                                                        non_blocking=True)
                        with torch.cuda.stream(s_out):  # step i-1's result
                            self.host_out[(r + 2) % 3].copy_(self.dev[(r + 2) % 3],
                                                             non_blocking=True)
                        run(self.dev[r], lw, buf)  # step i, in place
                        stream.wait_stream(s_in)
                        stream.wait_stream(s_out)
                    self.graphs[(lid, r)] = g

    def start(self):
        """Copy step 0's input (host_in[0]) to the device."""
        with torch.cuda.stream(self.stream):
            self.dev[0].copy_(self.host_in[0], non_blocking=True)

    def step(self, i: int, layer: int):
        """Enqueue step i on the layer with index `layer`."""
        with torch.cuda.stream(self.stream):
            self.graphs[(layer, i % 3)].replay()

    def finish(self, last: int):
        """Copy the last step's result to host_out[last % 3]."""
        with torch.cuda.stream(self.stream):
            self.host_out[last % 3].copy_(self.dev[last % 3], non_blocking=True)

    def release(self):
        for g in self.graphs.values():
            g.reset()
        self.graphs = {}
