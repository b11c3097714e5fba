"""Timed CPU baseline for bench.py: the reference's own CPU implementation of
one LM decoder layer's int8 linear set.  TEST/BENCH INFRASTRUCTURE ONLY.

Runs, through oracle/_ref/libovref.so (the reference's gemm.cpp/ops_cpu.cpp
built from source with OpenMP), the int8 branch of LM::run_layer
(cpp/src/model/lm.cpp:217-322) minus attention:

    rmsnorm_quantize_f32 -> linear_s8_nk_packed_q_sliced (q|k|v)
    -> linear_s8_nk_packed_add (o, quantises the attention input inside)
    -> rmsnorm_quantize_f32 -> linear_s8_nk_packed_q_sliced (gate|up)
    -> silu_mul_quantize_f32 -> linear_s8_nk_packed_q_add (down)

On a host without AVX-VNNI the reference itself runs its AVX2 fallback
(rmsnorm_into_f32 + linear_s8_nk with unquantised activations, mat.cpp:11-27,
lm.cpp:244-249); that path is timed instead and labelled "AVX2 (no VNNI)".
If the reference library is missing, the oracle's scalar C restatement is
timed and the result is labelled kind "port".
"""
from __future__ import annotations

import os
import time

import numpy as np

import oracle as O

HIDDEN, QD, KVD, INTER = 1024, 2048, 1024, 3072
SHAPES = [("q", QD, HIDDEN), ("k", KVD, HIDDEN), ("v", KVD, HIDDEN), ("o", HIDDEN, QD),
          ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]
OPS_PER_TOKEN = 2 * sum(n * k for _, n, k in SHAPES)


def _layer_weights(rng):
    w = {}
    for name, n, k in SHAPES:
        w[name] = (rng.integers(-127, 128, size=(n, k), dtype=np.int8),
                   (np.abs(rng.standard_normal(n)) * 0.02 / 127).astype(np.float32))
    return w


class RefLayer:
    """One layer's weights prepared the way the reference's loader does."""

    def __init__(self, w, mode: str):
        self.mode = mode
        self.ones = np.ones(HIDDEN, np.float32)
        if mode == "vnni":
            p = {k: O.RefPacked(*w[k]) for k, _, _ in SHAPES}
            self.qkv = O.ref_concat([p["q"], p["k"], p["v"]])
            self.gu = O.ref_concat([p["gate"], p["up"]])
            self.o, self.down = p["o"], p["down"]
        else:
            self.w = w

    def run(self, x: np.ndarray) -> np.ndarray:
        M = x.shape[0]
        if self.mode == "vnni":
            aq, asc = O.ref_rmsnorm_quantize(x, self.ones, 1e-6)
            q, k, v = O.ref_linear_q_sliced(self.qkv, [QD, KVD, KVD], aq, asc)
            x = self.o.linear(q, x)                       # o_proj.mul_add(attn, x)
            aq, asc = O.ref_rmsnorm_quantize(x, self.ones, 1e-6)
            gate, up = O.ref_linear_q_sliced(self.gu, [INTER, INTER], aq, asc)
            aq, asc = O.ref_silu_mul_quantize(gate, up)
            return self.down.linear_q(aq, asc, x)         # down.mul_q_add
        if self.mode == "avx2":
            return self._run_avx2(x, M)
        return self._run_port(x)

    def _mm(self, name, A):
        W, s = self.w[name]
        out = np.zeros((A.shape[0], W.shape[0]), np.float32)
        A = np.ascontiguousarray(A, np.float32)
        rc = O.ref_lib().ref_linear_s8_nk(A.shape[0], W.shape[0], W.shape[1], A.ctypes.data,
                                          W.ctypes.data, s.ctypes.data, out.ctypes.data)
        if rc:
            raise RuntimeError("linear_s8_nk failed")
        return out

    def _run_avx2(self, x, M):
        xn = O.ref_rmsnorm_into(x, self.ones, 1e-6)
        q = self._mm("q", xn)
        self._mm("k", xn)
        self._mm("v", xn)
        x = x + self._mm("o", q)
        xn = O.ref_rmsnorm_into(x, self.ones, 1e-6)
        act = O.ref_silu_mul(self._mm("gate", xn), self._mm("up", xn))
        return x + self._mm("down", act)

    def _run_port(self, x):
        aq, asc = O.rmsnorm_quantize(x, self.ones, 1e-6)
        q = O.linear_q(aq, asc, *self.w["q"], HIDDEN)
        O.linear_q(aq, asc, *self.w["k"], HIDDEN)
        O.linear_q(aq, asc, *self.w["v"], HIDDEN)
        aq2, asc2 = O.quantize(q)
        x = O.linear_q(aq2, asc2, *self.w["o"], QD, x)
        aq, asc = O.rmsnorm_quantize(x, self.ones, 1e-6)
        gate = O.linear_q(aq, asc, *self.w["gate"], HIDDEN)
        up = O.linear_q(aq, asc, *self.w["up"], HIDDEN)
        aq, asc = O.silu_mul_quantize(gate, up)
        return O.linear_q(aq, asc, *self.w["down"], INTER, x)


def host_cpu() -> dict:
    """The host CPU as the reference's baseline reports it: model name (from
    /proc/cpuinfo, as lscpu shows it) and whether it has AVX-VNNI, which
    decides the reference's int8 path (gemm.cpp:556-572)."""
    model, flags = None, set()
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k = k.strip()
                if k == "model name" and model is None:
                    model = v.strip()
                elif k == "flags" and not flags:
                    flags = set(v.split())
    except OSError:
        pass
    return {"cpu_model": model, "avx_vnni": "avx_vnni" in flags,
            "avx512_vnni": "avx512_vnni" in flags, "logical_cpus": os.cpu_count()}


def pick_mode() -> tuple[str, str]:
    """(mode, kind): what the reference itself would run on this host."""
    if O.ref_available():
        return ("vnni", "reference") if O.ref_vnni() else ("avx2", "reference")
    return ("port", "port")


def run(M: int = 400, layers: int = 4, max_steps: int = 1 << 30, budget_s: float = 10.0,
        warmup: int = 1, seed: int = 0) -> dict:
    """Time up to `max_steps` layer steps (rotating over `layers` weight sets)
    within `budget_s` seconds after `warmup` untimed steps.  Returns the
    throughput in int8 TOPS and a description of the sample."""
    mode, kind = pick_mode()
    if mode == "port":
        layers = 1
    rng = np.random.default_rng(seed)
    lw = [RefLayer(_layer_weights(rng), mode) for _ in range(layers)]
    x = rng.standard_normal((M, HIDDEN)).astype(np.float32)
    for i in range(warmup):
        lw[i % layers].run(x)
    steps = 0
    t0 = time.perf_counter()
    while steps < max_steps:
        lw[steps % layers].run(x)
        steps += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    ops = steps * M * OPS_PER_TOKEN
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    cores = 1 if mode == "port" else threads
    label = {"vnni": "reference AVX-VNNI int8 path (linear_s8_nk_packed*, OpenMP)",
             "avx2": "reference AVX2 (no VNNI) fallback, unquantised activations",
             "port": "oracle scalar C restatement, 1 thread"}[mode]
    return {
        "value": ops / dt / 1e12,
        "unit": "TOPS",
        "cores": cores,
        "kind": kind,
        "sample": f"{steps} layer steps (M={M}, {layers} weight sets) in {dt:.2f} s; {label}",
        "steps": steps,
        "seconds": dt,
        "host": host_cpu(),
    }
