"""Generate the golden vectors in this directory from the reference itself.

    python tests/golden/make_golden.py

Runs the reference's own CPU int8 path -- cpp/src/backend/cpu/gemm.cpp and
ops_cpu.cpp compiled from source into oracle/_ref/libovref.so by
oracle/Makefile -- on seeded inputs and stores inputs and outputs as .npz.
It needs an AVX-VNNI host (the reference's quantised path throws without it,
gemm.cpp:712).  The shapes follow the reference's own unit tests
(cpp/tests/test_gemm.cpp:462-508), which hit every M%4, N%8 and K%32 tail,
plus the BASELINE config-0 GEMM (M=256, K=1024, N=3072), stored as SHA-256
digests because its tensors are megabytes.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle as O  # noqa: E402

QUANT_CASES = [(7, 69), (8, 1024), (3, 33), (1, 9), (5, 7), (4, 3072)]
NORM_CASES = [(7, 33), (8, 1024), (2, 1030), (3, 7)]
SILU_CASES = [(7, 69), (8, 1024), (2, 3072), (3, 13)]
GEMM_CASES = [(4, 8, 16), (5, 17, 33), (9, 7, 69), (1, 33, 9), (2, 1024, 1024), (7, 69, 33),
              (130, 200, 96)]
EXACT_CASES = [(4, 8, 16), (5, 17, 33), (9, 7, 69), (1, 33, 9), (2, 256, 1024)]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def cfg0_inputs():
    """A [256,1024] ~ N(0,1); W [K=1024, N=3072] int8 uniform
    in [-127,127] (layout=1); scale = |N(0,0.02)|/127; seed 0."""
    rng = np.random.default_rng(0)
    A = rng.standard_normal((256, 1024), dtype=np.float32)
    W_kn = rng.integers(-127, 128, size=(1024, 3072), dtype=np.int8)
    scale = (np.abs(rng.standard_normal(3072)) * 0.02 / 127.0).astype(np.float32)
    return A, W_kn, scale


def exact_activations(rng, M, K):
    """test_gemm.cpp:122-126: multiples of 0.5 with 63.5 at each block start,
    so amax/127 == 0.5 and quantisation is lossless."""
    A = 0.5 * rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    A[:, ::32] = 63.5
    return A


def main():
    if not O.ref_vnni():
        raise SystemExit("the reference's quantised path needs AVX-VNNI on this host")
    rng = np.random.default_rng(1234)
    out = {}
    for i, (M, K) in enumerate(QUANT_CASES):
        A = (rng.standard_normal((M, K)) * 3).astype(np.float32)
        aq, asc = O.ref_quantize(A)
        out[f"quant{i}_A"], out[f"quant{i}_aq"], out[f"quant{i}_asc"] = A, aq, asc
    for i, (M, K) in enumerate(NORM_CASES):
        x = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        w = rng.uniform(0.1, 1.1, K).astype(np.float32)
        aq, asc = O.ref_rmsnorm_quantize(x, w, 1e-6)
        out[f"norm{i}_x"], out[f"norm{i}_w"] = x, w
        out[f"norm{i}_aq"], out[f"norm{i}_asc"] = aq, asc
    for i, (M, K) in enumerate(SILU_CASES):
        g = (rng.standard_normal((M, K)) * 2).astype(np.float32)
        u = rng.standard_normal((M, K)).astype(np.float32)
        aq, asc = O.ref_silu_mul_quantize(g, u)
        out[f"silu{i}_g"], out[f"silu{i}_u"], out[f"silu{i}_aq"], out[f"silu{i}_asc"] = g, u, aq, asc
    for i, (M, N, K) in enumerate(GEMM_CASES):
        A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        s = rng.uniform(1e-4, 1e-2, N).astype(np.float32)
        C0 = rng.uniform(-1, 1, (M, N)).astype(np.float32)
        rp = O.RefPacked(W, s)
        aq, asc = O.ref_quantize(A)
        out[f"gemm{i}_A"], out[f"gemm{i}_W"], out[f"gemm{i}_s"], out[f"gemm{i}_C0"] = A, W, s, C0
        out[f"gemm{i}_C"] = rp.linear_q(aq, asc)            # linear_s8_nk_packed_q
        out[f"gemm{i}_Cadd"] = rp.linear_q(aq, asc, C0)     # linear_s8_nk_packed_q_add
        out[f"gemm{i}_Cpk"] = rp.linear(A)                  # linear_s8_nk_packed
        out[f"gemm{i}_Cpkadd"] = rp.linear(A, C0)           # linear_s8_nk_packed_add
    for i, (M, N, K) in enumerate(EXACT_CASES):
        A = exact_activations(rng, M, K)
        W = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
        s = rng.uniform(1e-4, 1e-2, N).astype(np.float32)
        out[f"exact{i}_A"], out[f"exact{i}_W"], out[f"exact{i}_s"] = A, W, s
        out[f"exact{i}_C"] = O.RefPacked(W, s).linear(A)
    # sliced: test_gemm.cpp:240-297 (two slices of 128 and 64 columns) and the
    # three-way split of the LM's qkv shape (scaled down to 256|128|128).
    for i, (M, K, Ns) in enumerate([(7, 69, [128, 64]), (8, 1024, [128, 64]),
                                    (5, 256, [256, 128, 128])]):
        A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        parts, Ws, ss = [], [], []
        for n in Ns:
            W = rng.integers(-127, 128, size=(n, K), dtype=np.int8)
            s = rng.uniform(1e-4, 1e-2, n).astype(np.float32)
            parts.append(O.RefPacked(W, s))
            Ws.append(W)
            ss.append(s)
        aq, asc = O.ref_quantize(A)
        Cs = O.ref_linear_q_sliced(O.ref_concat(parts), Ns, aq, asc)
        out[f"sliced{i}_A"] = A
        out[f"sliced{i}_Ns"] = np.array(Ns, np.int64)
        for j in range(len(Ns)):
            out[f"sliced{i}_W{j}"], out[f"sliced{i}_s{j}"], out[f"sliced{i}_C{j}"] = Ws[j], ss[j], Cs[j]
    np.savez_compressed(os.path.join(HERE, "gemm_path.npz"), **out)

    # config 0 at full size: digests of the reference's outputs.
    A, W_kn, scale = cfg0_inputs()
    W_nk = np.ascontiguousarray(W_kn.T)
    aq, asc = O.ref_quantize(A)
    C = O.RefPacked(W_nk, scale).linear_q(aq, asc)
    with open(os.path.join(HERE, "cfg0_sha256.txt"), "w") as f:
        f.write("# BASELINE config 0 (seed 0, numpy default_rng), reference CPU VNNI outputs\n")
        f.write(f"inputs_A {sha(A)}\ninputs_W_kn {sha(W_kn)}\ninputs_scale {sha(scale)}\n")
        f.write(f"aq_u8 {sha(aq)}\nasc {sha(asc)}\nC {sha(C)}\n")
        f.write(f"C_sum {float(C.astype(np.float64).sum())!r}\n")
    print("wrote", os.path.join(HERE, "gemm_path.npz"))


if __name__ == "__main__":
    main()
