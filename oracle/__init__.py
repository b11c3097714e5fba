"""CPU checkers for the int8 LM GEMM path.  TEST INFRASTRUCTURE ONLY.

Two checkers live here, both driven through ctypes with numpy arrays:

* ``port``  -- liboracle.so, the scalar C restatement in ovb_oracle.c of the
  reference's CPU int8 path (cpp/src/backend/cpu/gemm.cpp:379-882 and
  cpp/src/backend/cpu/ops_cpu.cpp:75-198).  Always available once built.
* ``ref``   -- _ref/libovref.so, the reference's own gemm.cpp/ops_cpu.cpp
  compiled from source by oracle/Makefile.  Its int8 quantised path needs an
  AVX-VNNI host (cpu_vnni_available(), gemm.cpp:556-572); ``ref_vnni()`` says
  whether it can run here.
* ``ref_cuda`` -- _ref/libovref_cuda.so, the reference's CUDA LM runner source
  built for sm_100a, for its guided_sample_kernel (the GPU-side checker of
  the device sampler; device pointers, needs a GPU).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package.  The product (ovnative_b200) never does.

Activation format of both checkers is the reference's: aq = u8 (q + 128)
[M, Kb*32] with zero tail bytes, asc = fp32 [M, Kb], Kb = ceil(K/32).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_PORT_PATH = os.path.join(_HERE, "liboracle.so")
_REF_PATH = os.path.join(_HERE, "_ref", "libovref.so")
_REF_CUDA_PATH = os.path.join(_HERE, "_ref", "libovref_cuda.so")

_i64 = C.c_int64
_p = C.c_void_p


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def kblocks(K: int) -> int:
    return (K + 31) // 32


# --------------------------------------------------------------------- port
_port = None


def port_lib():
    global _port
    if _port is None:
        if not os.path.exists(_PORT_PATH):
            raise RuntimeError(f"oracle port not built: {_PORT_PATH} (run make -C oracle)")
        lib = C.CDLL(_PORT_PATH)
        for name, args in {
            "ovo_quantize_u8": [_i64, _i64, _p, _p, _p],
            "ovo_rmsnorm_quantize_u8": [_i64, _i64, _p, _p, C.c_float, _p, _p],
            "ovo_silu_mul_quantize_u8": [_i64, _i64, _p, _p, _p, _p],
            "ovo_block_products": [_i64, _i64, _i64, _p, _p, _p],
            "ovo_linear_q": [_i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, C.c_int],
            "ovo_rmsnorm_into": [_p, _p, _p, _i64, _i64, C.c_float],
            "ovo_silu_mul": [_p, _p, _p, _i64],
            "ovo_guided_sample": [_p, C.c_int, _p, C.c_int, C.c_int, C.c_int, C.c_float,
                                  C.c_float, C.c_int, C.c_int, _p, _p, _p],
        }.items():
            f = getattr(lib, name)
            f.argtypes = args
            f.restype = None
        _port = lib
    return _port


def _quant_out(M: int, K: int):
    Kb = kblocks(K)
    return np.zeros((M, Kb * 32), np.uint8), np.zeros((M, Kb), np.float32)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def quantize(A: np.ndarray):
    """quantize_a_u8 (gemm.cpp:379-430) -> (aq u8 [M,Kp], asc f32 [M,Kb])."""
    A = _f32(A)
    M, K = A.shape
    aq, asc = _quant_out(M, K)
    port_lib().ovo_quantize_u8(M, K, _ptr(A), _ptr(aq), _ptr(asc))
    return aq, asc


def rmsnorm_quantize(x: np.ndarray, w: np.ndarray, eps: float):
    """rmsnorm_quantize_avx2 (gemm.cpp:638-707)."""
    x, w = _f32(x), _f32(w)
    M, K = x.shape
    aq, asc = _quant_out(M, K)
    port_lib().ovo_rmsnorm_quantize_u8(M, K, _ptr(x), _ptr(w), eps, _ptr(aq), _ptr(asc))
    return aq, asc


def silu_mul_quantize(gate: np.ndarray, up: np.ndarray):
    """silu_mul_quant_avx2 (ops_cpu.cpp:144-198)."""
    gate, up = _f32(gate), _f32(up)
    M, K = gate.shape
    aq, asc = _quant_out(M, K)
    port_lib().ovo_silu_mul_quantize_u8(M, K, _ptr(gate), _ptr(up), _ptr(aq), _ptr(asc))
    return aq, asc


def block_products(aq: np.ndarray, W_nk: np.ndarray, K: int) -> np.ndarray:
    """Exact per-32-k int32 products P[m, n, b] (gemm.cpp:455-474)."""
    aq = np.ascontiguousarray(aq, np.uint8)
    W_nk = np.ascontiguousarray(W_nk, np.int8)
    M, N = aq.shape[0], W_nk.shape[0]
    P = np.zeros((M, N, kblocks(K)), np.int32)
    port_lib().ovo_block_products(M, N, K, _ptr(aq), _ptr(W_nk), _ptr(P))
    return P


def linear_q(aq, asc, W_nk, wscale, K: int, C_in=None) -> np.ndarray:
    """linear_s8_nk_packed_q / _q_add semantics (gemm.cpp:432-504).

    W_nk is the [N, K] int8 weight, wscale its per-output-row scale.  With
    C_in the result is added to it (residual epilogue)."""
    aq = np.ascontiguousarray(aq, np.uint8)
    asc = _f32(asc)
    W_nk = np.ascontiguousarray(W_nk, np.int8)
    wscale = _f32(wscale)
    M, N = aq.shape[0], W_nk.shape[0]
    if C_in is None:
        out = np.zeros((M, N), np.float32)
        acc = 0
    else:
        out = _f32(C_in).copy()
        acc = 1
    port_lib().ovo_linear_q(M, N, K, _ptr(aq), _ptr(asc), _ptr(W_nk), _ptr(wscale), _ptr(out), N,
                            acc)
    return out


def rmsnorm_into(x, w, eps: float) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    port_lib().ovo_rmsnorm_into(_ptr(out), _ptr(x), _ptr(w), x.shape[0], x.shape[1], eps)
    return out


def silu_mul(gate, up) -> np.ndarray:
    gate, up = _f32(gate), _f32(up)
    out = np.empty_like(gate)
    port_lib().ovo_silu_mul(_ptr(out), _ptr(gate), _ptr(up), gate.size)
    return out


# ---------------------------------------------------------------- reference
_ref = None


def ref_available() -> bool:
    return os.path.exists(_REF_PATH)


def ref_lib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"reference library not built: {_REF_PATH}")
        lib = C.CDLL(_REF_PATH)
        sig = {
            "ref_vnni_available": ([], C.c_int),
            "ref_kernel_name": ([], C.c_char_p),
            "ref_packed_bytes": ([_i64, _i64], _i64),
            "ref_wsum_elems": ([_i64, _i64], _i64),
            "ref_s8_nk_pack": ([_i64, _i64, _p, _p, _p], C.c_int),
            "ref_s8_nk_quantize": ([_i64, _i64, _p, _p, _p], C.c_int),
            "ref_rmsnorm_quantize": ([_i64, _i64, _p, _p, C.c_float, _p, _p], C.c_int),
            "ref_silu_mul_quantize": ([_i64, _i64, _p, _p, _p, _p], C.c_int),
            "ref_rmsnorm_into": ([_p, _p, _p, _i64, _i64, C.c_float], C.c_int),
            "ref_silu_mul": ([_p, _p, _p, _i64], C.c_int),
            "ref_linear_packed_q": ([_i64, _i64, _i64, _p, _p, _p, _p, _p, _p], C.c_int),
            "ref_linear_packed_q_add": ([_i64, _i64, _i64, _p, _p, _p, _p, _p, _p], C.c_int),
            "ref_linear_packed": ([_i64, _i64, _i64, _p, _p, _p, _p, _p], C.c_int),
            "ref_linear_packed_add": ([_i64, _i64, _i64, _p, _p, _p, _p, _p], C.c_int),
            "ref_linear_packed_q_sliced": ([_i64, _i64, _p, _p, _p, _p, _p, _p, _p, C.c_int],
                                           C.c_int),
            "ref_linear_s8_nk": ([_i64, _i64, _i64, _p, _p, _p, _p], C.c_int),
            "ref_attention_head": ([_p, _i64, _p, _p, _i64, _p, C.c_int, C.c_int, C.c_float,
                                    _p, _i64], C.c_int),
            "ref_ovw1_tensor": ([C.c_char_p, C.c_char_p, _p, _p, C.c_char_p, C.c_int], C.c_int),
            "ref_attention_layer": ([_p, _p, _p, _p, _i64, _i64, C.c_int, C.c_int, C.c_int,
                                     C.c_float, _p, _p, _p, _p, C.c_int], C.c_int),
            "ref_lm_create": ([C.c_char_p, C.c_int, C.c_char_p, C.c_int], _p),
            "ref_lm_destroy": ([_p], None),
            "ref_lm_forward_cfg": ([_p, C.c_int, C.c_int, _p, _p, _p, _p, _p, _p], C.c_int),
            "ref_lm_forward": ([_p, C.c_int, C.c_int, _p, _p, _p, _p, _p], C.c_int),
        }
        for name, (args, res) in sig.items():
            # a library built before a wrapper was added lacks its symbol: that
            # wrapper fails when called, the others keep working
            f = getattr(lib, name, None)
            if f is None:
                continue
            f.argtypes = args
            f.restype = res
        _ref = lib
    return _ref


def ref_vnni() -> bool:
    return ref_available() and bool(ref_lib().ref_vnni_available())


def _chk(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"reference {what} raised (AVX-VNNI missing or bad arguments)")


class RefPacked:
    """A [N, K] int8 weight packed by the reference's s8_nk_pack (gemm.cpp:584-621)."""

    def __init__(self, W_nk: np.ndarray, wscale: np.ndarray):
        lib = ref_lib()
        self.W = np.ascontiguousarray(W_nk, np.int8)
        self.N, self.K = self.W.shape
        self.scale = _f32(wscale)
        self.packed = np.zeros(lib.ref_packed_bytes(self.N, self.K), np.int8)
        self.wsum = np.zeros(lib.ref_wsum_elems(self.N, self.K), np.int32)
        _chk(lib.ref_s8_nk_pack(self.N, self.K, _ptr(self.W), _ptr(self.packed), _ptr(self.wsum)),
             "s8_nk_pack")

    def linear_q(self, aq, asc, C_in=None) -> np.ndarray:
        aq = np.ascontiguousarray(aq, np.uint8)
        asc = _f32(asc)
        M = aq.shape[0]
        lib = ref_lib()
        if C_in is None:
            out = np.zeros((M, self.N), np.float32)
            _chk(lib.ref_linear_packed_q(M, self.N, self.K, _ptr(aq), _ptr(asc), _ptr(self.packed),
                                         _ptr(self.wsum), _ptr(self.scale), _ptr(out)),
                 "linear_s8_nk_packed_q")
        else:
            out = _f32(C_in).copy()
            _chk(lib.ref_linear_packed_q_add(M, self.N, self.K, _ptr(aq), _ptr(asc),
                                             _ptr(self.packed), _ptr(self.wsum), _ptr(self.scale),
                                             _ptr(out)), "linear_s8_nk_packed_q_add")
        return out

    def linear(self, A, C_in=None) -> np.ndarray:
        A = _f32(A)
        M = A.shape[0]
        lib = ref_lib()
        if C_in is None:
            out = np.zeros((M, self.N), np.float32)
            _chk(lib.ref_linear_packed(M, self.N, self.K, _ptr(A), _ptr(self.packed),
                                       _ptr(self.wsum), _ptr(self.scale), _ptr(out)),
                 "linear_s8_nk_packed")
        else:
            out = _f32(C_in).copy()
            _chk(lib.ref_linear_packed_add(M, self.N, self.K, _ptr(A), _ptr(self.packed),
                                           _ptr(self.wsum), _ptr(self.scale), _ptr(out)),
                 "linear_s8_nk_packed_add")
        return out


def ref_concat(parts: list[RefPacked]) -> RefPacked:
    """combine_packed (lm.cpp:57-94): tiles concatenate, wsum interleaves per block."""
    c = RefPacked.__new__(RefPacked)
    c.W = np.concatenate([p.W for p in parts], 0)
    c.N, c.K = c.W.shape
    c.scale = np.concatenate([p.scale for p in parts])
    c.packed = np.concatenate([p.packed for p in parts])
    Kb = kblocks(c.K)
    npads = [(p.N + 7) // 8 * 8 for p in parts]
    c.wsum = np.concatenate([p.wsum.reshape(Kb, npad) for p, npad in zip(parts, npads)],
                            1).reshape(-1).copy()
    return c


def ref_linear_q_sliced(packed: RefPacked, Ns: list[int], aq, asc) -> list[np.ndarray]:
    aq = np.ascontiguousarray(aq, np.uint8)
    asc = _f32(asc)
    M = aq.shape[0]
    outs = [np.zeros((M, n), np.float32) for n in Ns]
    ns = (C.c_int64 * len(Ns))(*Ns)
    cs = (C.c_void_p * len(Ns))(*[o.ctypes.data for o in outs])
    _chk(ref_lib().ref_linear_packed_q_sliced(M, packed.K, _ptr(aq), _ptr(asc),
                                              _ptr(packed.packed), _ptr(packed.wsum),
                                              _ptr(packed.scale), C.cast(ns, C.c_void_p),
                                              C.cast(cs, C.c_void_p), len(Ns)),
         "linear_s8_nk_packed_q_sliced")
    return outs


def ref_quantize(A):
    A = _f32(A)
    M, K = A.shape
    aq, asc = _quant_out(M, K)
    _chk(ref_lib().ref_s8_nk_quantize(M, K, _ptr(A), _ptr(aq), _ptr(asc)), "s8_nk_quantize")
    return aq, asc


def ref_rmsnorm_quantize(x, w, eps: float):
    x, w = _f32(x), _f32(w)
    M, K = x.shape
    aq, asc = _quant_out(M, K)
    _chk(ref_lib().ref_rmsnorm_quantize(M, K, _ptr(x), _ptr(w), eps, _ptr(aq), _ptr(asc)),
         "rmsnorm_quantize_f32")
    return aq, asc


def ref_silu_mul_quantize(gate, up):
    gate, up = _f32(gate), _f32(up)
    M, K = gate.shape
    aq, asc = _quant_out(M, K)
    _chk(ref_lib().ref_silu_mul_quantize(M, K, _ptr(gate), _ptr(up), _ptr(aq), _ptr(asc)),
         "silu_mul_quantize_f32")
    return aq, asc


def ref_rmsnorm_into(x, w, eps: float):
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    _chk(ref_lib().ref_rmsnorm_into(_ptr(out), _ptr(x), _ptr(w), x.shape[0], x.shape[1], eps),
         "rmsnorm_into_f32")
    return out


def ref_silu_mul(gate, up):
    gate, up = _f32(gate), _f32(up)
    out = np.empty_like(gate)
    _chk(ref_lib().ref_silu_mul(_ptr(out), _ptr(gate), _ptr(up), gate.size), "silu_mul_f32")
    return out


# ------------------------------------------------------------- sampler
def guided_sample(cond: np.ndarray, uncond: np.ndarray, T: int, C_books: int, guidance: float,
                  penalty: float, mask_id: int = 1024, in_place: bool = False):
    """The guidance + argmax loop of cpp/src/model/tts.cpp:291-326 on
    token-major planes cond [cond_seq, C*V], uncond [uncond_seq, C*V].
    in_place=True reproduces the reference's in-place log_softmax of the mix
    (tts.cpp:313); False gives the log-probabilities it intends.  Returns
    (pred int32 [C, T], scores float32 [C, T]).  Restatement only (parity
    unpinned: no reference test or callable reference function covers it)."""
    cond = _f32(cond)
    uncond = _f32(uncond)
    V = cond.shape[1] // C_books
    assert cond.shape[1] == uncond.shape[1] == C_books * V
    assert cond.shape[0] >= T and uncond.shape[0] >= T
    pred = np.zeros((C_books, T), np.int32)
    scores = np.zeros((C_books, T), np.float32)
    scratch = np.zeros(4 * V, np.float32)
    port_lib().ovo_guided_sample(_ptr(cond), cond.shape[0], _ptr(uncond), C_books, V, T,
                                 guidance, penalty, mask_id, 1 if in_place else 0, _ptr(pred),
                                 _ptr(scores), _ptr(scratch))
    return pred, scores


# ----------------------------------------------------------- attention
def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, segs, n_heads: int, n_kv: int,
              D: int, scale: float, use_ref: bool | None = None) -> np.ndarray:
    """The reference's attention loop (cpp/src/model/lm.cpp:256-274): for each
    segment (bias [rows, rows] or None, rows, q_off, kv_off -- element offsets
    as in AttnSegment, lm.h:46-51) and query head h (kv head h / group),
    ov::attention_head_f32 (ops_cpu.cpp:907-943) on q [T, n_heads*D],
    k/v [T, n_kv*D], into out [T, n_heads*D].  Runs the reference library
    when it is built (use_ref None/True), else a float64 numpy restatement of
    the same formula."""
    q = _f32(q)
    k = _f32(k)
    v = _f32(v)
    QD, KVD = n_heads * D, n_kv * D
    out = np.zeros_like(q)
    group = n_heads // n_kv
    ref = ref_available() if use_ref is None else use_ref
    for bias, rows, q_off, kv_off in segs:
        b = None if bias is None else _f32(bias)
        for h in range(n_heads):
            kv = h // group
            qo = q_off + h * D
            ko = kv_off + kv * D
            if ref:
                base_q = q.ctypes.data + 4 * qo
                base_k = k.ctypes.data + 4 * ko
                base_v = v.ctypes.data + 4 * ko
                base_o = out.ctypes.data + 4 * qo
                _chk(ref_lib().ref_attention_head(base_q, QD, base_k, base_v, KVD,
                                                  None if b is None else _ptr(b), rows, D,
                                                  scale, base_o, QD), "attention_head_f32")
            else:
                Q = np.stack([q.reshape(-1)[qo + i * QD: qo + i * QD + D] for i in range(rows)])
                K = np.stack([k.reshape(-1)[ko + i * KVD: ko + i * KVD + D] for i in range(rows)])
                V = np.stack([v.reshape(-1)[ko + i * KVD: ko + i * KVD + D] for i in range(rows)])
                sc = (Q.astype(np.float64) @ K.astype(np.float64).T) * scale
                if b is not None:
                    sc = sc + b.astype(np.float64)
                m = sc.max(axis=1, keepdims=True)
                p = np.exp(sc - m)
                o = (p / p.sum(axis=1, keepdims=True)) @ V.astype(np.float64)
                o[m[:, 0] < -1e29] = 0.0
                for i in range(rows):
                    out.reshape(-1)[qo + i * QD: qo + i * QD + D] = o[i]
    return out


def ref_ovw1_tensor(path: str, name: str):
    """The reference's own OVW1 loader (ov::WeightFile::Open + Get + ComputeCrc,
    cpp/src/core/weight_file.cpp:124-222, built into oracle/_ref) on one
    tensor: (info dict, None) or (None, the loader's error message)."""
    info = np.zeros(10, np.int64)
    crc = np.zeros(2, np.uint32)
    err = C.create_string_buffer(512)
    rc = ref_lib().ref_ovw1_tensor(path.encode(), name.encode(), info.ctypes.data,
                                   crc.ctypes.data, err, 512)
    if rc != 0:
        return None, err.value.decode()
    return {"dtype": int(info[0]), "ndim": int(info[1]), "layout": int(info[2]),
            "quant": int(info[3]), "dims": [int(x) for x in info[4:8]], "nbytes": int(info[8]),
            "n_scales": int(info[9]), "crc": int(crc[0]), "crc_computed": int(crc[1])}, None


class RefLM:
    """The reference's own LM (cpp/src/model/lm.h:52-140, lm.cpp, built into
    oracle/_ref) on an OVW1 file: LMConfig defaults except n_layers."""

    def __init__(self, path: str, n_layers: int):
        self._h = None
        err = C.create_string_buffer(512)
        h = ref_lib().ref_lm_create(path.encode(), n_layers, err, 512)
        if not h:
            raise RuntimeError(f"reference LM: {err.value.decode()}")
        self._h = h
        self.C, self.V = 8, 1025

    def close(self):
        if self._h:
            ref_lib().ref_lm_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward_cfg(self, ids, amask, cond_attn, uncond_attn, pos) -> np.ndarray:
        """LM::forward_cfg: ids [C, rows] int64, amask [rows] u8, cond/uncond
        masks u8, pos [rows] int64 -> logits [rows, C*V]."""
        ids = np.ascontiguousarray(ids, np.int64)
        rows = ids.shape[1]
        cs, us = cond_attn.shape[0], uncond_attn.shape[0]
        out = np.zeros((rows, self.C * self.V), np.float32)
        args = [np.ascontiguousarray(a) for a in (amask, cond_attn, uncond_attn)]
        pos = np.ascontiguousarray(pos, np.int64)
        _chk(ref_lib().ref_lm_forward_cfg(self._h, cs, us, _ptr(ids), _ptr(args[0]), _ptr(args[1]),
                                          _ptr(args[2]), _ptr(pos), _ptr(out)), "LM::forward_cfg")
        return out

    def forward(self, ids, amask, attn, pos) -> np.ndarray:
        """LM::forward: ids [B, C, S], amask [B, S], attn [B, S, S], pos [B, S]
        -> logits [B, C, S, V]."""
        ids = np.ascontiguousarray(ids, np.int64)
        B, _, S = ids.shape
        out = np.zeros((B, self.C, S, self.V), np.float32)
        a = np.ascontiguousarray(amask, np.uint8)
        m = np.ascontiguousarray(attn, np.uint8)
        pos = np.ascontiguousarray(pos, np.int64)
        _chk(ref_lib().ref_lm_forward(self._h, B, S, _ptr(ids), _ptr(a), _ptr(m), _ptr(pos),
                                      _ptr(out)), "LM::forward")
        return out


def attention_layer(q: np.ndarray, k: np.ndarray, v: np.ndarray, segs, n_heads: int, n_kv: int,
                    D: int, scale: float) -> np.ndarray:
    """The reference's attention loop of LM::run_layer (cpp/src/model/lm.cpp:
    256-274) as it runs there: ov::attention_head_f32 for every (segment, kv
    head, query head) in one OpenMP loop over the host cores (oracle/_ref).
    Same arguments and result as `attention`."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.zeros_like(q)
    n = len(segs)
    biases = [None if b is None else _f32(b) for b, _, _, _ in segs]
    bp = (C.c_void_p * n)(*[None if b is None else b.ctypes.data for b in biases])
    rows = np.array([r for _, r, _, _ in segs], np.int32)
    qo = np.array([o for _, _, o, _ in segs], np.int64)
    ko = np.array([o for _, _, _, o in segs], np.int64)
    _chk(ref_lib().ref_attention_layer(_ptr(q), _ptr(k), _ptr(v), _ptr(out), n_heads * D,
                                       n_kv * D, n_heads, n_kv, D, scale, C.cast(bp, C.c_void_p),
                                       _ptr(rows), _ptr(qo), _ptr(ko), n),
         "attention loop of LM::run_layer")
    return out


# ----------------------------------------------- reference CUDA sampler
_ref_cuda = None


def ref_cuda_available() -> bool:
    return os.path.exists(_REF_CUDA_PATH)


def _ref_cuda_lib():
    global _ref_cuda
    if _ref_cuda is None:
        if not ref_cuda_available():
            raise RuntimeError(f"reference CUDA library not built: {_REF_CUDA_PATH}")
        lib = C.CDLL(_REF_CUDA_PATH)
        lib.ref_cuda_guided_sample.argtypes = [_p, C.c_int, _p, C.c_int, C.c_int, C.c_int,
                                               C.c_int, C.c_float, C.c_float, C.c_int, _p, _p,
                                               _p]
        lib.ref_cuda_guided_sample.restype = C.c_int
        lib.ref_cuda_lm_create.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_int]
        lib.ref_cuda_lm_create.restype = _p
        lib.ref_cuda_lm_destroy.argtypes = [_p]
        lib.ref_cuda_lm_destroy.restype = None
        lib.ref_cuda_lm_forward.argtypes = [_p, C.c_int, C.c_int, _p, _p, _p, _p, _p]
        lib.ref_cuda_lm_forward.restype = C.c_int
        _ref_cuda = lib
    return _ref_cuda


class RefCudaLM:
    """The reference's own CUDA LM runner (cpp/src/backend/cuda/cuda_lm.cu:
    790-1221, built from its source into oracle/_ref) on an OVW1 file in the
    [K, N] int8 encoding: LM::forward's arguments on host buffers."""

    def __init__(self, path: str, n_layers: int):
        self._h = None
        err = C.create_string_buffer(512)
        h = _ref_cuda_lib().ref_cuda_lm_create(path.encode(), n_layers, err, 512)
        if not h:
            raise RuntimeError(f"reference CUDA LM: {err.value.decode()}")
        self._h = h
        self.C, self.V = 8, 1025

    def close(self):
        if self._h:
            _ref_cuda_lib().ref_cuda_lm_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def forward(self, ids, amask, attn, pos) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int64)
        B, _, S = ids.shape
        out = np.zeros((B, self.C, S, self.V), np.float32)
        a = np.ascontiguousarray(amask, np.uint8)
        m = np.ascontiguousarray(attn, np.uint8)
        pos = np.ascontiguousarray(pos, np.int64)
        rc = _ref_cuda_lib().ref_cuda_lm_forward(self._h, B, S, _ptr(ids), _ptr(a), _ptr(m),
                                                 _ptr(pos), _ptr(out))
        _chk(rc, "LmRunner::forward")
        return out


def ref_cuda_guided_sample(cond, uncond, T: int, C_books: int, guidance: float, penalty: float,
                           mask_id: int = 1024):
    """The reference's own CUDA guided_sample_kernel (cpp/src/backend/cuda/
    cuda_lm.cu:679-758, launched as LmRunnerSampleThunk launches it) on
    token-major torch CUDA planes cond [cond_seq, C*V] / uncond
    [uncond_seq, C*V].  Returns (pred int32 [C, T], scores fp32 [C, T]) as
    torch CUDA tensors, ordered on torch's current stream."""
    import torch
    lib = _ref_cuda_lib()
    V = cond.shape[1] // C_books
    pred = torch.empty((C_books, T), dtype=torch.int32, device=cond.device)
    scores = torch.empty((C_books, T), dtype=torch.float32, device=cond.device)
    rc = lib.ref_cuda_guided_sample(cond.data_ptr(), cond.shape[0], uncond.data_ptr(),
                                          uncond.shape[0], C_books, V, T, guidance, penalty,
                                          mask_id, pred.data_ptr(), scores.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream)
    _chk(rc, "guided_sample_kernel launch")
    return pred, scores
