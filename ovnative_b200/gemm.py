"""Host-side mirror of the reference's GEMM backend contract for this path.

The functions here carry the names and argument meaning of
cpp/include/ovnative/ov_gemm.h (namespace ov) -- s8_nk_quantize,
rmsnorm_quantize_f32, silu_mul_quantize_f32, linear_s8_nk_packed_q[_add],
linear_s8_nk_packed_q_sliced, linear_s8_nk_packed[_add] -- but run on the
B200 through the C ABI (include/ovb200.h).  Tensors are torch CUDA tensors
(PyTorch is used for device memory and streams only); every call is ordered on
torch's current stream.

Error behaviour follows the reference: M/N/K <= 0 is a no-op
(gemm.cpp:761, :779, :832), argument errors raise ValueError where the
reference throws std::invalid_argument (gemm.cpp:786-788), and device or
launch failures raise RuntimeError (std::runtime_error in the reference).

Quantised activations: aq is int8 q (or the reference's u8 q+128 when
``u8=True``, for byte comparison), [M, 32*ceil(K/32)], asc fp32 [M, ceil(K/32)].
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dev_ptr(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return t.data_ptr()


def _rows_ok(t: torch.Tensor, name: str):
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with unit column stride")


def kblocks(K: int) -> int:
    return (K + 31) // 32


def s8_nk_quant_bytes(M: int, K: int) -> int:
    """ov::s8_nk_quant_bytes (ov_gemm.h:95)."""
    return int(L.lib().ovb_quant_bytes(M, K))


def s8_nk_quant_scales(M: int, K: int) -> int:
    """ov::s8_nk_quant_scales (ov_gemm.h:96)."""
    return int(L.lib().ovb_quant_scales(M, K))


def empty_quant(M: int, K: int, device=None):
    """Allocate (aq, asc) for M rows of K features."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    Kb = kblocks(K)
    return (torch.empty((M, Kb * 32), dtype=torch.int8, device=dev),
            torch.empty((M, Kb), dtype=torch.float32, device=dev))


class Weight:
    """A device-resident int8 weight with per-output-channel scales.

    Built from either OVW1 layout: ``from_nk`` ([N, K], layout=0) or
    ``from_kn`` ([K, N], layout=1).  Replaces ``Mat``'s packed VNNI tiles
    (mat.cpp:88-104 / s8_nk_pack) and the CUDA runner's dequantised copies
    (cuda_lm.cu:840-873).

    ``f16=True`` (OVB_WEIGHT_F16) also keeps an fp16 copy, and the GEMMs on
    this weight run the fp16 tensor-core mainloop: within rel-L2 ~3e-4 of
    the reference instead of bit-exact, several times faster.
    """

    def __init__(self, handle: int, N: int, K: int, f16: bool = False):
        self._h = handle
        self.N = N
        self.K = K
        self.f16 = f16

    @property
    def handle(self) -> int:
        if not self._h:
            raise ValueError("weight was destroyed")
        return self._h

    @classmethod
    def _create(cls, W, scale, layout: int, N: int, K: int, f16: bool) -> "Weight":
        out = C.c_void_p()
        flags = L.OVB_WEIGHT_F16 if f16 else 0
        if isinstance(W, torch.Tensor) and W.is_cuda:
            W = W.contiguous()
            scale = scale.to(device=W.device, dtype=torch.float32).contiguous()
            st = L.lib().ovb_weight_create(W.data_ptr(), layout, N, K, scale.data_ptr(),
                                           L.OVB_SRC_DEVICE | flags, _stream(), C.byref(out))
        else:
            Wn = np.ascontiguousarray(W.cpu().numpy() if isinstance(W, torch.Tensor) else W,
                                      dtype=np.int8)
            sn = np.ascontiguousarray(scale.cpu().numpy() if isinstance(scale, torch.Tensor)
                                      else scale, dtype=np.float32)
            st = L.lib().ovb_weight_create(Wn.ctypes.data, layout, N, K, sn.ctypes.data, flags,
                                           _stream(), C.byref(out))
        L.check(st)
        return cls(out.value, N, K, f16)

    @classmethod
    def from_nk(cls, W, scale, f16: bool = False) -> "Weight":
        N, K = W.shape
        return cls._create(W, scale, L.OVB_LAYOUT_NK, N, K, f16)

    @classmethod
    def from_kn(cls, W, scale, f16: bool = False) -> "Weight":
        K, N = W.shape
        return cls._create(W, scale, L.OVB_LAYOUT_KN, N, K, f16)

    @classmethod
    def from_f32(cls, W, layout: int = 1) -> "Weight":
        """An fp32 linear weight (ovb_weight_create_f32): the reference's fp32
        encoding, layout 1 [K, N] (tools/convert_weights.py:178-180) or
        layout 0 [N, K], held as fp16 with power-of-two channel scales.  Only
        the fp16 mainloop (linear_h / linear_f32) takes it."""
        Wn = np.ascontiguousarray(W.cpu().numpy() if isinstance(W, torch.Tensor) else W,
                                  dtype=np.float32)
        if Wn.ndim != 2:
            raise ValueError("expected a 2-D weight")
        N, K = (Wn.shape[1], Wn.shape[0]) if layout == L.OVB_LAYOUT_KN else Wn.shape
        out = C.c_void_p()
        L.check(L.lib().ovb_weight_create_f32(Wn.ctypes.data, layout, N, K, _stream(),
                                              C.byref(out)))
        w = cls(out.value, N, K, True)
        w.fp32 = True
        return w

    @classmethod
    def concat(cls, parts: list["Weight"]) -> "Weight":
        """combine_packed (lm.cpp:57-94): q|k|v or gate|up along N."""
        arr = (C.c_void_p * len(parts))(*[p.handle for p in parts])
        out = C.c_void_p()
        L.check(L.lib().ovb_weight_concat(C.cast(arr, C.c_void_p), len(parts), _stream(),
                                          C.byref(out)))
        return cls(out.value, sum(p.N for p in parts), parts[0].K, all(p.f16 for p in parts))

    @classmethod
    def gate_up(cls, gate: "Weight", up: "Weight") -> "Weight":
        """gate|up interleaved in 32-row blocks for the fused SiLU*up GEMMs
        (ovb_weight_gate_up)."""
        out = C.c_void_p()
        L.check(L.lib().ovb_weight_gate_up(gate.handle, up.handle, _stream(), C.byref(out)))
        w = cls(out.value, 2 * gate.N, gate.K, gate.f16 and up.f16)
        w.glu = True
        return w

    def export(self):
        """The device weight as ([N, K] int8, [N] fp32) numpy arrays."""
        W = np.zeros((self.N, self.K), np.int8)
        s = np.zeros(self.N, np.float32)
        L.check(L.lib().ovb_weight_export(self.handle, W.ctypes.data, s.ctypes.data))
        return W, s

    def close(self):
        if self._h:
            L.lib().ovb_weight_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------ quantisers
def _flags(u8: bool, f16: bool = False) -> int:
    if u8 and f16:
        raise ValueError("u8 and f16 outputs are exclusive")
    return (L.OVB_AQ_U8 if u8 else 0) | (L.OVB_AQ_F16 if f16 else 0)


def to_f16(A: torch.Tensor, out=None) -> torch.Tensor:
    """fp16 of A itself, [M, Kp] with a zero tail (OVB_AQ_F16_RAW): the
    activations of an fp32 weight."""
    _rows_ok(A, "A")
    M, K = A.shape
    a16 = out if out is not None else torch.empty((M, kblocks(K) * 32), dtype=torch.float16,
                                                  device=A.device)
    L.check(L.lib().ovb_quantize(M, K, _dev_ptr(A), A.stride(0), _dev_ptr(a16), None,
                                 L.OVB_AQ_F16_RAW, _stream()))
    return a16


def rmsnorm_f16(x: torch.Tensor, w: torch.Tensor, eps: float, out=None) -> torch.Tensor:
    """fp16 of rmsnorm_into_f32's output (ops_cpu.cpp:812-825; the same
    values rmsnorm_quantize_f32 quantises), [M, Kp] with a zero tail."""
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    M, K = x.shape
    a16 = out if out is not None else torch.empty((M, kblocks(K) * 32), dtype=torch.float16,
                                                  device=x.device)
    L.check(L.lib().ovb_rmsnorm_quantize(M, K, _dev_ptr(x), _dev_ptr(w.contiguous()), eps,
                                         _dev_ptr(a16), None, L.OVB_AQ_F16_RAW, _stream()))
    return a16


def empty_quant_f16(M: int, K: int, device=None):
    """Allocate (a16, asc) for M rows: a16 is [M, Kp] fp16 (OVB_AQ_F16 form)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    Kb = kblocks(K)
    return (torch.empty((M, Kb * 32), dtype=torch.float16, device=dev),
            torch.empty((M, Kb), dtype=torch.float32, device=dev))


def _quant_out(M, K, device, u8, out, f16=False):
    if out is not None:
        return out
    if f16:
        return empty_quant_f16(M, K, device)
    aq, asc = empty_quant(M, K, device)
    if u8:
        aq = aq.view(torch.uint8)
    return aq, asc


def s8_nk_quantize(A: torch.Tensor, u8: bool = False, out=None, f16: bool = False):
    """ov::s8_nk_quantize (ov_gemm.h:97): per-row, per-32-k quantisation.
    ``f16=True`` writes the dequantised fp16(q * asc) instead of q (input of
    linear_h)."""
    _rows_ok(A, "A")
    M, K = A.shape
    aq, asc = _quant_out(M, K, A.device, u8, out, f16)
    L.check(L.lib().ovb_quantize(M, K, _dev_ptr(A), A.stride(0), _dev_ptr(aq), _dev_ptr(asc),
                                 _flags(u8, f16), _stream()))
    return aq, asc


def rmsnorm_quantize_f32(x: torch.Tensor, w: torch.Tensor, eps: float, u8: bool = False,
                         out=None, f16: bool = False):
    """ov::rmsnorm_quantize_f32 (ov_gemm.h:118-119)."""
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    M, K = x.shape
    aq, asc = _quant_out(M, K, x.device, u8, out, f16)
    L.check(L.lib().ovb_rmsnorm_quantize(M, K, _dev_ptr(x), _dev_ptr(w.contiguous()), eps,
                                         _dev_ptr(aq), _dev_ptr(asc), _flags(u8, f16), _stream()))
    return aq, asc


def silu_mul_quantize_f32(gate: torch.Tensor, up: torch.Tensor, u8: bool = False, out=None,
                          f16: bool = False):
    """ov::silu_mul_quantize_f32 (ov_gemm.h:84-85)."""
    _rows_ok(gate, "gate")
    _rows_ok(up, "up")
    M, K = gate.shape
    aq, asc = _quant_out(M, K, gate.device, u8, out, f16)
    L.check(L.lib().ovb_silu_mul_quantize(M, K, _dev_ptr(gate), gate.stride(0), _dev_ptr(up),
                                          up.stride(0), _dev_ptr(aq), _dev_ptr(asc),
                                          _flags(u8, f16), _stream()))
    return aq, asc


# ----------------------------------------------------------------- GEMMs
def _out(M, w: Weight, C, device):
    if C is None:
        return torch.empty((M, w.N), dtype=torch.float32, device=device)
    _rows_ok(C, "C")
    return C


def linear_s8_nk_packed_q(aq: torch.Tensor, asc: torch.Tensor, w: Weight, C=None):
    """ov::linear_s8_nk_packed_q (ov_gemm.h:98-100): C = linear(aq, asc)."""
    M = aq.shape[0]
    C = _out(M, w, C, aq.device)
    L.check(L.lib().ovb_linear_q(M, w.handle, _dev_ptr(aq), _dev_ptr(asc), _dev_ptr(C),
                                 C.stride(0), 0, _stream()))
    return C


def linear_s8_nk_packed_q_add(aq: torch.Tensor, asc: torch.Tensor, w: Weight, C: torch.Tensor):
    """ov::linear_s8_nk_packed_q_add (ov_gemm.h:78-80): C += linear(aq, asc)."""
    _rows_ok(C, "C")
    L.check(L.lib().ovb_linear_q(aq.shape[0], w.handle, _dev_ptr(aq), _dev_ptr(asc),
                                 _dev_ptr(C), C.stride(0), 1, _stream()))
    return C


def linear_s8_nk_packed_q_sliced(aq: torch.Tensor, asc: torch.Tensor, w: Weight,
                                 Cs: list[torch.Tensor]):
    """ov::linear_s8_nk_packed_q_sliced (ov_gemm.h:109-111): one launch over a
    concatenated weight, slice i written to Cs[i] ([M, N_i], N_i % 64 == 0)."""
    for c in Cs:
        _rows_ok(c, "C")
    arr = (L.Slice * len(Cs))(*[L.Slice(c.shape[1], _dev_ptr(c), c.stride(0)) for c in Cs])
    L.check(L.lib().ovb_linear_q_sliced(aq.shape[0], w.handle, _dev_ptr(aq), _dev_ptr(asc), arr,
                                        len(Cs), _stream()))
    return Cs


def linear_h(a16: torch.Tensor, w: Weight, C=None, accumulate: bool = False):
    """The fp16 mainloop on dequantised activations (ovb_linear_h): a16 from a
    quantiser with ``f16=True``, w created with ``f16=True``."""
    M = a16.shape[0]
    C = _out(M, w, C, a16.device)
    L.check(L.lib().ovb_linear_h(M, w.handle, _dev_ptr(a16), _dev_ptr(C), C.stride(0),
                                 1 if accumulate else 0, _stream()))
    return C


def linear_h_sliced(a16: torch.Tensor, w: Weight, Cs: list[torch.Tensor]):
    """linear_h over a concatenated weight, slice i written to Cs[i]."""
    for c in Cs:
        _rows_ok(c, "C")
    arr = (L.Slice * len(Cs))(*[L.Slice(c.shape[1], _dev_ptr(c), c.stride(0)) for c in Cs])
    L.check(L.lib().ovb_linear_h_sliced(a16.shape[0], w.handle, _dev_ptr(a16), arr, len(Cs),
                                        _stream()))
    return Cs


def linear_h_qk_rope(a16: torch.Tensor, w: Weight, n_heads: int, n_kv: int, q_norm: torch.Tensor,
                     k_norm: torch.Tensor, eps: float, table: torch.Tensor, out=None):
    """The q|k|v GEMM with the per-head q/k RMSNorm + RoPE fused into its
    epilogue (ovb_linear_h_qk_rope): returns fp16 (q16 [M, n_heads*128], k16,
    v16 [M, n_kv*128]), the same bytes as linear_h_sliced into fp32 q / k / v
    followed by attention.qk_norm_rope_f16.  ``table`` from
    attention.rope_table."""
    M = a16.shape[0]
    if out is None:
        out = (torch.empty((M, n_heads * 128), dtype=torch.float16, device=a16.device),
               torch.empty((M, n_kv * 128), dtype=torch.float16, device=a16.device),
               torch.empty((M, n_kv * 128), dtype=torch.float16, device=a16.device))
    for t in (q_norm, k_norm, table, *out):
        if not t.is_contiguous():
            raise ValueError("q_norm, k_norm, table and the outputs must be contiguous")
    if table.dtype != torch.float32 or table.numel() < M * 128:
        raise ValueError("table must be float32 with 128 floats per row (rope_table)")
    q16, k16, v16 = out
    L.check(L.lib().ovb_linear_h_qk_rope(M, w.handle, _dev_ptr(a16), n_heads, n_kv, 128,
                                         _dev_ptr(q_norm), _dev_ptr(k_norm), float(eps),
                                         _dev_ptr(table), _dev_ptr(q16), _dev_ptr(k16),
                                         _dev_ptr(v16), _stream()))
    return out


def linear_f32(A: torch.Tensor, w: Weight, C=None, accumulate: bool = False):
    """ov::linear_f32 / linear_f32_ld with accumulate (Mat::mul / mul_add on
    an fp32 weight, mat.cpp:11-13, :39-43) on the fp16 tensor cores: A to
    fp16, then linear_h with a weight from Weight.from_f32."""
    a16 = to_f16(A)
    return linear_h(a16, w, C, accumulate)


def _silu_out(M, w: Weight, device, u8, f16, out):
    if out is not None:
        return out
    inter = w.N // 2
    if f16:
        return empty_quant_f16(M, inter, device)
    aq, asc = empty_quant(M, inter, device)
    return (aq.view(torch.uint8) if u8 else aq), asc


def linear_q_silu(aq: torch.Tensor, asc: torch.Tensor, w: Weight, out=None, u8: bool = False,
                  f16: bool = False):
    """gate|up GEMM fused with silu_mul_quantize_f32 on the int8 mainloop
    (bit-identical to the two reference calls).  Returns (q or fp16, scales)."""
    M = aq.shape[0]
    q, sc = _silu_out(M, w, aq.device, u8, f16, out)
    L.check(L.lib().ovb_linear_q_silu(M, w.handle, _dev_ptr(aq), _dev_ptr(asc), _dev_ptr(q),
                                      _dev_ptr(sc), _flags(u8, f16), _stream()))
    return q, sc


def linear_h_silu(a16: torch.Tensor, w: Weight, out=None, u8: bool = False, f16: bool = True):
    """The same on the fp16 mainloop (a16 = fp16(q*asc) activations)."""
    M = a16.shape[0]
    q, sc = _silu_out(M, w, a16.device, u8, f16, out)
    L.check(L.lib().ovb_linear_h_silu(M, w.handle, _dev_ptr(a16), _dev_ptr(q), _dev_ptr(sc),
                                      _flags(u8, f16), _stream()))
    return q, sc


def workspace_bytes(M: int, K: int) -> int:
    return int(L.lib().ovb_linear_workspace_bytes(M, K))


def _work(M, K, device, work):
    need = workspace_bytes(M, K)
    if work is None:
        work = torch.empty(max(need, 1), dtype=torch.uint8, device=device)
    return work, need


def linear_s8_nk_packed(A: torch.Tensor, w: Weight, C=None, work=None):
    """ov::linear_s8_nk_packed (ov_gemm.h:67-69): quantise A, then C = linear."""
    _rows_ok(A, "A")
    M = A.shape[0]
    C = _out(M, w, C, A.device)
    work, need = _work(M, w.K, A.device, work)
    L.check(L.lib().ovb_linear(M, w.handle, _dev_ptr(A), A.stride(0), _dev_ptr(C), C.stride(0),
                               0, _dev_ptr(work), work.numel(), _stream()))
    return C


def linear_s8_nk_packed_add(A: torch.Tensor, w: Weight, C: torch.Tensor, work=None):
    """ov::linear_s8_nk_packed_add (ov_gemm.h:73-75): C += linear(quantise(A))."""
    _rows_ok(A, "A")
    _rows_ok(C, "C")
    work, need = _work(A.shape[0], w.K, A.device, work)
    L.check(L.lib().ovb_linear(A.shape[0], w.handle, _dev_ptr(A), A.stride(0), _dev_ptr(C),
                               C.stride(0), 1, _dev_ptr(work), work.numel(), _stream()))
    return C


def block_products(aq: torch.Tensor, w: Weight) -> torch.Tensor:
    """Exact int32 per-32-k block products P[m, n, b] from the tensor-core mainloop."""
    M = aq.shape[0]
    P = torch.empty((M, w.N, kblocks(w.K)), dtype=torch.int32, device=aq.device)
    L.check(L.lib().ovb_block_products(M, w.handle, _dev_ptr(aq), _dev_ptr(P), _stream()))
    return P


def device_status() -> int:
    """Status word of the bounded device waits (0 = all completed); clears it."""
    st = L.lib().ovb_device_status(_stream())
    if st < 0:
        L.check(st)
    return st
