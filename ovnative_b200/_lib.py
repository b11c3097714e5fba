"""ctypes binding of libovb200.so (the C ABI declared in include/ovb200.h).

The library is loaded from this package directory only; when it is missing
or fails to load, every entry point raises -- there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libovb200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "ovb200.h")

OVB_OK = 0
OVB_ERR_INVALID_ARG = -1
OVB_ERR_INTERNAL = -4
OVB_LAYOUT_NK = 0
OVB_LAYOUT_KN = 1
OVB_SRC_DEVICE = 1
OVB_WEIGHT_F16 = 2
OVB_AQ_U8 = 1
OVB_AQ_F16 = 2
OVB_AQ_F16_RAW = 4

_i64 = C.c_int64
_p = C.c_void_p
_int = C.c_int


class Slice(C.Structure):
    _fields_ = [("N", C.c_int64), ("C", C.c_void_p), ("ldc", C.c_int64)]


class WeightSrc(C.Structure):
    """ovb_weight_src: one source of ovb_weight_create_batch."""
    _fields_ = [("W", C.c_void_p), ("layout", C.c_int), ("N", C.c_int64), ("K", C.c_int64),
                ("scale", C.c_void_p)]


class Ovw1Tensor(C.Structure):
    """ovb_ovw1_tensor: one tensor of a mapped OVW1 file."""
    _fields_ = [("name", C.c_char_p), ("name_len", C.c_int32), ("dtype", C.c_int32),
                ("ndim", C.c_int32), ("layout", C.c_int32), ("quant", C.c_int32),
                ("dims", C.c_int64 * 4), ("data", C.c_void_p), ("nbytes", C.c_int64),
                ("scales", C.c_void_p), ("n_scales", C.c_int64), ("crc", C.c_uint32)]


class GuidedPair(C.Structure):
    """ovb_guided_pair."""
    _fields_ = [("cond", C.c_void_p), ("cond_seq", C.c_int), ("uncond", C.c_void_p),
                ("uncond_seq", C.c_int), ("target_len", C.c_int)]


class AttnSegment(C.Structure):
    """ovb_attn_segment (the reference's AttnSegment, cpp/src/model/lm.h:46-51)."""
    _fields_ = [("bias", C.c_void_p), ("rows", C.c_int32), ("q_off", C.c_int64),
                ("kv_off", C.c_int64)]


# name -> (argtypes, restype)
SIGNATURES = {
    "ovb_abi_version": ([], _int),
    "ovb_last_error": ([], C.c_char_p),
    "ovb_device_status": ([_p], _int),
    "ovb_selftest_wait_timeout": ([_p], _int),
    "ovb_quant_bytes": ([_i64, _i64], _i64),
    "ovb_quant_scales": ([_i64, _i64], _i64),
    "ovb_weight_create": ([_p, _int, _i64, _i64, _p, _int, _p, C.POINTER(_p)], _int),
    "ovb_weight_concat": ([_p, _int, _p, C.POINTER(_p)], _int),
    "ovb_weight_destroy": ([_p], _int),
    "ovb_weight_shape": ([_p, C.POINTER(_i64), C.POINTER(_i64)], _int),
    "ovb_weight_export": ([_p, _p, _p], _int),
    "ovb_quantize": ([_i64, _i64, _p, _i64, _p, _p, _int, _p], _int),
    "ovb_rmsnorm_quantize": ([_i64, _i64, _p, _p, C.c_float, _p, _p, _int, _p], _int),
    "ovb_silu_mul_quantize": ([_i64, _i64, _p, _i64, _p, _i64, _p, _p, _int, _p], _int),
    "ovb_linear_q": ([_i64, _p, _p, _p, _p, _i64, _int, _p], _int),
    "ovb_linear_q_sliced": ([_i64, _p, _p, _p, C.POINTER(Slice), _int, _p], _int),
    "ovb_linear_h": ([_i64, _p, _p, _p, _i64, _int, _p], _int),
    "ovb_linear_q_silu": ([_i64, _p, _p, _p, _p, _p, _int, _p], _int),
    "ovb_linear_h_silu": ([_i64, _p, _p, _p, _p, _int, _p], _int),
    "ovb_weight_gate_up": ([_p, _p, _p, C.POINTER(_p)], _int),
    "ovb_linear_h_sliced": ([_i64, _p, _p, C.POINTER(Slice), _int, _p], _int),
    "ovb_rope_table": ([_p, _i64, _int, C.c_float, _p, _p], _int),
    "ovb_qk_norm_rope_f16": ([_i64, _p, _p, _p, _int, _int, _int, _p, _p, C.c_float, _p, _p, _p,
                              _p, _p], _int),
    "ovb_linear_h_qk_rope": ([_i64, _p, _p, _int, _int, _int, _p, _p, C.c_float, _p, _p, _p, _p,
                              _p], _int),
    "ovb_linear_workspace_bytes": ([_i64, _i64], C.c_size_t),
    "ovb_linear": ([_i64, _p, _p, _i64, _p, _i64, _int, _p, C.c_size_t, _p], _int),
    "ovb_linear_static": ([_i64, _p, _p, _i64, _p, _i64, _int, _p], _int),
    "ovb_block_products": ([_i64, _p, _p, _p, _p], _int),
    "ovb_guided_sample": ([_p, _int, _p, _int, _int, _int, _int, C.c_float, C.c_float, _int,
                           _p, _p, _p], _int),
    "ovb_guided_sample_batch": ([_int, _p, _int, _int, C.c_float, C.c_float, _int, _p, _p, _p],
                                _int),
    "ovb_ovw1_open": ([C.c_char_p, C.POINTER(_p)], _int),
    "ovb_ovw1_close": ([_p], _int),
    "ovb_ovw1_count": ([_p], _i64),
    "ovb_ovw1_header": ([_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                         C.POINTER(C.c_uint64)], _int),
    "ovb_ovw1_tensor_at": ([_p, _i64, C.POINTER(Ovw1Tensor)], _int),
    "ovb_ovw1_find": ([_p, C.c_char_p, C.POINTER(Ovw1Tensor)], _int),
    "ovb_ovw1_crc": ([_p, C.c_char_p, C.POINTER(C.c_uint32)], _int),
    "ovb_ovw1_weight": ([_p, C.c_char_p, _int, _p, C.POINTER(_p)], _int),
    "ovb_ovw1_weights": ([_p, C.POINTER(C.c_char_p), _int, _int, _p, C.POINTER(_p)], _int),
    "ovb_weight_create_batch": ([C.POINTER(WeightSrc), _int, _int, _p, C.POINTER(_p)], _int),
    "ovb_lm_create": ([C.c_char_p, _int, _p, C.POINTER(_p)], _int),
    "ovb_lm_destroy": ([_p], _int),
    "ovb_lm_config": ([_p, C.POINTER(_i64)], _int),
    "ovb_lm_reserve": ([_p, _i64, _i64], _int),
    "ovb_lm_logits": ([_p], _p),
    "ovb_lm_forward_cfg": ([_p, _int, _int, _p, _p, _p, _p, _p, _p, _p], _int),
    "ovb_lm_forward_cfg_device": ([_p, _int, _int, _p, _p, _p, _p, _p, _p], _int),
    "ovb_lm_forward_segments_device": ([_p, _int, _p, _p, _p, _p, _p, _p], _int),
    "ovb_weight_create_f32": ([_p, _int, _i64, _i64, _p, C.POINTER(_p)], _int),
    "ovb_lm_forward": ([_p, _int, _int, _p, _p, _p, _p, _p, _p], _int),
    "ovb_lm_sample": ([_p, _p, _int, _p, _int, _int, C.c_float, C.c_float, _int, _p, _p, _p],
                      _int),
    "ovb_attention": ([_p, _p, _p, _p, _i64, _i64, _int, _int, _int, C.c_float,
                       C.POINTER(AttnSegment), _int, _p], _int),
    "ovb_attention_h": ([_p, _p, _p, _p, _i64, _i64, _int, _int, _int, C.c_float,
                         C.POINTER(AttnSegment), _int, _p, _p], _int),
    "ovb_attention_h_q": ([_p, _p, _p, _i64, _i64, _int, _int, _int, C.c_float,
                           C.POINTER(AttnSegment), _int, _p, _p, _p, _int, _p], _int),
    "ovb_attention_tiles_bytes": ([_p, _int], C.c_size_t),
    "ovb_attention_tiles": ([_p, _int, _p, _p, C.c_size_t, _p], _int),
}

_lib = None


class OvbError(RuntimeError):
    """A non-OK status from the C ABI (OVB_ERR_INTERNAL and friends)."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"ovb status {status}: {msg}")
        self.status = status


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m ovnative_b200.build` "
                "(the CUDA extension is required, there is no CPU fallback)")
        h = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            f = getattr(h, name)
            f.argtypes = args
            f.restype = res
        _lib = h
    return _lib


def check(status: int) -> None:
    """Raise like the reference does: ValueError where it throws
    std::invalid_argument / rejects arguments, RuntimeError otherwise."""
    if status == OVB_OK:
        return
    msg = lib().ovb_last_error().decode(errors="replace")
    if status == OVB_ERR_INVALID_ARG:
        raise ValueError(msg)
    raise OvbError(status, msg)
