"""ovnative_b200 -- B200-native int8 LM GEMM path for OVNative.

The product is libovb200.so (CUDA kernels for sm_100a behind the C ABI in
include/ovb200.h).  This package loads it and mirrors the reference's
ov_gemm.h interface on torch CUDA tensors (gemm.py), and adds the per-layer
linear sequence of LM::run_layer (layer.py) used by the benchmark, and the
guided argmax pass of the TTS step (sampler.py) and the attention of a layer
(attention.py).
"""
from ._lib import LIB_PATH, OvbError, lib  # noqa: F401
from .gemm import (  # noqa: F401
    Weight,
    block_products,
    device_status,
    empty_quant,
    empty_quant_f16,
    linear_f32,
    linear_h,
    linear_h_qk_rope,
    linear_h_silu,
    linear_h_sliced,
    linear_q_silu,
    linear_s8_nk_packed,
    linear_s8_nk_packed_add,
    linear_s8_nk_packed_q,
    linear_s8_nk_packed_q_add,
    linear_s8_nk_packed_q_sliced,
    rmsnorm_f16,
    rmsnorm_quantize_f32,
    s8_nk_quant_bytes,
    s8_nk_quant_scales,
    s8_nk_quantize,
    silu_mul_quantize_f32,
    to_f16,
    workspace_bytes,
)
from .attention import (  # noqa: F401
    attention,
    attention_h,
    attention_h_q,
    attention_tiles,
    qk_norm_rope_f16,
    rope_table,
)
from .sampler import guided_sample, guided_sample_batch  # noqa: F401
