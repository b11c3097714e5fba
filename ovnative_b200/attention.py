"""The attention of one LM layer (ovb_attention) on torch CUDA tensors.

Mirrors the reference's loop in LM::run_layer (cpp/src/model/lm.cpp:256-274):
for every AttnSegment (cpp/src/model/lm.h:46-51) -- `rows` query rows at
element offset q_off of q/out, the matching keys/values at kv_off of k/v, an
optional additive bias [rows, rows] -- and every query head h (kv head
h // (n_heads // n_kv)), ov::attention_head_f32 (cpp/src/backend/cpu/
ops_cpu.cpp:907-943):

    out[s] = softmax_t(q[s] . k[t] * scale + bias[s, t]) v[t]

with a fully masked row (every score below -1e29) giving zeros.  head_dim is
128.  The products run on the tensor cores with fp16 inputs and fp32
accumulation (about 1e-3 relative to the fp32 reference).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

HEAD_DIM = 128


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, segs, n_heads: int, n_kv: int,
              scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """q [T, n_heads * 128], k / v [T', n_kv * 128]: contiguous fp32 CUDA
    tensors.  segs: iterable of (bias or None, rows, q_off, kv_off) with
    element offsets, as AttnSegment.  Returns out, laid out like q (rows that
    no segment covers are left as they were: zeros when out is None)."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda or t.dtype != torch.float32 or t.dim() != 2 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 2-D float32 CUDA tensor")
    if k.shape != v.shape:
        raise ValueError("k and v must have the same shape")
    if q.shape[1] != n_heads * HEAD_DIM or k.shape[1] != n_kv * HEAD_DIM:
        raise ValueError("q / k widths must be n_heads * 128 / n_kv * 128")
    if out is None:
        out = torch.zeros_like(q)
    elif out.shape != q.shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 tensor shaped like q")
    segs = list(segs)
    arr = (L.AttnSegment * max(1, len(segs)))()
    keep = []
    for i, (bias, rows, q_off, kv_off) in enumerate(segs):
        if rows < 0 or q_off < 0 or kv_off < 0:
            raise ValueError("negative segment field")
        if q_off + rows * q.shape[1] > q.numel() or kv_off + rows * k.shape[1] > k.numel():
            raise ValueError("segment runs past the end of q / k")
        bp = None
        if bias is not None:
            if (not bias.is_cuda or bias.dtype != torch.float32 or not bias.is_contiguous()
                    or bias.numel() != rows * rows):
                raise ValueError("bias must be a contiguous float32 CUDA tensor of rows * rows")
            keep.append(bias)
            bp = bias.data_ptr()
        arr[i] = L.AttnSegment(bp, int(rows), int(q_off), int(kv_off))
    L.check(L.lib().ovb_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                  q.shape[1], k.shape[1], n_heads, n_kv, HEAD_DIM, float(scale),
                                  C.cast(arr, C.POINTER(L.AttnSegment)), len(segs),
                                  torch.cuda.current_stream().cuda_stream))
    return out
