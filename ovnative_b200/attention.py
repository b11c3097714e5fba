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


def attention_tiles(seg_rows, masks: torch.Tensor) -> torch.Tensor:
    """The tile table (ovb_attention_tiles) of a segment list from its u8
    masks (1 = attend), the segments' [r, r] masks concatenated into one
    contiguous uint8 CUDA tensor.  Returns the device table (uint8)."""
    seg_rows = [int(r) for r in seg_rows]
    if not masks.is_cuda or masks.dtype != torch.uint8 or not masks.is_contiguous():
        raise ValueError("masks must be a contiguous uint8 CUDA tensor")
    if masks.numel() < sum(r * r for r in seg_rows):
        raise ValueError("masks holds fewer than sum(rows^2) entries")
    rows = (C.c_int32 * max(1, len(seg_rows)))(*seg_rows)
    nbytes = int(L.lib().ovb_attention_tiles_bytes(C.cast(rows, C.c_void_p), len(seg_rows)))
    tiles = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=masks.device)
    L.check(L.lib().ovb_attention_tiles(C.cast(rows, C.c_void_p), len(seg_rows), masks.data_ptr(),
                                        tiles.data_ptr(), tiles.numel(),
                                        torch.cuda.current_stream().cuda_stream))
    return tiles


def attention_h(q16: torch.Tensor, k16: torch.Tensor, v16: torch.Tensor, segs, n_heads: int,
                n_kv: int, scale: float, out: torch.Tensor | None = None,
                tiles: torch.Tensor | None = None) -> torch.Tensor:
    """ovb_attention_h: the same attention on fp16 q [T, n_heads * 128] and
    k / v [T', n_kv * 128] (contiguous CUDA tensors).  segs as for
    `attention` (biases ignored when `tiles`, from attention_tiles over the
    same segments, is given).  Returns fp32 out shaped like q."""
    for name, t in (("q", q16), ("k", k16), ("v", v16)):
        if not t.is_cuda or t.dtype != torch.float16 or t.dim() != 2 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 2-D float16 CUDA tensor")
    if k16.shape != v16.shape:
        raise ValueError("k and v must have the same shape")
    if q16.shape[1] != n_heads * HEAD_DIM or k16.shape[1] != n_kv * HEAD_DIM:
        raise ValueError("q / k widths must be n_heads * 128 / n_kv * 128")
    if out is None:
        out = torch.zeros(q16.shape, dtype=torch.float32, device=q16.device)
    segs = list(segs)
    arr = (L.AttnSegment * max(1, len(segs)))()
    keep = []
    for i, (bias, rows, q_off, kv_off) in enumerate(segs):
        if q_off + rows * q16.shape[1] > q16.numel() or kv_off + rows * k16.shape[1] > k16.numel():
            raise ValueError("segment runs past the end of q / k")
        bp = None
        if bias is not None and tiles is None:
            if (not bias.is_cuda or bias.dtype != torch.float32 or not bias.is_contiguous()
                    or bias.numel() != rows * rows):
                raise ValueError("bias must be a contiguous float32 CUDA tensor of rows * rows")
            keep.append(bias)
            bp = bias.data_ptr()
        arr[i] = L.AttnSegment(bp, int(rows), int(q_off), int(kv_off))
    L.check(L.lib().ovb_attention_h(q16.data_ptr(), k16.data_ptr(), v16.data_ptr(),
                                    out.data_ptr(), q16.shape[1], k16.shape[1], n_heads, n_kv,
                                    HEAD_DIM, float(scale),
                                    C.cast(arr, C.POINTER(L.AttnSegment)), len(segs),
                                    None if tiles is None else tiles.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream))
    return out


def attention_h_q(q16: torch.Tensor, k16: torch.Tensor, v16: torch.Tensor, segs, n_heads: int,
                  n_kv: int, scale: float, tiles: torch.Tensor | None = None, u8: bool = False,
                  f16: bool = False):
    """ovb_attention_h_q: attention_h with ovb_quantize of its output fused
    into the epilogue.  Returns (aq, asc) in the form the flags select (int8
    q, u8 q+128 or fp16 q*asc) for the q rows [T, n_heads * 128]."""
    from .gemm import empty_quant, empty_quant_f16
    T, QD = q16.shape
    if f16:
        aq, asc = empty_quant_f16(T, QD, q16.device)
    else:
        aq, asc = empty_quant(T, QD, q16.device)
        if u8:
            aq = aq.view(torch.uint8)
    segs = list(segs)
    arr = (L.AttnSegment * max(1, len(segs)))()
    keep = []
    for i, (bias, rows, q_off, kv_off) in enumerate(segs):
        bp = None
        if bias is not None and tiles is None:
            keep.append(bias)
            bp = bias.data_ptr()
        arr[i] = L.AttnSegment(bp, int(rows), int(q_off), int(kv_off))
    flags = (L.OVB_AQ_U8 if u8 else 0) | (L.OVB_AQ_F16 if f16 else 0)
    L.check(L.lib().ovb_attention_h_q(q16.data_ptr(), k16.data_ptr(), v16.data_ptr(), QD,
                                      k16.shape[1], n_heads, n_kv, HEAD_DIM, float(scale),
                                      C.cast(arr, C.POINTER(L.AttnSegment)), len(segs),
                                      None if tiles is None else tiles.data_ptr(), aq.data_ptr(),
                                      asc.data_ptr(), flags,
                                      torch.cuda.current_stream().cuda_stream))
    return aq, asc


def rope_table(pos: torch.Tensor, theta: float = 1e6) -> torch.Tensor:
    """The RoPE table of int64 positions ``pos`` [rows] (ovb_rope_table):
    [rows, 32, 2, 2] fp32, ``tab[r, j, 0, u]`` = cos and ``tab[r, j, 1, u]``
    = sin of angle i = 2j + u, pos * inv_freq[i], inv_freq[i] =
    theta^(-2i/128) rounded to fp32 (qk_norm_rope_f32's table,
    ops_cpu.cpp:945-986)."""
    if not pos.is_cuda or pos.dtype != torch.int64 or not pos.is_contiguous():
        raise ValueError("pos must be a contiguous int64 CUDA tensor")
    tab = torch.empty((pos.numel(), 32, 2, 2), dtype=torch.float32, device=pos.device)
    L.check(L.lib().ovb_rope_table(pos.data_ptr(), pos.numel(), HEAD_DIM, float(theta),
                                   tab.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return tab


def qk_norm_rope_f16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_norm: torch.Tensor,
                     k_norm: torch.Tensor, eps: float, table: torch.Tensor):
    """Per-head q / k RMSNorm + RoPE into fp16, v converted to fp16
    (ovb_qk_norm_rope_f16): q [rows, n_heads*128], k / v [rows, n_kv*128]
    contiguous fp32; returns (q16, k16, v16), the operands of attention_h."""
    for name, t in (("q", q), ("k", k), ("v", v), ("q_norm", q_norm), ("k_norm", k_norm),
                    ("table", table)):
        if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous float32 CUDA tensor")
    rows = q.shape[0]
    if table.numel() < rows * HEAD_DIM:
        raise ValueError("table must hold 128 floats per row (rope_table)")
    n_heads, n_kv = q.shape[1] // HEAD_DIM, k.shape[1] // HEAD_DIM
    q16 = torch.empty(q.shape, dtype=torch.float16, device=q.device)
    k16 = torch.empty(k.shape, dtype=torch.float16, device=q.device)
    v16 = torch.empty(v.shape, dtype=torch.float16, device=q.device)
    L.check(L.lib().ovb_qk_norm_rope_f16(rows, q.data_ptr(), k.data_ptr(), v.data_ptr(), n_heads,
                                         n_kv, HEAD_DIM, q_norm.data_ptr(), k_norm.data_ptr(),
                                         float(eps), table.data_ptr(), q16.data_ptr(),
                                         k16.data_ptr(), v16.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream))
    return q16, k16, v16
