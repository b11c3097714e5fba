"""OVW1 weight files: the reference's checkpoint format (docs/weight-format.en.md).

`OVW1File` maps a file through the C ABI (ovb_ovw1_*, the checks of
ov::WeightFile::Open, cpp/src/core/weight_file.cpp:124-206) and creates
device weights from its int8 linear tensors without a host repack
(`weight`, in place of make_linear, cpp/src/model/mat.cpp:69-106).

`write` produces a file in the same format from numpy arrays -- the role of
the reference's converter (tools/convert_weights.py) for synthetic
checkpoints: header, 64-byte descriptors, names, 64-byte aligned payloads,
per-output-channel fp32 scales, CRC32 of each payload.
"""
from __future__ import annotations

import ctypes as C
import struct
import zlib

import numpy as np
import torch

from . import _lib as L
from .gemm import Weight

MAGIC = b"OMNIVOIC"
DTYPES = {np.dtype(np.float32): 0, np.dtype(np.int8): 1, np.dtype(np.float16): 2,
          np.dtype(np.int64): 3}
NP_DTYPE = {v: k for k, v in DTYPES.items()}
HEADER_BYTES = 128
DESC_BYTES = 64


def _align(n: int, a: int = 64) -> int:
    return (n + a - 1) // a * a


def write(path: str, tensors: list, n_params: int | None = None, flags: int = 0) -> None:
    """tensors: (name, array, layout, scales or None) in file order.  layout 1
    marks a transposed linear weight ([K, N], one scale per column), 0 a
    row-major tensor ([N, K] int8: one scale per row).  A tensor with scales
    is recorded as quant = 1 (per-output-channel int8)."""
    names = b""
    entries = []
    for name, arr, layout, scales in tensors:
        a = np.asarray(arr, order="C")  # keeps 0-d tensors 0-d
        nb = name.encode()
        entries.append((len(names), len(nb), a, layout, scales))
        names += nb + b"\0"
    n = len(entries)
    index_off = HEADER_BYTES
    names_off = index_off + n * DESC_BYTES
    data_off = _align(names_off + len(names))
    off = data_off
    placed = []
    for name_off, name_len, a, layout, scales in entries:
        d_off = off
        off = _align(off + a.nbytes)
        a_off = 0
        if scales is not None:
            a_off = off
            off = _align(off + 4 * len(scales))
        placed.append((name_off, name_len, a, layout, scales, d_off, a_off))
    size = off
    buf = bytearray(size)
    has_i8 = any(e[2].dtype == np.int8 for e in entries)
    struct.pack_into("<8sIIIIQQQQQQ", buf, 0, MAGIC, 1, 1 if has_i8 else 0, n, HEADER_BYTES,
                     index_off, names_off, data_off, size, flags,
                     n_params if n_params is not None else sum(e[2].size for e in entries))
    buf[names_off:names_off + len(names)] = names
    for i, (name_off, name_len, a, layout, scales, d_off, a_off) in enumerate(placed):
        dims = list(a.shape) + [0] * (4 - a.ndim)
        raw = a.tobytes()
        struct.pack_into("<IIBBBB4IIQQQQ", buf, index_off + i * DESC_BYTES, name_off, name_len,
                         DTYPES[a.dtype], a.ndim, layout, 1 if scales is not None else 0, *dims,
                         0 if scales is None else len(scales), zlib.crc32(raw), d_off, len(raw),
                         a_off)
        buf[d_off:d_off + len(raw)] = raw
        if scales is not None:
            s = np.ascontiguousarray(scales, dtype=np.float32).tobytes()
            buf[a_off:a_off + len(s)] = s
    with open(path, "wb") as f:
        f.write(buf)


class OVW1File:
    """A mapped OVW1 file (ovb_ovw1_open); close() or the context manager
    unmaps it.  Tensor views (`array`) point into the mapping."""

    def __init__(self, path: str):
        h = C.c_void_p()
        L.check(L.lib().ovb_ovw1_open(path.encode(), C.byref(h)))
        self._h = h.value

    def close(self):
        if self._h:
            L.lib().ovb_ovw1_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return int(L.lib().ovb_ovw1_count(self._h))

    def header(self) -> dict:
        m, f, p = C.c_uint32(), C.c_uint64(), C.c_uint64()
        L.check(L.lib().ovb_ovw1_header(self._h, C.byref(m), C.byref(f), C.byref(p)))
        return {"dtype_mode": m.value, "flags": f.value, "n_params": p.value}

    def info(self, key) -> L.Ovw1Tensor:
        t = L.Ovw1Tensor()
        if isinstance(key, int):
            L.check(L.lib().ovb_ovw1_tensor_at(self._h, key, C.byref(t)))
        else:
            L.check(L.lib().ovb_ovw1_find(self._h, key.encode(), C.byref(t)))
        return t

    def names(self) -> list[str]:
        return [self.info(i).name.decode() for i in range(len(self))]

    def array(self, name: str) -> np.ndarray:
        """A read-only numpy view of the payload (valid while the file is open)."""
        t = self.info(name)
        shape = tuple(t.dims[k] for k in range(t.ndim))
        dt = NP_DTYPE[t.dtype]
        buf = (C.c_char * t.nbytes).from_address(t.data) if t.nbytes else b""
        a = np.frombuffer(buf, dtype=dt, count=int(np.prod(shape)) if shape else 1)
        return a.reshape(shape)

    def scales(self, name: str) -> np.ndarray | None:
        t = self.info(name)
        if not t.scales:
            return None
        return np.frombuffer((C.c_float * t.n_scales).from_address(t.scales), dtype=np.float32)

    def verify(self, name: str) -> bool:
        """ComputeCrc == StoredCrc (weight_file.cpp:220-224)."""
        c = C.c_uint32()
        L.check(L.lib().ovb_ovw1_crc(self._h, name.encode(), C.byref(c)))
        return c.value == self.info(name).crc

    def weights(self, names: list[str], f16: bool = False) -> list[Weight]:
        """Several int8 linear tensors at once (ovb_ovw1_weights: one device
        allocation, one synchronisation)."""
        n = len(names)
        arr = (C.c_char_p * max(n, 1))(*[x.encode() for x in names])
        out = (C.c_void_p * max(n, 1))()
        L.check(L.lib().ovb_ovw1_weights(self._h, arr, n, L.OVB_WEIGHT_F16 if f16 else 0,
                                         torch.cuda.current_stream().cuda_stream, out))
        ws = []
        for i, name in enumerate(names):
            t = self.info(name)
            N = t.dims[1] if t.layout == 1 else t.dims[0]
            K = t.dims[0] if t.layout == 1 else t.dims[1]
            ws.append(Weight(out[i], int(N), int(K), f16))
        return ws

    def weight(self, name: str, f16: bool = False) -> Weight:
        """The int8 linear tensor `name` as a device weight (either layout)."""
        t = self.info(name)
        out = C.c_void_p()
        L.check(L.lib().ovb_ovw1_weight(self._h, name.encode(), L.OVB_WEIGHT_F16 if f16 else 0,
                                        torch.cuda.current_stream().cuda_stream, C.byref(out)))
        N = t.dims[1] if t.layout == 1 else t.dims[0]
        K = t.dims[0] if t.layout == 1 else t.dims[1]
        return Weight(out.value, int(N), int(K), f16)


def random_lm(path: str, n_layers: int, vocab: int = 4096, seed: int = 0, hidden: int = 1024,
              n_heads: int = 16, n_kv: int = 8, inter: int = 3072, audio_vocab: int = 1025,
              codebooks: int = 8, heads_f32: bool = False, layout: str = "nk") -> None:
    """A random-weight checkpoint of the reference LM's shape and tensor names
    (cpp/src/model/lm.cpp:96-141): int8 [N, K] linear weights with
    per-output-channel scales |N(0, 0.02)| / 127 (the --int8-layout nk
    encoding, audio heads int8 as well), int8 embedding tables with row
    scales, RMSNorm gains 1 + N(0, 0.05), codebook offsets c * audio_vocab.
    ``heads_f32`` stores the audio heads as the reference's converter does
    by default (tools/convert_weights.py:326-327: kept fp32, written
    transposed [K, N] with layout 1, :178-180), values N(0, 0.02).
    ``layout="kn"`` writes the same integer weights in the converter's
    default int8 encoding instead ([K, N], one scale per column, layout 1,
    :170-176) -- the only one the reference's CUDA runner reads."""
    if layout not in ("nk", "kn"):
        raise ValueError("layout must be 'nk' or 'kn'")
    rng = np.random.default_rng(seed)
    D = 128

    def lin(N, K):
        return (rng.integers(-127, 128, size=(N, K), dtype=np.int8),
                (np.abs(rng.standard_normal(N)) * 0.02 / 127 + 1e-6).astype(np.float32))

    def gain(n):
        return (1 + 0.05 * rng.standard_normal(n)).astype(np.float32)

    ts = []
    W, s = lin(vocab, hidden)
    ts.append(("llm.embed_tokens.weight", W, 0, (s * 40).astype(np.float32)))
    W, s = lin(codebooks * audio_vocab, hidden)
    ts.append(("audio_embeddings.weight", W, 0, (s * 40).astype(np.float32)))
    W, s = lin(codebooks * audio_vocab, hidden)
    if heads_f32:
        Wf = (rng.standard_normal((codebooks * audio_vocab, hidden)) * 0.02).astype(np.float32)
        ts.append(("audio_heads.weight", np.ascontiguousarray(Wf.T), 1, None))
    elif layout == "kn":
        ts.append(("audio_heads.weight", np.ascontiguousarray(W.T), 1, s))
    else:
        ts.append(("audio_heads.weight", W, 0, s))
    ts.append(("llm.norm.weight", gain(hidden), 0, None))
    ts.append(("codebook_layer_offsets",
               (np.arange(codebooks, dtype=np.int64) * audio_vocab), 0, None))
    QD, KVD = n_heads * D, n_kv * D
    for i in range(n_layers):
        p = f"llm.layers.{i}."
        ts.append((p + "input_layernorm.weight", gain(hidden), 0, None))
        ts.append((p + "post_attention_layernorm.weight", gain(hidden), 0, None))
        ts.append((p + "self_attn.q_norm.weight", gain(D), 0, None))
        ts.append((p + "self_attn.k_norm.weight", gain(D), 0, None))
        for name, N, K in (("self_attn.q_proj", QD, hidden), ("self_attn.k_proj", KVD, hidden),
                           ("self_attn.v_proj", KVD, hidden), ("self_attn.o_proj", hidden, QD),
                           ("mlp.gate_proj", inter, hidden), ("mlp.up_proj", inter, hidden),
                           ("mlp.down_proj", hidden, inter)):
            W, s = lin(N, K)
            if layout == "kn":
                ts.append((p + name + ".weight", np.ascontiguousarray(W.T), 1, s))
            else:
                ts.append((p + name + ".weight", W, 0, s))
    write(path, ts)
