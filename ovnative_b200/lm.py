"""The whole LM forward on the device (ovb_lm_*), built from an OVW1 file.

Mirrors the reference's LM (cpp/src/model/lm.h:52-140): `forward_cfg` is
LM::forward_cfg (lm.cpp:403-454, the ragged CFG pair), `forward` is
LM::forward (lm.cpp:343-401, the CudaForwardFn hook's arguments).  Inputs and
logits are host numpy arrays, as the hook passes them; `forward_cfg_device`
takes torch CUDA tensors and leaves the logits on the device.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


class LM:
    def __init__(self, path: str, f16: bool = False):
        h = C.c_void_p()
        L.check(L.lib().ovb_lm_create(path.encode(), L.OVB_WEIGHT_F16 if f16 else 0,
                                      torch.cuda.current_stream().cuda_stream, C.byref(h)))
        self._h = h.value
        cfg = (C.c_int64 * 9)()
        L.check(L.lib().ovb_lm_config(self._h, cfg))
        keys = ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "inter", "vocab",
                "audio_vocab", "n_codebooks")
        self.config = dict(zip(keys, (int(x) for x in cfg)))
        self.C, self.V = self.config["n_codebooks"], self.config["audio_vocab"]

    def close(self):
        if self._h:
            L.lib().ovb_lm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_cfg(self, ids, amask, cond_attn, uncond_attn, pos) -> np.ndarray:
        """ids [C, rows] int64 (rows = cond + uncond, codebook-major), amask
        [rows] u8, cond_attn [cs, cs] u8, uncond_attn [us, us] u8, pos [rows]
        int64 -> logits [rows, C*V] fp32."""
        ids = np.ascontiguousarray(ids, np.int64)
        a = np.ascontiguousarray(amask, np.uint8)
        cm = np.ascontiguousarray(cond_attn, np.uint8)
        um = np.ascontiguousarray(uncond_attn, np.uint8)
        pos = np.ascontiguousarray(pos, np.int64)
        rows = ids.shape[1]
        out = np.empty((rows, self.C * self.V), np.float32)
        L.check(L.lib().ovb_lm_forward_cfg(self._h, cm.shape[0], um.shape[0], _p(ids), _p(a),
                                           _p(cm), _p(um), _p(pos), _p(out),
                                           torch.cuda.current_stream().cuda_stream))
        return out

    def forward_cfg_sample(self, ids, amask, cond_attn, uncond_attn, pos, target_len: int,
                           guidance: float = 2.0, layer_penalty: float = 5.0,
                           mask_id: int = 1024):
        """One TTS step the way the reference's CUDA path runs it (device
        sampling, tts.cpp:270-282): LM::forward_cfg on host inputs with the
        logits kept on the device, then the guided sampler on its two CFG
        planes (cond at its last target_len rows, uncond at its first),
        returning host (pred int32 [C, T], scores fp32 [C, T])."""
        ids = np.ascontiguousarray(ids, np.int64)
        a = np.ascontiguousarray(amask, np.uint8)
        cm = np.ascontiguousarray(cond_attn, np.uint8)
        um = np.ascontiguousarray(uncond_attn, np.uint8)
        pos = np.ascontiguousarray(pos, np.int64)
        cs, us = cm.shape[0], um.shape[0]
        stream = torch.cuda.current_stream().cuda_stream
        L.check(L.lib().ovb_lm_forward_cfg(self._h, cs, us, _p(ids), _p(a), _p(cm), _p(um), _p(pos),
                                           None, stream))
        base = L.lib().ovb_lm_logits(self._h)
        pred = np.empty((self.C, target_len), np.int32)
        scores = np.empty((self.C, target_len), np.float32)
        L.check(L.lib().ovb_lm_sample(self._h, base, cs, base + cs * self.C * self.V * 4, us,
                                      target_len, guidance, layer_penalty, mask_id, _p(pred),
                                      _p(scores), stream))
        return pred, scores

    def forward(self, ids, amask, attn, pos) -> np.ndarray:
        """ids [B, C, S], amask [B, S], attn [B, S, S], pos [B, S] -> logits
        [B, C, S, V]."""
        ids = np.ascontiguousarray(ids, np.int64)
        B, _, S = ids.shape
        a = np.ascontiguousarray(amask, np.uint8)
        m = np.ascontiguousarray(attn, np.uint8)
        pos = np.ascontiguousarray(pos, np.int64)
        out = np.empty((B, self.C, S, self.V), np.float32)
        L.check(L.lib().ovb_lm_forward(self._h, B, S, _p(ids), _p(a), _p(m), _p(pos), _p(out),
                                       torch.cuda.current_stream().cuda_stream))
        return out

    def reserve(self, rows: int, mask_elems: int):
        L.check(L.lib().ovb_lm_reserve(self._h, rows, mask_elems))

    def forward_cfg_device(self, ids, amask, cond_attn, uncond_attn, pos) -> torch.Tensor:
        """The same on CUDA tensors, stream-ordered; returns a view of the
        model's device logits [rows, C*V] (valid until the next forward)."""
        cs, us = cond_attn.shape[0], uncond_attn.shape[0]
        L.check(L.lib().ovb_lm_forward_cfg_device(
            self._h, cs, us, ids.data_ptr(), amask.data_ptr(), cond_attn.data_ptr(),
            uncond_attn.data_ptr(), pos.data_ptr(), torch.cuda.current_stream().cuda_stream))
        return _device_view(L.lib().ovb_lm_logits(self._h), cs + us, self.C * self.V)


    def forward_segments_device(self, seg_rows, ids, amask, masks, pos) -> torch.Tensor:
        """Several attention segments (e.g. the CFG pairs of several
        utterances) in one forward on CUDA tensors, stream-ordered:
        seg_rows a list of row counts, ids [C, rows] int64, amask [rows] u8,
        masks the segments' [r, r] u8 masks concatenated (1-D), pos [rows]
        int64.  Returns a view of the device logits [rows, C*V] (valid until
        the next forward)."""
        n = len(seg_rows)
        arr = (C.c_int32 * max(n, 1))(*[int(r) for r in seg_rows])
        L.check(L.lib().ovb_lm_forward_segments_device(
            self._h, n, C.cast(arr, C.c_void_p), ids.data_ptr(), amask.data_ptr(),
            masks.data_ptr(), pos.data_ptr(), torch.cuda.current_stream().cuda_stream))
        return _device_view(L.lib().ovb_lm_logits(self._h), int(sum(seg_rows)), self.C * self.V)


def _device_view(ptr: int, rows: int, cols: int) -> torch.Tensor:
    """A torch view of `rows x cols` fp32 device memory at `ptr` (no copy)."""
    class _Mem:
        __cuda_array_interface__ = {"shape": (rows, cols), "typestr": "<f4",
                                    "data": (ptr, False), "version": 3, "strides": None}
    return torch.as_tensor(_Mem(), device="cuda")
