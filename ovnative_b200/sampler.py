"""The guided (classifier-free guidance) argmax pass of a TTS step
(ovb_guided_sample) on torch CUDA tensors.

Mirrors the accelerator hook LM::CudaSampleFn (cpp/src/model/lm.h:106-108):
the reference's CPU loop cpp/src/model/tts.cpp:291-326 computes, for every
codebook c and target frame t,

    lp_c, lp_u = log_softmax(cond row), log_softmax(uncond row)
    mix = log_softmax(lp_c + g * (lp_c - lp_u))      (mix = lp_c if g == 0)
    mix[mask_id] = -inf; pred = argmax(mix); score = max(mix) - c * layer_penalty

with the cond row at token cond_seq - T + t and the uncond row at token t of
token-major [seq, C * V] logits planes.
"""
from __future__ import annotations

import torch

from . import _lib as L

MASK_ID = 1024  # the audio vocabulary's mask token (cpp/src/model/tts.cpp:17)


def guided_sample(cond: torch.Tensor, uncond: torch.Tensor, target_len: int, codebooks: int,
                  guidance: float, layer_penalty: float, mask_id: int = MASK_ID,
                  pred: torch.Tensor | None = None, scores: torch.Tensor | None = None):
    """cond [cond_seq, codebooks * V] and uncond [uncond_seq, codebooks * V],
    fp32 CUDA, rows contiguous.  Returns (pred int32, scores fp32), each
    [codebooks, target_len] (index c * target_len + t)."""
    for name, t in (("cond", cond), ("uncond", uncond)):
        if not t.is_cuda or t.dtype != torch.float32 or t.dim() != 2 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 2-D float32 CUDA tensor")
    if cond.shape[1] != uncond.shape[1] or cond.shape[1] % codebooks:
        raise ValueError("cond/uncond widths must both be codebooks * vocab")
    V = cond.shape[1] // codebooks
    if pred is None:
        pred = torch.empty((codebooks, target_len), dtype=torch.int32, device=cond.device)
    if scores is None:
        scores = torch.empty((codebooks, target_len), dtype=torch.float32, device=cond.device)
    L.check(L.lib().ovb_guided_sample(cond.data_ptr(), cond.shape[0], uncond.data_ptr(),
                                      uncond.shape[0], codebooks, V, target_len, float(guidance),
                                      float(layer_penalty), mask_id, pred.data_ptr(),
                                      scores.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return pred, scores


def guided_sample_batch(planes: list, codebooks: int, guidance: float, layer_penalty: float,
                        pred: torch.Tensor, scores: torch.Tensor, mask_id: int = MASK_ID):
    """guided_sample for several CFG pairs in one call (ovb_guided_sample_batch):
    planes = [(cond, uncond, target_len), ...] as for guided_sample; pair p's
    [codebooks, target_len] outputs follow pair p - 1's in the flat int32
    `pred` and float32 `scores`."""
    if not planes:
        return pred, scores
    pairs = (L.GuidedPair * len(planes))()
    V = None
    need = 0
    for i, (cond, uncond, T) in enumerate(planes):
        for name, t in (("cond", cond), ("uncond", uncond)):
            if not t.is_cuda or t.dtype != torch.float32 or t.dim() != 2 or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous 2-D float32 CUDA tensor")
        if cond.shape[1] != uncond.shape[1] or cond.shape[1] % codebooks:
            raise ValueError("cond/uncond widths must both be codebooks * vocab")
        if V is not None and cond.shape[1] // codebooks != V:
            raise ValueError("every pair needs the same vocabulary")
        V = cond.shape[1] // codebooks
        pairs[i] = L.GuidedPair(cond.data_ptr(), cond.shape[0], uncond.data_ptr(),
                                uncond.shape[0], int(T))
        need += codebooks * int(T)
    for name, t, dt in (("pred", pred, torch.int32), ("scores", scores, torch.float32)):
        if not t.is_cuda or t.dtype != dt or not t.is_contiguous() or t.numel() < need:
            raise ValueError(f"{name} must be a contiguous {dt} CUDA tensor of {need} values")
    L.check(L.lib().ovb_guided_sample_batch(len(planes), pairs, codebooks, V, float(guidance),
                                            float(layer_penalty), mask_id, pred.data_ptr(),
                                            scores.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))
    return pred, scores
