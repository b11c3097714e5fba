"""TTS steps over many utterances on one GPU: the per-step device work of the
reference's sampling loop, with several utterances' CFG pairs packed into
each LM forward.

The reference synthesises one utterance at a time (Pipeline::run_sampling,
cpp/src/model/tts.cpp:165-364).  On its CUDA path every one of the 32
diffusion steps runs LM::forward over a B = 2 batch (tts.cpp:260-266) -- the
conditional row is the whole prompt of S tokens, the unconditional row holds
the target slice in its first T positions (tts.cpp:172-204) -- followed by
the guided argmax pass on the device (lm.h:106-108, tts.cpp:278-286).  Only
the ids change from step to step (tts.cpp:354-359).

Here each CFG pair is two attention segments of S rows, and the pairs of
several utterances are packed into one forward
(ovb_lm_forward_segments_device): rows attend only inside their own segment
and every other step works row by row, so each utterance gets exactly the
logits of its own forward, while the GEMMs see thousands of rows instead of
2 S.  The guided sampler then runs once per pair on that pair's planes.
One CUDA graph per batch holds the forward and the samplers.

`shard.lpt_assign` decides which utterances a GPU owns; `pack_batches`
groups them into forwards of at most `max_rows` rows.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import sampler as SP
from .lm import LM

MASK_ID = SP.MASK_ID   # kMaskId (tts.cpp:17)
N_TEXT = 40            # text ids per prompt
TEXT_VOCAB = 151000    # text ids drawn from [0, 151000)
GUIDANCE = 2.0         # TtsOptions::guidance_scale default (tts.h:28)
LAYER_PENALTY = 5.0    # TtsOptions::layer_penalty default (tts.h:30)
STEPS = 32             # TtsOptions::num_steps default (tts.h:27)


def target_len(S: int) -> int:
    """Target frames of a prompt of S tokens with N_TEXT text ids and no
    reference audio (build_prompt's layout, tts.cpp:142-160)."""
    return max(1, int(S) - N_TEXT)


def cfg_pair_inputs(rng: np.random.Generator, S: int, C: int = 8, text_vocab: int = TEXT_VOCAB):
    """The B = 2 CFG inputs of one utterance as run_sampling builds them for
    the CUDA path (tts.cpp:172-204), as two packed segments of S rows:
    ids [C, 2S] (codebook-major), audio_mask [2S], the two [S, S] masks and
    positions [2S].  The prompt (build_prompt, tts.cpp:142-160): N_TEXT text
    ids in every codebook row, then T = S - N_TEXT masked audio frames."""
    T = target_len(S)
    prompt = np.full((C, S), MASK_ID, np.int64)
    prompt[:, :S - T] = rng.integers(0, min(text_vocab, TEXT_VOCAB), size=S - T)
    amask_p = np.zeros(S, np.uint8)
    amask_p[S - T:] = 1
    ids = np.full((C, 2 * S), MASK_ID, np.int64)
    ids[:, :S] = prompt                         # cond row: the whole prompt
    ids[:, S:S + T] = prompt[:, S - T:]         # uncond row: the target slice first
    amask = np.zeros(2 * S, np.uint8)
    amask[:S] = amask_p
    amask[S:S + T] = 1
    cond = np.ones((S, S), np.uint8)
    unc = np.zeros((S, S), np.uint8)
    unc[:T, :T] = 1                             # full attention inside the target slice
    idx = np.arange(T, S)
    unc[idx, idx] = 1                           # the unused tail sees itself
    pos = np.concatenate([np.arange(S), np.arange(S)]).astype(np.int64)
    return ids, amask, cond, unc, pos


def pack_batches(lengths: dict, uids: list, max_rows: int, max_pairs: int = 32) -> list:
    """Group utterances into forwards of at most `max_rows` rows (2 S per
    utterance) and `max_pairs` CFG pairs (two attention segments each): the
    fewest batches that can hold them, filled longest first onto the
    least-loaded batch, so that the batches of one GPU are about equal."""
    rows = {u: 2 * int(lengths[u]) for u in uids}
    if any(r > max_rows for r in rows.values()):
        raise ValueError("an utterance is longer than max_rows")
    n = max(1, -(-sum(rows.values()) // max_rows), -(-len(uids) // max_pairs))
    while True:
        bins = [[] for _ in range(n)]
        load = [0] * n
        ok = True
        for u in sorted(uids, key=lambda u: (-rows[u], u)):
            cand = [b for b in range(n) if load[b] + rows[u] <= max_rows and len(bins[b]) < max_pairs]
            if not cand:
                ok = False
                break
            b = min(cand, key=lambda b: (load[b], b))
            bins[b].append(u)
            load[b] += rows[u]
        if ok:
            return [b for b in bins if b]
        n += 1


@dataclass
class _Pair:
    uid: int
    S: int
    T: int
    row0: int
    out0: int  # offset of this pair's C * T predictions in the batch's outputs


class Batch:
    """The device state of one packed forward: inputs, outputs, pinned host
    mirrors for the end-to-end path, and the CUDA graph."""

    def __init__(self, lm: LM, lengths: dict, uids: list, rng: np.random.Generator,
                 dev: torch.device):
        text_vocab = lm.config["vocab"]
        C = lm.C
        self.lm = lm
        self.pairs, parts, r0, o0 = [], [], 0, 0
        for u in uids:
            S = int(lengths[u])
            T = target_len(S)
            self.pairs.append(_Pair(u, S, T, r0, o0))
            parts.append(cfg_pair_inputs(rng, S, C, text_vocab))
            r0 += 2 * S
            o0 += C * T
        self.rows, self.n_out = r0, o0
        self.seg_rows = [r for p in self.pairs for r in (p.S, p.S)]
        self.mask_elems = int(sum(r * r for r in self.seg_rows))
        ids = np.concatenate([p[0] for p in parts], axis=1)
        amask = np.concatenate([p[1] for p in parts])
        masks = np.concatenate([m.reshape(-1) for p in parts for m in (p[2], p[3])])
        pos = np.concatenate([p[4] for p in parts])
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        self.ids, self.amask, self.masks, self.pos = to(ids), to(amask), to(masks), to(pos)
        self.pred = torch.empty(self.n_out, dtype=torch.int32, device=dev)
        self.scores = torch.empty(self.n_out, dtype=torch.float32, device=dev)
        self.h_ids = torch.from_numpy(ids).pin_memory()
        self.h_pred = torch.empty(self.n_out, dtype=torch.int32).pin_memory()
        self.h_scores = torch.empty(self.n_out, dtype=torch.float32).pin_memory()
        self.graph = None

    def run(self):
        """Enqueue the forward and the pairs' samplers (one launch for all the
        pairs, ovb_guided_sample_batch) on the current stream."""
        lm, C = self.lm, self.lm.C
        logits = lm.forward_segments_device(self.seg_rows, self.ids, self.amask, self.masks,
                                            self.pos)
        SP.guided_sample_batch([(logits[p.row0:p.row0 + p.S],
                                 logits[p.row0 + p.S:p.row0 + 2 * p.S], p.T) for p in self.pairs],
                               C, GUIDANCE, LAYER_PENALTY, self.pred, self.scores, MASK_ID)

    def capture(self, stream: torch.cuda.Stream):
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self.run()

    def h2d_bytes(self) -> int:
        return self.h_ids.numel() * self.h_ids.element_size()

    def d2h_bytes(self) -> int:
        return self.n_out * 8

    def release(self):
        if self.graph is not None:
            self.graph.reset()
            self.graph = None


class Stepper:
    """All of one GPU's utterances, packed into batches, stepped together.

    `step()` is one diffusion step of every utterance with inputs resident
    on the device (graph replays); `step_e2e()` is the same step as a serving
    loop drives it: every batch's ids copied in from pinned host memory, the
    graph, and the predictions and scores copied back, then a host
    synchronisation (the next step's ids depend on them, tts.cpp:329-359).

    With `extra_lms` (further LM instances on the same checkpoint, each with
    its own forward buffers) the batches are dealt round-robin to lanes, one
    per LM, and each lane replays its graphs on a stream of its own: two
    independent forwards then share the GPU, so that one's kernels fill the
    SMs another's leave idle (the last tiles of a persistent GEMM, a kernel's
    launch and ramp).  `stream` orders the step: the lanes start after the
    work already queued on it, and it waits for all lanes at the end."""

    def __init__(self, lm: LM, lengths: dict, uids: list, dev: torch.device,
                 stream: torch.cuda.Stream, max_rows: int = 16384, seed: int = 0,
                 extra_lms=()):
        rng = np.random.default_rng(seed)
        self.lm, self.stream = lm, stream
        self.lms = [lm, *extra_lms]
        self.streams = [stream] + [torch.cuda.Stream(device=dev) for _ in extra_lms]
        self.groups = pack_batches(lengths, uids, max_rows) if uids else []
        self.lane = [i % len(self.lms) for i in range(len(self.groups))]
        self.batches = [Batch(self.lms[k], lengths, g, rng, dev)
                        for k, g in zip(self.lane, self.groups)]
        for k, m in enumerate(self.lms):
            mine = [b for b, lk in zip(self.batches, self.lane) if lk == k]
            if mine:
                m.reserve(max(b.rows for b in mine), max(b.mask_elems for b in mine))
        self.rows_per_step = sum(b.rows for b in self.batches)
        self.samplers = sum(len(b.pairs) for b in self.batches)  # pairs sampled per step

    def _lanes(self):
        return [(self.streams[k], b) for k, b in zip(self.lane, self.batches)]

    def warm_and_capture(self):
        for s, b in self._lanes():  # eager first: kernel attributes are set outside capture
            with torch.cuda.stream(s):
                b.run()
        torch.cuda.synchronize()
        for s, b in self._lanes():
            b.capture(s)

    def _fork(self):
        for s in self.streams[1:]:
            s.wait_stream(self.stream)

    def _join(self):
        for s in self.streams[1:]:
            self.stream.wait_stream(s)

    def step(self):
        self._fork()
        for s, b in self._lanes():
            with torch.cuda.stream(s):
                b.graph.replay()
        self._join()

    def step_e2e(self):
        self._fork()
        for s, b in self._lanes():
            with torch.cuda.stream(s):
                b.ids.copy_(b.h_ids, non_blocking=True)
                b.graph.replay()
                b.h_pred.copy_(b.pred, non_blocking=True)
                b.h_scores.copy_(b.scores, non_blocking=True)
        self._join()
        self.stream.synchronize()

    def h2d_bytes_per_step(self) -> int:
        return sum(b.h2d_bytes() for b in self.batches)

    def d2h_bytes_per_step(self) -> int:
        return sum(b.d2h_bytes() for b in self.batches)

    def results(self) -> dict:
        """uid -> (pred [C, T], scores [C, T]) from the last device step."""
        out = {}
        C = self.lm.C
        for b in self.batches:
            pred, scores = b.pred.cpu().numpy(), b.scores.cpu().numpy()
            for p in b.pairs:
                n = C * p.T
                out[p.uid] = (pred[p.out0:p.out0 + n].reshape(C, p.T),
                              scores[p.out0:p.out0 + n].reshape(C, p.T))
        return out

    def release(self):
        for b in self.batches:
            b.release()
