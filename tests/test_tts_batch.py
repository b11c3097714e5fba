"""Host logic of the batched TTS steps (ovnative_b200.tts_batch): the CFG
inputs follow the reference's CUDA-path construction (cpp/src/model/
tts.cpp:142-204) and the packing puts every utterance in exactly one forward
within its row and pair limits."""
from __future__ import annotations

import numpy as np
import pytest

from ovnative_b200 import shard
from ovnative_b200 import tts_batch as TB


def test_cfg_pair_inputs_follow_the_reference_layout():
    rng = np.random.default_rng(0)
    S, C = 90, 8
    T = TB.target_len(S)
    assert T == S - TB.N_TEXT
    ids, amask, cond, unc, pos = TB.cfg_pair_inputs(rng, S, C)
    assert ids.shape == (C, 2 * S) and amask.shape == (2 * S,) and pos.shape == (2 * S,)
    # prompt (build_prompt, tts.cpp:150-160): text ids in every codebook row,
    # then masked target frames, audio_mask 1 on the frames
    assert (ids[:, :S - T] == ids[0, :S - T]).all() and (ids[:, :S - T] < TB.TEXT_VOCAB).all()
    assert (ids[:, S - T:S] == TB.MASK_ID).all()
    assert (amask[:S - T] == 0).all() and (amask[S - T:S] == 1).all()
    # uncond row (tts.cpp:186-198): the target slice first, mask ids after it,
    # audio_mask 1 on the slice only; full attention inside the slice and the
    # diagonal for the unused tail
    assert (ids[:, S:S + T] == ids[:, S - T:S]).all() and (ids[:, S + T:] == TB.MASK_ID).all()
    assert (amask[S:S + T] == 1).all() and (amask[S + T:] == 0).all()
    assert cond.all()
    assert unc[:T, :T].all() and not unc[:T, T:].any()
    tail = unc[T:]
    assert (tail.sum(1) == 1).all() and all(tail[i, T + i] for i in range(S - T))
    # positions 0..S-1 in both rows (tts.cpp:200-202)
    assert (pos[:S] == np.arange(S)).all() and (pos[S:] == np.arange(S)).all()


@pytest.mark.parametrize("world", [1, 2, 8])
def test_pack_batches_covers_every_utterance_within_limits(world):
    lengths = dict(enumerate(shard.synthetic_utterances()))
    plan = shard.lpt_assign([lengths[i] for i in range(64)], world)
    for rank in range(world):
        uids = plan[rank]
        groups = TB.pack_batches(lengths, uids, max_rows=16384)
        flat = sorted(u for g in groups for u in g)
        assert flat == sorted(uids)
        rows = [sum(2 * lengths[u] for u in g) for g in groups]
        assert max(rows) <= 16384 and all(len(g) <= 32 for g in groups)
        # no more batches than needed, and the batches are about equal
        assert len(groups) <= -(-sum(rows) // 16384) + 1
        if len(groups) > 1:
            assert max(rows) - min(rows) <= 2 * 800
        assert groups == TB.pack_batches(lengths, uids, max_rows=16384)  # deterministic


def test_pack_batches_limits():
    lengths = {0: 900, 1: 10}
    with pytest.raises(ValueError):
        TB.pack_batches(lengths, [0, 1], max_rows=1000)
    many = {i: 10 for i in range(70)}
    groups = TB.pack_batches(many, list(many), max_rows=1 << 20, max_pairs=32)
    assert len(groups) == 3 and all(len(g) <= 32 for g in groups)
