"""Utterance-parallel sharding of the LM work across GPUs (one process per GPU).

The reference runs one utterance at a time on one device (cuda_lm.cu:793-798)
and has no distributed code.  Utterances are independent, so the B200 build
scales by data parallelism with no collective on the data path: each rank
owns whole CFG pairs -- the conditional and unconditional rows of one
utterance stay together (ragged CFG packing, tts.cpp:205-231) -- and every
rank holds a full copy of the int8 weights.

Assignment is longest-processing-time first: utterances sorted by estimated
cost, each given to the currently least-loaded rank (ties to the lowest rank),
which is deterministic, so every rank computes the same plan without talking.
If a rank fails, `requeue` moves its unfinished utterances to the survivors
by the same rule.
"""
from __future__ import annotations

import numpy as np

HIDDEN = 1024
N_LAYERS = 28
LINEAR_OPS_PER_TOKEN = 2 * 15_728_640  # 2 * sum(N*K) of one layer's seven projections
N_HEADS, HEAD_DIM = 16, 128


def cfg_rows(length: int) -> int:
    """Rows one utterance contributes to a step: its CFG pair, M = 2 * len."""
    return 2 * int(length)


def utterance_cost(length: int) -> float:
    """Work of one forward over an utterance's CFG pair: the linear layers
    (linear in rows) plus attention scores and context (quadratic in rows)."""
    m = cfg_rows(length)
    linear = m * LINEAR_OPS_PER_TOKEN * N_LAYERS
    attention = 4.0 * N_HEADS * HEAD_DIM * m * m * N_LAYERS
    return float(linear + attention)


def synthetic_utterances(n: int = 64, lo: int = 150, hi: int = 800, seed: int = 0) -> np.ndarray:
    """n utterance lengths uniform in [lo, hi] tokens."""
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n)


def lpt_assign(lengths, world: int, loads=None, ids=None) -> list[list[int]]:
    """Assign utterance ids to `world` ranks, longest-processing-time first."""
    if world <= 0:
        raise ValueError("world must be positive")
    lengths = list(int(x) for x in lengths)
    ids = list(range(len(lengths))) if ids is None else list(ids)
    loads = [0.0] * world if loads is None else list(loads)
    order = sorted(range(len(ids)), key=lambda i: (-utterance_cost(lengths[i]), ids[i]))
    plan: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        plan[r].append(ids[i])
        loads[r] += utterance_cost(lengths[i])
    return plan


def shard_for_rank(lengths, rank: int, world: int) -> list[int]:
    return lpt_assign(lengths, world)[rank]


def plan_loads(lengths, plan) -> list[float]:
    return [sum(utterance_cost(lengths[i]) for i in ids) for ids in plan]


def requeue(lengths, plan, dead: set[int], done: set[int]) -> list[list[int]]:
    """Move the unfinished utterances of failed ranks onto the live ranks.

    Live ranks keep what they have; the orphans are spread by LPT on top of
    the live ranks' current loads.  Failed ranks end with empty lists."""
    world = len(plan)
    live = [r for r in range(world) if r not in dead]
    if not live:
        raise RuntimeError("no live rank left")
    orphans = [i for r in dead for i in plan[r] if i not in done]
    new = [list(plan[r]) if r not in dead else [] for r in range(world)]
    loads = [plan_loads(lengths, [new[r]])[0] for r in live]
    extra = lpt_assign([lengths[i] for i in orphans], len(live), loads=loads, ids=orphans)
    for k, r in enumerate(live):
        new[r].extend(extra[k])
    return new
