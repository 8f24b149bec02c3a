"""Host model of the ranks' tagged-word exchange (``xchg_ll`` / ``ll_put`` / ``rank_reduce`` in
``csrc/nkm_qwen3_kernel.cuh``; the GPT-OSS kernel's ``put_part`` / ``rank_sum``).

Each exchange n of a kind has one word per (source rank, element) in every rank's region, in
slot n % 2, tagged n + 1. A rank stores its words of exchange n into every region, then waits
until its own region holds all ranks' words of exchange n with tag n + 1 and reads them. The
region is never cleared between exchanges. Two slots per kind are enough because a rank produces
exchange n + 2 only after reading every rank's exchange n + 1, and a rank produces exchange n + 1
only after reading exchange n.

The model runs the ranks' programs under random interleavings of single actions and checks:
* every read sees the value of its own exchange;
* no rank waits forever;
* launch sequences that run one kind alone (attention-only or MoE-only launches) keep both
  properties.

A planted mistake (one slot per kind) must be caught.
"""
import random

import pytest


def _run(world, program, slots, seed, elements=3):
    """Interleave the ranks' programs; returns None on success or a description of the fault."""
    rnd = random.Random(seed)
    region = [[[[0, 0] for _ in range(world * elements)] for _ in range(2 * slots)] for _ in range(world)]
    seq = {0: 0, 1: 0}

    def value(kind, n, src, e):
        return (kind, n, src, e)

    # per rank: list of exchanges (kind, n) in program order, and a cursor (exchange, phase, index)
    plans = []
    for r in range(world):
        counts = {0: 0, 1: 0}
        plan = []
        for kind in program:
            plan.append((kind, counts[kind]))
            counts[kind] += 1
        plans.append(plan)
    state = [[0, "put", 0] for _ in range(world)]  # exchange index, phase, element / destination cursor
    stalled = 0
    while any(s[0] < len(plans[r]) for r, s in enumerate(state)):
        r = rnd.randrange(world)
        s = state[r]
        if s[0] >= len(plans[r]):
            continue
        kind, n = plans[r][s[0]]
        slot = kind * slots + n % slots
        if s[1] == "put":  # one store: element s[2] % elements of this rank into region s[2] // elements
            q, e = divmod(s[2], elements)
            region[q][slot][r * elements + e] = [n + 1, value(kind, n, r, e)]
            s[2] += 1
            if s[2] == world * elements:
                s[1], s[2] = "get", 0
            stalled = 0
            continue
        # one load of its own region: word s[2] (source s[2] // elements)
        tag, v = region[r][slot][s[2]]
        if tag != n + 1:
            if tag > n + 1:
                return f"rank {r} exchange {(kind, n)}: slot already holds tag {tag}"
            stalled += 1
            if stalled > 200000:
                return "no rank can move"
            continue
        src, e = divmod(s[2], elements)
        if v != value(kind, n, src, e):
            return f"rank {r} read {v} in exchange {(kind, n)}"
        s[2] += 1
        stalled = 0
        if s[2] == world * elements:
            state[r] = [s[0] + 1, "put", 0]
    return None


def _programs():
    full = [0, 1] * 4                  # decode steps: O-projection then experts, per layer
    moe_only = [1] * 6                 # MoE-only launches back to back
    mixed = [0, 1, 0, 1, 1, 1, 0, 0, 1]  # launches with different stage subsets
    return {"full": full, "moe_only": moe_only, "mixed": mixed}


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("name", ["full", "moe_only", "mixed"])
def test_two_slots_per_kind_never_overwrite_unread_words(world, name):
    program = _programs()[name]
    for seed in range(30):
        fault = _run(world, program, slots=2, seed=seed)
        assert fault is None, (name, world, seed, fault)


def test_one_slot_per_kind_is_caught():
    """The model is not vacuous: with one slot a fast rank overwrites words a slow rank has not
    read yet, and some interleaving shows it."""
    faults = [_run(3, [1] * 6, slots=1, seed=seed) for seed in range(60)]
    assert any(f is not None for f in faults)
