"""The tensor-parallel exchange's slot-reuse argument, checked on the CPU.

Each rank's exchange region holds, per slot parity, one slot per sender; an
exchange k (epoch e_k) writes this rank's partial into every peer's slot of
parity k & 1, then waits until its own slots of that parity carry e_k from every
peer and reads them.  Two parities suffice because a rank cannot start exchange
k + 2 (and overwrite parity k & 1) before finishing k + 1, which needs every
peer's k + 1 data, which a peer sends only after finishing its exchange k.

This model runs N ranks as interleaved state machines under random schedules
and asserts that every read sees the data of its own exchange -- never a
later exchange's overwrite, never an earlier one's leftovers -- and that no
schedule deadlocks.
"""
from __future__ import annotations

import random

import pytest


def _epoch(step: int, instance: int) -> int:
    return (step << 9) + instance + 1


def run(nranks: int, steps: int, per_step: int, seed: int) -> int:
    rng = random.Random(seed)
    # slots[owner][parity][sender] = (epoch, value)
    slots = [[[(0, None)] * nranks for _ in range(2)] for _ in range(nranks)]
    # per rank: index of the current exchange and its phase ("send" or "wait")
    k = [0] * nranks
    phase = ["send"] * nranks
    total = steps * per_step
    reads = 0
    while any(x < total for x in k):
        r = rng.choice([i for i in range(nranks) if k[i] < total])
        step, inst = divmod(k[r], per_step)
        e, par = _epoch(step, inst), inst & 1
        if phase[r] == "send":
            # the kernel's stores land in the peers' regions one by one, in any order
            for j in rng.sample(range(nranks), nranks):
                if j != r:
                    slots[j][par][r] = (e, (k[r], r))
            phase[r] = "wait"
        else:
            if all(slots[r][par][j][0] == e for j in range(nranks) if j != r):
                for j in range(nranks):
                    if j != r:
                        assert slots[r][par][j][1] == (k[r], j), (r, j, k[r], slots[r][par][j])
                        reads += 1
                k[r] += 1
                phase[r] = "send"
            # else: keep polling (another rank gets scheduled)
    return reads


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_two_parities_never_lose_or_mix_a_partial(nranks):
    per_step = 8  # two exchanges per layer, four layers
    for seed in range(40):
        reads = run(nranks, steps=3, per_step=per_step, seed=seed)
        assert reads == nranks * (nranks - 1) * 3 * per_step


def test_one_slot_parity_would_not_be_enough():
    """With a single parity the same schedules lose data: a fast rank's next
    exchange overwrites a slot a slow peer has not read yet."""
    def run_one_parity(nranks, seed):
        rng = random.Random(seed)
        slots = [[(0, None)] * nranks for _ in range(nranks)]
        k, phase = [0] * nranks, ["send"] * nranks
        total = 16
        while any(x < total for x in k):
            r = rng.choice([i for i in range(nranks) if k[i] < total])
            e = k[r] + 1
            if phase[r] == "send":
                for j in range(nranks):
                    if j != r:
                        slots[j][r] = (e, (k[r], r))
                phase[r] = "wait"
            elif all(slots[r][j][0] >= e for j in range(nranks) if j != r):
                if any(slots[r][j][1] != (k[r], j) for j in range(nranks) if j != r):
                    return False
                k[r] += 1
                phase[r] = "send"
        return True

    assert not all(run_one_parity(2, seed) for seed in range(200))
