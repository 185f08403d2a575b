"""The run-time tile claims of the single-column kernel (the producer's tile
source in qgemv_roofline_b200/csrc/gemv_tma.cu, k_gemv_tma), restated step by
step and run over random interleavings of the CTAs on the CPU.

The kernel relies on three facts that this model checks for many grid and
matrix sizes: every tile of the matrix is streamed exactly once, each CTA
makes exactly one failing claim (so the launch's last claim has the ticket
T - 2G + G - 1, counting only claimable tiles), and that claim leaves the
counter at zero with no claim after it -- so the next launch on the same
counter starts from zero."""

import random

import pytest


def run_launch(T, G, ctr, rng):
    """One launch of G CTAs over T tiles; returns (tiles streamed, counter)."""
    nclaims = max(0, T - 2 * G) + G
    state = {"ctr": ctr, "after_reset": False, "resets": 0}
    seen = []

    def atomic_add():
        assert not state["after_reset"], "a claim after the launch's last claim"
        v = state["ctr"]
        state["ctr"] += 1
        return v

    ctas = [{"b": b, "t": 0, "have": False, "claim": 0, "done": False} for b in range(G)]
    live = list(range(G))
    while live:
        c = ctas[rng.choice(live)]
        t = c["t"]
        k = c["b"] + t * G if t < 2 else T
        if k >= T:
            # claims start after the dependency wait, i.e. from step 1 on
            assert t >= 1
            tk = c["claim"] if c["have"] else atomic_add()
            c["have"] = False
            if tk == nclaims - 1:
                state["ctr"] = 0
                state["after_reset"] = True
                state["resets"] += 1
            k = 2 * G + tk
        if k < T:
            seen.append(k)
            if t >= 1:  # claim the next step's tile a step ahead
                c["claim"] = atomic_add()
                c["have"] = True
            c["t"] += 1
        else:
            c["done"] = True
            live.remove(c["b"])
    assert state["resets"] == 1
    return seen, state["ctr"]


@pytest.mark.parametrize("T,G", [(1, 1), (2, 1), (3, 2), (5, 3), (250, 148), (296, 148),
                                 (297, 148), (1024, 148), (6144, 148), (6144, 296),
                                 (513, 296)])
def test_every_tile_once_and_counter_reset(T, G):
    rng = random.Random(T * 1000 + G)
    ctr = 0
    for _ in range(3):  # consecutive launches on one counter
        seen, ctr = run_launch(T, G, ctr, rng)
        assert sorted(seen) == list(range(T))
        assert ctr == 0


def test_random_sizes():
    rng = random.Random(7)
    for _ in range(200):
        G = rng.randint(1, 300)
        T = rng.randint(G, 4000)
        seen, ctr = run_launch(T, G, 0, rng)
        assert sorted(seen) == list(range(T)) and ctr == 0
