"""A CPU model of the persistent kernel's weight ring (csrc/f5_mega.cu:
producer, c_gemv4096's two consumer groups): mbarrier parity waits under
random schedules, with copies that land in any order.

An mbarrier wait on parity P passes while the barrier's current phase has
the other parity, so a waiter that is two phases behind passes at once.
The ring is correct when every consumer that passes its wait on a stage
finds the chunk it waited for there.  The stage-index assignment of chunks
to the two groups (stage s -> group s % 2, the kernel's) is correct at every
ring depth; the chunk-parity assignment (chunk j -> group j % 2) is correct
only at an even depth, and the model finds the early read at depths 3 and
5 (the kernel met it when forced to 3 stages: wrong tokens from step 1)."""
import random

import pytest


class Bar:
    """Completed-phase counter of an mbarrier with one arrival per phase."""

    def __init__(self):
        self.done = 0

    def try_wait(self, parity):
        return (self.done & 1) != parity


def run(ns, n_chunks, assign, seed):
    """-> number of consumer waits that passed on a stage not yet holding
    their chunk, over one random schedule."""
    rng = random.Random(seed)
    full = [Bar() for _ in range(ns)]
    empty = [Bar() for _ in range(ns)]
    content = [None] * ns
    inflight = []          # (stage, chunk) copies issued, not landed
    issued = 0
    nxt = {0: 0, 1: 0}     # each group's position in its own chunk list
    mine = {g: [c for c in range(n_chunks) if assign(c, ns) == g] for g in (0, 1)}
    bad = 0
    while True:
        moves = []
        if issued < n_chunks:
            s, lap = issued % ns, issued // ns
            if lap == 0 or empty[s].try_wait((lap - 1) & 1):
                moves.append("issue")
        if inflight:
            moves.append("land")
        for g in (0, 1):
            if nxt[g] < len(mine[g]):
                c = mine[g][nxt[g]]
                # the consumer knows nothing of the producer's progress:
                # it has only the barrier (c may not even be issued yet)
                if full[c % ns].try_wait((c // ns) & 1):
                    moves.append(g)
        if not moves:
            break
        m = rng.choice(moves)
        if m == "issue":
            inflight.append((issued % ns, issued))
            issued += 1
        elif m == "land":
            s, c = inflight.pop(rng.randrange(len(inflight)))
            content[s] = c
            full[s].done += 1
        else:
            c = mine[m][nxt[m]]
            s = c % ns
            if content[s] != c:
                bad += 1
            else:
                empty[s].done += 1   # the group's arrivals complete the phase
            nxt[m] += 1
            if content[s] != c:
                break                # the run is already wrong
    return bad


def by_stage(c, ns):
    return (c % ns) & 1


def by_chunk(c, ns):
    return c & 1


@pytest.mark.parametrize("ns", [2, 3, 4, 5, 6])
def test_stage_index_groups_never_read_early(ns):
    assert sum(run(ns, 40, by_stage, seed) for seed in range(300)) == 0


def test_chunk_parity_groups_are_correct_only_at_even_depth():
    for ns in (2, 4, 6):
        assert sum(run(ns, 40, by_chunk, seed) for seed in range(300)) == 0
    for ns in (3, 5):
        assert sum(run(ns, 40, by_chunk, seed) for seed in range(300)) > 0
