"""Model check of the peer-memory gather protocol (xq4_linear_sharded_fused
and the chain's sharded ops), on CPU.

Each rank's k-th collective call has epoch e = k + 1.  The call stores each of
its values into every peer's inbox half e % 2 as a (value, epoch) word, then
waits until every word it needs from each peer in its own half e % 2
carries epoch e, copies them, and ends.  The claim the design rests on: two
halves suffice, because a rank cannot start call k + 2 before every peer has
finished reading call k (call k + 1 ends only after the peers' words of call
k + 1 arrived, which they send only after finishing call k).  The model runs
the protocol step by step under random interleavings and random per-rank
delays, and checks that every word read belongs to the same call of the same
peer, and that every rank finishes every call (no deadlock).
"""
import random

import pytest


def _run(nranks, calls, slots, seed):
    rng = random.Random(seed)
    inbox = [dict() for _ in range(nranks)]  # rank -> {(half, peer, slot): (value, epoch)}
    state = [{"call": 0, "sent": 0, "read": 0} for _ in range(nranks)]

    def value(rank, call, slot):
        return (rank, call, slot)

    def step(r):
        """One atomic step of rank r; False if it cannot progress now."""
        st = state[r]
        if st["call"] >= calls:
            return False
        e = st["call"] + 1
        half = e % 2
        if st["sent"] < (nranks - 1) * slots:  # send the next word to the next peer
            i = st["sent"]
            q = [p for p in range(nranks) if p != r][i // slots]
            s = i % slots
            inbox[q][(half, r, s)] = (value(r, st["call"], s), e)
            st["sent"] += 1
            return True
        if st["read"] < (nranks - 1) * slots:  # read the next word, if it has arrived
            i = st["read"]
            q = [p for p in range(nranks) if p != r][i // slots]
            s = i % slots
            word = inbox[r].get((half, q, s))
            if word is None or word[1] != e:
                return False  # not there yet: wait
            assert word[0] == value(q, st["call"], s), (r, e, q, s, word)
            st["read"] += 1
            return True
        st["call"] += 1  # the launch ends
        st["sent"] = st["read"] = 0
        return True

    stall = 0
    while any(st["call"] < calls for st in state):
        r = rng.randrange(nranks)
        if rng.random() < 0.3:  # this rank is slow right now
            continue
        if step(r):
            stall = 0
        else:
            stall += 1
            assert stall < 10000 * nranks, "no rank can progress"
    return state


@pytest.mark.parametrize("nranks", [2, 3, 4])
def test_inbox_protocol(nranks):
    for seed in range(40):
        state = _run(nranks, calls=7, slots=3, seed=seed)
        assert all(st["call"] == 7 for st in state)


def test_one_half_is_not_enough():
    """With a single half (every call writes the same slots) a fast rank
    overwrites words a slow peer has not read yet; the model detects it, so
    the two-half argument is what the protocol relies on."""
    def single_half_run(seed):
        rng = random.Random(seed)
        inbox = [dict(), dict()]
        state = [{"call": 0, "sent": False, "read": False} for _ in range(2)]
        while any(st["call"] < 6 for st in state):
            r = rng.randrange(2)
            st, q = state[r], 1 - r
            if st["call"] >= 6:
                continue
            e = st["call"] + 1
            if not st["sent"]:
                inbox[q]["w"] = (r, st["call"], e)
                st["sent"] = True
            elif not st["read"]:
                word = inbox[r].get("w")
                if word is None or word[2] < e:
                    continue
                if word[2] != e:  # a newer call's word: the one this call needed is gone
                    return False
                st["read"] = True
            else:
                st["call"] += 1
                st["sent"] = st["read"] = False
        return True
    assert not all(single_half_run(seed) for seed in range(200))
