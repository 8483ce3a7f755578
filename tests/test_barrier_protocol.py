"""The decode kernel's grid barrier (grid_barrier in shardserve_b200/csrc/decode_attention.cu),
restated step for step as a model of its atomic operations on the one 64-bit counter, and run
under many random interleavings: CTAs held back as if not resident (placed only after the
others have left or at a random later point), waiters that give up after a random number of
polls, and the counter started just below its 48-bit arrival-field wrap.

What the kernel relies on, checked for every call:
* a CTA merges (answer 1 or 2) only after every CTA of its call has arrived, so every
  partial state it reads has been written;
* every CTA with merge items either merges them itself (1) or some CTA of the call merges
  every item (2) -- no item is left unmerged;
* no CTA waits for ever: a waiter leaves after its polls run out;
* the call adds exactly 2^16 to the arrival field, and the give-up field is back to zero
  after the call (or, once, holds the carry of an arrival-field wrap, which the next call's
  last arrival clears).
Calls do not overlap (the next call's CTAs arrive only after the previous grid completed).
"""
import random

TALLY = {"gave_up": 0, "merged_all": 0, "carry": 0}
Q = 1 << 16
GIVE = 1 << 48
MASK = GIVE - 1
M64 = (1 << 64) - 1


class Counter:
    def __init__(self, v=0):
        self.v = v & M64

    def fetch_add(self, x):
        old = self.v
        self.v = (self.v + x) & M64
        return old


def barrier(c, cta, n, wait, polls, log):
    """grid_barrier: yields between atomic steps; returns 0 / 1 / 2 (StopIteration value)."""
    add = Q - (n - 1) if cta == 0 else 1
    old = c.fetch_add(add)
    log["arrived"].add(cta)
    yield
    start = old & MASK & ~(Q - 1)

    def done(v):
        return ((v - start) & MASK) >= Q

    if done((old + add) & M64):
        g = old >> 48
        if g == 0:
            return 1 if wait else 0
        c.fetch_add(((-g) << 48) & M64)
        yield
        return 2
    if not wait:
        return 0
    left = polls
    while not done(c.v):  # acquire load
        yield
        left -= 1
        if left < 0:
            o2 = c.fetch_add(GIVE)
            yield
            if not done(o2):
                return 0
            c.fetch_add((-GIVE) & M64)
            yield
            return 1
    return 1


def run_call(c, n, rnd, held_back):
    wait = [rnd.random() < 0.7 for _ in range(n)]
    log = {"arrived": set()}
    gens = {i: barrier(c, i, n, wait[i], rnd.randint(0, 6), log) for i in range(n)}
    answer = {}
    late_start = {i: rnd.randint(0, 4 * n) for i in held_back}
    step = 0
    while gens:
        runnable = [i for i in gens if i not in held_back or
                    (late_start[i] >= 0 and step >= late_start[i]) or
                    all(j in held_back for j in gens)]
        i = rnd.choice(runnable)
        try:
            next(gens[i])
        except StopIteration as stop:
            answer[i] = stop.value
            del gens[i]
            if answer[i] in (1, 2):
                assert log["arrived"] == set(range(n)), "merge before every CTA arrived"
        step += 1
        assert step < 100000, "a CTA waits for ever"
    merged_all = any(a == 2 for a in answer.values())
    for i in range(n):
        if wait[i]:
            assert answer[i] == 1 or merged_all, f"CTA {i}'s items are left unmerged"
    TALLY["gave_up"] += sum(1 for i in range(n) if wait[i] and answer[i] == 0)
    TALLY["merged_all"] += merged_all
    return answer


def check_calls(start_value, calls, seed):
    rnd = random.Random(seed)
    c = Counter(start_value)
    carry_left = False
    for k in range(calls):
        n = rnd.randint(2, 7)
        held_back = set(rnd.sample(range(n), rnd.randint(0, min(2, n - 1))))
        before = c.v & MASK
        run_call(c, n, rnd, held_back)
        assert ((c.v & MASK) - before) & MASK == Q
        g = c.v >> 48
        assert g == 0 or (g == 1 and not carry_left), "give-ups left behind"
        carry_left = g == 1
        TALLY["carry"] += carry_left


def test_barrier_protocol_random_interleavings():
    TALLY.update(gave_up=0, merged_all=0)
    for seed in range(300):
        check_calls(0, 40, seed)
    # the give-up path and the merge of every item by the last arrival both ran
    assert TALLY["gave_up"] > 100 and TALLY["merged_all"] > 100


def test_barrier_protocol_across_the_arrival_field_wrap():
    TALLY.update(carry=0)
    for seed in range(300):
        check_calls(MASK + 1 - 3 * Q, 10, 1000 + seed)
    assert TALLY["carry"] > 0  # a wrap's carry was left for the next call and cleared there
