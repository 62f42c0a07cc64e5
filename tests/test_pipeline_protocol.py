"""A host model of the decode kernel's stage pipeline (paged_decode_kernel,
split form), checked over random schedules.

One producer fills STAGES slots in page order; each page's copy lands at an
arbitrary later time (copies may land out of order).  Two consumer sets take
the pages of each piece alternately (page i of a piece goes to set i % 2), so
with an odd number of stages consecutive rounds of a slot go to different
sets.  The mbarrier model follows the PTX rule for parity waits: a wait on
parity P passes when the current phase has the other parity, i.e. when the
phase with parity P among the current and the immediately preceding phase has
completed.

With plain parity waits a set can reach round r of a slot while round r - 1
(the other set's page) is still in flight; its wait then passes on round r - 2
and it reads a slot whose copy has not landed, and its release lands in the
wrong round.  The kernel's wait is gated on the slot's round tag, which the
producer writes before it issues the round; the model shows that form never
passes early and never over-arrives, for the same schedules."""
import random

import pytest

STAGES = 7
SETS = 2
WARPS = 2  # consumer warps per set (8 in the kernel; 2 show the same interleavings)


class MBarrier:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.tx = 0
        self.phase = 0  # index of the current (incomplete) phase
        self.bad = False  # an arrive on a phase with no arrivals left

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, tx=0):
        if self.pending == 0:
            self.bad = True
        self.tx += tx
        self.pending -= 1
        self._maybe_complete()

    def complete_tx(self, tx):
        self.tx -= tx
        self._maybe_complete()

    def try_wait(self, parity):
        return (self.phase & 1) != parity


def pages_of_set(pieces, s):
    """Split form of the 8-head kernel: page i of a piece goes to set i % 2."""
    out, kbase = [], 0
    for n in pieces:
        out += [kbase + i for i in range(s, n, SETS)]
        kbase += n
    return out


def run(units, consumers, count, gated, rng, stages=STAGES):
    """Producer fills `units` stage loads in order; consumer w takes the loads
    in consumers[w] in order; `count` consumers release each load."""
    full = [MBarrier(1) for _ in range(stages)]
    empty = [MBarrier(count) for _ in range(stages)]
    tag = [0] * stages
    landed = [False] * units
    in_flight = []
    nxt = 0  # producer's next load
    pos = [0] * len(consumers)
    early = False
    for _ in range(200 * units + 1000):
        acts = []
        if nxt < units and (nxt < stages or empty[nxt % stages].try_wait(((nxt // stages) - 1) & 1)):
            acts.append(("issue", None))
        acts += [("land", k) for k in range(len(in_flight))]
        for w, mine in enumerate(consumers):
            if pos[w] < len(mine):
                kk = mine[pos[w]]
                st, r = kk % stages, kk // stages
                ok = (tag[st] >> 1) >= r + 1 if gated else True
                if ok and full[st].try_wait(r & 1):
                    acts.append(("consume", w))
        if not acts:
            break
        kind, arg = rng.choice(acts)
        if kind == "issue":
            st = nxt % stages
            tag[st] = ((nxt // stages + 1) << 1) | 1
            full[st].arrive(tx=1)
            in_flight.append(nxt)
            nxt += 1
        elif kind == "land":
            kk = in_flight.pop(arg)
            landed[kk] = True
            full[kk % stages].complete_tx(1)
        else:
            kk = consumers[arg][pos[arg]]
            early |= not landed[kk]
            empty[kk % stages].arrive()
            pos[arg] += 1
    done = all(pos[w] == len(m) for w, m in enumerate(consumers))
    over = any(b.bad for b in full + empty)
    return early, over, done


def run_split(pieces, gated, rng):
    consumers = [pages_of_set(pieces, s) for s in range(SETS) for _ in range(WARPS)]
    return run(sum(pieces), consumers, WARPS, gated, rng)


def schedules(n):
    rng = random.Random(2024)
    for _ in range(n):
        pieces = [rng.randint(1, 40) for _ in range(rng.randint(1, 4))]
        yield pieces, random.Random(rng.randrange(1 << 30))


def test_plain_parity_waits_pass_early():
    """The failure the gate removes is reachable: some schedule lets a set
    pass its wait before its page landed."""
    found = False
    for pieces, rng in schedules(3000):
        early, over, _ = run_split(pieces, gated=False, rng=rng)
        if early or over:
            found = True
            break
    assert found


@pytest.mark.parametrize("seed_block", range(4))
def test_tag_gated_waits_are_exact(seed_block):
    for k, (pieces, rng) in enumerate(schedules(2000)):
        if k % 4 != seed_block:
            continue
        early, over, done = run_split(pieces, gated=True, rng=rng)
        assert not early, pieces
        assert not over, pieces
        assert done, pieces


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
def test_head_shard_kernel_plain_waits_are_exact(kv_heads):
    """paged_decode_heads_kernel: a stage holds 8 / kv_heads pages; way
    set * PS + o takes page o of every other stage (stages of set parity), and
    with an even number of stages (6) each warp takes every round of its
    slots, so plain parity waits are exact without a tag."""
    ps, stages = 8 // kv_heads, 6
    rng = random.Random(7 + kv_heads)
    for _ in range(300):
        n = rng.randint(1, 120)  # pages of the CTA's range
        units = (n + ps - 1) // ps
        consumers = [[kk for kk in range(units) if kk % 2 == st and kk * ps + o < n]
                     for st in range(2) for o in range(ps) for _ in range(kv_heads)]
        early, over, done = run(units, consumers, 8, gated=False,
                                rng=random.Random(rng.randrange(1 << 30)), stages=stages)
        assert not early and not over and done, n


def test_prefill_kernel_plain_waits_are_exact():
    """paged_prefill_kernel: every consumer warp takes every stage in order."""
    rng = random.Random(11)
    for _ in range(300):
        units = rng.randint(1, 60)
        consumers = [list(range(units)) for _ in range(4)]
        early, over, done = run(units, consumers, 4, gated=False,
                                rng=random.Random(rng.randrange(1 << 30)), stages=6)
        assert not early and not over and done, units
