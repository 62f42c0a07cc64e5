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


# ---------------------------------------------------------------------------
# paged_prefill_kernel: the whole protocol of one CTA, with two softmax sides
# (side s takes the chunks c with c % 2 == s) and the tensor-core operations
# as asynchronous work that completes in issue order.
#   producer : chunk c's K/V into stage c % KV_STAGES after kv_empty of c - KV_STAGES
#   MMA      : S(0), S(1); then per c: wait P(c), PV(c) into O[c % 2], commit
#              kv_empty(c), S(c + 2) (waits for its K/V); finally commit o_full
#   side s   : per own chunk c: wait s_full[s]; read S buffer s; maybe rescale
#              O[s]; write P buffer s; arrive p_full[s] (SIDE_WARPS arrivals);
#              at the end wait o_full and read O[0], O[1]
# Hazards checked: reading S(c) before it is computed or after S(c + 2)
# overwrote it; a PV reading a P buffer not yet (or no longer) holding its
# chunk; an O rescale while a PV into that O is outstanding; a K/V stage
# refilled before the MMAs that read it completed; the final read before
# every PV completed; and deadlock.
KV_STAGES = 4
SIDE_WARPS = 2  # 4 in the kernel; 2 show the same interleavings


def run_prefill(n_chunks, rng, sides=2, early_s=False):
    full = [MBarrier(1) for _ in range(KV_STAGES)]
    empty = [MBarrier(1) for _ in range(KV_STAGES)]
    s_full = [MBarrier(1) for _ in range(2)]
    p_full = [MBarrier(SIDE_WARPS) for _ in range(2)]
    o_full = MBarrier(1)
    kv_landed = {}          # chunk -> landed
    kv_slot = [None] * KV_STAGES   # chunk whose K/V a stage holds (issued)
    s_buf = [None, None]    # chunk whose S the buffer holds (completed MMA)
    p_buf = [None, None]    # chunk whose P the buffer holds (all warps wrote)
    p_writes = [0, 0]
    o_pending = [0, 0]      # PVs issued into O[s] and not completed
    queue = []              # tensor-core ops in issue order: (kind, chunk) or ("commit", bar)
    errors = []
    prod_next = 0
    in_flight = []
    # MMA thread program as a list of steps, advanced one at a time
    mma = {"pc": 0, "c": 0}
    steps = []
    steps.append(("S", 0))
    if n_chunks > 1:
        steps.append(("S", 1))
    for c in range(n_chunks):
        if early_s and c + 2 < n_chunks:  # the broken order: S(c + 2) before P(c) is ready
            steps += [("S", c + 2), ("waitP", c), ("PV", c), ("commit_empty", c)]
            continue
        steps += [("waitP", c), ("PV", c), ("commit_empty", c)]
        if c + 2 < n_chunks:
            steps.append(("S", c + 2))
    steps.append(("commit_o", None))
    # softmax warps: (side, warp) -> list of own chunks, position, phase within chunk
    warps = []
    for s in range(sides):
        own = list(range(s, n_chunks, 2))
        for w in range(SIDE_WARPS):
            warps.append({"side": s, "own": own, "i": 0, "stage": "wait", "final": False})

    def exec_op():
        kind, c = queue.pop(0)
        if kind == "S":
            if kv_slot[c % KV_STAGES] != c or not kv_landed.get(c):
                errors.append(f"S({c}) read K/V not landed")
            b = c % 2
            if s_buf[b] is not None and s_buf[b] != c - 2:
                errors.append(f"S({c}) overwrote buffer holding S({s_buf[b]})")
            s_buf[b] = c
            s_read[b] = 0
        elif kind == "PV":
            b = c % 2
            if p_buf[b] != c:
                errors.append(f"PV({c}) read P buffer holding {p_buf[b]}")
            if kv_slot[c % KV_STAGES] != c:
                errors.append(f"PV({c}) read a refilled V stage")
            o_pending[b] -= 1
        elif kind == "commit":
            c[0].arrive() if isinstance(c, tuple) else c.arrive()

    s_read = [0, 0]
    for _ in range(400 * (n_chunks + 4)):
        acts = []
        if prod_next < n_chunks:
            st = prod_next % KV_STAGES
            if prod_next < KV_STAGES or empty[st].try_wait(((prod_next // KV_STAGES) - 1) & 1):
                acts.append(("issue",))
        acts += [("land", k) for k in range(len(in_flight))]
        if queue:
            acts.append(("exec",))
        if mma["pc"] < len(steps):
            kind, c = steps[mma["pc"]]
            if kind == "S":
                if full[c % KV_STAGES].try_wait((c // KV_STAGES) & 1):
                    acts.append(("mma",))
            elif kind == "waitP":
                if p_full[c % 2].try_wait((c // 2) & 1):
                    acts.append(("mma",))
            else:
                acts.append(("mma",))
        for wi, w in enumerate(warps):
            if w["i"] < len(w["own"]):
                c = w["own"][w["i"]]
                if w["stage"] == "wait" and s_full[w["side"]].try_wait((c // 2) & 1):
                    acts.append(("warp", wi))
                elif w["stage"] != "wait":
                    acts.append(("warp", wi))
            elif not w["final"] and o_full.try_wait(0):
                acts.append(("final", wi))
        if not acts:
            break
        act = rng.choice(acts)
        if act[0] == "issue":
            c = prod_next
            kv_slot[c % KV_STAGES] = c
            kv_landed[c] = False
            full[c % KV_STAGES].arrive(tx=1)
            in_flight.append(c)
            prod_next += 1
        elif act[0] == "land":
            c = in_flight.pop(act[1])
            kv_landed[c] = True
            full[c % KV_STAGES].complete_tx(1)
        elif act[0] == "exec":
            exec_op()
        elif act[0] == "mma":
            kind, c = steps[mma["pc"]]
            mma["pc"] += 1
            if kind == "S":
                queue.append(("S", c))
                queue.append(("commit", s_full[c % 2]))
            elif kind == "PV":
                o_pending[c % 2] += 1
                queue.append(("PV", c))
            elif kind == "commit_empty":
                queue.append(("commit", empty[c % KV_STAGES]))
            elif kind == "commit_o":
                queue.append(("commit", o_full))
        elif act[0] == "warp":
            w = warps[act[1]]
            c = w["own"][w["i"]]
            b = w["side"]
            if w["stage"] == "wait":
                w["stage"] = "read"
            elif w["stage"] == "read":
                if s_buf[b] != c:
                    errors.append(f"side {b} read S buffer holding {s_buf[b]} for chunk {c}")
                w["stage"] = "rescale" if rng.random() < 0.3 and c >= 2 else "write"
            elif w["stage"] == "rescale":
                if o_pending[b]:
                    errors.append(f"rescale of O[{b}] at chunk {c} with a PV outstanding")
                w["stage"] = "write"
            elif w["stage"] == "write":
                if p_buf[b] is not None and p_buf[b] != c and o_pending[b]:
                    errors.append(f"P buffer {b} rewritten for chunk {c} before PV({p_buf[b]}) read it")
                p_writes[b] += 1
                if p_writes[b] == SIDE_WARPS:
                    p_buf[b] = c
                    p_writes[b] = 0
                p_full[b].arrive()
                w["stage"] = "wait"
                w["i"] += 1
        elif act[0] == "final":
            w = warps[act[1]]
            if any(o_pending) or queue and any(k == "PV" for k, _ in queue):
                errors.append("final read before every PV completed")
            w["final"] = True
    done = mma["pc"] == len(steps) and not queue and all(w["final"] for w in warps)
    bad = any(b.bad for b in full + empty + s_full + p_full + [o_full])
    return errors, bad, done


@pytest.mark.parametrize("n_chunks", [1, 2, 3, 4, 5, 8, 13, 30])
def test_prefill_two_sided_protocol(n_chunks):
    rng = random.Random(100 + n_chunks)
    for _ in range(200):
        errors, bad, done = run_prefill(n_chunks, random.Random(rng.randrange(1 << 30)))
        assert not errors, errors[:3]
        assert not bad and done


def test_prefill_model_catches_an_early_score_mma():
    """The model is not vacuous: issuing S(c + 2) before P(c) is ready lets it
    overwrite the S buffer that side c % 2 may still be reading."""
    rng = random.Random(7)
    found = 0
    for _ in range(300):
        errors, _, _ = run_prefill(8, random.Random(rng.randrange(1 << 30)), early_s=True)
        found += bool(errors)
    assert found > 0
