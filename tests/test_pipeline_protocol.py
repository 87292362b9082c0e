"""Randomised interleaving check of the fused attention kernel's mbarrier protocol
(csrc/attn_sm100.cu), on the CPU.

The kernel is persistent: one CTA works through several items (128-row query tiles), and the
tiles of all its items form one sequence g = 0, 1, ... through the K/V rings and S buffers
(slot g % NS, softmax group g % 2).  Its roles are modelled as generators: the producer (per
item: Q into buffer k % 2, the tile list into list buffer k % 2, then the K and V rings), two
S-issue threads (even / odd tiles), the P.V issue thread, and eight softmax warps in two groups
with a per-item epilogue (merge exchange, O read, O_FREE and LIST_EMPTY arrivals).  Each yields
("wait", barrier, n) - wait for completion n of a barrier - or ("do", action).  MMAs complete
in issue order per issuing thread, TMA copies in any order.  A barrier keeps its
completed-phase count c; a parity wait for completion n passes iff c % 2 != n % 2, which is only
correct while c is n or n + 1: every poll asserts that (else the hardware would pass a phase
early or wait forever).  Buffer hazards are asserted as the model runs: an S MMA reads the Q of
its own item and never overwrites P before its P.V has completed, P.V reads the P of its own
tile written by all four warps of the tile's group, K/V slots are refilled only after their
readers completed, a tile list is rebuilt only after all eleven readers released it, O is
rescaled only while no P.V into it is in flight, and an item's first P.V into O waits until the
previous item's epilogue has read it.
"""
import random

import pytest

NS = 4  # ring stages of the kernel (kStages)


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.c = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        assert self.pending >= 0, self.name
        if self.pending == 0:
            self.c += 1
            self.pending = self.count


def run(items, seed, rescale_p=0.2):
    """items: the tile counts of the work items one CTA processes, in order."""
    rng = random.Random(seed)
    B = {}
    for s in range(NS):
        for nm, cnt in (("KF", 1), ("KE", 1), ("VF", 1), ("SF", 1), ("PF", 4), ("PV", 1)):
            B[f"{nm}{s}"] = Bar(f"{nm}{s}", cnt)
    for lb in range(2):
        B[f"LF{lb}"] = Bar(f"LF{lb}", 1)
        B[f"LE{lb}"] = Bar(f"LE{lb}", 11)
        B[f"QF{lb}"] = Bar(f"QF{lb}", 1)
        B[f"QE{lb}"] = Bar(f"QE{lb}", 2)
    for q in range(4):
        B[f"M{q}"] = Bar(f"M{q}", 2)
    B["OF"] = Bar("OF", 8)
    total = sum(items)
    kslot, vslot, sbuf = [None] * NS, [None] * NS, [None] * NS
    pwritten = [set() for _ in range(NS)]
    qbuf = [None, None]       # item whose Q is in buffer lb
    lists = [None, None]      # item whose list is in buffer lb
    list_readers = [set(), set()]
    o = {"pv_done": [-1, -1], "pv_issued": [-1, -1], "last": -1, "o_item": [None, None], "o_read": set()}
    queues = {"S0": [], "S1": [], "PV": []}
    tma = []
    bases = [sum(items[:k]) for k in range(len(items))]

    def item_of(g):
        for k in range(len(items)):
            if bases[k] <= g < bases[k] + items[k]:
                return k
        raise AssertionError("tile outside items")

    def complete_tma(it):
        kind, s, i = it
        if kind == "K":
            kslot[s] = i
            B[f"KF{s}"].arrive()
        elif kind == "V":
            vslot[s] = i
            B[f"VF{s}"].arrive()
        else:  # Q for item i into buffer s
            qbuf[s] = i
            B[f"QF{s}"].arrive()

    def complete_mma(it):
        kind, g, commits = it
        if kind == "S":
            s = g % NS
            k = item_of(g)
            assert qbuf[k % 2] == k, ("Q buffer", qbuf, g)
            assert kslot[s] == g, ("K slot", kslot[s], g)
            assert sbuf[s] is None or sbuf[s] == ("Pdone", g - NS), ("S overwrite", sbuf[s], g)
            sbuf[s] = ("S", g)
            pwritten[s] = set()
        elif kind == "PV":
            s = g % NS
            grp = g % 2
            k = item_of(g)
            assert vslot[s] == g, ("V slot", vslot[s], g)
            assert sbuf[s] == ("S", g) and pwritten[s] == set(range(4 * grp, 4 * grp + 4)), ("P", sbuf[s], pwritten[s], g)
            # O_grp belongs to item k: the previous item's epilogue must have read it
            if o["o_item"][grp] != k:
                assert o["o_item"][grp] is None or o["o_read"] >= {(o["o_item"][grp], w) for w in range(8)}, ("O reuse", o, g)
                o["o_item"][grp] = k
            sbuf[s] = ("Pdone", g)
            o["pv_done"][grp] = g
            o["last"] = g
        for b in commits:
            B[b].arrive()

    def producer():
        # per item: Q (buffer k % 2, once item k - 2's S MMAs completed), then the tile list
        # (buffer k % 2, once item k - 2's readers released it), then the K and V tiles
        g = 0
        for k, n in enumerate(items):
            lb = k % 2
            if k >= 2:
                yield ("wait", f"QE{lb}", (k >> 1) - 1)
            yield ("do", lambda k=k, lb=lb: tma.append(("Q", lb, k)))
            if k >= 2:
                yield ("wait", f"LE{lb}", (k >> 1) - 1)

            def build(k=k, lb=lb):
                assert lists[lb] is None or list_readers[lb] >= set(range(11)), ("list reuse", lists, list_readers, k)
                lists[lb] = k
                list_readers[lb] = set()
                B[f"LF{lb}"].arrive()
            yield ("do", build)
            for i in range(n):
                gi = g + i
                s = gi % NS
                if gi >= NS:
                    yield ("wait", f"KE{s}", gi // NS - 1)
                yield ("do", lambda gi=gi, s=s: tma.append(("K", s, gi)))
                if gi >= NS:
                    yield ("wait", f"PV{s}", gi // NS - 1)
                yield ("do", lambda gi=gi, s=s: tma.append(("V", s, gi)))
            g += n

    def sissue(par):
        g = 0
        for k, n in enumerate(items):
            lb = k % 2
            yield ("wait", f"LF{lb}", k >> 1)
            yield ("wait", f"QF{lb}", k >> 1)
            for i in range(n):
                gi = g + i
                if gi % 2 != par:
                    continue
                s = gi % NS
                if gi >= NS:
                    yield ("wait", f"PV{s}", gi // NS - 1)
                yield ("wait", f"KF{s}", gi // NS)
                yield ("do", lambda gi=gi, s=s, par=par: queues[f"S{par}"].append(("S", gi, [f"SF{s}", f"KE{s}"])))
            # Q_EMPTY via commit: tracks this thread's MMAs so far
            yield ("do", lambda par=par, lb=lb: queues[f"S{par}"].append(("C", -1, [f"QE{lb}"])))
            yield ("do", lambda lb=lb, par=par: (list_readers[lb].add(8 + par), B[f"LE{lb}"].arrive()))
            g += n

    def pvissue():
        g = 0
        for k, n in enumerate(items):
            lb = k % 2
            yield ("wait", f"LF{lb}", k >> 1)
            if k >= 1:
                yield ("wait", "OF", k - 1)
            for i in range(n):
                gi = g + i
                s = gi % NS
                yield ("wait", f"PF{s}", gi // NS)
                yield ("wait", f"VF{s}", gi // NS)

                def issue(gi=gi, s=s):
                    o["pv_issued"][gi % 2] = gi
                    queues["PV"].append(("PV", gi, [f"PV{s}"]))
                yield ("do", issue)
            yield ("do", lambda lb=lb: (list_readers[lb].add(10), B[f"LE{lb}"].arrive()))
            g += n

    def softmax(w):
        quarter, grp = w & 3, w >> 2
        g = 0
        for k, n in enumerate(items):
            lb = k % 2
            yield ("wait", f"LF{lb}", k >> 1)
            last = -1
            for i in range(n):
                gi = g + i
                if gi % 2 != grp:
                    continue
                s = gi % NS
                yield ("wait", f"SF{s}", gi // NS)

                def read(gi=gi, s=s):
                    assert sbuf[s] == ("S", gi), ("softmax reads", sbuf[s], gi)
                yield ("do", read)
                if last >= 0 and rng.random() < rescale_p:
                    yield ("wait", f"PV{last % NS}", last // NS)

                    def resc(gi=gi, grp=grp, last=last):
                        assert o["pv_done"][grp] == last and o["pv_issued"][grp] == last, ("rescale", o, gi)
                    yield ("do", resc)

                def write(gi=gi, s=s, w=w):
                    assert sbuf[s] == ("S", gi)
                    pwritten[s].add(w)
                yield ("do", write)
                yield ("do", lambda s=s: B[f"PF{s}"].arrive())
                last = gi
            if last >= 0:
                yield ("wait", f"PV{last % NS}", last // NS)
            yield ("do", lambda q=quarter: B[f"M{q}"].arrive())
            yield ("wait", f"M{quarter}", k)

            def epi(k=k, n=n, g=g, w=w):
                # both groups' last PV of this item complete
                for x in range(2):
                    tiles = [gg for gg in range(g, g + n) if gg % 2 == x]
                    if tiles:
                        assert o["pv_done"][x] >= tiles[-1] and o["o_item"][x] == k, ("epilogue", o, k)
                o["o_read"].add((k, w))
            yield ("do", epi)
            yield ("do", lambda: B["OF"].arrive())
            yield ("do", lambda lb=lb, w=w: (list_readers[lb].add(w), B[f"LE{lb}"].arrive()))
            g += n

    roles = {"prod": producer(), "s0": sissue(0), "s1": sissue(1), "pv": pvissue()}
    for w in range(8):
        roles[f"sm{w}"] = softmax(w)
    cur = {k: None for k in roles}
    done = set()
    steps = 0
    while len(done) < len(roles) or any(queues.values()) or tma:
        steps += 1
        assert steps < 2000000, "deadlock " + str({k: cur[k] for k in roles if k not in done})
        choices = [k for k in roles if k not in done] + [q for q in queues if queues[q]]
        if tma:
            choices.append("_tma")
        k = rng.choice(choices)
        if k in queues:
            it = queues[k].pop(0)
            if it[0] == "C":
                for b in it[2]:
                    B[b].arrive()
            else:
                complete_mma(it)
            continue
        if k == "_tma":
            complete_tma(tma.pop(rng.randrange(len(tma))))
            continue
        if cur[k] is None:
            try:
                cur[k] = next(roles[k])
            except StopIteration:
                done.add(k)
                continue
        op = cur[k]
        if op[0] == "wait":
            _, b, n = op
            c = B[b].c
            assert c in (n, n + 1), (k, b, "completion", n, "count", c)
            if c % 2 != n % 2:
                cur[k] = None
        else:
            op[1]()
            cur[k] = None


ITEM_CASES = [[1], [2], [3, 1, 2], [5, 7, 1, 4], [9, 9, 9], [1, 1, 1, 1, 1], [2, 6, 3, 8, 1, 5],
              [4, 4, 4, 4], [12, 1, 13, 2, 7], [21]]


@pytest.mark.parametrize("items", ITEM_CASES, ids=lambda c: "-".join(map(str, c)))
def test_barrier_protocol_interleavings(items):
    for seed in range(40):
        run(items, seed)


def test_odd_stage_count_with_two_groups_is_unsafe():
    """With an odd stage count a slot alternates between the two softmax groups, and a group may
    test a slot's S_FULL a phase early: the model must catch that (the kernel uses NS = 4)."""
    global NS
    saved, NS = NS, 3
    try:
        failures = 0
        for seed in range(200):
            try:
                run([4, 3], seed)
            except AssertionError:
                failures += 1
        assert failures > 0
    finally:
        NS = saved
