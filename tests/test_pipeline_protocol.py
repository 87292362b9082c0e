"""Randomised interleaving check of the fused attention kernel's mbarrier protocol
(csrc/attn_sm100.cu), on the CPU.

The kernel's roles are modelled as generators: the TMA producer (Q, then the K and V rings), two
S-issue threads (even / odd tiles), the P.V issue thread, and eight softmax warps in two groups
taking alternate tiles.  Each yields ("wait", barrier, n) - wait for completion n of a barrier -
or ("do", action).  MMAs complete in issue order per issuing thread, TMA copies in any order.
A barrier keeps its completed-phase count c; a parity wait for completion n passes iff
c % 2 != n % 2, which is only correct while c is n or n + 1: every poll asserts that (else the
hardware would pass a phase early or wait forever).  Buffer hazards are asserted as the model
runs: an S MMA never overwrites P before its P.V has completed, P.V reads the P of its own tile
written by all four warps of the tile's group, K/V slots are refilled only after their readers
completed, and O is rescaled only while no P.V into it is in flight.
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


def run(ntiles, seed, rescale_p=0.2):
    rng = random.Random(seed)
    B = {"Q": Bar("Q", 1)}
    for s in range(NS):
        for nm, cnt in (("KF", 1), ("KE", 1), ("VF", 1), ("SF", 1), ("PF", 4), ("PV", 1)):
            B[f"{nm}{s}"] = Bar(f"{nm}{s}", cnt)
    for q in range(4):
        B[f"M{q}"] = Bar(f"M{q}", 2)
    kslot, vslot = [None] * NS, [None] * NS
    sbuf = [None] * NS
    pwritten = [set() for _ in range(NS)]
    o = {"pv_done": [-1, -1], "pv_issued": [-1, -1], "last": -1}
    queues = {"S0": [], "S1": [], "PV": []}
    tma = []
    

    def complete_tma(item):
        kind, s, i = item
        if kind == "K":
            kslot[s] = i
            B[f"KF{s}"].arrive()
        elif kind == "V":
            vslot[s] = i
            B[f"VF{s}"].arrive()
        else:
            B["Q"].arrive()

    def complete_mma(item):
        kind, i, commits = item
        s = i % NS
        if kind == "S":
            assert kslot[s] == i, ("K slot", kslot[s], "for S", i)
            assert sbuf[s] is None or sbuf[s] == ("Pdone", i - NS), ("S overwrite", sbuf[s], i)
            sbuf[s] = ("S", i)
            pwritten[s] = set()
        else:
            assert vslot[s] == i, ("V slot", vslot[s], "for PV", i)
            g = i % 2
            assert sbuf[s] == ("S", i) and pwritten[s] == set(range(4 * g, 4 * g + 4)), ("P", sbuf[s], pwritten[s], i)
            assert o["pv_done"][g] == (i - 2 if i >= 2 else -1) and o["last"] == i - 1, (o, i)
            sbuf[s] = ("Pdone", i)
            o["pv_done"][g] = i
            o["last"] = i
        for b in commits:
            B[b].arrive()

    def kprod():
        tma.append(("Q", 0, 0))
        for i in range(ntiles):
            s = i % NS
            if i >= NS:
                yield ("wait", f"KE{s}", i // NS - 1)

            def ld(i=i, s=s):
                assert i < NS or sbuf[s] in (("S", i - NS), ("Pdone", i - NS)), ("K reuse", sbuf[s], i)
                tma.append(("K", s, i))
            yield ("do", ld)
            if i >= NS:
                yield ("wait", f"PV{s}", i // NS - 1)

            def ldv(i=i, s=s):
                assert i < NS or o["pv_done"][(i - NS) % 2] >= i - NS
                tma.append(("V", s, i))
            yield ("do", ldv)

    def sissue(par):
        yield ("wait", "Q", 0)
        for i in range(par, ntiles, 2):
            s = i % NS
            if i >= NS:
                yield ("wait", f"PV{s}", i // NS - 1)
            yield ("wait", f"KF{s}", i // NS)
            yield ("do", lambda i=i, s=s, par=par: queues[f"S{par}"].append(("S", i, [f"SF{s}", f"KE{s}"])))

    def pvissue():
        for i in range(ntiles):
            s = i % NS
            yield ("wait", f"PF{s}", i // NS)
            yield ("wait", f"VF{s}", i // NS)

            def issue(i=i, s=s):
                o["pv_issued"][i % 2] = i
                queues["PV"].append(("PV", i, [f"PV{s}"]))
            yield ("do", issue)

    def softmax(w):
        quarter, g = w & 3, w >> 2
        last = -1
        for i in range(g, ntiles, 2):
            s = i % NS
            yield ("wait", f"SF{s}", i // NS)

            def read(i=i, s=s):
                assert sbuf[s] == ("S", i), ("softmax reads", sbuf[s], i)
            yield ("do", read)
            if last >= 0 and (rng.random() < rescale_p):
                yield ("wait", f"PV{last % NS}", last // NS)

                def resc(i=i, g=g):
                    assert o["pv_done"][g] == i - 2 and o["pv_issued"][g] == i - 2, ("rescale", o, i)
                yield ("do", resc)

            def write(i=i, s=s, w=w):
                assert sbuf[s] == ("S", i)
                pwritten[s].add(w)
            yield ("do", write)
            yield ("do", lambda s=s: B[f"PF{s}"].arrive())
            last = i
        if last >= 0:
            yield ("wait", f"PV{last % NS}", last // NS)
        yield ("do", lambda q=quarter: B[f"M{q}"].arrive())
        yield ("wait", f"M{quarter}", 0)

        def epi(g=g, last=last):
            assert o["pv_done"][g] == last
        yield ("do", epi)

    roles = {"k": kprod(), "s0": sissue(0), "s1": sissue(1), "pv": pvissue()}
    for w in range(8):
        roles[f"sm{w}"] = softmax(w)
    cur = {k: None for k in roles}
    done = set()
    steps = 0
    while len(done) < len(roles) or any(queues.values()) or tma:
        steps += 1
        assert steps < 500000, "deadlock " + str({k: cur[k] for k in roles if k not in done})
        choices = [k for k in roles if k not in done]
        choices += [q for q in queues if queues[q]]
        if tma:
            choices.append("_tma")
        k = rng.choice(choices)
        if k in queues:
            complete_mma(queues[k].pop(0))
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
    return True


@pytest.mark.parametrize("ntiles", [1, 2, 3, 4, 5, 7, 9, 13, 21])
def test_barrier_protocol_interleavings(ntiles):
    for seed in range(60):
        run(ntiles, seed)


def test_odd_stage_count_with_two_groups_is_unsafe():
    """With an odd stage count a slot alternates between the two softmax groups, and a group may
    test a slot's S_FULL a phase early: the model must catch that (the kernel uses NS = 4)."""
    global NS
    saved, NS = NS, 3
    try:
        failures = 0
        for seed in range(200):
            try:
                run(4, seed)
            except AssertionError:
                failures += 1
        assert failures > 0
    finally:
        NS = saved
