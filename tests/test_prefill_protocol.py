"""CPU model check of the prefill kernel's mbarrier protocol (prefill_bsa.cu).

The roles run as programs of steps: the K producer, the V producer, the
single-thread MMA issuer and each of the four softmax warps on its own (a
warp whose rows do not list a tile runs ahead of the others, so warps can
be at different key tiles; a P_FULL phase completes on its fourth arrival,
and an arrival for a later phase landing in an open phase is an error). A wait on (barrier, parity) passes when the
barrier's completion count has the other parity, as `mbarrier.try_wait.parity`
does. TMA copies complete in any order; MMAs and commits complete in issue
order. Random schedules must never deadlock and never break an ordering rule
(a stage overwritten while still read, S read before it is computed, O
rescaled or read out under a running P.V). A planted mistake -- a V-stage
wait whose parity names the wrong completion -- must be caught.
"""

import random

import pytest


WARPS = 4  # softmax warps; each arrives once per key tile on P_FULL[j%2]


def _programs(n, rnd, flawed=False, rescale_prob=0.3):
    def kp():                                  # K producer: K(j) -> stage j%2
        for j in range(n):
            if 2 <= j < 4:
                yield ("wait", ("PRO", j - 2), 0)
            if j >= 4:
                yield ("wait", ("DONE", j & 1), (j >> 1) & 1)          # S(j-2) is in C(j-4)
            yield ("check", lambda s, j=j: j < 2 or ("S", j - 2) in s, f"K{j} over a stage S{j - 2} reads")
            yield ("tma", ("KF", j & 1), ("K", j))

    def vp():                                  # V producer: V(j) -> stage j%2
        for j in range(n):
            if j >= 2:                         # P.V(j-2) is in C(j-2), DONE[j%2]'s (j//2)-th completion
                par = (j >> 1) & 1 if flawed else ((j >> 1) - 1) & 1   # flawed: counts one completion too many
                yield ("wait", ("DONE", j & 1), par)
            yield ("check", lambda s, j=j: j < 2 or ("PV", j - 2) in s, f"V{j} over a stage PV{j - 2} reads")
            yield ("tma", ("VF", j & 1), ("V", j))

    def mma():
        def s_(j):
            yield ("wait", ("KF", j & 1), (j >> 1) & 1)
            yield ("check", lambda s: ("K", j) in s, f"S{j} before K{j} landed")
            yield ("mma", ("S", j))

        def pv(i):
            yield ("wait", ("PF", i & 1), (i >> 1) & 1)
            yield ("wait", ("VF", i & 1), (i >> 1) & 1)
            yield ("check", lambda s: ("V", i) in s and all(("P", i, w) in s for w in range(WARPS)),
                   f"PV{i} before P{i} / V{i}")
            yield ("mma", ("PV", i))

        for j in range(min(2, n)):
            yield from s_(j)
            yield ("commit", ("PRO", j))
        for j in range(n):
            yield from pv(j)
            if j + 2 < n:
                yield from s_(j + 2)
            yield ("commit", ("DONE", j & 1))

    def softmax(w):
        for j in range(n):
            if j < 2:
                yield ("wait", ("PRO", j), 0)
            else:
                yield ("wait", ("DONE", j & 1), ((j >> 1) - 1) & 1)   # S(j) is in C(j-2)
            yield ("check", lambda s, j=j: ("S", j) in s, f"S{j} read before it is computed")
            if j >= 1 and rnd.random() < rescale_prob:
                yield ("wait", ("DONE", (j - 1) & 1), ((j - 1) >> 1) & 1)  # P.V(j-1) is in C(j-1)
                yield ("check", lambda s, j=j: ("PV", j - 1) in s, f"O rescaled under PV{j - 1}")
            yield ("done", ("P", j, w))
            yield ("arrive", ("PF", j & 1), j)
        if n >= 1:
            yield ("wait", ("DONE", (n - 1) & 1), ((n - 1) >> 1) & 1)
            yield ("check", lambda s: ("PV", n - 1) in s, "O read out under the last P.V")

    progs = {"kp": kp(), "vp": vp(), "mma": mma()}
    for w in range(WARPS):
        progs[f"softmax{w}"] = softmax(w)
    return progs


def _run(n, seed, flawed=False):
    rnd = random.Random(seed)
    count, done, tma, pipe, pend = {}, set(), [], [], {}
    progs = _programs(n, rnd, flawed)
    cur = {k: next(g, None) for k, g in progs.items()}
    while True:
        moves = [("role", k) for k, op in cur.items()
                 if op is not None and not (op[0] == "wait" and (count.get(op[1], 0) & 1) == op[2])]
        if tma:
            moves.append(("tma", None))
        if pipe:
            moves.append(("pipe", None))
        if not moves:
            return "ok" if all(op is None for op in cur.values()) else "deadlock"
        kind, k = rnd.choice(moves)
        if kind == "tma":
            bar_, tag = tma.pop(rnd.randrange(len(tma)))
            done.add(tag)
            count[bar_] = count.get(bar_, 0) + 1
            continue
        if kind == "pipe":
            what, x = pipe.pop(0)
            if what == "mma":
                done.add(x)
            else:
                count[x] = count.get(x, 0) + 1
            continue
        op = cur[k]
        if op[0] == "check" and not op[1](done):
            return "violation: " + op[2]
        if op[0] == "tma":
            tma.append((op[1], op[2]))
        elif op[0] in ("mma", "commit"):
            pipe.append((op[0], op[1]))
        elif op[0] == "done":
            done.add(op[1])
        elif op[0] == "arrive":
            got = pend.setdefault(op[1], [])
            if got and got[0] != op[2]:
                return f"violation: arrival for P{op[2]} in the phase of P{got[0]}"
            got.append(op[2])
            if len(got) == WARPS:
                pend[op[1]] = []
                count[op[1]] = count.get(op[1], 0) + 1
        cur[k] = next(progs[k], None)


@pytest.mark.parametrize("n", [0, 1, 2, 3, 4, 5, 8, 13])
def test_protocol_never_deadlocks_or_reorders(n):
    bad = [(seed, r) for seed in range(300) for r in [_run(n, seed)] if r != "ok"]
    assert not bad, bad[:3]


def test_the_checker_catches_a_wait_on_the_wrong_completion():
    results = {_run(n, seed, flawed=True) for n in (3, 4, 5, 6) for seed in range(300)}
    assert any(r.startswith("violation: V") for r in results), results
