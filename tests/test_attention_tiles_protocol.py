"""The barrier protocol of the persistent two-tile attention template, checked on the CPU.

``compiler/kernels/attention.py`` runs one persistent CTA per SM over units of NQ = 2
query tiles (one batch x head each).  Its roles: the TMA producer (per unit the two Q
tiles, each once the previous unit's last ``Q_t K^T`` is done -- ``q_empty`` -- then K_j
and V_j through a ring of R slots), one MMA-issuing thread (per unit ``S_t(0)``, then per
block ``O_t += P_t V_j`` and ``S_t(j + 1)``, its tcgen05 operations completing in issue
order), and one softmax warpgroup per tile (per block: S_t in, P_t out; per unit: the
epilogue reads O_t, before it hands over the next unit's first P_t).  The model replays
that protocol under random schedules, with the causal case's per-tile block counts, and
checks that no schedule
deadlocks, that every parity wait is satisfied by exactly the completion it means, and
that no Q slot, ring slot, S / P buffer or O accumulator is overwritten or read at the
wrong time.  Mistakes planted in the model must be caught.
"""

import random

import pytest


class _Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.done = name, count, 0, 0

    def arrive(self):
        self.pending += 1
        assert self.pending <= self.count, self.name
        if self.pending == self.count:
            self.pending = 0
            self.done += 1


def simulate(units, R, seed, plant=None):
    """``units``: per unit the key blocks of each tile (nbt_0 <= nbt_1); returns the
    violations of one random schedule."""
    rnd = random.Random(seed)
    NQ = 2
    B = {}
    for t in range(NQ):
        for n in ("q_full", "q_empty", "s", "p", "o"):
            B[(n, t)] = _Bar(f"{n}[{t}]", 1)
    for r in range(R):
        B[("full", r)] = _Bar(f"full[{r}]", 1)
        B[("empty", r)] = _Bar(f"empty[{r}]", 1)
    st = {"q": [None] * NQ, "qread": [0] * NQ, "ring": [None] * R, "rread": [0] * R,
          "S": [None] * NQ, "O": [None] * NQ, "O_read": [True] * NQ}
    pipe, tma, errors = [], [], []

    def wait(name, idx, k):
        b = B[(name, idx)]
        while True:
            if b.done >= k + 2 or b.done < k:
                errors.append(f"{b.name}: waiting for completion {k} at {b.done}")
                raise StopIteration
            if (b.done & 1) != (k & 1):
                return
            yield

    def land(bar, fn):
        tma.append((bar, fn))

    def producer():
        L = 0
        for ui, nbt in enumerate(units):
            for t in range(NQ):
                if ui > 0 and plant != "no_q_empty_wait":
                    yield from wait("q_empty", t, ui - 1)

                def qland(t=t, ui=ui):
                    if st["qread"][t]:
                        errors.append(f"Q_{t}({ui}) lands over a tile still read")
                    st["q"][t] = ui
                land(("q_full", t), qland)
            for j in range(nbt[-1]):
                for which in "kv":
                    slot = L % R
                    if L >= R:
                        yield from wait("empty", slot, L // R - 1)

                    def rland(slot=slot, tag=(which, ui, j)):
                        if st["rread"][slot]:
                            errors.append(f"{tag} lands over a slot still read")
                        st["ring"][slot] = tag
                    land(("full", slot), rland)
                    L += 1

    def mma():
        C = 0
        cntp = [0] * NQ

        def qk(t, ui, j, slot):
            st["qread"][t] += 1
            st["rread"][slot] += 1

            def op():
                st["qread"][t] -= 1
                st["rread"][slot] -= 1
                if st["q"][t] != ui:
                    errors.append(f"S_{t}({ui},{j}) reads Q of unit {st['q'][t]}")
                if st["ring"][slot] != ("k", ui, j):
                    errors.append(f"S_{t}({ui},{j}) reads {st['ring'][slot]}")
                if st["S"][t] is not None and st["S"][t][2] != "consumed":
                    errors.append(f"S_{t}({ui},{j}) overwrites live {st['S'][t]}")
                st["S"][t] = [ui, j, "scores"]
            pipe.append(("op", op))
            pipe.append(("commit", ("s", t)))

        for ui, nbt in enumerate(units):
            kslot = C % R
            yield from wait("full", kslot, C // R)
            for t in range(NQ):
                yield from wait("q_full", t, ui)
                qk(t, ui, 0, kslot)
                if nbt[t] == 1:
                    pipe.append(("commit", ("q_empty", t)))
            pipe.append(("commit", ("empty", kslot)))
            C += 1
            for jm in range(nbt[-1]):
                vslot = C % R
                yield from wait("full", vslot, C // R)
                C += 1
                more = jm + 1 < nbt[-1]
                kslot, kwaited = C % R, False
                for t in range(NQ):
                    if jm >= nbt[t]:
                        continue
                    yield from wait("p", t, cntp[t])
                    cntp[t] += 1
                    st["rread"][vslot] += 1

                    def pv(t=t, ui=ui, jm=jm, vslot=vslot):
                        st["rread"][vslot] -= 1
                        if st["ring"][vslot] != ("v", ui, jm):
                            errors.append(f"PV_{t}({ui},{jm}) reads {st['ring'][vslot]}")
                        if st["S"][t] != [ui, jm, "P"]:
                            errors.append(f"PV_{t}({ui},{jm}) reads P {st['S'][t]}")
                        if jm == 0 and not st["O_read"][t]:
                            errors.append(f"PV_{t}({ui},0) overwrites O still being read")
                        st["O"][t] = (ui, jm)
                        st["O_read"][t] = False
                        st["S"][t][2] = "consumed"
                    pipe.append(("op", pv))
                    pipe.append(("commit", ("o", t)))
                    if jm + 1 < nbt[t]:
                        if not kwaited:
                            yield from wait("full", kslot, C // R)
                            kwaited = True
                        qk(t, ui, jm + 1, kslot)
                        if jm + 1 == nbt[t] - 1 - (plant == "early_q_release"):
                            pipe.append(("commit", ("q_empty", t)))
                pipe.append(("commit", ("empty", vslot)))
                if more:
                    pipe.append(("commit", ("empty", kslot)))
                    C += 1

    def softmax(t):
        gcnt = 0
        for ui, nbt in enumerate(units):
            for jj in range(nbt[t]):
                yield from wait("s", t, gcnt)
                if st["S"][t] != [ui, jj, "scores"]:
                    errors.append(f"softmax_{t}({ui},{jj}) reads {st['S'][t]}")
                # the S commit covers the previous O_t += P_t V: a rescale may touch O_t
                if jj > 0 and st["O"][t] != (ui, jj - 1):
                    errors.append(f"softmax_{t}({ui},{jj}) sees O_t at {st['O'][t]}")
                yield
                st["S"][t][2] = "P"
                B[("p", t)].arrive()
                gcnt += 1
                yield
            yield from wait("o", t, gcnt - 1)
            if st["O"][t] != (ui, nbt[t] - 1):
                errors.append(f"epilogue_{t}({ui}) reads O at {st['O'][t]}")
            yield
            st["O_read"][t] = True

    agents = [producer(), mma(), softmax(0), softmax(1)]
    alive = list(range(len(agents)))
    stall = 0
    while alive or pipe or tma:
        choices = ([("agent", i) for i in alive] + ([("pipe", 0)] if pipe else [])
                   + ([("tma", 0)] if tma else []))
        kind, i = rnd.choice(choices)
        if kind == "pipe":
            what, x = pipe.pop(0)
            x() if what == "op" else B[x].arrive()
            stall = 0
        elif kind == "tma":
            bar, fn = tma.pop(rnd.randrange(len(tma)))
            fn()
            B[bar].arrive()
            stall = 0
        else:
            try:
                next(agents[i])
            except (StopIteration, RuntimeError):
                alive.remove(i)
            stall += 1
        if errors:
            return errors
        if stall > 20000:
            return [f"deadlock: agents {alive} still waiting"]
    return errors


def _units(rng, n, causal):
    out = []
    for _ in range(n):
        if causal:
            a = rng.randint(1, 4)
            out.append((a, a + rng.randint(0, 1)))
        else:
            b = rng.randint(1, 4)
            out.append((b, b))
    return out


def _cases():
    rng = random.Random(7)
    return [(_units(rng, n, causal), R) for causal in (False, True) for n in (1, 2, 4) for R in (2, 3, 5)]


def test_protocol_holds_under_random_schedules():
    for units, R in _cases():
        for seed in range(40):
            errs = simulate(units, R, seed)
            assert not errs, (units, R, seed, errs[:2])


@pytest.mark.parametrize("plant", ["no_q_empty_wait", "early_q_release"])
def test_planted_protocol_mistakes_are_caught(plant):
    caught = sum(bool(simulate(units, R, seed, plant)) for units, R in _cases() for seed in range(20))
    assert caught > 0, plant
