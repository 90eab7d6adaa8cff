"""The barrier protocol of the split-key attention schedule, checked on the CPU.

``compiler/kernels/attention_split.py`` coordinates five roles through mbarriers: the
TMA producer, one MMA-issuing thread per key half (``S_h`` then ``O_h += P_h V``, each
thread's tcgen05 operations completing in issue order, the two threads' operations in
no fixed order), and two softmax warpgroups that take turns on the MUFU pipe.  This
test replays that protocol as a discrete-event model under random schedules (TMA
completions and the two tensor-pipe streams interleaved arbitrarily) and checks:

* no schedule deadlocks;
* every parity wait is satisfied by exactly the completion it means -- the barrier is
  never two phases ahead or one behind when the parity is tested;
* every MMA reads the intended Q tile, K / V block and P block, and no ring slot, S
  buffer or O accumulator is overwritten while a reader still needs it.

Mistakes planted in the model (a missing wait, a wrong phase index) must be caught.
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


# the kernel's barrier arrays: (name, entries, arrivals per phase); one model agent
# stands for a whole warpgroup, so 128-thread barriers count one arrival per agent
BARS = [("q_full", 2, 1), ("q_empty", 2, 2), ("k_full", 2, 1), ("v_full", 2, 1),
        ("s_full", 4, 1), ("p_ready", 4, 1), ("o_done", 4, 1), ("o_free", 1, 2),
        ("xch", 2, 2), ("turn", 2, 1)]


def simulate(nblk, ntile, seed, plant=None):
    """One random schedule of a CTA with ``ntile`` tiles of ``nblk`` key blocks;
    returns the list of violations (empty when the protocol held)."""
    rnd = random.Random(seed)
    B = {(n, i): _Bar(f"{n}[{i}]", a) for n, c, a in BARS for i in range(c)}
    total = nblk * ntile
    st = {"q": [None, None], "k": [None, None], "v": [None, None], "kread": [0, 0],
          "vread": [0, 0], "S": [[None, None], [None, None]], "P": [[None, None], [None, None]],
          "O_pv": [-1, -1], "readers": {}}
    pipes, tma, errors = [[], []], [], []

    def wait(name, idx, k):
        """Wait for completion ``k`` of barrier ``name[idx]`` by its parity."""
        if plant == "phase_off_by_one" and name == "turn":
            k += 1
        b = B[(name, idx)]
        while True:
            if b.done >= k + 2 or b.done < k:
                errors.append(f"{b.name}: waiting for completion {k} at {b.done}")
                raise StopIteration
            if (b.done & 1) != (k & 1):
                return
            yield

    def producer():
        def load_q(it):
            s = it & 1
            if it >= 2:
                yield from wait("q_empty", s, it // 2 - 1)
            tma.append((("q_full", s), lambda: st["q"].__setitem__(s, it)))

        def load_k(g):
            it, j = divmod(g, nblk)
            if j == 0:
                yield from load_q(it)
            s = g & 1
            if g >= 2:
                for h in range(2):
                    yield from wait("s_full", 2 * h + s, g // 2 - 1)
            tma.append((("k_full", s), lambda: (st["kread"][s] and errors.append(f"K({g}) over a live slot"),
                                                st["k"].__setitem__(s, g))))

        def load_v(g):
            s = g & 1
            if g >= 2:
                for h in range(1 if plant == "v_reuse_one_half" else 2):
                    yield from wait("o_done", 2 * h + s, g // 2 - 1)
            tma.append((("v_full", s), lambda: (st["vread"][s] and errors.append(f"V({g}) over a live slot"),
                                                st["v"].__setitem__(s, g))))

        gk = 0
        for _ in range(2):
            yield from load_k(gk)
            gk += 1
        for gv in range(total):
            yield from load_v(gv)
            if gk < total:
                yield from load_k(gk)
                gk += 1

    def mma(h):
        pipe = pipes[h]

        def issue_s(g):
            it, j = divmod(g, nblk)
            s = g & 1
            if j == 0:
                yield from wait("q_full", it & 1, it // 2)
            yield from wait("k_full", s, g // 2)
            st["kread"][s] += 1

            def op():
                st["kread"][s] -= 1
                if st["q"][it & 1] != it:
                    errors.append(f"S_{h}({g}) reads the wrong Q tile")
                if st["k"][s] != g:
                    errors.append(f"S_{h}({g}) reads the wrong K block")
                prev = st["S"][s][h]
                if prev is not None and prev[1] != "consumed":
                    errors.append(f"S_{h}({g}) overwrites live scores {prev}")
                st["S"][s][h] = [g, "fresh"]
            pipe.append(("op", op))
            pipe.append(("commit", ("s_full", 2 * h + s)))
            if j == nblk - 1:
                pipe.append(("commit", ("q_empty", it & 1)))

        def issue_pv(g):
            it, j = divmod(g, nblk)
            s = g & 1
            if j == 0 and it > 0:
                yield from wait("o_free", 0, it - 1)
            yield from wait("v_full", s, g // 2)
            if plant != "no_p_wait":
                yield from wait("p_ready", 2 * h + s, g // 2)
            st["vread"][s] += 1

            def op():
                st["vread"][s] -= 1
                if st["v"][s] != g:
                    errors.append(f"PV_{h}({g}) reads the wrong V block")
                if st["P"][s][h] != g:
                    errors.append(f"PV_{h}({g}) reads P {st['P'][s][h]}")
                if j == 0 and it > 0 and st["readers"].get(it - 1) != {0, 1}:
                    errors.append(f"PV_{h}({g}) overwrites O still being read")
                st["O_pv"][h] = g
                st["P"][s][h] = "used"
                st["S"][s][h][1] = "consumed"
            pipe.append(("op", op))
            pipe.append(("commit", ("o_done", 2 * h + s)))

        gs = 0
        for _ in range(2):
            yield from issue_s(gs)
            gs += 1
        for gp in range(total):
            yield from issue_pv(gp)
            if gs < total:
                yield from issue_s(gs)
                gs += 1

    def softmax(h):
        for g in range(total):
            it, j = divmod(g, nblk)
            s = g & 1
            yield from wait("s_full", 2 * h + s, g // 2)
            if st["S"][s][h] is None or st["S"][s][h][0] != g:
                errors.append(f"softmax_{h}({g}) reads scores {st['S'][s][h]}")
            yield
            if j > 0 and rnd.random() < 0.3:          # a lazy rescale of O_h
                yield from wait("o_done", 2 * h + ((g - 1) & 1), (g - 1) // 2)
                if st["O_pv"][h] != g - 1:
                    errors.append(f"rescale_{h}({g}) sees O_{h} at block {st['O_pv'][h]}")
                yield
            if h == 0 and g > 0:
                yield from wait("turn", 1, g - 1)
            if h == 1:
                yield from wait("turn", 0, g)
            yield
            B[("turn", h)].arrive()
            st["P"][s][h] = g
            B[("p_ready", 2 * h + s)].arrive()
            yield
            if j == nblk - 1:
                if plant != "no_epilogue_wait":
                    yield from wait("o_done", 2 * h + s, g // 2)
                B[("xch", it & 1)].arrive()
                yield from wait("xch", it & 1, it // 2)
                if st["O_pv"] != [g, g]:
                    errors.append(f"epilogue_{h}({g}) reads O at blocks {st['O_pv']}")
                yield
                st["readers"].setdefault(it, set()).add(h)
                B[("o_free", 0)].arrive()

    agents = [producer(), mma(0), mma(1), softmax(0), softmax(1)]
    alive = list(range(len(agents)))
    stall = 0
    while alive or pipes[0] or pipes[1] or tma:
        choices = ([("agent", i) for i in alive] + [("pipe", k) for k in (0, 1) if pipes[k]]
                   + ([("tma", 0)] if tma else []))
        kind, i = rnd.choice(choices)
        if kind == "pipe":
            what, x = pipes[i].pop(0)
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


CASES = [(nblk, ntile) for nblk in (2, 3, 5) for ntile in (1, 2, 3)]


def test_protocol_holds_under_random_schedules():
    for nblk, ntile in CASES:
        for seed in range(60):
            errs = simulate(nblk, ntile, seed)
            assert not errs, (nblk, ntile, seed, errs[:2])


@pytest.mark.parametrize("plant", ["no_p_wait", "no_epilogue_wait", "v_reuse_one_half",
                                   "phase_off_by_one"])
def test_planted_protocol_mistakes_are_caught(plant):
    caught = sum(bool(simulate(nblk, ntile, seed, plant)) for nblk, ntile in CASES for seed in range(20))
    assert caught > 0, plant
