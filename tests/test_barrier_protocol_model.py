"""A model of the TMA kernel's ring protocol (paia-project_b200/csrc/gemv_tma.cuh) under bounded waits that give up,
checked on the CPU with random interleavings. An mbarrier phase completes when its pending arrivals reach zero and its
transaction (byte) count is zero; one more arrival on a phase that already sits at zero pending arrivals - possible
only for the byte-counted `full` barriers, whose phase waits there for its bytes - would take the count below zero.
The kernel's rules, modelled here: the producer's lane 0 arms a slot's `full` barrier (arrival + expected bytes) only
after its wait on the slot's `empty` barrier succeeded, and arrives on nothing after its first failed wait; the other
producer lanes issue the slot's copies (bytes that land later) and learn lane 0's failure one stage late (a shared
flag read at the end of each stage, BF16 / FP8; INT4 lanes, whose metadata copies arrive on `full` too, take lane 0's
status by a shuffle of the same stage before they arrive); a consumer warp waits on `full`, and releases the slot on `empty`
only while every `full` wait of its own has seen the phase complete. Any wait may give up while its phase is
incomplete. Checked: no arrival ever lands on a phase at zero pending arrivals, and no byte count leaves the
barrier's range. The model also shows that the earlier, unguarded rules (consumers release after a failed wait) break
the first check, so the test can tell the two apart."""
import random

TX_LIMIT = (1 << 20) - 1


class Barrier:
    def __init__(self, count):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0
        self.bad = None

    def _complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, tx=0):
        if self.pending == 0:
            self.bad = self.bad or "arrival on a phase at zero pending arrivals"
            return
        self.pending -= 1
        self.tx += tx
        if abs(self.tx) > TX_LIMIT:
            self.bad = self.bad or "transaction count out of range"
        self._complete()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        if abs(self.tx) > TX_LIMIT:
            self.bad = self.bad or "transaction count out of range"
        self._complete()

    def done(self, lap):
        """Phase `lap` (0-based) has completed."""
        return self.phase > lap


def run(seed, guarded=True, st=4, nc=4, stages=40, nbytes=65536, p_timeout=0.02, out=None, int4=False):
    """Returns the first broken-barrier finding (or None); out, if given, receives whether every stage was produced
    and consumed and every copy landed."""
    rng = random.Random(seed)
    # INT4: lane 0's expect-bytes arrival, the lanes' metadata cp.async arrivals (one, after their copies land) and
    # lane 0's closing arrival; BF16 / FP8: lane 0's expect-bytes arrival alone
    full = [Barrier(3 if int4 else 1) for _ in range(st)]
    empty = [Barrier(nc) for _ in range(st)]
    inflight = []                                   # (slot, bytes) copies issued, not landed
    prod_g = 0                                      # next stage the producer handles
    live0, lanes_live, stop_flag = True, True, False
    cons_g = [0] * nc
    seen = [True] * nc

    def wait(bar, lap):
        """A bounded wait: succeeds once the phase completed; may give up (at random) while it has not."""
        if bar.done(lap):
            return "ok"
        return "timeout" if rng.random() < p_timeout else "pending"

    steps = 0
    while steps < 20000 and (prod_g < stages or min(cons_g) < stages or inflight):
        steps += 1
        actor = rng.randrange(nc + 2)
        if actor == nc and prod_g < stages:                         # producer: one stage
            s, lap = prod_g % st, prod_g // st
            if guarded:
                if live0 and prod_g >= st:
                    w = wait(empty[s], lap - 1)
                    if w == "pending":
                        continue
                    if w == "timeout":                               # lane 0 stops and raises the shared flag
                        live0, stop_flag = False, True
                if live0:
                    full[s].arrive(tx=nbytes)                        # lane 0: arrival + expected bytes
                if lanes_live:                                       # the lanes' copies, with last stage's status
                    inflight.append((s, nbytes))
                if int4:
                    lanes_live = live0                              # a shuffle of lane 0's status, this stage
                    if lanes_live:
                        inflight.append((s, "arrive"))               # the lanes' cp.async arrival, when it lands
                        full[s].arrive()                             # lane 0's closing arrival
                else:
                    lanes_live = lanes_live and not stop_flag       # flag read at the end of the stage
            else:                                                    # carries on after a failed wait
                if prod_g >= st and wait(empty[s], lap - 1) == "pending":
                    continue
                full[s].arrive(tx=nbytes)
                inflight.append((s, nbytes))
                if int4:
                    inflight.append((s, "arrive"))
                    full[s].arrive()
            prod_g += 1
        elif actor == nc + 1 and inflight:                          # a copy lands
            k = rng.randrange(len(inflight))
            s, b = inflight.pop(k)
            if b == "arrive":
                full[s].arrive()
            else:
                full[s].complete_tx(b)
        elif actor < nc and cons_g[actor] < stages:                 # consumer warp: one stage
            g = cons_g[actor]
            s, lap = g % st, g // st
            if guarded and not seen[actor]:                          # a warp whose wait gave up waits no more
                cons_g[actor] += 1
                continue
            w = wait(full[s], lap)
            if w == "pending":
                continue
            ok = w == "ok"
            if guarded:
                seen[actor] = seen[actor] and ok
                if seen[actor]:
                    empty[s].arrive()
            else:
                empty[s].arrive()                                    # unguarded: releases after a failed wait
            cons_g[actor] += 1
        for b in full + empty:
            if b.bad:
                return b.bad
    if out is not None:
        out["complete"] = prod_g == stages and min(cons_g) == stages and not inflight
    return None


def test_guarded_protocol_never_breaks_a_barrier():
    for seed in range(1000):
        for p in (0.0, 0.01, 0.05, 0.3):
            assert run(seed, guarded=True, p_timeout=p) is None, (seed, p)
            assert run(seed, guarded=True, p_timeout=p, int4=True) is None, (seed, p, "int4")


def test_unguarded_protocol_is_caught():
    for int4 in (False, True):
        broken = sum(run(seed, guarded=False, p_timeout=0.05, int4=int4) is not None for seed in range(1000))
        assert broken > 0, int4


def test_no_timeouts_run_to_completion():
    """Without timeouts every stage is produced and consumed and every copy lands, both forms alike."""
    for seed in range(200):
        for guarded in (True, False):
            for int4 in (False, True):
                out = {}
                assert run(seed, guarded=guarded, p_timeout=0.0, out=out, int4=int4) is None
                assert out["complete"], (seed, guarded, int4)
