"""A model of the row-sharded tensor-parallel protocol (paia-project_b200/csrc/gemv_tma.cuh tp_enter / tp_leave /
tp_exchange_kernel, paia_gemv/tp.py), checked on the CPU with random interleavings of ranks and CTAs.

Every rank runs a stream: per call k, the TP GEMV (G CTAs; each CTA's epilogue starts only once the rank's previous
stream item has completed, as the grid-dependency wait makes it), then, in the deferred form, the exchange, then a
reader of the rank's own y. A CTA reads the rank's epoch e, counts itself among the readers, CTA 0 tells every rank
that this rank started call e + 1, the CTA waits until every other rank has started it too, and stores its rows into
every rank's y. Deferred form: CTA 0 advances the epoch once all the call's CTAs have read it; the exchange counts the
rank in on every rank's exchange block and waits for every rank's count. Complete form: every CTA counts in on every
rank; CTA 0 waits for all CTAs of every rank, then advances the epoch.

Checked at every reader: each row of y holds the value of this call from every source rank - an older value is a
store that has not landed (read-after-write), a newer one a peer's next call overwriting y while this rank still
reads it (write-after-read). The same model without the start handshake, and the deferred form without the
exchange, are caught, so the checks can tell them apart."""
import random


class Model:
    def __init__(self, world, G, calls, form, handshake=True, exchange=True, seed=0):
        self.W, self.G, self.C, self.form = world, G, calls, form
        self.handshake, self.exchange = handshake, exchange
        self.rng = random.Random(seed)
        self.epoch = [0] * world
        self.readers = [0] * world
        self.complete = [0] * world
        self.ready = [[0] * world for _ in range(world)]      # ready[at rank][from rank]
        self.arrive = [[0] * world for _ in range(world)]
        self.xepoch = [0] * world
        self.xarrive = [[0] * world for _ in range(world)]
        self.y = [[[-1] * G for _ in range(world)] for _ in range(world)]   # y[at rank][source rank][cta] = call
        self.items = []                                        # per rank: the stream of items
        for r in range(world):
            seq = []
            for k in range(calls):
                seq.append(("gemv", k))
                if form == "deferred" and exchange:
                    seq.append(("exchange", k))
                seq.append(("read", k))
            self.items.append(seq)
        self.pos = [0] * world                                 # current stream item of each rank
        self.cta = [None] * world                              # per rank: CTA states of the running GEMV
        self.error = None

    # ---- one rank's current item, advanced by one action
    def step(self, r):
        if self.pos[r] >= len(self.items[r]):
            return False
        kind, k = self.items[r][self.pos[r]]
        if kind == "gemv":
            return self.step_gemv(r, k)
        if kind == "exchange":
            return self.step_exchange(r)
        return self.step_read(r, k)

    def step_gemv(self, r, k):
        if self.cta[r] is None:
            self.cta[r] = [{"pc": 0, "e": None} for _ in range(self.G)]
        ctas = self.cta[r]
        live = [i for i, c in enumerate(ctas) if c["pc"] < 5]
        if not live:
            self.cta[r] = None
            self.pos[r] += 1
            return True
        i = self.rng.choice(live)
        c = ctas[i]
        if c["pc"] == 0:                                       # read the epoch, count in as a reader
            c["e"] = self.epoch[r]
            self.readers[r] += 1
            if i == 0:
                for q in range(self.W):
                    self.ready[q][r] += 1
            c["pc"] = 1
        elif c["pc"] == 1:                                     # wait until every other rank started call e + 1
            if self.handshake and any(self.ready[r][q] < c["e"] + 1 for q in range(self.W) if q != r):
                return False
            c["pc"] = 2
        elif c["pc"] == 2:                                     # store this CTA's rows into every rank's y
            for q in range(self.W):
                self.y[q][r][i] = k
            if self.form == "complete":
                for q in range(self.W):
                    self.arrive[q][r] += 1
            c["pc"] = 3
        elif c["pc"] == 3:                                     # leave
            if i == 0:
                if self.form == "deferred":
                    if self.readers[r] < (c["e"] + 1) * self.G:
                        return False
                else:
                    cc = self.complete[r]
                    if any(self.arrive[r][s] < (cc + 1) * self.G for s in range(self.W)):
                        return False
                    self.complete[r] = cc + 1
                self.epoch[r] = c["e"] + 1
            c["pc"] = 5
        return True

    def step_exchange(self, r):
        st = getattr(self, "_x", None)
        if st is None:
            self._x = st = [None] * self.W
        if st[r] is None:
            for q in range(self.W):
                self.xarrive[q][r] += 1
            st[r] = self.xepoch[r]
            return True
        e = st[r]
        if any(self.xarrive[r][s] < e + 1 for s in range(self.W)):
            return False
        self.xepoch[r] = e + 1
        st[r] = None
        self.pos[r] += 1
        return True

    def step_read(self, r, k):
        for s in range(self.W):
            for i in range(self.G):
                v = self.y[r][s][i]
                if v < k:
                    self.error = self.error or f"rank {r} call {k}: row of rank {s} still holds call {v}"
                elif v > k:
                    self.error = self.error or f"rank {r} call {k}: rank {s} overwrote it with call {v}"
        self.pos[r] += 1
        return True

    def run(self, max_steps=200000):
        for _ in range(max_steps):
            if self.error:
                return self.error
            pending = [r for r in range(self.W) if self.pos[r] < len(self.items[r])]
            if not pending:
                return None
            # skew: some ranks run much more often than others
            weights = [1 + 6 * (r % 2) for r in pending]
            r = self.rng.choices(pending, weights)[0]
            self.step(r)
        return self.error or "did not finish"


def test_deferred_form_is_race_free():
    for seed in range(300):
        for world in (2, 4, 8):
            assert Model(world, 3, 6, "deferred", seed=seed).run() is None, (seed, world)


def test_complete_form_is_race_free():
    for seed in range(300):
        for world in (2, 4, 8):
            assert Model(world, 3, 6, "complete", seed=seed).run() is None, (seed, world)


def test_without_the_start_handshake_a_fast_rank_overwrites():
    hits = sum("overwrote" in (Model(2, 3, 6, "complete", handshake=False, seed=s).run() or "")
               for s in range(300))
    assert hits > 0


def test_deferred_without_the_exchange_reads_stale_rows():
    hits = sum("still holds" in (Model(2, 3, 6, "deferred", exchange=False, seed=s).run() or "")
               for s in range(300))
    assert hits > 0
