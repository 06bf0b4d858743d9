"""CPU simulation of the mbarrier protocols of the ring-based kernels.

A discrete-event model of `k_enc_gemm` (fmd_enc_gemm.cu), `k_enc_attn`
(fmd_enc_attn.cu), the decoder's persistent `k_lm_head` ring with G
consumer groups (fmd_gemv.cu), the tensor-core lm_head `k_lm_head_tc`
(fmd_lm_head_tc.cu: converter groups, passes of two stages) and the Q8_0
converter hand-off of the projection GEMM `k_proj_tc` (fmd_proj_tc.cu):
every role (TMA producer, MMA issuer, epilogue / softmax
warps) runs as a coroutine, asynchronous work (TMA copies landing, MMA groups
completing and their tcgen05.commit arrivals) completes at random later
times, and the scheduler interleaves everything in random order. The model
follows the PTX semantics of a parity wait: `try_wait.parity(P)` succeeds
when the barrier's current (incomplete) phase has parity != P. Checked on
every interleaving:
  * no wait succeeds on an aliased phase (the phase it means has completed);
  * no wait falls two phases behind (which would never succeed on hardware);
  * no buffer (ring stage, accumulator, S / P / O tile) is overwritten while
    its previous contents are still to be read, and every read sees the
    contents of the step it expects;
  * the run finishes (no deadlock).
"""

from __future__ import annotations

import random

import pytest


class Bar:
    """An mbarrier: `count` arrivals plus transaction bytes complete a phase."""

    def __init__(self, name, count):
        self.name, self.count, self.pending, self.tx, self.done = name, count, count, 0, 0

    def arrive(self, expect_tx=0):
        self.tx += expect_tx
        self.pending -= 1
        assert self.pending >= 0, f"{self.name}: too many arrivals"
        self._flip()

    def complete_tx(self, n):
        self.tx -= n
        self._flip()

    def _flip(self):
        if self.pending == 0 and self.tx == 0:
            self.done += 1
            self.pending = self.count

    def try_wait(self, phase):
        """Wait for phase index `phase` with its parity, as the kernels do."""
        ok = (self.done & 1) != (phase & 1)
        if ok:
            assert self.done >= phase + 1, f"{self.name}: parity alias (waited phase {phase}, {self.done} done)"
        else:
            assert self.done <= phase + 1, f"{self.name}: waiter fell behind (phase {phase}, {self.done} done)"
        return ok


class Sim:
    """`hold`: tags of asynchronous completions (copy landings) that the
    scheduler keeps back for as long as anything else can run, the worst
    case of out-of-order landing."""

    def __init__(self, seed, hold=()):
        self.rng = random.Random(seed)
        self.roles = []
        self.events = []  # pending asynchronous completions (callables)
        self.hold = set(hold)
        self.held = set()  # ids of pending events that carry a held tag

    def spawn(self, gen):
        self.roles.append([gen, None])

    def later(self, fn, tag=None):
        if tag is not None and tag in self.hold:
            self.held.add(id(fn))
        self.events.append(fn)

    def run(self, limit=2_000_000):
        for _ in range(limit):
            live = [r for r in self.roles if r[0] is not None]
            if not live and not self.events:
                return
            choices = []
            for r in live:
                cond = r[1]
                if cond is None or cond():
                    choices.append(("role", r))
            free = [i for i, f in enumerate(self.events) if id(f) not in self.held]
            if choices or free:
                choices += [("event", i) for i in free]
            else:
                choices = [("event", i) for i in range(len(self.events))]
            assert choices, "deadlock: every role waits and nothing is in flight"
            kind, x = self.rng.choice(choices)
            if kind == "event":
                self.events.pop(x)()
            else:
                try:
                    x[1] = next(x[0])
                except StopIteration:
                    x[0] = None
        raise AssertionError("simulation did not finish")


class Buf:
    """A buffer whose contents are tagged; writers must find it released."""

    def __init__(self, name):
        self.name, self.tag, self.readers = name, None, 0

    def write(self, tag):
        assert self.readers == 0, f"{self.name}: overwritten while {self.readers} reads are pending"
        self.tag = tag

    def check(self, tag):
        assert self.tag == tag, f"{self.name}: read {self.tag}, expected {tag}"


# ---- k_enc_gemm ----------------------------------------------------------------------------
def gemm_protocol(sim, stages, n_tiles, nk, epi_warps=8, bug=None):
    """`bug` plants a protocol mistake in the model (to show the checks bite):
    "acc_early" waits one accumulator release too early, "ring_early" one
    ring release too early."""
    full = [Bar(f"full{s}", 1) for s in range(stages)]
    empty = [Bar(f"empty{s}", 1) for s in range(stages)]
    acc_full = [Bar(f"acc_full{b}", 1) for b in range(2)]
    acc_empty = [Bar(f"acc_empty{b}", epi_warps) for b in range(2)]
    ring = [Buf(f"stage{s}") for s in range(stages)]
    acc = [Buf(f"acc{b}") for b in range(2)]
    STAGE = 48 * 1024

    def producer():
        g = 0
        for t in range(n_tiles):
            for kb in range(nk):
                st = g % stages
                if g >= stages:
                    ph = g // stages - 1  # wait parity ((g / S) + 1) & 1 == the release of use g - S
                    if bug == "ring_early":
                        ph -= 1
                    yield lambda b=empty[st], p=ph: b.try_wait(p)
                full[st].arrive(expect_tx=STAGE)

                def land(st=st, tag=(t, kb)):
                    ring[st].write(tag)
                    full[st].complete_tx(STAGE)
                sim.later(land)
                g += 1

    pending = []  # completions of issued MMA groups; MMAs of one thread complete in issue order

    def drain_one():
        pending.pop(0)()

    def submit(fn):
        pending.append(fn)
        sim.later(drain_one)

    def mma():
        g = 0
        for i in range(n_tiles):
            buf = i & 1
            if i >= 2:
                ph = (i >> 1) - 1 + (1 if bug == "acc_early" else 0)
                yield lambda b=acc_empty[buf], p=ph: b.try_wait(p)
            acc[buf].write(("acc", i))  # the tile's first MMA overwrites the accumulator
            for kb in range(nk):
                st = g % stages
                yield lambda b=full[st], p=g // stages: b.try_wait(p)
                ring[st].check((i, kb))
                ring[st].readers += 1

                def mma_done(st=st):
                    ring[st].readers -= 1
                    empty[st].arrive()  # tcgen05.commit -> empty[st]
                submit(mma_done)
                g += 1
            submit(lambda buf=buf: acc_full[buf].arrive())  # commit after the k-loop

    def epilogue(w):
        for i in range(n_tiles):
            buf = i & 1
            yield lambda b=acc_full[buf], p=i >> 1: b.try_wait(p)
            acc[buf].check(("acc", i))
            acc[buf].readers += 1
            yield None  # tcgen05.ld + processing
            acc[buf].readers -= 1
            acc_empty[buf].arrive()

    sim.spawn(producer())
    sim.spawn(mma())
    for w in range(epi_warps):
        sim.spawn(epilogue(w))


@pytest.mark.parametrize("seed", range(40))
@pytest.mark.parametrize("stages,n_tiles,nk", [(4, 5, 16), (4, 3, 1), (6, 4, 3), (4, 1, 64), (2, 6, 5)])
def test_enc_gemm_protocol(seed, stages, n_tiles, nk):
    sim = Sim(seed * 7919 + stages * 31 + n_tiles * 17 + nk)
    gemm_protocol(sim, stages, n_tiles, nk)
    sim.run()


@pytest.mark.parametrize("bug", ["acc_early", "ring_early"])
def test_the_simulation_catches_a_planted_protocol_mistake(bug):
    failures = 0
    for seed in range(20):
        sim = Sim(seed)
        gemm_protocol(sim, 4, 5, 16, bug=bug)
        try:
            sim.run()
        except AssertionError:
            failures += 1
    assert failures == 20


# ---- k_enc_attn -----------------------------------------------------------------------------
def attn_protocol(sim, stages, n_tiles, rescale_at):
    """One CTA: producer (Q, then K/V tiles into a ring), MMA issuer (S_j = QK_j^T
    into S[j & 1], then PV_{j-1}), 128 softmax threads modelled as one role per
    warp (4) since each barrier counts 128 arrivals: a warp arrives 32 times.
    (The model also shows that the s_empty and p_empty waits are implied by the
    issue order -- PV_{j-2} waits for softmax j-2 before S_j is issued, and MMAs
    complete in issue order -- so they never block; the kernel keeps them as
    explicit guards.)"""
    q_full = Bar("q_full", 1)
    kv_full = [Bar(f"kv_full{s}", 1) for s in range(stages)]
    kv_empty = [Bar(f"kv_empty{s}", 1) for s in range(stages)]
    s_full = [Bar(f"s_full{b}", 1) for b in range(2)]
    s_empty = [Bar(f"s_empty{b}", 128) for b in range(2)]
    p_full = [Bar(f"p_full{b}", 128) for b in range(2)]
    p_empty = [Bar(f"p_empty{b}", 1) for b in range(2)]
    o_full, o_final = Bar("o_full", 1), Bar("o_final", 1)
    kv = [Buf(f"kv{s}") for s in range(stages)]
    S = [Buf(f"S{b}") for b in range(2)]
    P = [Buf(f"P{b}") for b in range(2)]
    O = Buf("O")
    inflight = []  # MMA groups in issue order; each completes only after its predecessors

    def issue(group_tag, reads, on_done):
        for b in reads:
            b.readers += 1
        inflight.append(group_tag)

        def done():
            assert inflight[0] == group_tag, "MMA groups complete in issue order"
            inflight.pop(0)
            for b in reads:
                b.readers -= 1
            on_done()
        return done

    def producer():
        q_full.arrive(expect_tx=1)
        sim.later(lambda: q_full.complete_tx(1))
        for j in range(n_tiles):
            st = j % stages
            if j >= stages:
                yield lambda b=kv_empty[st], p=j // stages - 1: b.try_wait(p)
            kv_full[st].arrive(expect_tx=2)

            def land(st=st, j=j):
                kv[st].write(("kv", j))
                kv_full[st].complete_tx(2)
            sim.later(land)

    pending = []  # completions of issued MMA groups, run strictly in issue order

    def drain_one():
        pending.pop(0)()

    def submit(fn):
        pending.append(fn)
        sim.later(drain_one)

    def mma():
        yield lambda: q_full.try_wait(0)

        def pv(i):
            pb = i & 1
            yield lambda b=p_full[pb], p=i >> 1: b.try_wait(p)
            P[pb].check(("P", i))
            st = i % stages
            kv[st].check(("kv", i))
            O.write(("O", i))

            def fin(pb=pb, st=st):
                o_full.arrive()
                p_empty[pb].arrive()
                kv_empty[st].arrive()
            submit(issue(("pv", i), [P[pb], kv[st]], fin))

        for j in range(n_tiles):
            st, sb = j % stages, j & 1
            yield lambda b=kv_full[st], p=j // stages: b.try_wait(p)
            if j >= 2:
                yield lambda b=s_empty[sb], p=(j >> 1) - 1: b.try_wait(p)
            kv[st].check(("kv", j))
            S[sb].write(("S", j))
            submit(issue(("s", j), [kv[st]], lambda sb=sb: s_full[sb].arrive()))
            if j >= 1:
                yield from pv(j - 1)
        yield from pv(n_tiles - 1)
        submit(issue(("final",), [], lambda: o_final.arrive()))

    def softmax(w):
        for j in range(n_tiles):
            sb = j & 1
            yield lambda b=s_full[sb], p=j >> 1: b.try_wait(p)
            S[sb].check(("S", j))
            S[sb].readers += 1
            yield None  # tcgen05.ld of the S tile
            S[sb].readers -= 1
            for _ in range(32):
                s_empty[sb].arrive()
            rescaling = j in rescale_at
            if rescaling:  # O of PVs 0 .. j-1 is rescaled in tensor memory (load, scale, store)
                yield lambda p=j - 1: o_full.try_wait(p)
                O.check(("O", j - 1))
                O.readers += 1
            if j >= 2:
                yield lambda b=p_empty[sb], p=(j - 2) >> 1: b.try_wait(p)
            P[sb].write(("P", j))
            if rescaling:
                O.readers -= 1  # tcgen05.st of the rescaled O waited before P is published
            for _ in range(32):
                p_full[sb].arrive()
        yield lambda: o_final.try_wait(0)
        O.check(("O", n_tiles - 1))

    sim.spawn(producer())
    sim.spawn(mma())
    for w in range(4):
        sim.spawn(softmax(w))


@pytest.mark.parametrize("seed", range(40))
@pytest.mark.parametrize("stages,n_tiles,rescale", [(3, 24, (1, 5, 23)), (3, 1, ()), (3, 2, (1,)), (3, 7, (2, 3, 4))])
def test_enc_attn_protocol(seed, stages, n_tiles, rescale):
    sim = Sim(seed * 104729 + n_tiles * 13 + len(rescale))
    attn_protocol(sim, stages, n_tiles, set(rescale))
    sim.run()


# ---- k_lm_head (decoder) ------------------------------------------------------------------
def lm_head_protocol(sim, G, stages, my_tiles, nkb, warps=8, layout="per_group"):
    """`k_lm_head`'s ring. The producer interleaves the k-blocks of G tiles
    (tile G*p + j is group j's p-th tile, so its k-block kb is the group's
    unit q = p*nkb + kb). `layout="per_group"` (the kernel): group j's unit q
    uses stage j*S/G + q % (S/G) in phase q // (S/G). `layout="shared"` (the
    earlier design): the u-th copy in issue order uses stage u % S in phase
    u // S, so with an odd tile count the groups share stages."""
    full = [Bar(f"full{s}", 1) for s in range(stages)]
    empty = [Bar(f"empty{s}", warps) for s in range(stages)]  # one group of 8 warps consumes a stage
    ring = [Buf(f"stage{s}") for s in range(stages)]
    sg = stages // G
    order = []  # (tile, kb) in issue order
    for p in range((my_tiles + G - 1) // G):
        in_grp = min(G, my_tiles - G * p)
        for kb in range(nkb):
            for j in range(in_grp):
                order.append((G * p + j, kb))

    def slot(u, tile, kb):
        if layout == "shared":
            return u % stages, u // stages
        q = (tile // G) * nkb + kb
        return (tile % G) * sg + q % sg, q // sg

    where = {tag: slot(u, *tag) for u, tag in enumerate(order)}
    uses = {}  # stage -> phases in issue order
    for tag in order:
        st, ph = where[tag]
        uses.setdefault(st, []).append(ph)
    for st, phs in uses.items():  # every stage cycles through consecutive phases
        assert phs == list(range(len(phs))), (layout, st, phs)

    def producer():
        for tag in order:
            st, ph = where[tag]
            if ph > 0:
                yield lambda b=empty[st], p=ph - 1: b.try_wait(p)
            full[st].arrive(expect_tx=1)

            def land(st=st, tag=tag):
                ring[st].write(tag)
                full[st].complete_tx(1)
            sim.later(land, tag=tag)

    def consumer(g, w):
        for i in range(g, my_tiles, G):
            for kb in range(nkb):
                st, ph = where[(i, kb)]
                yield lambda b=full[st], p=ph: b.try_wait(p)
                ring[st].check((i, kb))
                ring[st].readers += 1
                yield None  # the warp's fragment to registers
                ring[st].readers -= 1
                empty[st].arrive()

    sim.spawn(producer())
    for g in range(G):
        for w in range(warps):
            sim.spawn(consumer(g, w))


# The stage counts the launcher picks: Q8_0 16 (both variants), dense 8 for two
# groups (rounded down to a multiple of G) and 5 for one; a CTA owns 8 or 9 of
# the 1,187 vocabulary tiles on 148 SMs.
@pytest.mark.parametrize("seed", range(20))
@pytest.mark.parametrize("G,stages,my_tiles", [(2, 16, 8), (2, 16, 9), (2, 8, 8), (2, 8, 9), (2, 8, 1),
                                               (1, 16, 8), (1, 5, 9), (1, 5, 1)])
def test_lm_head_ring_protocol(seed, G, stages, my_tiles):
    sim = Sim(seed * 31 + G * 7 + stages * 3 + my_tiles)
    lm_head_protocol(sim, G, stages, my_tiles, nkb=16)
    sim.run()


def _last_tile_held_copy(G, stages, my_tiles, nkb):
    """The tag of the copy whose late landing exposes a shared ring: the first
    k-block group 0 streams alone for an odd last tile lands in a stage group
    1 used last; holding back the copy 7 units before it (in issue order)
    lets group 0 reach that stage while the other group's phase is open."""
    order = []
    for p in range((my_tiles + G - 1) // G):
        in_grp = min(G, my_tiles - G * p)
        for kb in range(nkb):
            for j in range(in_grp):
                order.append((G * p + j, kb))
    base = (my_tiles // G) * G * nkb  # first unit of the last (odd) tile
    return order[base - 7]


@pytest.mark.parametrize("seed", range(50))
@pytest.mark.parametrize("stages,nkb", [(16, 16), (8, 16)])
def test_per_group_rings_survive_a_late_copy(seed, stages, nkb):
    """With one copy held back until nothing else can run, the per-group
    rings of the kernel still never alias, for an odd tile count too."""
    held = _last_tile_held_copy(2, stages, 9, nkb)
    sim = Sim(seed, hold=[held])
    lm_head_protocol(sim, 2, stages, 9, nkb=nkb, layout="per_group")
    sim.run()


def test_a_shared_ring_aliases_under_a_late_copy():
    """The same schedule breaks the earlier shared-ring layout (stage u % S
    over the interleaved issue order): with 9 tiles the last tile's k-blocks
    reach stages the other group used last, and a wait passes on the other
    group's phase. The check must bite, or the passing test above proves
    nothing."""
    hits = 0
    for seed in range(50):
        sim = Sim(seed, hold=[_last_tile_held_copy(2, 16, 9, 16)])
        lm_head_protocol(sim, 2, 16, 9, nkb=16, layout="shared")
        try:
            sim.run()
        except AssertionError as e:
            assert "alias" in str(e) or "overwritten" in str(e) or "read" in str(e), e
            hits += 1
    assert hits > 0


def test_an_odd_stage_count_with_a_shared_ring_is_a_hazard():
    """The shared layout with 9 stages: consecutive uses of a stage alternate
    between the two groups and random landing orders already alias."""
    hits = 0
    for seed in range(300):
        sim = Sim(seed)
        lm_head_protocol(sim, 2, 9, 8, nkb=16, layout="shared")
        try:
            sim.run()
        except AssertionError:
            hits += 1
    assert hits > 0


# ---- k_lm_head_tc ---------------------------------------------------------------------------
def lm_head_tc_protocol(sim, NR, my_tiles, nkb, bug=None):
    """`k_lm_head_tc` (fmd_lm_head_tc.cu) on one CTA: a producer streams the
    packed stages into RAW ring slots; NG groups of 4 converter warps take
    stages g = grp, grp + NG, ... into CONV A slots; the MMA warp works in
    passes of two stages (p = g / 2), waiting for both stages' conv_full and,
    from the AP-th pass on, for acc_empty of pass p - AP, then one commit
    frees the pass's A slots (conv_free[p % CP]) and one hands over its
    accumulators (acc_full[p % AP]); 8 epilogue warps, four per stage
    parity, read a stage's accumulators and release the pass on
    acc_empty[p % AP] (count 8). Converters refill slot c of pass p only
    after conv_free of pass p - CP. `bug` plants a mistake: "conv_free_early"
    (a converter waits one release too early) or "acc_early" (the MMA warp
    waits one accumulator release too early)."""
    RAW, CONV, NG = (8, 4, 2) if NR == 32 else (4, 2, 1)
    ACC = 512 // NR
    AP, CP = ACC // 4, CONV // 2
    n_stages = my_tiles * nkb
    assert n_stages % 2 == 0 and nkb % 2 == 0
    full = [Bar(f"full{s}", 1) for s in range(RAW)]
    empty = [Bar(f"empty{s}", 4) for s in range(RAW)]
    conv_full = [Bar(f"conv_full{c}", 4) for c in range(CONV)]
    conv_free = [Bar(f"conv_free{q}", 1) for q in range(CP)]
    acc_full = [Bar(f"acc_full{r}", 1) for r in range(AP)]
    acc_empty = [Bar(f"acc_empty{r}", 8) for r in range(AP)]
    raw = [Buf(f"raw{s}") for s in range(RAW)]
    conv = [Buf(f"conv{c}") for c in range(CONV)]
    acc = [Buf(f"acc{r}") for r in range(AP)]

    def producer():
        for g in range(n_stages):
            s = g % RAW
            if g >= RAW:
                yield lambda b=empty[s], p=g // RAW - 1: b.try_wait(p)
            full[s].arrive(expect_tx=1)

            def land(s=s, g=g):
                raw[s].write(g)
                full[s].complete_tx(1)
            sim.later(land, tag=g)

    def converter(grp, w):
        for g in range(grp, n_stages, NG):
            s, c, p = g % RAW, g % CONV, g // 2
            if p >= CP:
                ph = p // CP - 1 - (1 if bug == "conv_free_early" else 0)
                if ph >= 0:
                    yield lambda b=conv_free[p % CP], q=ph: b.try_wait(q)
            yield lambda b=full[s], q=g // RAW: b.try_wait(q)
            raw[s].check(g)
            raw[s].readers += 1
            yield None  # fragments to registers
            raw[s].readers -= 1
            empty[s].arrive()
            conv[c].write(g)  # this warp's rows of the A tile
            yield None
            conv_full[c].arrive()

    pending = []

    def drain_one():
        pending.pop(0)()

    def mma():
        for g in range(0, n_stages, 2):
            p = g // 2
            yield lambda b=conv_full[g % CONV], q=g // CONV: b.try_wait(q)
            yield lambda b=conv_full[(g + 1) % CONV], q=(g + 1) // CONV: b.try_wait(q)
            if p >= AP:
                ph = p // AP - 1 - (1 if bug == "acc_early" else 0)
                if ph >= 0:
                    yield lambda b=acc_empty[p % AP], q=ph: b.try_wait(q)
            conv[g % CONV].check(g)
            conv[(g + 1) % CONV].check(g + 1)
            conv[g % CONV].readers += 1
            conv[(g + 1) % CONV].readers += 1
            acc[p % AP].write(p)

            def done(g=g, p=p):
                conv[g % CONV].readers -= 1
                conv[(g + 1) % CONV].readers -= 1
                conv_free[p % CP].arrive()
                acc_full[p % AP].arrive()
            pending.append(done)
            sim.later(drain_one)

    def epilogue(par, w):
        for i in range(my_tiles):
            for kb in range(par, nkb, 2):
                g = i * nkb + kb
                p = g // 2
                yield lambda b=acc_full[p % AP], q=p // AP: b.try_wait(q)
                acc[p % AP].check(p)
                acc[p % AP].readers += 1
                yield None  # tcgen05.ld of the stage's two accumulators
                acc[p % AP].readers -= 1
                acc_empty[p % AP].arrive()
            yield None  # the tile's logits and per-row best (named barriers)

    sim.spawn(producer())
    for grp in range(NG):
        for w in range(4):
            sim.spawn(converter(grp, w))
    sim.spawn(mma())
    for par in range(2):
        for w in range(4):
            sim.spawn(epilogue(par, w))


@pytest.mark.parametrize("seed", range(25))
@pytest.mark.parametrize("NR,my_tiles,nkb", [(32, 9, 16), (32, 8, 16), (32, 1, 2), (64, 9, 16), (64, 2, 4)])
def test_lm_head_tc_protocol(seed, NR, my_tiles, nkb):
    sim = Sim(seed * 131 + NR + my_tiles * 7 + nkb)
    lm_head_tc_protocol(sim, NR, my_tiles, nkb)
    sim.run()


@pytest.mark.parametrize("seed", range(10))
def test_lm_head_tc_protocol_survives_a_late_copy(seed):
    """One copy held back until nothing else can run (the converter group of
    its stage stalls, the other group and the MMA passes run ahead as far as
    the slots allow): no alias, no overwrite, no deadlock."""
    sim = Sim(seed, hold=[37])
    lm_head_tc_protocol(sim, 32, 4, 16)
    sim.run()


@pytest.mark.parametrize("bug", ["conv_free_early", "acc_early"])
def test_the_lm_head_tc_model_catches_a_planted_mistake(bug):
    failures = 0
    for seed in range(20):
        sim = Sim(seed)
        lm_head_tc_protocol(sim, 32, 3, 16, bug=bug)
        try:
            sim.run()
        except AssertionError as e:
            assert any(k in str(e) for k in ("alias", "overwritten", "read", "behind")), e
            failures += 1
    assert failures == 20


# ---- k_proj_tc with Q8_0 weights ------------------------------------------------------------
def proj_tc_q8_protocol(sim, stages, n_tiles, nk, conv_warps=8, epi_warps=8, bug=None):
    """`k_proj_tc` (fmd_proj_tc.cu) with Q8_0 weights: the producer's copy of
    a stage brings the activation tile and the int8 weight tile (full[st]);
    `conv_warps` converter warps each write their rows of the stage's 16-bit
    B tile and arrive on conv[st]; the MMA warp waits on both full[st] and
    conv[st], and its commit frees the stage (empty[st]) for the producer,
    whose next copy into that stage is what lets the converters overwrite
    its B tile; two accumulators hand tiles to the epilogue. `bug`:
    "conv_skip" (the MMA warp does not wait for the converters)."""
    full = [Bar(f"full{s}", 1) for s in range(stages)]
    empty = [Bar(f"empty{s}", 1) for s in range(stages)]
    conv = [Bar(f"conv{s}", conv_warps) for s in range(stages)]
    acc_full = [Bar(f"acc_full{b}", 1) for b in range(2)]
    acc_empty = [Bar(f"acc_empty{b}", epi_warps) for b in range(2)]
    ring = [Buf(f"stage{s}") for s in range(stages)]
    btile = [[Buf(f"b{s}.{w}") for w in range(conv_warps)] for s in range(stages)]
    acc = [Buf(f"acc{b}") for b in range(2)]

    def producer():
        g = 0
        for t in range(n_tiles):
            for kb in range(nk):
                st = g % stages
                if g >= stages:
                    yield lambda b=empty[st], p=g // stages - 1: b.try_wait(p)
                full[st].arrive(expect_tx=1)

                def land(st=st, tag=(t, kb)):
                    ring[st].write(tag)
                    full[st].complete_tx(1)
                sim.later(land)
                g += 1

    def converter(w):
        g = 0
        for t in range(n_tiles):
            for kb in range(nk):
                st = g % stages
                yield lambda b=full[st], p=g // stages: b.try_wait(p)
                ring[st].check((t, kb))
                btile[st][w].write((t, kb))  # this warp's rows of the 16-bit B tile
                yield None
                conv[st].arrive()
                g += 1

    pending = []

    def drain_one():
        pending.pop(0)()

    def mma():
        g = 0
        for i in range(n_tiles):
            buf = i & 1
            if i >= 2:
                yield lambda b=acc_empty[buf], p=(i >> 1) - 1: b.try_wait(p)
            acc[buf].write(("acc", i))
            for kb in range(nk):
                st = g % stages
                yield lambda b=full[st], p=g // stages: b.try_wait(p)
                if bug != "conv_skip":
                    yield lambda b=conv[st], p=g // stages: b.try_wait(p)
                ring[st].check((i, kb))
                for w in range(conv_warps):
                    btile[st][w].check((i, kb))
                    btile[st][w].readers += 1
                ring[st].readers += 1

                def done(st=st):
                    ring[st].readers -= 1
                    for w in range(conv_warps):
                        btile[st][w].readers -= 1
                    empty[st].arrive()
                pending.append(done)
                sim.later(drain_one)
                g += 1
            pending.append(lambda buf=buf: acc_full[buf].arrive())
            sim.later(drain_one)

    def epilogue(w):
        for i in range(n_tiles):
            buf = i & 1
            yield lambda b=acc_full[buf], p=i >> 1: b.try_wait(p)
            acc[buf].check(("acc", i))
            acc[buf].readers += 1
            yield None
            acc[buf].readers -= 1
            acc_empty[buf].arrive()

    sim.spawn(producer())
    for w in range(conv_warps):
        sim.spawn(converter(w))
    sim.spawn(mma())
    for w in range(epi_warps):
        sim.spawn(epilogue(w))


@pytest.mark.parametrize("seed", range(25))
@pytest.mark.parametrize("stages,n_tiles,nk", [(3, 4, 16), (5, 3, 16), (3, 1, 2), (5, 6, 4)])
def test_proj_tc_q8_protocol(seed, stages, n_tiles, nk):
    sim = Sim(seed * 17 + stages * 5 + n_tiles * 3 + nk)
    proj_tc_q8_protocol(sim, stages, n_tiles, nk)
    sim.run()


def test_the_proj_tc_model_catches_a_skipped_converter_wait():
    failures = 0
    for seed in range(20):
        sim = Sim(seed)
        proj_tc_q8_protocol(sim, 3, 3, 16, bug="conv_skip")
        try:
            sim.run()
        except AssertionError as e:
            assert "read" in str(e) or "overwritten" in str(e), e
            failures += 1
    assert failures == 20
