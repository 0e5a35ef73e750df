"""A CPU model of the tree kernel's barrier protocol (bc_tree_mma.cuh).

Every role of one CTA — the K and V producers, the S = Q K^T issuer, the two
softmax warpgroups and the P V issuer — is a generator that waits on
mbarriers by phase parity exactly as the kernel does (same stage, buffer and
parity formulas, one-row-tile and two-row-tile variants). A random scheduler
interleaves the roles and completes asynchronous work (TMA copies, MMAs)
after random delays: TMA copies in any order, MMAs in issue order per
issuing thread (what tcgen05.commit tracks). The model checks what the kernel relies on but cannot check
itself:

* no mbarrier ever completes two phases before a waiter looks (a parity wait
  would then read "not yet" and stall — the hazard behind a real stall that
  the per-buffer P barriers fixed);
* every role finishes (no deadlock) for every tile count;
* the data dependencies hold: S of a unit after its K tile landed and after
  the PV that last read its S/P buffer; P after S; PV after P and its V tile;
  a K or V stage refilled only after every unit that reads it is done.

It also models the speculative first copies: each producer fills the first
`spec_pre` stages of its ring (at most one pass) before the prologue knows the
CTA's real key range. If the guess holds, those fills are the tiles of record;
if not, it refills the same stages and every wait on one of those stages'
full barriers looks one phase further. Either way the producers let the
prologue end only once their speculative copies have landed: no consumer can
then look at a speculated stage before its first phase is complete (a parity
wait cannot tell the phase it wants from the one before that).
"""
import random

import pytest

K_STAGES, V_STAGES, S_BUFS = 5, 6, 4  # one-row-tile CTA (two-row-tile: 4, 5)


class Barrier:
    """mbarrier with an arrival count; `phase` counts completed phases."""

    def __init__(self, name, count=1):
        self.name, self.count, self.pending, self.phase = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def ready(self, wanted):
        """Wait for completion number `wanted` (0-based) by its parity, as the
        hardware does: try_wait.parity(p) succeeds while the barrier's current
        phase has the other parity. That is the right answer only within one
        phase of the waiter; either side of that window is an error here."""
        if self.phase > wanted + 1:
            raise AssertionError(f"{self.name}: phase {self.phase} ran two ahead of a "
                                 f"waiter for completion {wanted} (parity aliasing)")
        if self.phase < wanted:
            raise AssertionError(f"{self.name}: a waiter for completion {wanted} looked while "
                                 f"the barrier was at phase {self.phase} (parity aliasing: "
                                 f"the waiter is ahead)")
        return (self.phase & 1) != (wanted & 1)


def run_cta(ntiles, dual, seed, rescale_prob=0.1, zero_prob=0.2, s_bufs=S_BUFS,
            p_per_group=False, spec_pre=0, spec_ok=True, spec_gate=True):
    """One CTA's run; `s_bufs` and `p_per_group` (one "P written" barrier per
    softmax group instead of per S/P buffer) model earlier designs;
    `spec_pre` prefix tiles are copied speculatively, the guess holding or not
    (`spec_ok`; when it holds the guessed range is the real one); without
    `spec_gate` the prologue ends without waiting for those copies (the first,
    faulty version of the speculation)."""
    S_BUFS = s_bufs  # noqa: N806  (shadows the kernel's constant)
    rng = random.Random(seed)
    rt = 2 if dual else 1
    ks = K_STAGES - 1 if dual else K_STAGES
    vs = V_STAGES - 1 if dual else V_STAGES
    if spec_ok:
        assert spec_pre <= ntiles
    nspec_k, nspec_v = min(spec_pre, ks), min(spec_pre, vs)
    xk, xv = (0, 0) if spec_ok else (nspec_k, nspec_v)

    def k_done(i):  # completion index of k_full for tile i (the kernel's k_phase)
        return i // ks + (1 if i % ks < xk else 0)

    def v_done(i):
        return i // vs + (1 if i % vs < xv else 0)
    nunits = ntiles * rt
    k_full = [Barrier(f"k_full{s}") for s in range(ks)]
    k_empty = [Barrier(f"k_empty{s}") for s in range(ks)]
    v_full = [Barrier(f"v_full{s}") for s in range(vs)]
    v_empty = [Barrier(f"v_empty{s}") for s in range(vs)]
    s_full = [Barrier(f"s_full{b}") for b in range(S_BUFS)]
    s_free = [Barrier(f"s_free{b}") for b in range(S_BUFS)]
    p_full = [Barrier(f"p_full{b}") for b in range(S_BUFS)]  # 4 warps: one arrival here

    def p_bar(u, g_or_buf):  # the "P written" barrier of unit u and its completion index
        if p_per_group:
            return p_full[g_or_buf], (u >> 1)
        return p_full[u % S_BUFS], u // S_BUFS
    pv_done = [Barrier(f"pv_done{g}") for g in range(2)]
    pv_fin = Barrier("pv_fin")
    log = []          # (event, index) in completion order
    pending = []      # asynchronous completions: [due, seq, thread, callback]
    clock = [0]
    seq = [0]
    last_due = {}     # per issuing thread: completions stay in issue order

    def later(thread, fn, label):
        due = max(clock[0] + rng.randint(1, 6), last_due.get(thread, 0))
        last_due[thread] = due
        seq[0] += 1
        pending.append([due, seq[0], thread, fn, label])

    def tile_of(u):
        return (u >> 1, u & 1) if dual else (u, 0)

    def producer(parity, kind, full, empty, nst, nspec):
        spec = list(range(parity, nspec, 2))
        for i in spec:  # before the prologue knows the real range: stage i
            log.append((f"{kind}_issue" if spec_ok else f"{kind}_spec_issue", i))
            land = f"{kind}_land" if spec_ok else f"{kind}_spec_land"
            later(f"tma{len(log)}", lambda i=i, land=land: (log.append((land, i)),
                                                             full[i].arrive()), kind)
            yield
        if spec_gate or not spec_ok:  # the speculative copies land before the prologue ends
            for i in spec:          # (ungated, only a failed guess waited, before refilling)
                while not full[i].ready(0):
                    yield
        landed[f"{kind}{parity}"] = True
        yield from prologue_barrier()
        for i in range(parity, ntiles, 2):
            if spec_ok and i < nspec:
                continue
            st = i % nst
            if i >= nst:
                while not empty[st].ready(i // nst - 1):
                    yield
            log.append((f"{kind}_issue", i))
            later(f"tma{len(log)}", lambda st=st, i=i: (log.append((f"{kind}_land", i)),
                                                         full[st].arrive()), kind)
            yield

    def k_producer(parity):
        return producer(parity, "k", k_full, k_empty, ks, nspec_k)

    def v_producer(parity):
        return producer(parity, "v", v_full, v_empty, vs, nspec_v)

    landed = {"k0": False, "k1": False, "v0": False, "v1": False}

    def prologue_barrier():
        """The CTA barrier that ends the prologue: the producers pass it only
        once their speculative copies have landed, so every consumer starts
        with each speculated stage's first phase complete."""
        while spec_gate and not all(landed.values()):
            yield

    def s_issuer():
        yield from prologue_barrier()
        for u in range(nunits):
            i, g = tile_of(u)
            kst, sb = i % ks, u % S_BUFS
            while not ((u < S_BUFS or s_free[sb].ready((u - S_BUFS) // S_BUFS)) and
                       (g != 0 or k_full[kst].ready(k_done(i)))):
                yield
            log.append(("s_issue", u))

            def done(u=u, sb=sb, kst=kst, g=g):
                log.append(("s_done", u))
                s_full[sb].arrive()
                if g == rt - 1:
                    k_empty[kst].arrive()
            later("s_issuer", done, "s")
            yield

    def softmax(wg):
        yield from prologue_barrier()
        i0, di = (0, 1) if dual else (wg, 2)
        for i in range(i0, ntiles, di):
            buf = wg if dual else (i & 1)
            u = 2 * i + wg if dual else i
            sb = u % S_BUFS
            while not s_full[sb].ready(u // S_BUFS):
                yield
            log.append(("p_start", u))
            yield
            if rng.random() < zero_prob and (not dual or wg == 0):
                while not v_full[i % vs].ready(v_done(i)):  # zeroing V rows
                    yield
            if rng.random() < rescale_prob and i >= i0 + di:
                while not pv_done[buf].ready((i - i0 - di) // di):  # O rescale
                    yield
            log.append(("p_ready", u))
            p_bar(u, buf)[0].arrive()
            yield

    def pv_issuer():
        yield from prologue_barrier()
        for u in range(nunits):
            i, g = tile_of(u)
            vst, sb = i % vs, u % S_BUFS
            buf = g if dual else (i & 1)
            pb, pn = p_bar(u, buf)
            while not (pb.ready(pn) and (g != 0 or v_full[vst].ready(v_done(i)))):
                yield
            log.append(("pv_issue", u))

            def done(u=u, sb=sb, vst=vst, g=g, buf=buf):
                log.append(("pv_done", u))
                pv_done[buf].arrive()
                if g == rt - 1:
                    v_empty[vst].arrive()
                s_free[sb].arrive()
            later("pv_issuer", done, "pv")
            yield
        later("pv_issuer", lambda: pv_fin.arrive(), "fin")

    roles = [k_producer(0), k_producer(1), v_producer(0), v_producer(1), s_issuer(),
             softmax(0), softmax(1), pv_issuer()]
    live = list(roles)
    steps = 0
    while live or pending:
        steps += 1
        assert steps < 200000, "no progress: deadlock"
        clock[0] += 1
        # complete the asynchronous work that is due, oldest first
        pending.sort(key=lambda e: (e[0], e[1]))
        while pending and pending[0][0] <= clock[0]:
            pending.pop(0)[3]()
        rng.shuffle(live)
        for g in list(live)[:rng.randint(1, len(live))] if live else []:
            try:
                next(g)
            except StopIteration:
                live.remove(g)
    assert pv_fin.phase == 1
    return log


def check_order(log, ntiles, dual, spec_pre=0, spec_ok=True):
    rt = 2 if dual else 1
    ks = K_STAGES - 1 if dual else K_STAGES
    vs = V_STAGES - 1 if dual else V_STAGES
    at = {ev: n for n, ev in enumerate(log)}
    if not spec_ok:  # a stage's speculative copy landed before its refill
        for kind, nst in (("k", ks), ("v", vs)):
            for i in range(min(spec_pre, nst)):
                assert at[(f"{kind}_spec_land", i)] < at.get((f"{kind}_issue", i), len(log))
    for u in range(ntiles * rt):
        i = u // rt
        assert at[("k_land", i)] < at[("s_issue", u)]
        if u >= S_BUFS:
            assert at[("pv_done", u - S_BUFS)] < at[("s_issue", u)]
        assert at[("s_done", u)] < at[("p_start", u)] < at[("p_ready", u)] < at[("pv_issue", u)]
        assert at[("v_land", i)] < at[("pv_issue", u)]
    for i in range(ntiles):
        last = (i + 1) * rt - 1
        if i + ks < ntiles:  # K stage refilled after both row tiles' S
            assert at[("s_done", last)] < at[("k_issue", i + ks)]
        if i + vs < ntiles:  # V stage refilled after both row tiles' PV
            assert at[("pv_done", last)] < at[("v_issue", i + vs)]


@pytest.mark.parametrize("dual", [False, True])
@pytest.mark.parametrize("ntiles", [1, 2, 3, 4, 5, 7, 11, 17, 66])
def test_tree_pipeline_protocol(ntiles, dual):
    for seed in range(12):
        log = run_cta(ntiles, dual, seed * 7919 + ntiles)
        check_order(log, ntiles, dual)


def test_model_detects_parity_aliasing():
    """The model's check fires when a barrier runs two phases ahead."""
    b = Barrier("b")
    b.arrive()
    b.arrive()
    with pytest.raises(AssertionError, match="parity aliasing"):
        b.ready(0)


def test_model_finds_the_per_group_p_barrier_stall():
    """The earlier design — three S/P buffers and one "P written" barrier per
    softmax group — lets a group finish tiles i and i+2 before the PV issuer
    looks at tile i; the model reports it as parity aliasing (the stall the
    per-buffer barriers fixed)."""
    hits = 0
    for seed in range(40):
        try:
            run_cta(17, False, seed, s_bufs=3, p_per_group=True)
        except AssertionError as e:
            assert "parity aliasing" in str(e)
            hits += 1
    assert hits > 0


@pytest.mark.parametrize("dual", [False, True])
@pytest.mark.parametrize("ntiles,spec_pre,spec_ok", [
    (1, 1, True), (3, 3, True), (5, 5, True), (6, 5, True), (17, 5, True), (4, 2, True),
    (1, 5, False), (3, 5, False), (6, 5, False), (17, 3, False), (2, 1, False), (0, 4, False),
])
def test_speculative_first_copies(ntiles, spec_pre, spec_ok, dual):
    """Speculative first copies, the guess holding (they are the tiles of
    record) or failing (landed, refilled, waited for one phase further):
    no aliasing, no deadlock, every dependency in order."""
    for seed in range(12):
        log = run_cta(ntiles, dual, seed * 104729 + ntiles, spec_pre=spec_pre, spec_ok=spec_ok)
        check_order(log, ntiles, dual, spec_pre, spec_ok)


def test_model_finds_the_ungated_speculation():
    """Ending the prologue before the speculative copies land lets a consumer
    of a failed guess wait for a stage's second phase while its first is
    still pending (a parity wait then succeeds at once, on the wrong data) —
    what the first version of the speculation did on the GPU."""
    hits = 0
    for seed in range(40):
        try:
            run_cta(3, False, seed, spec_pre=5, spec_ok=False, spec_gate=False)
        except AssertionError as e:
            assert "parity aliasing" in str(e)
            hits += 1
    assert hits > 0
