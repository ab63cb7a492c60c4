"""Randomized simulation of the barrier protocols of the persistent attention
kernels (attn_fwd_persist_kernel, attn_bwd_dq_persist_kernel and the dK/dV
kernel in gollama_b200/csrc/attention_tc.cu) and of the CTA-pair GEMM
(gemm_tf32_pair_kernel in gollama_b200/csrc/gemm_tf32.cu).

Each role (TMA producer, score-MMA issuer, accumulate-MMA issuer, math warps)
is a generator transcribing the kernel's loops, the barrier each wait uses and
the phase parity it computes.  Barriers follow mbarrier semantics: a phase
completes when its arrival count is reached and its transaction bytes have
landed, and a parity wait succeeds while the barrier's current phase parity
differs from the one waited for.  TMA copies and tcgen05.commit arrivals
complete later, in random order.  Every wait checks that it did not wake
early, and every buffer reuse checks that its previous reader finished."""
import random


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.P, self.tx = name, count, count, 0, 0

    def arrive(self):
        self.pending -= 1
        self._maybe()

    def expect_tx(self, n):
        self.tx += n
        self.arrive()

    def complete_tx(self, n):
        self.tx -= n
        self._maybe()

    def _maybe(self):
        assert self.pending >= 0, self.name
        if self.pending == 0 and self.tx == 0:
            self.P += 1
            self.pending = self.count

    def ready(self, parity):
        return (self.P & 1) != parity


def _wait(bar, parity, use):
    while not bar.ready(parity):
        yield
    assert bar.P >= use + 1, (bar.name, bar.P, use)  # woke for the intended phase, not an earlier one


def _drive(roles, events, rnd, cap=2_000_000):
    live = dict(roles)
    for _ in range(cap):
        if not live and not events:
            return
        if events and (not live or rnd.random() < 0.5):
            events.pop(rnd.randrange(len(events)))()
        else:
            name = rnd.choice(list(live))
            try:
                next(live[name])
            except StopIteration:
                del live[name]
    raise AssertionError("deadlock")


def _in_order(q, fn, ev):
    """A tcgen05.commit of an issuing thread: it arrives once every MMA that
    thread issued before it has completed, so one thread's commits fire in
    issue order (an event that comes up early is put back)."""
    seq = q["issued"]
    q["issued"] += 1

    def fire():
        if q["fired"] != seq:
            ev.append(fire)
            return
        q["fired"] += 1
        fn()
    return fire


def forward(H, B, n_qt, grid, cta, seed):
    rnd = random.Random(seed)
    items = list(range(cta, H * B * n_qt, grid))
    qt_of = lambda it: n_qt - 1 - it // (H * B)
    bars = {(n, i): Bar(f"{n}{i}", 1) for n, k in [("q_full", 2), ("q_empty", 2), ("k_full", 2), ("k_empty", 2),
                                                       ("v_full", 2), ("v_empty", 2), ("s_full", 3), ("p_full", 3),
                                                       ("pv_done", 3), ("o_full", 2), ("o_empty", 2), ("xchg", 2)]
            for i in range(k)}
    b = lambda n, i: bars[(n, i)]
    ev = []
    st = {"S": [None] * 3, "O": [None] * 2, "pv": set(), "epi": set(), "sdone": set()}

    def tma():
        kv = 0
        for local, it in enumerate(items):
            qb = local & 1
            yield from _wait(b("q_empty", qb), ((local >> 1) & 1) ^ 1, (local >> 1) - 1)
            assert local < 2 or (local - 2) in st["sdone"]
            b("q_full", qb).expect_tx(1)
            ev.append(lambda qb=qb: b("q_full", qb).complete_tx(1))
            for _ in range(qt_of(it) + 1):
                s_, ph = kv & 1, (kv >> 1) & 1
                yield from _wait(b("k_empty", s_), ph ^ 1, (kv >> 1) - 1)
                b("k_full", s_).expect_tx(1)
                ev.append(lambda s_=s_: b("k_full", s_).complete_tx(1))
                yield from _wait(b("v_empty", s_), ph ^ 1, (kv >> 1) - 1)
                assert kv < 2 or (kv - 2) in st["pv"]
                b("v_full", s_).expect_tx(1)
                ev.append(lambda s_=s_: b("v_full", s_).complete_tx(1))
                kv += 1

    def smma():
        sq = 0
        for local, it in enumerate(items):
            qb = local & 1
            yield from _wait(b("q_full", qb), (local >> 1) & 1, local >> 1)
            for _ in range(qt_of(it) + 1):
                sb, s_ = sq % 3, sq & 1
                if sq >= 3:
                    yield from _wait(b("pv_done", sb), ((sq - 3) // 3) & 1, (sq - 3) // 3)
                    assert (sq - 3) in st["pv"]
                yield from _wait(b("k_full", s_), (sq >> 1) & 1, sq >> 1)
                st["S"][sb] = sq
                ev.append(lambda s_=s_: b("k_empty", s_).arrive())
                ev.append(lambda sb=sb: b("s_full", sb).arrive())
                sq += 1

            def qdone(qb=qb, local=local):
                st["sdone"].add(local)
                b("q_empty", qb).arrive()
            ev.append(qdone)

    def acc():
        sq = 0
        for local, it in enumerate(items):
            ob = local & 1
            yield from _wait(b("o_empty", ob), ((local >> 1) & 1) ^ 1, (local >> 1) - 1)
            assert local < 2 or (local - 2) in st["epi"]
            st["O"][ob] = local
            for _ in range(qt_of(it) + 1):
                sb, s_ = sq % 3, sq & 1
                yield from _wait(b("p_full", sb), (sq // 3) & 1, sq // 3)
                yield from _wait(b("v_full", s_), (sq >> 1) & 1, sq >> 1)
                assert st["S"][sb] == sq

                def done(s_=s_, sb=sb, sq=sq):
                    st["pv"].add(sq)
                    b("v_empty", s_).arrive()
                    b("pv_done", sb).arrive()
                ev.append(done)
                sq += 1
            ev.append(lambda ob=ob: b("o_full", ob).arrive())

    def math():
        sq = xc = 0
        for local, it in enumerate(items):
            ob = local & 1
            for j in range(qt_of(it) + 1):
                sb = sq % 3
                yield from _wait(b("s_full", sb), (sq // 3) & 1, sq // 3)
                assert st["S"][sb] == sq
                b("xchg", xc & 1).arrive()
                yield from _wait(b("xchg", xc & 1), (xc >> 1) & 1, xc >> 1)
                xc += 1
                if j > 0 and rnd.random() < 0.5:  # the row max grew: O is rescaled
                    yield from _wait(b("pv_done", (sq - 1) % 3), ((sq - 1) // 3) & 1, (sq - 1) // 3)
                    assert (sq - 1) in st["pv"] and st["O"][ob] == local
                b("p_full", sb).arrive()
                sq += 1
            b("xchg", xc & 1).arrive()
            yield from _wait(b("xchg", xc & 1), (xc >> 1) & 1, xc >> 1)
            xc += 1
            yield from _wait(b("o_full", ob), (local >> 1) & 1, local >> 1)
            assert st["O"][ob] == local
            st["epi"].add(local)
            b("o_empty", ob).arrive()

    _drive({"tma": tma(), "smma": smma(), "acc": acc(), "math": math()}, ev, rnd)


def dq(H, B, n_qt, S, grid, cta, seed, groups=1):
    """attn_bwd_dq_persist_kernel (groups=1) or attn_bwd_dq2_persist_kernel
    (groups=2: math group g takes the steps with kv % 2 == g; the group that
    ran an item's last step moves the next item's Q/dO and reads out dQ)."""
    rnd = random.Random(seed)
    items = list(range(cta, H * B * n_qt, grid))
    n_k64 = (S + 63) // 64
    nk_of = lambda it: min(n_k64, ((n_qt - 1 - it // (H * B)) * 128 + 128) // 64)
    bars = {(n, i): Bar(f"{n}{i}", 1) for n, k in [("qo_full", 1), ("qo_moved", 1), ("kv_full", 3),
                                                       ("kv_empty", 3), ("s_full", 2), ("dp_full", 2), ("p_full", 2),
                                                       ("set_free", 2), ("dq_full", 2), ("dq_empty", 2)]
            for i in range(k)}
    b = lambda n, i=0: bars[(n, i)]
    ev = []
    commits = {"issued": 0, "fired": 0}
    st = {"tmem_qo": None, "staging": None, "s": set(), "dp": set(), "dq": set(), "epi": set(), "buf": [None, None]}

    def tma():
        kv = 0
        for local, it in enumerate(items):
            if local > 0:
                yield from _wait(b("qo_moved"), (local - 1) & 1, local - 1)

            def land(local=local):
                st["staging"] = local
                b("qo_full").complete_tx(1)
            b("qo_full").expect_tx(1)
            ev.append(land)
            for _ in range(nk_of(it)):
                s_, ph = kv % 3, (kv // 3) & 1
                yield from _wait(b("kv_empty", s_), ph ^ 1, kv // 3 - 1)
                assert kv < 3 or (kv - 3) in st["dq"]
                b("kv_full", s_).expect_tx(1)
                ev.append(lambda s_=s_: b("kv_full", s_).complete_tx(1))
                kv += 1

    def smma():
        kv = 0
        for local, it in enumerate(items):
            yield from _wait(b("qo_moved"), local & 1, local)
            for _ in range(nk_of(it)):
                s_, ts = kv % 3, kv % 2
                yield from _wait(b("kv_full", s_), (kv // 3) & 1, kv // 3)
                yield from _wait(b("set_free", ts), ((kv // 2) & 1) ^ 1, kv // 2 - 1)
                assert (kv < 2 or (kv - 2) in st["dq"]) and st["tmem_qo"] == local

                def s_done(ts=ts, kv=kv):
                    st["s"].add(kv)
                    b("s_full", ts).arrive()

                def dp_done(ts=ts, kv=kv):
                    st["dp"].add(kv)
                    b("dp_full", ts).arrive()
                ev.append(_in_order(commits, s_done, ev))
                ev.append(_in_order(commits, dp_done, ev))
                kv += 1

    def acc():
        kv = 0
        for local, it in enumerate(items):
            ob = local & 1
            yield from _wait(b("dq_empty", ob), ((local >> 1) & 1) ^ 1, (local >> 1) - 1)
            assert local < 2 or (local - 2) in st["epi"]
            st["buf"][ob] = local
            for _ in range(nk_of(it)):
                ps, pts = kv % 3, kv % 2
                yield from _wait(b("p_full", pts), (kv // 2) & 1, kv // 2)

                def done(pts=pts, ps=ps, kv=kv):
                    st["dq"].add(kv)
                    b("set_free", pts).arrive()
                    b("kv_empty", ps).arrive()
                ev.append(done)
                kv += 1
            ev.append(lambda ob=ob: b("dq_full", ob).arrive())

    def math(g=0):
        kv = 0
        if items and g == 0:
            yield from _wait(b("qo_full"), 0, 0)
            assert st["staging"] == 0
            st["tmem_qo"] = 0
            b("qo_moved").arrive()
        for local, it in enumerate(items):
            for _ in range(nk_of(it)):
                ts = kv % 2
                if groups == 2 and ts != g:
                    kv += 1
                    continue
                yield from _wait(b("s_full", ts), (kv // 2) & 1, kv // 2)
                assert kv in st["s"]
                yield from _wait(b("dp_full", ts), (kv // 2) & 1, kv // 2)
                assert kv in st["dp"]
                b("p_full", ts).arrive()
                kv += 1
            if groups == 2 and (kv - 1) % 2 != g:
                continue  # the other group ran the item's last step
            if local + 1 < len(items):
                yield from _wait(b("qo_full"), (local + 1) & 1, local + 1)
                # Q and dO in TMEM are overwritten: every S and dP product of this item has completed
                assert st["staging"] == local + 1 and all(k in st["s"] and k in st["dp"] for k in range(kv))
                st["tmem_qo"] = local + 1
                b("qo_moved").arrive()
            ob = local & 1
            yield from _wait(b("dq_full", ob), (local >> 1) & 1, local >> 1)
            assert st["buf"][ob] == local
            st["epi"].add(local)
            b("dq_empty", ob).arrive()

    maths = {f"math{g}": math(g) for g in range(groups)}
    _drive({"tma": tma(), "smma": smma(), "acc": acc(), **maths}, ev, rnd)


def dkdv(n_heads, nq, seed, groups=1):
    """attn_bwd_dkdv_tc_kernel's protocol for one CTA: n_heads * nq steps of
    64 queries, three Q/dO stages (K and V land in the third and are copied
    to TMEM first), two TMEM sets, each step committed in halves (S^T then
    dP^T by the score issuer; P^T then dS^T by the math warps).  groups=2:
    attn_bwd_dkdv2_kernel, math group g takes the steps with it % 2 == g, both
    groups copy K and V, no lse/D staging barrier, and the halves of a TMEM
    set are released separately (s_free after dV, dp_free after dK)."""
    rnd = random.Random(seed)
    n_it = n_heads * nq
    bars = {(n, i): Bar(f"{n}{i}", 1) for n, k in [("kv_full", 1), ("qo_full", 3), ("qo_empty", 3),
                                                       ("s_full", 2), ("dp_full", 2), ("p_full", 2), ("ds_full", 2),
                                                       ("set_free", 2), ("s_free", 2), ("dp_free", 2),
                                                       ("acc_done", 1), ("ld_ready", 2)]
            for i in range(k)}
    bars[("kv_moved", 0)] = Bar("kv_moved", groups)
    b = lambda n, i=0: bars[(n, i)]
    ev = []
    smma_q, acc_q = {"issued": 0, "fired": 0}, {"issued": 0, "fired": 0}
    st = {"kv_in_stage2": False, "stage": [None] * 3, "S": set(), "dP": set(), "P": set(), "dS": set(),
          "dv": set(), "dk": set(), "acc_done": False}

    def tma():
        def land_kv():
            st["kv_in_stage2"] = True
            b("kv_full").complete_tx(1)
        b("kv_full").expect_tx(1)
        ev.append(land_kv)
        for it in range(n_it):
            s_, ph = it % 3, (it // 3) & 1
            if it == 2:
                yield from _wait(b("kv_moved"), 0, 0)
                st["kv_in_stage2"] = False
            yield from _wait(b("qo_empty", s_), ph ^ 1, it // 3 - 1)
            assert it < 3 or (it - 3) in st["dk"]

            def land(s_=s_, it=it):
                st["stage"][s_] = it
                b("qo_full", s_).complete_tx(1)
            b("qo_full", s_).expect_tx(1)
            ev.append(land)

    def smma():
        yield from _wait(b("kv_moved"), 0, 0)
        for it in range(n_it):
            s_, ts = it % 3, it % 2
            yield from _wait(b("qo_full", s_), (it // 3) & 1, it // 3)

            def s_done(ts=ts, it=it):
                st["S"].add(it)
                b("s_full", ts).arrive()

            def dp_done(ts=ts, it=it):
                st["dP"].add(it)
                b("dp_full", ts).arrive()
            if groups == 1:
                yield from _wait(b("set_free", ts), ((it // 2) & 1) ^ 1, it // 2 - 1)
                assert st["stage"][s_] == it and (it < 2 or (it - 2) in st["dk"])
                ev.append(s_done)
                ev.append(dp_done)
            else:
                # S^T overwrites P^T of step it - 2: dV must have read it
                yield from _wait(b("s_free", ts), ((it // 2) & 1) ^ 1, it // 2 - 1)
                assert st["stage"][s_] == it and (it < 2 or (it - 2) in st["dv"])
                ev.append(_in_order(smma_q, s_done, ev))
                # dP^T overwrites dS^T of step it - 2: dK must have read it
                yield from _wait(b("dp_free", ts), ((it // 2) & 1) ^ 1, it // 2 - 1)
                assert it < 2 or (it - 2) in st["dk"]
                ev.append(_in_order(smma_q, dp_done, ev))

    def acc():
        for it in range(n_it):
            s_, ts = it % 3, it % 2
            yield from _wait(b("p_full", ts), (it // 2) & 1, it // 2)
            assert it in st["P"] and st["stage"][s_] == it

            def dv_done(ts=ts, it=it):
                st["dv"].add(it)
                if groups == 2:
                    b("s_free", ts).arrive()
            ev.append(_in_order(acc_q, dv_done, ev))
            yield from _wait(b("ds_full", ts), (it // 2) & 1, it // 2)
            assert it in st["dS"]

            def done(ts=ts, s_=s_, it=it):
                st["dk"].add(it)
                b("set_free" if groups == 1 else "dp_free", ts).arrive()
                b("qo_empty", s_).arrive()
            ev.append(_in_order(acc_q, done, ev))

        def fin():
            # a commit arrives once every earlier MMA of its thread completed
            if len(st["dk"]) < n_it:
                ev.append(fin)
                return
            st["acc_done"] = True
            b("acc_done").arrive()
        ev.append(fin)

    def math(g=0):
        yield from _wait(b("kv_full"), 0, 0)
        assert st["kv_in_stage2"]
        b("kv_moved").arrive()
        for it in range(g, n_it, groups):
            ts = it % 2
            if groups == 1:
                b("ld_ready", it & 1).arrive()
                yield from _wait(b("ld_ready", it & 1), (it >> 1) & 1, it >> 1)
            yield from _wait(b("s_full", ts), (it // 2) & 1, it // 2)
            assert it in st["S"]
            st["P"].add(it)
            b("p_full", ts).arrive()
            yield from _wait(b("dp_full", ts), (it // 2) & 1, it // 2)
            assert it in st["dP"]
            st["dS"].add(it)
            b("ds_full", ts).arrive()
        yield from _wait(b("acc_done"), 0, 0)
        assert st["acc_done"] and len(st["dk"]) == n_it

    maths = {f"math{g}": math(g) for g in range(groups)}
    _drive({"tma": tma(), "smma": smma(), "acc": acc(), **maths}, ev, rnd)


def pair_gemm(k_blocks, seed, dyn=False, total_tiles=None, stages=6, ring=8, epi_warps=4, skip=0.0, counts=None):
    """gemm_tf32_pair_kernel (gollama_b200/csrc/gemm_tf32.cu) for one CTA pair.

    k_blocks[i]: the k-blocks of the pair's i-th tile (static order: the tiles
    the pair owns).  dyn: the dynamic order instead, where the leader's
    producer takes indices from a counter shared with other pairs (each index
    taken by another pair with probability `skip`) until total_tiles, and
    publishes them through a ring of `ring` slots in both CTAs; the peer's
    producer, the MMA issuer and the epilogue warps of both CTAs read them in
    order and release each slot on the leader's ring_empty.

    Barriers: full[s] (leader; the leader's producer arrives with expect_tx of
    both CTAs' copies, and the peer's copy may land before that arrival),
    empty[s] in each CTA (the MMA issuer's commit), tfull[b] in each CTA (the
    issuer's commit after a tile), tempty[b] (leader; one arrival per epilogue
    warp of either CTA).  Checked: every stage the MMAs read holds both CTAs'
    copies of the right (tile, k-block); no stage is refilled before the MMAs
    that read it completed; no accumulator is overwritten before every
    epilogue warp of both CTAs read it; no ring slot is rewritten before its
    ten readers took it; every tile reaches the epilogue of both CTAs once.
    counts: arrival counts to override (a planted mistake for the tests)."""
    rnd = random.Random(seed)
    bars = {}

    def b(name, i=0, cta=0):
        key = (name, i, cta)
        if key not in bars:
            count = {"tempty": 2 * epi_warps, "ring_empty": 2 + 2 * epi_warps, **(counts or {})}.get(name, 1)
            bars[key] = Bar(f"{name}{i}.{cta}", count)
        return bars[key]

    ev = []
    commits = {"issued": 0, "fired": 0}
    st = {
        "stage": [[None, None] for _ in range(stages)],  # (tile, kb) landed per CTA
        "stage_read": {},                                # stage fill index -> MMAs done
        "acc": [None, None],                             # tile index complete in accumulator b
        "drained": {},                                   # local tile -> epilogue warps done
        "ring": [[None] * ring, [None] * ring],           # published (index, tile) per CTA
        "ring_reads": {},                                # index -> readers done
        "seen": [[], []],                                # tiles per CTA's epilogue (warp 0)
        "counter": 0,
        "published": [],
    }

    def take():
        while st["counter"] < total_tiles and rnd.random() < skip:
            st["counter"] += 1          # another pair took this index
        t = st["counter"] if st["counter"] < total_tiles else -1
        st["counter"] += 1
        return t

    def consume(cta, i):
        slot = i % ring
        yield from _wait(b("ring_full", slot, cta), (i // ring) & 1, i // ring)
        idx, tile = st["ring"][cta][slot]
        assert idx == i, ("ring slot holds another index", cta, slot, idx, i)
        st["ring_reads"][i] = st["ring_reads"].get(i, 0) + 1
        b("ring_empty", slot).arrive()
        return tile

    def nkb(tile):
        return k_blocks[tile % len(k_blocks)]

    def get_tile(cta, i, reader=True):
        """the i-th tile of a role (-1: no more); in the dynamic order the
        leader's producer publishes it, every other role reads the ring"""
        if not dyn:
            return i if i < len(k_blocks) else -1
        if reader:
            return (yield from consume(cta, i))
        slot = i % ring
        yield from _wait(b("ring_empty", slot), ((i // ring) & 1) ^ 1, i // ring - 1)
        assert i < ring or st["ring_reads"].get(i - ring) == 2 + 2 * epi_warps, ("ring slot rewritten early", i)
        tile = take()
        for c in (0, 1):
            st["ring"][c][slot] = (i, tile)
        st["published"].append(tile)
        b("ring_full", slot, 0).arrive()
        b("ring_full", slot, 1).arrive()
        return tile

    def producer(cta):
        stage = f = i = 0
        phase = 0
        while True:
            tile = yield from get_tile(cta, i, reader=not (cta == 0))
            if tile < 0:
                return
            for kb in range(nkb(tile)):
                u = f // stages
                yield from _wait(b("empty", stage, cta), phase ^ 1, u - 1)
                assert u == 0 or st["stage_read"].get((cta, f - stages)), ("stage refilled before read", cta, f)
                if cta == 0:
                    b("full", stage).expect_tx(2)   # the pair's two copies

                def land(stage=stage, cta=cta, tile=tile, kb=kb):
                    st["stage"][stage][cta] = (tile, kb)
                    b("full", stage).complete_tx(1)
                ev.append(land)
                f += 1
                stage += 1
                if stage == stages:
                    stage, phase = 0, phase ^ 1
                yield
            i += 1

    def mma():
        stage = f = local = 0
        phase = 0
        while True:
            tile = yield from get_tile(0, local)
            if tile < 0:
                return
            buf, use = local & 1, local >> 1
            yield from _wait(b("tempty", buf), (use & 1) ^ 1, use - 1)
            assert local < 2 or st["drained"].get(local - 2) == 2 * epi_warps, ("accumulator overwritten", local)
            st["acc"][buf] = ("partial", local)
            for kb in range(nkb(tile)):
                yield from _wait(b("full", stage), phase, f // stages)
                assert st["stage"][stage] == [(tile, kb), (tile, kb)], ("stage contents", stage, st["stage"][stage])
                for c in (0, 1):
                    def freed(stage=stage, f=f, c=c):
                        st["stage_read"][(c, f)] = True
                        b("empty", stage, c).arrive()
                    ev.append(_in_order(commits, freed, ev))
                f += 1
                stage += 1
                if stage == stages:
                    stage, phase = 0, phase ^ 1
                yield
            for c in (0, 1):
                def done(buf=buf, local=local, c=c):
                    st["acc"][buf] = ("done", local)
                    b("tfull", buf, c).arrive()
                ev.append(_in_order(commits, done, ev))
            local += 1

    def epilogue(cta, w):
        local = 0
        while True:
            tile = yield from get_tile(cta, local)
            if tile < 0:
                return
            buf, use = local & 1, local >> 1
            yield from _wait(b("tfull", buf, cta), use & 1, use)
            assert st["acc"][buf] == ("done", local), ("accumulator not final", cta, w, local, st["acc"][buf])
            st["drained"][local] = st["drained"].get(local, 0) + 1
            b("tempty", buf).arrive()
            if w == 0:
                st["seen"][cta].append(tile)
            local += 1
            yield

    roles = {"prod0": producer(0), "prod1": producer(1), "mma": mma()}
    roles.update({f"epi{c}.{w}": epilogue(c, w) for c in (0, 1) for w in range(epi_warps)})
    _drive(roles, ev, rnd)
    want = [t for t in st["published"] if t >= 0] if dyn else list(range(len(k_blocks)))
    assert st["seen"][0] == want and st["seen"][1] == want, (st["seen"], want)
    if dyn:
        assert all(st["ring_reads"].get(i) == 2 + 2 * epi_warps for i in range(len(st["published"])))
    return want
