"""CPU model of the attention kernel's barrier protocol (wan2-ti2v-5b_b200/csrc/attn.cu).

The kernel's roles (TMA producer, UMMA issuer, two softmax warpgroups) hand work over through
mbarriers whose waits test only the parity of a phase.  A waiter that falls two phases behind its
barrier therefore cannot tell the phase it wants from the one two later: it blocks until the
latter, which may itself depend on the waiter (a deadlock that the kernel's bounded waits turn
into an error code and a wrong result).  This model replays a protocol with the kernel's barrier
counts, ring, issue order and in-order tensor-pipe completion (a commit arrives once every earlier
MMA is done) under randomised timings and checks that every run finishes.

* The shipped bf16 kernel: 128-key tiles, one S per query tile in TMEM with P written over it,
  so the next S of a tile is issued after that tile's P V (its softmax waits for it).
* A variant that was built and measured, then dropped (slower: its N = 64 QK MMAs with both
  operands in shared memory need more shared-memory bandwidth than the SM has): 64-key chunks with
  S double-buffered per tile.  There a softmax warpgroup can finish two chunks before the issuer
  takes the first P, so the P hand-off needs one barrier per S buffer; with one per tile the model
  deadlocks, as the kernel did.
"""
import random


class Bar:
    """An mbarrier: `count` arrivals complete a phase; try_wait.parity(p) succeeds once the
    current phase's parity differs from p."""

    def __init__(self, count):
        self.count, self.pending, self.phase = count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count

    def done(self, parity):
        return (self.phase & 1) != parity


def run(nkv, ring, p_full_per_buffer, seed, rescale_prob=0.2, chunked=True):
    """chunked=False: the shipped 128-key protocol; chunked=True: the 64-key double-buffered one."""
    rnd = random.Random(seed)
    nch = 2 * nkv if chunked else nkv
    kv_full = [Bar(1) for _ in range(ring)]
    kv_empty = [Bar(1) for _ in range(ring)]
    s_full = [Bar(1) for _ in range(4)]
    p_full = [Bar(1) for _ in range(4)]  # the four arriving warps of a warpgroup as one arrival
    pv_done = [Bar(1) for _ in range(2)]
    o_done = [Bar(1) for _ in range(2)]
    q_full = Bar(1)
    pipe = []  # tensor pipe: MMAs run in issue order; a commit arrives once everything before it is done

    def sf(t, c):
        return s_full[2 * t + (c & 1)] if chunked else s_full[2 * t]

    def sf_parity(c):
        return (c >> 1) & 1 if chunked else c & 1

    def pf(t, c):
        return p_full[2 * t + (c & 1)] if (chunked and p_full_per_buffer) else p_full[2 * t]

    def pf_parity(c):
        return (c >> 1) & 1 if (chunked and p_full_per_buffer) else c & 1

    def producer():
        q_full.arrive()
        for i in range(2 * nkv):  # K_0 V_0 K_1 V_1 ...
            slot, ph = i % ring, (i // ring) & 1
            yield ("wait", kv_empty[slot], ph ^ 1)
            yield ("work", rnd.randint(1, 5))
            kv_full[slot].arrive()

    def issuer():
        def kv_wait(i):
            return ("wait", kv_full[i % ring], (i // ring) & 1)

        def qk(t, c):  # chunked: K tile c // 2; shipped: K tile c
            tile = c >> 1 if chunked else c
            slot = (2 * tile) % ring
            pipe.append(["mma", rnd.randint(2, 4)])
            pipe.append(["commit", sf(t, c)])
            if t == 1 and (not chunked or c & 1):
                pipe.append(["commit", kv_empty[slot]])

        def pv(t, c):
            tile = c >> 1 if chunked else c
            slot = (2 * tile + 1) % ring
            pipe.append(["mma", rnd.randint(2, 4)])
            pipe.append(["commit", pv_done[t]])
            if t == 1 and (not chunked or c & 1):
                pipe.append(["commit", kv_empty[slot]])
            if c == nch - 1:
                pipe.append(["commit", o_done[t]])

        yield ("wait", q_full, 0)
        yield kv_wait(0)
        if chunked:
            qk(0, 0), qk(1, 0), qk(0, 1), qk(1, 1)
            for c in range(nch):
                if not c & 1:
                    yield kv_wait(c + 1)
                yield ("wait", pf(0, c), pf_parity(c))
                pv(0, c)
                if c + 2 < nch:
                    if not c & 1:
                        yield kv_wait(c + 2)
                    qk(0, c + 2)
                yield ("wait", pf(1, c), pf_parity(c))
                pv(1, c)
                if c + 2 < nch:
                    qk(1, c + 2)
        else:
            qk(0, 0), qk(1, 0)
            for j in range(nch):
                yield kv_wait(2 * j + 1)
                yield ("wait", pf(0, j), pf_parity(j))
                pv(0, j)
                if j + 1 < nch:
                    yield kv_wait(2 * j + 2)
                    qk(0, j + 1)
                yield ("wait", pf(1, j), pf_parity(j))
                pv(1, j)
                if j + 1 < nch:
                    qk(1, j + 1)

    def softmax(t):
        for c in range(nch):
            yield ("wait", sf(t, c), sf_parity(c))
            yield ("work", rnd.randint(1, 12))
            if chunked and c > 0 and rnd.random() < rescale_prob:  # O rescale: wait for P V_t(c - 1)
                yield ("wait", pv_done[t], (c - 1) & 1)
            pf(t, c).arrive()
        yield ("wait", o_done[t], 0)

    agents = {"producer": producer(), "issuer": issuer(), "softmax0": softmax(0), "softmax1": softmax(1)}
    state = dict.fromkeys(agents)
    busy = dict.fromkeys(agents, 0)
    finished = set()
    for _ in range(100000):
        if pipe:
            if pipe[0][0] == "mma":
                pipe[0][1] -= 1
                if pipe[0][1] <= 0:
                    pipe.pop(0)
            else:
                pipe.pop(0)[1].arrive()
                continue
        for k in rnd.sample(list(agents), len(agents)):
            if k in finished:
                continue
            if busy[k]:
                busy[k] -= 1
                continue
            it = state[k]
            if it is not None and it[0] == "wait" and not it[1].done(it[2]):
                continue
            try:
                nxt = next(agents[k])
            except StopIteration:
                finished.add(k)
                continue
            state[k] = nxt
            if nxt[0] == "work":
                busy[k], state[k] = nxt[1], None
        if len(finished) == len(agents) and not pipe:
            return True
    return False


def test_shipped_protocol_never_deadlocks():
    for ring in (3, 5):  # the e4m3 kernel's ring and the bf16 kernel's
        for nkv in range(1, 12):
            for seed in range(40):
                assert run(nkv, ring, False, seed * 97 + nkv, chunked=False), (ring, nkv, seed)


def test_double_buffered_variant_needs_a_p_barrier_per_buffer():
    for nkv in range(1, 10):
        for seed in range(40):
            assert run(nkv, 5, True, seed * 97 + nkv), (nkv, seed)
    # with one P barrier per query tile the same variant deadlocks: the model is sharp enough
    fails = sum(not run(nkv, 5, False, seed * 97 + nkv) for nkv in range(4, 10) for seed in range(60))
    assert fails > 0


def run_persistent(units_nkv, ring, seed):
    """The shipped bf16 kernel's persistent form (attn_persistent_kernel): one CTA walks several
    units (query-tile pairs) of nkv key tiles each.  Q has one buffer (reloaded once the unit's last
    QK is done: q_empty); the ring, s_full and the P barriers run on across units; the first P V of a
    unit waits for the softmax warps to have read the previous unit's O (o_free).  P is handed over
    in two parts: the first 96 key columns (p_part), on which the issuer starts the P V MMA, then the
    last 32 (p_full)."""
    rnd = random.Random(seed)
    kv_full = [Bar(1) for _ in range(ring)]
    kv_empty = [Bar(1) for _ in range(ring)]
    s_full, p_full = [Bar(1) for _ in range(2)], [Bar(1) for _ in range(2)]
    p_part = [Bar(1) for _ in range(2)]
    o_done, o_free = [Bar(1) for _ in range(2)], [Bar(1) for _ in range(2)]
    q_full, q_empty = Bar(1), Bar(1)
    pipe = []

    def producer():
        g = 0
        for i, nkv in enumerate(units_nkv):
            yield ("wait", q_empty, (i & 1) ^ 1)
            yield ("work", rnd.randint(1, 4))
            q_full.arrive()
            for _ in range(2 * nkv):
                slot, ph = g % ring, (g // ring) & 1
                yield ("wait", kv_empty[slot], ph ^ 1)
                yield ("work", rnd.randint(1, 5))
                kv_full[slot].arrive()
                g += 1

    def issuer():
        g = jg = 0
        for i, nkv in enumerate(units_nkv):
            def kv_wait(r):
                return ("wait", kv_full[r % ring], (r // ring) & 1)

            def qk(t, j):
                pipe.append(["mma", rnd.randint(2, 4)])
                pipe.append(["commit", s_full[t]])
                if t == 1:
                    pipe.append(["commit", kv_empty[(g + 2 * j) % ring]])
                    if j == nkv - 1:
                        pipe.append(["commit", q_empty])

            def pv_rest(t, j):
                pipe.append(["mma", rnd.randint(1, 2)])
                if t == 1:
                    pipe.append(["commit", kv_empty[(g + 2 * j + 1) % ring]])
                if j == nkv - 1:
                    pipe.append(["commit", o_done[t]])

            yield ("wait", q_full, i & 1)
            yield kv_wait(g)
            qk(0, 0), qk(1, 0)
            for j in range(nkv):
                yield kv_wait(g + 2 * j + 1)
                for t in (0, 1):
                    yield ("wait", p_part[t], (jg + j) & 1)
                    if j == 0:
                        yield ("wait", o_free[t], (i & 1) ^ 1)
                    pipe.append(["mma", rnd.randint(1, 3)])  # the P V K-steps over the first part
                    yield ("wait", p_full[t], (jg + j) & 1)
                    pv_rest(t, j)
                    if j + 1 < nkv:
                        if t == 0:
                            yield kv_wait(g + 2 * j + 2)
                        qk(t, j + 1)
            g += 2 * nkv
            jg += nkv

    def softmax(t):
        jg = 0
        for i, nkv in enumerate(units_nkv):
            for j in range(nkv):
                yield ("wait", s_full[t], (jg + j) & 1)
                yield ("work", rnd.randint(1, 9))
                p_part[t].arrive()
                yield ("work", rnd.randint(1, 3))
                p_full[t].arrive()
            yield ("wait", o_done[t], i & 1)
            yield ("work", rnd.randint(1, 6))  # the epilogue reads O_t
            o_free[t].arrive()
            jg += nkv

    return _drive({"producer": producer(), "issuer": issuer(), "softmax0": softmax(0), "softmax1": softmax(1)},
                  pipe, rnd)


def _drive(agents, pipe, rnd):
    state = dict.fromkeys(agents)
    busy = dict.fromkeys(agents, 0)
    finished = set()
    for _ in range(200000):
        if pipe:
            if pipe[0][0] == "mma":
                pipe[0][1] -= 1
                if pipe[0][1] <= 0:
                    pipe.pop(0)
            else:
                pipe.pop(0)[1].arrive()
                continue
        for k in rnd.sample(list(agents), len(agents)):
            if k in finished:
                continue
            if busy[k]:
                busy[k] -= 1
                continue
            it = state[k]
            if it is not None and it[0] == "wait" and not it[1].done(it[2]):
                continue
            try:
                nxt = next(agents[k])
            except StopIteration:
                finished.add(k)
                continue
            state[k] = nxt
            if nxt[0] == "work":
                busy[k], state[k] = nxt[1], None
        if len(finished) == len(agents) and not pipe:
            return True
    return False


def test_persistent_protocol_never_deadlocks():
    for seed in range(300):
        rnd = random.Random(seed)
        units = [rnd.randint(1, 6) for _ in range(rnd.randint(1, 6))]  # cross-attention units: 4 tiles
        assert run_persistent(units, 5, seed), (units, seed)
