"""The synchronisation protocol of the two-tile prefill attention kernel
(`prefill_attention_tc_pair_kernel`, `cheetah_b200/csrc/prefill_attention_tc.cuh`),
checked on the CPU over random interleavings (and, more briefly, that of the
one-tile kernels in the same file).

The kernel's actors are modelled step for step in the order the kernel runs
them: the TMA producer (four K/V stages), the MMA thread (S_A(0), S_B(0),
S_A(1), then per key tile j: PV_A(j), S_B(j+1), PV_B(j), commit of the K/V
stage, S_A(j+2)), the tensor pipe (MMAs complete in issue order; a commit
arrives when every earlier MMA has completed), the TMA engine, and the two
softmax groups (wait S, wait the previous P.V before touching O, release S,
release P). An mbarrier is modelled by its count of completed phases; a
parity wait for phase k passes when the count is k + 1 (mod 2), as
`mbarrier.try_wait.parity` does. Each run checks:

* every actor finishes (no deadlock) for 1..12 key tiles;
* whenever an actor polls a wait for phase k, the barrier has completed at
  most k + 1 phases (a barrier two phases ahead would alias the parity);
* no buffer is overwritten while a reader still needs it: a K/V stage is
  reloaded only after every MMA that reads it has completed, an S buffer is
  rewritten only after its previous group read it, and a group writes P_g(j)
  only after P.V(j-1) has read P_g(j-1).
"""

import random

import pytest

STAGES = 4   # kTpStages
SBUFS = 3    # kTpSBufs


class Barrier:
    def __init__(self, name):
        self.name = name
        self.done = 0  # completed phases

    def poll(self, phase):
        """A parity wait for `phase`: true iff that phase has completed."""
        assert self.done <= phase + 1, f"{self.name}: {self.done} phases done while waiting for phase {phase}"
        return self.done == phase + 1

    def complete(self):
        self.done += 1


class Model:
    def __init__(self, n_tiles, rng, mutation=None):
        self.n = n_tiles
        self.rng = rng
        self.mutation = mutation  # a deliberate protocol mistake (negative tests)
        self.q_full = Barrier("q_full")
        self.kv_full = [Barrier(f"kv_full[{s}]") for s in range(STAGES)]
        self.kv_empty = [Barrier(f"kv_empty[{s}]") for s in range(STAGES)]
        self.s_full = [Barrier(f"s_full[{b}]") for b in range(SBUFS)]
        self.s_empty = [Barrier(f"s_empty[{b}]") for b in range(SBUFS)]
        self.p_full = [Barrier(f"p_full[{g}]") for g in range(2)]
        self.o_full = [Barrier(f"o_full[{g}]") for g in range(2)]
        self.pipe = []          # issued, not completed tensor-pipe ops
        self.tma = []           # K/V (and Q) loads in flight
        self.stage_tile = [None] * STAGES     # tile held by each K/V stage
        self.readers = {}       # tile -> MMAs issued that read it and have not completed
        self.s_tile = [None] * SBUFS          # S tile n each buffer holds (None: free)
        self.p_read = [-1, -1]  # last j whose P_g the P.V has finished reading
        self.actors = [self.producer(), self.mma(), self.group(0), self.group(1)]

    # -- actors (generators yield while a wait does not pass) ---------------
    def wait(self, bar, phase):
        while not bar.poll(phase):
            yield

    def producer(self):
        self.tma.append(("q", None))
        for j in range(self.n):
            s = j % STAGES
            yield from self.wait(self.kv_empty[s], j // STAGES - 1)
            old = self.stage_tile[s]
            assert old is None or not self.readers.get(old), f"stage {s} reloaded while tile {old} is read"
            self.stage_tile[s] = j
            self.tma.append(("kv", j))
            yield

    def issue_s(self, g, j):
        n = 2 * j + g
        sb = n % SBUFS
        yield from self.wait(self.kv_full[j % STAGES], j // STAGES)
        yield from self.wait(self.s_empty[sb], n // SBUFS - 1)
        assert self.s_tile[sb] is None, f"S buffer {sb} rewritten while S tile {self.s_tile[sb]} is unread"
        self.s_tile[sb] = n
        self.readers[j] = self.readers.get(j, 0) + 1
        self.pipe.append(("s", g, j, sb))

    def s_full_of(self, g, n):
        """(barrier, phase) that signals S tile n = 2j + g."""
        if self.mutation == "per_group_s_full":
            return self.s_full[g], n // 2
        return self.s_full[n % SBUFS], n // SBUFS

    def issue_pv(self, g, j):
        yield from self.wait(self.p_full[g], j)
        self.readers[j] = self.readers.get(j, 0) + 1
        self.pipe.append(("pv", g, j, None))

    def mma(self):
        yield from self.wait(self.q_full, 0)
        yield from self.issue_s(0, 0)
        yield from self.issue_s(1, 0)
        if self.n >= 2:
            yield from self.issue_s(0, 1)
        for j in range(self.n):
            yield from self.issue_pv(0, j)
            if j + 1 < self.n:
                yield from self.issue_s(1, j + 1)
            yield from self.issue_pv(1, j)
            self.pipe.append(("commit", None, j, None))
            if j + 2 < self.n:
                yield from self.issue_s(0, j + 2)
            yield

    def group(self, g):
        for j in range(self.n):
            n = 2 * j + g
            sb = n % SBUFS
            yield from self.wait(*self.s_full_of(g, n))
            assert self.s_tile[sb] == n
            yield  # pass 1 (row max)
            if j > 0 and self.mutation != "no_o_wait":
                yield from self.wait(self.o_full[g], j - 1)
            # pass 2 writes P_g(j): P.V(j-1) must be done reading P_g(j-1).
            assert self.p_read[g] == j - 1, f"group {g} overwrote P while P.V({j - 1}) reads it"
            yield
            self.s_tile[sb] = None
            self.s_empty[sb].complete()
            self.p_full[g].complete()
            yield
        if self.n:
            yield from self.wait(self.o_full[g], self.n - 1)

    # -- asynchronous engines ------------------------------------------------
    def step_pipe(self):
        kind, g, j, sb = self.pipe.pop(0)
        if kind == "s":
            self.readers[j] -= 1
            self.s_full_of(g, 2 * j + g)[0].complete()
        elif kind == "pv":
            self.readers[j] -= 1
            self.p_read[g] = j
            self.o_full[g].complete()
        else:  # commit of tile j's stage: every earlier MMA has completed
            assert not self.readers.get(j), f"stage of tile {j} released with readers in flight"
            self.kv_empty[j % STAGES].complete()

    def step_tma(self):
        i = self.rng.randrange(len(self.tma))
        kind, j = self.tma.pop(i)
        if kind == "q":
            self.q_full.complete()
        else:
            self.kv_full[j % STAGES].complete()

    def run(self, max_steps=200000):
        live = list(self.actors)
        for _ in range(max_steps):
            choices = [("actor", a) for a in live]
            if self.pipe:
                choices.append(("pipe", None))
            if self.tma:
                choices.append(("tma", None))
            if not choices:
                return True
            kind, a = self.rng.choice(choices)
            if kind == "pipe":
                self.step_pipe()
            elif kind == "tma":
                self.step_tma()
            else:
                try:
                    next(a)
                except StopIteration:
                    live.remove(a)
        return False


class SingleTileModel(Model):
    """The one-query-tile kernels (`prefill_attention_tc_kernel`, head_dim 64,
    three K/V stages; `prefill_attention_tc2_kernel<128>`, two stages): S
    double-buffered by j & 1, the MMA thread issues S(j+1) before waiting for
    P(j), then P.V(j), o_full and the stage's commit; the softmax group
    releases S(j) right after reading it, waits for P.V(j-1) before touching
    O and P, then releases P(j)."""

    def __init__(self, n_tiles, rng, stages):
        self.stages = stages
        super().__init__(n_tiles, rng)
        self.kv_full = [Barrier(f"kv_full[{s}]") for s in range(stages)]
        self.kv_empty = [Barrier(f"kv_empty[{s}]") for s in range(stages)]
        self.stage_tile = [None] * stages
        self.s_full = [Barrier(f"s_full[{b}]") for b in range(2)]
        self.s_empty = [Barrier(f"s_empty[{b}]") for b in range(2)]
        self.s_tile = [None, None]
        self.actors = [self.producer(), self.mma(), self.group(0)]

    def producer(self):
        self.tma.append(("q", None))
        for j in range(self.n):
            s = j % self.stages
            yield from self.wait(self.kv_empty[s], j // self.stages - 1)
            old = self.stage_tile[s]
            assert old is None or not self.readers.get(old), f"stage {s} reloaded while tile {old} is read"
            self.stage_tile[s] = j
            self.tma.append(("kv", j))
            yield

    def issue_s(self, g, j):
        sb = j & 1
        yield from self.wait(self.kv_full[j % self.stages], j // self.stages)
        yield from self.wait(self.s_empty[sb], (j >> 1) - 1)
        assert self.s_tile[sb] is None, f"S buffer {sb} rewritten while S tile {self.s_tile[sb]} is unread"
        self.s_tile[sb] = j
        self.readers[j] = self.readers.get(j, 0) + 1
        self.pipe.append(("s", 0, j, sb))

    def mma(self):
        yield from self.wait(self.q_full, 0)
        yield from self.issue_s(0, 0)
        for j in range(self.n):
            if j + 1 < self.n:
                yield from self.issue_s(0, j + 1)
            yield from self.issue_pv(0, j)
            self.pipe.append(("commit", None, j, None))
            yield

    def group(self, g):
        for j in range(self.n):
            sb = j & 1
            yield from self.wait(self.s_full[sb], j >> 1)
            assert self.s_tile[sb] == j
            yield  # S read into registers
            self.s_tile[sb] = None
            self.s_empty[sb].complete()
            yield  # softmax
            if j > 0:
                yield from self.wait(self.o_full[0], j - 1)
            assert self.p_read[0] == j - 1, f"P overwritten while P.V({j - 1}) reads it"
            yield  # O rescaled or folded, P written
            self.p_full[0].complete()
            yield
        if self.n:
            yield from self.wait(self.o_full[0], self.n - 1)

    def step_pipe(self):
        kind, g, j, sb = self.pipe.pop(0)
        if kind == "s":
            self.readers[j] -= 1
            self.s_full[sb].complete()
        elif kind == "pv":
            self.readers[j] -= 1
            self.p_read[0] = j
            self.o_full[0].complete()
        else:
            assert not self.readers.get(j), f"stage of tile {j} released with readers in flight"
            self.kv_empty[j % self.stages].complete()

    def step_tma(self):
        i = self.rng.randrange(len(self.tma))
        kind, j = self.tma.pop(i)
        if kind == "q":
            self.q_full.complete()
        else:
            self.kv_full[j % self.stages].complete()


@pytest.mark.parametrize("stages", [3, 2])
@pytest.mark.parametrize("n_tiles", [1, 2, 3, 5, 8, 13])
def test_single_tile_kernels_protocol(stages, n_tiles):
    for seed in range(60):
        m = SingleTileModel(n_tiles, random.Random(7000 * stages + 100 * n_tiles + seed), stages)
        assert m.run(), f"no progress with {n_tiles} key tiles, {stages} stages (seed {seed})"
        assert m.o_full[0].done == n_tiles


@pytest.mark.parametrize("n_tiles", list(range(1, 13)))
def test_pair_kernel_protocol_finishes_without_aliasing_or_overwrites(n_tiles):
    for seed in range(60):
        m = Model(n_tiles, random.Random(1000 * n_tiles + seed))
        assert m.run(), f"no progress with {n_tiles} key tiles (seed {seed})"
        # Every phase that was produced was consumed.
        assert all(b.done == (n_tiles + STAGES - 1 - s) // STAGES for s, b in enumerate(m.kv_full))
        assert [b.done for b in m.o_full] == [n_tiles, n_tiles]


@pytest.mark.parametrize("mutation", ["no_o_wait", "per_group_s_full"])
def test_the_checks_catch_protocol_mistakes(mutation):
    """Two mistakes the kernel avoids are caught: writing P_g(j) without
    waiting for P.V(j-1) (it still reads P_g(j-1)), and one S-full barrier
    per group instead of one per S buffer (S_A(j+2) can complete before
    group A polls for S_A(j+1), two phases ahead of its wait)."""
    caught = 0
    for seed in range(200):
        m = Model(8, random.Random(seed), mutation)
        try:
            m.run()
        except AssertionError:
            caught += 1
    assert caught > 0
