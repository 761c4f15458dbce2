"""CPU models of the normal-mode dispatch and combine protocols across ranks, driven by random
schedules.

Each rank runs a sequence of dispatches, fresh (count step concurrent with the stage, then the pull)
or with a cached handle (stage, then the pull; no count step), as the runtime launches them. The
model keeps the flags of the control blocks and a version number per staged chunk, executes one
enabled action of one rank at a time in random order, and checks:
  * every chunk a pull reads holds the data of the pull's own dispatch (never a previous dispatch's
    rows, never those of a later one that overwrote the staging too early);
  * the epoch the count step derives from the control block (previous epoch + 1) equals the one the
    host passes to the stage (the host's dispatch ticket), across mixes of fresh and cached calls;
  * nothing deadlocks: every schedule finishes.
The waits mirror the kernels': the stage and the count step wait until every receiver has finished
pulling the previous dispatch; the count step exchanges readiness with every peer; the pull waits
per (source, chunk) for the staged flag of its epoch; the pull's end releases `pull_done` to every
source and, without a count step, records the epoch.

The combine model runs back-to-back combines: each rank's pushers wait until the destination has
finished its previous combine (`combine_ready`), store rows into its slots and announce them on the
token's arrival counter; its reducers wait for the token's exact contribution count, read the rows
and reset the counter; the rank's last block then records its sequence number and releases it to
every rank. Checked: every reduced row is the current combine's, every counter ends at zero, no
deadlock; a variant without the destination wait is caught.

The GEMM-combine model (the down projection whose epilogue stores into the sources' slots) runs
epochs of send then reduce on every rank: the GEMM waits per destination for the release of the
previous epoch, stores its rows and publishes its epoch; the source waits for every rank's epoch,
reads its slots and releases them. Checked: every slot read holds the current epoch's row, no
deadlock; a GEMM without the release wait is caught.
"""
import random

import pytest


class Rank:
    def __init__(self, r, world, chunks):
        self.r = r
        self.dispatch_epoch = 0
        self.ticket = 0
        self.pull_done = [0] * world          # written by receiver s after pulling my staging
        self.notify = [0] * world             # written by peer s in its count step
        self.staged = [[0] * chunks for _ in range(world)]  # staged[s][c]: source s released chunk c at epoch
        self.staging = [0] * chunks           # version (epoch) of each chunk's rows in my staging


def build_ops(rank, plan, world, chunks):
    """Per dispatch: [group of concurrent launches], then the pull. Each op is a generator of steps;
    a step is (condition, effect)."""
    ops = []
    for cached in plan:
        rank.ticket += 1
        e = rank.ticket
        group = [('stage', e)] if cached else [('count', e), ('stage', e)]
        ops.append(group)
        ops.append([('pull', e, cached)])
    return ops


def stage_steps(R, me, e, chunks):
    for s in range(len(R)):
        yield (lambda s=s: R[me].pull_done[s] >= e - 1), (lambda: None)
    for c in range(chunks):
        def write(c=c):
            R[me].staging[c] = e
            for dst in range(len(R)):
                R[dst].staged[me][c] = e
        yield (lambda: True), write


def count_steps(R, me, e_host, seen):
    def derive():
        seen.append((me, R[me].dispatch_epoch + 1, e_host))
    yield (lambda: True), derive
    for s in range(len(R)):
        yield (lambda s=s: R[me].pull_done[s] >= e_host - 1), (lambda: None)
    for s in range(len(R)):
        def publish(s=s):
            R[s].notify[me] = e_host
        yield (lambda: True), publish
    for s in range(len(R)):
        yield (lambda s=s: R[me].notify[s] >= e_host), (lambda: None)

    def done():
        R[me].dispatch_epoch = e_host
    yield (lambda: True), done


def pull_steps(R, me, e, cached, chunks, errors):
    for s in range(len(R)):
        for c in range(chunks):
            def read(s=s, c=c):
                if R[s].staging[c] != e:
                    errors.append((me, s, c, e, R[s].staging[c]))
            yield (lambda s=s, c=c: R[me].staged[s][c] >= e), read

    def finish():
        for s in range(len(R)):
            R[s].pull_done[me] = e
        if cached:
            R[me].dispatch_epoch = e
    yield (lambda: True), finish


def run(world, plans, chunks, seed):
    rng = random.Random(seed)
    R = [Rank(r, world, chunks) for r in range(world)]
    errors, seen = [], []
    queues = [build_ops(R[r], plans[r], world, chunks) for r in range(world)]
    active = [[] for _ in range(world)]  # generators of the current group, with their pending step
    for step in range(200000):
        for r in range(world):
            if not active[r] and queues[r]:
                group = queues[r].pop(0)
                gens = []
                for op in group:
                    if op[0] == 'stage':
                        g = stage_steps(R, r, op[1], chunks)
                    elif op[0] == 'count':
                        g = count_steps(R, r, op[1], seen)
                    else:
                        g = pull_steps(R, r, op[1], op[2], chunks, errors)
                    gens.append([g, next(g, None)])
                active[r] = [x for x in gens if x[1] is not None]
        enabled = [(r, i) for r in range(world) for i, (g, st) in enumerate(active[r]) if st[0]()]
        if not enabled:
            pending = any(active) or any(queues)
            assert not pending, f'deadlock at step {step}'
            return errors, seen
        r, i = rng.choice(enabled)
        g, st = active[r][i]
        st[1]()
        nxt = next(g, None)
        if nxt is None:
            active[r].pop(i)
        else:
            active[r][i][1] = nxt
    raise AssertionError('schedule did not finish')


@pytest.mark.parametrize('seed', range(12))
@pytest.mark.parametrize('world', [1, 2, 3])
def test_dispatch_protocol_fresh_and_cached(seed, world):
    rng = random.Random(100 * seed + world)
    n = 6
    # every rank issues the same sequence of fresh / cached dispatches (a cached handle replays a
    # fresh dispatch on every rank together); the first one is always fresh
    plan = [False] + [rng.random() < 0.5 for _ in range(n - 1)]
    errors, seen = run(world, [plan] * world, chunks=3, seed=seed)
    assert not errors, errors[:5]
    assert all(derived == host for _, derived, host in seen), seen


def test_model_detects_a_missing_receiver_wait():
    """Sanity check of the model: a stage that does not wait for the receivers' previous pull lets a
    slow receiver read rows of the next dispatch."""
    global stage_steps
    original = stage_steps

    def no_wait(R, me, e, chunks):
        for c in range(chunks):
            def write(c=c):
                R[me].staging[c] = e
                for dst in range(len(R)):
                    R[dst].staged[me][c] = e
            yield (lambda: True), write
    stage_steps = no_wait
    try:
        bad = 0
        for seed in range(40):
            errors, _ = run(2, [[False, True, True, True]] * 2, chunks=2, seed=seed)
            bad += bool(errors)
        assert bad > 0
    finally:
        stage_steps = original


# ------------------------------------------------------------------------------------------------
# Combine: push rows into the destination's slots, announce arrivals, reduce, release the slots.
# ------------------------------------------------------------------------------------------------
class CRank:
    def __init__(self, world, tokens):
        self.seq = 0                                    # combines this rank has completed
        self.ready = [0] * world                        # ready[d]: d's completed combines (d writes)
        self.arrival = [0] * tokens                     # per own token: contributions landed
        self.slot = [[0] * tokens for _ in range(world)]  # slot[s][t]: version of source s's row for my token t


def combine_push_steps(C, me, k, routes):
    """Pushers of rank `me` for combine k: rows of the tokens it received, back to their source."""
    start_seq = C[me].seq
    for d, t in routes:
        yield (lambda d=d: C[me].ready[d] >= start_seq), (lambda: None)

        def store(d=d, t=t):
            C[d].slot[me][t] = k
        yield (lambda: True), store

        def announce(d=d, t=t):
            C[d].arrival[t] += 1
        yield (lambda: True), announce


def combine_reduce_steps(C, me, k, contributors, errors):
    for t, srcs in enumerate(contributors):
        if not srcs:
            continue
        yield (lambda t=t, n=len(srcs): C[me].arrival[t] == n), (lambda: None)

        def reduce(t=t, srcs=srcs):
            for s in srcs:
                if C[me].slot[s][t] != k:
                    errors.append((me, s, t, k, C[me].slot[s][t]))
            C[me].arrival[t] = 0
        yield (lambda: True), reduce


def run_combines(world, tokens, n_combines, seed):
    rng = random.Random(seed)
    C = [CRank(world, tokens) for _ in range(world)]
    errors = []
    plans = []
    for k in range(1, n_combines + 1):
        # which ranks hold a row of each source token (at least its own rank in half the cases)
        holders = [[sorted(rng.sample(range(world), rng.randint(0, world))) for _ in range(tokens)] for _ in range(world)]
        plans.append(holders)
    queue = [[k for k in range(1, n_combines + 1)] for _ in range(world)]
    active = [[] for _ in range(world)]  # [generator, pending step] of the current combine's roles
    ending = [None] * world
    for step in range(400000):
        for r in range(world):
            if not active[r] and ending[r] is None and queue[r]:
                k = queue[r].pop(0)
                holders = plans[k - 1]
                routes = [(d, t) for d in range(world) for t in range(tokens) if r in holders[d][t]]
                rng.shuffle(routes)
                gens = [combine_push_steps(C, r, k, routes),
                        combine_reduce_steps(C, r, k, [holders[r][t] for t in range(tokens)], errors)]
                active[r] = [[g, next(g, None)] for g in gens]
                active[r] = [x for x in active[r] if x[1] is not None]
                ending[r] = k
        enabled = [(r, i) for r in range(world) for i, (g, st) in enumerate(active[r]) if st[0]()]
        finishing = [r for r in range(world) if not active[r] and ending[r] is not None]
        if not enabled and not finishing:
            assert not any(queue), f'deadlock at step {step}'
            return errors, C
        pick = rng.randrange(len(enabled) + len(finishing))
        if pick >= len(enabled):
            r = finishing[pick - len(enabled)]
            C[r].seq = ending[r]                  # the last block: seq, then release to every rank
            for s in range(world):
                C[s].ready[r] = ending[r]
            ending[r] = None
            continue
        r, i = enabled[pick]
        g, st = active[r][i]
        st[1]()
        nxt = next(g, None)
        if nxt is None:
            active[r].pop(i)
        else:
            active[r][i][1] = nxt
    raise AssertionError('schedule did not finish')


@pytest.mark.parametrize('seed', range(12))
@pytest.mark.parametrize('world', [1, 2, 3])
def test_combine_protocol_back_to_back(seed, world):
    errors, C = run_combines(world, tokens=4, n_combines=5, seed=seed)
    assert not errors, errors[:5]
    assert all(c.seq == 5 for c in C) and all(a == 0 for c in C for a in c.arrival)


def test_combine_model_detects_a_missing_ready_wait():
    """Sanity check of the model: pushers that do not wait for the destination's previous combine
    overwrite rows it has not reduced yet."""
    global combine_push_steps
    original = combine_push_steps

    def no_wait(C, me, k, routes):
        for d, t in routes:
            def store(d=d, t=t):
                C[d].slot[me][t] = k
            yield (lambda: True), store

            def announce(d=d, t=t):
                C[d].arrival[t] += 1
            yield (lambda: True), announce
    combine_push_steps = no_wait
    try:
        bad = 0
        for seed in range(40):
            try:
                errors, _ = run_combines(2, tokens=3, n_combines=4, seed=seed)
            except AssertionError:
                errors = ['deadlock']  # an early arrival can also leave a counter that never matches
            bad += bool(errors)
        assert bad > 0
    finally:
        combine_push_steps = original


# ------------------------------------------------------------------------------------------------
# Down projection -> combine (parallel/gemm_combine.py): every rank's GEMM stores rows into the
# slots of the tokens' source ranks and publishes its epoch (gc_done); each source waits for every
# rank's epoch, reduces its slots and releases them (gc_free); the next epoch's GEMM waits, per
# destination, until that destination released the previous epoch.
# ------------------------------------------------------------------------------------------------
class GRank:
    def __init__(self, world, tokens):
        self.done = [0] * world       # done[s]: last epoch whose rows s stored into my slots (s writes)
        self.free = [0] * world       # free[d]: last epoch d finished reducing (d writes)
        self.slot = [[0] * tokens for _ in range(world)]  # slot[s][t]: epoch of the row s stored for my token t


def gc_send_steps(G, me, e, routes):
    """The GEMM of epoch e on rank `me`: waits for every destination's release of epoch e - 1, stores
    its rows (destination, token) in any order, then the last CTA publishes e to every rank."""
    world = len(G)
    for d in range(world):
        yield (lambda d=d: G[me].free[d] >= e - 1), (lambda: None)
    for d, t in routes:
        def store(d=d, t=t):
            G[d].slot[me][t] = e
        yield (lambda: True), store

    def publish():
        for d in range(world):
            G[d].done[me] = e
    yield (lambda: True), publish


def gc_reduce_steps(G, me, e, expected, errors):
    """The reduce of epoch e on rank `me`: waits for every rank's epoch, reads each expected slot,
    then releases its slots to every rank."""
    world = len(G)
    for s in range(world):
        yield (lambda s=s: G[me].done[s] >= e), (lambda: None)
    for s, t in expected:
        def read(s=s, t=t):
            if G[me].slot[s][t] != e:
                errors.append((me, s, t, e, G[me].slot[s][t]))
        yield (lambda: True), read

    def release():
        for d in range(world):
            G[d].free[me] = e
    yield (lambda: True), release


def run_gemm_combine(world, tokens, epochs, seed, send_steps=None):
    send_steps = send_steps or gc_send_steps
    rng = random.Random(seed)
    G = [GRank(world, tokens) for _ in range(world)]
    errors = []
    plans = []  # plans[e-1][r]: (destination, token) rows rank r sends at epoch e
    for _ in range(epochs):
        routes = [[] for _ in range(world)]
        for s in range(world):
            for t in range(tokens):
                for r in rng.sample(range(world), rng.randint(0, world)):
                    routes[r].append((s, t))
        for r in range(world):
            rng.shuffle(routes[r])
        plans.append(routes)
    # per rank: a stream of operations send(1), reduce(1), send(2), ... each a generator
    queues = []
    for r in range(world):
        q = []
        for e in range(1, epochs + 1):
            expected = [(s, t) for s in range(world) for (d, t) in plans[e - 1][s] if d == r]
            q.append(('send', e, plans[e - 1][r]))
            q.append(('reduce', e, expected))
        queues.append(q)
    current = [None] * world
    for step in range(500000):
        for r in range(world):
            if current[r] is None and queues[r]:
                kind, e, arg = queues[r].pop(0)
                g = send_steps(G, r, e, arg) if kind == 'send' else gc_reduce_steps(G, r, e, arg, errors)
                current[r] = [g, next(g)]
        enabled = [r for r in range(world) if current[r] is not None and current[r][1][0]()]
        if not enabled:
            assert all(c is None for c in current) and not any(queues), f'deadlock at step {step}'
            return errors, G
        r = rng.choice(enabled)
        g, st = current[r]
        st[1]()
        nxt = next(g, None)
        current[r] = None if nxt is None else [g, nxt]
    raise AssertionError('schedule did not finish')


@pytest.mark.parametrize('seed', range(12))
@pytest.mark.parametrize('world', [1, 2, 3, 4])
def test_gemm_combine_protocol_epochs(seed, world):
    errors, G = run_gemm_combine(world, tokens=3, epochs=5, seed=seed)
    assert not errors, errors[:5]
    assert all(x == 5 for g in G for x in g.done) and all(x == 5 for g in G for x in g.free)


def test_gemm_combine_model_detects_a_missing_release_wait():
    """Sanity check of the model: a GEMM that does not wait for the destinations' release of the
    previous epoch overwrites slots a slow source has not reduced yet."""
    def no_wait(G, me, e, routes):
        for d, t in routes:
            def store(d=d, t=t):
                G[d].slot[me][t] = e
            yield (lambda: True), store

        def publish():
            for d in range(len(G)):
                G[d].done[me] = e
        yield (lambda: True), publish
    bad = 0
    for seed in range(60):
        errors, _ = run_gemm_combine(2, tokens=3, epochs=4, seed=seed, send_steps=no_wait)
        bad += bool(errors)
    assert bad > 0
