"""CPU model of the mbarrier phase protocol used by the tcgen05 kernels, driven by random schedules.

An mbarrier completes a phase when its expected arrivals have arrived; `try_wait.parity(P)` succeeds
once the phase with parity P has completed, so waiting on parity ((i / depth) & 1) ^ 1 passes at
once for the first `depth` uses (the idiom every ring here uses). The models check, over many random
interleavings of the roles, the rings whose ordering the kernels rely on:
  * the tile-id queue of the fused dispatch -> GEMM kernel (one producer, the MMA warp and eight
    epilogue warps, depth 4): every consumer reads every id in order, no slot is overwritten before
    all nine consumers read it, and the sentinel ends every consumer;
  * the shared-memory stage ring (TMA producer -> MMA, depth S) and the 2 or 4 TMEM accumulators
    (MMA -> eight epilogue warps) of the grouped GEMMs: stages and accumulators are never reused
    before they are released;
  * the pull ring of the fused kernel (slots freed kLag rows late, a failed wait partway, the
    drain of loads in flight before its shared memory is reused);
  * the order of the fused kernel's epilogue scale reads after the rows landed.
"""
import random

import pytest


class MBarrier:
    def __init__(self, count):
        self.count = count
        self.pending = count
        self.phase = 0  # number of completed phases

    def arrive(self):
        assert self.pending > 0
        self.pending -= 1
        if self.pending == 0:
            self.phase += 1
            self.pending = self.count


def _done(bar, parity):
    """`mbarrier.try_wait.parity(parity)`: the hardware tracks only the parity of the current
    (incomplete) phase, and the wait succeeds when it differs from `parity`."""
    return (bar.phase & 1) != parity


@pytest.mark.parametrize('seed', range(40))
def test_tile_queue_protocol(seed):
    rng = random.Random(seed)
    Q, consumers, tiles = 4, 9, rng.randint(0, 25)
    qfull = [MBarrier(1) for _ in range(Q)]
    qempty = [MBarrier(consumers) for _ in range(Q)]
    slots = [None] * Q
    seq = list(range(tiles)) + [-1]
    prod = {'q': 0, 'done': False}
    cons = [{'q': 0, 'read': [], 'done': False} for _ in range(consumers)]
    reads_left = {}  # slot -> consumers that still have to read its current value

    for step in range(100000):
        actors = [('p', None)] if not prod['done'] else []
        actors += [('c', i) for i in range(consumers) if not cons[i]['done']]
        if not actors:
            break
        kind, i = rng.choice(actors)
        if kind == 'p':
            q = prod['q']
            s = q % Q
            if _done(qempty[s], ((q // Q) & 1) ^ 1):
                assert reads_left.get(s, 0) == 0, 'slot overwritten before every consumer read it'
                slots[s] = seq[q]
                reads_left[s] = consumers
                qfull[s].arrive()
                prod['q'] += 1
                prod['done'] = seq[q] == -1
        else:
            c = cons[i]
            q = c['q']
            s = q % Q
            if _done(qfull[s], (q // Q) & 1):
                t = slots[s]
                reads_left[s] -= 1
                qempty[s].arrive()
                c['q'] += 1
                if t < 0:
                    c['done'] = True
                else:
                    c['read'].append(t)
    assert prod['done'] and all(c['done'] for c in cons)
    for c in cons:
        assert c['read'] == list(range(tiles))


@pytest.mark.parametrize('seed', range(40))
@pytest.mark.parametrize('n_acc', [2, 4])
def test_stage_ring_and_accumulators(seed, n_acc):
    """n_acc TMEM accumulators rotate over the K blocks (the FP8 GEMM keeps 512 / N of them)."""
    rng = random.Random(seed)
    S, KB, tiles, epi = rng.choice([4, 6, 8]), rng.randint(1, 6), rng.randint(1, 6), 8
    full = [MBarrier(1) for _ in range(S)]
    empty = [MBarrier(1) for _ in range(S)]
    tfull = [MBarrier(1) for _ in range(n_acc)]
    tempty = [MBarrier(epi) for _ in range(n_acc)]
    total = tiles * KB
    stage_owner = [None] * S     # k-block whose data is in the stage
    acc_owner = [None] * n_acc   # k-block whose partial is in the accumulator
    acc_reads = [0] * n_acc
    prod = {'g': 0}
    mma = {'g': 0}
    epis = [{'g': 0} for _ in range(epi)]
    for step in range(200000):
        actors = []
        if prod['g'] < total:
            actors.append('p')
        if mma['g'] < total:
            actors.append('m')
        actors += [i for i in range(epi) if epis[i]['g'] < total]
        if not actors:
            break
        a = rng.choice(actors)
        if a == 'p':
            g = prod['g']
            s = g % S
            if _done(empty[s], ((g // S) & 1) ^ 1):
                assert stage_owner[s] is None, 'stage refilled before the MMA released it'
                stage_owner[s] = g
                full[s].arrive()  # the TMA bytes landed
                prod['g'] += 1
        elif a == 'm':
            g = mma['g']
            s, b = g % S, g % n_acc
            if _done(tempty[b], ((g // n_acc) & 1) ^ 1) and _done(full[s], (g // S) & 1):
                assert stage_owner[s] == g and acc_owner[b] is None
                acc_owner[b] = g
                acc_reads[b] = 0
                stage_owner[s] = None
                empty[s].arrive()   # tcgen05.commit -> stage free
                tfull[b].arrive()   # tcgen05.commit -> accumulator ready
                mma['g'] += 1
        else:
            e = epis[a]
            g = e['g']
            b = g % n_acc
            if _done(tfull[b], (g // n_acc) & 1):
                assert acc_owner[b] == g, 'epilogue read an accumulator of another k-block'
                acc_reads[b] += 1
                if acc_reads[b] == epi:
                    acc_owner[b] = None
                tempty[b].arrive()
                e['g'] += 1
    assert prod['g'] == mma['g'] == total and all(e['g'] == total for e in epis)


@pytest.mark.parametrize('seed', range(60))
def test_pull_ring_lagged_release_and_drain(seed):
    """The pull ring of the fused dispatch -> GEMM kernel: the producer TMA-loads rows into S slots;
    the consumer frees a slot only kLag rows after it took it (its stores may still read the slot),
    so the ring runs iff S > kLag. A wait that expires stops the producer: it issues nothing more
    and then waits for every load it issued (the last use of each slot) before the ring's shared
    memory is reused. Loads land at random times (a separate actor)."""
    rng = random.Random(seed)
    lag = 4
    S = rng.choice([lag + 1, lag + 2, 8])
    rows = rng.randint(0, 40)
    fail_at = rng.choice([None, None, rng.randint(0, max(0, rows - 1))])  # consumer stops at this row
    full = [MBarrier(1) for _ in range(S)]
    empty = [MBarrier(1) for _ in range(S)]
    slot_row = [None] * S      # row whose load targets the slot
    in_flight = set()          # rows whose loads have not landed
    prod = {'k': 0, 'failed': False, 'issued': 0, 'drained': False}
    cons = {'k': 0, 'done': False}
    for step in range(200000):
        actors = []
        if not prod['drained']:
            actors.append('p')
        if not cons['done']:
            actors.append('c')
        if in_flight:
            actors.append('land')
        if not actors:
            break
        a = rng.choice(actors)
        if a == 'land':
            k = rng.choice(sorted(in_flight))
            in_flight.discard(k)
            full[k % S].arrive()
        elif a == 'p':
            k = prod['k']
            if not prod['failed'] and k < rows:
                s = k % S
                if k < S or _done(empty[s], ((k // S) - 1) & 1):
                    assert slot_row[s] is None or slot_row[s] <= k - S, 'slot reused before its row was released'
                    assert all(r % S != s for r in in_flight), 'two loads in flight into one slot'
                    slot_row[s] = k
                    in_flight.add(k)
                    prod['k'] += 1
                    prod['issued'] += 1
                elif cons['done']:
                    prod['failed'] = True  # nobody will free the slot: the bounded wait expires
            else:
                # drain: the last use of every slot has landed before the memory is reused
                issued = prod['issued']
                if all(_done(full[k % S], (k // S) & 1) for k in range(max(0, issued - S), issued)):
                    assert not in_flight, 'drain passed with a load still in flight'
                    prod['drained'] = True
        else:
            k = cons['k']
            if k >= rows or (fail_at is not None and k == fail_at):
                cons['done'] = True   # finished, or its wait on row k expired
                continue
            s = k % S
            if _done(full[s], (k // S) & 1):
                assert slot_row[s] == k and k not in in_flight
                if k >= lag:
                    empty[(k - lag) % S].arrive()
                cons['k'] += 1
    assert prod['drained'] and cons['done'] and not in_flight
    if fail_at is None:
        assert cons['k'] == rows and prod['issued'] == rows


@pytest.mark.parametrize('epilogue_acquires', [True, False])
def test_tile_scales_read_after_rows_landed(epilogue_acquires):
    """The GEMM producer of the fused kernel publishes a tile id before it waits for the tile's rows
    to land; the epilogue reads the rows' scales with plain loads. Only an acquire of the landed
    counter by the epilogue itself orders those loads after the rows. Without it, some schedule
    reads a scale before its row landed (the case the kernel guards against)."""
    violations = 0
    for seed in range(200):
        rng = random.Random(seed)
        rows = 3
        landed = 0
        pushed = False
        prod_waited = False
        epi_state = 'wait_id'
        bad = False
        while epi_state != 'done':
            a = rng.choice(['pull', 'prod', 'epi'])
            if a == 'pull' and landed < rows:
                landed += 1
            elif a == 'prod':
                if not pushed:
                    pushed = True
                elif not prod_waited and landed == rows:
                    prod_waited = True
            elif a == 'epi':
                if epi_state == 'wait_id' and pushed:
                    epi_state = 'acquire' if epilogue_acquires else 'read'
                elif epi_state == 'acquire' and landed == rows:
                    epi_state = 'read'
                elif epi_state == 'read':
                    bad |= landed < rows
                    epi_state = 'done'
        violations += bad
    if epilogue_acquires:
        assert violations == 0
    else:
        assert violations > 0
