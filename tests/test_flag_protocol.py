"""Host emulation of the tensor-parallel all-reduce flag protocol (CPU threads as ranks).

The decode / verify / draft steps of ``parallel.tp`` exchange row partials through two
receive buffers per rank (O and down).  All-reduce number k of a step uses epoch
``step * stride + k``; odd k write the O buffer, even k the down buffer; a sender writes its
partial into every rank's slot, then releases its flag there; a rank reduces once every
sender's flag reached the epoch.  Writes are safe only if a rank never writes a peer's slot
before the peer has consumed the previous content of that slot.  The emulation checks that
invariant for the schedules the engine uses (steps with an even number of all-reduces) and
shows the race the even-count rule prevents (an odd count lets two consecutive all-reduces
hit the same buffer).  The same is done for the slot reuse of open-loop prefill/decode serving
(``parallel.pd``): request i goes to decode slot i mod S, and the prefill rank waits on the
slot's free flag (released by the decoder after request i - S) before pushing.
"""
import threading
import time

import pytest

STRIDE = 1024


class Device:
    """Per-rank receive slots and flags; records protocol violations."""

    def __init__(self, world):
        self.world = world
        self.lock = threading.Lock()
        # (owner, buffer, sender) -> (epoch written, epoch consumed)
        self.slots = {(o, b, s): (0, 0) for o in range(world) for b in "OD" for s in range(world)}
        self.flags = {(o, b, s): 0 for o in range(world) for b in "OD" for s in range(world)}
        self.violations = []

    def write(self, owner, buf, sender, epoch):
        with self.lock:
            written, consumed = self.slots[(owner, buf, sender)]
            if written != consumed:
                self.violations.append((owner, buf, sender, written, epoch))
            self.slots[(owner, buf, sender)] = (epoch, consumed)

    def signal(self, owner, buf, sender, epoch):
        with self.lock:
            self.flags[(owner, buf, sender)] = max(self.flags[(owner, buf, sender)], epoch)

    def wait_and_consume(self, owner, buf, epoch, deadline=5.0):
        t0 = time.time()
        while True:
            with self.lock:
                if all(self.flags[(owner, buf, s)] >= epoch for s in range(self.world)):
                    for s in range(self.world):
                        written, _ = self.slots[(owner, buf, s)]
                        self.slots[(owner, buf, s)] = (written, written)
                    return
            if time.time() - t0 > deadline:
                raise TimeoutError("bounded wait ran out")
            time.sleep(0)


def run_rank(dev, rank, program, delays, consume_delays=None):
    step = 0
    for n_ar in program:
        for k in range(1, n_ar + 1):
            buf = "O" if k % 2 else "D"
            epoch = step * STRIDE + k
            time.sleep(delays(rank, step, k))
            for owner in range(dev.world):  # partial rows to every rank's slot for this sender
                dev.write(owner, buf, rank, epoch)
            for owner in range(dev.world):
                dev.signal(owner, buf, rank, epoch)
            if consume_delays is not None:
                time.sleep(consume_delays(rank, step, k))
            dev.wait_and_consume(rank, buf, epoch)  # the owner reduces its slots
        step += 1  # each step (or captured graph) advances the shared step counter once


def emulate(world, program, delays, consume_delays=None):
    dev = Device(world)
    threads = [threading.Thread(target=run_rank, args=(dev, r, program, delays, consume_delays))
               for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    return dev.violations


@pytest.mark.parametrize("world", [2, 4])
def test_even_all_reduce_counts_never_overwrite_unconsumed_slots(world):
    L = 3
    # decode steps (2 per layer), a 5-row verify (2 per layer), a gamma=4 proposal (3 per token)
    program = [2 * L, 2 * L, 3 * 4, 2 * L, 3 * 4, 2 * L]

    def skewed(rank, step, k):  # rank 0 runs ahead, the last rank lags at every all-reduce
        return 0.0 if rank == 0 else 0.0005 * rank

    assert emulate(world, program, skewed) == []

    import random

    rng = random.Random(world)
    assert emulate(world, program, lambda r, s, k: rng.random() * 0.0005) == []


def test_odd_all_reduce_count_races():
    """A graph with an odd number of all-reduces (gamma = 3 -> 9) ends and the next starts on
    the same buffer: a fast rank overwrites a slow rank's unconsumed slot."""
    def slow_last_reduce(rank, step, k):  # rank 1 is slow to reduce the step's last all-reduce
        return 0.05 if (rank == 1 and step == 0 and k == 9) else 0.0

    violations = emulate(2, [9, 2], lambda r, s, k: 0.0, slow_last_reduce)
    assert violations, "the odd count should let two consecutive all-reduces share a buffer"
    # the same slow reduce with an even count (10) is safe: the next step starts on the other buffer
    assert emulate(2, [10, 2], lambda r, s, k: 0.0,
                   lambda r, s, k: 0.05 if (r == 1 and s == 0 and k == 10) else 0.0) == []


class PDSlots:
    """Decode-side slots and flags of one prefill/decode pair (``parallel.pd`` open-loop serving)."""

    def __init__(self, n_slots):
        self.lock = threading.Lock()
        self.content = {s: (0, True) for s in range(n_slots)}  # slot -> (request epoch, consumed)
        self.ready = {s: 0 for s in range(n_slots)}            # completion flag (epoch)
        self.free = {s: 0 for s in range(n_slots)}             # prefill-side free flag (epoch)
        self.violations = []

    def _wait(self, cond, deadline=5.0):
        t0 = time.time()
        while True:
            with self.lock:
                if cond():
                    return
            if time.time() - t0 > deadline:
                raise TimeoutError("bounded wait gave up")
            time.sleep(0.0002)


def _serve_pair(n_requests, n_slots, *, wait_free=True, seed=0):
    import random

    dev = PDSlots(n_slots)
    rng = random.Random(seed)
    pre_delay = [rng.random() * 0.002 for _ in range(n_requests)]
    dec_delay = [0.002 + rng.random() * 0.004 for _ in range(n_requests)]

    def prefill():
        for i in range(n_requests):
            s, e = i % n_slots, i + 1
            if wait_free and i >= n_slots:  # the decoder released the slot's previous request
                dev._wait(lambda: dev.free[s] >= e - n_slots)
            time.sleep(pre_delay[i])
            with dev.lock:
                old, consumed = dev.content[s]
                if not consumed:
                    dev.violations.append(("overwrite", s, old, e))
                dev.content[s] = (e, False)
                dev.ready[s] = e

    def decode():
        for i in range(n_requests):
            s, e = i % n_slots, i + 1
            dev._wait(lambda: dev.ready[s] >= e)
            time.sleep(dec_delay[i])  # the decode reads the slot for a while
            with dev.lock:
                got, _ = dev.content[s]
                if got != e:
                    dev.violations.append(("read", s, got, e))
                dev.content[s] = (got, True)
                dev.free[s] = e

    threads = [threading.Thread(target=prefill), threading.Thread(target=decode)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(10)
    return dev.violations


@pytest.mark.parametrize("n_slots", [1, 2, 3])
def test_pd_slot_reuse_waits_for_the_decoder(n_slots):
    """Request i of a prefill/decode pair goes to slot i mod S; the prefill rank pushes into a slot only
    after the decoder released the slot's previous request, so no pushed K/V is overwritten unread."""
    for seed in range(3):
        assert _serve_pair(24, n_slots, seed=seed) == []


def test_pd_slot_reuse_without_the_free_flag_races():
    """Dropping the free-flag wait lets a fast prefill overwrite a slot the decoder is still reading."""
    assert any(_serve_pair(24, 2, wait_free=False, seed=s) for s in range(3))


def test_pd_tp_mode_list():
    import pytest

    from sparsecache_b200.parallel.pd_tp import parse_modes

    assert parse_modes("push", 0.0) == ["push"]
    assert parse_modes("push", 2.0) == ["poisson"]  # the single-mode form with a rate
    assert parse_modes("push,nccl,poisson", 2.0) == ["push", "nccl", "poisson"]
    assert parse_modes(" nccl , push ", 0.0) == ["nccl", "push"]
    for bad, rate in (("push,poisson", 0.0), ("tcp", 0.0), ("", 0.0), ("push,push", 0.0)):
        with pytest.raises(ValueError):
            parse_modes(bad, rate)
