"""ZeRO-3 prefetching parameter gather: slot and plan bookkeeping with a stand-in for the native
stream/event/copy object (CPU; the copies themselves are exercised by the GPU engine tests)."""

from __future__ import annotations

import torch

from cs244c_llama_zero_b200.parallel.zero.base import CommClock
from cs244c_llama_zero_b200.parallel.zero.stage3 import _PullGather


class FakeNative:
    def __init__(self):
        self.log = []
        self.pg = None

    def prefetch(self, ctx, slot, off, nbytes, dst, cat, timed):
        assert self.pg.bound[slot] is None, "prefetch into a slot that a module still uses"
        self.log.append(("prefetch", slot, off))

    def gather_now(self, ctx, slot, off, nbytes, dst, cat, timed):
        assert self.pg.bound[slot] is None
        self.log.append(("now", slot, off))

    def acquire(self, slot):
        self.log.append(("acquire", slot))

    def release(self, slot):
        self.log.append(("release", slot))

    def mark_ready(self):
        self.log.append(("ready",))

    def join(self):
        self.log.append(("join",))

    def take_times(self):
        return [0.0, 0.0], [0, 0]


class FakeHandle:
    def __init__(self, name, shard):
        self.name = name
        self.param_shard = shard
        self.chunk = shard.numel()
        self.padded_numel = 2 * self.chunk
        self.full_param_bytes = 2 * self.padded_numel
        self.materialized = False


class FakeCollectives:
    def __init__(self, base):
        self.base = base
        self.barriers = 0

    def locate_symmetric(self, t):
        return "ctx", (t.data_ptr() - self.base) * 1  # byte offsets of a uint8 store

    def barrier(self):
        self.barriers += 1


class FakeEngine:
    def __init__(self, names, chunk=64):
        self.device = torch.device("cpu")
        self.world_size = 2
        self.store = torch.zeros(len(names) * chunk, dtype=torch.uint8)
        self._handle_order = [FakeHandle(n, self.store[i * chunk:(i + 1) * chunk]) for i, n in enumerate(names)]
        self.clock = CommClock(self.device)
        self.collectives = FakeCollectives(self.store.data_ptr())


def _setup(names=("emb", "l0", "l1", "norm")):
    eng = FakeEngine(names)
    native = FakeNative()
    slots = [torch.zeros(2 * 64, dtype=torch.uint8) for _ in range(2)]
    pg = _PullGather(eng, eng.store, slots, native=native)
    native.pg = pg
    return eng, pg, native, {h.name: h for h in eng._handle_order}


def _step(pg, h, order):
    """Run forward then backward of a module sequence, each module gathered, used and released."""
    pg.begin_forward()
    calls = [(n, "forward") for n in order] + [(n, "backward") for n in reversed(order)]
    for name, phase in calls:
        handle = h[name]
        full = pg.materialize(handle, phase)
        assert full is not None and full.numel() == handle.padded_numel
        handle.materialized = True
        pg.release(handle)
        handle.materialized = False


def _kinds(log):
    return [e[0] for e in log]


def test_second_step_is_fully_prefetched():
    eng, pg, native, h = _setup()
    order = ["emb", "l0", "l1", "norm", "emb"]  # tied LM head reuses the embedding handle
    pg.after_store_write(next_plan=False)
    _step(pg, h, order)
    assert _kinds(native.log).count("now") == 10 and "prefetch" not in _kinds(native.log)
    pg.before_store_write()
    pg.after_store_write(next_plan=True)
    assert native.log[-1][0] == "prefetch"  # the next step's first module, right after the barrier
    native.log.clear()
    _step(pg, h, order)
    kinds = _kinds(native.log)
    assert "now" not in kinds, native.log
    assert kinds.count("acquire") == 10 and kinds.count("prefetch") == 9
    assert eng.collectives.barriers == 2


def test_mismatched_order_falls_back_to_direct_gathers():
    eng, pg, native, h = _setup()
    pg.after_store_write(next_plan=False)
    _step(pg, h, ["emb", "l0", "l1", "norm"])
    pg.before_store_write()
    pg.after_store_write(next_plan=True)
    native.log.clear()
    _step(pg, h, ["emb", "l1", "l0", "norm"])  # a different module order than the recorded plan
    kinds = _kinds(native.log)
    assert kinds[0] == "acquire"          # the prefetched first module is still used
    assert "now" in kinds                 # later ones are gathered on demand
    assert pg.plan is None and kinds.count("acquire") + kinds.count("now") == 8
    # the step after follows the new order again with prefetches only
    pg.before_store_write()
    pg.after_store_write(next_plan=True)
    native.log.clear()
    _step(pg, h, ["emb", "l1", "l0", "norm"])
    assert "now" not in _kinds(native.log)


def test_store_write_joins_and_drops_pending_prefetches():
    eng, pg, native, h = _setup()
    pg.after_store_write(next_plan=False)
    _step(pg, h, ["emb", "l0"])
    pg.before_store_write()
    pg.after_store_write(next_plan=True)
    assert pg.pending  # first module prefetched
    pg.before_store_write()  # e.g. load_state_dict rewrites the store
    assert not pg.pending and native.log[-1] == ("join",)


def test_gathers_appear_in_the_collective_trace():
    eng, pg, native, h = _setup(("emb", "l0"))
    records = []
    pg.record_gather = lambda *rec: records.append(rec)  # what TracingCollectives.record_external receives
    pg.after_store_write(next_plan=False)
    _step(pg, h, ["emb", "l0"])
    labels = [r[1] for r in records]
    assert labels == ["stage3.forward.allgather.emb", "stage3.forward.allgather.l0",
                      "stage3.backward.allgather.l0", "stage3.backward.allgather.emb"]
    assert all(r[0] == "allgather" and r[2] == 64 and r[3] == 128 for r in records)
