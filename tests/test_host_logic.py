"""Host-side logic of the B200 backend on the CPU: the paged prefix cache's LRU bookkeeping (same
contract as engine/backend/prefix_cache.py, with block references instead of
clones), per-slot seeds (engine/backend/executor.py:45-52) and the replica
router, including a world-size-2 gloo run."""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_stateful_b200.runtime.replicas import ReplicaRouter, assign_sessions, max_over_ranks, share_routing

from .conftest import GOLDEN


# ----------------------------------------------------------------------------- prefix cache
class _FakeSched:
    def __init__(self):
        self.dropped = []
        self.entries = []
        self.status = torch.zeros(1, dtype=torch.int32)

    def make_entry(self, slot, n):
        blocks = torch.arange(-(-n // 16), dtype=torch.int32) + 100 * slot
        self.entries.append((slot, n))
        return blocks

    def drop_blocks(self, blocks):
        self.dropped.append(blocks.tolist())

    def share_prefix(self, slot, blocks, n):
        self.shared = (slot, blocks.tolist(), n)


class _FakePool:
    def __init__(self):
        self._sched = _FakeSched()
        self._pending_drops = []

    def flush_drops(self):
        while self._pending_drops:
            self._sched.drop_blocks(self._pending_drops.pop())


def _cache(**kw):
    from test_stateful_b200.runtime.pool import PagedPrefixKVCache
    return PagedPrefixKVCache(_FakePool(), **kw)


def test_prefix_cache_lru_and_block_references():
    c = _cache(max_entries=2)
    assert c.get("x") is None and c.get(None) is None
    c.put("a", 1, 20)
    c.put("b", 2, 17)
    assert c.get("a").prefix_len == 20          # refreshes a
    c.put("c", 3, 5)                            # evicts b, dropping its block references
    assert c.get("b") is None
    assert c._pool._sched.dropped == [[200, 201]]
    assert c.stats["hits"] == 1 and c.stats["misses"] == 3 and c.size == 2
    assert c.invalidate("a") and not c.invalidate("a")
    c.clear()
    assert c.size == 0


def test_prefix_cache_disabled_and_too_long():
    c = _cache(max_entries=0)
    c.put("k", 1, 5)
    assert c.size == 0
    c = _cache(max_entries=4, max_prefix_len=10)
    c.put("long", 1, 20)
    assert c.size == 0 and c._pool._sched.entries == []


def test_prefix_restore_points_slot_at_blocks():
    from test_stateful_b200.runtime.pool import SlotState
    c = _cache()
    c.put("k", 3, 40)
    slot = SlotState(slot_id=7)
    c.restore(slot, c.get("k"))
    assert c._pool._sched.shared == (7, [300, 301, 302], 40)
    assert slot.past_len == 40 and slot.position_offset == 0


# ----------------------------------------------------------------------------- seeds
def test_stable_sampling_seed_matches_reference():
    from test_stateful_b200.runtime.executor import stable_sampling_seed
    z = np.load(os.path.join(GOLDEN, "seeds.npz"), allow_pickle=False)
    for base, sess, seg, want in zip(z["base"], z["session"], z["segment"], z["seed"]):
        assert stable_sampling_seed(int(base), str(sess), int(seg)) == int(want)


# ----------------------------------------------------------------------------- replicas
def test_router_affinity_and_least_loaded():
    r = ReplicaRouter(3, capacity=2)
    assert r.route("s1", "p") == 0
    assert r.route("s2", None) == 1
    assert r.route("s3", "p") == 0       # prefix affinity
    assert r.route("s4", "p") == 2       # home full -> least loaded
    r.release("s1")
    assert r.route("s5", "p") == 0
    assert (r.route("s6", None), r.route("s7", None)) == (1, 2)
    with pytest.raises(RuntimeError):
        r.route("s8", None)


def _worker(rank, world, path, q):
    dist.init_process_group("gloo", init_method=f"file://{path}", rank=rank, world_size=world)
    sessions = [(f"s{i}", f"p{i % 3}") for i in range(10)]
    mine, table = share_routing(sessions, rank, world, capacity=8)
    worst = max_over_ranks(1.5 + rank, world)
    counts = torch.tensor([len(mine)])
    dist.all_reduce(counts)
    q.put((rank, [s for s, _ in mine], table, worst, int(counts.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_routing_and_max_timing():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "rdzv")
        procs = [ctx.Process(target=_worker, args=(r, 2, path, q)) for r in range(2)]
        for p in procs:
            p.start()
        res = sorted(q.get(timeout=120) for _ in procs)
        for p in procs:
            p.join(timeout=60)
    (r0, mine0, table0, w0, n0), (r1, mine1, table1, w1, n1) = res
    assert table0 == table1 == assign_sessions([(f"s{i}", f"p{i % 3}") for i in range(10)], 2, 8)
    assert sorted(mine0 + mine1) == sorted(f"s{i}" for i in range(10))
    assert n0 == n1 == 10
    assert w0 == w1 == 2.5


def test_code2wav_implicit_convolution_rule():
    """Which code2wav convolutions read the history buffer directly (and so get 64-channel
    padded taps in their packed weights): rows per frame a multiple of 128, or a largest call
    of >= 512 rows per stream padded to whole 128-row tiles by at most 1/8 (the device rule,
    ``c2w_implicit_rows``)."""
    from test_stateful_b200.runtime.code2wav import implicit_rows

    t_in, t_blk = [4, 32, 160, 640], [32, 160, 640, 1920]  # decoder blocks, rows per frame
    assert [implicit_rows(t, 1) for t in t_in] == [False, False, False, True]
    assert [implicit_rows(t, 1) for t in t_blk] == [False, False, True, True]
    assert [implicit_rows(t, 25) for t in t_in] == [False, True, True, True]   # 100 < 512 rows
    assert [implicit_rows(t, 25) for t in t_blk] == [True, True, True, True]   # 800 -> 896: 12 %
    assert implicit_rows(100, 6)       # 600 rows -> 640: pads 40 <= 600 / 8
    assert not implicit_rows(70, 7)    # 490 rows: below 512
    assert not implicit_rows(40, 13)   # 520 rows -> 640: pads 120 > 65
