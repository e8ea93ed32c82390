"""The whole-box workload's host side on the CPU: the seeded arrival list (Poisson rate,
prompt and frame ranges, the shared-prefix fraction) and the serving loop's phases
(admit, one prefill chunk per iteration, decode, retire) against a stand-in executor
that records every call.  No GPU: the loop only calls the executor's public surface."""

from types import SimpleNamespace

import torch

from test_stateful_b200.runtime.serving_loop import Request, cfg5_requests, percentile, serve_replica


def test_cfg5_requests_distribution_and_determinism():
    a, pa = cfg5_requests(2000, 200.0, 5)
    b, pb = cfg5_requests(2000, 200.0, 5)
    assert [r.arrival for r in a] == [r.arrival for r in b] and all(torch.equal(x, y) for x, y in zip(pa, pb))
    arr = [r.arrival for r in a]
    assert arr[0] == 0.0 and all(x <= y for x, y in zip(arr, arr[1:]))
    rate = (len(arr) - 1) / arr[-1]
    assert 185.0 < rate < 215.0  # Poisson at 200 req/s
    share = sum(r.prefix is not None for r in a) / len(a)
    assert 0.27 < share < 0.33
    assert {r.prefix for r in a if r.prefix is not None} == set(range(8))
    assert all(8 <= r.ids.numel() <= 128 for r in a)
    assert all(25 <= r.frames <= 250 for r in a)
    assert len(pa) == 8 and all(p.numel() == 96 for p in pa)


class _Clock:
    def __init__(self, dt):
        self.t, self.dt = 0.0, dt

    def __call__(self):
        self.t += self.dt
        return self.t

    def sleep(self, s):
        self.t += s


class _Pool:
    def __init__(self, n):
        self.slots = [SimpleNamespace(slot_id=i, past_len=0, frame_idx=0, segment_idx=0) for i in range(n)]
        self.free = list(range(n))[::-1]
        self.max_in_use = 0

    @property
    def free_count(self):
        return len(self.free)

    def allocate(self, sid):
        if not self.free:
            return None
        s = self.slots[self.free.pop()]
        s.past_len = s.frame_idx = 0
        self.max_in_use = max(self.max_in_use, len(self.slots) - len(self.free))
        return s

    def release(self, i):
        assert i not in self.free
        self.free.append(i)

    def init_kv_tensors(self, slot):
        pass


class _Cache:
    def __init__(self, log):
        self.entries, self.log = {}, log

    def get(self, key):
        return self.entries.get(key)

    def put(self, key, slot_id, n):
        self.entries[key] = SimpleNamespace(prefix_len=n)
        self.log.append(("put", key, slot_id, n))

    def restore(self, slot, entry):
        slot.past_len = entry.prefix_len
        self.log.append(("restore", slot.slot_id))

    def clear(self):
        self.entries.clear()


class _Executor:
    """Records the calls; a prefill appends its rows, a decode step one row per slot."""

    def __init__(self, n_slots):
        self._device = torch.device("cpu")
        self.kv_pool = _Pool(n_slots)
        self.log = []
        self.batches = []

    def make_prefix_cache(self, max_entries, max_prefix_len):
        return _Cache(self.log)

    def set_text_embedding(self, slot, emb):
        pass

    def prefill_prefix_only(self, slot, e):
        slot.past_len += e.shape[1]
        self.log.append(("prefix_only", slot.slot_id, e.shape[1]))

    def prefill_from_prefix(self, slot, e):
        slot.past_len += e.shape[1]
        slot.frame_idx += 1
        self.log.append(("from_prefix", slot.slot_id, e.shape[1]))
        return b"", False

    def iter_prefill(self, slot, e, chunk, keep_kv=False):
        n = e.shape[1]
        if not keep_kv:
            assert slot.past_len == 0
        for start in range(0, n, chunk):
            slot.past_len += min(chunk, n - start)
            self.log.append(("suffix" if keep_kv else "chunk", slot.slot_id, min(chunk, n - start)))
            if start + chunk < n:
                yield None
        slot.frame_idx += 1
        yield b"", False

    def launch_decode_step(self, slots):
        assert len({s.slot_id for s in slots}) == len(slots)
        self.batches.append([s.slot_id for s in slots])
        return SimpleNamespace(wait=lambda: None)

    @staticmethod
    def advance(slots):
        for s in slots:
            s.past_len += 1
            s.frame_idx += 1


def test_serve_replica_phases_and_accounting():
    reqs, prefixes = cfg5_requests(40, 400.0, 7, prefix_len=16, lo=8, hi=100, fmin=1, fmax=12)
    ex = _Executor(6)
    clk = _Clock(1e-4)
    table = torch.randn(4096, 4)
    st = serve_replica(ex, reqs, prefixes, table, torch.zeros(4), prefill_chunk=32, clock=clk, sleep=clk.sleep)
    assert st.completed == len(reqs)
    assert st.frames == sum(r.frames for r in reqs)
    assert len(st.ttfa_s) == len(reqs) and min(st.ttfa_s) >= 0.0
    assert ex.kv_pool.free_count == 6 and ex.kv_pool.max_in_use <= 6
    assert st.max_running <= 6 and st.decode_steps == len(ex.batches)
    # every prompt's rows reached the engine exactly once, in chunks of <= 32
    rows = {}
    for e in ex.log:
        if e[0] in ("chunk", "suffix"):
            rows[e[0]] = rows.get(e[0], 0) + e[2]
    assert rows.get("chunk", 0) == sum(r.ids.numel() for r in reqs if r.prefix is None)
    assert rows.get("suffix", 0) == sum(r.ids.numel() for r in reqs if r.prefix is not None)
    assert all(e[2] <= 32 for e in ex.log if e[0] in ("chunk", "suffix"))
    # the first request of each prefix prefills and caches it; later ones restore
    used = {r.prefix for r in reqs if r.prefix is not None}
    assert st.prefix_misses == len(used) == sum(e[0] == "put" for e in ex.log)
    assert st.prefix_hits == sum(r.prefix is not None for r in reqs) - len(used)
    # a request runs for its frames: decode steps per slot session = frames - 1
    assert sum(len(b) for b in ex.batches) == sum(r.frames - 1 for r in reqs)


def test_serve_replica_waits_for_arrivals():
    reqs = [Request("a", 0.0, torch.arange(10), None, 3), Request("b", 5.0, torch.arange(10), None, 2)]
    ex = _Executor(2)
    clk = _Clock(1e-3)
    st = serve_replica(ex, reqs, [], torch.randn(16, 4), torch.zeros(4), prefill_chunk=64, clock=clk,
                       sleep=clk.sleep)
    assert st.completed == 2 and st.frames == 5
    assert st.wall_s >= 5.0  # the second request is served after it arrives
    assert percentile([3.0, 1.0, 2.0], 50) == 2.0 and percentile([], 50) is None
