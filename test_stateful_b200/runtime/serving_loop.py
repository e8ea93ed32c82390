"""Continuous-batching serving loop of one replica, for the whole-box workload.

The reference's ``EngineLoop._run`` (engine/backend/engine_loop.py:281-324) repeats the
same phases every iteration: admit the sessions that arrived, prefill at most one request
(``_try_prefill_one``, :498 — a prefix-cache hit restores the cached KV and prefills only the
request's suffix, a miss prefills the prefix, caches it and then the suffix, :801-835,
893-928), launch one decode step over the running slots (``launch_decode_step``), wait for it,
and retire the sessions that are done.  ``serve_replica`` runs those phases over a timed list
of arrivals against a ``B200Executor``; prompts (the suffix after a shared prefix included)
are prefilled in chunks (``iter_prefill``: one engine step per chunk), so a long prompt holds
the running streams back by one chunk per iteration, not by the whole prompt.

A request here is what reaches the decode path: its arrival time, its prompt ids (after the
shared prefix, if it has one), the index of its shared prefix, and the number of codec frames
to generate (the first comes from the prefill).  The text front end, the gateway and the
per-session audio assembly are outside the path and not modelled.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from .. import workload


@dataclass
class Request:
    rid: str
    arrival: float                 # seconds after the start of the run
    ids: torch.Tensor              # prompt ids after the shared prefix (the whole prompt without one)
    prefix: Optional[int] = None   # index of the shared prefix, or None
    frames: int = 1                # codec frames to generate, the prefill's frame included


@dataclass
class ServeStats:
    frames: int = 0                # codec frames generated (prefill frames included)
    decode_steps: int = 0
    wall_s: float = 0.0            # first arrival to the last frame
    completed: int = 0
    max_running: int = 0
    prefix_hits: int = 0
    prefix_misses: int = 0
    prefill_calls: int = 0         # engine steps spent on prompts
    ttfa_s: List[float] = field(default_factory=list)   # arrival -> first frame, per request
    step_s: List[float] = field(default_factory=list)   # wall time of each decode step


def cfg5_requests(n: int, rate: float, seed: int, prefix_len: int = 96, n_prefixes: int = 8, share: float = 0.3,
                  lo: int = 8, hi: int = 128, fmin: int = 25, fmax: int = 250
                  ) -> Tuple[List[Request], List[torch.Tensor]]:
    """The whole-box workload's arrivals: a Poisson process of ``rate`` requests/s (the first at
    t = 0), prompts of U{lo..hi} random ids, U{fmin..fmax} frames (2-20 s of audio at 12.5 Hz),
    and a fraction ``share`` of the requests opening with one of ``n_prefixes`` random
    ``prefix_len``-id prefixes.  Returns ``(requests, prefixes)``; seeded, the same on every rank."""
    if n < 1 or rate <= 0:
        raise ValueError("need n >= 1 and rate > 0")
    g = workload._gen(seed, 29)
    gaps = torch.empty(n, dtype=torch.float64).exponential_(generator=g) / rate
    arrivals = torch.cumsum(gaps, 0) - gaps[0]
    prefixes = [torch.randint(0, workload.TEXT_VOCAB, (prefix_len,), generator=g) for _ in range(n_prefixes)]
    reqs = []
    for i in range(n):
        shared = float(torch.rand((), generator=g, dtype=torch.float64)) < share
        k = int(torch.randint(0, n_prefixes, (), generator=g))
        length = int(torch.randint(lo, hi + 1, (), generator=g))
        ids = torch.randint(0, workload.TEXT_VOCAB, (length,), generator=g)
        frames = int(torch.randint(fmin, fmax + 1, (), generator=g))
        reqs.append(Request(f"req-{i}", float(arrivals[i]), ids, k if shared else None, frames))
    return reqs, prefixes


def prefix_key(req: Request) -> Optional[str]:
    return None if req.prefix is None else f"prefix-{req.prefix}"


def serve_replica(ex, requests: Sequence[Request], prefixes: Sequence[torch.Tensor], table: torch.Tensor,
                  pad: torch.Tensor, prefill_chunk: int = 64, clock: Callable[[], float] = time.perf_counter,
                  sleep: Callable[[float], None] = time.sleep) -> ServeStats:
    """Serve ``requests`` (arrival times relative to the call) on one executor until every one
    has produced its frames.  ``table`` maps prompt ids to input embeddings and ``pad`` is the
    text embedding added to every frame (``workload.text_table`` / ``tts_pad_embed``)."""
    dev = ex._device
    pool = ex.kv_pool
    prefix_len = int(prefixes[0].numel()) if len(prefixes) else 0
    cache = ex.make_prefix_cache(max_entries=max(1, len(prefixes)), max_prefix_len=max(512, prefix_len))

    def emb(ids: torch.Tensor) -> torch.Tensor:
        return table[ids.to(table.device)].to(dev).unsqueeze(0)

    queue = deque(sorted(requests, key=lambda r: r.arrival))
    waiting: deque = deque()
    running: list = []
    made: dict = {}
    goal: dict = {}
    prefill = None  # (request, slot, generator of iter_prefill steps)
    st = ServeStats()
    t0 = clock()
    while queue or waiting or running or prefill is not None:
        now = clock() - t0
        while queue and queue[0].arrival <= now:  # phase 1: admit
            waiting.append(queue.popleft())
        if prefill is None and waiting and pool.free_count > 0:  # phase 2: start a prefill
            req = waiting.popleft()
            slot = pool.allocate(req.rid)
            slot.segment_idx = 0
            pool.init_kv_tensors(slot)  # a new session: its token counts start at zero
            ex.set_text_embedding(slot, pad)
            key = prefix_key(req)
            if key is not None:
                entry = cache.get(key)
                if entry is None:  # miss: prefill the prefix, cache it by block reference
                    st.prefix_misses += 1
                    ex.prefill_prefix_only(slot, emb(prefixes[req.prefix]))
                    cache.put(key, slot.slot_id, prefix_len)
                    st.prefill_calls += 1
                else:
                    st.prefix_hits += 1
                    cache.restore(slot, entry)
                gen = ex.iter_prefill(slot, emb(req.ids), prefill_chunk, keep_kv=True)  # the suffix
            else:
                gen = ex.iter_prefill(slot, emb(req.ids), prefill_chunk)
            prefill = (req, slot, gen)
        if prefill is not None:  # one prefill chunk per iteration
            req, slot, gen = prefill
            st.prefill_calls += 1
            if next(gen) is not None:  # the prompt is in and its first frame sampled
                st.ttfa_s.append(clock() - t0 - req.arrival)
                st.frames += 1
                made[slot.slot_id] = 1
                goal[slot.slot_id] = req.frames
                if req.frames > 1:
                    running.append(slot)
                else:
                    pool.release(slot.slot_id)
                    st.completed += 1
                prefill = None
        if running:  # phase 3: one decode step of every running stream
            ts = clock()
            ex.launch_decode_step(running).wait()
            ex.advance(running)
            st.step_s.append(clock() - ts)
            st.decode_steps += 1
            st.frames += len(running)
            st.max_running = max(st.max_running, len(running))
            keep = []
            for s in running:  # phase 4: retire
                made[s.slot_id] += 1
                if made[s.slot_id] >= goal[s.slot_id]:
                    pool.release(s.slot_id)
                    st.completed += 1
                else:
                    keep.append(s)
            running = keep
        elif prefill is None and not waiting and queue:  # idle until the next arrival
            sleep(max(0.0, queue[0].arrival - (clock() - t0)))
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    st.wall_s = clock() - t0
    cache.clear()
    return st


def percentile(xs: Sequence[float], q: float) -> Optional[float]:
    if not xs:
        return None
    s = sorted(xs)
    i = min(len(s) - 1, max(0, int(round(q / 100.0 * (len(s) - 1)))))
    return float(s[i])
