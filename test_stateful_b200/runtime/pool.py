"""Paged KV pool and prefix cache behind the reference's ``KVCachePool`` /
``PrefixKVCache`` interfaces.

The reference pool (engine/backend/kv_cache_pool.py:192-566) hands out whole
per-session slots backed by a slot-contiguous tensor, and its prefix cache
(engine/backend/prefix_cache.py:43-159) stores cloned KV tensors that a hit
copies into the slot (engine/backend/engine_loop.py:823-835).  Here slots are
still the unit the engine loop schedules (same LIFO slot free list, same
``SlotState`` fields), but KV lives in 16-token blocks owned by the device
allocator of ``libqtts_b200.so``: a prefix-cache entry is a list of block ids
holding a reference, and a hit points the new slot at those blocks
(copy-on-write on the first write into a shared partial block).
"""

from __future__ import annotations

import logging
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import List, Optional

import torch

from .. import ops

logger = logging.getLogger(__name__)


@dataclass
class SlotState:
    """Host-side bookkeeping of one session slot: the fields and methods of the reference's
    ``SlotKVState`` (kv_cache_pool.py:63-189) that the engine loop reads and writes.  The
    talker KV is paged (``talker_kv`` stays ``None``; the pool's ``_talker_kv_pool`` view
    serves the loop's prefix reads and restores), and the code2wav state lives on the device,
    so ``c2w_kv`` stays ``None`` and the conv-state lists stay empty: ``pingpong_ready`` is
    False and the loop's state copies have nothing to do."""

    slot_id: int
    session_id: Optional[str] = None
    segment_idx: int = -1
    is_free: bool = True
    prefill_source: str = ""
    talker_kv: Optional[torch.Tensor] = None
    past_len: int = 0
    position_offset: int = 0
    c2w_kv: Optional[torch.Tensor] = None
    c2w_conv_states: Optional[list] = None
    c2w_transconv_states: Optional[list] = None
    frame_idx: int = 0
    _c2w_conv_write: Optional[list] = None
    _c2w_transconv_write: Optional[list] = None
    next_embed: Optional[torch.Tensor] = None
    last_codec_sum: Optional[torch.Tensor] = None
    token_counts: Optional[torch.Tensor] = None
    trailing: list = field(default_factory=list)
    text_idx: int = 0
    token_queue: list = field(default_factory=list)
    steadystream_replay_embeds: list = field(default_factory=list)
    steadystream_full_codecs: list = field(default_factory=list)
    c2w_voiced_snapshot: Optional[dict] = None
    pad_start_frame: int = -1
    pad_consecutive_silence: int = 0
    sampling_seed: Optional[int] = None
    sampling_generator: Optional[torch.Generator] = None
    last_active_time: float = field(default_factory=time.monotonic)

    def reset(self) -> None:
        self.session_id = None
        self.segment_idx = -1
        self.prefill_source = ""
        self.talker_kv = None
        self.past_len = 0
        self.position_offset = 0
        self.c2w_kv = None
        self.c2w_conv_states = None
        self.c2w_transconv_states = None
        self.frame_idx = 0
        self._c2w_conv_write = None
        self._c2w_transconv_write = None
        self.next_embed = None
        self.last_codec_sum = None
        self.token_counts = None
        self.trailing = []
        self.text_idx = 0
        self.token_queue = []
        self.steadystream_replay_embeds = []
        self.steadystream_full_codecs = []
        self.c2w_voiced_snapshot = None
        self.pad_start_frame = -1
        self.pad_consecutive_silence = 0
        self.sampling_seed = None
        self.sampling_generator = None
        self.last_active_time = time.monotonic()

    @property
    def has_c2w_states(self) -> bool:
        return self.c2w_kv is not None

    @property
    def pingpong_ready(self) -> bool:
        return self._c2w_conv_write is not None

    def init_pingpong_buffers(self) -> None:
        """kv_cache_pool.py:145-154: write-side copies of host conv states (none here)."""
        if self.c2w_conv_states:
            self._c2w_conv_write = [t.clone() for t in self.c2w_conv_states]
        if self.c2w_transconv_states:
            self._c2w_transconv_write = [t.clone() for t in self.c2w_transconv_states]

    def flip_c2w_buffers(self) -> None:
        self.c2w_conv_states, self._c2w_conv_write = self._c2w_conv_write, self.c2w_conv_states
        self.c2w_transconv_states, self._c2w_transconv_write = (self._c2w_transconv_write,
                                                                self.c2w_transconv_states)

    def copy_c2w_and_flip(self, conv_sources: list, transconv_sources: list) -> None:
        if self._c2w_conv_write is not None:
            for j, src in enumerate(conv_sources):
                if src is not None:
                    self._c2w_conv_write[j].copy_(src)
        if self._c2w_transconv_write is not None:
            for j, src in enumerate(transconv_sources):
                if src is not None:
                    self._c2w_transconv_write[j].copy_(src)
        self.flip_c2w_buffers()

    def touch(self) -> None:
        self.last_active_time = time.monotonic()

    @property
    def idle_seconds(self) -> float:
        return time.monotonic() - self.last_active_time


class PagedKVCachePool:
    """Slot allocator + paged KV state (``KVCachePool`` API)."""

    def __init__(self, model, max_slots: int):
        self._model = model
        self._pool = model.pool
        self._sched = ops.Sched(self._pool)
        self._max_slots = max_slots
        self._cfg = model.cfg
        self._slots: List[SlotState] = [SlotState(slot_id=i) for i in range(max_slots)]
        self._free_slots: List[int] = list(range(max_slots))
        self._pending_drops: List[torch.Tensor] = []
        self._closed = False
        self._preallocate = True
        # the engine loop's prefix reads and restores index this like the reference's
        # slot-contiguous tensor (engine_loop.py:823-835, 952-964); here they take and
        # share block references
        self._talker_kv_pool = PagedTalkerKV(self)

    # -- block references released by handles (see BlockRefs) ----------------
    def flush_drops(self) -> None:
        """Drop the block references of prefix handles that went away since the last call."""
        while self._pending_drops:
            blocks = self._pending_drops.pop()
            if not self._closed:
                self._sched.drop_blocks(blocks)

    def close(self) -> None:
        """The device state is going away (executor shutdown): references released later are
        not sent to it."""
        self._closed = True
        self._pending_drops.clear()

    # -- KVCachePool surface -------------------------------------------------
    @property
    def max_seq_len(self) -> int:
        return self._cfg.pool.max_seq_len

    @property
    def free_count(self) -> int:
        return len(self._free_slots)

    @property
    def used_count(self) -> int:
        return self._max_slots - len(self._free_slots)

    @property
    def utilization(self) -> float:
        return 0.0 if self._max_slots == 0 else self.used_count / self._max_slots

    @property
    def free_blocks(self) -> int:
        return int(self._pool.free_top.item())

    def allocate(self, session_id: str) -> Optional[SlotState]:
        """Same LIFO choice as kv_cache_pool.py:269-306; no KV zeroing is needed
        because a paged slot starts with an empty block table."""
        self.flush_drops()
        if not self._free_slots:
            return None
        sid = self._free_slots.pop()
        slot = self._slots[sid]
        slot.reset()
        slot.session_id = session_id
        slot.is_free = False
        return slot

    def release(self, slot_id: int) -> None:
        slot = self._slots[slot_id]
        if slot.is_free:
            return
        self.flush_drops()
        self._sched.release(slot_id)
        slot.reset()
        slot.is_free = True
        self._free_slots.append(slot_id)

    def get(self, slot_id: int) -> SlotState:
        return self._slots[slot_id]

    def get_by_session(self, session_id: str) -> Optional[SlotState]:
        for s in self._slots:
            if not s.is_free and s.session_id == session_id:
                return s
        return None

    def active_slots(self) -> List[SlotState]:
        return [s for s in self._slots if not s.is_free]

    def init_kv_tensors(self, slot: SlotState) -> None:
        self._model_counts_reset(slot.slot_id)

    def reset_for_new_segment(self, slot: SlotState) -> None:
        slot.text_idx = 0
        slot.trailing = []
        slot.next_embed = None
        slot.last_codec_sum = None
        slot.token_queue = []
        slot.pad_start_frame = -1
        slot.pad_consecutive_silence = 0
        slot.sampling_seed = None

    def scatter_prefill_kv(self, slot_id: int, kv: torch.Tensor, seq_len: int) -> None:
        """Append ``kv [1, L*2, H, >=seq_len, D]`` to an empty slot (kv_cache_pool.py:383-395)."""
        if self._slots[slot_id].past_len != 0:
            raise ValueError("scatter_prefill_kv needs an empty slot")
        self._append_rows(slot_id, kv[0, :, :, :seq_len].permute(2, 0, 1, 3))
        self._slots[slot_id].past_len = seq_len

    def scatter_talker_kv_delta(self, slot_ids, delta_kv: Optional[torch.Tensor], original_past_lens) -> None:
        """kv_cache_pool.py:480-498.  The B200 step already stored its KV in the
        pool, so the executor's outputs carry ``batch_talker_kv=None``; explicit
        deltas (e.g. from another backend) are appended here."""
        if delta_kv is None:
            return
        cap = self.max_seq_len
        for i, (sid, pl) in enumerate(zip(slot_ids, original_past_lens)):
            if pl >= cap:
                continue
            n = min(int(delta_kv.shape[3]), cap - pl)
            self._append_rows(sid, delta_kv[i, :, :, :n].permute(2, 0, 1, 3))

    def gather_talker_kv(self, slot_ids, max_past_len: int) -> torch.Tensor:
        """``[B, L*2, H, max_past_len, D]`` zero-padded (kv_cache_pool.py:410-420)."""
        t = self._cfg.talker
        out = torch.zeros(len(slot_ids), 2 * t.num_layers, t.kv_heads, max_past_len, t.head_dim,
                          device=self._pool.kv.device, dtype=torch.float16)
        for i, sid in enumerate(slot_ids):
            n = min(int(self._pool.seq_len[sid].item()), max_past_len)
            if n > 0:
                out[i, :, :, :n] = self._sched.gather(sid, n)
        return out

    def find_eviction_candidate(self, max_idle_sec: float = 10.0) -> Optional[SlotState]:
        best = None
        for s in self._slots:
            if s.is_free or s.idle_seconds < max_idle_sec:
                continue
            if best is None or s.idle_seconds > best.idle_seconds:
                best = s
        return best

    def force_evict(self, slot_id: int) -> Optional[str]:
        slot = self._slots[slot_id]
        if slot.is_free:
            return None
        sid = slot.session_id
        logger.warning("Force-evicting slot %d (session=%s)", slot_id, sid)
        self.release(slot_id)
        return sid

    # -- paged helpers -------------------------------------------------------
    def _append_rows(self, slot_id: int, rows: torch.Tensor) -> None:
        """rows ``[n, L*2, Hkv, D]``: reserve n positions, then write them."""
        n = rows.shape[0]
        slots = torch.tensor([slot_id], dtype=torch.int32, device=self._pool.kv.device)
        mapping, _, _, cs, cd = self._sched.append(slots, n)
        self._sched.copy_blocks(cs, cd)
        self._sched.scatter(rows.to(torch.float16).contiguous(), mapping)
        st = int(self._sched.status.item())
        if st != 0:
            raise ValueError(f"KV append failed with status {st}")

    def _model_counts_reset(self, slot_id: int) -> None:
        hook = getattr(self, "counts_reset_hook", None)
        if hook is not None:
            hook(slot_id)


class BlockRefs:
    """One device reference on each KV block of a cached prefix.  Handles that share it keep
    it alive; when the last one goes away the blocks are queued on the pool and their
    references dropped at the pool's next host call (never from inside the garbage collector,
    which may run while a CUDA graph is being captured)."""

    def __init__(self, pool, blocks: torch.Tensor):
        self.pool = pool
        self.blocks = blocks

    def __del__(self):
        q = getattr(self.pool, "_pending_drops", None)
        if q is not None:
            q.append(self.blocks)


class PagedKVHandle:
    """The first ``prefix_len`` positions of a talker KV, as references to paged blocks.

    It stands where the reference passes a cloned ``[1, L*2, Hkv, n, D]`` tensor: what
    ``_read_prefix_kv`` returns and ``PrefixKVCache.put`` stores (engine_loop.py:952-964,
    prefix_cache.py:101-148), and what ``_restore_prefix_cache`` assigns into the pool
    (engine_loop.py:823-835).  ``clone()`` shares the references instead of copying KV;
    indexing ``[0, :, :, :n, :]`` gives the first n positions."""

    def __init__(self, refs: BlockRefs, prefix_len: int, shape_tail=(0, 0, 0)):
        self._refs = refs
        self.prefix_len = int(prefix_len)
        self._tail = shape_tail  # (L*2, Hkv, D)

    @property
    def blocks(self) -> torch.Tensor:
        return self._refs.blocks[: -(-self.prefix_len // 16)]

    @property
    def shape(self) -> tuple:
        l2, h, d = self._tail
        return (1, l2, h, self.prefix_len, d)

    def clone(self) -> "PagedKVHandle":
        return PagedKVHandle(self._refs, self.prefix_len, self._tail)

    def contiguous(self) -> "PagedKVHandle":
        return self

    def __getitem__(self, key) -> "PagedKVHandle":
        n = _positions(key, self.prefix_len)
        return PagedKVHandle(self._refs, min(n, self.prefix_len), self._tail)


def _positions(key, default: int) -> int:
    """The stop of the position slice (4th index) of a ``[b, l, h, :n, d]`` subscript."""
    if isinstance(key, tuple) and len(key) >= 4 and isinstance(key[3], slice):
        sl = key[3]
        if sl.start not in (None, 0) or sl.step not in (None, 1):
            raise ValueError("paged KV views take positions [0, n) only")
        return default if sl.stop is None else int(sl.stop)
    return default


def _slot_of(key) -> int:
    first = key[0] if isinstance(key, tuple) else key
    if isinstance(first, slice):
        if first.stop is not None and first.start is not None and first.stop - first.start != 1:
            raise ValueError("paged KV views address one slot at a time")
        return int(first.start or 0)
    return int(first)


class PagedTalkerKV:
    """``kv_pool._talker_kv_pool`` of the paged pool: answers the two subscripts the engine
    loop applies to the reference's ``[slots, L*2, Hkv, max_seq, D]`` tensor.

    * ``pool[slot:slot+1, :, :, :n, :]`` (``_read_prefix_kv``) takes a reference on the
      slot's first ceil(n/16) blocks and returns a ``PagedKVHandle``;
    * ``pool[slot, :, :, :n, :] = handle`` (``_restore_prefix_cache``) points the empty slot
      at the handle's blocks (copy-on-write of a shared partial block happens on the slot's
      first write); assigning a tensor ``[L*2, Hkv, n, D]`` instead writes its rows into the
      slot's own blocks."""

    def __init__(self, pool: "PagedKVCachePool"):
        self._p = pool

    @property
    def shape(self) -> tuple:
        t, c = self._p._cfg.talker, self._p._cfg.pool
        return (self._p._max_slots, 2 * t.num_layers, t.kv_heads, c.max_seq_len, t.head_dim)

    def _tail(self):
        t = self._p._cfg.talker
        return (2 * t.num_layers, t.kv_heads, t.head_dim)

    def __getitem__(self, key) -> PagedKVHandle:
        slot = _slot_of(key)
        have = self._p._slots[slot].past_len
        n = _positions(key, have)
        if n < 1 or n > have:
            raise ValueError(f"slot {slot} holds {have} positions, {n} requested")
        self._p.flush_drops()
        blocks = self._p._sched.make_entry(slot, n)
        return PagedKVHandle(BlockRefs(self._p, blocks), n, self._tail())

    def __setitem__(self, key, value) -> None:
        slot = _slot_of(key)
        if isinstance(value, PagedKVHandle):
            n = min(_positions(key, value.prefix_len), value.prefix_len)
            self._p.flush_drops()
            self._p._sched.share_prefix(slot, value.blocks, n)
            st = int(self._p._sched.status.item())
            if st != 0:
                raise ValueError(f"prefix restore into slot {slot} failed (status {st})")
            return
        kv = value[0] if value.dim() == 5 else value          # [L*2, Hkv, n, D]
        n = min(_positions(key, kv.shape[2]), kv.shape[2])
        self._p._append_rows(slot, kv[:, :, :n].permute(2, 0, 1, 3))


@dataclass(frozen=True)
class PagedPrefixEntry:
    """A cached prefix (``PrefixCacheEntry``, prefix_cache.py:33-40): ``talker_kv`` is a
    handle holding references on the prefix's blocks."""

    key: str
    talker_kv: PagedKVHandle
    prefix_len: int
    created_at: float
    hit_count: int = 0

    @property
    def blocks(self) -> torch.Tensor:
        return self.talker_kv.blocks


class PagedPrefixKVCache:
    """LRU of cached prefixes (``PrefixKVCache`` API and semantics, prefix_cache.py:43-159).

    ``put(key, kv, prefix_len)`` takes the handle the pool's ``_talker_kv_pool`` view returned
    (or a slot id, whose first ``prefix_len`` positions are referenced) and keeps a shared
    reference instead of a clone; ``restore(slot, entry)`` points an empty slot at the blocks
    instead of copying them; eviction / ``invalidate`` / ``clear`` drop the entry, and the
    blocks return to the free stack once no slot or handle uses them.  The reference's own
    ``PrefixKVCache`` works on this pool too: it stores the handle's ``clone()``.
    """

    def __init__(self, pool: PagedKVCachePool, max_entries: int = 16, max_prefix_len: int = 512):
        self._pool = pool
        self._max_entries = max_entries
        self._max_prefix_len = max_prefix_len
        self._cache: "OrderedDict[str, PagedPrefixEntry]" = OrderedDict()
        self._total_hits = 0
        self._total_misses = 0

    @property
    def size(self) -> int:
        return len(self._cache)

    @property
    def max_prefix_len(self) -> int:
        return self._max_prefix_len

    @property
    def stats(self) -> dict:
        return {"size": self.size, "max_entries": self._max_entries, "hits": self._total_hits,
                "misses": self._total_misses,
                "hit_rate": self._total_hits / max(1, self._total_hits + self._total_misses)}

    def get(self, key: Optional[str]) -> Optional[PagedPrefixEntry]:
        if key is None or key not in self._cache:
            self._total_misses += 1
            return None
        self._cache.move_to_end(key)
        self._total_hits += 1
        e = self._cache[key]
        object.__setattr__(e, "hit_count", e.hit_count + 1)
        return e

    def put(self, key: Optional[str], talker_kv, prefix_len: int) -> None:
        """Cache the first ``prefix_len`` positions of ``talker_kv``: a ``PagedKVHandle`` (as
        the engine loop reads it from the pool) or a slot id holding them."""
        if key is None or self._max_entries <= 0 or prefix_len > self._max_prefix_len:
            return
        if key in self._cache:
            self._cache.move_to_end(key)
            return
        while len(self._cache) >= self._max_entries:
            self._cache.popitem(last=False)
        if isinstance(talker_kv, PagedKVHandle):
            handle = talker_kv[0, :, :, :prefix_len, :]
        else:
            blocks = self._pool._sched.make_entry(int(talker_kv), prefix_len)
            handle = PagedKVHandle(BlockRefs(self._pool, blocks), prefix_len, _tail_of(self._pool))
        self._cache[key] = PagedPrefixEntry(key=key, talker_kv=handle, prefix_len=prefix_len,
                                            created_at=time.monotonic())
        _flush(self._pool)

    def restore(self, slot: SlotState, entry) -> None:
        """engine_loop._restore_prefix_cache without the copy; ``entry`` is a cached entry or
        a handle (e.g. ``entry.talker_kv[0, :, :, :n, :]`` for a shorter prefix)."""
        _flush(self._pool)
        self._pool._sched.share_prefix(slot.slot_id, entry.blocks, entry.prefix_len)
        st = int(self._pool._sched.status.item())
        if st != 0:
            raise ValueError(f"prefix restore into slot {slot.slot_id} failed (status {st})")
        slot.past_len = entry.prefix_len
        slot.position_offset = 0

    def invalidate(self, key: str) -> bool:
        found = self._cache.pop(key, None) is not None
        _flush(self._pool)
        return found

    def clear(self) -> None:
        self._cache.clear()
        _flush(self._pool)


def _flush(pool) -> None:
    flush = getattr(pool, "flush_drops", None)
    if flush is not None:
        flush()


def _tail_of(pool) -> tuple:
    cfg = getattr(pool, "_cfg", None)
    if cfg is None:
        return (0, 0, 0)
    t = cfg.talker
    return (2 * t.num_layers, t.kv_heads, t.head_dim)
