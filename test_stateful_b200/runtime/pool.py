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
    """Host-side bookkeeping of one session slot (fields of ``SlotKVState``,
    kv_cache_pool.py:63-135, minus the per-slot KV tensors, which are paged)."""

    slot_id: int
    session_id: Optional[str] = None
    segment_idx: int = -1
    is_free: bool = True
    prefill_source: str = ""
    past_len: int = 0
    position_offset: int = 0
    frame_idx: int = 0
    next_embed: Optional[torch.Tensor] = None
    last_codec_sum: Optional[torch.Tensor] = None
    trailing: list = field(default_factory=list)
    text_idx: int = 0
    token_queue: list = field(default_factory=list)
    pad_start_frame: int = -1
    pad_consecutive_silence: int = 0
    sampling_seed: Optional[int] = None
    last_active_time: float = field(default_factory=time.monotonic)

    def reset(self) -> None:
        self.session_id = None
        self.segment_idx = -1
        self.prefill_source = ""
        self.past_len = 0
        self.position_offset = 0
        self.frame_idx = 0
        self.next_embed = None
        self.last_codec_sum = None
        self.trailing = []
        self.text_idx = 0
        self.token_queue = []
        self.pad_start_frame = -1
        self.pad_consecutive_silence = 0
        self.sampling_seed = None
        self.last_active_time = time.monotonic()

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
        self._preallocate = True
        self._talker_kv_pool = None  # paged: there is no slot-contiguous tensor

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


@dataclass(frozen=True)
class PagedPrefixEntry:
    """A cached prefix: the block ids holding it (one reference each) + length."""

    key: str
    blocks: torch.Tensor
    prefix_len: int
    created_at: float
    hit_count: int = 0


class PagedPrefixKVCache:
    """LRU of prefix block lists (``PrefixKVCache`` API, prefix_cache.py:43-159).

    ``put`` takes a reference on the first ceil(prefix_len/16) blocks of a slot
    instead of cloning KV; ``restore(slot, entry)`` points an empty slot at the
    blocks instead of copying them; eviction / ``invalidate`` / ``clear`` drop
    the references so unused blocks return to the free stack.
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

    def put(self, key: Optional[str], slot_id: int, prefix_len: int) -> None:
        """Cache the first ``prefix_len`` positions of ``slot_id`` (which must hold them)."""
        if key is None or self._max_entries <= 0 or prefix_len > self._max_prefix_len:
            return
        if key in self._cache:
            self._cache.move_to_end(key)
            return
        while len(self._cache) >= self._max_entries:
            _, old = self._cache.popitem(last=False)
            self._pool._sched.drop_blocks(old.blocks)
        blocks = self._pool._sched.make_entry(slot_id, prefix_len)
        self._cache[key] = PagedPrefixEntry(key=key, blocks=blocks, prefix_len=prefix_len,
                                            created_at=time.monotonic())

    def restore(self, slot: SlotState, entry: PagedPrefixEntry) -> None:
        """engine_loop._restore_prefix_cache without the copy."""
        self._pool._sched.share_prefix(slot.slot_id, entry.blocks, entry.prefix_len)
        st = int(self._pool._sched.status.item())
        if st != 0:
            raise ValueError(f"prefix restore into slot {slot.slot_id} failed (status {st})")
        slot.past_len = entry.prefix_len
        slot.position_offset = 0

    def invalidate(self, key: str) -> bool:
        e = self._cache.pop(key, None)
        if e is None:
            return False
        self._pool._sched.drop_blocks(e.blocks)
        return True

    def clear(self) -> None:
        for e in self._cache.values():
            self._pool._sched.drop_blocks(e.blocks)
        self._cache.clear()
