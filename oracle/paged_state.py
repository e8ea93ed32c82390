"""Paged KV pool state: block allocator, block tables, slot mapping, prefix refcount/COW.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference pool is slot-contiguous (engine/backend/kv_cache_pool.py:235-246)
and its prefix cache clones and copies KV (engine/backend/prefix_cache.py:138-144,
engine/backend/engine_loop.py:823-835).  The B200 pool stores the same logical
KV in 16-token blocks.  This module is the sequential statement of that
allocator; the device kernels must reproduce its block tables, slot mappings,
refcounts and free stack bit for bit, and the logical KV read back through its
block tables must equal what the reference ``KVCachePool.gather_talker_kv``
returns after the same operations (tests/golden/pool_ops.npz).

Semantics (shared with the CUDA kernels):

* The free list is a LIFO stack, initialised so the first pop returns block 0
  (the reference's slot free list is also LIFO, kv_cache_pool.py:221, 273).
* ``append(slots, n_new)`` walks the streams in batch order and, for each new
  token position ``t``, uses ``table[slot][t // bs]``; an unassigned entry pops
  a fresh block (refcount 1); a block still shared (refcount > 1) at the first
  write pops a fresh block, records a copy ``(src, dst)`` and drops one
  reference to ``src``.  It is all-or-nothing: if any stream would pass the
  per-sequence capacity or the stack runs dry, nothing changes and an error is
  returned.
* ``share_prefix`` points an empty slot at a cached entry's blocks (refcount+1
  each); ``make_entry`` takes a reference on a slot's first blocks; ``release``
  and ``drop_entry`` drop references in table order and push blocks that reach
  zero.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np

OK = 0
ERR_CAPACITY = -3
ERR_POOL_EXHAUSTED = -4
ERR_BAD_ARG = -1


class PagedState:
    def __init__(self, num_blocks: int, block_size: int, max_slots: int, max_blocks_per_seq: int):
        self.num_blocks = num_blocks
        self.bs = block_size
        self.max_slots = max_slots
        self.mbps = max_blocks_per_seq
        self.free: List[int] = list(range(num_blocks - 1, -1, -1))
        self.refcount = np.zeros(num_blocks, dtype=np.int32)
        self.table = np.full((max_slots, max_blocks_per_seq), -1, dtype=np.int32)
        self.seq_len = np.zeros(max_slots, dtype=np.int32)

    # -- helpers -------------------------------------------------------------
    @property
    def free_top(self) -> int:
        return len(self.free)

    def free_stack_array(self) -> np.ndarray:
        """Stack contents bottom→top, as the device array holds them in [0, top)."""
        return np.asarray(self.free, dtype=np.int32)

    def _decref(self, b: int) -> None:
        self.refcount[b] -= 1
        assert self.refcount[b] >= 0
        if self.refcount[b] == 0:
            self.free.append(int(b))

    # -- operations ----------------------------------------------------------
    def append(self, slots: Sequence[int], n_new: int) -> Tuple[int, np.ndarray, List[Tuple[int, int]]]:
        """Reserve KV positions for ``n_new`` tokens per stream.

        Returns ``(status, slot_mapping [B * n_new], cow_pairs)``.  Runs on a
        copy of the state and commits only when every stream succeeded.
        """
        slots = [int(s) for s in slots]
        cap = self.mbps * self.bs
        fail = np.full(len(slots) * n_new, -1, np.int64)
        for s in slots:
            if int(self.seq_len[s]) + n_new > cap:
                return ERR_CAPACITY, fail, []
        free = list(self.free)
        refcount = self.refcount.copy()
        table = self.table.copy()
        seq_len = self.seq_len.copy()
        mapping = np.empty(len(slots) * n_new, dtype=np.int64)
        cow: List[Tuple[int, int]] = []
        for i, s in enumerate(slots):
            pos = int(seq_len[s])
            for j in range(n_new):
                t = pos + j
                bi = t // self.bs
                blk = int(table[s, bi])
                if blk < 0 or (j == 0 and refcount[blk] > 1):
                    if not free:
                        return ERR_POOL_EXHAUSTED, fail, []
                    new = free.pop()
                    refcount[new] = 1
                    if blk >= 0:
                        cow.append((blk, new))
                        refcount[blk] -= 1  # stays >= 1, nothing is pushed
                    table[s, bi] = new
                    blk = new
                mapping[i * n_new + j] = blk * self.bs + t % self.bs
            seq_len[s] = pos + n_new
        self.free, self.refcount, self.table, self.seq_len = free, refcount, table, seq_len
        return OK, mapping, cow

    def share_prefix(self, slot: int, blocks: Sequence[int], prefix_len: int) -> int:
        if self.seq_len[slot] != 0 or (self.table[slot] >= 0).any():
            return ERR_BAD_ARG
        nb = (prefix_len + self.bs - 1) // self.bs
        if nb > len(blocks) or nb > self.mbps:
            return ERR_BAD_ARG
        for i in range(nb):
            b = int(blocks[i])
            self.table[slot, i] = b
            self.refcount[b] += 1
        self.seq_len[slot] = prefix_len
        return OK

    def make_entry(self, slot: int, prefix_len: int) -> List[int]:
        nb = (prefix_len + self.bs - 1) // self.bs
        blocks = [int(b) for b in self.table[slot, :nb]]
        for b in blocks:
            self.refcount[b] += 1
        return blocks

    def drop_entry(self, blocks: Sequence[int]) -> None:
        for b in blocks:
            self._decref(int(b))

    def release(self, slot: int) -> None:
        for bi in range(self.mbps):
            b = int(self.table[slot, bi])
            if b >= 0:
                self._decref(b)
                self.table[slot, bi] = -1
        self.seq_len[slot] = 0


class PagedKV:
    """Block storage ``[num_blocks, L2, Hkv, bs, D]`` driven by a ``PagedState``."""

    def __init__(self, state: PagedState, l2: int, hkv: int, d: int, dtype=np.float32):
        self.st = state
        self.data = np.zeros((state.num_blocks, l2, hkv, state.bs, d), dtype=dtype)

    def write(self, mapping: np.ndarray, kv: np.ndarray) -> None:
        """``kv [n, L2, Hkv, D]`` for ``n`` mapped positions (``-1`` skipped)."""
        bs = self.st.bs
        for i, m in enumerate(mapping):
            if m < 0:
                continue
            self.data[m // bs, :, :, m % bs, :] = kv[i]

    def copy_blocks(self, cow: Sequence[Tuple[int, int]]) -> None:
        for src, dst in cow:
            self.data[dst] = self.data[src]

    def gather(self, slot: int, n: int) -> np.ndarray:
        """Logical KV ``[L2, Hkv, n, D]`` of a slot's first ``n`` positions."""
        bs = self.st.bs
        out = np.zeros((self.data.shape[1], self.data.shape[2], n, self.data.shape[4]), self.data.dtype)
        for t in range(n):
            b = int(self.st.table[slot, t // bs])
            out[:, :, t, :] = self.data[b, :, :, t % bs, :]
        return out
