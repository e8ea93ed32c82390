"""Pin the paged-pool oracle against the reference slot-contiguous pool.

``tests/golden/pool_ops.npz`` records an op sequence run on the reference
``KVCachePool`` (engine/backend/kv_cache_pool.py:269-341, 383-395, 480-498)
and ``PrefixKVCache`` (engine/backend/prefix_cache.py:81-148) with the prefix
restore of engine/backend/engine_loop.py:823-835.  Replaying it on the paged
state must give the same logical KV for every live slot.
"""

import os

import numpy as np
import pytest

from oracle.paged_state import PagedState, PagedKV, OK, ERR_CAPACITY, ERR_POOL_EXHAUSTED

from .conftest import GOLDEN


def replay(z, block_size=4, num_blocks=64):
    L, H, D, S = (int(z[k]) for k in ("L", "H", "D", "S"))
    st = PagedState(num_blocks, block_size, 4, S // block_size)
    kv = PagedKV(st, 2 * L, H, D)
    toks = z["kv_tokens"].reshape(-1, 2 * L, H, D)
    cur = 0
    entry = None
    snaps = {}
    n_decode = 0
    for row in z["ops"]:
        op = int(row[0])
        if op == 0:
            continue
        if op == 1:
            slot, n = int(row[1]), int(row[2])
            status, m, cow = st.append([slot], n)
            assert status == OK
            kv.copy_blocks(cow)
            kv.write(m, toks[cur:cur + n]); cur += n
        elif op == 2:
            entry = st.make_entry(int(row[1]), int(row[2]))
        elif op == 3:
            assert st.share_prefix(int(row[1]), entry, int(row[2])) == OK
        elif op == 4:
            nb = int(row[1])
            slots = [int(s) for s in row[2:2 + nb]]
            status, m, cow = st.append(slots, 1)
            assert status == OK
            kv.copy_blocks(cow)
            kv.write(m, toks[cur:cur + nb]); cur += nb
            n_decode += 1
            if n_decode == 15:
                snaps = {s: kv.gather(s, int(st.seq_len[s])) for s in range(4) if st.seq_len[s] > 0}
        elif op == 5:
            st.release(int(row[1]))
    assert cur == toks.shape[0]
    return st, kv, snaps


@pytest.mark.parametrize("block_size", [4, 16])
def test_replay_matches_reference_pool(block_size):
    z = np.load(os.path.join(GOLDEN, "pool_ops.npz"))
    st, kv, snaps = replay(z, block_size=block_size)
    keys1 = [k for k in z.files if k.startswith("snap1_slot")]
    for k in keys1:
        slot = int(k[len("snap1_slot"):])
        n = int(z[f"snap1_len{slot}"])
        np.testing.assert_array_equal(snaps[slot][:, :, :n], z[k])
    for k in [k for k in z.files if k.startswith("final_slot")]:
        slot = int(k[len("final_slot"):])
        n = int(z[f"final_len{slot}"])
        assert int(st.seq_len[slot]) == n
        np.testing.assert_array_equal(kv.gather(slot, n), z[k])


def test_refcounts_and_free_stack_consistent():
    z = np.load(os.path.join(GOLDEN, "pool_ops.npz"))
    st, kv, _ = replay(z, block_size=4)
    # every block is either free or referenced; the free stack has no duplicates
    free = st.free_stack_array()
    assert len(set(free.tolist())) == len(free)
    assert all(st.refcount[b] == 0 for b in free)
    used = [b for b in range(st.num_blocks) if st.refcount[b] > 0]
    assert len(used) + len(free) == st.num_blocks


def test_shared_partial_block_cow_and_last_sharer_writes_in_place():
    st = PagedState(32, 4, 4, 8)
    assert st.append([0], 6)[0] == OK          # blocks 0,1 ; block 1 holds 2 tokens
    e = st.make_entry(0, 6)                      # entry refs blocks 0,1
    assert st.share_prefix(1, e, 6) == OK
    assert st.share_prefix(2, e, 6) == OK
    st.drop_entry(e)                             # block 1 now shared by slots 0,1,2 (refcount 3)
    status, m, cow = st.append([1, 2, 0], 1)
    assert status == OK
    # slot 1 and 2 copy, slot 0 (last sharer, refcount back to 1) writes in place
    assert [c[0] for c in cow] == [1, 1]
    assert m[2] == 1 * 4 + 2
    assert st.refcount[1] == 1


def test_all_or_nothing_errors():
    st = PagedState(3, 4, 2, 2)
    assert st.append([0], 9)[0] == ERR_CAPACITY
    assert st.append([0], 8)[0] == OK
    before = (list(st.free), st.refcount.copy(), st.table.copy(), st.seq_len.copy())
    status, m, cow = st.append([1], 5)   # needs 2 blocks, 1 left
    assert status == ERR_POOL_EXHAUSTED and (m == -1).all()
    assert st.free == before[0] and (st.table == before[2]).all() and (st.seq_len == before[3]).all()
