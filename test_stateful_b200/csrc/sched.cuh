// On-device ragged scheduler step over the paged KV pool.
//
// The reference keeps each session's KV slot-contiguous and, every step,
// gathers the whole past into a padded batch and scatters the delta back
// (engine/backend/kv_cache_pool.py:410-420, 480-498); a prefix-cache hit
// copies the cached KV into the slot (engine/backend/engine_loop.py:823-835).
// Here KV lives in fixed-size blocks; a step only reserves positions:
//
//   append:  for each stream (batch order) and each new token, use the block
//            table entry; an unassigned entry pops a block from the LIFO free
//            stack; a block still shared at the first write (refcount > 1,
//            i.e. a prefix block another slot or the prefix cache holds) is
//            copied to a fresh block (copy-on-write) and one reference dropped.
//
// Sequential semantics, parallel execution: thread i handles stream i.  The
// number of pops each stream needs is known up front except for shared
// blocks, where stream i copies iff refcount - k_i > 1, k_i being the number
// of earlier streams in the batch whose first write lands in the same block
// (each earlier copier dropped one reference).  An exclusive scan of the pop
// counts gives every stream its slice of the stack top, so the assignment is
// identical to popping one stream at a time (oracle/paged_state.py).
#pragma once

#include "common.cuh"

namespace qtts {

struct SchedView {
    int32_t* free_stack;
    int32_t* free_top;
    int32_t* refcount;
    int32_t* table;
    int32_t* seq_len;
    int32_t* pos_off;
    int num_blocks, bs, max_slots, mbps;
};

inline SchedView view_of(const qtts_paged_state* s) {
    return SchedView{s->free_stack, s->free_top, s->refcount, s->block_table, s->seq_len, s->position_offset,
                     s->num_blocks, s->block_size, s->max_slots, s->max_blocks_per_seq};
}

__global__ void sched_init_kernel(SchedView v) {
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nth = gridDim.x * blockDim.x;
    for (int i = tid; i < v.num_blocks; i += nth) {
        v.free_stack[i] = v.num_blocks - 1 - i;
        v.refcount[i] = 0;
    }
    for (int i = tid; i < v.max_slots * v.mbps; i += nth) v.table[i] = -1;
    for (int i = tid; i < v.max_slots; i += nth) {
        v.seq_len[i] = 0;
        v.pos_off[i] = 0;
    }
    if (tid == 0) *v.free_top = v.num_blocks;
}

constexpr int kSchedThreads = 1024;

__global__ void __launch_bounds__(kSchedThreads) sched_append_kernel(SchedView v, const int32_t* __restrict__ slots,
                                                                     int n_rows, int n_new,
                                                                     int32_t* __restrict__ mapping,
                                                                     int32_t* __restrict__ row_ctx,
                                                                     int32_t* __restrict__ row_pos,
                                                                     int32_t* __restrict__ cow_src,
                                                                     int32_t* __restrict__ cow_dst,
                                                                     int32_t* __restrict__ status) {
    __shared__ int s_blk0[kSchedThreads];
    __shared__ int s_scan[kSchedThreads];
    __shared__ int s_err;
    const int i = threadIdx.x;
    griddep_wait();
    griddep_launch();
    const bool active = i < n_rows;
    int slot = 0, pos = 0, bi0 = 0, blk0 = -1, need = 0;
    bool cow = false, bad = false;
    if (i == 0) s_err = QTTS_OK;
    if (active) {
        slot = slots[i];
        if (slot < 0 || slot >= v.max_slots) {
            bad = true;
        } else {
            pos = v.seq_len[slot];
            if (pos + n_new > v.mbps * v.bs) bad = true;
            bi0 = pos / v.bs;
            if (!bad) blk0 = v.table[slot * v.mbps + bi0];
        }
    }
    s_blk0[i] = (active && !bad) ? blk0 : -1;
    __syncthreads();
    if (active && bad) atomicCAS(&s_err, QTTS_OK, QTTS_ERR_CAPACITY);
    if (active && !bad) {
        if (blk0 < 0) {
            need = 1;
        } else {
            int k = 0;
            for (int j = 0; j < i; ++j) k += (s_blk0[j] == blk0);
            cow = v.refcount[blk0] - k > 1;
            need = cow ? 1 : 0;
        }
        const int first_boundary = (bi0 + 1) * v.bs;
        if (pos + n_new > first_boundary) need += (pos + n_new - 1 - first_boundary) / v.bs + 1;
    }
    // inclusive scan of need (Hillis-Steele over the block)
    s_scan[i] = need;
    __syncthreads();
    for (int off = 1; off < kSchedThreads; off <<= 1) {
        const int add = i >= off ? s_scan[i - off] : 0;
        __syncthreads();
        s_scan[i] += add;
        __syncthreads();
    }
    const int total = s_scan[kSchedThreads - 1];
    const int excl = s_scan[i] - need;
    const int top = *v.free_top;
    if (i == 0 && s_err == QTTS_OK && total > top) s_err = QTTS_ERR_POOL_EXHAUSTED;
    __syncthreads();
    const int err = s_err;
    if (err != QTTS_OK) {
        for (int e = i; e < n_rows * n_new; e += kSchedThreads) {
            mapping[e] = -1;
            row_ctx[e] = 0;
            row_pos[e] = 0;
        }
        if (active) {
            cow_src[i] = -1;
            cow_dst[i] = -1;
        }
        if (i == 0) *status = err;
        return;
    }
    if (active) {
        int base = top - 1 - excl;  // this stream's pops: free_stack[base], [base-1], ...
        cow_src[i] = -1;
        cow_dst[i] = -1;
        int32_t* row = v.table + slot * v.mbps;
        if (blk0 < 0) {
            const int b = v.free_stack[base--];
            v.refcount[b] = 1;
            row[bi0] = b;
        } else if (cow) {
            const int b = v.free_stack[base--];
            v.refcount[b] = 1;
            row[bi0] = b;
            cow_src[i] = blk0;
            cow_dst[i] = b;
            atomicSub(&v.refcount[blk0], 1);
        }
        for (int bi = bi0 + 1; bi * v.bs < pos + n_new; ++bi) {
            const int b = v.free_stack[base--];
            v.refcount[b] = 1;
            row[bi] = b;
        }
    }
    __syncthreads();  // table rows written, every pop read
    for (int e = i; e < n_rows * n_new; e += kSchedThreads) {
        const int r = e / n_new, j = e % n_new;
        const int s = slots[r];
        const int t = v.seq_len[s] + j;
        mapping[e] = v.table[s * v.mbps + t / v.bs] * v.bs + t % v.bs;
        row_ctx[e] = t + 1;
        row_pos[e] = v.pos_off[s] + t;
    }
    __syncthreads();  // seq_len read above before it is advanced
    if (active) v.seq_len[slot] = pos + n_new;
    if (i == 0) {
        *v.free_top = top - total;
        *status = QTTS_OK;
    }
}

__global__ void sched_share_prefix_kernel(SchedView v, int slot, const int32_t* blocks, int prefix_len,
                                          int32_t* status) {
    const int nb = (prefix_len + v.bs - 1) / v.bs;
    int err = QTTS_OK;
    if (slot < 0 || slot >= v.max_slots || nb > v.mbps || prefix_len < 0 || v.seq_len[slot] != 0) err = QTTS_ERR_INVALID;
    for (int i = 0; err == QTTS_OK && i < v.mbps; ++i)
        if (v.table[slot * v.mbps + i] >= 0) err = QTTS_ERR_INVALID;
    for (int i = 0; err == QTTS_OK && i < nb; ++i)
        if (blocks[i] < 0 || blocks[i] >= v.num_blocks || v.refcount[blocks[i]] <= 0) err = QTTS_ERR_INVALID;
    if (err == QTTS_OK) {
        for (int i = 0; i < nb; ++i) {
            v.table[slot * v.mbps + i] = blocks[i];
            v.refcount[blocks[i]] += 1;
        }
        v.seq_len[slot] = prefix_len;
    }
    if (status) *status = err;
}

__global__ void sched_make_entry_kernel(SchedView v, int slot, int prefix_len, int32_t* blocks_out) {
    const int nb = (prefix_len + v.bs - 1) / v.bs;
    for (int i = 0; i < nb; ++i) {
        const int b = v.table[slot * v.mbps + i];
        blocks_out[i] = b;
        if (b >= 0) v.refcount[b] += 1;
    }
}

__device__ __forceinline__ void sched_decref(SchedView& v, int b) {
    if (b < 0 || b >= v.num_blocks) return;
    if (--v.refcount[b] == 0) v.free_stack[(*v.free_top)++] = b;
}

__global__ void sched_drop_blocks_kernel(SchedView v, const int32_t* blocks, int n) {
    for (int i = 0; i < n; ++i) sched_decref(v, blocks[i]);
}

__global__ void sched_release_kernel(SchedView v, int slot) {
    for (int i = 0; i < v.mbps; ++i) {
        const int b = v.table[slot * v.mbps + i];
        if (b >= 0) {
            sched_decref(v, b);
            v.table[slot * v.mbps + i] = -1;
        }
    }
    v.seq_len[slot] = 0;
    v.pos_off[slot] = 0;
}

}  // namespace qtts
