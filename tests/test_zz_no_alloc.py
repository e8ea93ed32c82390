"""qtts_paged_attention_noalloc: paged attention for callers that cannot
allocate device memory when they run it (a plugin host that owns every
allocation, or a latency-bound thread that must not call cudaMalloc).  It keeps
its split-KV partials in a static device array of the library instead of
caller scratch.  This file is collected last so that a stopping run has
already run every other test; it also passes on its own in a fresh process.
"""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

from test_stateful_b200 import _lib  # noqa: E402

DEV = "cuda"
HKV, HQ, L, NB, MBPS, BS = 8, 16, 4, 600, 128, 16


def _case(seed, ctxs, d):
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn(NB, L, 2, HKV, BS, d, generator=g).to(torch.float16).to(DEV)
    table = torch.stack([torch.randperm(NB, generator=g)[:MBPS] for _ in ctxs]).to(torch.int32).to(DEV)
    q = torch.randn(len(ctxs), HQ, d, generator=g).to(DEV)
    ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    rows = torch.arange(len(ctxs), dtype=torch.int32, device=DEV)
    return kv, table, q, ctx, rows


def _with_caller_scratch(kv, table, q, ctx, rows, layer, max_ctx):
    R, _, d = q.shape
    n_blocks = -(-max_ctx // BS)
    splits = max(1, -(-n_blocks // _lib.ATTN_SPLIT_BLOCKS))
    ws_o = torch.empty(R * HQ * splits * d, device=DEV)
    ws_ml = torch.empty(R * HQ * splits * 2, device=DEV)
    out = torch.empty(R, HQ * d, device=DEV, dtype=torch.bfloat16)
    out_lo = torch.empty_like(out)
    rc = _lib.load().qtts_paged_attention(q.data_ptr(), R, HQ, HKV, d, kv.data_ptr(), layer, L, BS, NB,
                                          table.data_ptr(), MBPS, rows.data_ptr(), ctx.data_ptr(), max_ctx, 0,
                                          ws_o.data_ptr(), ws_ml.data_ptr(), out.data_ptr(), out_lo.data_ptr(),
                                          _lib.stream_ptr())
    _lib.check(rc, "paged_attention")
    return out.float() + out_lo.float()


def _without_scratch(kv, table, q, ctx, rows, layer, max_ctx):
    R, _, d = q.shape
    out = torch.empty(R, HQ * d, device=DEV, dtype=torch.bfloat16)
    out_lo = torch.empty_like(out)
    rc = _lib.load().qtts_paged_attention_noalloc(q.data_ptr(), R, HQ, HKV, d, kv.data_ptr(), layer, L, BS, NB,
                                                  table.data_ptr(), MBPS, rows.data_ptr(), ctx.data_ptr(), max_ctx,
                                                  out.data_ptr(), out_lo.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "paged_attention_noalloc")
    return out.float() + out_lo.float()


def test_noalloc_matches_caller_scratch_on_two_calls_in_a_row():
    # two consecutive calls with different shapes: the second reuses the static
    # array the first one wrote, and must not see any of its contents
    cases = [(1, [1, 16, 17, 300, 1024, 2048], 128, 3, 2048),
             (2, [5, 255, 256, 257, 999], 64, 1, 1024)]
    for seed, ctxs, d, layer, max_ctx in cases:
        kv, table, q, ctx, rows = _case(seed, ctxs, d)
        want = _with_caller_scratch(kv, table, q, ctx, rows, layer, max_ctx)
        got = _without_scratch(kv, table, q, ctx, rows, layer, max_ctx)
        torch.cuda.synchronize()
        torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-4)
    assert _lib.device_error() == 0


def test_noalloc_takes_every_head_dim_up_to_the_limit():
    # rows x heads x splits x head_dim exactly at the 1 Mi-float limit for head_dim 64 and 32:
    # the (max, sum) area scales with 1/head_dim, so the smallest head_dim needs the most of it
    for seed, d, n_rows in ((4, 64, 128), (5, 32, 256)):
        max_ctx = MBPS * BS                      # 2048 keys -> 8 splits of 16 blocks
        assert n_rows * HQ * 8 * d == 1 << 20
        g = torch.Generator().manual_seed(seed)
        ctxs = torch.randint(1, max_ctx + 1, (n_rows,), generator=g).tolist()
        kv, table, q, ctx, rows = _case(seed, ctxs, d)
        want = _with_caller_scratch(kv, table, q, ctx, rows, 2, max_ctx)
        got = _without_scratch(kv, table, q, ctx, rows, 2, max_ctx)
        torch.cuda.synchronize()
        torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-4)
    assert _lib.device_error() == 0


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    kv, table, q, ctx, rows = _case(3, [16] * 4, 128)
    big_rows = 600  # 600 rows x 16 heads x 1 split x 128 > 1 Mi partials
    qb = torch.zeros(big_rows, HQ, 128, device=DEV)
    rb = torch.zeros(big_rows, dtype=torch.int32, device=DEV)
    cb = torch.full((big_rows,), 16, dtype=torch.int32, device=DEV)
    out = torch.empty(big_rows, HQ * 128, device=DEV, dtype=torch.bfloat16)
    rc = _lib.load().qtts_paged_attention_noalloc(qb.data_ptr(), big_rows, HQ, HKV, 128, kv.data_ptr(), 0, L, BS,
                                                  NB, table.data_ptr(), MBPS, rb.data_ptr(), cb.data_ptr(), 16,
                                                  out.data_ptr(), None, _lib.stream_ptr())
    assert rc == _lib.ERR_INVALID
    assert "static scratch" in _lib.last_error()
