"""Kernel parity on the B200: each entry point of libqtts_b200.so against the
CPU oracle (integer/index work: bit-exact) or an fp32 torch statement of the
same op (floating point: tolerance in each test)."""

import ctypes as C
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import model as M  # noqa: E402
from oracle.paged_state import PagedState, OK  # noqa: E402
from test_stateful_b200 import _lib, ops  # noqa: E402
from test_stateful_b200.config import EngineConfig, PagedPoolConfig, TalkerConfig  # noqa: E402
from test_stateful_b200.runtime.model import PagedPoolTensors, rope_tables  # noqa: E402

DEV = "cuda"


def _gen(seed):
    return torch.Generator(device="cpu").manual_seed(seed)


def _rand(shape, seed, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(shape, generator=_gen(seed)) * scale).to(dtype).to(DEV)


# --------------------------------------------------------------------- GEMM
GEMM_SHAPES = [(64, 4096, 2048), (64, 2048, 6144), (37, 1024, 2048), (128, 2048, 1024), (200, 512, 256),
               (1, 3072, 2048), (17, 128, 64)]


@pytest.mark.parametrize("M_,N,K", GEMM_SHAPES)
def test_gemm_f32_matches_fp32_matmul(M_, N, K):
    x = _rand((M_, K), 1)
    w = _rand((N, K), 2, 0.05)
    y = ops.gemm(x, w, _lib.EPI_F32)
    ref = x.float() @ w.float().T
    torch.testing.assert_close(y, ref, rtol=1e-3, atol=1e-3)  # fp32 accumulation of exact bf16 products


@pytest.mark.parametrize("M_,N,K", [(64, 2048, 2048), (37, 1024, 6144), (200, 512, 1024)])
def test_gemm_hilo_operand_recovers_fp32_activation(M_, N, K):
    """W·hi + W·lo in one pass: the error against an fp32 activation is far below bf16 rounding."""
    x = torch.randn(M_, K, generator=_gen(21)).to(DEV)
    w = _rand((N, K), 22, 0.05)
    hi, lo = ops.split_hilo(x)
    y = ops.gemm(hi, w, _lib.EPI_F32, x_lo=lo)
    ref = x.double() @ w.double().T
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    plain = ops.gemm(hi, w, _lib.EPI_F32)
    err_plain = float((plain.double() - ref).abs().max() / ref.abs().max())
    assert err < 5e-5, err
    assert err < err_plain / 20, (err, err_plain)


def test_gemm_swiglu_hilo_output():
    from test_stateful_b200.runtime.model import _interleave_gate_up
    H, I = 2048, 6144
    x = torch.randn(64, H, generator=_gen(23)).to(DEV)
    hi, lo = ops.split_hilo(x)
    g = _rand((I, H), 24, 0.05)
    u = _rand((I, H), 25, 0.05)
    w = _interleave_gate_up(g, u)
    out_lo = torch.empty(64, I, device=DEV, dtype=torch.bfloat16)
    y = ops.gemm(hi, w, _lib.EPI_SWIGLU, x_lo=lo, out_lo=out_lo)
    ref = torch.nn.functional.silu(x.double() @ g.double().T) * (x.double() @ u.double().T)
    got = y.double() + out_lo.double()
    assert float((got - ref).abs().max() / ref.abs().max()) < 1e-4


def test_gemm_bf16_bias_and_residual():
    x = _rand((64, 1024), 3)
    w = _rand((2048, 1024), 4, 0.05)
    b = _rand((2048,), 5, 0.1)
    y = ops.gemm(x, w, _lib.EPI_BF16, bias=b)
    ref = x.float() @ w.float().T + b.float()
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=1e-2)  # bf16 output rounding
    r0 = torch.randn(64, 2048, generator=_gen(6)).to(DEV)
    r = r0.clone()
    ops.gemm(x, w, _lib.EPI_RESIDUAL, out=r)
    torch.testing.assert_close(r, r0 + x.float() @ w.float().T, rtol=1e-3, atol=1e-3)


def test_gemm_swiglu_interleaved():
    from test_stateful_b200.runtime.model import _interleave_gate_up
    H, I = 1024, 3072
    x = _rand((64, H), 7)
    g = _rand((I, H), 8, 0.05)
    u = _rand((I, H), 9, 0.05)
    w = _interleave_gate_up(g, u)
    y = ops.gemm(x, w, _lib.EPI_SWIGLU)
    gf, uf = x.float() @ g.float().T, x.float() @ u.float().T
    ref = torch.nn.functional.silu(gf) * uf
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-3)


@pytest.mark.parametrize("D,Hq,Hkv,H", [(128, 16, 8, 2048), (64, 16, 8, 1024)])
def test_gemm_qkv_rope_epilogue(D, Hq, Hkv, H):
    Mr = 64
    L, layer, nb = 3, 1, 32
    x = _rand((Mr, H), 10)
    w = _rand(((Hq + 2 * Hkv) * D, H), 11, 0.05)
    qn = (1 + 0.1 * torch.randn(D, generator=_gen(12))).to(torch.bfloat16).to(DEV)
    kn = (1 + 0.1 * torch.randn(D, generator=_gen(13))).to(torch.bfloat16).to(DEV)
    cos, sin = rope_tables(D, 1e6, 1024, DEV)
    pos = torch.randint(0, 1000, (Mr,), generator=_gen(14)).to(torch.int32).to(DEV)
    perm = torch.randperm(nb * 16, generator=_gen(15))[:Mr].to(torch.int32)
    mapping = perm.clone()
    mapping[5] = -1
    mapping = mapping.to(DEV)
    pool = torch.zeros(nb, L, 2, Hkv, 16, D, device=DEV, dtype=torch.float16)
    q_out = torch.empty(Mr, Hq * D, device=DEV, dtype=torch.float32)
    e = _lib.QkvEpilogue(Hq, Hkv, D, qn.data_ptr(), kn.data_ptr(), 1e-6, cos.data_ptr(), sin.data_ptr(), 1024,
                         pos.data_ptr(), mapping.data_ptr(), pool.data_ptr(), layer, L, 16)
    ops.gemm(x, w, _lib.EPI_QKV_ROPE, out=q_out, qkv=e)
    torch.cuda.synchronize()
    y = (x.float() @ w.float().T).cpu()
    q = y[:, :Hq * D].view(Mr, Hq, D)
    k = y[:, Hq * D:(Hq + Hkv) * D].view(Mr, Hkv, D)
    v = y[:, (Hq + Hkv) * D:].view(Mr, Hkv, D)
    q = M.rms_norm(q, qn.float().cpu(), 1e-6)
    k = M.rms_norm(k, kn.float().cpu(), 1e-6)
    c, s = M.rope_cos_sin(pos.long().cpu().unsqueeze(1), D, 1e6)   # [M,1,D]
    q = q * c + M.rotate_half(q) * s
    k = k * c + M.rotate_half(k) * s
    torch.testing.assert_close(q_out.cpu().view(Mr, Hq, D), q, rtol=1e-3, atol=1e-3)  # q stays fp32
    pc = pool.float().cpu()
    for m in range(Mr):
        sm = int(mapping[m])
        if sm < 0:
            continue
        blk, off = sm // 16, sm % 16
        torch.testing.assert_close(pc[blk, layer, 0, :, off], k[m], rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(pc[blk, layer, 1, :, off], v[m], rtol=2e-2, atol=2e-2)
    # row 5 had no slot: its position must be untouched (zeros) everywhere
    assert int((pool[:, layer].float().abs().sum(dim=(1, 2, 4)) > 0).sum()) == Mr - 1


# --------------------------------------------------------------------- attention
@pytest.mark.parametrize("D", [128, 64])
def test_paged_attention_ragged(D):
    Hkv, Hq, L, layer, nb, mbps = 8, 16, 2, 1, 300, 80
    ctxs = [1, 15, 16, 17, 100, 255, 256, 257, 700, 1024, 1280]
    R = len(ctxs)
    g = _gen(20)
    kv = (torch.randn(nb, L, 2, Hkv, 16, D, generator=g)).to(torch.float16).to(DEV)
    table = torch.full((R, mbps), -1, dtype=torch.int32)
    perm = torch.randperm(nb, generator=g)
    i = 0
    for r, c in enumerate(ctxs):
        n = -(-c // 16)
        table[r, :n] = perm[i:i + n] if i + n <= nb else torch.randint(0, nb, (n,), generator=g)
        i = (i + n) % (nb - 100)
    q = torch.randn(R, Hq, D, generator=g).to(DEV)
    row_slot = torch.arange(R, dtype=torch.int32, device=DEV)
    row_ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    out_lo = torch.empty(R, Hq * D, device=DEV, dtype=torch.bfloat16)
    out = ops.paged_attention(q, kv, layer, table.to(DEV), row_slot, row_ctx, max_ctx=mbps * 16, out_lo=out_lo)
    out = out.float() + out_lo.float()
    kvc, qc = kv.float().cpu(), q.float().cpu()
    for r, c in enumerate(ctxs):
        blocks = table[r, : -(-c // 16)].long()
        K = kvc[blocks, layer, 0].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c]
        V = kvc[blocks, layer, 1].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c]
        K = K.repeat_interleave(2, 0)
        V = V.repeat_interleave(2, 0)
        p = torch.softmax((qc[r].unsqueeze(1) @ K.transpose(1, 2)).squeeze(1) / D ** 0.5, dim=-1)
        ref = (p.unsqueeze(1) @ V).squeeze(1).reshape(-1)
        torch.testing.assert_close(out[r].cpu(), ref, rtol=1e-3, atol=1e-4)  # fp32 softmax/PV, hi+lo output


@pytest.mark.parametrize("split", [0, 2])
def test_paged_prefill_attention_query_tiles(split):
    """Chunked prefill (qtts_paged_attention_prefill): streams of S query rows with causal key
    counts past + t + 1 (talker_unified_modules.py:282-294), S not a multiple of the 8-token
    tile, pasts that start mid-block, several splits per row (split = 2 blocks) or one
    (default 16), against an fp32 torch statement of the same attention and against the
    one-row-per-query decode kernel."""
    D, Hkv, Hq, L, layer, nb, mbps = 128, 8, 16, 2, 1, 400, 40
    S = 21
    pasts = [0, 37, 300, 5]
    n = len(pasts)
    g = _gen(33)
    kv = (torch.randn(nb, L, 2, Hkv, 16, D, generator=g)).to(torch.float16).to(DEV)
    table = torch.full((n, mbps), -1, dtype=torch.int32)
    perm = torch.randperm(nb, generator=g)
    for b, pl in enumerate(pasts):
        k = -(-(pl + S) // 16)
        table[b, :k] = perm[b * mbps: b * mbps + k]
    R = n * S
    q = torch.randn(R, Hq, D, generator=g).to(DEV)
    row_slot = torch.tensor([b for b in range(n) for _ in range(S)], dtype=torch.int32, device=DEV)
    ctxs = [pl + t + 1 for pl in pasts for t in range(S)]
    row_ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    max_ctx = mbps * 16
    sb = split or _lib.ATTN_SPLIT_BLOCKS
    splits = max(1, -(-(-(-max_ctx // 16)) // sb))
    ws_o = torch.empty(R * Hq * splits * D, device=DEV)
    ws_ml = torch.empty(R * Hq * splits * 2, device=DEV)
    out = torch.empty(R, Hq * D, device=DEV, dtype=torch.bfloat16)
    out_lo = torch.empty_like(out)
    tdev = table.to(DEV)
    rc = _lib.load().qtts_paged_attention_prefill(q.data_ptr(), R, S, Hq, Hkv, D, kv.data_ptr(), layer, L, 16, nb,
                                                  tdev.data_ptr(), mbps, row_slot.data_ptr(), row_ctx.data_ptr(),
                                                  max_ctx, split, ws_o.data_ptr(), ws_ml.data_ptr(), out.data_ptr(),
                                                  out_lo.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "paged_attention_prefill")
    got = (out.float() + out_lo.float()).cpu()
    dec_lo = torch.empty_like(out)
    dec = ops.paged_attention(q, kv, layer, tdev, row_slot, row_ctx, max_ctx, out_lo=dec_lo, split_blocks=split)
    dec = (dec.float() + dec_lo.float()).cpu()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    kvc, qc = kv.float().cpu(), q.float().cpu()
    for r, c in enumerate(ctxs):
        b = r // S
        blocks = table[b, : -(-c // 16)].long()
        K = kvc[blocks, layer, 0].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c].repeat_interleave(2, 0)
        V = kvc[blocks, layer, 1].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c].repeat_interleave(2, 0)
        p = torch.softmax((qc[r].unsqueeze(1) @ K.transpose(1, 2)).squeeze(1) / D ** 0.5, dim=-1)
        ref = (p.unsqueeze(1) @ V).squeeze(1).reshape(-1)
        torch.testing.assert_close(got[r], ref, rtol=1e-3, atol=1e-4)
        torch.testing.assert_close(got[r], dec[r], rtol=1e-3, atol=1e-4)


@pytest.mark.skipif(os.environ.get("QTTS_PREFILL_UMMA") == "0", reason="query-tile form reads stale tails")
@pytest.mark.parametrize("pasts", [[0, 700, 33, 64], [700]], ids=["4streams", "1stream_splits"])
def test_paged_prefill_long_chunks_stale_tail(pasts):
    """Chunked prefill past one 64-query group (S = 150: groups of 64, 64 and 22 queries) with
    pasts that start mid-block and up to 850 keys, against an fp32 torch statement.  Every pool
    entry the streams do not own, and the tail of each stream's last block past its last key,
    holds NaN: keys past a row's count must contribute exactly nothing (the tcgen05 form zeroes
    V past the group's keys before P . V).  One stream gives 24 (group, kv head) CTAs, so the
    tcgen05 form splits each group's keys over several CTAs and folds them in a second kernel."""
    D, Hkv, Hq, L, layer, nb, mbps = 128, 8, 16, 2, 0, 400, 64
    S = 150
    n = len(pasts)
    g = _gen(35)
    kv = torch.full((nb, L, 2, Hkv, 16, D), float("nan"), dtype=torch.float16)
    table = torch.full((n, mbps), -1, dtype=torch.int32)
    perm = torch.randperm(nb, generator=g)
    for b, pl in enumerate(pasts):
        k = -(-(pl + S) // 16)
        table[b, :k] = perm[b * mbps: b * mbps + k]
        keys = torch.randn(2, Hkv, k * 16, D, generator=g).to(torch.float16)
        keys[:, :, pl + S:] = float("nan")
        kv[table[b, :k].long(), layer] = keys.reshape(2, Hkv, k, 16, D).permute(2, 0, 1, 3, 4)
    kv = kv.to(DEV)
    R = n * S
    q = torch.randn(R, Hq, D, generator=g).to(DEV)
    row_slot = torch.tensor([b for b in range(n) for _ in range(S)], dtype=torch.int32, device=DEV)
    ctxs = [pl + t + 1 for pl in pasts for t in range(S)]
    row_ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    max_ctx = mbps * 16
    splits = -(-(max_ctx // 16) // _lib.ATTN_SPLIT_BLOCKS)
    ws_o = torch.empty(R * Hq * splits * D, device=DEV)
    ws_ml = torch.empty(R * Hq * splits * 2, device=DEV)
    out = torch.empty(R, Hq * D, device=DEV, dtype=torch.bfloat16)
    out_lo = torch.empty_like(out)
    tdev = table.to(DEV)
    rc = _lib.load().qtts_paged_attention_prefill(q.data_ptr(), R, S, Hq, Hkv, D, kv.data_ptr(), layer, L, 16, nb,
                                                  tdev.data_ptr(), mbps, row_slot.data_ptr(), row_ctx.data_ptr(),
                                                  max_ctx, 0, ws_o.data_ptr(), ws_ml.data_ptr(), out.data_ptr(),
                                                  out_lo.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "paged_attention_prefill")
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    got = (out.float() + out_lo.float()).cpu()
    assert torch.isfinite(got).all()
    kvc, qc = kv.float().cpu(), q.float().cpu()
    for r, c in enumerate(ctxs):
        b = r // S
        blocks = table[b, : -(-c // 16)].long()
        K = kvc[blocks, layer, 0].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c].repeat_interleave(2, 0)
        V = kvc[blocks, layer, 1].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :c].repeat_interleave(2, 0)
        p = torch.softmax((qc[r].unsqueeze(1) @ K.transpose(1, 2)).squeeze(1) / D ** 0.5, dim=-1)
        ref = (p.unsqueeze(1) @ V).squeeze(1).reshape(-1)
        torch.testing.assert_close(got[r], ref, rtol=1e-3, atol=1e-4)


@pytest.mark.skipif(os.environ.get("QTTS_PREFILL_UMMA") is not None, reason="already a forced run")
def test_prefill_query_tile_form():
    """Chunked prefill with two query heads per KV head runs on the tcgen05 kernel by default;
    the mma.sync query-tile kernel stays available (QTTS_PREFILL_UMMA=0, read once per
    process): rerun the prefill tests in a child process with it."""
    import subprocess
    import sys

    env = dict(os.environ, QTTS_PREFILL_UMMA="0")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider", "-k",
                        "prefill and not tile_form and not without_splits and not umma_forms", os.path.abspath(__file__)], env=env,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.skipif(os.environ.get("QTTS_PREFILL_UMMA") is not None, reason="already a forced run")
@pytest.mark.parametrize("form", ["1", "2"])
def test_prefill_umma_forms(form):
    """The tcgen05 prefill has two forms — 64-key tiles with Q and P in shared memory (1) and
    128-key tiles with Q and P as TMEM operands (2) — picked by chunk length unless
    QTTS_PREFILL_UMMA forces one (read once per process): rerun the prefill kernel tests in a
    child process with each forced, so both see every case."""
    import subprocess
    import sys

    env = dict(os.environ, QTTS_PREFILL_UMMA=form)
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider", "-k",
                        "paged_prefill", os.path.abspath(__file__)], env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.skipif(os.environ.get("QTTS_PREFILL_UMMA") is not None or os.environ.get("QTTS_PREFILL_SPLITS")
                    is not None, reason="already a forced run")
def test_prefill_umma_without_splits():
    """The tcgen05 prefill splits a group's keys over several CTAs when the grid is small
    (QTTS_PREFILL_SPLITS caps the count, read once per process): rerun the prefill tests in a
    child process with splitting off, so both the split and the one-CTA forms are covered."""
    import subprocess
    import sys

    env = dict(os.environ, QTTS_PREFILL_SPLITS="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider", "-k",
                        "prefill and not tile_form and not without_splits and not umma_forms", os.path.abspath(__file__)], env=env,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


# --------------------------------------------------------------------- scheduler
def _pool(num_blocks=16, max_slots=6, mbps=8):
    cfg = EngineConfig(talker=TalkerConfig(num_layers=1, kv_heads=1, head_dim=8),
                       pool=PagedPoolConfig(block_size=16, num_blocks=num_blocks, max_slots=max_slots,
                                            max_seq_len=mbps * 16))
    return PagedPoolTensors(cfg, DEV)


def _assert_state_equal(pool, st: PagedState):
    torch.cuda.synchronize()
    top = int(pool.free_top.item())
    assert top == st.free_top
    assert np.array_equal(pool.free_stack[:top].cpu().numpy(), st.free_stack_array())
    assert np.array_equal(pool.refcount.cpu().numpy(), st.refcount)
    assert np.array_equal(pool.block_table.cpu().numpy(), st.table)
    assert np.array_equal(pool.seq_len.cpu().numpy(), st.seq_len)


def test_sched_matches_oracle_bit_exact():
    pool = _pool()
    pool.init()
    sch = ops.Sched(pool)
    st = PagedState(16, 16, 6, 8)
    rng = np.random.default_rng(0)

    def append(slots, n):
        s_dev = torch.tensor(slots, dtype=torch.int32, device=DEV)
        m, ctx, pos, cs, cd = sch.append(s_dev, n)
        status, m_ref, cow = st.append(slots, n)
        torch.cuda.synchronize()
        assert int(sch.status.item()) == status
        assert np.array_equal(m.cpu().numpy().astype(np.int64), m_ref)
        got = [(int(a), int(b)) for a, b in zip(cs.cpu(), cd.cpu()) if a >= 0]
        assert got == cow
        _assert_state_equal(pool, st)
        return status

    assert append([0], 37) == OK
    assert append([1], 5) == OK
    entry_dev = sch.make_entry(0, 21)
    entry = st.make_entry(0, 21)
    torch.cuda.synchronize()
    assert entry_dev.cpu().tolist() == entry
    _assert_state_equal(pool, st)
    for slot in (2, 3):
        sch.share_prefix(slot, entry_dev, 21)
        assert st.share_prefix(slot, entry, 21) == OK
        _assert_state_equal(pool, st)
    # shared partial block: slots 2, 3 copy; slot 0 is past it
    for _ in range(20):
        batch = list(rng.permutation([0, 1, 2, 3]))
        assert append(batch, 1) == OK
    sch.release(1)
    st.release(1)
    _assert_state_equal(pool, st)
    sch.drop_blocks(entry_dev)
    st.drop_entry(entry)
    _assert_state_equal(pool, st)
    assert append([4, 1], 16) == OK
    # capacity error: all-or-nothing
    assert append([0, 4], 200) == -3
    # exhaustion error: all-or-nothing
    assert append([5], 8 * 16) == -4


# --------------------------------------------------------------------- sampling
def test_sample_talker_head_matches_oracle():
    R, V = 64, 3072
    g = _gen(30)
    logits = torch.randn(R, V, generator=g)
    counts = (torch.rand(R, V, generator=g) < 0.05).long() * torch.randint(1, 4, (R, V), generator=g)
    gum = M.gumbel_from_uniform(torch.rand(R, 50, generator=g))
    temp = torch.full((R, 1), 0.9)
    pen = torch.full((R, 1), 1.05)
    tok_ref, counts_ref = M.talker_sample(logits, counts, gum, temp, pen, eos_id=2150)
    c_dev = counts.to(DEV)
    tok = ops.sample(logits.to(DEV), 50, gumbel=gum.to(DEV), temperature=temp.to(DEV).view(-1),
                     penalty=pen.to(DEV).view(-1), counts=c_dev, eos_id=2150)
    assert torch.equal(tok.cpu(), tok_ref)
    assert torch.equal(c_dev.cpu(), counts_ref)


def test_sample_greedy_and_cp_select():
    R, V = 64, 2048
    g = _gen(31)
    logits = torch.randn(R, V, generator=g)
    gum = M.gumbel_from_uniform(torch.rand(R, 15, 50, generator=g))
    temp = torch.full((R, 1), 0.9)
    for s in (0, 7, 14):
        ref = M.topk_select(logits, temp, gum[:, s], 50)
        tok = ops.sample(logits.to(DEV), 50, gumbel=gum[:, s].contiguous().to(DEV), temperature=temp.view(-1).to(DEV))
        assert torch.equal(tok.cpu(), ref)
    zeros = torch.zeros(R, 50)
    tok = ops.sample(logits.to(DEV), 50, gumbel=zeros.to(DEV))
    assert torch.equal(tok.cpu(), logits.argmax(-1))


def test_sample_philox_noise_is_deterministic_and_keyed():
    R, V = 8, 2048
    logits = torch.zeros(R, V, device=DEV)
    key = torch.arange(R, dtype=torch.int64, device=DEV) * 7 + 3
    a = ops.sample(logits, 50, seed=123, noise_key=key, step=5)
    b = ops.sample(logits, 50, seed=123, noise_key=key, step=5)
    c = ops.sample(logits, 50, seed=123, noise_key=key, step=6)
    assert torch.equal(a, b)
    assert not torch.equal(a, c)
    assert int(a.min()) >= 0 and int(a.max()) < V


# --------------------------------------------------------------------- small ops
def test_rmsnorm_and_codec_sum():
    H = 2048
    x = torch.randn(64, H, generator=_gen(40)).to(DEV)
    w = (1 + 0.1 * torch.randn(H, generator=_gen(41))).to(torch.bfloat16).to(DEV)
    y = ops.rmsnorm(x, w, 1e-6)
    torch.testing.assert_close(y.float(), M.rms_norm(x, w.float(), 1e-6), rtol=1e-2, atol=1e-2)
    t0 = _rand((3072, H), 42, 0.02)
    tc = _rand((15, 2048, H), 43, 0.02)
    codes = torch.cat([torch.randint(0, 3072, (64, 1), generator=_gen(44)),
                       torch.randint(0, 2048, (64, 15), generator=_gen(45))], 1).to(DEV)
    text = torch.randn(64, H, generator=_gen(46)).to(DEV) * 0.02
    cs, nx = ops.codec_sum(codes, t0, tc, text)
    W = {"talker.codec_embedding.weight": t0.float().cpu()}
    for s in range(15):
        W[f"cp.codec_embedding.{s}.weight"] = tc[s].float().cpu()
    ref = M.codec_sum(M.stacked_codec_table(W, 15), codes.cpu())
    torch.testing.assert_close(cs.cpu(), ref, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(nx.cpu(), ref + text.cpu(), rtol=1e-6, atol=1e-7)  # next input stays fp32


@pytest.mark.skipif(os.environ.get("QTTS_GEMM_PUSH") is not None or os.environ.get("QTTS_GEMM_BN32") is not None,
                    reason="already a forced run")
@pytest.mark.parametrize("knob", ["QTTS_GEMM_PUSH", "QTTS_GEMM_BN32"])
def test_gemm_opt_in_variants(knob):
    """The push form of the split-K reduction and 32-token tiles are opt-in (read once per
    process); rerun the GEMM tests in a child process with each on."""
    import subprocess
    import sys

    env = dict(os.environ, **{knob: "1"})
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider", "-k", "gemm",
                        os.path.abspath(__file__)], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.skipif(os.environ.get("QTTS_ATTN_ROWS") is not None, reason="already a forced run")
def test_attention_split_form():
    """head_dim 128 decode attention runs one CTA per (row, kv head) by default; the split form
    (paged_attn_tc_kernel + attn_combine_kernel) stays available (QTTS_ATTN_ROWS=0, read once per
    process): rerun the attention tests in a child process with it."""
    import subprocess
    import sys

    env = dict(os.environ, QTTS_ATTN_ROWS="0")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider", "-k",
                        "attention and not split_form", os.path.abspath(__file__)], env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


# --------------------------------------------------------------------- bounded device waits
def test_bounded_wait_runs_out_and_returns_a_status():
    """The failure path of every mbarrier wait in the library: a wait on a phase that nothing
    completes gives up after its limit, records the device error word and returns; the
    context stays usable (a second launch that does arrive succeeds)."""
    import time

    lib = _lib.load()
    status = torch.full((1,), 12345, dtype=torch.int32, device=DEV)
    assert _lib.device_error() == 0
    t0 = time.perf_counter()
    _lib.check(lib.qtts_selftest_bounded_wait(20_000_000, 0, status.data_ptr(), _lib.stream_ptr()), "selftest")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status.item()) == _lib.ERR_TIMEOUT
    assert waited >= 0.015, waited  # it did wait about the limit (20 ms), then returned
    assert _lib.device_error() == 7  # DEV_ERR_SELFTEST_WAIT; reading clears the word
    assert _lib.device_error() == 0
    status.fill_(12345)
    _lib.check(lib.qtts_selftest_bounded_wait(20_000_000, 1, status.data_ptr(), _lib.stream_ptr()), "selftest")
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.OK
    assert _lib.device_error() == 0
    # out-of-range limits are refused on the host
    assert lib.qtts_selftest_bounded_wait(0, 0, status.data_ptr(), _lib.stream_ptr()) == _lib.ERR_INVALID
    assert lib.qtts_selftest_bounded_wait(3_000_000_000, 0, status.data_ptr(), _lib.stream_ptr()) == _lib.ERR_INVALID
