"""Kernel-level Python API over the C ABI (torch tensors in, torch tensors out).

Each function launches one entry point of ``libqtts_b200.so`` on the current
CUDA stream.  Inputs must already be CUDA tensors of the stated dtype; there
is no CPU path.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libqtts_b200 kernels take CUDA tensors only")


def split_hilo(x: torch.Tensor):
    """fp32 activation -> (hi, lo) bf16 pair with hi + lo ~ x."""
    hi = x.to(torch.bfloat16)
    return hi, (x - hi.float()).to(torch.bfloat16)


def gemm(x: torch.Tensor, w: torch.Tensor, epilogue: int = _lib.EPI_F32, out: Optional[torch.Tensor] = None,
         bias: Optional[torch.Tensor] = None, qkv: Optional[_lib.QkvEpilogue] = None,
         x_lo: Optional[torch.Tensor] = None, out_lo: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``(x [+ x_lo]) [M,K] bf16 · w [N,K]^T`` with a fused epilogue (see ``_lib.EPI_*``)."""
    _need_cuda(x, w, out, bias, x_lo, out_lo)
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        if epilogue == _lib.EPI_F32:
            out = torch.empty(M, N, device=x.device, dtype=torch.float32)
        elif epilogue == _lib.EPI_BF16:
            out = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
        elif epilogue == _lib.EPI_SWIGLU:
            out = torch.empty(M, N // 2, device=x.device, dtype=torch.bfloat16)
        else:
            raise ValueError("this epilogue needs an explicit out tensor")
    rc = _lib.load().qtts_gemm(x.data_ptr(), _lib.ptr(x_lo), M, K, w.data_ptr(), N, epilogue, out.data_ptr(),
                               _lib.ptr(out_lo), _lib.ptr(bias), C.byref(qkv) if qkv is not None else None,
                               _lib.stream_ptr())
    _lib.check(rc, "gemm")
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, rows: Optional[int] = None, ld: Optional[int] = None,
            out: Optional[torch.Tensor] = None, out_lo: Optional[torch.Tensor] = None) -> torch.Tensor:
    _need_cuda(x, w)
    H = w.shape[0]
    M = rows if rows is not None else x.numel() // H
    ld = ld if ld is not None else H
    if out is None:
        out = torch.empty(M, H, device=x.device, dtype=torch.bfloat16)
    _lib.check(_lib.load().qtts_rmsnorm(x.data_ptr(), M, H, ld, w.data_ptr(), eps, out.data_ptr(),
                                        _lib.ptr(out_lo), _lib.stream_ptr()), "rmsnorm")
    return out


def paged_attention(q: torch.Tensor, kv_pool: torch.Tensor, layer: int, block_table: torch.Tensor,
                    row_slot: torch.Tensor, row_ctx: torch.Tensor, max_ctx: int,
                    out: Optional[torch.Tensor] = None, ws_o: Optional[torch.Tensor] = None,
                    ws_ml: Optional[torch.Tensor] = None, out_lo: Optional[torch.Tensor] = None,
                    split_blocks: int = 0) -> torch.Tensor:
    """``q [R, Hq, D]`` fp32 over ``kv_pool [blocks, L, 2, Hkv, 16, D]`` fp16; ``split_blocks``
    KV blocks per split (0: the library default)."""
    _need_cuda(q, kv_pool, block_table, row_slot, row_ctx)
    R, Hq, D = q.shape
    nb, L, _, Hkv, bs, _ = kv_pool.shape
    n_blocks = -(-max_ctx // bs)
    splits = max(1, -(-n_blocks // (split_blocks or _lib.ATTN_SPLIT_BLOCKS)))
    if out is None:
        out = torch.empty(R, Hq * D, device=q.device, dtype=torch.bfloat16)
    if ws_o is None:
        ws_o = torch.empty(R * Hq * splits * D, device=q.device, dtype=torch.float32)
    if ws_ml is None:
        ws_ml = torch.empty(R * Hq * splits * 2, device=q.device, dtype=torch.float32)
    rc = _lib.load().qtts_paged_attention(q.data_ptr(), R, Hq, Hkv, D, kv_pool.data_ptr(), layer, L, bs, nb,
                                          block_table.data_ptr(), block_table.shape[-1], row_slot.data_ptr(),
                                          row_ctx.data_ptr(), max_ctx, split_blocks, ws_o.data_ptr(), ws_ml.data_ptr(),
                                          out.data_ptr(), _lib.ptr(out_lo), _lib.stream_ptr())
    _lib.check(rc, "paged_attention")
    return out


def paged_attention_prefill(q: torch.Tensor, kv_pool: torch.Tensor, layer: int, block_table: torch.Tensor,
                            row_slot: torch.Tensor, row_ctx: torch.Tensor, max_ctx: int, rows_per_stream: int,
                            out: Optional[torch.Tensor] = None, ws_o: Optional[torch.Tensor] = None,
                            ws_ml: Optional[torch.Tensor] = None, out_lo: Optional[torch.Tensor] = None,
                            split_blocks: int = 0) -> torch.Tensor:
    """Chunked-prefill attention (head_dim 128): ``q [R, Hq, D]`` holds ``R / rows_per_stream``
    streams of ``rows_per_stream`` consecutive query rows each (row_ctx causal: past + t + 1);
    the 8-query tiles of a stream share every KV block they read."""
    _need_cuda(q, kv_pool, block_table, row_slot, row_ctx)
    R, Hq, D = q.shape
    nb, L, _, Hkv, bs, _ = kv_pool.shape
    n_blocks = -(-max_ctx // bs)
    splits = max(1, -(-n_blocks // (split_blocks or _lib.ATTN_SPLIT_BLOCKS)))
    if out is None:
        out = torch.empty(R, Hq * D, device=q.device, dtype=torch.bfloat16)
    if ws_o is None:
        ws_o = torch.empty(R * Hq * splits * D, device=q.device, dtype=torch.float32)
    if ws_ml is None:
        ws_ml = torch.empty(R * Hq * splits * 2, device=q.device, dtype=torch.float32)
    rc = _lib.load().qtts_paged_attention_prefill(q.data_ptr(), R, rows_per_stream, Hq, Hkv, D, kv_pool.data_ptr(),
                                                  layer, L, bs, nb, block_table.data_ptr(), block_table.shape[-1],
                                                  row_slot.data_ptr(), row_ctx.data_ptr(), max_ctx, split_blocks,
                                                  ws_o.data_ptr(), ws_ml.data_ptr(), out.data_ptr(), _lib.ptr(out_lo),
                                                  _lib.stream_ptr())
    _lib.check(rc, "paged_attention_prefill")
    return out


def sample(logits: torch.Tensor, topk: int, gumbel: Optional[torch.Tensor] = None, temperature=None, penalty=None,
           counts: Optional[torch.Tensor] = None, eos_id: int = -1, seed: int = 0,
           noise_key: Optional[torch.Tensor] = None, step: int = 0, tok_out: Optional[torch.Tensor] = None,
           tok_ld: int = 1) -> torch.Tensor:
    """Talker head when ``counts`` is given (suppress + penalty + counts update), else CP select."""
    _need_cuda(logits, gumbel, temperature, penalty, counts, noise_key)
    R, V = logits.shape
    if tok_out is None:
        tok_out = torch.empty(R, device=logits.device, dtype=torch.int64)
        tok_ld = 1
    rc = _lib.load().qtts_sample(logits.data_ptr(), R, V, logits.stride(0), topk, _lib.ptr(gumbel),
                                 gumbel.stride(0) if gumbel is not None else 0, seed, _lib.ptr(noise_key), step,
                                 _lib.ptr(temperature), _lib.ptr(penalty), _lib.ptr(counts), eos_id,
                                 tok_out.data_ptr(), tok_ld, _lib.stream_ptr())
    _lib.check(rc, "sample")
    return tok_out


def philox_gumbel(seed: int, keys: torch.Tensor, frames: torch.Tensor, stage: int, cols: int = 50) -> torch.Tensor:
    """The Gumbel rows the samplers draw in-kernel for per-row ``keys`` (int64) and frame
    counters ``frames`` (int32) at ``stage`` (0: talker head, 1 + s: code-predictor stage s)."""
    _need_cuda(keys, frames)
    R = keys.numel()
    out = torch.empty(R, cols, device=keys.device, dtype=torch.float32)
    _lib.check(_lib.load().qtts_philox_gumbel(int(seed) & ((1 << 64) - 1), keys.data_ptr(), frames.data_ptr(), stage,
                                              R, cols, out.data_ptr(), _lib.stream_ptr()), "philox_gumbel")
    return out


def codec_sum(codes: torch.Tensor, talker_table: torch.Tensor, cp_tables: torch.Tensor,
              text_add: Optional[torch.Tensor] = None):
    """Returns ``(codec_sum fp32 [R,H], next_x fp32 [R,H])``."""
    _need_cuda(codes, talker_table, cp_tables, text_add)
    R, G = codes.shape
    V0, H = talker_table.shape
    Vc = cp_tables.shape[1]
    cs = torch.empty(R, H, device=codes.device, dtype=torch.float32)
    nx = torch.empty(R, H, device=codes.device, dtype=torch.float32)
    rc = _lib.load().qtts_codec_sum(codes.data_ptr(), R, G, talker_table.data_ptr(), V0, cp_tables.data_ptr(), Vc, H,
                                    _lib.ptr(text_add), cs.data_ptr(), nx.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "codec_sum")
    return cs, nx


class Sched:
    """Paged-state operations on a ``runtime.model.PagedPoolTensors``."""

    def __init__(self, pool):
        self.pool = pool
        self.lib = _lib.load()
        dev = pool.free_stack.device
        self.status = torch.zeros(1, device=dev, dtype=torch.int32)

    def append(self, slots: torch.Tensor, n_new: int):
        n = slots.numel()
        dev = slots.device
        mapping = torch.empty(n * n_new, device=dev, dtype=torch.int32)
        ctx = torch.empty_like(mapping)
        pos = torch.empty_like(mapping)
        cs = torch.empty(n, device=dev, dtype=torch.int32)
        cd = torch.empty_like(cs)
        rc = self.lib.qtts_sched_append(C.byref(self.pool.state), slots.data_ptr(), n, n_new, mapping.data_ptr(),
                                        ctx.data_ptr(), pos.data_ptr(), cs.data_ptr(), cd.data_ptr(),
                                        self.status.data_ptr(), _lib.stream_ptr())
        _lib.check(rc, "sched_append")
        return mapping, ctx, pos, cs, cd

    def copy_blocks(self, cs: torch.Tensor, cd: torch.Tensor):
        rc = self.lib.qtts_kv_copy_blocks(self.pool.kv.data_ptr(), self.pool.block_elems, self.pool.kv.shape[0],
                                          cs.data_ptr(), cd.data_ptr(), cs.numel(), _lib.stream_ptr())
        _lib.check(rc, "kv_copy_blocks")

    def share_prefix(self, slot: int, blocks: torch.Tensor, prefix_len: int):
        rc = self.lib.qtts_sched_share_prefix(C.byref(self.pool.state), slot, blocks.data_ptr(), prefix_len,
                                              self.status.data_ptr(), _lib.stream_ptr())
        _lib.check(rc, "sched_share_prefix")

    def make_entry(self, slot: int, prefix_len: int) -> torch.Tensor:
        bs = self.pool.state.block_size
        out = torch.empty(max(1, -(-prefix_len // bs)), device=self.pool.free_stack.device, dtype=torch.int32)
        rc = self.lib.qtts_sched_make_entry(C.byref(self.pool.state), slot, prefix_len, out.data_ptr(),
                                            _lib.stream_ptr())
        _lib.check(rc, "sched_make_entry")
        return out[: -(-prefix_len // bs)]

    def drop_blocks(self, blocks: torch.Tensor):
        rc = self.lib.qtts_sched_drop_blocks(C.byref(self.pool.state), blocks.data_ptr(), blocks.numel(),
                                             _lib.stream_ptr())
        _lib.check(rc, "sched_drop_blocks")

    def release(self, slot: int):
        _lib.check(self.lib.qtts_sched_release(C.byref(self.pool.state), slot, _lib.stream_ptr()), "sched_release")

    def scatter(self, rows: torch.Tensor, mapping: torch.Tensor):
        """rows ``[n, L*2, Hkv, D]`` bf16 into the pool."""
        L2, Hkv, D = rows.shape[1:]
        rc = self.lib.qtts_kv_scatter(self.pool.kv.data_ptr(), C.byref(self.pool.state), L2 // 2, Hkv, D,
                                      rows.data_ptr(), mapping.data_ptr(), rows.shape[0], _lib.stream_ptr())
        _lib.check(rc, "kv_scatter")

    def gather(self, slot: int, n: int) -> torch.Tensor:
        kv = self.pool.kv
        L, Hkv, D = kv.shape[1], kv.shape[3], kv.shape[5]
        out = torch.empty(2 * L, Hkv, n, D, device=kv.device, dtype=torch.float16)
        rc = self.lib.qtts_kv_gather(kv.data_ptr(), C.byref(self.pool.state), L, Hkv, D, slot, n, out.data_ptr(),
                                     _lib.stream_ptr())
        _lib.check(rc, "kv_gather")
        return out
