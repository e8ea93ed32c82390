"""Single-kernel timing on small cases that still exceed L2 (126 MB).

    python microbench.py attention [--rows 64] [--ctx-mean 520] [--launches 50]
    python microbench.py prefill-attention [--streams 8] [--prefill-chunk 128] [--past 384]
    python microbench.py gemm [--n 12288] [--k 2048] [--m 64] [--launches 50]
    python microbench.py code2wav [--rows 64] [--launches 50] [--chunk 25]

Prints one JSON line with the mean launch time (CUDA events) and the
achieved bandwidth over the kernel's algorithmic bytes:
* attention: K+V bytes of every visible key of one layer (fp16) + q/out;
* gemm: the weight bytes (bf16) + activation hi/lo operands + fp32 output.
Inputs cycle through enough copies that every launch reads from HBM.  The
same command is the small case for an ``ncu --set full`` capture.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

from test_stateful_b200 import _lib, ops  # noqa: E402


def bench_attention(rows: int, ctx_mean: int, launches: int, layers: int = 4, seed: int = 0, split: int = 0,
                    spread: float = 0.5):
    """Decode attention over `rows` rows with contexts U[mean (1 - spread), mean (1 + spread)]
    (spread 0: every row at the mean)."""
    dev = "cuda"
    g = torch.Generator().manual_seed(seed)
    lo, hi = max(1, int(ctx_mean * (1 - spread))), max(1, int(ctx_mean * (1 + spread)))
    ctx = torch.randint(lo, hi + 1, (rows,), generator=g)
    nblk = [-(-int(c) // 16) for c in ctx]
    mbps = max(nblk)
    total = sum(nblk)
    kv = torch.randn(total, layers, 2, 8, 16, 128, generator=g).to(torch.float16).to(dev)
    table = torch.full((rows, mbps), -1, dtype=torch.int32)
    perm = torch.randperm(total, generator=g)
    off = 0
    for r, n in enumerate(nblk):
        table[r, :n] = perm[off:off + n].to(torch.int32)
        off += n
    table = table.to(dev)
    q = torch.randn(rows, 16, 128, generator=g).to(dev)
    row_slot = torch.arange(rows, dtype=torch.int32, device=dev)
    row_ctx = ctx.to(torch.int32).to(dev)
    out = torch.empty(rows, 16 * 128, device=dev, dtype=torch.bfloat16)
    out_lo = torch.empty_like(out)
    max_ctx = mbps * 16
    for i in range(3):
        ops.paged_attention(q, kv, i % layers, table, row_slot, row_ctx, max_ctx, out=out, out_lo=out_lo,
                                    split_blocks=split)
    torch.cuda.synchronize()
    # captured in a CUDA graph: the per-call host path is not timed
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(launches):
                ops.paged_attention(q, kv, i % layers, table, row_slot, row_ctx, max_ctx, out=out, out_lo=out_lo,
                                    split_blocks=split)
        graph.replay()
        s.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        graph.replay()
        e1.record(s)
        s.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / launches
    algo = int(ctx.sum()) * 2 * 8 * 128 * 2 + rows * 16 * 128 * (4 + 4)
    rows_form = os.environ.get("QTTS_ATTN_ROWS") != "0"
    kernel = "paged_attn_tc_row_kernel (CTA per row x kv head)" if rows_form else "paged_attn_tc_kernel + combine"
    return {"kernel": kernel, "split_blocks": split or 16, "rows": rows, "ctx_sum": int(ctx.sum()), "launch_us": sec * 1e6,
            "algorithmic_bytes": algo, "achieved_gbs": algo / sec / 1e9}


def bench_prefill_attention(streams: int, chunk: int, past: int, launches: int, layers: int = 8, seed: int = 0,
                            split: int = 0):
    """One prompt chunk per stream: ``chunk`` query rows at positions past .. past + chunk - 1
    (causal key counts past + t + 1), every stream's blocks scattered over the pool.  Times the
    query-tile prefill kernel and, for comparison, the decode kernel given the same rows (one
    row per query, each re-reading its whole context).  Bytes counted once per launch: the K+V
    of every key the chunk sees + q in / out ("unique")."""
    dev = "cuda"
    g = torch.Generator().manual_seed(seed)
    ctx_end = past + chunk
    nblk = -(-ctx_end // 16)
    total = streams * nblk
    kv = torch.randn(total, layers, 2, 8, 16, 128, generator=g).to(torch.float16).to(dev)
    perm = torch.randperm(total, generator=g).to(torch.int32)
    table = perm.view(streams, nblk).contiguous().to(dev)
    R = streams * chunk
    q = torch.randn(R, 16, 128, generator=g).to(dev)
    row_slot = torch.tensor([b for b in range(streams) for _ in range(chunk)], dtype=torch.int32, device=dev)
    row_ctx = torch.tensor([past + t + 1 for _ in range(streams) for t in range(chunk)], dtype=torch.int32,
                           device=dev)
    max_ctx = nblk * 16
    out = torch.empty(R, 16 * 128, device=dev, dtype=torch.bfloat16)
    out_lo = torch.empty_like(out)

    def timed(fn):
        for i in range(3):
            fn(i % layers)
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for i in range(launches):
                    fn(i % layers)
            graph.replay()
            s.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            graph.replay()
            e1.record(s)
            s.synchronize()
        return e0.elapsed_time(e1) / 1e3 / launches

    t_pre = timed(lambda l: ops.paged_attention_prefill(q, kv, l, table, row_slot, row_ctx, max_ctx, chunk, out=out,
                                                        out_lo=out_lo, split_blocks=split))
    t_dec = timed(lambda l: ops.paged_attention(q, kv, l, table, row_slot, row_ctx, max_ctx, out=out, out_lo=out_lo,
                                                split_blocks=split))
    unique = streams * ctx_end * 2 * 8 * 128 * 2 + R * 16 * 128 * (4 + 4)
    # causal score + PV multiply-adds of every (query, head, visible key): 2 x 2 x D flops each
    flops = streams * 16 * 4 * 128 * sum(past + t + 1 for t in range(chunk))
    umma = os.environ.get("QTTS_PREFILL_UMMA") != "0"
    kernel = "paged_prefill_umma_kernel (tcgen05, 64-query groups)" if umma else "paged_prefill_tc_kernel (8-query tiles)"
    return {"kernel": kernel, "streams": streams, "chunk": chunk, "past": past,
            "split_blocks": split or 16, "launch_us": t_pre * 1e6, "unique_bytes": unique,
            "achieved_unique_gbs": unique / t_pre / 1e9, "causal_tflops": flops / t_pre / 1e12,
            "prefill_tokens_per_s": R / t_pre,
            "decode_kernel_same_rows_us": t_dec * 1e6, "speedup_vs_decode_rows": t_dec / t_pre}


def bench_gemm(n: int, k: int, m: int, launches: int, seed: int = 0, plain: bool = False):
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(seed)
    copies = max(2, -(-300_000_000 // (n * k * 2)))  # > 2x L2 of distinct weights
    ws = [torch.randn(n, k, generator=g, device=dev).mul_(0.02).to(torch.bfloat16) for _ in range(copies)]
    x = torch.randn(m, k, generator=g, device=dev)
    hi, lo = ops.split_hilo(x)
    out = torch.empty(m, n, device=dev)
    if plain:  # one bf16 MMA per k-slice instead of the hi/lo pair
        lo = None
    for i in range(3):
        ops.gemm(hi, ws[i % copies], _lib.EPI_F32, out=out, x_lo=lo)
    torch.cuda.synchronize()
    # captured in a CUDA graph: the per-call host path (tensor-map encoding) is not timed
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(launches):
                ops.gemm(hi, ws[i % copies], _lib.EPI_F32, out=out, x_lo=lo)
        graph.replay()
        s.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        graph.replay()
        e1.record(s)
        s.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / launches
    algo = n * k * 2 + m * k * 4 + m * n * 4
    return {"kernel": "gemm_tc_kernel<64,4,bf16>" if plain else "gemm_tc_kernel<64,3,hi/lo>", "n": n, "k": k,
            "m": m, "launch_us": sec * 1e6,
            "algorithmic_bytes": algo, "achieved_gbs": algo / sec / 1e9,
            "tflops": 2 * 2 * m * n * k / sec / 1e12}


def bench_code2wav(rows: int, launches: int, seed: int = 0, chunk: int = 1):
    """One code2wav call (full decoder widths) for `rows` streams x `chunk` frames,
    captured in a CUDA graph and replayed; frames/s = rows * chunk / call time."""
    from test_stateful_b200 import weights as wmod
    from test_stateful_b200.config import Code2WavConfig
    from test_stateful_b200.runtime.code2wav import DeviceCode2Wav
    dev = "cuda"
    cfg = Code2WavConfig()
    dec = DeviceCode2Wav(cfg, wmod.make_code2wav_weights(cfg, seed), dev, max_slots=rows, max_frames=4096,
                         max_chunk=chunk)
    slots = torch.arange(rows, dtype=torch.int32, device=dev)
    dec.reset(slots)
    g = torch.Generator(device=dev).manual_seed(seed)
    codes = torch.randint(0, cfg.codebook_size, (rows, chunk, 16), generator=g, device=dev)
    wav = torch.empty(rows, chunk * cfg.samples_per_frame, device=dev)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        dec.step(codes, slots, wav, stream=s, frames=chunk)
        s.synchronize()
        first = wav.double()
        first_sum, first_abs = float(first.sum()), float(first.abs().sum())
        for _ in range(2):
            dec.step(codes, slots, wav, stream=s, frames=chunk)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            dec.step(codes, slots, wav, stream=s, frames=chunk)
        for _ in range(3):
            graph.replay()
        s.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(launches):
            graph.replay()
        e1.record(s)
        s.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / launches
    flops = 5.1e9 * rows * chunk
    out = {"kernel": "code2wav step", "rows": rows, "chunk": chunk, "step_us": sec * 1e6,
           "frames_per_s": rows * chunk / sec,
           "kernels_per_step": dec.last_launches, "approx_tflops": flops / sec / 1e12,
           "wav_absmean": float(wav.abs().mean()), "first_call_sum": first_sum, "first_call_abs_sum": first_abs}
    dec.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["attention", "prefill-attention", "gemm", "code2wav"])
    ap.add_argument("--streams", type=int, default=8, help="prefill-attention: streams with one chunk each")
    ap.add_argument("--prefill-chunk", type=int, default=128, help="prefill-attention: query rows per stream")
    ap.add_argument("--past", type=int, default=384, help="prefill-attention: positions before the chunk")
    ap.add_argument("--rows", type=int, default=64)
    ap.add_argument("--ctx-mean", type=int, default=520)
    ap.add_argument("--ctx-spread", type=float, default=0.5, help="attention: contexts U[mean(1-s), mean(1+s)]")
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--m", type=int, default=64)
    ap.add_argument("--launches", type=int, default=50)
    ap.add_argument("--split", type=int, default=0, help="attention: KV blocks per split (0: library default)")
    ap.add_argument("--chunk", type=int, default=1, help="code2wav: frames per stream per call")
    ap.add_argument("--plain", action="store_true", help="gemm: plain bf16 activations (no lo operand)")
    a = ap.parse_args()
    if a.what == "attention":
        r = bench_attention(a.rows, a.ctx_mean, a.launches, split=a.split, spread=a.ctx_spread)
    elif a.what == "prefill-attention":
        r = bench_prefill_attention(a.streams, a.prefill_chunk, a.past, a.launches, split=a.split)
    elif a.what == "code2wav":
        r = bench_code2wav(a.rows, a.launches, chunk=a.chunk)
    else:
        r = bench_gemm(a.n, a.k, a.m, a.launches, plain=a.plain)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
