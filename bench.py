#!/usr/bin/env python3
"""Codec frames/s/GPU of the continuous-batching decode step (64 ragged streams, 512 steps).

Workload (seeded synthetic, no dataset): 64 concurrent streams per GPU, prompt
lengths U{16..512} whose first min(96, L) token ids are a shared prefix
(prefix-cache hit: the prefix blocks are shared, partial blocks copied on the
first write), random-init weights of the Qwen3-TTS talker (28 layers, hidden
2048, 16/8 heads, d128, SwiGLU 6144, codec vocab 3072) and the 15-stage code
predictor (5 layers, hidden 1024), 16-token KV blocks in an 8192-block pool,
top-k 50 / temperature 0.9 sampling with in-kernel Philox noise.

One step = one decode step for all 64 streams (talker + sampling + code
predictor + codec sum + streaming code2wav), i.e. 64 codec frames and 64 x 1920
waveform samples — the unit of work of the reference's fused
talker+code2wav plan.  ``value`` replays the captured decode step with
everything resident on the device; ``e2e`` goes through the public executor
call (``B200Executor.launch_decode_step`` -> ``GPUFuture.wait``) with the
per-step text embeddings copied from pinned host memory and the codec frames
and audio chunks copied back every step.

``--impl reference`` times the CPU oracle (a restatement of the reference's
PyTorch modules, fp32) on the host cores.  Under torchrun each rank is an
independent replica (request-sharded, no collective on the decode path).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "codec frames/sec/GPU at 64 ragged streams (1/2/4/8 B200); p50 step latency"
UNIT = "frames/s"
STREAMS = 64
PREFIX = 96
SEED = 1


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=512)  # the benchmark workload: 512 decode steps
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--profile", action="store_true",
                    help="timed region only, inside an NVTX range 'timed' (for ncu --nvtx-include timed/); "
                         "no CPU baseline, e2e or roofline pass")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ----------------------------------------------------------------------------- workload
def build_workload(device):
    from test_stateful_b200 import workload
    from test_stateful_b200.config import EngineConfig
    from test_stateful_b200.runtime.executor import B200Executor

    steps_total = ARGS.warmup + ARGS.steps + ARGS.e2e_steps + 2
    max_seq = 512 + steps_total + 16
    ex = B200Executor(device_id=device.index or 0, max_batch_size=STREAMS + 1, max_seq_len=max_seq,
                      model_config=EngineConfig(), do_sample=True, temperature=0.9, repetition_penalty=1.05,
                      random_seed=SEED, num_blocks=8192, weight_seed=SEED, max_prefill_rows=512)
    ex.load()
    t = ex._config.talker
    prompts = workload.shared_prefix_prompts(STREAMS, 16, 512, PREFIX, SEED)
    table = workload.text_table(t.hidden_size, SEED, device=device)
    pad = workload.tts_pad_embed(t.hidden_size, SEED, device=device)
    pool = ex.kv_pool
    cache = ex.make_prefix_cache(max_entries=4, max_prefix_len=512)
    # the shared prefix: prefill once into a holder slot, cache its blocks, free the slot
    holder = pool.allocate("prefix-holder")
    longest = max(prompts, key=len)
    ex.prefill_prefix_only(holder, table[longest[:PREFIX].to(device)].unsqueeze(0))
    cache.put("shared-96", holder.slot_id, PREFIX)
    pool.release(holder.slot_id)
    entry = cache.get("shared-96")
    slots = []
    for i, ids in enumerate(prompts):
        s = pool.allocate(f"stream-{i}")
        s.segment_idx = 0
        n_shared = min(PREFIX, len(ids))
        cache.restore(s, entry) if n_shared == PREFIX else _share_partial(cache, s, entry, n_shared)
        suffix = ids[n_shared:]
        if len(suffix) > 0:
            ex.prefill_from_prefix(s, table[suffix.to(device)].unsqueeze(0))
        else:
            ex._configure_sampling(s)
            ex.next_x[s.slot_id].copy_(pad)
        ex.set_text_embedding(s, pad)
        slots.append(s)
    torch.cuda.synchronize(device)
    return ex, slots, prompts, pad


def _share_partial(cache, slot, entry, n):
    """A prompt shorter than the prefix shares ceil(n/16) prefix blocks; the
    last one is partial and gets copied on the first write (copy-on-write)."""
    from test_stateful_b200.runtime.pool import PagedPrefixEntry
    part = PagedPrefixEntry(key=entry.key, blocks=entry.blocks[: -(-n // 16)], prefix_len=n,
                            created_at=entry.created_at)
    cache.restore(slot, part)


# ----------------------------------------------------------------------------- roofline helpers
def attention_roofline(ex, slots, peaks):
    """Paged decode attention at the workload's final state, timed with CUDA events."""
    from test_stateful_b200 import ops
    m = ex.model
    t = ex._config.talker
    dev = m.pool.kv.device
    n = len(slots)
    ctx = torch.tensor([s.past_len for s in slots], dtype=torch.int32, device=dev)
    row_slot = torch.tensor([s.slot_id for s in slots], dtype=torch.int32, device=dev)
    q = torch.randn(n, t.num_heads, t.head_dim, device=dev)
    max_ctx = ex._config.pool.max_blocks_per_seq * 16
    out = torch.empty(n, t.num_heads * t.head_dim, device=dev, dtype=torch.bfloat16)
    nb = -(-max_ctx // 16)
    splits = max(1, -(-nb // 1))  # scratch for any split size
    ws_o = torch.empty(n * t.num_heads * splits * t.head_dim, device=dev)
    ws_ml = torch.empty(n * t.num_heads * splits * 2, device=dev)
    table = m.pool.block_table

    split = int(os.environ.get("QTTS_ATTN_SPLIT", "8"))  # the engine's split size

    def run(layer):
        ops.paged_attention(q, m.pool.kv, layer, table, row_slot, ctx, max_ctx, out=out, ws_o=ws_o, ws_ml=ws_ml,
                            split_blocks=split)

    for layer in range(3):
        run(layer)
    torch.cuda.synchronize()
    # all layers of the pool, twice, captured in a CUDA graph and replayed on one stream
    reps = 2 * t.num_layers
    gs = torch.cuda.Stream()
    with torch.cuda.stream(gs):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gs):
            for i in range(reps):
                run(i % t.num_layers)
        graph.replay()
        gs.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(gs)
        graph.replay()
        e1.record(gs)
        gs.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    kv_bytes = int(ctx.sum()) * 2 * t.kv_heads * t.head_dim * 2      # K+V of one layer
    qo_bytes = n * t.num_heads * t.head_dim * (4 + 2)
    algo = kv_bytes + qo_bytes
    gbs = algo / sec / 1e9
    peak = peaks.get("hbm_gbs")
    # DRAM traffic per launch: an ncu capture of the same kernel on 64 rows at mean context 858
    # read 228.13 MB + wrote 5.01 MB for 225.93 MB of algorithmic bytes
    # (profiles/paged_attn_kernel_d128_64rows_ctx520.md); traffic grows with the blocks read,
    # so this launch's traffic is scaled from that ratio
    traffic_ratio = (228.13 + 5.01) / 225.93
    return {"kernel": "paged_attn_tc_kernel + attn_combine_kernel", "bound": "hbm", "achieved": round(gbs, 1),
            "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 3) if peak else None,
            "traffic": int(algo * traffic_ratio),
            "traffic_source": "ncu dram__bytes_read+write of a 64-row, mean-context-858 capture, scaled by bytes",
            "algorithmic_bytes_per_launch": algo, "launch_us": round(sec * 1e6, 2),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_oracle_rate(n_streams=4, ctx=256, steps=40, warmup=1):
    """The oracle (fp32, all host threads) on a bounded sample of the workload:
    ``warmup`` untimed then ``steps`` timed decode steps of ``n_streams`` streams starting
    at context ``ctx`` (about 10 s of CPU work at the default)."""
    from oracle.engine import OracleEngine
    from oracle import model as M
    from test_stateful_b200 import weights as wmod
    from test_stateful_b200.config import EngineConfig
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = EngineConfig()
    t, c = cfg.talker, cfg.cp
    W = wmod.make_talker_weights(t, SEED, dtype=torch.float32)
    W.update(wmod.make_cp_weights(c, SEED, dtype=torch.float32))
    eng = OracleEngine(W, t, c)
    g = torch.Generator().manual_seed(0)
    for i in range(n_streams):
        eng.k[i] = [torch.randn(t.kv_heads, ctx, t.head_dim, generator=g) * 0.5 for _ in range(t.num_layers)]
        eng.v[i] = [torch.randn(t.kv_heads, ctx, t.head_dim, generator=g) * 0.5 for _ in range(t.num_layers)]
        eng.past[i] = ctx
    x = torch.randn(n_streams, t.hidden_size, generator=g) * 0.02
    counts = torch.zeros(n_streams, t.codec_vocab_size, dtype=torch.long)
    temp = torch.full((n_streams, 1), 0.9)
    pen = torch.full((n_streams, 1), 1.05)
    t0 = None
    for k in range(warmup + steps):
        if k == warmup:
            t0 = time.perf_counter()
        gum = M.gumbel_from_uniform(torch.rand(n_streams, 50, generator=g))
        cgum = M.gumbel_from_uniform(torch.rand(n_streams, c.num_stages, 50, generator=g))
        r = eng.decode(list(range(n_streams)), x, counts, gum, cgum, temp, pen)
        x = r["codec_sum"]
        counts = r["counts"]
    dt = time.perf_counter() - t0
    frames = n_streams * steps
    return {"value": round(frames / dt, 3), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{steps} decode steps x {n_streams} streams at context {ctx}, full 28-layer talker + "
                      f"15-stage code predictor (reference full recompute), fp32, {torch.get_num_threads()} threads",
            "seconds": round(dt, 2)}


# ----------------------------------------------------------------------------- main arms
def run_reference(rank, world):
    if rank != 0:
        return
    # the arm's own --steps / --warmup; each step is a two-stream sample of the 64-stream step
    # (0.1-0.2 s of CPU work on 16 threads, so the default 512 steps end within about two minutes)
    base = cpu_oracle_rate(n_streams=2, steps=max(1, ARGS.steps), warmup=ARGS.warmup)
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": world,
            "steps": ARGS.steps, "warmup": ARGS.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg2 decode step (bounded CPU sample)", "streams": STREAMS},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200(rank, world, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=600))
    ex, slots, prompts, pad = build_workload(dev)
    n = len(slots)
    stream = ex._stream

    # warm-up: eager step, capture, replays
    for _ in range(max(1, ARGS.warmup)):
        ex.launch_decode_step(slots).wait()
    launches = ex.prepare_replay(slots)  # CUDA graphs of the step (stream A: talker + CP; B: code2wav)
    for _ in range(2):
        ex.replay_step(n)
    torch.cuda.synchronize(dev)

    # ---- timed region: K replays, inputs resident (KV + weights >> L2: no flush needed)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    # Step k's code2wav (stream B) overlaps step k + 1's talker and code predictor (stream A);
    # the timed region runs from before step 0 to the end of the last step's code2wav.
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(ARGS.steps + 1)]
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    with torch.cuda.stream(stream):
        evs[0].record(stream)
    last_b = None
    for k in range(ARGS.steps):
        ev_a, last_b = ex.replay_step(n)
        with torch.cuda.stream(stream):
            evs[k + 1].record(stream)  # stream A's part of step k done
    with torch.cuda.stream(stream):
        stream.wait_event(last_b)
        end.record(stream)
    torch.cuda.synchronize(dev)
    torch.cuda.nvtx.range_pop()
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    for s in slots:
        s.past_len += ARGS.steps
        s.frame_idx += ARGS.steps
    per_step = [evs[k].elapsed_time(evs[k + 1]) for k in range(ARGS.steps)]
    total_ms = evs[0].elapsed_time(end)
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    frames = n * ARGS.steps * world
    value = frames / (total_ms / 1e3)
    if ARGS.profile:
        if rank == 0:
            print(json.dumps({"profile_run": True, "value": round(value, 1), "unit": UNIT,
                              "ms_per_step": round(total_ms / ARGS.steps, 4), "kernels_per_step": launches}))
        ex._graphs.clear()
        ex.shutdown()
        return

    # ---- e2e through the executor call with host buffers
    t_host = pad.float().cpu().expand(n, -1).contiguous().pin_memory()
    idx = torch.tensor([s.slot_id for s in slots], dtype=torch.long, device=dev)
    staged = torch.empty_like(t_host, device=dev)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    # one step of lookahead, as a serving loop runs it: step k + 1 is launched (its text
    # input copied from pinned host memory first) before step k's codes and audio are read
    t0 = time.perf_counter()
    pending = None
    for _ in range(ARGS.e2e_steps):
        with torch.cuda.stream(stream):
            staged.copy_(t_host, non_blocking=True)
            ex.text_add.index_copy_(0, idx, staged)
        fut = ex.launch_decode_step(slots)
        if pending is not None:
            out = pending.wait()
            _ = out.full_codec, out.audio_chunks
        pending = fut
    out = pending.wait()
    _ = out.full_codec, out.audio_chunks
    torch.cuda.synchronize(dev)
    e2e_sec = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_sec], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_sec = float(t.item())
    e2e_value = n * ARGS.e2e_steps * world / e2e_sec
    h2d = t_host.numel() * 4 + n * 4
    d2h = n * (1 + ex._config.cp.num_stages) * 8 + 4 + n * ex._config.c2w.samples_per_frame * 4

    peaks = load_peaks()
    roof = attention_roofline(ex, slots, peaks)
    ctx_now = [s.past_len for s in slots]
    cpu = None
    if rank == 0 and not ARGS.no_cpu_baseline:
        cpu = cpu_oracle_rate()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": ARGS.steps,
            "warmup": ARGS.warmup, "ms_per_step": round(total_ms / ARGS.steps, 4),
            "p50_step_ms": round(statistics.median(per_step), 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2: 64 ragged streams/GPU, ctx U{16..512} + 96-token shared prefix, "
                                   "8192 x 16-token KV blocks, top-k 50 / T 0.9 Philox sampling",
                       "streams_per_gpu": n, "parallelism": f"replicas x{world} (request-sharded, no collective)",
                       "l2": "inputs larger than L2 (KV ~4 GB + weights ~3 GB read per step)",
                       "step": "talker 28 layers + sampling + 15-stage code predictor + codec sum + "
                               "streaming code2wav (1920 samples/stream)",
                       "pipeline": "two streams: step k's code2wav overlaps step k+1's talker + code predictor; "
                                   "timed from step 0's start to the last step's code2wav end",
                       "ctx_mean_end": round(sum(ctx_now) / len(ctx_now), 1)},
            "gpu_launches": launches * ARGS.steps,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": ARGS.e2e_steps, "path": "B200Executor.launch_decode_step -> GPUFuture.wait",
                    "lookahead": "step k+1 launched before step k's results are read"},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    ex._graphs.clear()
    ex.shutdown()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    global ARGS
    ARGS = parse()
    rank, world, local = dist_env()
    if ARGS.impl == "reference":
        run_reference(rank, world)
        return
    run_b200(rank, world, local)


if __name__ == "__main__":
    main()
