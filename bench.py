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
PyTorch modules, fp32: talker, sampling head, code predictor with its full
per-stage recompute, streaming code2wav) on the host cores, on the same 64
streams and config.  Under torchrun each rank is an independent replica
(request-sharded, no collective on the decode path); rank 0 times the CPU
baseline only after every rank has left the process group.
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


def workload_config(world: int) -> dict:
    """The ``config`` both arms print (the same dict, so the two lines compare like for like)."""
    return {"workload": "cfg2: 64 ragged streams/GPU, ctx U{16..512} + 96-token shared prefix, "
                        "8192 x 16-token KV blocks, top-k 50 / T 0.9 sampling, 512 decode steps",
            "streams_per_gpu": STREAMS, "parallelism": f"replicas x{world} (request-sharded, no collective)",
            "l2": "inputs larger than L2 (KV ~4 GB + weights ~3 GB read per step)",
            "step": "talker 28 layers + sampling + 15-stage code predictor + codec sum + "
                    "streaming code2wav (1920 samples/stream)"}


def host_threads() -> int:
    """Host cores this process may run on (the GPU box's cgroup/affinity, not the machine's)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


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
    ap.add_argument("--roofline-only", action="store_true",
                    help="build the workload, run the roofline passes once and print them (the small case "
                         "for an ncu DRAM capture of the attention and GEMM kernels)")
    ap.add_argument("--num-blocks", type=int, default=8192,
                    help="KV pool blocks (8192 = the benchmark's pool; the streams use about 2300)")
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "cfg5"],
                    help="cfg2: the decode-step benchmark (default); cfg5: whole-box serving run — "
                         "128 requests/GPU arriving as a Poisson process at 25 req/s/GPU (200 req/s on 8 GPUs)")
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

    steps_total = ARGS.warmup + ARGS.steps + E2E_WARMUP + ARGS.e2e_steps + 2
    max_seq = 512 + steps_total + 16
    ex = B200Executor(device_id=device.index or 0, max_batch_size=STREAMS + 1, max_seq_len=max_seq,
                      model_config=EngineConfig(), do_sample=True, temperature=0.9, repetition_penalty=1.05,
                      random_seed=SEED, num_blocks=ARGS.num_blocks, weight_seed=SEED, max_prefill_rows=512)
    ex.load()
    t = ex._config.talker
    prompts = workload.shared_prefix_prompts(STREAMS, 16, 512, PREFIX, SEED)
    table = workload.text_table(t.hidden_size, SEED, device=device)
    pad = workload.tts_pad_embed(t.hidden_size, SEED, device=device)
    slots, _ = workload.setup_shared_prefix_streams(ex, prompts, table, pad, PREFIX)
    return ex, slots, prompts, pad


# ----------------------------------------------------------------------------- roofline helpers
# DRAM traffic per launch from an ncu capture of the same kernels on this workload
# (bench.py --roofline-only --num-blocks 2600, dram__bytes_read.sum + dram__bytes_write.sum):
# attention read 44 404 792 + wrote 1 986 bytes per launch for 43 307 008 unique KV bytes (the
# 96-token prefix every row shares is read from DRAM once), GEMM 26 023 022 + 570 bytes per
# launch for 27 262 976 algorithmic bytes (its activations stay in L2).  Traffic scales with the
# unique blocks read (attention) and the weight bytes (GEMM).
E2E_WARMUP = 3  # untimed steps through the executor call before the e2e timing
ATTN_TRAFFIC_PER_UNIQUE = (44404792 + 1986) / 43307008
GEMM_TRAFFIC_RATIO = (26023022 + 570) / 27262976


def _replay_timed(fn, reps):
    """Capture ``reps`` calls of ``fn(i)`` in a CUDA graph on a side stream, warm it, and time
    one replay with CUDA events on that stream; returns seconds per call."""
    gs = torch.cuda.Stream()
    with torch.cuda.stream(gs):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=gs):
            for i in range(reps):
                fn(i)
        graph.replay()
        gs.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(gs)
        graph.replay()
        e1.record(gs)
        gs.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def attention_roofline(ex, slots, peaks):
    """Paged decode attention at the workload's current state (every layer of the pool,
    twice), timed with CUDA events.  Algorithmic bytes count each row's visible keys (the
    shared prefix once per row, as the reference's per-stream gather reads it); unique bytes
    count every KV block once, with the most keys any row reads from it."""
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
    ws_o = torch.empty(n * t.num_heads * nb * t.head_dim, device=dev)   # scratch for any split size
    ws_ml = torch.empty(n * t.num_heads * nb * 2, device=dev)
    table = m.pool.block_table
    split = int(os.environ.get("QTTS_ATTN_SPLIT", "8"))  # the engine's split size

    def run(i):
        ops.paged_attention(q, m.pool.kv, i % t.num_layers, table, row_slot, ctx, max_ctx, out=out, ws_o=ws_o,
                            ws_ml=ws_ml, split_blocks=split)

    for layer in range(3):
        run(layer)
    torch.cuda.synchronize()
    sec = _replay_timed(run, 2 * t.num_layers)
    per_key = 2 * t.kv_heads * t.head_dim * 2                 # K+V of one layer, fp16
    kv_bytes = int(ctx.sum()) * per_key
    qo_bytes = n * t.num_heads * t.head_dim * (4 + 2)
    algo = kv_bytes + qo_bytes
    # unique blocks: the most keys any row reads from each block id
    tab = table[row_slot.long()].cpu()
    keys_in_block = {}
    for r, c in enumerate(ctx.cpu().tolist()):
        for j in range(-(-c // 16)):
            b = int(tab[r, j])
            keys_in_block[b] = max(keys_in_block.get(b, 0), min(16, c - 16 * j))
    unique = sum(keys_in_block.values()) * per_key + qo_bytes
    gbs = algo / sec / 1e9
    peak = peaks.get("hbm_gbs")
    kernel = ("paged_attn_tc_row_kernel (one CTA per row and kv head)" if os.environ.get("QTTS_ATTN_ROWS", "1") != "0"
              else "paged_attn_tc_kernel + attn_combine_kernel")
    return {"kernel": kernel, "bound": "hbm", "achieved": round(gbs, 1),
            "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 3) if peak else None,
            "traffic": int(unique * ATTN_TRAFFIC_PER_UNIQUE),
            "traffic_source": "ncu dram__bytes_read+write per launch over unique KV bytes, scaled to this launch",
            "algorithmic_bytes_per_launch": algo, "unique_bytes_per_launch": unique,
            "achieved_unique": round(unique / sec / 1e9, 1),
            "frac_unique": round(unique / sec / 1e9 / peak, 3) if peak else None,
            "ctx_mean": round(float(ctx.float().mean()), 1), "launch_us": round(sec * 1e6, 2),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}


def gemm_roofline(ex, peaks):
    """The dominant kernel of the step, gemm_tc_kernel<64,3,hi/lo> (about two thirds of the
    step's launch time), on the talker's projections: the 28 layers' QKV, O, gate/up and down
    weights of the loaded model at M = 64 tokens with bf16 hi/lo activation operands, one
    CUDA graph of all 112 launches (weights 2.83 GB > L2, so every launch streams from HBM),
    timed with CUDA events.  Plain fp32 epilogues stand in for the step's fused ones (QKV norm
    + RoPE + KV store, SwiGLU, residual); their extra bytes are a few MB per step."""
    from test_stateful_b200 import _lib, ops
    m = ex.model
    t = ex._config.talker
    dev = m.w_qkv.device
    g = torch.Generator(device=dev).manual_seed(0)
    acts = {}
    for K in sorted({t.hidden_size, t.q_size, t.intermediate_size}):
        acts[K] = ops.split_hilo(torch.randn(STREAMS, K, generator=g, device=dev))
    shapes = []
    for l in range(t.num_layers):
        for w in (m.w_qkv[l], m.w_o[l], m.w_gate_up[l], m.w_down[l]):
            shapes.append(w)
    outs = {}
    for w in shapes:
        outs.setdefault(w.shape[0], torch.empty(STREAMS, w.shape[0], device=dev))

    def run(i):
        w = shapes[i % len(shapes)]
        hi, lo = acts[w.shape[1]]
        ops.gemm(hi, w, _lib.EPI_F32, out=outs[w.shape[0]], x_lo=lo)

    for i in range(4):
        run(i)
    torch.cuda.synchronize()
    sec = _replay_timed(run, len(shapes))
    algo = sum(w.shape[0] * w.shape[1] * 2 + STREAMS * w.shape[1] * 4 + STREAMS * w.shape[0] * 4
               for w in shapes) / len(shapes)
    gbs = algo / sec / 1e9
    peak = peaks.get("hbm_gbs")
    return {"kernel": "gemm_tc_kernel<64,3,hi/lo> (talker QKV/O/gate-up/down, M = 64)", "bound": "hbm",
            "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 3) if peak else None,
            "traffic": int(algo * GEMM_TRAFFIC_RATIO),
            "traffic_source": "ncu dram__bytes_read+write per launch over algorithmic bytes, scaled to this launch",
            "algorithmic_bytes_per_launch": int(algo), "launches": len(shapes),
            "launch_us": round(sec * 1e6, 2), "talker_projections_ms": round(sec * len(shapes) * 1e3, 3),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ----------------------------------------------------------------------------- CPU baseline
class CpuStep:
    """The oracle (fp32 CPU restatement of the reference's talker, sampling head, code
    predictor with its full per-stage recompute, codec sum and streaming code2wav) set up on
    the benchmark's streams: their cfg2 context lengths, KV of random values (the values do not
    change the work), all host threads.  ``step(n)`` runs one decode step of the first n
    streams, code2wav included, and returns its seconds."""

    def __init__(self):
        from oracle.engine import OracleEngine
        from oracle import code2wav as OC
        from test_stateful_b200 import weights as wmod, workload
        from test_stateful_b200.config import EngineConfig
        torch.set_num_threads(host_threads())
        cfg = EngineConfig()
        t, c = cfg.talker, cfg.cp
        W = wmod.make_talker_weights(t, SEED, dtype=torch.float32)
        W.update(wmod.make_cp_weights(c, SEED, dtype=torch.float32))
        self.Wc = wmod.make_code2wav_weights(cfg.c2w, SEED, dtype=torch.float32)
        self.cfg, self.OC = cfg, OC
        self.eng = OracleEngine(W, t, c)
        g = torch.Generator().manual_seed(0)
        lengths = [len(p) for p in workload.shared_prefix_prompts(STREAMS, 16, 512, PREFIX, SEED)]
        for i, n in enumerate(lengths):
            self.eng.k[i] = [torch.randn(t.kv_heads, n, t.head_dim, generator=g) * 0.5 for _ in range(t.num_layers)]
            self.eng.v[i] = [torch.randn(t.kv_heads, n, t.head_dim, generator=g) * 0.5 for _ in range(t.num_layers)]
            self.eng.past[i] = n
        self.c2w_state = [OC.Code2WavState(cfg.c2w) for _ in range(STREAMS)]
        self.x = torch.randn(STREAMS, t.hidden_size, generator=g) * 0.02
        self.counts = torch.zeros(STREAMS, t.codec_vocab_size, dtype=torch.long)
        self.g = g
        self.lengths = lengths

    def step(self, n: int) -> float:
        from oracle import model as M
        c = self.cfg.cp
        t0 = time.perf_counter()
        gum = M.gumbel_from_uniform(torch.rand(n, 50, generator=self.g))
        cgum = M.gumbel_from_uniform(torch.rand(n, c.num_stages, 50, generator=self.g))
        r = self.eng.decode(list(range(n)), self.x[:n], self.counts[:n], gum, cgum, torch.full((n, 1), 0.9),
                            torch.full((n, 1), 1.05))
        for i in range(n):
            self.OC.decode_chunk(self.Wc, self.cfg.c2w, r["full_codec"][i].view(-1, 1), self.c2w_state[i])
        self.x[:n] = r["codec_sum"]
        self.counts[:n] = r["counts"]
        return time.perf_counter() - t0


def cpu_baseline_rate(n_streams=STREAMS, steps=6, warmup=1):
    """``cpu_baseline`` of the GPU arm: ``steps`` timed decode steps of the oracle over the
    benchmark's first ``n_streams`` streams (about 15-30 s of CPU work at the default)."""
    cs = CpuStep()
    for _ in range(warmup):
        cs.step(n_streams)
    dt = sum(cs.step(n_streams) for _ in range(steps))
    return {"value": round(n_streams * steps / dt, 3), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{steps} decode steps of the benchmark's first {n_streams} streams (cfg2 contexts, "
                      f"{sum(cs.lengths[:n_streams]) / n_streams:.0f} mean), full 28-layer talker + 15-stage code "
                      f"predictor (the reference's full recompute) + streaming code2wav, fp32, "
                      f"{torch.get_num_threads()} threads",
            "seconds": round(dt, 2)}


# ----------------------------------------------------------------------------- main arms
def run_reference(rank, world):
    """The reference arm: the oracle port of the reference's CPU path on this box's host cores,
    same workload and config as the GPU arm.  Each of the arm's --warmup + --steps steps is one
    decode step (code2wav included) of the first n of the 64 streams, n chosen after the first
    warm-up step so the whole arm ends in about ``budget`` seconds; frames/s = n * steps / time."""
    if rank != 0:
        return
    budget = 150.0
    cs = CpuStep()
    probe_n = 8
    t_probe = cs.step(probe_n)  # counts as the first warm-up step
    per_step = budget / max(1, ARGS.steps + ARGS.warmup)
    n = max(1, min(STREAMS, int(per_step / (t_probe / probe_n))))
    for _ in range(max(0, ARGS.warmup - 1)):
        cs.step(n)
    dt = sum(cs.step(n) for _ in range(ARGS.steps))
    value = n * ARGS.steps / dt
    base = {"value": round(value, 3), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{ARGS.steps} decode steps of the benchmark's first {n} of {STREAMS} streams (cfg2 contexts), "
                      f"full 28-layer talker + 15-stage code predictor (the reference's full recompute) + streaming "
                      f"code2wav, fp32, {torch.get_num_threads()} threads",
            "seconds": round(dt, 2)}
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": world,
            "steps": ARGS.steps, "warmup": ARGS.warmup, "ms_per_step": round(dt / ARGS.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(world), "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200(rank, world, local):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    ex, slots, prompts, pad = build_workload(dev)
    n = len(slots)
    stream = ex._stream
    peaks = load_peaks()

    if ARGS.roofline_only:
        torch.cuda.nvtx.range_push("roofline")  # for ncu --nvtx --nvtx-include roofline/
        roof = {"gemm": gemm_roofline(ex, peaks), "attention": attention_roofline(ex, slots, peaks)}
        torch.cuda.nvtx.range_pop()
        if rank == 0:
            print(json.dumps({"roofline_only": True, **roof}), flush=True)
        ex._graphs.clear()
        ex.shutdown()
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    # warm-up: eager step, capture, replays
    for _ in range(max(1, ARGS.warmup)):
        ex.launch_decode_step(slots).wait()
        ex.advance(slots)
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
        if world > 1:
            torch.distributed.destroy_process_group()
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
    def e2e_loop(steps):
        pending = None
        for _ in range(steps):
            with torch.cuda.stream(stream):
                staged.copy_(t_host, non_blocking=True)
                ex.text_add.index_copy_(0, idx, staged)
            fut = ex.launch_decode_step(slots)
            ex.advance(slots)  # the loop's per-slot counters, before the next launch
            if pending is not None:
                out = pending.wait()
                _ = out.full_codec, out.audio_chunks
            pending = fut
        out = pending.wait()
        _ = out.full_codec, out.audio_chunks

    # untimed warm-up of this path (its first use loads the copy and index kernels' modules,
    # ~20 ms once, which would otherwise be charged to the timed steps)
    e2e_loop(E2E_WARMUP)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    e2e_loop(ARGS.e2e_steps)
    torch.cuda.synchronize(dev)
    e2e_sec = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_sec], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_sec = float(t.item())
    e2e_value = n * ARGS.e2e_steps * world / e2e_sec
    h2d = t_host.numel() * 4 + n * 4
    d2h = n * (1 + ex._config.cp.num_stages) * 8 + 4 + n * ex._config.c2w.samples_per_frame * 4

    roof_gemm = gemm_roofline(ex, peaks)
    roof_attn = attention_roofline(ex, slots, peaks)
    ctx_now = [s.past_len for s in slots]
    ex._graphs.clear()
    ex.shutdown()
    if world > 1:
        # every rank is done with the GPU and with collectives before rank 0 spends host time
        # on the CPU baseline: no rank waits in a collective meanwhile
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    cpu = None if ARGS.no_cpu_baseline else cpu_baseline_rate()
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": ARGS.steps,
        "warmup": ARGS.warmup, "ms_per_step": round(total_ms / ARGS.steps, 4),
        "p50_step_ms": round(statistics.median(per_step), 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(world),
        "ctx_mean_end": round(sum(ctx_now) / len(ctx_now), 1),
        "pipeline": "two streams: step k's code2wav overlaps step k+1's talker + code predictor; "
                    "timed from step 0's start to the last step's code2wav end",
        "gpu_launches": launches * ARGS.steps,
        "roofline": roof_gemm,
        "roofline_attention": roof_attn,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": ARGS.e2e_steps, "warmup": E2E_WARMUP,
                "path": "B200Executor.launch_decode_step -> GPUFuture.wait",
                "lookahead": "step k+1 launched before step k's results are read"},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


CFG5_PER_GPU = 128          # requests (streams) per GPU
CFG5_RATE_PER_GPU = 25.0    # requests/s per GPU: 200 req/s over 8 GPUs
CFG5_SEED = 5


def run_cfg5(rank, world, local):
    """BASELINE configs[4] on this box's GPUs: the whole-box request stream (128 x world
    requests at 25 x world req/s, prompts U{8..128} ids, 25-250 frames, 30 % opening with one of
    8 shared 96-id prefixes) is routed once (``ReplicaRouter``: least-loaded, prefix affinity)
    and every rank serves its share with ``serve_replica`` (chunked prefill interleaved with
    decode; talker, code predictor, sampling and code2wav per step).  Wall-clock timing: the
    run is paced by the arrivals, so the device is idle between them by design."""
    from test_stateful_b200 import workload
    from test_stateful_b200.config import EngineConfig
    from test_stateful_b200.runtime.executor import B200Executor
    from test_stateful_b200.runtime.replicas import max_over_ranks, share_routing
    from test_stateful_b200.runtime.serving_loop import cfg5_requests, percentile, prefix_key, serve_replica

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    reqs, prefixes = cfg5_requests(CFG5_PER_GPU * world, CFG5_RATE_PER_GPU * world, CFG5_SEED)
    mine_sessions, _ = share_routing([(r.rid, prefix_key(r)) for r in reqs], rank, world, CFG5_PER_GPU)
    mine_ids = {sid for sid, _key in mine_sessions}
    mine = [r for r in reqs if r.rid in mine_ids]
    cfg = EngineConfig()
    ex = B200Executor(device_id=local, max_batch_size=CFG5_PER_GPU, max_seq_len=512, model_config=cfg,
                      do_sample=True, temperature=0.9, random_seed=CFG5_SEED + rank, num_blocks=ARGS.num_blocks,
                      weight_seed=SEED)
    ex.load()
    t = cfg.talker
    table = workload.text_table(t.hidden_size, SEED, device=dev)
    pad = workload.tts_pad_embed(t.hidden_size, SEED, device=dev)
    ex.warmup()
    t_cap = time.perf_counter()
    ex.capture_graphs(range(1, CFG5_PER_GPU + 1))
    t_cap = time.perf_counter() - t_cap
    if world > 1:
        torch.distributed.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    st = serve_replica(ex, mine, prefixes, table, pad, prefill_chunk=64)
    clk = clocks.stop()
    wall = max_over_ranks(st.wall_s, world, device=dev)
    frames = st.frames
    if world > 1:
        tot = torch.tensor([float(frames), float(st.completed)], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(tot)
        frames, completed = int(tot[0].item()), int(tot[1].item())
    else:
        completed = st.completed
    ex._graphs.clear()
    ex.shutdown()
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    value = frames / wall
    line = {
        "metric": "codec frames/s, whole-box serving (cfg5): Poisson arrivals, chunked prefill interleaved with "
                  "decode, talker + code predictor + sampling + code2wav per step",
        "value": round(value, 1), "unit": UNIT, "n_gpus": world, "per_gpu": round(value / world, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Poisson arrivals and random prompt ids; random-init weights)",
        "config": {"workload": "cfg5: 128 requests/GPU at 25 req/s/GPU (200 req/s on 8 GPUs), prompts U{8..128} "
                               "ids, 25-250 frames (2-20 s), 30% open with one of 8 shared 96-id prefixes",
                   "requests": len(reqs), "parallelism": f"replicas x{world} (ReplicaRouter: least-loaded, "
                                                          "prefix affinity; no collective)",
                   "prefill_chunk": 64, "graphs_captured": f"batch sizes 1..{CFG5_PER_GPU} ({t_cap:.1f} s)"},
        "wall_s": round(wall, 3), "frames": frames, "completed": completed,
        "rank0": {"requests": len(mine), "frames": st.frames, "decode_steps": st.decode_steps,
                  "max_running": st.max_running, "prefill_calls": st.prefill_calls,
                  "prefix_hits": st.prefix_hits, "prefix_misses": st.prefix_misses,
                  "ttfa_ms_p50": round(1e3 * percentile(st.ttfa_s, 50), 2),
                  "ttfa_ms_p90": round(1e3 * percentile(st.ttfa_s, 90), 2),
                  "step_ms_p50": round(1e3 * percentile(st.step_s, 50), 3) if st.step_s else None,
                  "step_ms_p90": round(1e3 * percentile(st.step_s, 90), 3) if st.step_s else None,
                  "audio_s_per_wall_s": round(st.frames / 12.5 / st.wall_s, 1)},
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def main():
    global ARGS
    ARGS = parse()
    rank, world, local = dist_env()
    if ARGS.impl == "reference":
        run_reference(rank, world)
        return
    if ARGS.workload == "cfg5":
        run_cfg5(rank, world, local)
        return
    run_b200(rank, world, local)


if __name__ == "__main__":
    main()
