"""The serving loop on the B200 (tiny config): Poisson arrivals faster than the replica
drains them, chunked prefill interleaved with decode, shared prefixes served from the prefix
cache.  Every request produces its frames, the pool's slots and KV blocks all come back
afterwards (no leaked reference), and the per-batch-size CUDA graphs captured ahead of time
are the ones the steps replay."""

import pytest
import torch

pytestmark = pytest.mark.gpu

from test_stateful_b200 import weights as wmod, workload  # noqa: E402
from test_stateful_b200.config import tiny_engine_config  # noqa: E402
from test_stateful_b200.runtime.executor import B200Executor  # noqa: E402
from test_stateful_b200.runtime.serving_loop import cfg5_requests, serve_replica  # noqa: E402


def test_serving_loop_completes_and_returns_every_block():
    cfg = tiny_engine_config()
    W = wmod.make_talker_weights(cfg.talker, 4)
    W.update(wmod.make_cp_weights(cfg.cp, 4))
    Wc = wmod.make_code2wav_weights(cfg.c2w, 4)
    ex = B200Executor(max_batch_size=6, max_seq_len=160, model_config=cfg, do_sample=True, temperature=0.9,
                      random_seed=3, num_blocks=96, weights=W, c2w_weights=Wc, max_prefill_rows=64)
    ex.load()
    try:
        pool = ex.kv_pool
        free0 = pool.free_blocks
        reqs, prefixes = cfg5_requests(14, 300.0, 11, prefix_len=32, n_prefixes=2, share=0.4, lo=8, hi=70,
                                       fmin=2, fmax=14)
        hidden = cfg.talker.hidden_size
        table = workload.text_table(hidden, 4, device="cuda")
        pad = workload.tts_pad_embed(hidden, 4, device="cuda")
        ex.capture_graphs(range(1, 7))
        graphs = {n: ex._graphs[n] for n in range(1, 7)}
        st = serve_replica(ex, reqs, prefixes, table, pad, prefill_chunk=24)
        assert st.completed == len(reqs)
        assert st.frames == sum(r.frames for r in reqs)
        assert st.prefix_hits + st.prefix_misses == sum(r.prefix is not None for r in reqs)
        assert st.prefix_misses >= 1 and st.max_running >= 2
        assert all(ex._graphs[n] is graphs[n] for n in graphs)  # no capture during the run
        assert pool.free_count == 6
        pool.flush_drops()
        assert pool.free_blocks == free0  # every stream's and every cached prefix's blocks are back
        print(f"serving: {st.completed} requests, {st.frames} frames, {st.decode_steps} steps, "
              f"max running {st.max_running}, prefix hits {st.prefix_hits}/{st.prefix_hits + st.prefix_misses}")
    finally:
        ex._graphs.clear()
        ex.shutdown()
