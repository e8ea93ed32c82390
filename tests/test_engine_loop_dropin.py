"""The reference's own engine loop, unmodified, driving this backend's host layer (CPU).

``EngineLoop`` (engine/backend/engine_loop.py:184-2561) is imported from the
reference checkout together with its ``PrefixKVCache``, ``MLFQScheduler`` and
request/result types, and runs in its own thread exactly as ``TTSEngine``
starts it (engine/server.py:289-306).  It drives a ``B200Executor`` whose host
logic is the product's — the ``PagedKVCachePool`` with its paged
``_talker_kv_pool`` view and block-reference handles, slot bookkeeping,
``prefill`` / ``prefill_prefix_only`` / ``launch_decode_step`` /
``GPUFuture.wait`` / ``StepOutput`` — and whose device actions (the engine step,
code2wav, state writes on CUDA streams) are replaced by a CPU stand-in built
here: a deterministic toy model on small tensors, with the paged allocator
played by ``oracle.paged_state``.  The device kernels behind those actions are
tested on the GPU against the oracle elsewhere; this file tests the boundary.

Scenario (the reference test harness's pattern, tests/unit/test_engine_loop_pipeline.py):
three sessions arrive before the loop starts — two with the same voice (the
first misses the prefix cache and takes the split prefix-only prefill, the
second hits it and restores the prefix by block reference), one without a
cacheable prefix (full prefill) — and each streams audio until the toy model
emits EOS.  Checked: every session ends with SESSION_DONE after its audio
chunks; the hit shares the miss's prefix blocks; each decode step's input row is
what the loop computed (codec sum of the previous frame + the next trailing
text row, then tts_pad); newly primed streams get their sampling state set on
their first decode step; all blocks return to the free stack once the cache is
cleared.
"""

import queue
import sys
import time
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle.paged_state import PagedState
from test_stateful_b200.config import PagedPoolConfig, tiny_engine_config
from test_stateful_b200.runtime.executor import B200Executor
from test_stateful_b200.runtime.pool import PagedKVCachePool

from .conftest import reference_root

REF = reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="reference checkout not available")

FRAMES = 6          # the toy model emits EOS on the 6th decode frame of a stream
VOICE_LEN = 20      # cacheable voice prefix: one full 16-token block + a partial one


class _OracleSched:
    """The paged allocator played by the CPU restatement (block tables, refcounts, COW)."""

    def __init__(self, cfg):
        p = cfg.pool
        self.st = PagedState(p.num_blocks, p.block_size, p.max_slots, p.max_blocks_per_seq)
        self.status = torch.zeros(1, dtype=torch.int32)
        self.log = []

    def make_entry(self, slot, n):
        blocks = self.st.make_entry(slot, n)
        self.log.append(("make_entry", slot, n, list(blocks)))
        return torch.tensor(blocks, dtype=torch.int32)

    def share_prefix(self, slot, blocks, n):
        self.log.append(("share_prefix", slot, blocks.tolist(), n))
        self.status[0] = self.st.share_prefix(slot, blocks.tolist(), n)

    def drop_blocks(self, blocks):
        self.st.drop_entry(blocks.tolist())

    def release(self, slot):
        self.st.release(slot)


class _CpuStandInExecutor(B200Executor):
    """``B200Executor`` with its device actions replaced by a deterministic toy model on CPU
    tensors; every host-side method the engine loop calls is the product's."""

    def __init__(self, cfg, monkeypatch, max_batch=4, max_seq_len=128):
        # the product constructor requires a CUDA device; set the same fields on the CPU
        self._device = torch.device("cpu")
        self._config = cfg
        cfg.pool = PagedPoolConfig(block_size=16, num_blocks=48, max_slots=max_batch, max_seq_len=max_seq_len)
        self._max_batch, self._max_seq_len, self._max_input_len = max_batch, max_seq_len, 256
        self._do_sample, self._temperature, self._repetition_penalty, self._random_seed = True, 0.9, 1.05, 7
        self._weights = self._c2w_weights = None
        # a decoder stands in so the futures carry audio; its work happens in _enqueue_step
        self._use_graphs, self._enable_c2w = False, True
        self._c2w = SimpleNamespace(close=lambda: None)
        self._stream = self._c2w_stream = None
        self._model, self._graphs, self._embedding_weights = None, {}, None
        self._parity, self._done_a, self._done_b = 0, [None, None], [None, None]
        monkeypatch.setattr(torch.Tensor, "pin_memory", lambda t: t)  # no pinned memory without a GPU
        self._alloc_state()
        t = cfg.talker
        fake_model = SimpleNamespace(cfg=cfg, pool=SimpleNamespace(free_stack=torch.zeros(1, dtype=torch.int32),
                                                                   free_top=torch.zeros(1, dtype=torch.int32),
                                                                   kv=torch.zeros(1)))
        self._kv_pool = PagedKVCachePool(fake_model, max_batch)
        self._kv_pool._sched = _OracleSched(cfg)
        self._kv_pool.counts_reset_hook = self._reset_slot_state
        g = torch.Generator().manual_seed(3)
        self.codec_table = (torch.randn(2048, t.hidden_size, generator=g) * 0.05).to(torch.bfloat16).float()
        self.steps = []        # (session, frame, input row, code0)
        self.fresh_log = []    # (session, frame) of streams started by _stage_host_inputs
        self.moved_log = []
        self.cow = []

    # -- toy model ---------------------------------------------------------------
    def _frame(self, slot, x):
        f = slot.frame_idx
        code0 = self._config.talker.codec_eos_id if f >= FRAMES - 1 else int(x.abs().sum() * 1e3) % 2000
        codes = torch.full((16,), 7, dtype=torch.int64)
        codes[0] = code0
        return codes

    def _emit(self, par, row, slot, x):
        codes = self._frame(slot, x)
        sid = slot.slot_id
        self.codes_buf[par][row] = codes
        self.codes_host_buf[par][row] = codes
        cs = self.codec_table[int(codes[0]) % 2048]
        self.codec_sum_buf[par][sid] = cs
        self.next_x[sid] = cs + self.text_add[sid]
        self.counts[sid, int(codes[0])] += 1
        self.wav_host_buf[par][row] = 0.1 * torch.sin(torch.arange(self.wav_host_buf.shape[-1]) * 0.05 + sid)
        self.steps.append((slot.session_id, slot.frame_idx, x.clone(), int(codes[0])))

    # -- device actions --------------------------------------------------------
    def _write_sampling_state(self, sid, seed):
        self.noise_key[sid] = seed
        self.noise_step[sid] = 0
        self.temperature[sid] = self._temperature
        self.penalty[sid] = self._repetition_penalty

    def _reset_slot_state(self, slot_id):
        self.counts[slot_id].zero_()

    def set_text_embedding(self, slot, emb):
        self.text_add[slot.slot_id] = 0 if emb is None else emb.reshape(-1).float()

    def _prefill_call(self, slot, embeds, sample):
        seq = int(embeds.shape[-2]) if embeds.dim() == 3 else int(embeds.shape[0])
        st = self._kv_pool._sched.st
        rc, _, cow = st.append([slot.slot_id], seq)
        assert rc == 0
        self.cow += [(slot.session_id, c) for c in cow]
        if sample:
            self._emit(2, 0, slot, embeds.reshape(seq, -1)[-1].float())
        slot.past_len += seq

    def _first_frame_audio(self, slot):
        return self.wav_host_buf[2][0].numpy().tobytes()

    def _apply_host_inputs(self, moved, fresh):
        for s in moved:
            self.next_x[s.slot_id] = s.next_embed.reshape(-1).float()
        self.moved_log += [(s.session_id, s.frame_idx) for s in moved]
        self.fresh_log += [(s.session_id, s.frame_idx) for s in fresh]

    def _enqueue_step(self, n, upload, graphs=None):
        par = self._parity
        self._parity ^= 1
        ids = self.slots_host_buf[par][:n].tolist()
        slots = [self._kv_pool.get(i) for i in ids]
        for s in slots:  # the batch append is sequential in batch order; per slot to attribute copies
            rc, _, cow = self._kv_pool._sched.st.append([s.slot_id], 1)
            assert rc == 0
            self.cow += [(s.session_id, c) for c in cow]
        for row, s in enumerate(slots):
            self._emit(par, row, s, self.next_x[s.slot_id].clone())
            self.noise_step[s.slot_id] += 1
        self.status_host_buf[par].zero_()
        return par, None, None


class _Builder:
    """Prompt plans from token ids (the reference test harness's stub idea): voice ``v`` is a
    fixed 20-row prefix; the text rows come from a table; speaker "nocache" has no cacheable
    prefix and is prefilled whole."""

    def __init__(self, H):
        g = torch.Generator().manual_seed(11)
        self.table = (torch.randn(64, H, generator=g) * 0.05).to(torch.bfloat16)
        self.eos = (torch.randn(1, 1, H, generator=g) * 0.05).to(torch.bfloat16)
        self.w = SimpleNamespace(tts_pad_embed=(torch.randn(1, 1, H, generator=g) * 0.05).to(torch.bfloat16))
        self.voices = {}

    def _voice(self, speaker):
        if speaker not in self.voices:
            g = torch.Generator().manual_seed(len(self.voices) + 100)
            self.voices[speaker] = (torch.randn(1, VOICE_LEN, self.table.shape[1], generator=g) * 0.05).to(
                torch.bfloat16)
        return self.voices[speaker]

    def compute_cache_key(self, task_type, language, speaker, *args, **kwargs):
        return None if speaker == "nocache" else f"voice:{speaker}"

    def _trailing(self, token_ids, include_eos):
        rows = [self.table[t].view(1, 1, -1) for t in token_ids[1:]]
        return rows + ([self.eos] if include_eos else [])

    def build_plan_from_ids(self, *, token_ids, speaker=None, include_eos=True, **kwargs):
        from engine.backend.prefill import PrefillPlan
        voice = self._voice(speaker)
        first = self.table[token_ids[0]].view(1, 1, -1)
        full = torch.cat([voice, first], dim=1)
        if speaker == "nocache":
            return PrefillPlan(prefill_embeds=full, trailing=self._trailing(token_ids, include_eos))
        return PrefillPlan(prefill_embeds=full, trailing=self._trailing(token_ids, include_eos),
                           prefix_cache_key=f"voice:{speaker}", cacheable_prefix_embeds=voice.clone(),
                           request_prefill_embeds=first.clone())

    def build_suffix_from_ids(self, token_ids, include_eos=True):
        return self.table[token_ids[0]].view(1, 1, -1), self._trailing(token_ids, include_eos)


class _ImmediateLoop:
    def call_soon_threadsafe(self, callback, *args):
        callback(*args)


def test_reference_engine_loop_drives_the_b200_host_layer(monkeypatch):
    # after this repository's own packages (the reference has a ``tests`` package too), and only
    # for the duration of this test
    monkeypatch.setattr(sys, "path", sys.path + [str(REF)])
    from engine.backend.engine_loop import EngineLoop
    from engine.core.types import EngineRequest, RequestType, ResultType

    cfg = tiny_engine_config(num_layers=2)
    ex = _CpuStandInExecutor(cfg, monkeypatch)
    builder = _Builder(cfg.talker.hidden_size)
    loop = EngineLoop(engine_inbox=queue.Queue(), async_loop=_ImmediateLoop(), executor=ex,
                      prefill_builder=builder, max_batch_size=4, prefix_cache_max_entries=4)
    sessions = {"miss": ("A", [5, 6, 7, 8]), "hit": ("A", [9, 10, 11]), "full": ("nocache", [12, 13])}
    results = {k: queue.Queue() for k in sessions}
    for sid, (speaker, tokens) in sessions.items():
        for req in (EngineRequest(type=RequestType.NEW_SESSION, session_id=sid, speaker_key=speaker,
                                  task_type="custom_voice", result_queue=results[sid]),
                    EngineRequest(type=RequestType.START_TOKENS, session_id=sid, segment_idx=0, token_ids=tokens),
                    EngineRequest(type=RequestType.SEGMENT_TOKENS_DONE, session_id=sid, segment_idx=0),
                    EngineRequest(type=RequestType.SESSION_TOKENS_DONE, session_id=sid)):
            loop._inbox.put(req)
    got = {k: [] for k in sessions}
    loop.start()
    try:
        deadline = time.monotonic() + 30
        while time.monotonic() < deadline and not all(
                any(r.type == ResultType.SESSION_DONE for r in got[k]) for k in sessions):
            for k, q in results.items():
                while not q.empty():
                    got[k].append(q.get_nowait())
            time.sleep(0.01)
    finally:
        loop.stop()
    for k in sessions:
        types = [r.type for r in got[k]]
        assert ResultType.ERROR not in types, (k, [r.error_msg for r in got[k] if r.type == ResultType.ERROR])
        assert types[-1] == ResultType.SESSION_DONE, (k, types)
        chunks = [r.audio_bytes for r in got[k] if r.type == ResultType.AUDIO_CHUNK]
        # split prefills stream FRAMES decode frames; the full prefill adds its first frame
        assert len(chunks) >= FRAMES - 1 and all(len(c) == cfg.c2w.samples_per_frame * 4 for c in chunks), k

    sched = ex._kv_pool._sched
    # one prefix-only prefill (the miss) cached by reference; the hit shared those blocks
    makes = [e for e in sched.log if e[0] == "make_entry"]
    shares = [e for e in sched.log if e[0] == "share_prefix"]
    assert [m[2] for m in makes] == [VOICE_LEN] and len(shares) == 1 and shares[0][3] == VOICE_LEN
    assert shares[0][2] == makes[0][3]  # the hit points its slot at the blocks the miss cached
    # the partial prefix block is copied on the first write of each stream that shares it
    assert {s for s, _ in ex.cow} >= {"miss:0", "hit:0"}
    # streams primed by the loop (prefix-only prefill, cache hit) start on their first decode step
    assert sorted(ex.fresh_log) == [("hit:0", 0), ("miss:0", 0)]
    # every decode input is the loop's: first text row, then codec sum of the previous frame +
    # the next trailing row, then tts_pad once the text is used up
    pad = builder.w.tts_pad_embed.reshape(-1).float()
    for k, (speaker, tokens) in sessions.items():
        rows = [(f, x, c) for s, f, x, c in ex.steps if s == f"{k}:0"]
        trailing = [t.reshape(-1).float() for t in builder._trailing(tokens, True)]
        prev = None
        for f, x, code0 in rows:
            if prev is None:
                if k != "full":
                    torch.testing.assert_close(x, builder.table[tokens[0]].float())
            else:
                want_text = trailing[f - 1] if f - 1 < len(trailing) else pad
                torch.testing.assert_close(x, ex.codec_table[prev % 2048] + want_text)
            prev = code0
        assert rows[-1][2] == cfg.talker.codec_eos_id and rows[-1][0] == FRAMES - 1
    # the batch inputs the loop set were all taken from its slots
    assert len(ex.moved_log) == sum(1 for s, f, _, _ in ex.steps if not (s == "full:0" and f == 0))
    # every slot is back; once the loop's prefix cache lets go, every block is free again
    assert ex._kv_pool.free_count == 4
    loop._prefix_cache.clear()
    ex._kv_pool.flush_drops()
    assert sched.st.free_top == cfg.pool.num_blocks and int(np.abs(sched.st.refcount).sum()) == 0
