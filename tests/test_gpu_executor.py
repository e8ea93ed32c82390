"""The executor surface end to end on the B200: prefill -> decode steps
(eager, captured, replayed) with code2wav in the step; audio chunks checked
against the fp32 oracle decoding the same codec frames (SNR >= 30 dB)."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import code2wav as OC  # noqa: E402
from test_stateful_b200 import _lib, weights as wmod  # noqa: E402
from test_stateful_b200.config import tiny_engine_config  # noqa: E402
from test_stateful_b200.runtime.executor import B200Executor  # noqa: E402

DEV = "cuda"


def _snr(ref, out):
    ref = np.asarray(ref, np.float64)
    return 10 * np.log10((ref ** 2).sum() / max(((np.asarray(out, np.float64) - ref) ** 2).sum(), 1e-30))


def test_executor_decode_steps_emit_audio_matching_oracle():
    cfg = tiny_engine_config()
    W = wmod.make_talker_weights(cfg.talker, 3)
    W.update(wmod.make_cp_weights(cfg.cp, 3))
    Wc = wmod.make_code2wav_weights(cfg.c2w, 3)  # CPU generator: the values the oracle uses
    ex = B200Executor(max_batch_size=4, max_seq_len=96, model_config=cfg, do_sample=True, temperature=0.9,
                      random_seed=5, num_blocks=64, weights=W, c2w_weights=Wc, max_prefill_rows=64)
    ex.load()
    pool = ex.kv_pool
    g = torch.Generator().manual_seed(0)
    slots, frames, audio = [], [], []
    for i, n in enumerate((7, 12)):
        s = pool.allocate(f"s{i}")
        a, _ = ex.prefill(s, (torch.randn(1, n, cfg.talker.hidden_size, generator=g) * 0.02).to(DEV))
        slots.append(s)
        frames.append([ex.codes[0].cpu().clone()])
        audio.append([np.frombuffer(a, np.float32)])
    for _ in range(6):  # eager, capture, replays
        out = ex.launch_decode_step(slots).wait()
        ex.advance(slots)
        for i in range(len(slots)):
            frames[i].append(out.full_codec[i].clone())
            audio[i].append(np.frombuffer(out.audio_chunks[i], np.float32))
    assert _lib.device_error() == 0
    W = wmod.to_fp32(Wc)
    for i in range(len(slots)):
        st = OC.Code2WavState(cfg.c2w)
        ref = [OC.decode_chunk(W, cfg.c2w, f.view(-1, 1), st).numpy() for f in frames[i]]
        got = np.concatenate(audio[i])
        assert got.size == len(frames[i]) * cfg.c2w.samples_per_frame
        s = _snr(np.concatenate(ref), got)
        assert s >= 30.0, (i, s)
    assert ex.make_zero_conv_states() == [] and not ex.apply_c2w_warm_state(slots[0], None, None, None, 0)
    ex.shutdown()


def test_executor_lookahead_matches_sequential_steps():
    """Launching step k+1 before reading step k (code2wav of step k then overlaps step k+1's
    talker on the second stream, and the two steps use different buffer parities) gives the
    same codes and audio, bit for bit, as launching and waiting one step at a time."""
    cfg = tiny_engine_config()
    W = wmod.make_talker_weights(cfg.talker, 4)
    W.update(wmod.make_cp_weights(cfg.cp, 4))
    Wc = wmod.make_code2wav_weights(cfg.c2w, 4)

    def run(lookahead):
        ex = B200Executor(max_batch_size=4, max_seq_len=96, model_config=cfg, do_sample=True, temperature=0.9,
                          random_seed=7, num_blocks=64, weights=dict(W), c2w_weights=dict(Wc), max_prefill_rows=64)
        ex.load()
        g = torch.Generator().manual_seed(1)
        slots = []
        for i, n in enumerate((5, 9, 14)):
            s = ex.kv_pool.allocate(f"s{i}")
            ex.prefill(s, (torch.randn(1, n, cfg.talker.hidden_size, generator=g) * 0.02).to(DEV))
            slots.append(s)
        codes, audio = [], []
        pending = None
        for _ in range(8):  # eager, capture, replays
            fut = ex.launch_decode_step(slots)
            ex.advance(slots)
            if not lookahead:
                out = fut.wait()
                codes.append(out.full_codec.clone())
                audio.append(list(out.audio_chunks))
                continue
            if pending is not None:
                out = pending.wait()
                codes.append(out.full_codec.clone())
                audio.append(list(out.audio_chunks))
            pending = fut
        if lookahead:
            out = pending.wait()
            codes.append(out.full_codec.clone())
            audio.append(list(out.audio_chunks))
        assert _lib.device_error() == 0
        ex.shutdown()
        return codes, audio

    c_seq, a_seq = run(False)
    c_la, a_la = run(True)
    for k in range(len(c_seq)):
        assert torch.equal(c_seq[k], c_la[k]), k
        assert a_seq[k] == a_la[k], k


def test_chunked_prefill_interleaved_with_decode():
    """Chunked prefill (engine steps of 8 prompt tokens, only the last one sampling) gives the
    first frame of a single-shot prefill, and running its chunks between decode steps of other
    streams leaves those streams' codes and audio unchanged (greedy, so both runs are
    deterministic)."""
    cfg = tiny_engine_config()
    W = wmod.make_talker_weights(cfg.talker, 6)
    W.update(wmod.make_cp_weights(cfg.cp, 6))
    Wc = wmod.make_code2wav_weights(cfg.c2w, 6)
    g = torch.Generator().manual_seed(3)
    prompts = [(torch.randn(1, n, cfg.talker.hidden_size, generator=g) * 0.02) for n in (9, 13, 21)]

    def run(chunked):
        ex = B200Executor(max_batch_size=4, max_seq_len=96, model_config=cfg, do_sample=False, random_seed=2,
                          num_blocks=64, weights=dict(W), c2w_weights=dict(Wc), max_prefill_rows=64)
        ex.load()
        old = []
        for i, p in enumerate(prompts[:2]):
            s = ex.kv_pool.allocate(f"s{i}")
            ex.prefill(s, p.to(DEV))
            old.append(s)
        new = ex.kv_pool.allocate("new")
        outs = []
        if chunked:
            it = ex.iter_prefill(new, prompts[2].to(DEV), chunk=8)
            first = None
            for _ in range(3):  # 21 tokens: chunks of 8, 8, 5 between decode steps of the others
                out = ex.launch_decode_step(old).wait()
                ex.advance(old)
                outs.append((out.full_codec.clone(), list(out.audio_chunks)))
                first = next(it)
            assert first is not None
        else:
            for _ in range(3):
                out = ex.launch_decode_step(old).wait()
                ex.advance(old)
                outs.append((out.full_codec.clone(), list(out.audio_chunks)))
            first = ex.prefill(new, prompts[2].to(DEV))
        logits = ex.logits[0].float().cpu().clone()
        codes0 = ex.codes[0].cpu().clone()
        nxt = ex.launch_decode_step(old + [new]).wait()
        assert _lib.device_error() == 0
        ex.shutdown()
        return outs, first, logits, codes0, nxt

    o_seq, f_seq, l_seq, c_seq, n_seq = run(False)
    o_chk, f_chk, l_chk, c_chk, n_chk = run(True)
    for (ca, aa), (cb, ab) in zip(o_seq, o_chk):  # the running streams are untouched
        assert torch.equal(ca, cb)
        assert aa == ab
    rel = float((l_seq - l_chk).abs().max() / l_seq.abs().max())
    assert rel < 1e-3, rel  # split-K order differs with the chunk's row count
    assert torch.equal(c_seq, c_chk)
    assert f_seq[1] == f_chk[1]
    assert _snr(np.frombuffer(f_seq[0], np.float32), np.frombuffer(f_chk[0], np.float32)) >= 30.0
    assert torch.equal(n_seq.full_codec, n_chk.full_codec)
