"""Pin the code2wav oracle against the reference's own streaming wrapper.

``tests/golden/code2wav_tiny.npz`` was written by ``make_golden.py`` running
``Code2WavStreamingWrapper`` (scripts/export/code2wav_streaming.py:595-856)
batched at T=1 the way the fused step drives it: two slots that start 9
steps apart (ragged past lengths, -inf bias on the left padding), 78 steps so
the first slot's KV window (72) wraps, per-slot conv/transconv state carried
between steps.
"""

import os

import numpy as np
import torch

from oracle import code2wav as C
from test_stateful_b200 import weights as wmod
from test_stateful_b200.config import Code2WavConfig, tiny_code2wav_config

from .conftest import GOLDEN


def test_code2wav_oracle_matches_reference_stream():
    z = np.load(os.path.join(GOLDEN, "code2wav_tiny.npz"))
    cfg = tiny_code2wav_config()
    W = wmod.to_fp32(wmod.make_code2wav_weights(cfg, int(z["seed"])))
    codes, active, wav = z["codes"], z["active"], z["wav"]
    assert wav.shape[-1] == cfg.samples_per_frame == 1920
    for s in range(codes.shape[1]):
        st = C.Code2WavState(cfg)
        n = 0
        for t in range(codes.shape[0]):
            if not active[t, s]:
                continue
            w = C.decode_chunk(W, cfg, torch.from_numpy(codes[t, s]).view(-1, 1), st).numpy()
            np.testing.assert_allclose(w, wav[t, s], rtol=0, atol=2e-5)
            n += 1
        assert n == int(active[:, s].sum())
        if n > cfg.window:
            assert st.kv[0][0].shape[2] == cfg.window - 1  # the window wrapped


def test_code2wav_chunk_equals_frames():
    """A T-frame chunk through the oracle equals T single-frame steps (the
    chunked cfg4 path and the T=1 fused path produce the same waveform)."""
    cfg = tiny_code2wav_config()
    W = wmod.to_fp32(wmod.make_code2wav_weights(cfg, 3))
    g = torch.Generator().manual_seed(0)
    codes = torch.randint(0, cfg.codebook_size, (cfg.num_codebooks, 6), generator=g)
    a, b = C.Code2WavState(cfg), C.Code2WavState(cfg)
    chunk = C.decode_chunk(W, cfg, codes, a)
    frames = torch.cat([C.decode_chunk(W, cfg, codes[:, t:t + 1], b) for t in range(6)])
    torch.testing.assert_close(chunk, frames, rtol=0, atol=2e-5)


def test_code2wav_state_shapes_match_reference_layout():
    """17 conv + 4 transconv states with the shapes of get_initial_state_shapes
    (code2wav_streaming.py:159-193) at the full configuration."""
    cfg = Code2WavConfig()
    st = C.Code2WavState(cfg)
    conv = [tuple(t.shape[1:]) for t in st.conv]
    assert conv[:4] == [(512, 2), (1024, 6), (1024, 6), (1024, 6)]
    assert conv[4:7] == [(768, 6), (768, 18), (768, 54)]
    assert conv[13:16] == [(96, 6), (96, 18), (96, 54)]
    assert conv[16] == (96, 6)
    assert [tuple(t.shape[1:]) for t in st.trans] == [(768, 8), (384, 5), (192, 4), (96, 3)]
    assert cfg.samples_per_frame == 1920


def test_code2wav_oracle_matches_reference_chunked_stream():
    """Chunked semantics: chunks of T frames (here 25, 25, 25, 7) with carried state;
    each chunk sees at most window - T past frames plus its own frames causally.  Fixture
    from the reference wrapper, two slots with ragged pasts (wav stored as fp16)."""
    z = np.load(os.path.join(GOLDEN, "code2wav_chunked_tiny.npz"))
    cfg = tiny_code2wav_config()
    W = wmod.to_fp32(wmod.make_code2wav_weights(cfg, int(z["seed"])))
    codes, chunks, start1 = z["codes"], z["chunks"].tolist(), int(z["start1"])
    for s_, ref in ((0, z["wav0"]), (1, z["wav1"])):
        st = C.Code2WavState(cfg)
        f, out = 0, []
        for call, T in enumerate(chunks):
            if s_ == 1 and call < start1:
                continue
            out.append(C.decode_chunk(W, cfg, torch.from_numpy(codes[s_, :, f:f + T]).long(), st).numpy())
            f += T
        got = np.concatenate(out)
        assert got.shape == ref.shape
        np.testing.assert_allclose(got, ref.astype(np.float32), rtol=0, atol=1.5e-3)


def _warm_fixture():
    z = np.load(os.path.join(GOLDEN, "code2wav_warm_tiny.npz"))
    conv = [torch.from_numpy(z[f"conv_{j}"]) for j in range(17)]
    trans = [torch.from_numpy(z[f"trans_{b}"]) for b in range(4)]
    return z, torch.from_numpy(z["kv"]), conv, trans, int(z["frame"])


def test_code2wav_oracle_continues_reference_warm_state():
    """``code2wav_warm_tiny.npz``: the wrapper's state after 80 frames (the warm state
    ``Executor.apply_c2w_warm_state`` receives) and the 10 frames it decodes next.  The oracle,
    started from that state, decodes the same 10 frames."""
    z, kv, conv, trans, frame = _warm_fixture()
    cfg = tiny_code2wav_config()
    W = wmod.to_fp32(wmod.make_code2wav_weights(cfg, int(z["seed"])))
    st = C.Code2WavState(cfg)
    st.kv = [(kv[:, 2 * l], kv[:, 2 * l + 1]) for l in range(cfg.num_layers)]
    st.conv = [x.clone() for x in conv]
    st.trans = [x.clone() for x in trans]
    st.frame = frame
    codes = z["codes"]
    for i in range(z["wav"].shape[0]):
        w = C.decode_chunk(W, cfg, torch.from_numpy(codes[frame + i]).view(-1, 1), st).numpy()
        np.testing.assert_allclose(w, z["wav"][i], rtol=0, atol=2e-5)


def test_warm_state_conversion_to_decoder_layout():
    """``warm_state_parts`` on the reference's warm state (CPU): every window frame lands at
    position frame % window of its (layer, k/v, head) row; conv contexts become rows, zero
    padded; each transposed conv's previous input row, recovered by least squares from the
    bias-free overlap tail, reproduces that tail through the fp32 weights."""
    from test_stateful_b200.runtime.code2wav import expected_state_layout, pack_code2wav, warm_state_parts

    z, kv, conv, trans, frame = _warm_fixture()
    cfg = tiny_code2wav_config()
    Wd = wmod.make_code2wav_weights(cfg, int(z["seed"]))
    W = wmod.to_fp32(Wd)
    P = pack_code2wav(cfg, Wd, "cpu")
    layout = expected_state_layout(cfg, 1)
    parts = warm_state_parts(cfg, P, layout, kv, conv, trans, frame, "cpu")
    assert [tuple(p.shape) for p in parts] == [(r, e) for r, e, _, _ in layout]
    L, H, Wn, D = cfg.num_layers, cfg.num_heads, cfg.window, cfg.head_dim
    ring = parts[0].float().view(2 * L, H, Wn, D)
    T = kv.shape[3]
    for i in (0, T // 2, T - 1):
        f = frame - T + i
        torch.testing.assert_close(ring[:, :, f % Wn], kv[0, :, :, i].to(torch.float16).float())
    assert float(ring[:, :, frame % Wn].abs().max()) == 0.0  # the next frame's position is still free
    for j in range(17):
        rows, row_elems, valid, _ = layout[1 + j]
        got = parts[1 + j].float()
        ref = conv[j][0].t()
        want = ref if parts[1 + j].dtype == torch.float32 else ref.to(torch.bfloat16).float()
        torch.testing.assert_close(got[:, :valid], want)
        if row_elems > valid:
            assert float(got[:, valid:].abs().max()) == 0.0
    for b, (cin, cout, s) in enumerate(cfg.block_dims()):
        x = parts[18 + b].float()[0, :cin]
        w = W[f"c2w.decoder.{1 + b}.transconv.weight"]  # [cin, cout, 2s]
        tail = torch.einsum("i,icp->cp", x, w[:, :, s:])
        ref = trans[b][0]
        rel = float((tail - ref).abs().max() / ref.abs().max())
        assert rel < 2e-2, (b, rel)  # bf16 packed weights, bf16 state row
