"""Pin the CPU oracle against fixtures produced by the reference's own modules.

The fixtures were written by ``tests/golden/make_golden.py`` running
``TalkerUnifiedFusedONNX`` (scripts/export/talker_unified_modules.py:323-401),
``CodePredictorUnrolled`` (scripts/export/utils.py:852-1042),
``CodecEmbeddingSum`` (scripts/python/codec_embedding_sum.py:56-83) and the
reference ``KVCachePool``/``PrefixKVCache`` on the CPU.
"""

import os

import numpy as np
import pytest
import torch

from oracle import model as M
from oracle.engine import run_trajectory
from test_stateful_b200 import weights as wmod, workload
from test_stateful_b200.config import EngineConfig, tiny_engine_config

from .conftest import GOLDEN


def _weights(cfg, seed):
    W = wmod.make_talker_weights(cfg.talker, seed)
    W.update(wmod.make_cp_weights(cfg.cp, seed))
    return wmod.to_fp32(W)


def test_fused_tiny_single_call():
    z = np.load(os.path.join(GOLDEN, "fused_tiny.npz"))
    cfg = tiny_engine_config(int(z["num_layers"]))
    t, c = cfg.talker, cfg.cp
    W = _weights(cfg, int(z["seed"]))
    past = torch.from_numpy(z["past"])
    L = t.num_layers
    pk = [past[:, 2 * l] for l in range(L)]
    pv = [past[:, 2 * l + 1] for l in range(L)]
    lens = z["past_lens"].tolist()
    pos = torch.tensor(lens).unsqueeze(1)
    r = M.fused_step(W, t, c, torch.from_numpy(z["embeds"]), pos, pk, pv, lens,
                     torch.from_numpy(z["counts"]), torch.from_numpy(z["gumbel"]),
                     torch.from_numpy(z["cp_gumbel"]), torch.from_numpy(z["temperature"]),
                     torch.from_numpy(z["penalty"]))
    np.testing.assert_allclose(r["logits"].numpy(), z["out_logits"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(r["hidden"].numpy(), z["out_hidden"], rtol=1e-4, atol=1e-5)
    assert np.array_equal(r["full_codec"].numpy(), z["out_full_codec"])
    assert np.array_equal(r["counts"].numpy(), z["out_counts"])
    np.testing.assert_allclose(r["codec_sum"].numpy(), z["out_codec_sum"][:, 0], rtol=1e-5, atol=1e-6)
    delta = z["out_delta"]
    for l in range(L):
        np.testing.assert_allclose(r["new_k"][l].numpy(), delta[:, 2 * l], rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(r["new_v"][l].numpy(), delta[:, 2 * l + 1], rtol=1e-4, atol=1e-5)


def _traj_inputs(z, cfg):
    lengths = z["lengths"].tolist()
    seed = int(z["seed"])
    table = workload.text_table(cfg.talker.hidden_size, seed)
    pad = workload.tts_pad_embed(cfg.talker.hidden_size, seed)
    ids = workload.prompt_ids(lengths, seed)
    assert np.array_equal(np.concatenate([x.numpy() for x in ids]), z["prompt_ids"])
    return [table[x] for x in ids], pad


@pytest.mark.parametrize("name", ["traj_tiny_sampled.npz", "traj_tiny_greedy.npz"])
def test_tiny_trajectory(name):
    z = np.load(os.path.join(GOLDEN, name))
    cfg = tiny_engine_config(num_layers=2)
    W = _weights(cfg, int(z["seed"]))
    embeds, pad = _traj_inputs(z, cfg)
    steps = int(z["steps"])
    codes, logits = run_trajectory(W, cfg.talker, cfg.cp, embeds, steps, pad, z["gumbel"], z["cp_gumbel"],
                                   float(z["temperature"]), float(z["penalty"]))
    assert np.array_equal(codes, z["codes"])
    np.testing.assert_allclose(logits, z["step_logits"], rtol=1e-3, atol=1e-4)


@pytest.mark.slow
def test_cfg1_full_greedy():
    """The CPU reference case: full 28-layer talker, seed 0, fp32, 4 ragged prompts, 32 greedy steps."""
    path = os.path.join(GOLDEN, "cfg1_full_greedy.npz")
    if not os.path.exists(path):
        pytest.skip("cfg1 fixture not generated")
    z = np.load(path)
    cfg = EngineConfig()
    W = _weights(cfg, int(z["seed"]))
    embeds, pad = _traj_inputs(z, cfg)
    steps = int(z["steps"])
    B = len(embeds)
    gz = np.zeros((steps + 1, B, 50), np.float32)
    cgz = np.zeros((steps + 1, B, cfg.cp.num_stages, 50), np.float32)
    codes, logits = run_trajectory(W, cfg.talker, cfg.cp, embeds, steps, pad, gz, cgz,
                                   float(z["temperature"]), float(z["penalty"]))
    assert np.array_equal(codes, z["codes"])
    np.testing.assert_allclose(logits, z["step_logits"], rtol=2e-3, atol=2e-4)


def test_philox_restatement_known_answers():
    """oracle/noise.py's Philox4x32-10 against the published known-answer vectors of the
    generator (Random123 distribution, kat_vectors: philox4x32_10)."""
    from oracle import noise

    cases = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
             ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
             ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
              (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in cases:
        got = tuple(int(v) for v in noise.philox4x32_10(*ctr, *key))
        assert got == want
    # the transform: u in (0, 1), Gumbel = -log(-log(clamp(u, 1e-8, 1)))
    u = noise.uniform(7, [1, 2, 3], [0, 1, 2], 0, 64)
    assert u.min() > 0.0 and u.max() < 1.0
    g = noise.gumbel(7, [1, 2, 3], [0, 1, 2], 0, 64)
    assert np.allclose(g, -np.log(-np.log(np.clip(u, 1e-8, 1.0))), rtol=1e-6)
