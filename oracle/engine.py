"""A sequential CPU engine over the oracle model — TEST INFRASTRUCTURE ONLY.

Restates the prefill/decode flow of engine/backend/executor.py (prefill
759-877, launch_decode_step 1087-1183, _build_fused_inputs 1259-1469) and the
delta-KV append of engine/backend/engine_loop.py:2086-2092, with each stream's
KV held contiguously as the reference pool does.
"""

from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np
import torch

from . import model as M


class OracleEngine:
    def __init__(self, W: Dict[str, torch.Tensor], tcfg, ccfg):
        self.W = W
        self.t = tcfg
        self.c = ccfg
        self.table = M.stacked_codec_table(W, ccfg.num_stages)
        self.k: Dict[int, List[torch.Tensor]] = {}
        self.v: Dict[int, List[torch.Tensor]] = {}
        self.past: Dict[int, int] = {}

    def _empty(self):
        return [torch.zeros(self.t.kv_heads, 0, self.t.head_dim) for _ in range(self.t.num_layers)]

    def prefill(self, sid: int, embeds: torch.Tensor, counts, gumbel, cp_gumbel, temp, pen):
        """``embeds [S, H]`` for one stream; returns the fused outputs (batch 1)."""
        S = embeds.shape[0]
        empty = [torch.zeros(1, self.t.kv_heads, 0, self.t.head_dim) for _ in range(self.t.num_layers)]
        pos = torch.arange(S).unsqueeze(0)
        r = M.fused_step(self.W, self.t, self.c, embeds.unsqueeze(0), pos, empty, empty, [0], counts.unsqueeze(0),
                         gumbel, cp_gumbel, temp, pen, self.table)
        self.k[sid] = [r["new_k"][l][0] for l in range(self.t.num_layers)]
        self.v[sid] = [r["new_v"][l][0] for l in range(self.t.num_layers)]
        self.past[sid] = S
        return r

    def share_prefix(self, dst: int, src: int, n: int) -> None:
        """Stream ``dst`` starts from the first ``n`` KV positions of ``src``: the copy a
        prefix-cache hit makes (engine/backend/engine_loop.py:823-835)."""
        self.k[dst] = [k[:, :n].clone() for k in self.k[src]]
        self.v[dst] = [v[:, :n].clone() for v in self.v[src]]
        self.past[dst] = n

    def extend(self, sid: int, embeds: torch.Tensor, counts, gumbel, cp_gumbel, temp, pen, force=None):
        """``embeds [S, H]`` appended to stream ``sid``'s KV in one fused call (batch 1):
        Executor.prefill_from_prefix (engine/backend/executor.py:952-1081)."""
        S = embeds.shape[0]
        P = self.past[sid]
        pos = (torch.arange(S) + P).unsqueeze(0)
        pk = [k.unsqueeze(0) for k in self.k[sid]]
        pv = [v.unsqueeze(0) for v in self.v[sid]]
        r = M.fused_step(self.W, self.t, self.c, embeds.unsqueeze(0), pos, pk, pv, [P], counts.unsqueeze(0),
                         gumbel, cp_gumbel, temp, pen, self.table, force=force)
        for l in range(self.t.num_layers):
            self.k[sid][l] = torch.cat([self.k[sid][l], r["new_k"][l][0]], dim=1)
            self.v[sid][l] = torch.cat([self.v[sid][l], r["new_v"][l][0]], dim=1)
        self.past[sid] = P + S
        return r

    def decode(self, sids: Sequence[int], embeds: torch.Tensor, counts, gumbel, cp_gumbel, temp, pen, force=None):
        """One batched decode step; ``embeds [B, H]``; ``force``: see ``model.fused_step``."""
        B = len(sids)
        lens = [self.past[s] for s in sids]
        P = max(lens)
        pk, pv = [], []
        for l in range(self.t.num_layers):
            kk = torch.zeros(B, self.t.kv_heads, P, self.t.head_dim)
            vv = torch.zeros_like(kk)
            for i, s in enumerate(sids):
                kk[i, :, :lens[i]] = self.k[s][l]
                vv[i, :, :lens[i]] = self.v[s][l]
            pk.append(kk)
            pv.append(vv)
        pos = torch.tensor(lens).unsqueeze(1)
        r = M.fused_step(self.W, self.t, self.c, embeds.unsqueeze(1), pos, pk, pv, lens, counts,
                         gumbel, cp_gumbel, temp, pen, self.table, force=force)
        for i, s in enumerate(sids):
            for l in range(self.t.num_layers):
                self.k[s][l] = torch.cat([self.k[s][l], r["new_k"][l][i]], dim=1)
                self.v[s][l] = torch.cat([self.v[s][l], r["new_v"][l][i]], dim=1)
            self.past[s] += 1
        return r


def run_trajectory(W, tcfg, ccfg, prompt_embeds: Sequence[torch.Tensor], steps: int, pad: torch.Tensor,
                   gumbel: np.ndarray, cp_gumbel: np.ndarray, temperature: float, penalty: float):
    """Same flow as tests/golden/make_golden.py ``run_trajectory`` on the oracle.

    ``gumbel [steps+1, B, 50]``, ``cp_gumbel [steps+1, B, 15, 50]`` are the
    noise rows the reference run drew.  Returns ``codes [B, steps+1, 16]`` and
    ``step_logits [steps+1, B, V]``.
    """
    eng = OracleEngine(W, tcfg, ccfg)
    B = len(prompt_embeds)
    V = tcfg.codec_vocab_size
    codes = np.zeros((B, steps + 1, 1 + ccfg.num_stages), np.int64)
    step_logits = np.zeros((steps + 1, B, V), np.float32)
    nxt, counts = [], []
    for i, e in enumerate(prompt_embeds):
        r = eng.prefill(i, e, torch.zeros(V, dtype=torch.long), torch.from_numpy(gumbel[0, i:i + 1]),
                        torch.from_numpy(cp_gumbel[0, i:i + 1]), torch.full((1, 1), temperature),
                        torch.full((1, 1), penalty))
        codes[i, 0] = r["full_codec"][0].numpy()
        step_logits[0, i] = r["logits"][0, -1].numpy()
        nxt.append(r["codec_sum"][0] + pad)
        counts.append(r["counts"][0])
    for step in range(1, steps + 1):
        r = eng.decode(list(range(B)), torch.stack(nxt), torch.stack(counts), torch.from_numpy(gumbel[step]),
                       torch.from_numpy(cp_gumbel[step]), torch.full((B, 1), temperature),
                       torch.full((B, 1), penalty))
        codes[:, step] = r["full_codec"].numpy()
        step_logits[step] = r["logits"][:, -1].numpy()
        nxt = [r["codec_sum"][i] + pad for i in range(B)]
        counts = [r["counts"][i] for i in range(B)]
    return codes, step_logits
