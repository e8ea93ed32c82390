#!/usr/bin/env python3
"""Generate the golden fixtures by running the REFERENCE's own code on the CPU.

Run once, in a checkout that has the reference tree next to it:

    python tests/golden/make_golden.py --reference <path to the reference checkout>

and, for the oracle-extended 512-step greedy horizon (no reference needed):

    python tests/golden/make_golden.py --only cfg1_long

It imports, from the reference tree:

* ``scripts/export/talker_unified_modules.py``: ``TalkerUnifiedONNX``,
  ``TalkerUnifiedFusedONNX`` (talker + sampling head + code predictor + codec sum)
* ``scripts/export/utils.py``: ``CodePredictorUnrolled``
* ``scripts/python/codec_embedding_sum.py``: ``CodecEmbeddingSum``
* ``engine/backend/kv_cache_pool.py``: ``KVCachePool``, ``ModelConfig``
* ``engine/backend/prefix_cache.py``: ``PrefixKVCache``
* ``engine/backend/batch_helper.py``: ``padded_attention_bias``

The upstream ``qwen_tts`` package those modules wrap is absent (its git
submodule is empty), so the model objects handed to them are stand-ins built
from ``transformers``' Qwen3 layers with exactly the attributes the reference
reads, loaded with the seeded weights of ``test_stateful_b200.weights``.

Outputs (``tests/golden/*.npz``) are small; the tests never read the
reference tree.
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from test_stateful_b200.config import EngineConfig, tiny_engine_config  # noqa: E402
from test_stateful_b200 import weights as wmod  # noqa: E402
from test_stateful_b200 import workload  # noqa: E402


def import_reference(ref: Path):
    for p in (ref, ref / "scripts" / "export", ref / "scripts" / "python"):
        sys.path.insert(0, str(p))
    import talker_unified_modules as tum
    import utils as export_utils
    import codec_embedding_sum as ces
    from engine.backend import kv_cache_pool, prefix_cache, batch_helper
    return tum, export_utils, ces, kv_cache_pool, prefix_cache, batch_helper


# ----------------------------------------------------------------------------
# stand-in model objects with the attributes the reference modules read
# ----------------------------------------------------------------------------

def _qwen3_config(hidden, heads, kv_heads, head_dim, inter, eps, theta, n_layers):
    from transformers import Qwen3Config
    c = Qwen3Config(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads,
                    head_dim=head_dim, intermediate_size=inter, rms_norm_eps=eps, rope_theta=theta,
                    num_hidden_layers=n_layers, hidden_act="silu", attention_bias=False)
    c._attn_implementation = "eager"
    return c


def _load_layer(layer, W, p):
    sd = {}
    for name in ("input_layernorm.weight", "post_attention_layernorm.weight",
                 "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                 "self_attn.o_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                 "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"):
        sd[name] = W[p + name]
    layer.load_state_dict(sd, strict=True)


def build_standins(cfg: EngineConfig, W):
    from transformers.models.qwen3.modeling_qwen3 import (Qwen3DecoderLayer, Qwen3RMSNorm,
                                                          Qwen3RotaryEmbedding)
    t, c = cfg.talker, cfg.cp
    tc = _qwen3_config(t.hidden_size, t.num_heads, t.kv_heads, t.head_dim, t.intermediate_size,
                       t.rms_eps, t.rope_theta, t.num_layers)
    half = t.head_dim // 2
    mrope = [half // 4, (3 * half) // 8, half - half // 4 - (3 * half) // 8]
    talker = nn.Module()
    talker.layers = nn.ModuleList()
    for i in range(t.num_layers):
        layer = Qwen3DecoderLayer(tc, i)
        _load_layer(layer, W, f"talker.layers.{i}.")
        layer.self_attn.rope_scaling = {"mrope_section": mrope, "interleaved": False}
        talker.layers.append(layer)
    talker.norm = Qwen3RMSNorm(t.hidden_size, eps=t.rms_eps)
    talker.norm.weight.data.copy_(W["talker.norm.weight"])
    talker.rotary_emb = Qwen3RotaryEmbedding(tc)
    codec_head = nn.Linear(t.hidden_size, t.codec_vocab_size, bias=False)
    codec_head.weight.data.copy_(W["talker.codec_head.weight"])
    talker_codec_emb = nn.Embedding(t.codec_vocab_size, t.hidden_size)
    talker_codec_emb.weight.data.copy_(W["talker.codec_embedding.weight"])

    cc = _qwen3_config(c.hidden_size, c.num_heads, c.kv_heads, c.head_dim, c.intermediate_size,
                       c.rms_eps, c.rope_theta, c.num_layers)
    cp = nn.Module()
    cp.config = cc
    cp.model = nn.Module()
    cp.model.layers = nn.ModuleList()
    for i in range(c.num_layers):
        layer = Qwen3DecoderLayer(cc, i)
        _load_layer(layer, W, f"cp.layers.{i}.")
        cp.model.layers.append(layer)
    cp.model.norm = Qwen3RMSNorm(c.hidden_size, eps=c.rms_eps)
    cp.model.norm.weight.data.copy_(W["cp.norm.weight"])
    cp.model.rotary_emb = Qwen3RotaryEmbedding(cc)
    cp.model.codec_embedding = nn.ModuleList()
    cp.lm_head = nn.ModuleList()
    for s in range(c.num_stages):
        e = nn.Embedding(c.vocab_size, c.talker_hidden_size)
        e.weight.data.copy_(W[f"cp.codec_embedding.{s}.weight"])
        cp.model.codec_embedding.append(e)
        h = nn.Linear(c.hidden_size, c.vocab_size, bias=False)
        h.weight.data.copy_(W[f"cp.lm_head.{s}.weight"])
        cp.lm_head.append(h)
    cp.small_to_mtp_projection = nn.Linear(c.talker_hidden_size, c.hidden_size, bias=True)
    cp.small_to_mtp_projection.weight.data.copy_(W["cp.projection.weight"])
    cp.small_to_mtp_projection.bias.data.copy_(W["cp.projection.bias"])
    return talker, codec_head, talker_codec_emb, cp


def build_fused(ref_mods, cfg, W):
    tum, export_utils, ces, *_ = ref_mods
    talker, codec_head, talker_codec_emb, cp = build_standins(cfg, W)
    backbone = tum.TalkerUnifiedONNX(talker, codec_head, emit_delta_kv=True).eval()
    cp_unrolled = export_utils.CodePredictorUnrolled(cp, talker_codec_emb, logits_topk=tum.LOGITS_TOPK).eval()
    stacked = ces.CodecEmbeddingSum.stack_weights(
        talker_codec_emb.weight.data, [e.weight.data for e in cp.model.codec_embedding])
    csum = ces.CodecEmbeddingSum(stacked).eval()
    fused = tum.TalkerUnifiedFusedONNX(backbone, cp_unrolled, csum, vocab_size=cfg.talker.codec_vocab_size,
                                       codec_eos_token_id=cfg.talker.codec_eos_id).eval()
    return fused


def fp32_weights(cfg, seed):
    W = wmod.make_talker_weights(cfg.talker, seed)
    W.update(wmod.make_cp_weights(cfg.cp, seed))
    return wmod.to_fp32(W)


# ----------------------------------------------------------------------------
# a minimal engine driver over the reference KVCachePool (executor.py flow)
# ----------------------------------------------------------------------------

class RefDriver:
    """Prefill + batched decode the way Executor/EngineLoop drive the fused graph.

    prefill: dummy past KV of length 1 masked by the bias (executor.py:790-797,
    1275-1281, 1400-1405), delta KV scattered with ``scatter_prefill_kv``
    (executor.py:838-844); decode: ``gather_talker_kv`` + ``padded_attention_bias``
    (executor.py:1116-1122, 1283-1288), delta appended with
    ``scatter_talker_kv_delta`` (engine_loop.py:2086-2092).
    """

    def __init__(self, ref_mods, cfg, W, max_slots, max_seq):
        _, _, _, kvp, _, bh = ref_mods
        self.bh = bh
        self.cfg = cfg
        self.fused = build_fused(ref_mods, cfg, W)
        t = cfg.talker
        mc = kvp.ModelConfig(num_layers=t.num_layers, kv_heads=t.kv_heads, head_dim=t.head_dim,
                             max_seq_len=max_seq, hidden_size=t.hidden_size, dtype=torch.float32,
                             codec_vocab_size=t.codec_vocab_size)
        self.pool = kvp.KVCachePool(max_slots=max_slots, config=mc, device=torch.device("cpu"))

    def _call(self, embeds, pos, counts, gumbel, cp_gumbel, temp, pen, bias, past):
        L2 = past.shape[1]
        past_list = [past[:, i] for i in range(L2)]
        with torch.no_grad():
            out = self.fused(embeds, pos, counts, gumbel, cp_gumbel, temp, pen, bias, *past_list)
        codec_sum, full_codec, hidden, logits, counts2, *present = out
        return dict(codec_sum=codec_sum, full_codec=full_codec, hidden=hidden, logits=logits,
                    counts=counts2, delta=torch.stack(present, dim=1))

    def prefill(self, slot, embeds, counts, gumbel, cp_gumbel, temp, pen):
        t = self.cfg.talker
        S = embeds.shape[1]
        pos = torch.arange(S).view(1, 1, S, 1).expand(1, 3, S, 1).contiguous()
        bias = self.bh.padded_attention_bias(torch.zeros(1, dtype=torch.long), S, 1,
                                             torch.device("cpu"), torch.float32)
        past = torch.zeros(1, 2 * t.num_layers, t.kv_heads, 1, t.head_dim)
        r = self._call(embeds, pos, counts, gumbel, cp_gumbel, temp, pen, bias, past)
        self.pool.scatter_prefill_kv(slot.slot_id, r["delta"], S)
        slot.past_len = S
        return r

    def decode(self, slots, embeds, counts, gumbel, cp_gumbel, temp, pen):
        ids = [s.slot_id for s in slots]
        past_lens = [s.past_len for s in slots]
        P = max(past_lens)
        past = self.pool.gather_talker_kv(ids, P)
        bias = self.bh.padded_attention_bias(torch.tensor(past_lens), 1, P, torch.device("cpu"),
                                             torch.float32)
        pos = torch.tensor(past_lens).view(-1, 1, 1, 1).expand(-1, 3, 1, 1).contiguous()
        r = self._call(embeds, pos, counts, gumbel, cp_gumbel, temp, pen, bias, past)
        self.pool.scatter_talker_kv_delta(ids, r["delta"], past_lens)
        for s in slots:
            s.past_len += 1
        r["past_lens"] = past_lens
        return r


def run_trajectory(ref_mods, cfg, seed, lengths, steps, do_sample, noise_seed=None):
    """Prefill each stream, then ``steps`` batched decode steps; returns arrays."""
    W = fp32_weights(cfg, seed)
    t, c = cfg.talker, cfg.cp
    B = len(lengths)
    drv = RefDriver(ref_mods, cfg, W, max_slots=B, max_seq=max(lengths) + steps + 1)
    table = workload.text_table(t.hidden_size, seed)
    pad = workload.tts_pad_embed(t.hidden_size, seed)
    ids = workload.prompt_ids(lengths, seed)
    gnoise = torch.Generator().manual_seed(noise_seed if noise_seed is not None else seed + 7)
    temp_v, pen_v = (0.9, 1.05) if do_sample else (1.0, 1.05)

    def noise(n):
        if not do_sample:
            return torch.zeros(n, 50), torch.zeros(n, c.num_stages, 50)
        u = torch.rand(n, 50, generator=gnoise).clamp(1e-8, 1.0)
        cu = torch.rand(n, c.num_stages, 50, generator=gnoise).clamp(1e-8, 1.0)
        return -torch.log(-torch.log(u)), -torch.log(-torch.log(cu))

    codes = np.zeros((B, steps + 1, 1 + c.num_stages), np.int64)
    logits0 = np.zeros((B, t.codec_vocab_size), np.float32)
    hidden0 = np.zeros((B, t.hidden_size), np.float32)
    gumbels = np.zeros((steps + 1, B, 50), np.float32)
    cp_gumbels = np.zeros((steps + 1, B, c.num_stages, 50), np.float32)
    step_logits = np.zeros((steps + 1, B, t.codec_vocab_size), np.float32)
    slots, nxt, counts = [], [], []
    for i, n in enumerate(lengths):
        slot = drv.pool.allocate(f"s{i}")
        slots.append(slot)
        g, cg = noise(1)
        gumbels[0, i], cp_gumbels[0, i] = g[0].numpy(), cg[0].numpy()
        r = drv.prefill(slot, table[ids[i]].unsqueeze(0), torch.zeros(1, t.codec_vocab_size, dtype=torch.long),
                        g, cg, torch.full((1, 1), temp_v), torch.full((1, 1), pen_v))
        codes[i, 0] = r["full_codec"][0].numpy()
        logits0[i] = r["logits"][0, -1].numpy()
        step_logits[0, i] = r["logits"][0, -1].numpy()
        hidden0[i] = r["hidden"][0, -1].numpy()
        nxt.append(r["codec_sum"][0, 0] + pad)
        counts.append(r["counts"][0])
    for step in range(1, steps + 1):
        g, cg = noise(B)
        gumbels[step], cp_gumbels[step] = g.numpy(), cg.numpy()
        embeds = torch.stack(nxt).unsqueeze(1)
        r = drv.decode(slots, embeds, torch.stack(counts), g, cg, torch.full((B, 1), temp_v),
                       torch.full((B, 1), pen_v))
        codes[:, step] = r["full_codec"].numpy()
        step_logits[step] = r["logits"][:, -1].numpy()
        nxt = [r["codec_sum"][i, 0] + pad for i in range(B)]
        counts = [r["counts"][i] for i in range(B)]
    return dict(codes=codes, logits0=logits0, hidden0=hidden0, gumbel=gumbels, cp_gumbel=cp_gumbels,
                step_logits=step_logits, lengths=np.asarray(lengths, np.int64),
                prompt_ids=np.concatenate([x.numpy() for x in ids]), seed=np.int64(seed),
                steps=np.int64(steps), do_sample=np.int64(int(do_sample)),
                temperature=np.float32(temp_v), penalty=np.float32(pen_v))


def make_fused_tiny(ref_mods, out):
    """Single fused calls at the tiny config: prefill, ragged decode (sampled)."""
    cfg = tiny_engine_config(num_layers=2)
    t, c = cfg.talker, cfg.cp
    W = fp32_weights(cfg, seed=3)
    fused = build_fused(ref_mods, cfg, W)
    bh = ref_mods[5]
    g = torch.Generator().manual_seed(5)
    B, P = 3, 12
    past_lens = [5, 9, 12]
    past = torch.randn(B, 2 * t.num_layers, t.kv_heads, P, t.head_dim, generator=g)
    for b, pl in enumerate(past_lens):
        past[b, :, :, pl:] = 0.0
    embeds = torch.randn(B, 1, t.hidden_size, generator=g) * 0.5
    counts = torch.randint(0, 2, (B, t.codec_vocab_size), generator=g)
    gum = -torch.log(-torch.log(torch.rand(B, 50, generator=g).clamp(1e-8, 1)))
    cgum = -torch.log(-torch.log(torch.rand(B, c.num_stages, 50, generator=g).clamp(1e-8, 1)))
    temp = torch.full((B, 1), 0.9)
    pen = torch.full((B, 1), 1.05)
    bias = bh.padded_attention_bias(torch.tensor(past_lens), 1, P, torch.device("cpu"), torch.float32)
    pos = torch.tensor(past_lens).view(-1, 1, 1, 1).expand(-1, 3, 1, 1).contiguous()
    with torch.no_grad():
        r = fused(embeds, pos, counts, gum, cgum, temp, pen, bias, *[past[:, i] for i in range(2 * t.num_layers)])
    codec_sum, full_codec, hidden, logits, counts2, *present = r
    np.savez_compressed(out, past=past.numpy(), past_lens=np.asarray(past_lens), embeds=embeds.numpy(),
                        counts=counts.numpy(), gumbel=gum.numpy(), cp_gumbel=cgum.numpy(),
                        temperature=temp.numpy(), penalty=pen.numpy(),
                        out_codec_sum=codec_sum.numpy(), out_full_codec=full_codec.numpy(),
                        out_hidden=hidden.numpy(), out_logits=logits.numpy(), out_counts=counts2.numpy(),
                        out_delta=torch.stack(present, dim=1).numpy(), seed=np.int64(3), num_layers=np.int64(2))


def make_pool_ops(ref_mods, out):
    """KVCachePool + PrefixKVCache op sequence with random KV (the paged pool's pin).

    Ops mirror the engine: allocate (LIFO, zeroes the slot), prefill scatter,
    prefix put (a clone of ``[0, prefix_len)``), prefix hit restore
    (engine_loop.py:823-835), decode delta appends, release, re-allocate.
    """
    _, _, _, kvp, pc, _ = ref_mods
    L, H, D, S = 2, 2, 4, 48
    mc = kvp.ModelConfig(num_layers=L, kv_heads=H, head_dim=D, max_seq_len=S, dtype=torch.float32)
    pool = kvp.KVCachePool(max_slots=4, config=mc, device=torch.device("cpu"))
    cache = pc.PrefixKVCache(max_entries=2, max_prefix_len=32)
    g = torch.Generator().manual_seed(11)
    ops = []   # (name, args...) encoded as int rows: [op, slot, n, aux]
    kvs = []

    def rnd(n):
        t = torch.randn(1, 2 * L, H, n, D, generator=g)
        kvs.append(t[0].permute(2, 0, 1, 3).reshape(n, -1).numpy())   # [n, L2*H*D] per token
        return t

    A = pool.allocate("A"); ops.append([0, A.slot_id, 0, 0])
    kv = rnd(21); pool.scatter_prefill_kv(A.slot_id, kv, 21); A.past_len = 21; ops.append([1, A.slot_id, 21, 0])
    cache.put("key", pool._talker_kv_pool[A.slot_id:A.slot_id + 1, :, :, :19].clone(), 19); ops.append([2, A.slot_id, 19, 0])
    B = pool.allocate("B"); ops.append([0, B.slot_id, 0, 0])
    e = cache.get("key")
    pool._talker_kv_pool[B.slot_id, :, :, :e.prefix_len] = e.talker_kv[0, :, :, :e.prefix_len]
    B.past_len = e.prefix_len; ops.append([3, B.slot_id, e.prefix_len, 0])
    C = pool.allocate("C"); ops.append([0, C.slot_id, 0, 0])
    pool._talker_kv_pool[C.slot_id, :, :, :e.prefix_len] = e.talker_kv[0, :, :, :e.prefix_len]
    C.past_len = e.prefix_len; ops.append([3, C.slot_id, e.prefix_len, 0])
    for step in range(15):
        batch = [A, B, C] if step % 3 else [C, A, B]
        d = torch.randn(len(batch), 2 * L, H, 1, D, generator=g)
        for i in range(len(batch)):
            kvs.append(d[i].permute(2, 0, 1, 3).reshape(1, -1).numpy())
        pool.scatter_talker_kv_delta([s.slot_id for s in batch], d, [s.past_len for s in batch])
        ops.append([4, len(batch)] + [s.slot_id for s in batch] + [0] * (4 - len(batch)))
        for s in batch:
            s.past_len += 1
    snap1 = {s.slot_id: pool.gather_talker_kv([s.slot_id], s.past_len)[0].numpy() for s in (A, B, C)}
    lens1 = {s.slot_id: s.past_len for s in (A, B, C)}
    pool.release(A.slot_id); ops.append([5, A.slot_id, 0, 0])
    Dd = pool.allocate("D"); ops.append([0, Dd.slot_id, 0, 0])
    kv = rnd(7); pool.scatter_prefill_kv(Dd.slot_id, kv, 7); Dd.past_len = 7; ops.append([1, Dd.slot_id, 7, 0])
    for step in range(10):
        batch = [Dd, B]
        d = torch.randn(2, 2 * L, H, 1, D, generator=g)
        for i in range(2):
            kvs.append(d[i].permute(2, 0, 1, 3).reshape(1, -1).numpy())
        pool.scatter_talker_kv_delta([s.slot_id for s in batch], d, [s.past_len for s in batch])
        ops.append([4, 2, Dd.slot_id, B.slot_id, 0, 0])
        for s in batch:
            s.past_len += 1
    final = {s.slot_id: pool.gather_talker_kv([s.slot_id], s.past_len)[0].numpy() for s in (Dd, B, C)}
    lens2 = {s.slot_id: s.past_len for s in (Dd, B, C)}
    width = max(len(o) for o in ops)
    ops_arr = np.array([o + [0] * (width - len(o)) for o in ops], np.int64)
    payload = dict(ops=ops_arr, kv_tokens=np.concatenate(kvs, 0), L=L, H=H, D=D, S=S)
    for k, v in snap1.items():
        payload[f"snap1_slot{k}"] = v
        payload[f"snap1_len{k}"] = lens1[k]
    for k, v in final.items():
        payload[f"final_slot{k}"] = v
        payload[f"final_len{k}"] = lens2[k]
    np.savez_compressed(out, **payload)


# ----------------------------------------------------------------------------
# code2wav: stand-in decoder tree for scripts/export/code2wav_streaming.py
# ----------------------------------------------------------------------------

class SnakeBeta(nn.Module):
    """The wrapper patches every module of this class NAME (code2wav_streaming.py:562-592)."""

    def __init__(self, alpha, beta):
        super().__init__()
        self.alpha = nn.Parameter(alpha.clone())
        self.beta = nn.Parameter(beta.clone())

    def forward(self, x):
        a = torch.exp(self.alpha.view(1, -1, 1))
        s = torch.sin(x * a)
        return x + s * s * torch.exp(-self.beta.view(1, -1, 1))


class _CausalConv(nn.Module):
    """``.conv`` and a left ``.padding`` are what streaming_causal_conv reads."""

    def __init__(self, w, b, dilation=1, groups=1):
        super().__init__()
        cout, cin_g, k = w.shape
        self.conv = nn.Conv1d(cin_g * groups, cout, k, dilation=dilation, groups=groups)
        self.conv.weight.data.copy_(w)
        self.conv.bias.data.copy_(b)
        self.padding = (k - 1) * dilation

    def forward(self, x):
        return self.conv(nn.functional.pad(x, (self.padding, 0)))


class _CausalTransConv(nn.Module):
    def __init__(self, w, b, stride):
        super().__init__()
        cin, cout, k = w.shape
        self.conv = nn.ConvTranspose1d(cin, cout, k, stride=stride)
        self.conv.weight.data.copy_(w)
        self.conv.bias.data.copy_(b)
        self.right_pad = k - stride

    def forward(self, x):
        y = self.conv(x)
        return y[..., :-self.right_pad] if self.right_pad > 0 else y


class _Scale(nn.Module):
    def __init__(self, s):
        super().__init__()
        self.scale = nn.Parameter(s.clone())

    def forward(self, x):
        return self.scale * x


class _Codebook(nn.Module):
    """embedding = embedding_sum / cluster_usage.clamp(min=epsilon) (code2wav_streaming.py:227-229)."""

    def __init__(self, table):
        super().__init__()
        self.register_buffer("embedding_sum", table * 2.0)
        self.register_buffer("cluster_usage", torch.full((table.shape[0],), 2.0))
        self.epsilon = 1e-5

    def decode(self, codes):
        emb = self.embedding_sum / self.cluster_usage.clamp(min=self.epsilon).unsqueeze(1)
        return nn.functional.embedding(codes, emb).transpose(1, 2)


def _linear(W, name, bias=False):
    w = W[name + ".weight"]
    m = nn.Linear(w.shape[1], w.shape[0], bias=bias)
    m.weight.data.copy_(w.reshape(w.shape[0], w.shape[1]))
    if bias:
        m.bias.data.copy_(W[name + ".bias"])
    return m


def build_code2wav_standin(c, W):
    """A module tree with exactly the attributes Code2WavStreamingWrapper reads
    (quantizer.rvq_*.{n_q, vq.layers[i]._codebook, output_proj}, pre_conv,
    pre_transformer.{input_proj, rotary_emb, layers, norm, output_proj},
    upsample[i] = (transconv, convnext), decoder[0..6], config)."""
    import types
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm

    def rvq(part, tables):
        r = nn.Module()
        r.n_q = len(tables)
        r.vq = nn.Module()
        r.vq.layers = nn.ModuleList()
        for t in tables:
            layer = nn.Module()
            layer._codebook = _Codebook(t)
            r.vq.layers.append(layer)
        w = W[f"c2w.{part}.output_proj.weight"]
        r.output_proj = nn.Conv1d(w.shape[1], w.shape[0], 1)
        r.output_proj.weight.data.copy_(w)
        r.output_proj.bias.data.copy_(W[f"c2w.{part}.output_proj.bias"])
        return r

    dec = nn.Module()
    dec.config = types.SimpleNamespace(
        codebook_dim=c.codebook_dim, latent_dim=c.latent_dim, decoder_dim=c.decoder_dim,
        num_key_value_heads=c.kv_heads, num_attention_heads=c.num_heads, head_dim=c.head_dim,
        hidden_size=c.hidden_size, num_hidden_layers=c.num_layers, _attn_implementation="eager")
    q = nn.Module()
    q.n_q_semantic, q.n_q_acoustic = 1, c.num_codebooks - 1
    q.rvq_first = rvq("rvq_first", [W["c2w.rvq_first.codebook.0"]])
    q.rvq_rest = rvq("rvq_rest", [W[f"c2w.rvq_rest.codebook.{i}"] for i in range(c.num_codebooks - 1)])
    dec.quantizer = q
    dec.pre_conv = _CausalConv(W["c2w.pre_conv.weight"], W["c2w.pre_conv.bias"])

    p = "c2w.pre_transformer."
    pt = nn.Module()
    pt.input_proj = _linear(W, p + "input_proj", bias=True)
    pt.rotary_emb = nn.Module()
    pt.rotary_emb.register_buffer(
        "inv_freq", 1.0 / (c.rope_theta ** (torch.arange(0, c.head_dim, 2, dtype=torch.int64).float() / c.head_dim)))
    pt.rotary_emb.attention_scaling = 1.0
    pt.layers = nn.ModuleList()
    for i in range(c.num_layers):
        lp = f"{p}layers.{i}."
        layer = nn.Module()
        layer.input_layernorm = Qwen3RMSNorm(c.hidden_size, eps=c.rms_eps)
        layer.input_layernorm.weight.data.copy_(W[lp + "input_layernorm.weight"])
        layer.post_attention_layernorm = Qwen3RMSNorm(c.hidden_size, eps=c.rms_eps)
        layer.post_attention_layernorm.weight.data.copy_(W[lp + "post_attention_layernorm.weight"])
        a = nn.Module()
        for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(a, n, _linear(W, lp + "self_attn." + n))
        a.q_norm = Qwen3RMSNorm(c.head_dim, eps=c.rms_eps)
        a.q_norm.weight.data.copy_(W[lp + "self_attn.q_norm.weight"])
        a.k_norm = Qwen3RMSNorm(c.head_dim, eps=c.rms_eps)
        a.k_norm.weight.data.copy_(W[lp + "self_attn.k_norm.weight"])
        a.head_dim, a.layer_idx = c.head_dim, i
        a.num_key_value_groups = c.num_heads // c.kv_heads
        a.scaling = c.head_dim ** -0.5
        layer.self_attn = a
        layer.self_attn_layer_scale = _Scale(W[lp + "self_attn_layer_scale.scale"])
        layer.mlp_layer_scale = _Scale(W[lp + "mlp_layer_scale.scale"])
        mlp = nn.Module()
        for n in ("gate_proj", "up_proj", "down_proj"):
            setattr(mlp, n, _linear(W, lp + "mlp." + n))
        mlp.forward = types.MethodType(
            lambda self, x: self.down_proj(nn.functional.silu(self.gate_proj(x)) * self.up_proj(x)), mlp)
        layer.mlp = mlp
        pt.layers.append(layer)
    pt.norm = Qwen3RMSNorm(c.hidden_size, eps=c.rms_eps)
    pt.norm.weight.data.copy_(W[p + "norm.weight"])
    pt.output_proj = _linear(W, p + "output_proj", bias=True)
    dec.pre_transformer = pt

    dec.upsample = nn.ModuleList()
    for i, s in enumerate(c.upsample_ratios):
        u = f"c2w.upsample.{i}."
        tconv = _CausalTransConv(W[u + "transconv.weight"], W[u + "transconv.bias"], s)
        cn = nn.Module()
        cn.dwconv = _CausalConv(W[u + "convnext.dwconv.weight"], W[u + "convnext.dwconv.bias"],
                                groups=c.latent_dim)
        cn.norm = nn.LayerNorm(c.latent_dim, eps=c.ln_eps)
        cn.norm.weight.data.copy_(W[u + "convnext.norm.weight"])
        cn.norm.bias.data.copy_(W[u + "convnext.norm.bias"])
        cn.pwconv1 = _linear(W, u + "convnext.pwconv1", bias=True)
        cn.act = nn.GELU()
        cn.pwconv2 = _linear(W, u + "convnext.pwconv2", bias=True)
        cn.gamma = nn.Parameter(W[u + "convnext.gamma"].clone())
        dec.upsample.append(nn.ModuleList([tconv, cn]))

    d = nn.ModuleList([_CausalConv(W["c2w.decoder.0.weight"], W["c2w.decoder.0.bias"])])
    for b, (cin, cout, s) in enumerate(c.block_dims()):
        k = f"c2w.decoder.{1 + b}."
        blk = nn.Module()
        mods = [SnakeBeta(W[k + "snake.alpha"], W[k + "snake.beta"]),
                _CausalTransConv(W[k + "transconv.weight"], W[k + "transconv.bias"], s)]
        for j, dil in enumerate(c.dilations):
            r = f"{k}res.{j}."
            ru = nn.Module()
            ru.act1 = SnakeBeta(W[r + "act1.alpha"], W[r + "act1.beta"])
            ru.conv1 = _CausalConv(W[r + "conv1.weight"], W[r + "conv1.bias"], dilation=dil)
            ru.act2 = SnakeBeta(W[r + "act2.alpha"], W[r + "act2.beta"])
            ru.conv2 = _CausalConv(W[r + "conv2.weight"], W[r + "conv2.bias"])
            mods.append(ru)
        blk.block = nn.ModuleList(mods)
        d.append(blk)
    d.append(SnakeBeta(W["c2w.decoder.5.alpha"], W["c2w.decoder.5.beta"]))
    d.append(_CausalConv(W["c2w.decoder.6.weight"], W["c2w.decoder.6.bias"]))
    dec.decoder = d
    return dec.eval()


def make_code2wav(ref: Path, out, seed=5, steps=78, starts=(0, 9)):
    """Batched T=1 streaming decode the way the fused step drives the wrapper:
    per-slot delta KV appended and trimmed to window-1 frames (executor.py:68-79),
    left-padded past KV with a -inf bias on the padding (executor.py:1374-1441),
    cache_position = each slot's frame index (executor.py:1298-1301)."""
    sys.path.insert(0, str(ref / "scripts" / "export"))
    import code2wav_streaming as c2ws
    from test_stateful_b200.config import tiny_code2wav_config
    c = tiny_code2wav_config()
    W = wmod.to_fp32(wmod.make_code2wav_weights(c, seed))
    dec = build_code2wav_standin(c, W)
    wrap = c2ws.Code2WavStreamingWrapper(dec, window_size=c.window, emit_delta_kv=True).eval()
    shapes = c2ws.get_initial_state_shapes(dec, batch_size=1)
    conv_shapes = [s for n, s in shapes if n.startswith("conv_state")]
    trans_shapes = [s for n, s in shapes if n.startswith("transconv")]
    n_slots = len(starts)
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(0, c.codebook_size, (steps, n_slots, c.num_codebooks), generator=g)
    kv = [None] * n_slots                      # [1, 2L, H, S, hd] past per slot
    conv = [[torch.zeros(s) for s in conv_shapes] for _ in range(n_slots)]
    trans = [[torch.zeros(s) for s in trans_shapes] for _ in range(n_slots)]
    frame = [0] * n_slots
    wav = np.zeros((steps, n_slots, c.samples_per_frame), np.float32)
    active = np.zeros((steps, n_slots), bool)
    max_past = c.window - 1
    L2 = 2 * c.num_layers
    with torch.no_grad():
        for t in range(steps):
            act = [i for i in range(n_slots) if t >= starts[i]]
            lens = [0 if kv[i] is None else min(kv[i].shape[3], max_past) for i in act]
            P = max(1, max(lens))
            bias = torch.zeros(len(act), 1, 1, P + 1)
            past = []
            for bi, (i, sl) in enumerate(zip(act, lens)):
                bias[bi, :, :, :P - sl] = float("-inf")
                k = kv[i] if kv[i] is not None else torch.zeros(1, L2, c.kv_heads, 0, c.head_dim)
                past.append(nn.functional.pad(k[:, :, :, -max_past:], (0, 0, P - sl, 0)))
            past = torch.cat(past, 0)
            states = [past[:, j] for j in range(L2)]
            states += [torch.cat([conv[i][j] for i in act], 0) for j in range(len(conv_shapes))]
            states += [torch.cat([trans[i][j] for i in act], 0) for j in range(len(trans_shapes))]
            cpos = torch.tensor([[float(frame[i])] for i in act])
            outs = wrap(codes[t, act].unsqueeze(-1), cpos, bias, *states)
            delta = torch.stack(outs[1:1 + L2], dim=1)
            nc = outs[1 + L2:1 + L2 + len(conv_shapes)]
            nt = outs[1 + L2 + len(conv_shapes):]
            for bi, i in enumerate(act):
                wav[t, i] = outs[0][bi].numpy()
                active[t, i] = True
                d = delta[bi:bi + 1]
                kv[i] = d if kv[i] is None else torch.cat([kv[i], d], 3)[:, :, :, -max_past:]
                conv[i] = [x[bi:bi + 1].clone() for x in nc]
                trans[i] = [x[bi:bi + 1].clone() for x in nt]
                frame[i] += 1
    np.savez_compressed(out, codes=codes.numpy().astype(np.int32), active=active, wav=wav,
                        seed=np.int64(seed), starts=np.asarray(starts, np.int32))


def make_cfg1_long(out, steps=512):
    """The CPU reference case's streams (seed 0, prompts {37, 64, 91, 128}, greedy) for ``steps``
    decode steps, run by the ORACLE (oracle/engine.py): the reference's own modules pin the
    oracle over the first 32 steps (cfg1_full_greedy.npz); this fixture extends the horizon to
    the 512-step agreement bar.  Stores the greedy codes and every 64th step's logits (fp16)."""
    from oracle.engine import run_trajectory as oracle_trajectory
    cfg = EngineConfig()
    seed, lengths = 0, [37, 64, 91, 128]
    t, c = cfg.talker, cfg.cp
    W = fp32_weights(cfg, seed)
    table = workload.text_table(t.hidden_size, seed)
    pad = workload.tts_pad_embed(t.hidden_size, seed)
    ids = workload.prompt_ids(lengths, seed)
    B = len(lengths)
    g = np.zeros((steps + 1, B, 50), np.float32)
    cg = np.zeros((steps + 1, B, c.num_stages, 50), np.float32)
    t0 = time.time()
    codes, step_logits = oracle_trajectory(W, t, c, [table[i] for i in ids], steps, pad, g, cg, 1.0, 1.05)
    every = 64
    keep = np.arange(0, steps + 1, every)
    np.savez_compressed(out, codes=codes.astype(np.int16), logit_steps=keep.astype(np.int32),
                        step_logits=step_logits[keep].astype(np.float16), lengths=np.asarray(lengths, np.int64),
                        seed=np.int64(seed), steps=np.int64(steps), do_sample=np.int64(0),
                        temperature=np.float32(1.0), penalty=np.float32(1.05))
    print(f"cfg1_long: {steps} steps in {time.time() - t0:.0f}s", flush=True)


def make_code2wav_chunked(ref: Path, out, seed=6, chunks=(25, 25, 25, 7), start1=1):
    """Multi-frame chunks through the reference wrapper (25-frame chunks with carried state): per call T frames per
    slot, past KV capped at window - T frames (the executor's max_past = window - chunk_T,
    executor.py:1374-1380), bias = -inf on each slot's left padding plus the causal mask inside
    the chunk, delta KV appended.  Slot 1 joins at call ``start1`` (ragged pasts)."""
    sys.path.insert(0, str(ref / "scripts" / "export"))
    import code2wav_streaming as c2ws
    from test_stateful_b200.config import tiny_code2wav_config
    c = tiny_code2wav_config()
    W = wmod.to_fp32(wmod.make_code2wav_weights(c, seed))
    dec = build_code2wav_standin(c, W)
    wrap = c2ws.Code2WavStreamingWrapper(dec, window_size=c.window, emit_delta_kv=True).eval()
    shapes = c2ws.get_initial_state_shapes(dec, batch_size=1)
    conv_shapes = [s for n, s in shapes if n.startswith("conv_state")]
    trans_shapes = [s for n, s in shapes if n.startswith("transconv")]
    L2 = 2 * c.num_layers
    g = torch.Generator().manual_seed(seed)
    total = sum(chunks)
    codes = torch.randint(0, c.codebook_size, (2, c.num_codebooks, total), generator=g)
    kv = [None, None]
    conv = [[torch.zeros(s) for s in conv_shapes] for _ in range(2)]
    trans = [[torch.zeros(s) for s in trans_shapes] for _ in range(2)]
    frame = [0, 0]
    wav = [[], []]
    with torch.no_grad():
        for call, T in enumerate(chunks):
            act = [0] + ([1] if call >= start1 else [])
            max_past = c.window - T
            lens = [0 if kv[i] is None else min(kv[i].shape[3], max_past) for i in act]
            P = max(1, max(lens))
            bias = torch.zeros(len(act), 1, T, P + T)
            bias[:, :, :, P:] = torch.triu(torch.full((T, T), float("-inf")), diagonal=1)
            past = []
            for bi, (i, sl) in enumerate(zip(act, lens)):
                bias[bi, :, :, :P - sl] = float("-inf")
                k = kv[i] if kv[i] is not None else torch.zeros(1, L2, c.kv_heads, 0, c.head_dim)
                past.append(nn.functional.pad(k[:, :, :, k.shape[3] - sl:], (0, 0, P - sl, 0)))
            past = torch.cat(past, 0)
            states = [past[:, j] for j in range(L2)]
            states += [torch.cat([conv[i][j] for i in act], 0) for j in range(len(conv_shapes))]
            states += [torch.cat([trans[i][j] for i in act], 0) for j in range(len(trans_shapes))]
            cpos = torch.stack([torch.arange(frame[i], frame[i] + T, dtype=torch.float32) for i in act])
            cds = torch.stack([codes[i, :, frame[i]:frame[i] + T] for i in act])
            outs = wrap(cds, cpos, bias, *states)
            delta = torch.stack(outs[1:1 + L2], dim=1)
            nc = outs[1 + L2:1 + L2 + len(conv_shapes)]
            nt = outs[1 + L2 + len(conv_shapes):]
            for bi, i in enumerate(act):
                wav[i].append(outs[0][bi].numpy())
                d = delta[bi:bi + 1]
                kv[i] = d if kv[i] is None else torch.cat([kv[i], d], 3)[:, :, :, -(c.window - 1):]
                conv[i] = [x[bi:bi + 1].clone() for x in nc]
                trans[i] = [x[bi:bi + 1].clone() for x in nt]
                frame[i] += T
    np.savez_compressed(out, codes=codes.numpy().astype(np.int32), chunks=np.asarray(chunks, np.int32),
                        start1=np.int32(start1), seed=np.int64(seed),
                        wav0=np.concatenate(wav[0]).astype(np.float16), wav1=np.concatenate(wav[1]).astype(np.float16))


def make_code2wav_warm(ref: Path, out, seed=7, warm=80, cont=10):
    """A warm state as the reference hands it to ``Executor.apply_c2w_warm_state``
    (engine/backend/executor.py:715-757): one stream decoded frame by frame through the wrapper
    for ``warm`` frames from zero state (past KV kept at window - 1 frames, as the executor
    crops it), its state recorded — KV [1, 2L, H, T, hd], the 17 conv states, the 4 transposed-
    conv overlap tails, the frame index — then ``cont`` more frames decoded from it (their audio
    is what a backend given that state must reproduce)."""
    sys.path.insert(0, str(ref / "scripts" / "export"))
    import code2wav_streaming as c2ws
    from test_stateful_b200.config import tiny_code2wav_config
    c = tiny_code2wav_config()
    W = wmod.to_fp32(wmod.make_code2wav_weights(c, seed))
    dec = build_code2wav_standin(c, W)
    wrap = c2ws.Code2WavStreamingWrapper(dec, window_size=c.window, emit_delta_kv=True).eval()
    shapes = c2ws.get_initial_state_shapes(dec, batch_size=1)
    conv = [torch.zeros(s) for n, s in shapes if n.startswith("conv_state")]
    trans = [torch.zeros(s) for n, s in shapes if n.startswith("transconv")]
    L2 = 2 * c.num_layers
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(0, c.codebook_size, (warm + cont, c.num_codebooks), generator=g)
    kv = None
    max_past = c.window - 1
    rec = None
    wav = []
    with torch.no_grad():
        for t in range(warm + cont):
            if t == warm:
                rec = (kv.clone(), [x.clone() for x in conv], [x.clone() for x in trans], t)
            sl = 0 if kv is None else kv.shape[3]
            P = max(1, sl)
            bias = torch.zeros(1, 1, 1, P + 1)
            bias[:, :, :, :P - sl] = float("-inf")
            k = kv if kv is not None else torch.zeros(1, L2, c.kv_heads, 0, c.head_dim)
            past = nn.functional.pad(k, (0, 0, P - sl, 0))
            states = [past[:, j] for j in range(L2)] + conv + trans
            outs = wrap(codes[t].view(1, -1, 1), torch.tensor([[float(t)]]), bias, *states)
            d = torch.stack(outs[1:1 + L2], dim=1)
            kv = d if kv is None else torch.cat([kv, d], 3)[:, :, :, -max_past:]
            conv = [x.clone() for x in outs[1 + L2:1 + L2 + len(conv)]]
            trans = [x.clone() for x in outs[1 + L2 + len(conv):]]
            if t >= warm:
                wav.append(outs[0][0].numpy())
    kv0, conv0, trans0, frame0 = rec
    arrays = {f"conv_{j}": x.numpy() for j, x in enumerate(conv0)}
    arrays.update({f"trans_{b}": x.numpy() for b, x in enumerate(trans0)})
    np.savez_compressed(out, codes=codes.numpy().astype(np.int32), kv=kv0.numpy(), frame=np.int32(frame0),
                        wav=np.stack(wav).astype(np.float32), seed=np.int64(seed), **arrays)


def make_seeds(out):
    """Per-(session, segment) sampling seeds from engine/backend/executor.py:45-52."""
    from engine.backend import executor as ref_executor
    base, sess, seg, seed = [], [], [], []
    for b in (0, 1, 1234567):
        for s in ("s0", "session-42", "slot:3"):
            for g in (-1, 0, 7):
                base.append(b)
                sess.append(s)
                seg.append(g)
                seed.append(ref_executor._stable_sampling_seed(b, s, g))
    np.savez_compressed(out, base=np.asarray(base, np.int64), session=np.asarray(sess),
                        segment=np.asarray(seg, np.int64), seed=np.asarray(seed, np.uint64))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    ap.add_argument("--skip-full", action="store_true")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    if args.only == "cfg1_long":  # oracle-only
        make_cfg1_long(HERE / "cfg1_long_greedy.npz")
        return
    if args.reference is None:
        ap.error("--reference is required")
    ref_mods = import_reference(args.reference.resolve())
    if args.only == "seeds":
        make_seeds(HERE / "seeds.npz")
        return
    if args.only == "code2wav":
        make_code2wav(args.reference.resolve(), HERE / "code2wav_tiny.npz")
        make_code2wav_chunked(args.reference.resolve(), HERE / "code2wav_chunked_tiny.npz")
        make_code2wav_warm(args.reference.resolve(), HERE / "code2wav_warm_tiny.npz")
        return
    if args.only == "code2wav_warm":
        make_code2wav_warm(args.reference.resolve(), HERE / "code2wav_warm_tiny.npz")
        return
    make_code2wav(args.reference.resolve(), HERE / "code2wav_tiny.npz")
    make_code2wav_chunked(args.reference.resolve(), HERE / "code2wav_chunked_tiny.npz")
    make_code2wav_warm(args.reference.resolve(), HERE / "code2wav_warm_tiny.npz")
    make_seeds(HERE / "seeds.npz")
    t0 = time.time()
    make_fused_tiny(ref_mods, HERE / "fused_tiny.npz")
    make_pool_ops(ref_mods, HERE / "pool_ops.npz")
    tiny = tiny_engine_config(num_layers=2)
    np.savez_compressed(HERE / "traj_tiny_sampled.npz",
                        **run_trajectory(ref_mods, tiny, seed=4, lengths=[5, 13, 21], steps=12, do_sample=True))
    np.savez_compressed(HERE / "traj_tiny_greedy.npz",
                        **run_trajectory(ref_mods, tiny, seed=4, lengths=[5, 13, 21], steps=12, do_sample=False))
    print(f"tiny fixtures done in {time.time() - t0:.1f}s", flush=True)
    if not args.skip_full:
        # the CPU reference case: full talker, seed 0, fp32, prompts {37,64,91,128}, 32 greedy steps
        t0 = time.time()
        r = run_trajectory(ref_mods, EngineConfig(), seed=0, lengths=[37, 64, 91, 128], steps=32, do_sample=False)
        r.pop("gumbel"); r.pop("cp_gumbel")
        np.savez_compressed(HERE / "cfg1_full_greedy.npz", **r)
        print(f"cfg1 done in {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
