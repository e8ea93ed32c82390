"""fp32 CPU restatement of the talker, sampling head, code predictor and codec sum.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Each function cites the reference lines it restates.  Weights are the dicts
produced by ``test_stateful_b200.weights`` (HF-style names), widened to fp32.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

Tensor = torch.Tensor


# ----------------------------------------------------------------------------
# building blocks
# ----------------------------------------------------------------------------

def rms_norm(x: Tensor, w: Tensor, eps: float) -> Tensor:
    """Qwen3RMSNorm in fp32: ``w * x * rsqrt(mean(x^2) + eps)``."""
    x32 = x.float()
    var = x32.pow(2).mean(-1, keepdim=True)
    return w.float() * (x32 * torch.rsqrt(var + eps))


def rope_cos_sin(positions: Tensor, head_dim: int, theta: float) -> Tuple[Tensor, Tensor]:
    """cos/sin tables ``[B, S, D]`` for integer positions ``[B, S]``.

    talker_unified_modules.py:87-108 builds ``freqs = pos * inv_freq`` and
    ``emb = cat(freqs, freqs)``; the three mRoPE axes carry the same position
    (engine/backend/executor.py:1290-1296), so the section mix at 111-139
    selects identical values and the result is standard RoPE.
    """
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = positions.to(torch.float32).unsqueeze(-1) * inv_freq.view(1, 1, -1)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: Tensor) -> Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """``x [B, h, S, D]``, ``cos/sin [B, S, D]`` (talker_unified_modules.py:142-156)."""
    return x * cos.unsqueeze(1) + rotate_half(x) * sin.unsqueeze(1)


def linear(x: Tensor, w: Tensor, b: Optional[Tensor] = None) -> Tensor:
    return F.linear(x, w, b)


# ----------------------------------------------------------------------------
# talker (TalkerUnifiedONNX.forward, talker_unified_modules.py:243-320)
# ----------------------------------------------------------------------------

def _attention_layer(W: Dict[str, Tensor], p: str, x: Tensor, cos: Tensor, sin: Tensor,
                     past_k: Tensor, past_v: Tensor, mask: Tensor, n_heads: int, n_kv: int,
                     head_dim: int, eps: float) -> Tuple[Tensor, Tensor, Tensor]:
    """talker_unified_modules.py:159-201 (and utils.py:919-945 for the predictor)."""
    B, S, _ = x.shape
    q = linear(x, W[p + "self_attn.q_proj.weight"]).view(B, S, n_heads, head_dim)
    k = linear(x, W[p + "self_attn.k_proj.weight"]).view(B, S, n_kv, head_dim)
    v = linear(x, W[p + "self_attn.v_proj.weight"]).view(B, S, n_kv, head_dim)
    q = rms_norm(q, W[p + "self_attn.q_norm.weight"], eps).transpose(1, 2)
    k = rms_norm(k, W[p + "self_attn.k_norm.weight"], eps).transpose(1, 2)
    v = v.transpose(1, 2)
    q = apply_rope(q, cos, sin)
    k = apply_rope(k, cos, sin)
    full_k = torch.cat([past_k, k], dim=2)
    full_v = torch.cat([past_v, v], dim=2)
    rep = n_heads // n_kv
    kk = full_k.repeat_interleave(rep, dim=1)
    vv = full_v.repeat_interleave(rep, dim=1)
    scores = torch.matmul(q, kk.transpose(2, 3)) * (head_dim ** -0.5) + mask
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32)
    o = torch.matmul(probs, vv).transpose(1, 2).reshape(B, S, n_heads * head_dim)
    return linear(o, W[p + "self_attn.o_proj.weight"]), k, v


def _mlp(W: Dict[str, Tensor], p: str, x: Tensor) -> Tensor:
    g = linear(x, W[p + "mlp.gate_proj.weight"])
    u = linear(x, W[p + "mlp.up_proj.weight"])
    return linear(F.silu(g) * u, W[p + "mlp.down_proj.weight"])


def ragged_mask(past_lens: Sequence[int], padded_past: int, S: int) -> Tensor:
    """Additive mask ``[B, 1, S, P+S]``.

    Padding columns ``past_len_b <= j < P`` are masked
    (engine/backend/batch_helper.py:48-66) and so are causal-future columns
    (talker_unified_modules.py:282-288).
    """
    B = len(past_lens)
    total = padded_past + S
    mask = torch.zeros(B, 1, S, total)
    cols = torch.arange(total)
    for b, pl in enumerate(past_lens):
        pad = (cols < padded_past) & (cols >= int(pl))
        mask[b, 0, :, pad] = float("-inf")
    rows = torch.arange(S).unsqueeze(1) + padded_past
    causal = cols.unsqueeze(0) > rows
    mask = mask.masked_fill(causal.view(1, 1, S, total), float("-inf"))
    return mask


def talker_forward(W: Dict[str, Tensor], cfg, embeds: Tensor, positions: Tensor,
                   past_k: List[Tensor], past_v: List[Tensor], past_lens: Sequence[int]):
    """One talker pass over ``S`` new tokens per stream.

    ``embeds [B, S, H]``, ``positions [B, S]`` (position_offset + past_len + i),
    ``past_k/v[l] [B, Hkv, P, D]`` padded to a common ``P`` with ``past_lens``
    valid entries.  Returns ``(hidden_norm [B,S,H], logits [B,S,V],
    new_k[l] [B,Hkv,S,D], new_v[l])`` like the delta-KV outputs of
    talker_unified_modules.py:309-320.
    """
    B, S, _ = embeds.shape
    P = past_k[0].shape[2] if past_k else 0
    cos, sin = rope_cos_sin(positions, cfg.head_dim, cfg.rope_theta)
    mask = ragged_mask(past_lens, P, S)
    x = embeds.float()
    new_k, new_v = [], []
    for i in range(cfg.num_layers):
        p = f"talker.layers.{i}."
        h = rms_norm(x, W[p + "input_layernorm.weight"], cfg.rms_eps)
        a, k, v = _attention_layer(W, p, h, cos, sin, past_k[i], past_v[i], mask,
                                   cfg.num_heads, cfg.kv_heads, cfg.head_dim, cfg.rms_eps)
        x = x + a
        h = rms_norm(x, W[p + "post_attention_layernorm.weight"], cfg.rms_eps)
        x = x + _mlp(W, p, h)
        new_k.append(k)
        new_v.append(v)
    hidden = rms_norm(x, W["talker.norm.weight"], cfg.rms_eps)
    logits = linear(hidden, W["talker.codec_head.weight"])
    return hidden, logits, new_k, new_v


# ----------------------------------------------------------------------------
# sampling head (TalkerUnifiedFusedONNX.forward, talker_unified_modules.py:349-388)
# ----------------------------------------------------------------------------

def suppress_mask(vocab: int, eos_id: int) -> Tensor:
    """talker_unified_modules.py:349-355: ids ``[V-1024, V)`` except EOS."""
    m = torch.zeros(vocab, dtype=torch.bool)
    m[vocab - 1024:] = True
    m[eos_id] = False
    return m


def talker_sample(logits_last: Tensor, token_counts: Tensor, gumbel: Tensor, temperature: Tensor,
                  penalty: Tensor, eos_id: int, topk: int = 50) -> Tuple[Tensor, Tensor]:
    """Suppress → repetition penalty → top-k → /T → +Gumbel → argmax → counts += 1.

    ``logits_last [B, V]`` fp32, ``token_counts [B, V]`` int64,
    ``gumbel [B, topk]``, ``temperature/penalty [B, 1]``.
    """
    V = logits_last.shape[-1]
    g0 = logits_last.float().masked_fill(suppress_mask(V, eos_id), -1e9)
    penalized = torch.where(g0 > 0, g0 / penalty, g0 * penalty)
    g0 = torch.where(token_counts > 0, penalized, g0)
    vals, idx = g0.topk(topk, dim=-1)
    vals = vals / temperature
    sel = (vals + gumbel).argmax(dim=-1)
    tok = idx.gather(1, sel.unsqueeze(1)).squeeze(1)
    counts = token_counts + F.one_hot(tok, V).to(token_counts.dtype)
    return tok, counts


def topk_select(logits: Tensor, temperature: Tensor, gumbel: Optional[Tensor], topk: int = 50) -> Tensor:
    """CodePredictorUnrolled._select_token (utils.py:986-1001)."""
    if gumbel is None:
        return logits.argmax(dim=-1)
    k = min(topk, logits.shape[-1])
    vals, idx = logits.topk(k, dim=-1)
    sel = (vals / temperature + gumbel[:, :k]).argmax(dim=-1)
    return idx.gather(1, sel.unsqueeze(1)).squeeze(1)


# ----------------------------------------------------------------------------
# code predictor (CodePredictorUnrolled, utils.py:852-1042)
# ----------------------------------------------------------------------------

def cp_transformer(W: Dict[str, Tensor], cfg, x: Tensor) -> Tensor:
    """utils.py:962-984: full causal pass over ``x [B, S, H]``, positions 0..S-1."""
    B, S, _ = x.shape
    pos = torch.arange(S).unsqueeze(0).expand(B, S)
    cos, sin = rope_cos_sin(pos, cfg.head_dim, cfg.rope_theta)
    mask = ragged_mask([0] * B, 0, S)
    empty = torch.zeros(B, cfg.kv_heads, 0, cfg.head_dim)
    h = x.float()
    for i in range(cfg.num_layers):
        p = f"cp.layers.{i}."
        n = rms_norm(h, W[p + "input_layernorm.weight"], cfg.rms_eps)
        a, _, _ = _attention_layer(W, p, n, cos, sin, empty, empty, mask,
                                   cfg.num_heads, cfg.kv_heads, cfg.head_dim, cfg.rms_eps)
        h = h + a
        n = rms_norm(h, W[p + "post_attention_layernorm.weight"], cfg.rms_eps)
        h = h + _mlp(W, p, n)
    return rms_norm(h, W["cp.norm.weight"], cfg.rms_eps)


def code_predictor(W: Dict[str, Tensor], cfg, talker_codec_emb: Tensor, past_hidden: Tensor,
                   tok0: Tensor, cp_gumbel: Optional[Tensor], temperature: Optional[Tensor],
                   force: Optional[Tensor] = None, stage_logits: Optional[list] = None) -> Tensor:
    """utils.py:1003-1042 (full recompute each stage, exactly as the reference).

    ``past_hidden [B, 1, Ht]`` is the talker's normalised last hidden state,
    ``tok0 [B]``; returns ``[B, num_stages]`` int64.  Test hooks: ``force
    [B, 1+num_stages]`` feeds stage ``s+1`` the token ``force[:, s+1]`` instead
    of the sampled one (teacher forcing); ``stage_logits`` collects each
    stage's logits.
    """
    proj_w, proj_b = W["cp.projection.weight"], W["cp.projection.bias"]
    e0 = talker_codec_emb[tok0].unsqueeze(1)
    seq = linear(torch.cat([past_hidden.float(), e0], dim=1), proj_w, proj_b)
    out = []
    for s in range(cfg.num_stages):
        h = cp_transformer(W, cfg, seq)
        logits = linear(h[:, -1, :], W[f"cp.lm_head.{s}.weight"])
        if stage_logits is not None:
            stage_logits.append(logits)
        noise = None if cp_gumbel is None else cp_gumbel[:, s, :]
        tok = topk_select(logits, temperature, noise, cfg.logits_topk)
        out.append(tok)
        if s < cfg.num_stages - 1:
            nxt = tok if force is None else force[:, s + 1]
            e = W[f"cp.codec_embedding.{s}.weight"][nxt].unsqueeze(1)
            seq = torch.cat([seq, linear(e, proj_w, proj_b)], dim=1)
    return torch.stack(out, dim=1)


# ----------------------------------------------------------------------------
# codec embedding sum (scripts/python/codec_embedding_sum.py:25-83)
# ----------------------------------------------------------------------------

def stacked_codec_table(W: Dict[str, Tensor], num_stages: int) -> Tensor:
    """[16, V_talker, H]: talker table then the CP tables zero-padded (25-53)."""
    t = W["talker.codec_embedding.weight"].float()
    parts = [t]
    for s in range(num_stages):
        w = W[f"cp.codec_embedding.{s}.weight"].float()
        pad = torch.zeros_like(t)
        pad[: w.shape[0]] = w
        parts.append(pad)
    return torch.stack(parts, dim=0)


def codec_sum(table: Tensor, codes: Tensor) -> Tensor:
    """``Σ_g table[g, codes[:, g]]`` (codec_embedding_sum.py:71-83)."""
    G = codes.shape[1]
    g = torch.arange(G).unsqueeze(0).expand(codes.shape[0], G)
    return table[g, codes].sum(dim=1)


# ----------------------------------------------------------------------------
# one fused decode step (TalkerUnifiedFusedONNX.forward + codec sum)
# ----------------------------------------------------------------------------

def fused_step(W, tcfg, ccfg, embeds, positions, past_k, past_v, past_lens, token_counts,
               gumbel, cp_gumbel, temperature, penalty, table=None, force=None):
    """talker_unified_modules.py:357-401 for ``S`` new tokens per stream.

    Returns a dict with ``hidden, logits, new_k, new_v, tok0, counts,
    cp_tokens, full_codec, codec_sum``.  Test hook: ``force [B, 1+num_stages]``
    makes the code predictor consume ``force[:, 0]`` as tok0 and ``force[:, s]``
    after stage s-1 (teacher forcing); the returned tokens are still this
    step's own samples, and ``counts`` is updated with them.
    """
    hidden, logits, new_k, new_v = talker_forward(W, tcfg, embeds, positions, past_k, past_v, past_lens)
    tok0, counts = talker_sample(logits[:, -1, :], token_counts, gumbel, temperature, penalty,
                                 tcfg.codec_eos_id, tcfg.logits_topk)
    cp_tok = code_predictor(W, ccfg, W["talker.codec_embedding.weight"], hidden[:, -1:, :],
                            tok0 if force is None else force[:, 0], cp_gumbel, temperature, force=force)
    full = torch.cat([tok0.unsqueeze(1), cp_tok], dim=1)
    if table is None:
        table = stacked_codec_table(W, ccfg.num_stages)
    csum = codec_sum(table, full)
    return dict(hidden=hidden, logits=logits, new_k=new_k, new_v=new_v, tok0=tok0, counts=counts,
                cp_tokens=cp_tok, full_codec=full, codec_sum=csum)


def gumbel_from_uniform(u: Tensor) -> Tensor:
    """engine/backend/executor.py:1238-1251: ``-log(-log(clamp(u, 1e-8, 1)))``."""
    u = u.clamp(1e-8, 1.0)
    return -torch.log(-torch.log(u))
