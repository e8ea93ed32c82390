"""Streaming code2wav decoder, fp32 CPU restatement — TEST INFRASTRUCTURE ONLY.

Restates ``Code2WavStreamingWrapper.forward`` (scripts/export/code2wav_streaming.py:708-810)
with the reference's own state formats: a sliding-window KV cache per layer
(29-66; the executor keeps at most window-1 = 71 past frames,
engine/backend/executor.py:1415-1441), 17 causal-conv left contexts (73-93,
shapes 159-193) and 4 bias-free transposed-conv overlaps (96-138).  Weights
are the dicts of ``test_stateful_b200.weights.code2wav_param_specs``.
"""

from __future__ import annotations

import math
from typing import Dict, List

import torch
import torch.nn.functional as F

from .model import rms_norm

Tensor = torch.Tensor


def snake(x: Tensor, alpha: Tensor, beta: Tensor) -> Tensor:
    """SnakeBeta as patched for export (562-592): x + sin(x e^a)^2 e^-b, per channel."""
    a = torch.exp(alpha.float()).view(1, -1, 1)
    binv = torch.exp(-beta.float()).view(1, -1, 1)
    s = torch.sin(x * a)
    return x + s * s * binv


def causal_conv(x: Tensor, state: Tensor, w: Tensor, b: Tensor, dilation: int = 1, groups: int = 1):
    """streaming_causal_conv (73-93): conv(cat(state, x)); new state = last (k-1)*d columns."""
    full = torch.cat([state, x], dim=-1)
    out = F.conv1d(full, w.float(), b.float(), dilation=dilation, groups=groups)
    pad = (w.shape[-1] - 1) * dilation
    return out, full[..., -pad:]


def causal_transconv(x: Tensor, overlap: Tensor, w: Tensor, b: Tensor, stride: int):
    """streaming_causal_transconv (96-138): overlap-add of the bias-free tail."""
    raw = F.conv_transpose1d(x, w.float(), b.float(), stride=stride)
    rp = w.shape[-1] - stride
    if rp <= 0:
        return raw, overlap
    out = torch.cat([raw[..., :rp] + overlap, raw[..., rp:-rp]], dim=-1)
    return out, raw[..., -rp:] - b.float().view(1, -1, 1)


def rope_cos_sin(pos: Tensor, head_dim: int, theta: float):
    """_build_decoder_rope_embeddings_export (288-306), attention_scaling 1."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    f = pos.float().unsqueeze(-1) * inv.view(1, 1, -1)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos(), emb.sin()


def _rot(x: Tensor) -> Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


class Code2WavState:
    """Per-stream streaming state in the reference layouts (batch of one)."""

    def __init__(self, cfg):
        L, D0 = cfg.latent_dim, cfg.decoder_dim
        self.kv: List[tuple] = [(torch.zeros(1, cfg.kv_heads, 0, cfg.head_dim),
                                 torch.zeros(1, cfg.kv_heads, 0, cfg.head_dim)) for _ in range(cfg.num_layers)]
        convs = [(cfg.codebook_dim, 2), (L, 6), (L, 6), (L, 6)]
        for cin, cout, _ in cfg.block_dims():
            convs += [(cout, 6 * d) for d in cfg.dilations]
        convs.append((cfg.block_dims()[-1][1], 6))
        self.conv = [torch.zeros(1, c, k) for c, k in convs]
        self.trans = [torch.zeros(1, cout, s) for _, cout, s in cfg.block_dims()]
        self.frame = 0


def decode_chunk(W: Dict[str, Tensor], cfg, codes: Tensor, st: Code2WavState) -> Tensor:
    """One stream, ``codes [16, T]`` -> wav ``[T * 1920]``; updates ``st``.  A chunk of T
    frames sees at most window - T past frames plus the chunk's own frames causally.

    code2wav_streaming.py:708-810 with the quantizer table path (681-706), the
    transformer layer (367-391) and attention (323-364)."""
    T = codes.shape[-1]
    codes = codes.clamp(0, cfg.codebook_size - 1).long()       # export_09...:146
    first = W["c2w.rvq_first.codebook.0"].float()[codes[0]]     # [T, d]
    rest = sum(W[f"c2w.rvq_rest.codebook.{g}"].float()[codes[1 + g]] for g in range(cfg.num_codebooks - 1))
    q = F.conv1d(first.t().unsqueeze(0), W["c2w.rvq_first.output_proj.weight"].float(),
                 W["c2w.rvq_first.output_proj.bias"].float())
    q = q + F.conv1d(rest.t().unsqueeze(0), W["c2w.rvq_rest.output_proj.weight"].float(),
                     W["c2w.rvq_rest.output_proj.bias"].float())
    h, st.conv[0] = causal_conv(q, st.conv[0], W["c2w.pre_conv.weight"], W["c2w.pre_conv.bias"])
    # ---- transformer with a sliding-window cache
    p = "c2w.pre_transformer."
    x = F.linear(h.transpose(1, 2), W[p + "input_proj.weight"].float(), W[p + "input_proj.bias"].float())
    pos = torch.arange(st.frame, st.frame + T).unsqueeze(0)
    cos, sin = rope_cos_sin(pos, cfg.head_dim, cfg.rope_theta)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    # past + chunk keys must fit the window: the caller keeps at most window - T past frames
    # (executor.py:1374-1380 with FUSED_CHUNK_T = T)
    st.kv = [(k[:, :, -(cfg.window - T):] if T < cfg.window else k[:, :, :0],
              v[:, :, -(cfg.window - T):] if T < cfg.window else v[:, :, :0]) for k, v in st.kv]
    P = st.kv[0][0].shape[2]
    cols = torch.arange(P + T)
    rows = torch.arange(T).unsqueeze(1) + P
    mask = torch.where(cols.unsqueeze(0) > rows, float("-inf"), 0.0).view(1, 1, T, P + T)
    nh, hd = cfg.num_heads, cfg.head_dim
    for i in range(cfg.num_layers):
        q_ = f"{p}layers.{i}."
        n = rms_norm(x, W[q_ + "input_layernorm.weight"], cfg.rms_eps)
        qq = F.linear(n, W[q_ + "self_attn.q_proj.weight"].float()).view(1, T, nh, hd)
        kk = F.linear(n, W[q_ + "self_attn.k_proj.weight"].float()).view(1, T, cfg.kv_heads, hd)
        vv = F.linear(n, W[q_ + "self_attn.v_proj.weight"].float()).view(1, T, cfg.kv_heads, hd).transpose(1, 2)
        qq = rms_norm(qq, W[q_ + "self_attn.q_norm.weight"], cfg.rms_eps).transpose(1, 2)
        kk = rms_norm(kk, W[q_ + "self_attn.k_norm.weight"], cfg.rms_eps).transpose(1, 2)
        qq = qq * cos + _rot(qq) * sin
        kk = kk * cos + _rot(kk) * sin
        pk, pv = st.kv[i]
        fk, fv = torch.cat([pk, kk], dim=2), torch.cat([pv, vv], dim=2)
        rep = nh // cfg.kv_heads
        a = torch.softmax(qq @ fk.repeat_interleave(rep, 1).transpose(2, 3) / math.sqrt(hd) + mask, dim=-1)
        o = (a @ fv.repeat_interleave(rep, 1)).transpose(1, 2).reshape(1, T, nh * hd)
        o = F.linear(o, W[q_ + "self_attn.o_proj.weight"].float())
        x = x + W[q_ + "self_attn_layer_scale.scale"].float() * o
        n = rms_norm(x, W[q_ + "post_attention_layernorm.weight"], cfg.rms_eps)
        m = F.linear(F.silu(F.linear(n, W[q_ + "mlp.gate_proj.weight"].float()))
                     * F.linear(n, W[q_ + "mlp.up_proj.weight"].float()), W[q_ + "mlp.down_proj.weight"].float())
        x = x + W[q_ + "mlp_layer_scale.scale"].float() * m
        keep = cfg.window - 1  # at most window - 1 past frames are ever visible (T >= 1)
        st.kv[i] = (fk[:, :, -keep:], fv[:, :, -keep:])
    x = rms_norm(x, W[p + "norm.weight"], cfg.rms_eps)
    h = F.linear(x, W[p + "output_proj.weight"].float(), W[p + "output_proj.bias"].float()).transpose(1, 2)
    # ---- upsampling: transposed conv (2, 2) + ConvNeXt (812-832)
    for i, s in enumerate(cfg.upsample_ratios):
        u = f"c2w.upsample.{i}."
        h, _ = causal_transconv(h, None, W[u + "transconv.weight"], W[u + "transconv.bias"], s)
        inp = h
        h, st.conv[1 + i] = causal_conv(h, st.conv[1 + i], W[u + "convnext.dwconv.weight"],
                                        W[u + "convnext.dwconv.bias"], groups=h.shape[1])
        h = h.transpose(1, 2)
        h = F.layer_norm(h, (h.shape[-1],), W[u + "convnext.norm.weight"].float(),
                         W[u + "convnext.norm.bias"].float(), cfg.ln_eps)
        h = F.gelu(F.linear(h, W[u + "convnext.pwconv1.weight"].float(), W[u + "convnext.pwconv1.bias"].float()))
        h = F.linear(h, W[u + "convnext.pwconv2.weight"].float(), W[u + "convnext.pwconv2.bias"].float())
        h = (W[u + "convnext.gamma"].float() * h).transpose(1, 2)
        h = inp + h
    # ---- decoder (783-799, blocks 834-856)
    h, st.conv[3] = causal_conv(h, st.conv[3], W["c2w.decoder.0.weight"], W["c2w.decoder.0.bias"])
    for b, (cin, cout, s) in enumerate(cfg.block_dims()):
        k = f"c2w.decoder.{1 + b}."
        h = snake(h, W[k + "snake.alpha"], W[k + "snake.beta"])
        h, st.trans[b] = causal_transconv(h, st.trans[b], W[k + "transconv.weight"], W[k + "transconv.bias"], s)
        for j, d in enumerate(cfg.dilations):
            r = f"{k}res.{j}."
            res = h
            t = snake(h, W[r + "act1.alpha"], W[r + "act1.beta"])
            t, st.conv[4 + 3 * b + j] = causal_conv(t, st.conv[4 + 3 * b + j], W[r + "conv1.weight"],
                                                   W[r + "conv1.bias"], dilation=d)
            t = snake(t, W[r + "act2.alpha"], W[r + "act2.beta"])
            t = F.conv1d(t, W[r + "conv2.weight"].float(), W[r + "conv2.bias"].float())
            h = res + t
    h = snake(h, W["c2w.decoder.5.alpha"], W["c2w.decoder.5.beta"])
    wav, st.conv[16] = causal_conv(h, st.conv[16], W["c2w.decoder.6.weight"], W["c2w.decoder.6.bias"])
    st.frame += T
    return wav.reshape(-1).clamp(-1.0, 1.0)
