"""Seeded random-init weights for the talker and the code predictor.

There is no network and no checkpoint, so every run (tests, fixtures, bench)
uses random-init weights of the reference architecture.  Each tensor gets its
own generator seeded from ``(seed, name)`` through a stable hash, so any subset
of the model (for example the first four layers) holds the same values as the
full model, on any machine with this torch build.  The values depend on the
generator's device: tensors made with ``device="cuda"`` (fast, used by the
benchmark) differ from the CPU ones the oracle and the parity tests use.

Names follow the module paths the reference reads:
``talker.layers.{i}.self_attn.q_proj.weight`` etc. mirror
``talker_model.layers[i].self_attn.q_proj`` (scripts/export/talker_unified_modules.py:170-228),
``cp.*`` mirrors ``CodePredictorUnrolled`` (scripts/export/utils.py:867-881).
"""

from __future__ import annotations

import hashlib
from typing import Dict, Iterator, Tuple

import torch

from .config import CodePredictorConfig, TalkerConfig

LINEAR_STD = 0.02
EMBED_STD = 0.02
NORM_JITTER = 0.05


def _tensor_seed(seed: int, name: str) -> int:
    h = hashlib.blake2b(digest_size=8)
    h.update(str(int(seed)).encode())
    h.update(b"\0")
    h.update(name.encode())
    return int.from_bytes(h.digest(), "little") & ((1 << 63) - 1)


def talker_param_specs(cfg: TalkerConfig, layers=None) -> Iterator[Tuple[str, tuple, str]]:
    """(name, shape, kind) for every talker tensor; kind is linear/embed/norm."""
    H, D = cfg.hidden_size, cfg.head_dim
    yield "talker.codec_embedding.weight", (cfg.codec_vocab_size, H), "embed"
    for i in (range(cfg.num_layers) if layers is None else layers):
        p = f"talker.layers.{i}."
        yield p + "input_layernorm.weight", (H,), "norm"
        yield p + "self_attn.q_proj.weight", (cfg.q_size, H), "linear"
        yield p + "self_attn.k_proj.weight", (cfg.kv_size, H), "linear"
        yield p + "self_attn.v_proj.weight", (cfg.kv_size, H), "linear"
        yield p + "self_attn.o_proj.weight", (H, cfg.q_size), "linear"
        yield p + "self_attn.q_norm.weight", (D,), "norm"
        yield p + "self_attn.k_norm.weight", (D,), "norm"
        yield p + "post_attention_layernorm.weight", (H,), "norm"
        yield p + "mlp.gate_proj.weight", (cfg.intermediate_size, H), "linear"
        yield p + "mlp.up_proj.weight", (cfg.intermediate_size, H), "linear"
        yield p + "mlp.down_proj.weight", (H, cfg.intermediate_size), "linear"
    yield "talker.norm.weight", (H,), "norm"
    yield "talker.codec_head.weight", (cfg.codec_vocab_size, H), "linear"


def cp_param_specs(cfg: CodePredictorConfig) -> Iterator[Tuple[str, tuple, str]]:
    H, D = cfg.hidden_size, cfg.head_dim
    yield "cp.projection.weight", (H, cfg.talker_hidden_size), "linear"
    yield "cp.projection.bias", (H,), "bias"
    for s in range(cfg.num_stages):
        yield f"cp.codec_embedding.{s}.weight", (cfg.vocab_size, cfg.talker_hidden_size), "embed"
    for i in range(cfg.num_layers):
        p = f"cp.layers.{i}."
        yield p + "input_layernorm.weight", (H,), "norm"
        yield p + "self_attn.q_proj.weight", (cfg.num_heads * D, H), "linear"
        yield p + "self_attn.k_proj.weight", (cfg.kv_heads * D, H), "linear"
        yield p + "self_attn.v_proj.weight", (cfg.kv_heads * D, H), "linear"
        yield p + "self_attn.o_proj.weight", (H, cfg.num_heads * D), "linear"
        yield p + "self_attn.q_norm.weight", (D,), "norm"
        yield p + "self_attn.k_norm.weight", (D,), "norm"
        yield p + "post_attention_layernorm.weight", (H,), "norm"
        yield p + "mlp.gate_proj.weight", (cfg.intermediate_size, H), "linear"
        yield p + "mlp.up_proj.weight", (cfg.intermediate_size, H), "linear"
        yield p + "mlp.down_proj.weight", (H, cfg.intermediate_size), "linear"
    yield "cp.norm.weight", (H,), "norm"
    for s in range(cfg.num_stages):
        yield f"cp.lm_head.{s}.weight", (cfg.vocab_size, H), "linear"


def code2wav_param_specs(cfg) -> Iterator[Tuple[str, tuple, object]]:
    """Decoder tensors, named after the module paths code2wav_streaming.py reads
    (``decoder.quantizer.rvq_first``, ``decoder.pre_conv``, ``decoder.pre_transformer``,
    ``decoder.upsample[i]``, ``decoder.decoder[j]``).  Conv weights use the
    torch layouts (Conv1d ``[out, in, k]``, ConvTranspose1d ``[in, out, k]``) and
    a 1/sqrt(fan-in) scale so the signal stays O(1) through the stack; the last
    conv is scaled down so the waveform sits inside the [-1, 1] clamp."""
    V, d, cd, L, H = cfg.codebook_size, cfg.vq_dim, cfg.codebook_dim, cfg.latent_dim, cfg.hidden_size
    hd, I = cfg.head_dim, cfg.intermediate_size

    def conv(out_c, in_c, k, gain=1.0):
        return ("normal", gain / (in_c * k) ** 0.5, 0.0)

    def small(std):
        return ("normal", std, 0.0)

    yield "c2w.rvq_first.codebook.0", (V, d), small(1.0)
    for i in range(cfg.num_codebooks - 1):
        yield f"c2w.rvq_rest.codebook.{i}", (V, d), small(1.0)
    for part in ("rvq_first", "rvq_rest"):
        yield f"c2w.{part}.output_proj.weight", (cd, d, 1), conv(cd, d, 1)
        yield f"c2w.{part}.output_proj.bias", (cd,), small(0.02)
    yield "c2w.pre_conv.weight", (L, cd, 3), conv(L, cd, 3)
    yield "c2w.pre_conv.bias", (L,), small(0.02)
    p = "c2w.pre_transformer."
    yield p + "input_proj.weight", (H, L), conv(H, L, 1)
    yield p + "input_proj.bias", (H,), small(0.02)
    for i in range(cfg.num_layers):
        q = f"{p}layers.{i}."
        yield q + "input_layernorm.weight", (H,), "norm"
        yield q + "self_attn.q_proj.weight", (cfg.num_heads * hd, H), conv(0, H, 1)
        yield q + "self_attn.k_proj.weight", (cfg.kv_heads * hd, H), conv(0, H, 1)
        yield q + "self_attn.v_proj.weight", (cfg.kv_heads * hd, H), conv(0, H, 1)
        yield q + "self_attn.o_proj.weight", (H, cfg.num_heads * hd), conv(0, cfg.num_heads * hd, 1)
        yield q + "self_attn.q_norm.weight", (hd,), "norm"
        yield q + "self_attn.k_norm.weight", (hd,), "norm"
        yield q + "self_attn_layer_scale.scale", (H,), ("normal", 0.02, 0.1)
        yield q + "post_attention_layernorm.weight", (H,), "norm"
        yield q + "mlp.gate_proj.weight", (I, H), conv(0, H, 1)
        yield q + "mlp.up_proj.weight", (I, H), conv(0, H, 1)
        yield q + "mlp.down_proj.weight", (H, I), conv(0, I, 1)
        yield q + "mlp_layer_scale.scale", (H,), ("normal", 0.02, 0.1)
    yield p + "norm.weight", (H,), "norm"
    yield p + "output_proj.weight", (L, H), conv(L, H, 1)
    yield p + "output_proj.bias", (L,), small(0.02)
    for i, _ in enumerate(cfg.upsample_ratios):
        u = f"c2w.upsample.{i}."
        yield u + "transconv.weight", (L, L, 2), conv(L, L, 1)
        yield u + "transconv.bias", (L,), small(0.02)
        yield u + "convnext.dwconv.weight", (L, 1, 7), conv(L, 1, 7)
        yield u + "convnext.dwconv.bias", (L,), small(0.02)
        yield u + "convnext.norm.weight", (L,), "norm"
        yield u + "convnext.norm.bias", (L,), small(0.02)
        yield u + "convnext.pwconv1.weight", (cfg.convnext_mult * L, L), conv(0, L, 1)
        yield u + "convnext.pwconv1.bias", (cfg.convnext_mult * L,), small(0.02)
        yield u + "convnext.pwconv2.weight", (L, cfg.convnext_mult * L), conv(0, cfg.convnext_mult * L, 1)
        yield u + "convnext.pwconv2.bias", (L,), small(0.02)
        yield u + "convnext.gamma", (L,), ("normal", 0.02, 0.1)
    D0 = cfg.decoder_dim
    yield "c2w.decoder.0.weight", (D0, L, 7), conv(D0, L, 7)
    yield "c2w.decoder.0.bias", (D0,), small(0.02)
    for b, (cin, cout, s) in enumerate(cfg.block_dims()):
        k = f"c2w.decoder.{1 + b}."
        yield k + "snake.alpha", (cin,), small(0.1)
        yield k + "snake.beta", (cin,), small(0.1)
        yield k + "transconv.weight", (cin, cout, 2 * s), conv(cout, cin, 2)
        yield k + "transconv.bias", (cout,), small(0.02)
        for j, _ in enumerate(cfg.dilations):
            r = f"{k}res.{j}."
            yield r + "act1.alpha", (cout,), small(0.1)
            yield r + "act1.beta", (cout,), small(0.1)
            yield r + "conv1.weight", (cout, cout, 7), conv(cout, cout, 7, 0.5)
            yield r + "conv1.bias", (cout,), small(0.02)
            yield r + "act2.alpha", (cout,), small(0.1)
            yield r + "act2.beta", (cout,), small(0.1)
            yield r + "conv2.weight", (cout, cout, 1), conv(cout, cout, 1, 0.5)
            yield r + "conv2.bias", (cout,), small(0.02)
    last = cfg.block_dims()[-1][1]
    yield "c2w.decoder.5.alpha", (last,), small(0.1)
    yield "c2w.decoder.5.beta", (last,), small(0.1)
    yield "c2w.decoder.6.weight", (1, last, 7), conv(1, last, 7, 0.1)
    yield "c2w.decoder.6.bias", (1,), small(0.01)


def make_code2wav_weights(cfg, seed: int, device="cpu", dtype=torch.bfloat16):
    return make_weights(code2wav_param_specs(cfg), seed, device, dtype)


def _make(name: str, shape: tuple, kind, seed: int, device, dtype) -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(_tensor_seed(seed, name))
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if isinstance(kind, tuple):  # ("normal", std, mean)
        t.mul_(kind[1]).add_(kind[2])
    elif kind == "linear":
        t.mul_(LINEAR_STD)
    elif kind == "embed":
        t.mul_(EMBED_STD)
    elif kind == "bias":
        t.mul_(LINEAR_STD)
    elif kind == "norm":
        t.mul_(NORM_JITTER).add_(1.0)
    return t.to(dtype)


def make_weights(specs, seed: int, device="cpu", dtype=torch.bfloat16) -> Dict[str, torch.Tensor]:
    """Materialise every tensor of ``specs``.

    With ``dtype=torch.bfloat16`` the values are the ones the B200 path runs
    on; the oracle uses the same bf16 values widened to fp32 so that a parity
    test measures kernel error and not weight rounding.
    """
    return {name: _make(name, shape, kind, seed, device, dtype) for name, shape, kind in specs}


def make_talker_weights(cfg: TalkerConfig, seed: int, device="cpu", dtype=torch.bfloat16, layers=None):
    return make_weights(talker_param_specs(cfg, layers), seed, device, dtype)


def make_cp_weights(cfg: CodePredictorConfig, seed: int, device="cpu", dtype=torch.bfloat16):
    return make_weights(cp_param_specs(cfg), seed, device, dtype)


def to_fp32(weights: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    return {k: v.float() for k, v in weights.items()}
