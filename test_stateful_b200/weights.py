"""Seeded random-init weights for the talker and the code predictor.

There is no network and no checkpoint, so every run (tests, fixtures, bench)
uses random-init weights of the reference architecture.  Each tensor gets its
own generator seeded from ``(seed, name)`` through a stable hash, so any subset
of the model (for example the first four layers) holds the same values as the
full model, on any machine with this torch build.

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


def _make(name: str, shape: tuple, kind: str, seed: int, device, dtype) -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(_tensor_seed(seed, name))
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if kind == "linear":
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
