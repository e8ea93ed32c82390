"""Model and pool configuration for the B200 decode backend.

The field names follow the reference's ``ModelConfig``
(engine/backend/kv_cache_pool.py:36-60) so that a ``b200`` backend can be
constructed from the same manifest values.  Two groups are added that the
reference keeps inside its TensorRT plan: the code-predictor architecture
(scripts/export/utils.py:852-1042) and the paged-KV pool geometry, which has
no counterpart in the slot-contiguous reference pool.
"""

from __future__ import annotations

from dataclasses import dataclass, field, asdict


@dataclass
class TalkerConfig:
    """Qwen3 talker (scripts/export/talker_unified_modules.py:231-320)."""

    num_layers: int = 28
    hidden_size: int = 2048
    num_heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 6144
    codec_vocab_size: int = 3072
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6
    codec_eos_id: int = 2150
    logits_topk: int = 50

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def kv_bytes_per_token(self) -> int:
        """K+V bytes of one token over all layers, bf16."""
        return self.num_layers * 2 * self.kv_heads * self.head_dim * 2


@dataclass
class CodePredictorConfig:
    """15-stage residual codebook predictor (scripts/export/utils.py:852-1042)."""

    num_layers: int = 5
    hidden_size: int = 1024
    num_heads: int = 16
    kv_heads: int = 8
    head_dim: int = 64
    intermediate_size: int = 3072
    vocab_size: int = 2048
    num_stages: int = 15
    talker_hidden_size: int = 2048
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6
    logits_topk: int = 50

    @property
    def max_seq(self) -> int:
        # positions 0..num_stages: [h_last, emb(tok0), emb_1(t1), ...]
        return self.num_stages + 1


@dataclass
class Code2WavConfig:
    """Streaming code2wav decoder (scripts/export/code2wav_streaming.py:595-856).

    Fixed by the reference: 16 codebooks of 2048 entries (1 semantic + 15
    acoustic, codes clamped to 2047 — export_09_talker_code2wav_fused.py:146),
    codebook_dim 512, latent 1024, hidden 1024, 8 layers, 16 kv heads x 64,
    window 72, decoder_dim 1536, upsampling (2, 2) then strides (8, 5, 4, 3),
    residual dilations (1, 3, 9) (code2wav_streaming.py:159-193,
    docs/code2wav_state_size.md, tests/unit/test_conv1d_subpixel.py:98-104).
    Not fixed by any reference file (the qwen_tts decoder is absent), chosen
    here: RVQ vector width 256, SwiGLU MLP 3072, ConvNeXt expansion 4 with
    GELU, RMSNorm eps 1e-5, LayerNorm eps 1e-6, RoPE theta 10000.
    """

    num_codebooks: int = 16
    codebook_size: int = 2048
    vq_dim: int = 256
    codebook_dim: int = 512
    latent_dim: int = 1024
    hidden_size: int = 1024
    num_layers: int = 8
    num_heads: int = 16
    kv_heads: int = 16
    head_dim: int = 64
    intermediate_size: int = 3072
    window: int = 72
    rms_eps: float = 1.0e-5
    rope_theta: float = 10000.0
    decoder_dim: int = 1536
    upsample_ratios: tuple = (2, 2)
    upsample_rates: tuple = (8, 5, 4, 3)
    dilations: tuple = (1, 3, 9)
    convnext_mult: int = 4
    ln_eps: float = 1.0e-6

    @property
    def samples_per_frame(self) -> int:
        n = 1
        for r in tuple(self.upsample_ratios) + tuple(self.upsample_rates):
            n *= r
        return n

    def block_dims(self):
        """(in, out, stride) of the four decoder blocks."""
        out = []
        for b, s in enumerate(self.upsample_rates):
            out.append((self.decoder_dim // (2 ** b), self.decoder_dim // (2 ** (b + 1)), s))
        return out


def tiny_code2wav_config() -> Code2WavConfig:
    """Narrow channels, same strides/kernels/window: the fixture configuration.
    Widths stay multiples of the GEMM tiles where the full model's are
    (projections of 128, head_dim 32, decoder channels multiples of 8)."""
    return Code2WavConfig(vq_dim=16, codebook_dim=64, latent_dim=128, hidden_size=128, num_layers=2, num_heads=4,
                          kv_heads=4, head_dim=32, intermediate_size=256, decoder_dim=128, convnext_mult=2)


@dataclass
class PagedPoolConfig:
    """Geometry of the paged talker KV pool (no counterpart in the reference)."""

    block_size: int = 16
    num_blocks: int = 8192
    max_slots: int = 64
    max_seq_len: int = 1024

    @property
    def max_blocks_per_seq(self) -> int:
        return (self.max_seq_len + self.block_size - 1) // self.block_size


@dataclass
class EngineConfig:
    talker: TalkerConfig = field(default_factory=TalkerConfig)
    cp: CodePredictorConfig = field(default_factory=CodePredictorConfig)
    pool: PagedPoolConfig = field(default_factory=PagedPoolConfig)
    c2w: Code2WavConfig = field(default_factory=Code2WavConfig)

    def to_dict(self) -> dict:
        return asdict(self)

    # -- the flat fields of the reference's ModelConfig (engine/backend/kv_cache_pool.py:36-60),
    #    which the engine loop reads from ``executor._config`` (engine_loop.py:242-243, 2105)
    @property
    def num_layers(self) -> int:
        return self.talker.num_layers

    @property
    def kv_heads(self) -> int:
        return self.talker.kv_heads

    @property
    def head_dim(self) -> int:
        return self.talker.head_dim

    @property
    def hidden_size(self) -> int:
        return self.talker.hidden_size

    @property
    def max_seq_len(self) -> int:
        return self.pool.max_seq_len

    @property
    def dtype(self):
        import torch
        return torch.bfloat16

    @property
    def codec_vocab_size(self) -> int:
        return self.talker.codec_vocab_size

    @property
    def logits_topk(self) -> int:
        return self.talker.logits_topk

    @property
    def cp_num_stages(self) -> int:
        return self.cp.num_stages

    @property
    def n_c2w_layers(self) -> int:
        return self.c2w.num_layers

    @property
    def c2w_kv_heads(self) -> int:
        return self.c2w.kv_heads

    @property
    def c2w_head_dim(self) -> int:
        return self.c2w.head_dim

    @property
    def c2w_sliding_window(self) -> int:
        return self.c2w.window


def tiny_engine_config(num_layers: int = 2) -> EngineConfig:
    """A small configuration with the talker's vocab and head layout intact.

    Used by the CPU tests and the golden-vector fixtures: the vocab (3072,
    suppress range [2048, 3072), EOS 2150) and the GQA ratio are kept because
    the sampling head and the attention kernels depend on them.
    """
    return EngineConfig(
        talker=TalkerConfig(num_layers=num_layers, hidden_size=256, num_heads=4, kv_heads=2,
                            head_dim=64, intermediate_size=512),
        cp=CodePredictorConfig(num_layers=2, hidden_size=128, num_heads=4, kv_heads=2, head_dim=32,
                               intermediate_size=256, talker_hidden_size=256),
        pool=PagedPoolConfig(block_size=16, num_blocks=64, max_slots=8, max_seq_len=256),
        c2w=tiny_code2wav_config(),
    )
