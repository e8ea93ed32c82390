"""Seeded synthetic inputs for the benchmark configurations.

No dataset is involved: prompts are uniform-random token ids mapped through a
seeded random text-embedding table (the reference maps text ids through
``text_embedding`` + ``ResizeMLP``, engine/backend/prefill.py:34-236; that
projection is per-request host work outside the decode path, so a seeded
table of the talker's hidden width stands in for it).  ``tts_pad`` is the
embedding the engine adds once the text is exhausted
(engine/backend/engine_loop.py:2191-2197).
"""

from __future__ import annotations

from typing import List, Sequence

import torch

TEXT_VOCAB = 4096


def _gen(seed: int, salt: int, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((int(seed) * 1_000_003 + salt) & ((1 << 62) - 1))
    return g


def text_table(hidden: int, seed: int, device="cpu") -> torch.Tensor:
    return torch.randn(TEXT_VOCAB, hidden, generator=_gen(seed, 11, device), device=device) * 0.02


def tts_pad_embed(hidden: int, seed: int, device="cpu") -> torch.Tensor:
    return torch.randn(hidden, generator=_gen(seed, 13, device), device=device) * 0.02


def prompt_ids(lengths: Sequence[int], seed: int) -> List[torch.Tensor]:
    g = _gen(seed, 17)
    return [torch.randint(0, TEXT_VOCAB, (int(n),), generator=g) for n in lengths]


def shared_prefix_prompts(n_streams: int, lo: int, hi: int, prefix_len: int, seed: int) -> List[torch.Tensor]:
    """Benchmark prompts: lengths U{lo..hi}; the first ``min(prefix_len, L)`` ids are common."""
    g = _gen(seed, 19)
    lengths = torch.randint(lo, hi + 1, (n_streams,), generator=g).tolist()
    prefix = torch.randint(0, TEXT_VOCAB, (prefix_len,), generator=g)
    out = []
    for n in lengths:
        suffix = torch.randint(0, TEXT_VOCAB, (max(0, n - prefix_len),), generator=g)
        out.append(torch.cat([prefix[: min(prefix_len, n)], suffix]))
    return out
