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


def setup_shared_prefix_streams(ex, prompts: Sequence[torch.Tensor], table: torch.Tensor, pad: torch.Tensor,
                                prefix_len: int, key: str = "shared-prefix", record: bool = False):
    """The benchmark's stream set-up on a ``B200Executor`` (cfg2): the common prefix
    (``prompts[i][:prefix_len]``) is prefilled once into a holder slot and cached by block
    reference, and the holder is freed; each stream then restores the cached prefix from the
    prefix cache (no KV copy) — a prompt shorter than the prefix shares ceil(L/16) of its
    blocks, the last one partial and copied on the stream's first write — and prefills its
    own suffix (sampling its first frame) or, with no suffix, starts decoding from ``pad``.
    Every stream's text embedding is ``pad``, its first frame included.  Returns
    ``(slots, first)``: ``first[i]`` is ``(codes [16], logits [V])`` of stream i's prefill
    (``None`` without a suffix) when ``record`` is set, else ``None``."""
    dev = ex._device
    pool = ex.kv_pool
    cache = ex.make_prefix_cache(max_entries=4, max_prefix_len=max(512, prefix_len))
    holder = pool.allocate("prefix-holder")
    longest = max(prompts, key=len)
    ex.prefill_prefix_only(holder, table[longest[:prefix_len].to(table.device)].to(dev).unsqueeze(0))
    cache.put(key, holder.slot_id, prefix_len)
    pool.release(holder.slot_id)
    entry = cache.get(key)
    slots, first = [], []
    for i, ids in enumerate(prompts):
        s = pool.allocate(f"stream-{i}")
        s.segment_idx = 0
        n_shared = min(prefix_len, len(ids))
        # the whole cached prefix, or (prompt shorter than it) its first n_shared positions
        cache.restore(s, entry if n_shared == prefix_len else entry.talker_kv[0, :, :, :n_shared, :])
        suffix = ids[n_shared:]
        # the text embedding added to the codec sum of each frame, the first one included
        ex.set_text_embedding(s, pad)
        if len(suffix) > 0:
            ex.prefill_from_prefix(s, table[suffix.to(table.device)].to(dev).unsqueeze(0))
            if record:
                first.append((ex.codes[0].cpu().clone(), ex.logits[0].cpu().clone()))
        else:
            ex._configure_sampling(s)
            ex.next_x[s.slot_id].copy_(pad.to(dev))
            if record:
                first.append(None)
        slots.append(s)
    torch.cuda.synchronize(dev)
    return slots, (first if record else None)
