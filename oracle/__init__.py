"""CPU oracle for the B200 decode backend — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithms of the Qwen3-TTS
standalone engine's decode hot path:

* ``oracle.model``       — talker forward, sampling head, code predictor and
  codec embedding sum, in fp32 torch
  (scripts/export/talker_unified_modules.py, scripts/export/utils.py:852-1042,
  scripts/python/codec_embedding_sum.py).
* ``oracle.paged_state`` — the paged KV pool's block allocator, block tables,
  slot mapping and prefix-block refcount/copy-on-write, in plain Python/numpy,
  pinned against the reference's slot-contiguous ``KVCachePool``
  (engine/backend/kv_cache_pool.py) and ``PrefixKVCache``
  (engine/backend/prefix_cache.py).
* ``oracle.code2wav``    — the streaming code2wav decoder
  (scripts/export/code2wav_streaming.py).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import it, and only as the checker or the timed CPU baseline.
The product path (``test_stateful_b200``) never imports it.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own PyTorch
modules (imported from the reference checkout, with seeded random-init
stand-ins for the absent ``qwen_tts`` package) and its ``KVCachePool`` /
``PrefixKVCache`` on small cases and stores the outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this package against
them.
"""
