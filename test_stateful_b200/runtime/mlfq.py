"""Multi-level feedback queue batch ordering (host side, unchanged semantics).

Same contract as the reference scheduler (engine/core/mlfq.py:29-173): three
levels, a segment starts at level 0, moves to level 1 after ``q1_threshold``
decode steps and to level 2 after ``q2_threshold``; a batch takes level 0 then
1 then 2, first-come first-served inside a level, up to ``max_batch``; every
``aging_interval`` global steps, level-2 segments not scheduled for
``starvation_limit`` steps go back to level 0.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional


@dataclass
class MLFQConfig:
    q1_threshold: int = 50
    q2_threshold: int = 200
    aging_interval: int = 100
    starvation_limit: int = 50


@dataclass
class MLFQMeta:
    level: int = 0
    decode_steps: int = 0
    last_scheduled_at: int = 0
    steps_since_schedule: int = 0

    def reset(self) -> None:
        self.level = 0
        self.decode_steps = 0
        self.steps_since_schedule = 0


class MLFQScheduler:
    def __init__(self, config: Optional[MLFQConfig] = None):
        self._cfg = config or MLFQConfig()
        self._global_step = 0

    @property
    def global_step(self) -> int:
        return self._global_step

    def on_segment_created(self, meta: MLFQMeta) -> None:
        meta.reset()

    def on_segment_boundary(self, meta: MLFQMeta) -> None:
        meta.reset()

    def on_step_done(self, meta: MLFQMeta) -> None:
        meta.decode_steps += 1
        meta.steps_since_schedule += 1
        if meta.level == 0 and meta.decode_steps >= self._cfg.q1_threshold:
            meta.level = 1
        elif meta.level == 1 and meta.decode_steps >= self._cfg.q2_threshold:
            meta.level = 2

    def on_scheduled(self, meta: MLFQMeta) -> None:
        meta.last_scheduled_at = self._global_step
        meta.steps_since_schedule = 0

    def select_batch(self, candidates: List, max_batch: int, *, get_meta: Callable) -> List:
        levels = ([], [], [])
        for seg in candidates:
            levels[min(2, max(0, get_meta(seg).level))].append(seg)
        chosen: List = []
        for bucket in levels:
            for seg in bucket:
                if len(chosen) >= max_batch:
                    return chosen
                self.on_scheduled(get_meta(seg))
                chosen.append(seg)
        return chosen

    def tick(self, all_metas: Optional[List[MLFQMeta]] = None) -> int:
        self._global_step += 1
        if not all_metas or self._cfg.aging_interval <= 0 or self._global_step % self._cfg.aging_interval:
            return 0
        boosted = 0
        for meta in all_metas:
            if meta.level >= 2 and meta.steps_since_schedule >= self._cfg.starvation_limit:
                meta.level = 0
                meta.steps_since_schedule = 0
                boosted += 1
        return boosted
