"""Multi-path parallel thinking (reference ``mamformer/thinking.py``).

N paths branch from the prompt cache (each blind to the others), each ends at
``<|think_end|>`` or its budget; then a summary phase and an answer phase.  Modes and budgets
(per path / summary): NoThink 0, FastThink 2 x 128 / 64, CoreThink 3 x 341 / 128,
DeepThink 5 x 819 / 256.  Control token ids 3..7 (think_start, think_end, answer_start,
answer_end, summary_start).
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from typing import List, Optional

_MODE_TABLE = {
    # mode: (paths, budget per path, summary budget)
    "NoThink": (0, 0, 0),
    "FastThink": (2, 128, 64),
    "CoreThink": (3, 341, 128),
    "DeepThink": (5, 819, 256),
}


class ThinkingMode(Enum):
    NoThink = "NoThink"
    FastThink = "FastThink"
    CoreThink = "CoreThink"
    DeepThink = "DeepThink"

    @property
    def num_paths(self) -> int:
        return _MODE_TABLE[self.value][0]

    @property
    def default_budget(self) -> int:
        return _MODE_TABLE[self.value][1]

    @property
    def default_summary_budget(self) -> int:
        return _MODE_TABLE[self.value][2]

    @classmethod
    def from_string(cls, s: str) -> "ThinkingMode":
        for m in cls:
            if m.value.lower() == str(s).lower():
                return m
        raise ValueError(f"Unknown thinking mode '{s}'. Available: {[m.value for m in cls]}")


@dataclass
class ThinkingConfig:
    mode: ThinkingMode = ThinkingMode.NoThink
    num_paths: int = 0
    think_budget: int = 0
    summary_budget: int = 0
    enabled: bool = False
    show_thinking: bool = False
    early_stop: bool = True
    think_start_token_id: int = 3
    think_end_token_id: int = 4
    answer_start_token_id: int = 5
    answer_end_token_id: int = 6
    summary_start_token_id: int = 7

    @property
    def effective_num_paths(self) -> int:
        return self.num_paths if self.num_paths > 0 else self.mode.num_paths

    @property
    def effective_budget(self) -> int:
        return self.think_budget if self.think_budget > 0 else self.mode.default_budget

    @property
    def effective_summary_budget(self) -> int:
        return self.summary_budget if self.summary_budget > 0 else self.mode.default_summary_budget

    @property
    def is_active(self) -> bool:
        return self.enabled and self.mode != ThinkingMode.NoThink

    @property
    def total_think_budget(self) -> int:
        return self.effective_num_paths * self.effective_budget

    @classmethod
    def disabled(cls) -> "ThinkingConfig":
        return cls(mode=ThinkingMode.NoThink, enabled=False)

    @classmethod
    def from_preset(cls, mode: str = "NoThink", budget: int = 0, num_paths: int = 0,
                    summary_budget: int = 0, show_thinking: bool = False) -> "ThinkingConfig":
        m = ThinkingMode.from_string(mode)
        return cls(mode=m, think_budget=budget, num_paths=num_paths, summary_budget=summary_budget,
                   enabled=m != ThinkingMode.NoThink, show_thinking=show_thinking)

    def validate(self) -> None:
        if self.think_budget < 0:
            raise ValueError(f"think_budget must be >= 0, got {self.think_budget}")
        if self.num_paths < 0:
            raise ValueError(f"num_paths must be >= 0, got {self.num_paths}")
        if self.enabled and self.mode == ThinkingMode.NoThink:
            raise ValueError("thinking enabled=True but mode=NoThink")

    def summary(self) -> str:
        n, b, s = self.effective_num_paths, self.effective_budget, self.effective_summary_budget
        return (f"ThinkingConfig(mode={self.mode.value}, paths={n}, budget_per_path={b}, "
                f"total_think={n * b}, summary_budget={s})")


class MultiPathController:
    """Phase bookkeeping: prompt -> path:i ... -> summary -> answer -> done."""

    def __init__(self, config: ThinkingConfig):
        self.config = config
        self.num_paths = config.effective_num_paths
        self._path_tokens: List[List[int]] = [[] for _ in range(self.num_paths)]
        self._path_counts: List[int] = [0] * self.num_paths
        self._path_budget_forced: List[bool] = [False] * self.num_paths
        self._summary_tokens: List[int] = []
        self._summary_count = 0
        self._summary_budget_forced = False
        self._answer_tokens: List[int] = []
        self._phase = "prompt"
        self._current_path = -1
        self._all_paths_done = False

    @property
    def phase(self) -> str:
        return self._phase

    @property
    def current_path(self) -> int:
        return self._current_path

    @property
    def is_done(self) -> bool:
        return self._phase == "done"

    @property
    def path_done(self) -> bool:
        return not self._phase.startswith("path:") and self._phase != "prompt"

    @property
    def summary_done(self) -> bool:
        return self._phase not in ("summary", "prompt")

    @property
    def answer_done(self) -> bool:
        return self._phase not in ("answer", "prompt")

    def start_path(self, path_idx: int) -> None:
        if path_idx < self.num_paths:
            self._phase = f"path:{path_idx}"
            self._current_path = path_idx

    def _end_current_path(self) -> None:
        if self._current_path + 1 >= self.num_paths:
            self._all_paths_done = True
            self._phase = "paths_done"
        else:
            self._phase = "between_paths"

    def start_summary(self) -> None:
        self._phase = "summary"

    def start_answer(self) -> None:
        self._phase = "answer"

    def record_path_token(self, path_idx: int, token_id: int) -> Optional[str]:
        self._path_tokens[path_idx].append(token_id)
        if token_id == self.config.think_end_token_id:
            self._end_current_path()
            return "end_path"
        self._path_counts[path_idx] += 1
        if self._path_counts[path_idx] >= self.config.effective_budget:
            self._path_budget_forced[path_idx] = True
            return "budget_exceeded"
        return None

    def record_summary_token(self, token_id: int) -> Optional[str]:
        self._summary_tokens.append(token_id)
        self._summary_count += 1
        if self._summary_count >= self.config.effective_summary_budget:
            self._summary_budget_forced = True
            self._phase = "summary_done"
            return "end_summary"
        return None

    def record_answer_token(self, token_id: int) -> Optional[str]:
        if token_id in (self.config.answer_end_token_id, 2):
            self._phase = "done"
            return "end_answer"
        self._answer_tokens.append(token_id)
        return None

    def get_think_start_token(self) -> int:
        return self.config.think_start_token_id

    def get_think_end_token(self) -> int:
        return self.config.think_end_token_id

    def get_summary_start_token(self) -> int:
        return self.config.summary_start_token_id

    def get_answer_start_token(self) -> int:
        return self.config.answer_start_token_id

    def finalize(self) -> dict:
        return {"all_paths": self._path_tokens, "path_counts": self._path_counts,
                "path_budget_forced": self._path_budget_forced,
                "summary_tokens": self._summary_tokens, "summary_count": self._summary_count,
                "summary_budget_forced": self._summary_budget_forced,
                "answer_tokens": self._answer_tokens, "total_think_tokens": sum(self._path_counts),
                "phase": self._phase}

    def __repr__(self) -> str:
        return (f"MultiPathController(phase={self._phase}, paths={self._path_counts}/{self.num_paths}, "
                f"summary={self._summary_count}/{self.config.effective_summary_budget}, "
                f"answer={len(self._answer_tokens)})")
