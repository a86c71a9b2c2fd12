"""Multi-path parallel thinking: modes, budgets and the decode-time phase tracker.

Behaviour follows the reference's thinking mode (``mamformer/thinking.py``: modes 52-104,
config 107-234, controller 237-454): N reasoning paths branch from the prompt's cache and do
not see each other; each path stops at ``<|think_end|>`` or at its token budget; then a summary
of bounded length and an answer follow.  The public surface (mode names and budgets, the
config fields and ``effective_*`` helpers, the controller's method names, the event strings
``"end_path"`` / ``"budget_exceeded"`` / ``"end_summary"`` / ``"end_answer"`` and the keys of
``finalize()``) is kept so that generation code written for either framework drives this one.

The controller is written here as a table-driven state machine over :class:`Phase`: every
transition is one row of ``_TRANSITIONS`` and an illegal transition raises, so a caller that
records an answer token before the answer phase starts finds out at once.

Control token ids (from the tokenizer): 3 think_start, 4 think_end, 5 answer_start,
6 answer_end, 7 summary_start; id 2 (EOS) also ends the answer.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, List, NamedTuple, Optional

EOS_TOKEN_ID = 2


class _Budget(NamedTuple):
    paths: int
    per_path: int
    summary: int


# (number of paths, tokens per path, summary tokens) per mode
_BUDGETS: Dict[str, _Budget] = {
    "NoThink": _Budget(0, 0, 0),
    "FastThink": _Budget(2, 128, 64),
    "CoreThink": _Budget(3, 341, 128),
    "DeepThink": _Budget(5, 819, 256),
}


class ThinkingMode(Enum):
    NoThink = "NoThink"
    FastThink = "FastThink"
    CoreThink = "CoreThink"
    DeepThink = "DeepThink"

    @property
    def budget(self) -> _Budget:
        return _BUDGETS[self.value]

    @property
    def num_paths(self) -> int:
        return self.budget.paths

    @property
    def default_budget(self) -> int:
        return self.budget.per_path

    @property
    def default_summary_budget(self) -> int:
        return self.budget.summary

    @classmethod
    def from_string(cls, s: str) -> "ThinkingMode":
        by_name = {m.value.lower(): m for m in cls}
        mode = by_name.get(str(s).lower())
        if mode is None:
            raise ValueError(f"Unknown thinking mode '{s}'. Available: {[m.value for m in cls]}")
        return mode


def _override_or(value: int, fallback: int) -> int:
    """A positive explicit setting wins; 0 means 'use the mode's default'."""
    return value if value > 0 else fallback


@dataclass
class ThinkingConfig:
    """Thinking settings.  ``num_paths`` / ``think_budget`` / ``summary_budget`` of 0 select the
    mode's defaults; ``enabled`` is the master switch."""

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
        return _override_or(self.num_paths, self.mode.num_paths)

    @property
    def effective_budget(self) -> int:
        return _override_or(self.think_budget, self.mode.default_budget)

    @property
    def effective_summary_budget(self) -> int:
        return _override_or(self.summary_budget, self.mode.default_summary_budget)

    @property
    def is_active(self) -> bool:
        return self.enabled and self.mode is not ThinkingMode.NoThink

    @property
    def total_think_budget(self) -> int:
        return self.effective_num_paths * self.effective_budget

    @classmethod
    def disabled(cls) -> "ThinkingConfig":
        return cls()

    @classmethod
    def from_preset(cls, mode: str = "NoThink", budget: int = 0, num_paths: int = 0,
                    summary_budget: int = 0, show_thinking: bool = False) -> "ThinkingConfig":
        m = ThinkingMode.from_string(mode)
        return cls(mode=m, num_paths=num_paths, think_budget=budget, summary_budget=summary_budget,
                   enabled=m is not ThinkingMode.NoThink, show_thinking=show_thinking)

    def validate(self) -> None:
        problems = []
        if self.think_budget < 0:
            problems.append(f"think_budget must be >= 0, got {self.think_budget}")
        if self.num_paths < 0:
            problems.append(f"num_paths must be >= 0, got {self.num_paths}")
        if self.enabled and self.mode is ThinkingMode.NoThink:
            problems.append("thinking enabled=True but mode=NoThink")
        if problems:
            raise ValueError("; ".join(problems))

    def summary(self) -> str:
        paths, per, summ = self.effective_num_paths, self.effective_budget, self.effective_summary_budget
        return (f"ThinkingConfig(mode={self.mode.value}, paths={paths}, budget_per_path={per}, "
                f"total_think={paths * per}, summary_budget={summ})")


class Phase(Enum):
    PROMPT = "prompt"
    PATH = "path"                  # rendered as "path:<index>"
    BETWEEN_PATHS = "between_paths"
    PATHS_DONE = "paths_done"
    SUMMARY = "summary"
    SUMMARY_DONE = "summary_done"
    ANSWER = "answer"
    DONE = "done"


# Allowed (from, to) transitions.  start_path may also restart a path from any earlier phase
# (the batched generator records paths one after another, after all were sampled).
_TRANSITIONS = {
    Phase.PROMPT: {Phase.PATH, Phase.SUMMARY, Phase.ANSWER},
    Phase.PATH: {Phase.PATH, Phase.BETWEEN_PATHS, Phase.PATHS_DONE, Phase.SUMMARY, Phase.ANSWER},
    Phase.BETWEEN_PATHS: {Phase.PATH, Phase.SUMMARY, Phase.ANSWER},
    Phase.PATHS_DONE: {Phase.PATH, Phase.SUMMARY, Phase.ANSWER},
    Phase.SUMMARY: {Phase.SUMMARY_DONE, Phase.ANSWER, Phase.SUMMARY},
    Phase.SUMMARY_DONE: {Phase.ANSWER, Phase.SUMMARY},
    Phase.ANSWER: {Phase.DONE, Phase.ANSWER},
    Phase.DONE: {Phase.ANSWER},
}


@dataclass
class _Segment:
    """Tokens of one path or of the summary, with the count against its budget (the path's
    closing think_end token is kept in ``tokens`` but not counted)."""
    tokens: List[int] = field(default_factory=list)
    counted: int = 0
    hit_budget: bool = False


class MultiPathController:
    """Tracks one thinking decode: paths, then summary, then answer.

    Drive it with ``start_path(i)`` / ``record_path_token(i, tok)`` for each path,
    ``start_summary()`` / ``record_summary_token(tok)``, ``start_answer()`` /
    ``record_answer_token(tok)``; each ``record_*`` call returns ``None`` (keep going) or an
    event string telling the caller to stop that phase.  ``finalize()`` returns the tokens and
    counters."""

    def __init__(self, config: ThinkingConfig):
        self.config = config
        self.num_paths = config.effective_num_paths
        self._paths = [_Segment() for _ in range(self.num_paths)]
        self._summary = _Segment()
        self._answer: List[int] = []
        self._state = Phase.PROMPT
        self._active_path = -1

    # -- state -------------------------------------------------------------------------------
    def _go(self, nxt: Phase) -> None:
        if nxt not in _TRANSITIONS[self._state]:
            raise RuntimeError(f"thinking controller: cannot go from {self.phase} to {nxt.value}")
        self._state = nxt

    @property
    def phase(self) -> str:
        if self._state is Phase.PATH:
            return f"path:{self._active_path}"
        return self._state.value

    @property
    def current_path(self) -> int:
        return self._active_path

    @property
    def is_done(self) -> bool:
        return self._state is Phase.DONE

    @property
    def path_done(self) -> bool:
        return self._state not in (Phase.PATH, Phase.PROMPT)

    @property
    def summary_done(self) -> bool:
        return self._state not in (Phase.SUMMARY, Phase.PROMPT)

    @property
    def answer_done(self) -> bool:
        return self._state not in (Phase.ANSWER, Phase.PROMPT)

    # -- transitions --------------------------------------------------------------------------
    def start_path(self, path_idx: int) -> None:
        if not 0 <= path_idx < self.num_paths:
            return
        self._go(Phase.PATH)
        self._active_path = path_idx

    def start_summary(self) -> None:
        self._go(Phase.SUMMARY)

    def start_answer(self) -> None:
        self._go(Phase.ANSWER)

    # -- token recording ----------------------------------------------------------------------
    def record_path_token(self, path_idx: int, token_id: int) -> Optional[str]:
        seg = self._paths[path_idx]
        seg.tokens.append(token_id)
        if token_id == self.config.think_end_token_id:
            last = path_idx + 1 >= self.num_paths
            self._go(Phase.PATHS_DONE if last else Phase.BETWEEN_PATHS)
            return "end_path"
        seg.counted += 1
        if seg.counted >= self.config.effective_budget:
            seg.hit_budget = True
            return "budget_exceeded"
        return None

    def record_summary_token(self, token_id: int) -> Optional[str]:
        seg = self._summary
        seg.tokens.append(token_id)
        seg.counted += 1
        if seg.counted < self.config.effective_summary_budget:
            return None
        seg.hit_budget = True
        self._go(Phase.SUMMARY_DONE)
        return "end_summary"

    def record_answer_token(self, token_id: int) -> Optional[str]:
        if token_id == self.config.answer_end_token_id or token_id == EOS_TOKEN_ID:
            self._go(Phase.DONE)
            return "end_answer"
        self._answer.append(token_id)
        return None

    # -- control tokens -----------------------------------------------------------------------
    def get_think_start_token(self) -> int:
        return self.config.think_start_token_id

    def get_think_end_token(self) -> int:
        return self.config.think_end_token_id

    def get_summary_start_token(self) -> int:
        return self.config.summary_start_token_id

    def get_answer_start_token(self) -> int:
        return self.config.answer_start_token_id

    # -- results ------------------------------------------------------------------------------
    def finalize(self) -> dict:
        counts = [s.counted for s in self._paths]
        return {
            "all_paths": [list(s.tokens) for s in self._paths],
            "path_counts": counts,
            "path_budget_forced": [s.hit_budget for s in self._paths],
            "summary_tokens": list(self._summary.tokens),
            "summary_count": self._summary.counted,
            "summary_budget_forced": self._summary.hit_budget,
            "answer_tokens": list(self._answer),
            "total_think_tokens": sum(counts),
            "phase": self.phase,
        }

    def __repr__(self) -> str:
        counts = [s.counted for s in self._paths]
        return (f"MultiPathController(phase={self.phase}, paths={counts}/{self.num_paths}, "
                f"summary={self._summary.counted}/{self.config.effective_summary_budget}, "
                f"answer={len(self._answer)})")
