"""Routing decisions as data, shared by the PyTorch overlay and the vLLM layer.

Every "should this call run on zcutlass?" decision in the drop-in packages is
an ordered table of `Rule`s -- a reason string and a test that is true when
the call must fall back -- read by one evaluator, `first_reason`. The reason
strings and the order in which they are tried are the reference's interface
(its users aggregate them in serving reports), so each table cites the
reference lines it keeps; the code around them is this package's own.

Also here: the tally of hits, misses and reasons (`Tally`), the shape-family
buckets (decode / prefill / large / fallback) and the environment switches
the reference's packages read.
"""

from __future__ import annotations

import math
import os
from collections import Counter
from dataclasses import dataclass
from typing import Any, Callable, Iterable, Optional, Sequence


@dataclass(frozen=True)
class Rule:
    """`reason` is reported when `test(subject)` is true."""

    reason: str
    test: Callable[[Any], bool]


def first_reason(rules: Sequence[Rule], subject: Any) -> Optional[str]:
    """The reason of the first rule (in table order) whose test holds, else None."""
    return next((r.reason for r in rules if r.test(subject)), None)


class Tally:
    """Hit / miss counts and a count per fallback reason."""

    def __init__(self) -> None:
        self.hits = 0
        self._reasons: Counter[str] = Counter()

    @property
    def misses(self) -> int:
        return sum(self._reasons.values())

    @property
    def fallback_reasons(self) -> dict[str, int]:
        return dict(self._reasons)

    @property
    def total(self) -> int:
        return self.hits + self.misses

    @property
    def hit_rate(self) -> float:
        return self.hits / self.total if self.total else 0.0

    def record_hit(self) -> None:
        self.hits += 1

    def record_miss(self, reason: str) -> None:
        self._reasons[reason] += 1

    def absorb(self, other: "Tally") -> None:
        self.hits += other.hits
        self._reasons.update(other._reasons)

    def __repr__(self) -> str:
        return f"{type(self).__name__}(hits={self.hits}, misses={self.misses}, fallback_reasons={self.fallback_reasons})"


# ---------------------------------------------------------------- shape families

@dataclass(frozen=True)
class Bucket:
    family: str
    m_lo: int
    m_hi: float  # inclusive; math.inf for open-ended


def classify(m: int, n: int, k: int, buckets: Iterable[Bucket], min_n: int, min_k: int) -> str:
    """The family of an (m, n, k) GEMM: the first bucket holding m, when n and k
    reach their minimums; otherwise "fallback"."""
    if n < min_n or k < min_k:
        return "fallback"
    return next((b.family for b in buckets if b.m_lo <= m <= b.m_hi), "fallback")


# Default buckets of the reference (python/zcutlass_torch/overlay.py:75-82,
# python/zcutlass_vllm/route_logger.py:42-49): N, K >= 1024 and M in these ranges.
DEFAULT_BUCKETS = (Bucket("decode", 0, 16), Bucket("prefill", 32, 256), Bucket("large", 512, math.inf))


def default_family(m: int, n: int, k: int) -> str:
    return classify(m, n, k, DEFAULT_BUCKETS, 1024, 1024)


# ---------------------------------------------------------------- environment

_FALSE_WORDS = frozenset({"", "0", "false", "False", "FALSE", "no", "No", "NO"})


def env_flag(name: str, default: bool = False) -> bool:
    """A switch the way the reference reads one: unset -> default; empty,
    0, false or no (any of their usual spellings) -> off; anything else -> on."""
    raw = os.environ.get(name)
    return default if raw is None else raw not in _FALSE_WORDS


def env_list(name: str, default: tuple[str, ...] = ()) -> tuple[str, ...]:
    """A comma-separated list (blank entries dropped); unset or blank -> default."""
    raw = os.environ.get(name, "")
    if not raw.strip():
        return default
    return tuple(p.strip() for p in raw.split(",") if p.strip())


def env_word(name: str, default: str) -> str:
    """A lower-cased, stripped word."""
    return os.environ.get(name, default).strip().lower()
