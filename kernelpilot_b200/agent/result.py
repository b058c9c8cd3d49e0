"""The outcome of evaluating one candidate kernel, as the sandboxed worker writes it
and an optimisation loop reads it (kernelpilot/agent/result.py:1-46: same stages,
fields, score and dict form, so results written by either side read the same)."""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

# How far a candidate got; only "ok" candidates may ever be kept as the best.
STAGES = ("no_code", "rejected", "compile", "correctness", "benchmark", "timeout", "crash", "ok")


@dataclass
class EvalResult:
    stage: str
    error: str | None = None
    compile_log: str = ""
    # failed correctness checks (CheckResult dicts), a few at most
    failures: list[dict] = field(default_factory=list)
    checks_passed: int = 0
    # one row per benchmark shape: shape, ms, torch_ms, speedup, gbs, tflops, pct_*
    bench: list[dict] = field(default_factory=list)
    profile: dict = field(default_factory=dict)
    duration_s: float = 0.0

    def __post_init__(self) -> None:
        if self.stage not in STAGES:
            raise ValueError(f"unknown stage {self.stage!r}; expected one of {STAGES}")

    @property
    def ok(self) -> bool:
        return self.stage == "ok"

    @property
    def score(self) -> float | None:
        """Geometric mean of the speed-ups over PyTorch on the benchmark shapes."""
        speedups = [r["speedup"] for r in self.bench if r.get("speedup")]
        if not self.ok or not speedups:
            return None
        return math.exp(sum(math.log(s) for s in speedups) / len(speedups))

    def to_dict(self) -> dict:
        d = asdict(self)
        d["score"] = self.score
        return d

    @classmethod
    def from_dict(cls, d: dict) -> EvalResult:
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})
