"""Per-request sampling parameters.

Mirrors the reference's ``SamplingParams`` (``src/sampling_params.py:6-30``):
the same fields, defaults and validation errors, plus the two knobs the
B200 sampler adds: ``repetition_penalty`` (applied over the set of token ids
already in the sequence) and ``seed`` (keys the per-request Philox stream;
``None`` uses the sampler's own seed).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_p: float | None = None
    top_k: int | None = None
    min_p: float | None = None
    max_tokens: int = 128
    min_tokens: int = 0
    ignore_eos: bool = False
    repetition_penalty: float = 1.0
    seed: int | None = None

    def __post_init__(self) -> None:
        # same checks and messages as src/sampling_params.py:16-30
        if self.max_tokens < 0:
            raise ValueError(f"max_tokens must be >= 0, got {self.max_tokens}")
        if self.min_tokens < 0:
            raise ValueError(f"min_tokens must be >= 0, got {self.min_tokens}")
        if self.min_tokens > self.max_tokens:
            raise ValueError("min_tokens must not exceed max_tokens")
        if self.temperature < 0:
            raise ValueError(f"temperature must be >= 0, got {self.temperature}")
        if self.top_p is not None and not (0.0 < self.top_p <= 1.0):
            raise ValueError(f"top_p must be in (0, 1], got {self.top_p}")
        if self.top_k is not None and self.top_k == 0:
            raise ValueError("top_k=0 is invalid; use None to disable")
        if self.min_p is not None and not (0.0 <= self.min_p <= 1.0):
            raise ValueError(f"min_p must be in [0, 1], got {self.min_p}")
        if not (self.repetition_penalty > 0.0):
            raise ValueError(f"repetition_penalty must be > 0, got {self.repetition_penalty}")
        if self.seed is not None and not (0 <= self.seed < 2**64):
            raise ValueError(f"seed must be in [0, 2^64), got {self.seed}")
