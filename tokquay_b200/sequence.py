"""Per-request state shared by the allocator, the step driver and any engine.

Same data contract as the reference (tokquay/sequence.py:9-81): the fields and
their meaning are the interface the scheduler and engine are written against,
so they are kept as they are.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass, field


class SequenceStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"


@dataclass(frozen=True)
class SamplingParams:
    """Generation settings of one request; ``temperature == 0`` is greedy
    (tokquay/sequence.py:15-31)."""

    max_tokens: int = 16
    temperature: float = 0.0
    top_k: int = 0
    ignore_eos: bool = False
    seed: int | None = None

    def __post_init__(self) -> None:
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if self.top_k < 0:
            raise ValueError("top_k must be >= 0")


@dataclass
class Sequence:
    """One request (tokquay/sequence.py:34-81).

    ``num_cached_tokens`` leading positions already have K/V in the pool; the
    next step feeds ``token_ids[num_cached_tokens:]``.  ``block_table[i]`` is
    the pool block holding positions ``[i*bs, (i+1)*bs)``.
    """

    seq_id: int
    prompt_token_ids: list[int]
    output_token_ids: list[int] = field(default_factory=list)
    block_table: list[int] = field(default_factory=list)
    status: SequenceStatus = SequenceStatus.WAITING
    num_cached_tokens: int = 0
    sampling: SamplingParams = field(default_factory=SamplingParams)
    finish_reason: str | None = None

    def __post_init__(self) -> None:
        if not self.prompt_token_ids:
            raise ValueError("prompt must contain at least one token")

    @property
    def token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.output_token_ids

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def num_uncached_tokens(self) -> int:
        return self.num_tokens - self.num_cached_tokens

    def tokens_slice(self, begin: int, end: int) -> list[int]:
        """``token_ids[begin:end]`` without building the whole concatenation
        (a decode step needs only the last token)."""
        p = len(self.prompt_token_ids)
        if begin >= p:
            return self.output_token_ids[begin - p:end - p]
        if end <= p:
            return self.prompt_token_ids[begin:end]
        return self.prompt_token_ids[begin:] + self.output_token_ids[:end - p]

    def append_token(self, token_id: int) -> None:
        self.output_token_ids.append(token_id)

    def reset_for_recompute(self) -> None:
        """Forget cache state after the allocator freed the blocks (preemption)."""
        self.block_table = []
        self.num_cached_tokens = 0
        self.status = SequenceStatus.WAITING
