"""A host-only stand-in for the engine, for the serving front end's CPU tests.

It has the engine surface the replica loop uses (``add_request``,
``abort_request``, ``has_unfinished``, ``step``, ``scheduler``, ``allocator``,
``model.cfg.vocab_size``) and a fixed rule for its tokens: token t of a request
is ``(sum(prompt) + t) % vocab``.  Every running request gets one token per
step; a request finishes with "length" at ``max_tokens``.  Failures are made on
the host: ``fail_after`` steps raise, ``exit_after`` steps end the process.
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass
from types import SimpleNamespace

from tokquay_b200.engine import TokenEvent
from tokquay.scheduler import RequestRejected, Scheduler, SchedulerConfig
from tokquay.sequence import Sequence


def expected_tokens(prompt: list[int], n: int, vocab: int = 1000) -> list[int]:
    return [(sum(prompt) + t) % vocab for t in range(n)]


class _Pool:
    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks, self.block_size = num_blocks, block_size
        self.num_free_blocks = num_blocks

    def blocks_needed(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)


class EchoEngine:
    def __init__(self, vocab: int = 1000, num_blocks: int = 64, block_size: int = 16, max_model_len: int = 256,
                 step_s: float = 0.0, fail_after: int | None = None, exit_after: int | None = None):  # fmt: skip
        self.allocator = _Pool(num_blocks, block_size)
        self.scheduler = Scheduler(self.allocator, SchedulerConfig(max_model_len=max_model_len))
        self.model = SimpleNamespace(cfg=SimpleNamespace(vocab_size=vocab))
        self.vocab, self.step_s = vocab, step_s
        self.fail_after, self.exit_after = fail_after, exit_after
        self.steps = 0
        self._next = 0

    def add_request(self, prompt_token_ids, params) -> Sequence:
        seq = Sequence(self._next, list(prompt_token_ids), sampling=params)
        why = self.scheduler.rejection_reason(seq)
        if why:
            raise RequestRejected(why)
        self._next += 1
        self.scheduler.running.append(seq)
        return seq

    def abort_request(self, seq: Sequence) -> None:
        self.scheduler.running.remove(seq)

    def has_unfinished(self) -> bool:
        return bool(self.scheduler.running)

    def step(self) -> list[TokenEvent]:
        self.steps += 1
        if self.fail_after is not None and self.steps > self.fail_after:
            raise RuntimeError("injected step failure")
        if self.exit_after is not None and self.steps > self.exit_after:
            os._exit(3)
        if self.step_s:
            time.sleep(self.step_s)
        events = []
        for seq in list(self.scheduler.running):
            tok = (sum(seq.prompt_token_ids) + len(seq.output_token_ids)) % self.vocab
            seq.output_token_ids.append(tok)
            done = len(seq.output_token_ids) >= seq.sampling.max_tokens
            if done:
                self.scheduler.running.remove(seq)
            events.append(TokenEvent(seq.seq_id, tok, "length" if done else None))
        return events


@dataclass(frozen=True)
class EchoFactory:
    """Picklable factory: one ``EchoEngine`` per replica.  Replicas are
    labelled (the router's ``devices``); ``fail`` / ``exit`` map a label to
    the steps after which that replica raises / exits."""

    step_s: float = 0.0
    max_model_len: int = 256
    fail: tuple[tuple[str, int], ...] = ()
    exit: tuple[tuple[str, int], ...] = ()

    def __call__(self, label):
        return EchoEngine(step_s=self.step_s, max_model_len=self.max_model_len,
                          fail_after=dict(self.fail).get(label), exit_after=dict(self.exit).get(label))  # fmt: skip
