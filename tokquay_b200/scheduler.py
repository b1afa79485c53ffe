"""Continuous-batching scheduler over the paged pool (the caller of the hot path).

Restates the reference's scheduling policy (tokquay/scheduler.py:1-35, :82-190)
so that a step sequence -- which requests run, which are preempted, which
blocks they get -- is the same decision for decision, given the same token
streams.  The policy:

* every step is either a prefill step over newly admitted requests (when at
  least one waiting request can be admitted) or a decode step over every
  running sequence -- never both;
* admission is first-come first-served and stops at the first waiting request
  that does not fit: the running-sequence cap, the step budget counted in
  padded tokens (batch size x longest row), and the free blocks, keeping
  ``watermark_blocks`` spare while other sequences run;
* a decode step that cannot get a block for some sequence evicts the newest
  running sequence (preemption by recompute): its blocks are freed, it keeps
  its generated tokens and goes back to the front of the waiting queue;
* a request whose worst-case context can never fit is refused when added.

The allocator and sequences are this package's (same contract as the
reference's), so block tables and allocator state follow the reference's bit
for bit.

``SchedulerConfig.mixed_prefill_tokens > 0`` switches to an opt-in policy
that is not the reference's (chunked prefill): each step runs every decoding
sequence together with up to that many prompt tokens -- the next chunk of
every running sequence still in its prompt, then newly admitted requests --
in one mixed launch of the paged path.  Admission (FCFS, no skipping, blocks
for the whole prompt reserved up front, watermark) and preemption (the newest
running sequence, by recompute) follow the same rules as above.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from tokquay_b200.kv_cache import BlockAllocator
from tokquay_b200.sequence import Sequence, SequenceStatus

__all__ = ["RequestRejected", "SchedulerConfig", "ScheduledBatch", "Scheduler"]


class RequestRejected(ValueError):
    """The request can never be served with this configuration."""


@dataclass
class SchedulerConfig:
    """Limits of one engine (tokquay/scheduler.py:46-57)."""

    max_num_seqs: int = 64
    max_num_batched_tokens: int = 2048  # per step, in padded tokens: rows x longest row
    max_model_len: int = 1024
    watermark_blocks: int = 1
    # Opt-in, not the reference's policy: > 0 runs every decoding sequence and
    # up to this many prompt tokens (chunks of prompts) in each step.
    mixed_prefill_tokens: int = 0

    def __post_init__(self) -> None:
        if self.max_num_seqs < 1 or self.max_num_batched_tokens < self.max_num_seqs:
            raise ValueError("need max_num_seqs >= 1 and max_num_batched_tokens >= max_num_seqs")
        if self.mixed_prefill_tokens < 0:
            raise ValueError("mixed_prefill_tokens must be >= 0")


@dataclass
class ScheduledBatch:
    """One step's sequences.  ``padded_tokens`` is fixed when the batch is made
    (the step itself changes the sequences' uncached counts).  ``new_lens``:
    the tokens each sequence feeds (None: all of its uncached tokens, as every
    step of the reference's policy does)."""

    seqs: list[Sequence]
    is_prefill: bool
    preempted: list[Sequence] = field(default_factory=list)
    new_lens: list[int] | None = None
    padded_tokens: int = field(init=False)

    def __post_init__(self) -> None:
        widest = max(self.new_lens) if self.new_lens else max(s.num_uncached_tokens for s in self.seqs)
        self.padded_tokens = len(self.seqs) * widest


class Scheduler:
    """Decides, step by step, which sequences run (tokquay/scheduler.py:71-190)."""

    def __init__(self, allocator: BlockAllocator, config: SchedulerConfig | None = None):
        self.allocator = allocator
        self.config = config or SchedulerConfig()
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []  # admission order; the last is the newest
        self.num_preemptions = 0
        self.num_discarded_positions = 0  # cached positions preemption threw away

    # ---- requests --------------------------------------------------------------------
    def max_context(self, seq: Sequence) -> int:
        """The most positions ``seq`` can hold in the cache: its prompt and every
        output token but the last (which is returned, never cached)."""
        return len(seq.prompt_token_ids) + seq.sampling.max_tokens - 1

    def rejection_reason(self, seq: Sequence) -> str | None:
        cfg = self.config
        need = self.max_context(seq)
        if need > cfg.max_model_len:
            return f"prompt + max_tokens needs {need} positions but the model supports {cfg.max_model_len}"
        blocks = self.allocator.blocks_needed(need)
        if blocks > self.allocator.num_blocks:
            return f"needs {blocks} KV blocks but the pool only has {self.allocator.num_blocks}"
        if need > cfg.max_num_batched_tokens:  # a preempted sequence is prefilled again in one step
            return f"needs {need} tokens in one step but max_num_batched_tokens is {cfg.max_num_batched_tokens}"
        return None

    def add_request(self, seq: Sequence) -> None:
        why = self.rejection_reason(seq)
        if why is not None:
            raise RequestRejected(why)
        seq.status = SequenceStatus.WAITING
        self.waiting.append(seq)

    def has_unfinished(self) -> bool:
        return bool(self.waiting) or bool(self.running)

    def finish(self, seq: Sequence, reason: str) -> None:
        self.running.remove(seq)
        self.allocator.free(seq)
        seq.status = SequenceStatus.FINISHED
        seq.finish_reason = reason

    def abort(self, seq: Sequence) -> None:
        """Drop a request wherever it is (queued, preempted, running); a no-op
        once it has finished.  Its blocks go back to the pool."""
        if seq.status is SequenceStatus.FINISHED:
            return
        (self.running if seq in self.running else self.waiting).remove(seq)
        self.allocator.free(seq)  # nothing to free for a queued sequence
        seq.status = SequenceStatus.FINISHED
        seq.finish_reason = "abort"

    # ---- one decision ----------------------------------------------------------------
    def schedule(self) -> ScheduledBatch | None:
        """The next step's batch, or None when there is nothing to run."""
        if self.config.mixed_prefill_tokens > 0:
            return self._mixed_step()
        if self.waiting:
            fresh = self._admit()
            if fresh:
                self.running += fresh
                return ScheduledBatch(fresh, is_prefill=True)
        if not self.running:
            return None
        return self._decode_step()

    def _admit(self) -> list[Sequence]:
        """Admit from the head of the queue while the head fits (FCFS, no skipping)."""
        cfg, pool = self.config, self.allocator
        fresh: list[Sequence] = []
        widest = 0
        while self.waiting and len(self.running) + len(fresh) < cfg.max_num_seqs:
            head = self.waiting[0]
            rows = head.num_tokens  # nothing of it is cached: prompt, plus outputs after a preemption
            if (len(fresh) + 1) * max(widest, rows) > cfg.max_num_batched_tokens:
                break
            spare = cfg.watermark_blocks if (self.running or fresh) else 0
            if pool.blocks_needed(rows) + spare > pool.num_free_blocks:
                break
            self.waiting.popleft()
            pool.allocate(head)
            head.status = SequenceStatus.RUNNING
            widest = max(widest, rows)
            fresh.append(head)
        return fresh

    def _decode_step(self) -> ScheduledBatch:
        """Give every running sequence a slot for its next token, evicting the
        newest sequences while the pool has none."""
        pool, running = self.allocator, self.running
        evicted: list[Sequence] = []
        k = 0
        while k < len(running):
            seq = running[k]
            if pool.can_append_slot(seq):
                pool.append_slot(seq)
                k += 1
                continue
            victim = running.pop()  # the newest; the sequence itself when it is the newest
            self._preempt(victim)
            evicted.append(victim)
            # retry `seq` unless it was the victim (then k now points past the end)
        # Only a lone oldest sequence can be evicted, and then the whole pool is
        # free for it (rejection at add time guarantees it fits).
        assert running, "scheduler evicted every running sequence"
        return ScheduledBatch(list(running), is_prefill=False, preempted=evicted)

    def _mixed_step(self) -> ScheduledBatch | None:
        """The opt-in chunked-prefill policy: every running sequence gets the
        slots for its next tokens (evicting the newest running sequence while
        the pool has none, as a decode step does); decoding sequences feed one
        token, sequences still in their prompt feed their next chunk out of the
        step's ``mixed_prefill_tokens`` (admission order), and what is left of
        that budget admits requests from the head of the queue."""
        cfg, pool, running = self.config, self.allocator, self.running
        evicted: list[Sequence] = []
        k = 0
        while k < len(running):
            seq = running[k]
            if pool.can_append_slot(seq):
                pool.append_slot(seq)
                k += 1
                continue
            victim = running.pop()
            self._preempt(victim)
            evicted.append(victim)
        budget = cfg.mixed_prefill_tokens
        seqs: list[Sequence] = []
        lens: list[int] = []
        for seq in running:
            left = seq.num_uncached_tokens
            n = 1 if left == 1 else min(left, budget)
            if n <= 0:
                continue  # still in its prompt, no budget left this step
            if left > 1:
                budget -= n
            seqs.append(seq)
            lens.append(n)
        while self.waiting and budget > 0 and len(running) < cfg.max_num_seqs:
            head = self.waiting[0]
            rows = head.num_tokens  # nothing of it is cached: prompt, plus outputs after a preemption
            spare = cfg.watermark_blocks if running else 0
            if pool.blocks_needed(rows) + spare > pool.num_free_blocks:
                break
            self.waiting.popleft()
            pool.allocate(head)
            head.status = SequenceStatus.RUNNING
            running.append(head)
            n = min(rows, budget)
            budget -= n
            seqs.append(head)
            lens.append(n)
        if not seqs:
            return None
        return ScheduledBatch(seqs, is_prefill=False, preempted=evicted, new_lens=lens)

    def _preempt(self, seq: Sequence) -> None:
        self.num_discarded_positions += seq.num_cached_tokens  # recomputed on readmission
        self.allocator.free(seq)
        seq.reset_for_recompute()  # keeps the outputs; status WAITING
        self.waiting.appendleft(seq)  # front of the queue: arrival order is kept
        self.num_preemptions += 1
