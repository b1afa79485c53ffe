"""Opt-in chunked-prefill scheduling over the paged path.

The reference's scheduler (tokquay/scheduler.py) is the default and runs
unchanged: ``Engine`` uses it as it is whenever ``mixed_prefill_tokens`` is 0.
Its policy alternates steps: a step that admits prompts runs only prompts
(tokquay/scheduler.py:9-17), so every running sequence waits through it.

``SchedulerConfig(mixed_prefill_tokens=P)`` with P > 0 selects ``Scheduler``
below, a subclass that keeps every rule of the reference's -- FCFS admission
without skipping, blocks for the whole prompt reserved at admission, the
watermark, preemption of the newest running sequence by recompute, the
up-front rejections -- and changes only what one step holds: every decoding
sequence plus up to P prompt tokens, first the next chunk of each running
sequence still in its prompt (admission order), then requests admitted from
the head of the queue.  The paged attention kernel runs the prompt chunks
(causal, from any cached start) and the decode rows in one launch per layer.
"""

from __future__ import annotations

from dataclasses import dataclass

from tokquay_b200._host import ref_scheduler, ref_sequence

__all__ = ["RequestRejected", "SchedulerConfig", "ScheduledBatch", "MixedBatch", "Scheduler"]

RequestRejected = ref_scheduler.RequestRejected
ScheduledBatch = ref_scheduler.ScheduledBatch
_RUNNING = ref_sequence.SequenceStatus.RUNNING


@dataclass
class SchedulerConfig(ref_scheduler.SchedulerConfig):
    """The reference's limits (tokquay/scheduler.py:46-57) plus
    ``mixed_prefill_tokens``: > 0 opts in to chunked prefill with that many
    prompt tokens per step; 0 is the reference's policy."""

    mixed_prefill_tokens: int = 0

    def __post_init__(self) -> None:
        super().__post_init__()
        if self.mixed_prefill_tokens < 0:
            raise ValueError("mixed_prefill_tokens must be >= 0")


@dataclass
class MixedBatch(ScheduledBatch):
    """A chunked-prefill step: ``new_lens[i]`` tokens of ``seqs[i]`` are fed
    (1 for a decoding sequence, a prompt chunk otherwise).  ``padded_tokens``
    counts rows x longest row, as the reference's batch does."""

    new_lens: list[int] | None = None

    def __post_init__(self) -> None:
        self.padded_tokens = len(self.seqs) * max(self.new_lens)


class Scheduler(ref_scheduler.Scheduler):
    """The reference scheduler with the opt-in chunked-prefill step."""

    def __init__(self, allocator, config: SchedulerConfig):
        if config.mixed_prefill_tokens <= 0:
            raise ValueError("this scheduler is the chunked-prefill policy: mixed_prefill_tokens must be > 0 "
                             "(use tokquay.scheduler.Scheduler for the alternating policy)")
        super().__init__(allocator, config)

    def schedule(self) -> MixedBatch | None:
        """Grow every running sequence's table for its next tokens (evicting the
        newest running sequences while the pool is short, as the reference's
        decode step does), then fill the step's prompt-token budget: running
        sequences still in their prompt first, then the queue's head, FCFS."""
        cfg, pool, running = self.config, self.allocator, self.running
        evicted = self._schedule_decode().preempted if running else []
        budget = cfg.mixed_prefill_tokens
        seqs, lens = [], []
        for seq in running:
            left = seq.num_uncached_tokens
            take = 1 if left == 1 else min(left, budget)
            if take <= 0:
                continue  # mid-prompt, and this step's prompt budget is spent
            if left > 1:
                budget -= take
            seqs.append(seq)
            lens.append(take)
        while budget > 0 and self.waiting and len(running) < cfg.max_num_seqs:
            head = self.waiting[0]
            need = head.num_tokens  # nothing of it is cached (prompt, plus outputs after a preemption)
            spare = cfg.watermark_blocks if running else 0
            if pool.blocks_needed(need) + spare > pool.num_free_blocks:
                break  # FCFS: never skip ahead of the head of the queue
            self.waiting.popleft()
            pool.allocate(head)
            head.status = _RUNNING
            running.append(head)
            take = min(need, budget)
            budget -= take
            seqs.append(head)
            lens.append(take)
        if not seqs:
            return None
        return MixedBatch(seqs, is_prefill=False, preempted=evicted, new_lens=lens)
