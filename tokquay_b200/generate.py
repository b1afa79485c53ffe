"""Step drivers over the paged cache (tokquay/generate.py:63-120).

``paged_forward`` keeps the reference signature and contract: one batched
step, next-token logits ``[B, V]`` back, ``num_cached_tokens`` advanced.
"""

from __future__ import annotations

import torch

from tokquay_b200._host import ref_sequence
from tokquay_b200.kv_cache import BlockAllocator, DevicePagedBatch, PackedStep, _hostpack
from tokquay_b200.model import GPT2, argmax_rows

Sequence, SequenceStatus = ref_sequence.Sequence, ref_sequence.SequenceStatus


@torch.no_grad()
def paged_forward(
    model: GPT2,
    allocator: BlockAllocator,
    seqs: list[Sequence],
    new_lens: list[int] | None = None,
) -> torch.Tensor:
    """Run one batched step over paged KV and return next-token logits ``[B, vocab]``.

    Sequence ``i`` feeds ``token_ids[num_cached_tokens : num_cached_tokens + n_i]``
    (``n_i`` defaults to everything uncached), so prefill and decode mix freely.
    Blocks must already cover the sequences.  Advances ``num_cached_tokens``.
    """
    runner = getattr(model, "graph_runner", None)
    if runner is not None and runner.allocator is allocator:
        logits = runner.try_run(seqs, new_lens)  # a decode step: replay a captured CUDA graph
        if logits is not None:
            _advance_after_replay(seqs)
            return logits
    return _eager_forward(model, allocator, seqs, new_lens)


def _eager_forward(model: GPT2, allocator: BlockAllocator, seqs: list[Sequence],
                   new_lens: list[int] | None) -> torch.Tensor:  # fmt: skip
    lens = new_lens or [s.num_uncached_tokens for s in seqs]
    batch = DevicePagedBatch(allocator, None, None, None, packed=PackedStep.from_sequences(seqs, lens))
    logits = model.forward_paged(batch, last_only=True)[:, 0]
    for s, n in zip(seqs, lens):
        s.num_cached_tokens += n
    return logits


def _eager_greedy(model: GPT2, allocator: BlockAllocator, seqs: list[Sequence],
                  new_lens: list[int] | None) -> torch.Tensor:  # fmt: skip
    """Greedy tokens of one eager step (int64 ``[B]`` on the device): the fused
    LM head when the model has it on and the batch fits it, else the logits'
    ``tq_argmax_rows``.  Advances ``num_cached_tokens``."""
    from tokquay_b200 import _lib

    if not (model.fused_lm_head and len(seqs) <= _lib.LM_HEAD_MAX_ROWS):
        return argmax_rows(_eager_forward(model, allocator, seqs, new_lens))
    lens = new_lens or [s.num_uncached_tokens for s in seqs]
    batch = DevicePagedBatch(allocator, None, None, None, packed=PackedStep.from_sequences(seqs, lens))
    tokens = torch.empty(batch.B, dtype=torch.int64, device=allocator.pool.device)
    model.forward_paged(batch, last_only=True, greedy_out=tokens)
    for s, n in zip(seqs, lens):
        s.num_cached_tokens += n
    return tokens


def _advance_after_replay(seqs: list[Sequence]) -> None:
    if _hostpack is not None and hasattr(_hostpack, "advance_cached"):
        _hostpack.advance_cached(seqs)  # the native packer kept this step's lengths
    else:
        for s in seqs:
            s.num_cached_tokens += 1


@torch.no_grad()
def paged_greedy_step(
    model: GPT2,
    allocator: BlockAllocator,
    seqs: list[Sequence],
    new_lens: list[int] | None = None,
) -> list[int]:
    """One batched step with greedy sampling: each sequence's next token,
    ``paged_forward(...).argmax(-1).tolist()`` (the greedy rows of
    tokquay/engine.py:189-194), advancing ``num_cached_tokens`` the same way.
    A decode step that a captured CUDA graph covers returns the graph's own
    argmax: no ``[B, vocab]`` logits copy and no second argmax launch, one
    ``B x 8``-byte device-to-host read."""
    runner = getattr(model, "graph_runner", None)
    if runner is not None and runner.allocator is allocator:
        tokens = runner.try_run_greedy(seqs, new_lens)
        if tokens is not None:
            _advance_after_replay(seqs)
            return tokens.tolist()
    return _eager_greedy(model, allocator, seqs, new_lens).tolist()


@torch.no_grad()
def paged_greedy_decode(
    model: GPT2,
    allocator: BlockAllocator,
    seqs: list[Sequence],
    n_steps: int,
) -> list[list[int]]:
    """``n_steps`` greedy steps of a fixed batch: after each step every
    sequence gets its token appended (``append_token``), and every step but
    the last is followed by ``allocator.append_slot`` -- the loop of
    tokquay/generate.py:109-119 for a batch that runs ``n_steps`` more tokens.
    The first step feeds each sequence's uncached tokens, every later step one.
    Returns the new tokens per sequence.

    With captured CUDA graphs the steps are pipelined one ahead of the host:
    step k+1 is planned while step k runs and takes step k's tokens from the
    device, so the GPU does not wait for the host between steps."""
    runner = getattr(model, "graph_runner", None)
    if runner is not None and runner.allocator is allocator:
        out = runner.decode_steps(seqs, n_steps)
        if out is not None:
            return out
    out: list[list[int]] = [[] for _ in seqs]
    for k in range(n_steps):
        toks = paged_greedy_step(model, allocator, seqs)
        for s, o, t in zip(seqs, out, toks):
            s.append_token(t)
            o.append(t)
            if k + 1 < n_steps:
                allocator.append_slot(s)
    return out


@torch.no_grad()
def paged_greedy_generate(
    model: GPT2,
    allocator: BlockAllocator,
    prompts: list[list[int]],
    max_new_tokens: int,
) -> list[list[int]]:
    """Greedy-decode several prompts together (tokquay/generate.py:90-120): one
    prefill batch, then decode steps; a sequence's blocks are freed as soon as
    it has ``max_new_tokens`` outputs."""
    seqs = [Sequence(i, list(p)) for i, p in enumerate(prompts)]
    for s in seqs:
        allocator.allocate(s)
        s.status = SequenceStatus.RUNNING
    # Every sequence runs the same number of steps (max_new_tokens, at least
    # one), so the batch never changes: the prefill step, then the decode
    # steps as one pipelined run.
    paged_greedy_decode(model, allocator, seqs, 1)
    if max_new_tokens > 1:
        for s in seqs:
            allocator.append_slot(s)
        paged_greedy_decode(model, allocator, seqs, max_new_tokens - 1)
    for s in seqs:
        allocator.free(s)
        s.status = SequenceStatus.FINISHED
    return [s.output_token_ids for s in seqs]
