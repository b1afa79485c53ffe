"""The allocation-free paged-attention entry point, through the C ABI.

``tq_paged_attention_noalloc`` is for callers that cannot allocate device
memory (or hand over scratch) when they run attention: a host runtime that
passes this library only the tensors it already owns, such as a serving
process held to a fixed memory budget.  Its split-K scratch is a fixed array
inside the library.  These tests check that it gives the same rows as the
allocating entry point, twice in a row on the same shared scratch, and that a
plan too large for that scratch is refused before anything is launched.

This file is collected last so that a failure here (with ``-x``) still leaves
every other test run; it also passes on its own in a fresh process.
"""

import math
import random

import pytest
import torch

from tokquay_b200 import _lib
from tokquay_b200.kv_cache import BlockAllocator, DevicePagedBatch, cdiv
from tokquay_b200.model import GPT2Config

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

ATTN_RTOL = 2e-5  # the attention tolerance of tests/test_gpu_kernels.py, relative to max |out|


def _batch(seed: int):
    """Long decodes (split over several warps, so the scratch is used) next to
    a few prefill chunks, over a fragmented pool."""
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=2, n_head=12)
    bs = 16
    rng = random.Random(seed)
    alloc = BlockAllocator(cfg, 8 * 64 + 64, bs, device="cuda")
    random.Random(seed).shuffle(alloc._free)
    alloc.pool.normal_(generator=torch.Generator(device="cuda").manual_seed(seed))
    tables, start, new = [], [], []
    for _ in range(6):  # decodes of up to 1000 keys
        s = rng.randint(600, 999)
        tables.append(alloc._take(cdiv(s + 1, bs)))
        start.append(s)
        new.append(1)
    for _ in range(2):  # prefill chunks after a cached prefix
        s, n = rng.randint(0, 200), rng.randint(2, 40)
        tables.append(alloc._take(cdiv(s + n, bs)))
        start.append(s)
        new.append(n)
    batch = DevicePagedBatch(alloc, tables, start, new)
    assert 0 < batch.num_partials <= _lib.NOALLOC_MAX_PARTIALS
    return cfg, alloc, batch


def _noalloc(batch: DevicePagedBatch, layer: int, q: torch.Tensor, out: torch.Tensor, num_partials: int) -> int:
    a = batch.allocator
    return _lib.load().tq_paged_attention_noalloc(
        out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), a.pool.data_ptr(), a.num_blocks,
        a.cfg.n_layer, a.cfg.n_head, a.block_size, a.cfg.d_head, layer, batch.block_tables_i32.data_ptr(),
        batch.table_stride, batch.attn_plan.data_ptr(), batch.n_ctas, num_partials,
        1.0 / math.sqrt(a.cfg.d_head), torch.cuda.current_stream().cuda_stream)  # fmt: skip


def test_noalloc_matches_the_allocating_entry_point_on_two_calls_in_a_row():
    cfg, alloc, batch = _batch(0)
    C = cfg.n_embd
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(1)
    for call, layer in enumerate([1, 0]):  # second call reuses the scratch the first one left behind
        qkv = torch.randn(batch.N, 3 * C, device="cuda", generator=g)
        want = torch.full((batch.N, C), float("nan"), device="cuda")
        batch.attend_rows(layer, qkv, want, stream)
        got = torch.full((batch.N, C), float("nan"), device="cuda")
        _lib.check(_noalloc(batch, layer, qkv, got, batch.num_partials), "tq_paged_attention_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(want).all() and torch.isfinite(got).all(), call
        err = (got - want).abs().max().item()
        assert err <= ATTN_RTOL * want.abs().max().item(), (call, err)
    assert _lib.device_status() == 0


def test_noalloc_refuses_a_plan_beyond_its_scratch():
    cfg, alloc, batch = _batch(2)
    out = torch.zeros(batch.N, cfg.n_embd, device="cuda")
    qkv = torch.zeros(batch.N, 3 * cfg.n_embd, device="cuda")
    st = _noalloc(batch, 0, qkv, out, _lib.NOALLOC_MAX_PARTIALS + 1)
    assert st == _lib.TQ_ERR_CAPACITY
    assert str(_lib.NOALLOC_MAX_PARTIALS) in _lib.last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # refused before anything ran
    assert _lib.device_status() == 0


def test_noalloc_merges_split_prompt_tiles():
    """A plan whose prompt tiles are cut over their keys: the no-allocation
    entry point merges their pieces after the grid, as the allocating one does."""
    prev = _lib.prompt_tiles()
    try:
        _lib.prompt_tiles(16, 1500, 200, 4)
        cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=1, n_head=12)
        bs = 16
        rng = random.Random(5)
        alloc = BlockAllocator(cfg, 6 * 64, bs, device="cuda")
        random.Random(5).shuffle(alloc._free)
        alloc.pool.normal_(generator=torch.Generator(device="cuda").manual_seed(5))
        tables, start, new = [], [], []
        for s, n in ((0, 236), (rng.randint(100, 400), 170)) + tuple((rng.randint(16, 500), 1) for _ in range(8)):
            tables.append(alloc._take(cdiv(s + n, bs)))
            start.append(s)
            new.append(n)
        batch = DevicePagedBatch(alloc, tables, start, new)
        assert batch.tile_merges > 0 and 0 < batch.num_partials <= _lib.NOALLOC_MAX_PARTIALS
        C = cfg.n_embd
        stream = torch.cuda.current_stream().cuda_stream
        qkv = torch.randn(batch.N, 3 * C, device="cuda", generator=torch.Generator(device="cuda").manual_seed(6))
        want = torch.full((batch.N, C), float("nan"), device="cuda")
        batch.attend_rows(0, qkv, want, stream)
        got = torch.full((batch.N, C), float("nan"), device="cuda")
        _lib.check(_noalloc(batch, 0, qkv, got, batch.num_partials), "tq_paged_attention_noalloc")
        torch.cuda.synchronize()
        assert torch.isfinite(want).all() and torch.isfinite(got).all()
        err = (got - want).abs().max().item()
        assert err <= ATTN_RTOL * want.abs().max().item(), err
        assert _lib.device_status() == 0
    finally:
        _lib.prompt_tiles(prev, 1500, 200, 1)
