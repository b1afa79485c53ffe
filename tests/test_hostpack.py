"""The native step packer (``_hostpack``, tokquay_b200/csrc/hostpack.c) gives
exactly what the Python packer gives, for any mix of prefill and decode rows.
CPU only."""

import random

import numpy as np
import pytest

from tokquay_b200 import kv_cache
from tokquay_b200.kv_cache import PackedStep
from tokquay.sequence import Sequence

hostpack = pytest.importorskip("tokquay_b200._hostpack")


def python_pack(seqs, new_lens):
    saved = kv_cache._hostpack
    kv_cache._hostpack = None
    try:
        return PackedStep.from_sequences(seqs, new_lens)
    finally:
        kv_cache._hostpack = saved


def random_seqs(rng, n):
    seqs = []
    for i in range(n):
        s = Sequence(i, [rng.randrange(50257) for _ in range(rng.randint(1, 60))])
        for _ in range(rng.randint(0, 30)):
            s.append_token(rng.randrange(50257))
        s.block_table = [rng.randrange(10_000) for _ in range(rng.randint(0, 40))]
        s.num_cached_tokens = rng.randint(0, s.num_tokens - 1)
        seqs.append(s)
    return seqs


@pytest.mark.parametrize("seed", range(20))
def test_native_packer_matches_python(seed):
    rng = random.Random(seed)
    seqs = random_seqs(rng, rng.randint(1, 40))
    for new_lens in (None, [rng.randint(1, s.num_uncached_tokens) for s in seqs]):
        got = PackedStep.from_sequences(seqs, new_lens)
        want = python_pack(seqs, new_lens)
        for name in PackedStep.__slots__:
            np.testing.assert_array_equal(getattr(got, name), getattr(want, name), err_msg=name)


def test_native_packer_rejects_what_the_planner_must_see():
    s = Sequence(0, [1, 2, 3])
    s.num_cached_tokens = 1
    with pytest.raises(ValueError):
        PackedStep.from_sequences([s], [5])  # more tokens than the sequence has
    with pytest.raises(ValueError):
        PackedStep.from_sequences([], None)


@pytest.mark.parametrize("seed", range(8))
def test_native_pack_and_plan_matches_the_python_path(seed):
    """plan_sequences (pack in C, then tq_plan_step) writes the plan that
    from_sequences + plan_packed writes, with and without fixed capacities."""
    from tokquay_b200 import _lib
    from tokquay_b200.kv_cache import MIN_SPLIT_CHUNKS, attention_warps, plan_packed

    rng = random.Random(100 + seed)
    seqs = random_seqs(rng, rng.randint(1, 30))
    for s in seqs:  # a valid step: tables cover every sequence, block ids in the pool
        s.block_table = [rng.randrange(4000) for _ in range(-(-s.num_tokens // 16))]
    new_lens = [rng.randint(1, s.num_uncached_tokens) for s in seqs]
    n_ctas = rng.choice([1, 7, 148])
    caps = np.array([64, 4096, 64, 64 * 12 * 16 + n_ctas * attention_warps(), 64, 4096 * 12 * 8], np.int32)
    for cp in (None, caps):
        want, wl = plan_packed(16, 4000, 12, PackedStep.from_sequences(seqs, new_lens), 50257, n_ctas,
                               MIN_SPLIT_CHUNKS, caps=cp)  # fmt: skip
        out = np.full(int(wl[_lib.PLAN_TOTAL_INTS]), -7, np.int32)
        layout = np.zeros(_lib.PLAN_LAYOUT_LEN, np.int32)
        st = hostpack.plan_sequences(_lib.function_address("tq_plan_step"), seqs, new_lens, 16, 4000, 12, 50257,
                                     n_ctas, MIN_SPLIT_CHUNKS, 0 if cp is None else cp.ctypes.data, out.ctypes.data,
                                     out.size, layout.ctypes.data)  # fmt: skip
        assert st == 0
        np.testing.assert_array_equal(layout, wl)
        used = int(wl[_lib.PLAN_USED_INTS])
        np.testing.assert_array_equal(out[:used], want[:used])
    # a batch the planner rejects comes back as its status, the message in tq_last_error
    short = Sequence(99, [1, 2, 3, 4, 5])
    short.block_table = [0]
    st = hostpack.plan_sequences(_lib.function_address("tq_plan_step"), [short], None, 4, 4000, 12, 50257, 1, 8, 0,
                                 out.ctypes.data, out.size, layout.ctypes.data)  # fmt: skip
    assert st == _lib.TQ_ERR_INVALID and "cannot hold 5 tokens" in _lib.last_error()
    # one the packer rejects raises before the planner runs
    bad = seqs[0]
    with pytest.raises(ValueError):
        hostpack.plan_sequences(_lib.function_address("tq_plan_step"), [bad], [bad.num_uncached_tokens + 5], 16,
                                4000, 12, 50257, 1, 8, 0, out.ctypes.data, out.size, layout.ctypes.data)  # fmt: skip


def test_decode_only_planning_and_advance():
    """decode_max_ctx: a step with a prefill row, or a context past the limit,
    comes back as -2 with nothing planned; a decode step is planned and
    advance_cached moves every sequence on by its one token."""
    from tokquay_b200 import _lib
    from tokquay_b200.kv_cache import MIN_SPLIT_CHUNKS

    fn = _lib.function_address("tq_plan_step")
    seqs = []
    for i in range(5):
        s = Sequence(i, list(range(10 + i)))
        s.num_cached_tokens = s.num_tokens - 1
        s.block_table = list(range(i * 4, i * 4 + 4))
        seqs.append(s)
    out = np.zeros(1 << 16, np.int32)
    layout = np.zeros(_lib.PLAN_LAYOUT_LEN, np.int32)
    args = (16, 64, 12, 0, 3, MIN_SPLIT_CHUNKS, 0, out.ctypes.data, out.size, layout.ctypes.data)
    assert hostpack.plan_sequences(fn, seqs, None, *args, 64) == 0
    before = [s.num_cached_tokens for s in seqs]
    hostpack.advance_cached(seqs)
    assert [s.num_cached_tokens for s in seqs] == [b + 1 for b in before]
    with pytest.raises(RuntimeError):
        hostpack.advance_cached(seqs)  # only once per planned step
    for s in seqs:  # one more token each: still a decode step
        s.append_token(7)
    assert hostpack.plan_sequences(fn, seqs, None, *args, 14) == -2  # context 15 > 14
    seqs[2].num_cached_tokens -= 3  # a prefill-like row (4 new tokens)
    assert hostpack.plan_sequences(fn, seqs, None, *args, 64) == -2
    with pytest.raises(RuntimeError):
        hostpack.advance_cached(seqs)  # nothing was planned
    assert hostpack.plan_sequences(fn, seqs, None, *args) == 0  # no decode check: planned
