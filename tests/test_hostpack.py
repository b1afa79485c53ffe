"""The native step packer (``_hostpack``, tokquay_b200/csrc/hostpack.c) gives
exactly what the Python packer gives, for any mix of prefill and decode rows.
CPU only."""

import random

import numpy as np
import pytest

from tokquay_b200 import kv_cache
from tokquay_b200.kv_cache import PackedStep
from tokquay_b200.sequence import Sequence

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
