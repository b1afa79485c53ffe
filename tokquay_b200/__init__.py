"""B200-native (sm_100a) paged-attention hot path for Tokquay's paged forward.

A drop-in for Tokquay's paged path: the reference package ``tokquay`` must be
importable (``tokquay_b200._host``), and its ``Sequence``, scheduler and engine
run unchanged over this package's allocator and model.

Public surface, mirroring the reference's modules:

* ``GPT2Config`` (the reference's), ``GPT2``     (tokquay/model.py)
* ``BlockAllocator`` (a subclass of the reference's), ``BatchedKV``,
  ``OutOfBlocksError``, ``DevicePagedBatch``      (tokquay/kv_cache.py)
* ``Sequence``, ``SamplingParams``, ``SequenceStatus``: the reference's
                                                  (tokquay/sequence.py)
* ``paged_forward``, ``paged_greedy_generate``   (tokquay/generate.py),
  ``paged_greedy_step`` (one step + greedy tokens), ``paged_greedy_decode``
  (a fixed batch's greedy steps, pipelined over CUDA graphs)

The CUDA kernels live in ``libtokquay_b200.so`` (C ABI: include/tokquay_b200.h),
built in-tree by ``python -m tokquay_b200.build``.
"""

from tokquay_b200._host import ref_sequence

Sequence, SamplingParams, SequenceStatus = ref_sequence.Sequence, ref_sequence.SamplingParams, ref_sequence.SequenceStatus

from tokquay_b200.kv_cache import (  # noqa: F401
    BatchedKV,
    BlockAllocator,
    DevicePagedBatch,
    OutOfBlocksError,
    cdiv,
)
from tokquay_b200.model import GPT2, GPT2Config  # noqa: F401
from tokquay_b200.generate import (  # noqa: F401
    paged_forward,
    paged_greedy_decode,
    paged_greedy_generate,
    paged_greedy_step,
)

__all__ = [
    "BatchedKV",
    "BlockAllocator",
    "DevicePagedBatch",
    "GPT2",
    "GPT2Config",
    "OutOfBlocksError",
    "SamplingParams",
    "Sequence",
    "SequenceStatus",
    "cdiv",
    "paged_forward",
    "paged_greedy_decode",
    "paged_greedy_step",
    "paged_greedy_generate",
]
