"""CPU oracle for the paged-attention hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference Tokquay algorithm that the CUDA
path replaces: the block-pool K/V scatter, the dense per-step gather, masked
softmax attention and the GPT-2 forward around it.  It exists to check the
product, never to be the product: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it.  Nothing under ``tokquay_b200/`` imports it, and the product raises when
its CUDA library is missing instead of falling back here.

Parity pin: ``tests/test_oracle_golden.py`` checks this restatement against
golden vectors produced by the unmodified reference implementation
(``tests/golden/make_golden.py`` imports the reference and records its outputs).
"""

from oracle.paged_ref import (  # noqa: F401
    OracleBatch,
    cdiv,
    gather,
    gelu_tanh,
    gpt2_forward,
    layer_norm,
    masked_attention,
    paged_forward,
    write,
)
