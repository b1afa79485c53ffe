"""Seeded synthetic workloads for the BASELINE configurations.

Everything is derived from integer seeds with numpy's PCG64 and Python's
``random.Random``, so the same case can be rebuilt bit for bit on any machine
(the fixture generator, the CPU tests and the GPU box) without storing weights
or pools.  There are no real GPT-2 weights or prompts here: weights are
random-init N(0, 0.02) and token ids are uniform over the vocabulary.

The builders are written against the ``Sequence`` / ``BlockAllocator``
interface only, so the same function sets up a case for this package and for
the reference implementation (block tables then have to come out identical).
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field

import numpy as np

# GPT-2 124M and a small model with the same head size for fast cases.
GPT2_SMALL = dict(vocab_size=50257, n_positions=1024, n_embd=768, n_layer=12, n_head=12)
MINI = dict(vocab_size=512, n_positions=128, n_embd=128, n_layer=2, n_head=2)


def param_specs(cfg) -> list[tuple[str, tuple[int, ...]]]:
    """State-dict names and shapes of the GPT-2 model, in a fixed order."""
    C, V, P, L = cfg.n_embd, cfg.vocab_size, cfg.n_positions, cfg.n_layer
    specs: list[tuple[str, tuple[int, ...]]] = [("wte.weight", (V, C)), ("wpe.weight", (P, C))]
    for i in range(L):
        p = f"h.{i}."
        specs += [
            (p + "ln_1.weight", (C,)), (p + "ln_1.bias", (C,)),
            (p + "attn.c_attn.weight", (3 * C, C)), (p + "attn.c_attn.bias", (3 * C,)),
            (p + "attn.c_proj.weight", (C, C)), (p + "attn.c_proj.bias", (C,)),
            (p + "ln_2.weight", (C,)), (p + "ln_2.bias", (C,)),
            (p + "mlp.c_fc.weight", (4 * C, C)), (p + "mlp.c_fc.bias", (4 * C,)),
            (p + "mlp.c_proj.weight", (C, 4 * C)), (p + "mlp.c_proj.bias", (C,)),
        ]  # fmt: skip
    specs += [("ln_f.weight", (C,)), ("ln_f.bias", (C,))]
    return specs


def random_weights(cfg, seed: int, init: str = "normal") -> dict[str, np.ndarray]:
    """float32 weights.  ``init="normal"``: every parameter N(0, 0.02) (the
    BASELINE's random init).  ``init="gpt2"``: the same draws, but LayerNorm
    weights 1 and all biases / LayerNorm shifts 0 (larger activations, larger
    logit gaps: a stricter numerical check)."""
    if init not in ("normal", "gpt2"):
        raise ValueError(init)
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in param_specs(cfg):
        w = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
        if init == "gpt2":
            if name.endswith(".bias"):
                w = np.zeros(shape, np.float32)
            elif ".ln_" in name or name.startswith("ln_f"):
                w = np.ones(shape, np.float32)
        out[name] = w
    return out


def load_weights(model, weights: dict[str, np.ndarray], dtype=None) -> None:
    """Copy numpy weights into a torch GPT-2 (this package's or the reference's)."""
    import torch

    sd = {k: torch.from_numpy(v) for k, v in weights.items()}
    if dtype is not None:
        sd = {k: v.to(dtype) for k, v in sd.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    if missing or unexpected:
        raise KeyError(f"state dict mismatch: missing {missing}, unexpected {unexpected}")


def block_values(block_shape: tuple[int, ...], seed: int, block: int, scale: float = 1.0) -> np.ndarray:
    """Contents of pool block ``block``: N(0, scale^2), from the stream (seed, block)."""
    v = np.random.default_rng([seed, block]).standard_normal(block_shape, dtype=np.float32)
    return v * np.float32(scale) if scale != 1.0 else v


def fill_pool_blocks(pool, blocks, seed: int, scale: float = 1.0) -> None:
    """Fill the given blocks of ``pool`` (a numpy array or torch tensor, any
    device) with their seeded values."""
    shape = tuple(pool.shape[1:])
    for b in sorted(set(int(x) for x in blocks)):
        vals = block_values(shape, seed, b, scale)
        if isinstance(pool, np.ndarray):
            pool[b] = vals.astype(pool.dtype, copy=False)
        else:
            import torch

            pool[b].copy_(torch.from_numpy(vals).to(pool.dtype))


def shuffle_free_list(alloc, seed: int) -> None:
    """Fragment block tables: shuffle the free list with ``random.Random(seed)``
    (the adversarial fixture of tests/test_phase3_paged.py:52-59)."""
    random.Random(seed).shuffle(alloc._free)


@dataclass
class StepCase:
    """One paged step: sequences (with blocks) and how many tokens each feeds."""

    seqs: list
    new_lens: list[int]
    meta: dict = field(default_factory=dict)

    @property
    def block_tables(self) -> list[list[int]]:
        return [list(s.block_table) for s in self.seqs]


def decode_case(SequenceCls, alloc, n_seqs: int, ctx_range: tuple[int, int], vocab: int, seed: int,
                free_seed: int | None = None, shard: tuple[int, int] = (0, 1)) -> StepCase:  # fmt: skip
    """Decode step (configs 1, 2, 4): ``n_seqs`` sequences with context lengths
    uniform in ``ctx_range`` and uniform token ids, all from ``random.Random(seed)``;
    each owns blocks for its whole context and has ``ctx-1`` positions cached,
    so the step feeds its last token.  ``shard=(r, n)`` keeps sequences
    r, r+n, r+2n, ... of that batch (one replica's share, config 4)."""
    rng = random.Random(seed)
    ctx = [rng.randint(*ctx_range) for _ in range(n_seqs)]
    toks = [[rng.randrange(vocab) for _ in range(c)] for c in ctx]
    r, n = shard
    ctx, toks = ctx[r::n], toks[r::n]
    shuffle_free_list(alloc, seed if free_seed is None else free_seed)
    seqs = []
    for i, (c, t) in enumerate(zip(ctx, toks)):
        s = SequenceCls(i, t)
        alloc.allocate(s)
        s.num_cached_tokens = c - 1
        seqs.append(s)
    return StepCase(seqs, [1] * len(seqs), {"ctx": ctx})


def mixed_case(SequenceCls, alloc, n_prefill: int, n_decode: int, len_range: tuple[int, int], vocab: int,
               seed: int) -> StepCase:  # fmt: skip
    """Mixed step (config 3): ``n_prefill`` fresh prompts (start 0, whole prompt)
    and ``n_decode`` decoding sequences, lengths uniform in ``len_range``, in a
    seeded interleaved order."""
    rng = random.Random(seed)
    kinds = ["p"] * n_prefill + ["d"] * n_decode
    rng.shuffle(kinds)
    lens = [rng.randint(*len_range) for _ in kinds]
    toks = [[rng.randrange(vocab) for _ in range(n)] for n in lens]
    shuffle_free_list(alloc, seed)
    seqs, new_lens = [], []
    for i, (k, n, t) in enumerate(zip(kinds, lens, toks)):
        s = SequenceCls(i, t)
        alloc.allocate(s)
        if k == "d":
            s.num_cached_tokens = n - 1
            new_lens.append(1)
        else:
            new_lens.append(n)
        seqs.append(s)
    return StepCase(seqs, new_lens, {"kinds": kinds, "lens": lens})


def used_blocks(case: StepCase) -> list[int]:
    return sorted({b for s in case.seqs for b in s.block_table})


# BASELINE.json configs (GPT-2 124M, fp32, random init).
CONFIGS = {
    1: dict(n_seqs=8, ctx_range=(16, 256), block_size=16, num_blocks=1024),
    # 1,024 blocks cannot hold 64 contexts of up to 512 tokens (+100 decode
    # steps), so config 2 runs on 2,048 blocks, for the reference and this build alike.
    2: dict(n_seqs=64, ctx_range=(16, 512), block_size=16, num_blocks=2048, steps=100),
    3: dict(n_prefill=4, n_decode=60, len_range=(16, 256), block_sizes=(16, 32), num_blocks=1024),
    4: dict(n_seqs=512, ctx_range=(256, 1024), block_size=32, pool_bytes=150e9),
}

# Config 4's parity case: every 8th of its 512 sequences (the share of one of
# eight replicas) on a pool of 4,096 blocks (9.7 GB), a size the reference's
# dense-gather forward also runs at on a host.
CFG4_SUBSET = dict(shard=(0, 8), num_blocks=4096, steps=3)
