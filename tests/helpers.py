"""Helpers shared by the CPU and GPU tests: golden fixtures and case rebuilding.

Weights and pool contents are rebuilt from the seeds recorded in
``tests/golden/golden.json`` (see tests/golden/make_golden.py); integer data
(token ids, block tables) come from the fixture itself.
"""

from __future__ import annotations

import functools
import json
import random
from pathlib import Path
from types import SimpleNamespace

import numpy as np

from tokquay_b200 import workloads as W
from tokquay_b200.model import GPT2Config
from tokquay.sequence import Sequence

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"

# CUDA fp32 path vs the reference's fp32 logits: the north-star bound.
LOGITS_ATOL = 1e-4
# numpy oracle (fp32) vs the reference (torch fp32 on the CPU): different
# summation orders only.
ORACLE_F32_ATOL = 1e-5
# float64 runs agree to rounding noise (tests/test_phase3_paged.py uses 1e-9).
F64_ATOL = 1e-9


@functools.lru_cache(maxsize=None)
def load_golden() -> SimpleNamespace:
    meta = json.loads((GOLDEN_DIR / "golden.json").read_text())
    with np.load(GOLDEN_DIR / "golden.npz") as z:
        arrays = {k: z[k] for k in z.files}
    return SimpleNamespace(meta=meta, cases=meta["cases"], arrays=arrays)


def cfg_of(case: dict) -> GPT2Config:
    return GPT2Config(**case["cfg"]) if "cfg" in case else GPT2Config(**W.GPT2_SMALL)


@functools.lru_cache(maxsize=None)
def gpt2_small_weights() -> dict[str, np.ndarray]:
    return W.random_weights(GPT2Config(**W.GPT2_SMALL), 0, "normal")


def weights_of(case: dict) -> dict[str, np.ndarray]:
    if "cfg" not in case and case["weights_seed"] == 0 and case["init"] == "normal":
        return gpt2_small_weights()
    return W.random_weights(cfg_of(case), case["weights_seed"], case["init"])


def pool_shape(cfg: GPT2Config, num_blocks: int, bs: int) -> tuple[int, ...]:
    return (num_blocks, cfg.n_layer, 2, cfg.n_head, bs, cfg.d_head)


def mixed_prompt_lists(case: dict, vocab: int):
    """Token lists of a config-3 case, regenerated the way workloads.mixed_case draws them."""
    rng = random.Random(case["seed"])
    kinds = ["p"] * case["n_prefill"] + ["d"] * case["n_decode"]
    rng.shuffle(kinds)
    lens = [rng.randint(*case["len_range"]) for _ in kinds]
    toks = [[rng.randrange(vocab) for _ in range(n)] for n in lens]
    return kinds, lens, toks


def decode_token_lists(n_seqs: int, ctx_range, vocab: int, seed: int):
    rng = random.Random(seed)
    ctx = [rng.randint(*ctx_range) for _ in range(n_seqs)]
    toks = [[rng.randrange(vocab) for _ in range(c)] for c in ctx]
    return ctx, toks


def build_config_case(name: str, golden, SequenceCls=Sequence, alloc=None):
    """Rebuild the sequences of config case ``name`` with their golden block
    tables.  With ``alloc`` (an allocator of this package) the tables are
    produced by the allocator instead, and returned for comparison."""
    case = golden.cases[name]
    cfg = GPT2Config(**W.GPT2_SMALL)
    if name.startswith("cfg3"):
        kinds, lens, toks = mixed_prompt_lists(case, cfg.vocab_size)
        if alloc is not None:
            sc = W.mixed_case(SequenceCls, alloc, case["n_prefill"], case["n_decode"], tuple(case["len_range"]),
                              cfg.vocab_size, seed=case["seed"])  # fmt: skip
            return sc.seqs, sc.new_lens
        seqs, new_lens = [], []
        for i, (k, n, t) in enumerate(zip(kinds, lens, toks)):
            s = SequenceCls(i, t)
            s.block_table = list(case["tables"][i])
            if k == "d":
                s.num_cached_tokens = n - 1
                new_lens.append(1)
            else:
                new_lens.append(n)
            seqs.append(s)
        return seqs, new_lens
    if alloc is not None:
        sc = W.decode_case(SequenceCls, alloc, case["n_seqs"], tuple(case["ctx_range"]), cfg.vocab_size,
                           seed=case["seed"])  # fmt: skip
        return sc.seqs, sc.new_lens
    ctx, toks = decode_token_lists(case["n_seqs"], tuple(case["ctx_range"]), cfg.vocab_size, case["seed"])
    tables = case["tables"] if "tables" in case else case["steps"][0]["tables"]
    seqs = []
    for i, (c, t) in enumerate(zip(ctx, toks)):
        s = SequenceCls(i, t)
        s.block_table = list(tables[i])
        s.num_cached_tokens = c - 1
        seqs.append(s)
    return seqs, [1] * len(seqs)


def numpy_pool(cfg: GPT2Config, num_blocks: int, bs: int, blocks, seed: int, scale: float = 1.0,
               dtype=np.float32) -> np.ndarray:  # fmt: skip
    pool = np.zeros(pool_shape(cfg, num_blocks, bs), dtype=dtype)
    W.fill_pool_blocks(pool, blocks, seed, scale)
    return pool


def logits_cols(logits: np.ndarray, stride: int) -> np.ndarray:
    return np.asarray(logits)[:, ::stride]
