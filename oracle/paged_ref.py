"""numpy restatement of Tokquay's paged forward (TEST INFRASTRUCTURE ONLY).

Every function names the reference lines it restates (paths are relative to the
Tokquay project root).  The algorithm is kept as the reference has it -- build
padded index tensors, scatter the new K/V, gather each sequence's blocks into a
dense copy, run masked softmax attention over the padded key axis -- because
this module is the parity oracle and the CPU baseline for that algorithm, not a
fast implementation of it.

Weights are a ``dict[str, np.ndarray]`` keyed like the reference model's
``state_dict`` (``wte.weight``, ``h.0.attn.c_attn.weight`` ...), linear weights
in ``nn.Linear`` layout ``[out, in]``.  Arithmetic runs in the dtype of the
arrays given (float32 for parity with the fp32 path, float64 for the
noise-free self-consistency checks the reference's own tests make).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


def cdiv(a: int, b: int) -> int:
    """Ceiling division (tokquay/kv_cache.py:30-31)."""
    return -(-a // b)


# ----------------------------------------------------------------------------- per-step view
@dataclass
class OracleBatch:
    """Index arrays of one step, as ``PagedBatch.__init__`` builds them
    (tokquay/kv_cache.py:174-226)."""

    B: int
    T: int
    nb: int
    max_ctx: int
    block_tables: np.ndarray  # int64 [B, nb], padded with block 0 (kv_cache.py:200-201)
    positions: np.ndarray  # int64 [B, T] (kv_cache.py:205)
    last_idx: np.ndarray  # int64 [B] (kv_cache.py:206)
    mask: np.ndarray  # bool [B, 1, T, nb*bs] (kv_cache.py:213-214)
    w_b: np.ndarray  # scatter targets of the valid new tokens (kv_cache.py:217-226)
    w_t: np.ndarray
    w_blk: np.ndarray
    w_off: np.ndarray

    @classmethod
    def build(cls, block_size: int, block_tables: list[list[int]], start: list[int], new_lens: list[int]):
        # Validation and its error messages follow kv_cache.py:182-191.
        if not block_tables or not (len(block_tables) == len(start) == len(new_lens)):
            raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
        if min(new_lens) < 1:
            raise ValueError("every sequence must feed at least one token")
        bs = block_size
        ctx = [s + n for s, n in zip(start, new_lens)]
        for b, (tbl, c) in enumerate(zip(block_tables, ctx)):
            if len(tbl) < cdiv(c, bs):
                raise ValueError(f"sequence {b}: {len(tbl)} blocks cannot hold {c} tokens")
        B, T = len(block_tables), max(new_lens)
        nb = max(cdiv(c, bs) for c in ctx)
        padded = [list(tbl[:nb]) + [0] * (nb - len(tbl[:nb])) for tbl in block_tables]
        tables = np.asarray(padded, dtype=np.int64).reshape(B, nb)
        start_a = np.asarray(start, dtype=np.int64)
        ctx_a = np.asarray(ctx, dtype=np.int64)
        positions = start_a[:, None] + np.arange(T, dtype=np.int64)[None, :]
        last_idx = np.asarray([n - 1 for n in new_lens], dtype=np.int64)
        k_pos = np.arange(nb * bs, dtype=np.int64)[None, None, :]
        mask = ((k_pos <= positions[:, :, None]) & (k_pos < ctx_a[:, None, None]))[:, None]
        w_b, w_t, w_blk, w_off = [], [], [], []
        for b, (tbl, s, n) in enumerate(zip(block_tables, start, new_lens)):
            for t in range(n):
                p = s + t
                w_b.append(b)
                w_t.append(t)
                w_blk.append(tbl[p // bs])
                w_off.append(p % bs)
        as64 = lambda x: np.asarray(x, dtype=np.int64)  # noqa: E731
        return cls(B, T, nb, max(ctx), tables, positions, last_idx, mask,
                   as64(w_b), as64(w_t), as64(w_blk), as64(w_off))  # fmt: skip


def write(pool: np.ndarray, layer: int, k: np.ndarray, v: np.ndarray, batch: OracleBatch) -> None:
    """Scatter the valid new K/V rows ``[B, H, T, d]`` into the pool
    (tokquay/kv_cache.py:228-232).  ``pool`` is ``[NB, L, 2, H, bs, d]``."""
    pool[batch.w_blk, layer, 0, :, batch.w_off] = k[batch.w_b, :, batch.w_t]
    pool[batch.w_blk, layer, 1, :, batch.w_off] = v[batch.w_b, :, batch.w_t]


def gather(pool: np.ndarray, layer: int, batch: OracleBatch) -> tuple[np.ndarray, np.ndarray]:
    """Dense copy of every sequence's blocks, ``[B, H, nb*bs, d]`` for K and V
    (tokquay/kv_cache.py:234-242)."""
    out = []
    for kv in (0, 1):
        g = pool[batch.block_tables, layer, kv]  # [B, nb, H, bs, d]
        g = g.transpose(0, 2, 1, 3, 4)  # [B, H, nb, bs, d]
        out.append(np.ascontiguousarray(g).reshape(batch.B, g.shape[1], -1, g.shape[-1]))
    return out[0], out[1]


# ----------------------------------------------------------------------------- math
def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray, eps: float) -> np.ndarray:
    """``nn.LayerNorm`` over the last axis: biased variance, eps inside the root
    (used at tokquay/model.py:122-123 and :180)."""
    mean = x.mean(axis=-1, keepdims=True)
    xc = x - mean
    var = (xc * xc).mean(axis=-1, keepdims=True)
    return xc / np.sqrt(var + x.dtype.type(eps)) * w + b


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """GELU with the tanh approximation, ``F.gelu(approximate="tanh")``
    (tokquay/model.py:110)."""
    t = x.dtype.type
    c = t(math.sqrt(2.0 / math.pi))
    # 0.5 * x * (1 + tanh(c * (x + 0.044715 * x * x * x))), evaluated in the
    # same order, in place (fewer temporaries; the same rounding step by step).
    a = x * t(0.044715)
    a *= x
    a *= x
    a += x
    a *= c
    np.tanh(a, out=a)
    a += t(1.0)
    out = x * t(0.5)
    out *= a
    return out


def linear(x: np.ndarray, w: np.ndarray, b: np.ndarray | None) -> np.ndarray:
    """``nn.Linear``: ``x @ w.T + b`` with ``w`` in ``[out, in]`` layout."""
    y = x @ w.T
    return y + b if b is not None else y


def masked_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, allowed: np.ndarray) -> np.ndarray:
    """``softmax(q kᵀ / sqrt(d), masked) v`` over ``[B, H, T, S]`` scores
    (tokquay/model.py:94-96).  Fully masked rows (padded queries whose slots
    lie beyond every key) give NaN, as in the reference; callers discard them."""
    d = q.shape[-1]
    scores = (q @ np.swapaxes(k, -1, -2)) / q.dtype.type(math.sqrt(d))
    scores = np.where(allowed, scores, -np.inf)
    with np.errstate(invalid="ignore"):
        m = scores.max(axis=-1, keepdims=True)
        p = np.exp(scores - m)
        p = p / p.sum(axis=-1, keepdims=True)
    return p @ v


# ----------------------------------------------------------------------------- model
def gpt2_forward(
    weights: dict[str, np.ndarray],
    cfg,
    input_ids: np.ndarray,
    pool: np.ndarray,
    batch: OracleBatch,
    last_only: bool = True,
) -> np.ndarray:
    """Paged GPT-2 forward: ``input_ids [B, T]`` -> logits ``[B, 1|T, V]``
    (tokquay/model.py:136-181 with the paged branch of Attention.forward,
    :67-78 and :94-99; Block.forward :121-124; MLP.forward :108-110).

    ``cfg`` needs ``n_layer, n_head, n_embd, n_positions, layer_norm_eps``.
    """
    B, T = input_ids.shape
    if (B, T) != (batch.B, batch.T):  # model.py:157-158
        raise ValueError(f"input_ids {tuple(input_ids.shape)} does not match batch {(batch.B, batch.T)}")
    if batch.max_ctx > cfg.n_positions:  # model.py:159-160
        raise ValueError(f"sequence length {batch.max_ctx} exceeds n_positions={cfg.n_positions}")
    W = weights
    C, H = cfg.n_embd, cfg.n_head
    d = C // H
    eps = cfg.layer_norm_eps
    pos = np.minimum(batch.positions, cfg.n_positions - 1)  # model.py:163
    x = W["wte.weight"][input_ids] + W["wpe.weight"][pos]  # model.py:172
    for i in range(cfg.n_layer):
        p = f"h.{i}."
        h = layer_norm(x, W[p + "ln_1.weight"], W[p + "ln_1.bias"], eps)
        qkv = linear(h, W[p + "attn.c_attn.weight"], W[p + "attn.c_attn.bias"])  # model.py:69
        q, k, v = (qkv[..., j * C:(j + 1) * C].reshape(B, T, H, d).transpose(0, 2, 1, 3) for j in range(3))
        write(pool, i, k, v, batch)  # model.py:76
        kd, vd = gather(pool, i, batch)  # model.py:77
        a = masked_attention(q, kd, vd, batch.mask)  # model.py:94-96
        a = a.transpose(0, 2, 1, 3).reshape(B, T, C)  # model.py:98
        x = x + linear(a, W[p + "attn.c_proj.weight"], W[p + "attn.c_proj.bias"])  # model.py:99, :122
        h = layer_norm(x, W[p + "ln_2.weight"], W[p + "ln_2.bias"], eps)
        h = gelu_tanh(linear(h, W[p + "mlp.c_fc.weight"], W[p + "mlp.c_fc.bias"]))
        x = x + linear(h, W[p + "mlp.c_proj.weight"], W[p + "mlp.c_proj.bias"])  # model.py:123
    if last_only:
        x = x[np.arange(B), batch.last_idx][:, None]  # model.py:179
    x = layer_norm(x, W["ln_f.weight"], W["ln_f.bias"], eps)  # model.py:180
    return x @ W["wte.weight"].T  # tied LM head, model.py:181


def paged_forward(weights, cfg, pool, block_size, seqs, new_lens=None) -> np.ndarray:
    """One batched step over paged KV; returns ``[B, V]`` next-token logits and
    advances ``num_cached_tokens`` (tokquay/generate.py:63-87).

    ``seqs`` are objects with ``token_ids``, ``num_cached_tokens``,
    ``num_uncached_tokens`` and ``block_table`` (any ``Sequence``-like type).
    """
    lens = new_lens or [s.num_uncached_tokens for s in seqs]
    starts = [s.num_cached_tokens for s in seqs]
    batch = OracleBatch.build(block_size, [s.block_table for s in seqs], starts, lens)
    rows = []
    for s, n in zip(seqs, lens):
        row = list(s.token_ids[s.num_cached_tokens:s.num_cached_tokens + n])
        rows.append(row + [0] * (batch.T - n))  # generate.py:80-82
    ids = np.asarray(rows, dtype=np.int64)
    logits = gpt2_forward(weights, cfg, ids, pool, batch, last_only=True)[:, 0]
    for s, n in zip(seqs, lens):
        s.num_cached_tokens += n
    return logits
