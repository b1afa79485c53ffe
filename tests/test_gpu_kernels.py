"""Kernel-level parity on the GPU, through the C ABI.

* KV write: bit-exact against a torch scatter of the same rows.
* Paged attention (decode and causal prefill rows mixed, split-K or not):
  against a float64 torch reference of softmax(q k^T / sqrt(d)) v over each
  row's keys 0..position, on a pool whose unused slots hold NaN -- so any
  read of a slot outside a sequence's causal range poisons the result.
* Fused LayerNorm / bias / GELU / residual: against torch fp32 ops.
"""

import math
import random

import numpy as np
import pytest
import torch

from tokquay_b200 import _lib
from tokquay_b200.kv_cache import BlockAllocator, DevicePagedBatch, attention_warps, cdiv
from tokquay_b200.model import GPT2Config

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

ATTN_RTOL = 2e-5  # fp32 online softmax vs a float64 reference, relative to max |out|


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _mixed_batch(rng, alloc, n_seqs, max_ctx, prefill_frac):
    """Random sequences: some decode one token after a cached context, some
    prefill a chunk starting at an arbitrary cached position."""
    bs = alloc.block_size
    tables, start, new = [], [], []
    for _ in range(n_seqs):
        if rng.random() < prefill_frac:
            n = rng.randint(2, 70)
            s = rng.randint(0, max(0, max_ctx - n))
        else:
            n = 1
            s = rng.randint(0, max_ctx - 1)
        tables.append(alloc._take(cdiv(s + n, bs)))
        start.append(s)
        new.append(n)
    return tables, start, new


def _reference_attention(pool, layer, q, tables, start, new, bs):
    """float64 per-row softmax attention over keys 0..position (the semantics
    of tokquay/model.py:94-96 with the mask of tokquay/kv_cache.py:213-214)."""
    H, d = pool.shape[3], pool.shape[5]
    out = torch.empty(q.shape[0], H * d, dtype=torch.float64, device=q.device)
    row = 0
    for tbl, s, n in zip(tables, start, new):
        ctx = s + n
        idx = torch.tensor(tbl[:cdiv(ctx, bs)], device=q.device)
        k = pool[idx, layer, 0].permute(1, 0, 2, 3).reshape(H, -1, d)[:, :ctx].double()
        v = pool[idx, layer, 1].permute(1, 0, 2, 3).reshape(H, -1, d)[:, :ctx].double()
        qq = q[row:row + n].view(n, H, d).transpose(0, 1).double()  # [H, n, d]
        sc = qq @ k.transpose(1, 2) / math.sqrt(d)
        pos = torch.arange(s, s + n, device=q.device)[:, None]
        sc = sc.masked_fill(torch.arange(ctx, device=q.device)[None, :] > pos, float("-inf"))
        out[row:row + n] = (torch.softmax(sc, -1) @ v).transpose(0, 1).reshape(n, H * d)
        row += n
    return out


@pytest.mark.parametrize("bs", [1, 4, 16, 32, 64, 256])
@pytest.mark.parametrize("kind", ["decode", "mixed", "prefill"])
@pytest.mark.parametrize("seed", [0, 1])
def test_paged_attention_matches_float64_reference(bs, kind, seed):
    rng = random.Random(seed * 100 + bs)
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=256, n_layer=2, n_head=4)
    max_ctx = 700
    n_seqs = {"decode": 37, "mixed": 21, "prefill": 6}[kind]
    frac = {"decode": 0.0, "mixed": 0.3, "prefill": 1.0}[kind]
    num_blocks = n_seqs * cdiv(max_ctx + 2, bs) + 8
    alloc = BlockAllocator(cfg, num_blocks, bs, device="cuda")
    random.Random(seed).shuffle(alloc._free)
    g = torch.Generator(device="cuda").manual_seed(seed)
    alloc.pool.normal_(generator=g)
    tables, start, new = _mixed_batch(rng, alloc, n_seqs, max_ctx, frac)
    # Poison every slot at or beyond each sequence's context: masked keys must never be read.
    for tbl, s, n in zip(tables, start, new):
        ctx = s + n
        for j, blk in enumerate(tbl):
            lo = max(0, ctx - j * bs)
            if lo < bs:
                alloc.pool[blk, :, :, :, lo:] = float("nan")
    for blk in alloc._free:
        alloc.pool[blk] = float("nan")
    batch = DevicePagedBatch(alloc, tables, start, new)
    C = cfg.n_embd
    layer = 1
    # q rows live inside a wider [N, 3C] buffer, as the c_attn output does.
    qkv = torch.randn(batch.N, 3 * C, device="cuda", generator=g)
    out = torch.full((batch.N, C), float("nan"), device="cuda")
    batch.attend_rows(layer, qkv, out, _stream())
    torch.cuda.synchronize()
    want = _reference_attention(alloc.pool, layer, qkv[:, :C], tables, start, new, bs)
    assert torch.isfinite(out).all()
    err = (out.double() - want).abs().max().item()
    assert err <= ATTN_RTOL * want.abs().max().item(), (err, batch.split_chunks, batch.num_combine)
    assert _lib.device_status() == 0


def test_paged_attention_config4_full_size():
    """BASELINE config 4 at its full shape -- 512 decoding sequences, contexts
    U[256, 1024], block size 32, GPT-2 124M's 12 layers x 12 heads -- on a pool
    sized to the batch (~25 GB, every other slot NaN), one launch per tested
    layer on the grid the bench uses; every row of every head against the
    float64 reference."""
    rng = random.Random(4)
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=12, n_head=12)
    bs, n_seqs = 32, 512
    ctx = [rng.randint(256, 1024) for _ in range(n_seqs)]
    alloc = BlockAllocator(cfg, sum(cdiv(c, bs) for c in ctx) + 16, bs, device="cuda")
    random.Random(5).shuffle(alloc._free)
    g = torch.Generator(device="cuda").manual_seed(4)
    alloc.pool.normal_(generator=g)
    tables = [alloc._take(cdiv(c, bs)) for c in ctx]
    start, new = [c - 1 for c in ctx], [1] * n_seqs
    for tbl, c in zip(tables, ctx):  # slots past each context
        if c % bs:
            alloc.pool[tbl[-1], :, :, :, c % bs:] = float("nan")
    if alloc._free:
        alloc.pool[torch.tensor(alloc._free, device="cuda")] = float("nan")
    batch = DevicePagedBatch(alloc, tables, start, new)
    C = cfg.n_embd
    try:
        for layer in (0, 11):
            q = torch.randn(n_seqs, C, device="cuda", generator=g)
            out = torch.full((n_seqs, C), float("nan"), device="cuda")
            batch.attend_rows(layer, q, out, _stream())
            torch.cuda.synchronize()
            assert torch.isfinite(out).all(), layer
            worst, scale = 0.0, 0.0
            for b0 in range(0, n_seqs, 64):  # the reference in slices of 64 sequences
                sl = slice(b0, b0 + 64)
                want = _reference_attention(alloc.pool, layer, q[sl], tables[sl], start[sl], new[sl], bs)
                worst = max(worst, (out[sl].double() - want).abs().max().item())
                scale = max(scale, want.abs().max().item())
            assert worst <= ATTN_RTOL * scale, (layer, worst, scale)
        assert _lib.device_status() == 0
    finally:
        del batch, alloc
        torch.cuda.empty_cache()


def test_paged_attention_split_k_is_exercised():
    """Few long decodes force split-K + combine; compare with the unsplit run."""
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=1, n_head=12)
    alloc = BlockAllocator(cfg, 8 * 64 + 4, 16, device="cuda")
    alloc.pool.normal_()
    tables = [alloc._take(64) for _ in range(8)]
    start, new = [1000 + i for i in range(8)], [1] * 8
    batch = DevicePagedBatch(alloc, tables, start, new)
    assert batch.num_combine == 8 and batch.split_chunks >= 2
    qkv = torch.randn(8, 3 * 768, device="cuda")
    out = torch.empty(8, 768, device="cuda")
    batch.attend_rows(0, qkv, out, _stream())
    want = _reference_attention(alloc.pool, 0, qkv[:, :768], tables, start, new, 16)
    assert (out.double() - want).abs().max().item() <= ATTN_RTOL * want.abs().max().item()


def _merge_kinds(batch) -> set[int]:
    """Merge flags of the plan's work items: 0 whole, 1 cut inside a CTA, 2
    split across CTAs, 3 both (the decode bit, 4, is left out)."""
    L = batch.layout
    plan = batch.plan.cpu().numpy()
    nw = batch.n_ctas * attention_warps()
    o = int(L[_lib.PLAN_OFF_ITEMS])
    first = plan[o:o + 16 * nw].reshape(nw, 16)[:, :8]  # first items: 8 words + 8 block ids
    offs = plan[o + 16 * nw:o + 17 * nw + 1]
    ro = o + 16 * nw + (nw + 8) // 8 * 8
    rest = plan[ro:ro + 8 * int(offs[-1])].reshape(-1, 8)
    words = [w[2] for w in first if w[4] != 0] + [w[2] for w in rest]
    return {(int(np.uint32(x)) >> 24) & 3 for x in words}


@pytest.mark.parametrize("n_ctas", [1, 5, 37, 148, 400])
def test_paged_attention_any_grid(n_ctas):
    """Whatever the grid, the cuts -- merged in shared memory inside a CTA,
    through split-K scratch across CTAs, or both -- give the float64 result."""
    rng = random.Random(n_ctas)
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=1, n_head=12)
    alloc = BlockAllocator(cfg, 40 * 64 + 8, 16, device="cuda")
    random.Random(1).shuffle(alloc._free)
    alloc.pool.normal_()
    tables, start, new = [], [], []
    for i in range(40):
        s = rng.choice([rng.randint(0, 60), rng.randint(300, 1000)])
        n = rng.choice([1, 1, 1, 7])
        tables.append(alloc._take(cdiv(s + n, 16)))
        start.append(s)
        new.append(n)
    batch = DevicePagedBatch(alloc, tables, start, new, n_ctas=n_ctas)
    kinds = _merge_kinds(batch)
    if n_ctas >= 37:
        assert 1 in kinds or 3 in kinds  # some pair is cut between warps of a CTA
    qkv = torch.randn(batch.N, 3 * 768, device="cuda")
    out = torch.full((batch.N, 768), float("nan"), device="cuda")
    batch.attend_rows(0, qkv, out, _stream())
    torch.cuda.synchronize()
    want = _reference_attention(alloc.pool, 0, qkv[:, :768], tables, start, new, 16)
    assert torch.isfinite(out).all()
    assert (out.double() - want).abs().max().item() <= ATTN_RTOL * want.abs().max().item(), kinds
    assert _lib.device_status() == 0


@pytest.mark.parametrize("bs", [1, 4, 16, 32, 128])
def test_kv_write_is_bit_exact(bs):
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=3, n_head=12)
    rng = random.Random(bs)
    alloc = BlockAllocator(cfg, 200, bs, device="cuda")
    random.Random(3).shuffle(alloc._free)
    alloc.pool.normal_()
    before = alloc.pool.clone()
    tables, start, new = [], [], []
    for _ in range(9):
        s, n = rng.randint(0, 300), rng.choice([1, 1, 17, 40])
        if cdiv(s + n, bs) > alloc.num_free_blocks:
            break
        tables.append(alloc._take(cdiv(s + n, bs)))
        start.append(s)
        new.append(n)
    batch = DevicePagedBatch(alloc, tables, start, new)
    qkv = torch.randn(batch.N, 3 * 768, device="cuda")
    layer = 2
    batch.write_rows(layer, qkv, 768, 1536, _stream())
    torch.cuda.synchronize()
    want = before.clone()
    row = 0
    for tbl, s, n in zip(tables, start, new):
        for t in range(n):
            p = s + t
            blk, off = tbl[p // bs], p % bs
            want[blk, layer, 0, :, off] = qkv[row, 768:1536].view(12, 64)
            want[blk, layer, 1, :, off] = qkv[row, 1536:].view(12, 64)
            row += 1
    assert torch.equal(alloc.pool, want)


@pytest.mark.parametrize("n_parts", [1, 3, 4])
@pytest.mark.parametrize("bs", [4, 16, 32])
def test_qkv_bias_kv_write_matches_the_unfused_path(n_parts, bs):
    """c_attn epilogue fused with the KV write == bias_gelu (no GELU) + kv_write,
    bit for bit: same q rows, same pool, nothing else in the pool touched."""
    lib = _lib.load()
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=3, n_head=12)
    rng = random.Random(bs * 10 + n_parts)
    alloc = BlockAllocator(cfg, 120, bs, device="cuda")
    random.Random(5).shuffle(alloc._free)
    alloc.pool.normal_()
    tables, start, new = [], [], []
    for _ in range(7):
        s, n = rng.randint(0, 200), rng.choice([1, 1, 9])
        if cdiv(s + n, bs) > alloc.num_free_blocks:
            break
        tables.append(alloc._take(cdiv(s + n, bs)))
        start.append(s)
        new.append(n)
    batch = DevicePagedBatch(alloc, tables, start, new)
    N, C = batch.N, 768
    g = torch.Generator(device="cuda").manual_seed(bs)
    parts = torch.randn(n_parts, N, 3 * C, device="cuda", generator=g)
    bias = torch.randn(3 * C, device="cuda", generator=g)
    st = _stream()
    # unfused: sum + bias into qkv, then scatter K/V
    pool0 = alloc.pool.clone()
    qkv = torch.empty(N, 3 * C, device="cuda")
    _lib.check(lib.tq_bias_gelu(qkv.data_ptr(), parts.data_ptr(), n_parts, N * 3 * C, bias.data_ptr(), 3 * C, 0,
                                batch.count_ptr(0), N, st), "tq_bias_gelu")  # fmt: skip
    batch.write_rows(2, qkv, C, 2 * C, st)
    want_pool = alloc.pool.clone()
    alloc.pool.copy_(pool0)
    q = torch.full((N, C), float("nan"), device="cuda")
    batch.write_qkv_rows(2, parts, n_parts, N * 3 * C, bias, q, st)
    torch.cuda.synchronize()
    assert torch.equal(q, qkv[:, :C])
    assert torch.equal(alloc.pool, want_pool)
    assert _lib.device_status() == 0


def _ln(x, w, b, eps):
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w, b, eps)


@pytest.mark.parametrize("C", [128, 768, 1024])
def test_fused_row_kernels_match_torch(C):
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(C)
    N, V, P, eps = 37, 500, 64, 1e-5
    dev = "cuda"
    r = lambda *s: torch.randn(*s, device=dev, generator=g)  # noqa: E731
    wte, wpe, w, b = r(V, C), r(P, C), r(C), r(C)
    ids = torch.randint(0, V, (N,), device=dev, dtype=torch.int32, generator=g)
    pos = torch.randint(0, P, (N,), device=dev, dtype=torch.int32, generator=g)
    n_dev = torch.tensor([N, 0, 0, 0], dtype=torch.int32, device=dev)
    x, xa = torch.empty(N, C, device=dev), torch.empty(N, C, device=dev)
    s = _stream()
    _lib.check(lib.tq_embed_layernorm(x.data_ptr(), xa.data_ptr(), ids.data_ptr(), pos.data_ptr(), wte.data_ptr(),
                                      wpe.data_ptr(), V, P, w.data_ptr(), b.data_ptr(), eps, C, n_dev.data_ptr(), N,
                                      s), "embed")  # fmt: skip
    x_ref = wte[ids.long()] + wpe[pos.long()]
    torch.testing.assert_close(x, x_ref, rtol=0, atol=0)
    torch.testing.assert_close(xa, _ln(x_ref, w, b, eps), rtol=1e-5, atol=1e-5)

    y, bias = r(N, C), r(C)
    x0 = x.clone()
    _lib.check(lib.tq_bias_residual_layernorm(x.data_ptr(), xa.data_ptr(), y.data_ptr(), 1, 0, bias.data_ptr(),
                                              w.data_ptr(), b.data_ptr(), eps, C, n_dev.data_ptr(), N, s),
               "bias_residual_ln")  # fmt: skip
    x1 = x0 + (y + bias)
    torch.testing.assert_close(x, x1, rtol=0, atol=0)
    torch.testing.assert_close(xa, _ln(x1, w, b, eps), rtol=1e-5, atol=1e-5)
    xa_before = xa.clone()
    _lib.check(lib.tq_bias_residual_layernorm(x.data_ptr(), None, y.data_ptr(), 1, 0, bias.data_ptr(), None, None,
                                              eps, C, n_dev.data_ptr(), N, s), "bias_residual")  # fmt: skip
    torch.testing.assert_close(x, x1 + (y + bias), rtol=0, atol=0)
    assert torch.equal(xa, xa_before)
    # split-K partial sums of the linear output: x += (y_0 + y_1 + y_2) + bias
    parts = r(3, N, C)
    x2 = x.clone()
    _lib.check(lib.tq_bias_residual_layernorm(x.data_ptr(), xa.data_ptr(), parts.data_ptr(), 3, N * C,
                                              bias.data_ptr(), w.data_ptr(), b.data_ptr(), eps, C, n_dev.data_ptr(),
                                              N, s), "bias_residual_ln parts")  # fmt: skip
    x3 = x2 + (((parts[0] + parts[1]) + parts[2]) + bias)
    torch.testing.assert_close(x, x3, rtol=0, atol=0)
    torch.testing.assert_close(xa, _ln(x3, w, b, eps), rtol=1e-5, atol=1e-5)

    rows = torch.tensor([5, 0, 36, 17], dtype=torch.int32, device=dev)
    out = torch.empty(4, C, device=dev)
    n4 = torch.tensor([4], dtype=torch.int32, device=dev)
    _lib.check(lib.tq_layernorm_rows(out.data_ptr(), x.data_ptr(), rows.data_ptr(), w.data_ptr(), b.data_ptr(), eps, C,
                                     n4.data_ptr(), 4, s), "layernorm_rows")  # fmt: skip
    torch.testing.assert_close(out, _ln(x[rows.long()], w, b, eps), rtol=1e-5, atol=1e-5)


def test_bias_gelu_matches_torch():
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    h = torch.randn(53, 3072, device="cuda", generator=g) * 3
    bias = torch.randn(3072, device="cuda", generator=g)
    want = torch.nn.functional.gelu(h + bias, approximate="tanh")
    n = torch.tensor([53], dtype=torch.int32, device="cuda")
    _lib.check(lib.tq_bias_gelu(h.data_ptr(), h.data_ptr(), 1, 0, bias.data_ptr(), 3072, 1, n.data_ptr(), 53,
                                _stream()), "gelu")  # fmt: skip
    torch.testing.assert_close(h, want, rtol=1e-5, atol=1e-6)
    # split-K partial sums into a separate output, with and without the GELU
    parts = torch.randn(4, 53, 3072, device="cuda", generator=g)
    total = ((parts[0] + parts[1]) + parts[2]) + parts[3]
    out = torch.empty(53, 3072, device="cuda")
    for act, ref in ((1, torch.nn.functional.gelu(total + bias, approximate="tanh")), (0, total + bias)):
        _lib.check(lib.tq_bias_gelu(out.data_ptr(), parts.data_ptr(), 4, 53 * 3072, bias.data_ptr(), 3072, act,
                                    n.data_ptr(), 53, _stream()), "gelu parts")  # fmt: skip
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)


def test_abi_rejects_bad_arguments():
    """Validation happens on the host and returns a status; nothing launches."""
    lib = _lib.load()
    pool = torch.zeros(4, 1, 2, 1, 16, 64, device="cuda")
    n = torch.tensor([1], dtype=torch.int32, device="cuda")
    st = lib.tq_kv_write(pool.data_ptr(), 4, 1, 1, 16, 32, 0, pool.data_ptr(), 192, 64, 128, n.data_ptr(),
                         n.data_ptr(), 1, None)  # head_dim 32: unsupported
    assert st == _lib.TQ_ERR_UNSUPPORTED and "head_dim" in _lib.last_error()
    st = lib.tq_kv_write(pool.data_ptr() + 4, 4, 1, 1, 16, 64, 0, pool.data_ptr(), 192, 64, 128, n.data_ptr(),
                         n.data_ptr(), 1, None)  # misaligned pool
    assert st == _lib.TQ_ERR_INVALID
    st = lib.tq_bias_gelu(pool.data_ptr(), pool.data_ptr(), 1, 0, pool.data_ptr(), 6, 1, n.data_ptr(), 1, None)
    assert st == _lib.TQ_ERR_INVALID
    assert _lib.device_status() == 0


@pytest.mark.parametrize("V", [1, 3, 31, 1024, 8193, 50257])
def test_argmax_rows_matches_torch(V):
    """tq_argmax_rows picks what torch.argmax(-1) picks: first of equal maxima,
    NaN as the largest value, all -inf rows at index 0."""
    from tokquay_b200.model import argmax_rows

    g = torch.Generator(device="cuda").manual_seed(V)
    x = torch.randn(37, V, device="cuda", generator=g)
    if V > 10:
        x[3, V // 3] = x[3, V // 2] = 1e9  # a tie: the first index wins
        x[5, 7] = float("nan")
        x[5, 9] = float("nan")
        x[8, 4] = float("inf")
    x[6] = float("-inf")
    x[7] = 2.0
    got = argmax_rows(x)
    assert torch.equal(got, x.argmax(-1))
    # a view with a row stride larger than V, rows limited by a device count
    wide = torch.randn(20, V + 5, device="cuda", generator=g)
    out = torch.full((20,), -1, dtype=torch.int64, device="cuda")
    n = torch.tensor([13], dtype=torch.int32, device="cuda")
    argmax_rows(wide[:, :V], out=out, d_num_rows=n.data_ptr(), max_rows=20)
    assert torch.equal(out[:13], wide[:13, :V].argmax(-1)) and (out[13:] == -1).all()


def _item_flags(batch) -> list[int]:
    """Flag byte of every work item of the batch's plan (first items included)."""
    L = batch.layout
    plan = batch.plan.cpu().numpy()
    nw = batch.n_ctas * attention_warps()
    o = int(L[_lib.PLAN_OFF_ITEMS])
    first = plan[o:o + 16 * nw].reshape(nw, 16)[:, :8]
    offs = plan[o + 16 * nw:o + 17 * nw + 1]
    ro = o + 16 * nw + (nw + 8) // 8 * 8
    rest = plan[ro:ro + 8 * int(offs[-1])].reshape(-1, 8)
    words = [w[2] for w in first if w[4] != 0] + [w[2] for w in rest]
    return [(int(np.uint32(x)) >> 24) for x in words]


@pytest.fixture
def tile_knobs():
    prev = _lib.prompt_tiles()
    yield _lib.prompt_tiles
    _lib.prompt_tiles(prev, 1500, 200, 1)


@pytest.mark.parametrize("bs", [4, 16, 64])
@pytest.mark.parametrize("shape", ["prefill_split", "beside_decode", "decode_split", "tiles_off"])
def test_prompt_tiles_match_float64_reference(bs, shape, tile_knobs):
    """Long prompt chunks (cached prefixes of 0-600 keys, 100-256 rows) on the
    tensor-core tiles: prompt rows alone (long tiles cut into pieces whose
    partials the merge kernel combines after the grid), the same beside a
    decode row (whole tiles, and cut into pieces), and with tiles off (2-row
    warp items) -- every row against float64, NaN in every slot past each
    context."""
    pieces = {"prefill_split": 8, "decode_split": 4}.get(shape, 1)
    tile_knobs(0 if shape == "tiles_off" else 16, 1500, 200, pieces)
    rng = random.Random(bs)
    cfg = GPT2Config(vocab_size=64, n_positions=1024, n_embd=768, n_layer=1, n_head=12)
    alloc = BlockAllocator(cfg, 4 * cdiv(1024, bs) + 8, bs, device="cuda")
    random.Random(2).shuffle(alloc._free)
    g = torch.Generator(device="cuda").manual_seed(bs)
    alloc.pool.normal_(generator=g)
    tables, start, new = [], [], []
    for s, n in ((0, 256), (rng.randint(100, 600), rng.randint(100, 200)), (rng.randint(0, 300), 128)):
        tables.append(alloc._take(cdiv(s + n, bs)))
        start.append(s)
        new.append(n)
    if shape in ("beside_decode", "decode_split"):
        c = rng.randint(100, 700)
        tables.append(alloc._take(cdiv(c, bs)))
        start.append(c - 1)
        new.append(1)
    for tbl, s, n in zip(tables, start, new):
        ctx = s + n
        for j, blk in enumerate(tbl):
            lo = max(0, ctx - j * bs)
            if lo < bs:
                alloc.pool[blk, :, :, :, lo:] = float("nan")
    if alloc._free:
        alloc.pool[torch.tensor(alloc._free, device="cuda")] = float("nan")
    batch = DevicePagedBatch(alloc, tables, start, new)
    flags = _item_flags(batch)
    n_tile = sum(f & 8 != 0 for f in flags)
    n_split = sum(f & 8 != 0 and f & 2 != 0 for f in flags)
    if shape == "tiles_off":
        assert n_tile == 0
    elif shape == "beside_decode":
        assert n_tile > 0 and n_split == 0 and batch.tile_merges == 0
    else:
        assert n_split > 0 and batch.tile_merges > 0
    C = cfg.n_embd
    qkv = torch.randn(batch.N, 3 * C, device="cuda", generator=g)
    out = torch.full((batch.N, C), float("nan"), device="cuda")
    for _ in range(2):  # twice: the scratch (counters at zero) serves the next launch
        batch.attend_rows(0, qkv, out, _stream())
        torch.cuda.synchronize()
        want = _reference_attention(alloc.pool, 0, qkv[:, :C], tables, start, new, bs)
        assert torch.isfinite(out).all()
        err = (out.double() - want).abs().max().item()
        assert err <= ATTN_RTOL * want.abs().max().item(), (shape, err)
    assert _lib.device_status() == 0
