"""GPT-2 with the paged forward on the B200 kernels.

Parameter names and shapes are the reference's (tokquay/model.py:24-35,
:59-134), so a ``state_dict`` moves between the two models unchanged.  The
paged forward (tokquay/model.py:136-181) runs on ragged rows -- only the N
real new tokens of the step, never the reference's padded ``B x T`` -- with:

* the fp32 linears on torch matmul (cuBLAS SGEMM; TF32 must stay off), split
  over K-slices at decode batch sizes (``split_k_for``), with the slices'
  partial sums added by the fused kernel that consumes the linear's output;
* ``tq_embed_layernorm``, ``tq_bias_residual_layernorm``, ``tq_bias_gelu`` and
  ``tq_layernorm_rows`` for everything elementwise around them;
* ``tq_qkv_bias_kv_write`` (c_attn bias, q out, K/V straight into the pool)
  + ``tq_paged_attention`` for the attention over the pool.

In the last layer only each sequence's last row is carried past attention
when ``last_only`` is set: the other rows' K/V are already in the pool and
their outputs would be discarded (model.py:179).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from tokquay_b200 import _lib
from tokquay_b200._host import ref_model
from tokquay_b200.kv_cache import DevicePagedBatch

GPT2Config = ref_model.GPT2Config  # the reference's config (tokquay/model.py:24-35)


class Attention(nn.Module):
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        self.c_attn = nn.Linear(cfg.n_embd, 3 * cfg.n_embd)
        self.c_proj = nn.Linear(cfg.n_embd, cfg.n_embd)


class MLP(nn.Module):
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        self.c_fc = nn.Linear(cfg.n_embd, 4 * cfg.n_embd)
        self.c_proj = nn.Linear(4 * cfg.n_embd, cfg.n_embd)


class Block(nn.Module):
    def __init__(self, cfg: GPT2Config):
        super().__init__()
        self.ln_1 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_eps)
        self.attn = Attention(cfg)
        self.ln_2 = nn.LayerNorm(cfg.n_embd, eps=cfg.layer_norm_eps)
        self.mlp = MLP(cfg)


def _tf32_off() -> bool:
    return not torch.backends.cuda.matmul.allow_tf32 and torch.get_float32_matmul_precision() == "highest"


def argmax_rows(logits: torch.Tensor, out: torch.Tensor | None = None, d_num_rows: int | None = None,
                max_rows: int | None = None) -> torch.Tensor:
    """Greedy tokens ``logits.argmax(-1)`` (int64) of a ``[rows, V]`` fp32
    tensor in one kernel (``tq_argmax_rows``; ties and NaN as torch picks them).
    ``d_num_rows`` (a device int32 address) limits the rows, for graph capture."""
    if logits.dim() != 2 or logits.dtype != torch.float32 or logits.stride(1) != 1:
        raise ValueError("argmax_rows needs a [rows, V] float32 tensor with unit column stride")
    rows = logits.shape[0] if max_rows is None else max_rows
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=logits.device)
    lib = _lib.load()
    count = d_num_rows
    if count is None:
        count_t = torch.full((1,), rows, dtype=torch.int32, device=logits.device)
        count = count_t.data_ptr()
    _lib.check(lib.tq_argmax_rows(logits.data_ptr(), logits.stride(0), logits.shape[1], out.data_ptr(), count, rows,
                                  torch.cuda.current_stream(logits.device).cuda_stream), "tq_argmax_rows")  # fmt: skip
    return out


def split_k_for(rows: int, k: int, n: int) -> int:
    """How many K-slices an fp32 linear of ``rows x k @ k x n`` is split into.

    At decode batch sizes cuBLAS's fp32 GEMM runs a handful of CTAs down the
    whole K loop; one batched matmul over K-slices fills the GPU and the
    slices' partial sums are added by the fused kernel that consumes the
    output.  Chosen from B200 measurements of torch.mm vs torch.bmm over
    K-slices for GPT-2's linears (rows 8 / 64 / 512) and of whole decode
    steps: finer splits make a matmul alone faster (c_fc and mlp.c_proj at 64
    rows by ~1.3 us with 8 / 32 slices), but the consumers' extra partial-sum
    reads cost more than that in the step."""
    if rows > 128:
        s = 4 if k >= 2048 else 1
    else:
        s = 16 if k >= 2048 else (8 if n <= 1024 else 4)
    while s > 1 and (k % s or k // s < 64):
        s //= 2
    return s


class GPT2(nn.Module):
    def __init__(self, cfg: GPT2Config | None = None):
        super().__init__()
        # Optional measurement hooks: ``attention_timer(layer, start)`` is called
        # right before (start=True) and after (start=False) every attention
        # launch, on the launching stream, so a caller can record CUDA events
        # around it (also inside a graph capture); ``kernel_launches`` counts this
        # package's kernel launches (GEMMs and other torch ops are not counted).
        self.attention_timer = None
        self.kernel_launches = 0
        self.last_h2d_bytes = 0  # plan bytes the last forward's batch copied to the device
        self.graph_runner = None  # set by use_cuda_graphs()
        # Opt-in, not the reference's LM head: greedy-token steps run ln_f, the
        # tied LM head and the argmax as one fp32 CUDA-core kernel
        # (tq_lm_head_argmax) instead of torch's fp32 matmul + tq_argmax_rows,
        # for batches of up to 64 sequences.
        self.fused_lm_head = False
        self._lm_scratch: torch.Tensor | None = None
        self._wt: dict[str, tuple] = {}  # name -> (parameter version, contiguous W^T)
        self.cfg = cfg or GPT2Config()
        self.wte = nn.Embedding(self.cfg.vocab_size, self.cfg.n_embd)
        self.wpe = nn.Embedding(self.cfg.n_positions, self.cfg.n_embd)
        self.h = nn.ModuleList(Block(self.cfg) for _ in range(self.cfg.n_layer))
        self.ln_f = nn.LayerNorm(self.cfg.n_embd, eps=self.cfg.layer_norm_eps)

    def use_cuda_graphs(self, allocator, buckets=None, max_ctx: int | None = None):
        """Replay decode steps over ``allocator``'s pool as captured CUDA graphs
        (``paged_forward`` then uses them for every all-decode batch that fits a
        bucket).  Returns the runner; graphs are captured on first use."""
        from tokquay_b200.graphs import DEFAULT_BUCKETS, DecodeGraphRunner

        self.graph_runner = DecodeGraphRunner(self, allocator, buckets or DEFAULT_BUCKETS, max_ctx)
        allocator.graph_runner = self.graph_runner  # batch_for stages decode steps for it
        return self.graph_runner

    def _weight_t(self, name: str, w: torch.Tensor) -> torch.Tensor:
        """Contiguous ``[in, out]`` copy of a linear weight, rebuilt if the
        parameter was changed in place."""
        hit = self._wt.get(name)
        if hit is None or hit[0] != w._version or hit[1].device != w.device:
            hit = (w._version, w.detach().t().contiguous())
            self._wt[name] = hit
        return hit[1]

    def _wte_t_padded(self) -> tuple[torch.Tensor, int]:
        """``wte`` transposed to ``[C, vstride]`` with zero columns past the
        vocabulary, vstride a whole number of the fused head's column slices;
        rebuilt if the embedding changes."""
        w = self.wte.weight
        hit = self._wt.get("wte_pad")
        if hit is None or hit[0] != w._version or hit[1].device != w.device:
            V, C = w.shape
            slice_ = _lib.LM_HEAD_SLICE
            vstride = -(-V // slice_) * slice_
            wt = torch.zeros(C, vstride, dtype=torch.float32, device=w.device)
            wt[:, :V] = w.detach().t()
            hit = (w._version, wt)
            self._wt["wte_pad"] = hit
        return hit[1], hit[1].shape[1]

    def lm_head_greedy(self, x: torch.Tensor, rows_ptr: int | None, n_rows_ptr: int, max_rows: int,
                       tokens: torch.Tensor, stream: int) -> None:
        """``tokens[r] = argmax((ln_f(x[rows[r]])) @ wte.T)`` for the device's
        row count (``n_rows_ptr``), up to ``max_rows`` <= 64: one kernel, no
        logits tensor (tokquay/model.py:179-181 + tokquay/engine.py:189-194)."""
        lib = _lib.load()
        wt, vstride = self._wte_t_padded()
        if self._lm_scratch is None or self._lm_scratch.device != x.device:
            self._lm_scratch = torch.zeros(_lib.LM_HEAD_SCRATCH_BYTES, dtype=torch.uint8, device=x.device)
        cfg = self.cfg
        _lib.check(lib.tq_lm_head_argmax(
            tokens.data_ptr(), None, x.data_ptr(), x.stride(0), rows_ptr, self.ln_f.weight.data_ptr(),
            self.ln_f.bias.data_ptr(), cfg.layer_norm_eps, cfg.n_embd, wt.data_ptr(), vstride, cfg.vocab_size,
            self._lm_scratch.data_ptr(), n_rows_ptr, max_rows, stream), "tq_lm_head_argmax")  # fmt: skip

    @staticmethod
    def _linear_parts(x: torch.Tensor, wt: torch.Tensor) -> tuple[torch.Tensor, int, int]:
        """``x @ wt`` as ``n_parts`` split-K partial sums laid out ``part_stride``
        floats apart (torch fp32 matmul; TF32 stays off)."""
        rows, k = x.shape
        n = wt.shape[1]
        s = split_k_for(rows, k, n)
        if s == 1:
            return torch.mm(x, wt), 1, 0
        parts = torch.bmm(x.view(rows, s, k // s).transpose(0, 1), wt.view(s, k // s, n))  # [s, rows, n]
        return parts, s, rows * n

    # ---- reference-shaped entry point --------------------------------------------------
    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, cache: DevicePagedBatch, last_only: bool = False) -> torch.Tensor:
        """``input_ids [B, T]`` (right-padded, as the reference takes them) ->
        logits ``[B, T, V]`` (or ``[B, 1, V]`` with ``last_only``), the call the
        reference's ``paged_forward`` makes (tokquay/generate.py:84).  Logits of
        padded slots are zero.  Only the paged path exists in this package:
        ``cache`` is the step view ``BlockAllocator.batch_for`` returned (a
        ``DevicePagedBatch``, or a decode step staged into a CUDA graph)."""
        from tokquay_b200.graphs import GraphStepBatch

        graph_step = isinstance(cache, GraphStepBatch)
        if not (graph_step or isinstance(cache, DevicePagedBatch)):
            raise TypeError("this model runs the paged forward only: pass the step view of "
                            "tokquay_b200.BlockAllocator.batch_for")
        B, T = input_ids.shape
        if (B, T) != (cache.B, cache.T):
            raise ValueError(f"input_ids {tuple(input_ids.shape)} does not match batch {(cache.B, cache.T)}")
        if graph_step:
            if cache.runner.model is not self:
                raise ValueError("the step was staged for another model's CUDA graphs")
            return cache.replay(input_ids)
        b, t = cache._valid_bt()
        ids = input_ids.to(cache.pool.device)[b, t].to(torch.int32).contiguous()
        return self.forward_paged(cache, last_only=last_only, ids=ids)

    # ---- hot path ------------------------------------------------------------------------
    @torch.no_grad()
    def forward_paged(self, batch: DevicePagedBatch, last_only: bool = True,
                      ids: torch.Tensor | None = None, greedy_out: torch.Tensor | None = None) -> torch.Tensor | None:  # fmt: skip
        """Paged forward over the batch's ragged rows.  ``ids`` (int32 ``[N]``
        on the device) defaults to the token ids the batch was planned with.
        Returns ``[B, 1, V]`` (``last_only``) or ``[B, T, V]``.  With
        ``greedy_out`` (int64 ``[B]``), ``fused_lm_head`` on and at most 64
        sequences, the greedy tokens go there instead and None is returned."""
        cfg = self.cfg
        if batch.max_ctx > cfg.n_positions:  # tokquay/model.py:159-160
            raise ValueError(f"sequence length {batch.max_ctx} exceeds n_positions={cfg.n_positions}")
        if not _tf32_off():
            raise RuntimeError("TF32 matmul is enabled; the fp32 paged forward needs it off "
                               "(torch.backends.cuda.matmul.allow_tf32 = False, precision 'highest')")
        if ids is None:
            ids = batch.token_ids
            if ids is None:
                raise ValueError("the batch carries no token ids; pass ids")
        lib = _lib.load()
        dev = batch.pool.device
        stream = torch.cuda.current_stream(dev).cuda_stream
        self.last_h2d_bytes = batch.h2d_bytes
        # Activations and launches are sized for rows_alloc / seqs_alloc: the
        # step's own N and B, or a workspace's capacities when the step is being
        # captured as a CUDA graph (the kernels read the true counts on the device).
        C, eps, N, B = cfg.n_embd, cfg.layer_norm_eps, batch.rows_alloc, batch.seqs_alloc
        if not last_only and (N, B) != (batch.N, batch.B):
            raise ValueError("all-position logits need a batch sized to its own rows")
        n_ptr, b_ptr = batch.count_ptr(0), batch.count_ptr(3)
        x = torch.empty(N, C, dtype=torch.float32, device=dev)
        xa = torch.empty(N, C, dtype=torch.float32, device=dev)
        h0 = self.h[0].ln_1
        _lib.check(lib.tq_embed_layernorm(
            x.data_ptr(), xa.data_ptr(), ids.data_ptr(), batch.row_positions.data_ptr(),
            self.wte.weight.data_ptr(), self.wpe.weight.data_ptr(), cfg.vocab_size, cfg.n_positions,
            h0.weight.data_ptr(), h0.bias.data_ptr(), eps, C, n_ptr, N, stream), "tq_embed_layernorm")  # fmt: skip

        rows, rows_ptr = N, n_ptr
        for i, blk in enumerate(self.h):
            last = i == cfg.n_layer - 1
            att = blk.attn
            p = f"h.{i}."
            parts, ns, ps = self._linear_parts(xa, self._weight_t(p + "c_attn", att.c_attn.weight))
            q = torch.empty(N, C, dtype=torch.float32, device=dev)
            batch.write_qkv_rows(i, parts, ns, ps, att.c_attn.bias, q, stream)  # q out, K/V into the pool
            a = torch.empty(N, C, dtype=torch.float32, device=dev)
            if self.attention_timer is not None:
                self.attention_timer(i, True)
                batch.attend_rows(i, q, a, stream)
                self.attention_timer(i, False)
            else:
                batch.attend_rows(i, q, a, stream)
            if last and last_only and N != B:
                # Only the last row of each sequence is sampled from (model.py:179).
                sel = batch.last_rows
                a, x = a.index_select(0, sel), x.index_select(0, sel)
                xa = torch.empty(B, C, dtype=torch.float32, device=dev)
                rows, rows_ptr = B, b_ptr
            y, ns, ps = self._linear_parts(a, self._weight_t(p + "c_proj", att.c_proj.weight))
            _lib.check(lib.tq_bias_residual_layernorm(
                x.data_ptr(), xa.data_ptr(), y.data_ptr(), ns, ps, att.c_proj.bias.data_ptr(),
                blk.ln_2.weight.data_ptr(), blk.ln_2.bias.data_ptr(), eps, C, rows_ptr, rows, stream),
                "tq_bias_residual_layernorm")  # fmt: skip
            parts, ns, ps = self._linear_parts(xa, self._weight_t(p + "c_fc", blk.mlp.c_fc.weight))
            hid = parts if ns == 1 else torch.empty(rows, 4 * C, dtype=torch.float32, device=dev)
            _lib.check(lib.tq_bias_gelu(hid.data_ptr(), parts.data_ptr(), ns, ps, blk.mlp.c_fc.bias.data_ptr(),
                                        4 * C, 1, rows_ptr, rows, stream), "tq_bias_gelu")  # fmt: skip
            y, ns, ps = self._linear_parts(hid, self._weight_t(p + "mlp.c_proj", blk.mlp.c_proj.weight))
            nxt = None if last else self.h[i + 1].ln_1
            _lib.check(lib.tq_bias_residual_layernorm(
                x.data_ptr(), xa.data_ptr(), y.data_ptr(), ns, ps, blk.mlp.c_proj.bias.data_ptr(),
                nxt.weight.data_ptr() if nxt is not None else None,
                nxt.bias.data_ptr() if nxt is not None else None, eps, C, rows_ptr, rows, stream),
                "tq_bias_residual_layernorm")  # fmt: skip

        # embed + per layer (qkv bias + kv write, attention, 2x bias_residual, gelu) + final LN
        self.kernel_launches += 2 + cfg.n_layer * 5
        if last_only and greedy_out is not None and self.fused_lm_head and B <= _lib.LM_HEAD_MAX_ROWS:
            sel_ptr = None if rows == B else batch.last_rows.data_ptr()
            self.lm_head_greedy(x, sel_ptr, b_ptr, B, greedy_out, stream)  # in place of the final LN's count
            return None
        if last_only:
            xf = torch.empty(B, C, dtype=torch.float32, device=dev)
            sel_ptr = None if rows == B else batch.last_rows.data_ptr()
            _lib.check(lib.tq_layernorm_rows(xf.data_ptr(), x.data_ptr(), sel_ptr, self.ln_f.weight.data_ptr(),
                                             self.ln_f.bias.data_ptr(), eps, C, b_ptr, B, stream),
                       "tq_layernorm_rows")  # fmt: skip
            return torch.mm(xf, self._weight_t("wte", self.wte.weight)).unsqueeze(1)  # tied LM head, model.py:181
        xf = torch.empty(N, C, dtype=torch.float32, device=dev)
        _lib.check(lib.tq_layernorm_rows(xf.data_ptr(), x.data_ptr(), None, self.ln_f.weight.data_ptr(),
                                         self.ln_f.bias.data_ptr(), eps, C, n_ptr, N, stream),
                   "tq_layernorm_rows")  # fmt: skip
        logits = torch.mm(xf, self._weight_t("wte", self.wte.weight))
        out = torch.zeros(B, batch.T, cfg.vocab_size, dtype=torch.float32, device=dev)
        b, t = batch._valid_bt()
        out[b, t] = logits
        return out
