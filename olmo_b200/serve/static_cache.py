"""
Fixed-shape decoding state for the generation engine: preallocated key/value windows, one decode step whose tensor
shapes never change, and (on a GPU) one CUDA graph per attention length bucket.

Why.  Decoding through ``OLMo.forward`` with concatenated caches changes a shape every step; every new length pays
for fresh library heuristics and allocator traffic, and a step is a few hundred small launches.  Here a step always
sees ``[rows, 1]`` tokens, ``[rows, kv_heads, window, head_dim]`` caches and a ``[rows, 1, 1, window]`` additive bias;
what changes between steps is *content* (the write column, the per-row rotary index, the bias), held in device tensors
the captured graph reads.  Attention reads the first ``length`` columns only, ``length`` rounded up to a bucket, so a
short batch does not pay for the whole window.

Layout.  Row ``r`` of the window belongs to one request (or is idle).  All rows write their new token at the same
column ``cur``; a row's earlier tokens sit directly to the left of ``cur`` and everything else in the row is masked.
Keys are stored already rotated by their token's index in its own sequence, so moving rows sideways (to make room for
a longer prompt, or to reclaim the left part of the window) needs no arithmetic on the values.
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..models.blocks import StaticKV

__all__ = ["StaticWindow", "supports_static_window"]


def supports_static_window(config) -> bool:
    """Rotary models with ungrouped blocks (every released OLMo architecture)."""
    return bool(config.rope) and not config.alibi and config.block_group_size == 1


class StaticWindow:
    def __init__(self, model, rows: int, window: Optional[int] = None, bucket: int = 128, cuda_graphs: Optional[bool] = None,
                 fused: Optional[bool] = None):
        cfg = model.config
        assert supports_static_window(cfg)
        self.model, self.config = model, cfg
        param = next(model.parameters())
        self.device, self.dtype = param.device, (param.dtype if param.dtype.is_floating_point else torch.bfloat16)
        self.rows = rows
        self.window = min(window or cfg.max_sequence_length, cfg.max_sequence_length)
        self.bucket = max(1, min(bucket, self.window))
        self.cuda_graphs = (self.device.type == "cuda") if cuda_graphs is None else (cuda_graphs and self.device.type == "cuda")
        hd, n_kv, n_layers = cfg.d_model // cfg.n_heads, cfg.effective_n_kv_heads, cfg.n_layers
        shape = (rows, n_kv, self.window, hd)
        self.k = [torch.zeros(shape, dtype=self.dtype, device=self.device) for _ in range(n_layers)]
        self.v = [torch.zeros(shape, dtype=self.dtype, device=self.device) for _ in range(n_layers)]
        self.floor = torch.finfo(self.dtype).min
        self.bias = torch.full((rows, 1, 1, self.window), self.floor, dtype=self.dtype, device=self.device)
        self.tokens = torch.zeros(rows, 1, dtype=torch.long, device=self.device)
        self.pos = torch.zeros(1, dtype=torch.long, device=self.device)
        self.rope_pos = torch.zeros(rows, dtype=torch.long, device=self.device)
        self.logits = torch.zeros(rows, cfg.embedding_size or cfg.vocab_size, dtype=torch.float32, device=self.device)
        self.cur = 0  # next write column
        self.used: List[bool] = [False] * rows
        self.first_col: List[int] = [0] * rows  # leftmost live column of each used row
        self.fused = self._fused_ok() if fused is None else (fused and self._fused_ok())
        self._graphs: Dict[int, "torch.cuda.CUDAGraph"] = {}
        self._pool = None
        self.graph_replays = 0
        # angle tables up to the context length exist before anything is captured
        block0 = model.transformer.blocks[0]
        block0.rotary_emb.get_rotary_embedding(cfg.max_sequence_length, self.device)

    # ------------------------------------------------------------------------------------ slots
    @property
    def free_rows(self) -> int:
        return self.used.count(False)

    def kv_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)

    def release(self, row: int) -> None:
        self.used[row] = False
        self.bias[row].fill_(self.floor)
        if not any(self.used):
            self.cur = 0

    # -------------------------------------------------------------------------------- movement
    def _shift(self, by: int) -> None:
        """Move every row's live columns ``by`` to the right (``by`` < 0: to the left)."""
        cur, new = self.cur, self.cur + by
        assert 0 <= new <= self.window and (by > 0 or -by <= min(self.first_col[r] for r in range(self.rows) if self.used[r]))
        src = slice(max(0, -by), cur)
        dst = slice(max(0, -by) + by, new)
        for t in self.k + self.v:
            t[:, :, dst] = t[:, :, src].clone()
        moved = self.bias[..., src].clone()
        self.bias.fill_(self.floor)
        self.bias[..., dst] = moved
        self.first_col = [c + by if u else 0 for c, u in zip(self.first_col, self.used)]
        self.cur = new

    def compact(self, force: bool = False) -> None:
        """Reclaim the columns left of every live row.  Cheap check, the copy runs only when at least one bucket (or,
        with ``force``, anything) can be won back."""
        live = [self.first_col[r] for r in range(self.rows) if self.used[r]]
        if not live:
            self.cur = 0
            return
        slack = min(live)
        if slack >= self.bucket or (force and slack > 0):
            self._shift(-slack)

    # ------------------------------------------------------------------------------- admission
    def admit(self, kv: Sequence[Tuple[torch.Tensor, torch.Tensor]], mask: torch.Tensor, first_tokens: torch.Tensor) -> List[int]:
        """Place freshly prefilled sequences into free rows.  ``kv`` is what ``OLMo.forward(use_cache=True)`` returned
        for a left-padded batch (keys before the rotary embedding, ``[n, kv_heads, p, head_dim]``), ``mask`` its
        ``[n, p]`` padding mask, ``first_tokens`` the token each sequence feeds next.  Returns the rows used."""
        n, p = mask.shape
        rows = [r for r in range(self.rows) if not self.used[r]][:n]
        assert len(rows) == n and p < self.window
        if self.cur >= self.window:
            self.compact(force=True)
        if p > self.cur:
            if any(self.used):
                self._shift(p - self.cur)
            self.cur = p
        lo, hi = self.cur - p, self.cur
        index = torch.tensor(rows, device=self.device)
        lengths = mask.sum(dim=1).long()
        token_index = (torch.arange(p, device=self.device)[None, :] - (p - lengths)[:, None]).clamp_min(0)  # [n, p]
        rotary = self.model.transformer.blocks[0].rotary_emb
        sin, cos = rotary.get_rotary_embedding(self.config.max_sequence_length, self.device)
        sin, cos = sin[0, 0][token_index][:, None], cos[0, 0][token_index][:, None]  # [n, 1, p, head_dim]
        full = self.config.rope_full_precision
        for layer, (keys, values) in enumerate(kv):
            k_ = keys.float() if full else keys
            rotated = rotary.apply_rotary_pos_emb(sin.type_as(k_), cos.type_as(k_), k_)
            self.k[layer][index, :, lo:hi] = rotated.to(self.dtype)
            self.v[layer][index, :, lo:hi] = values.to(self.dtype)
        row_bias = torch.full((n, 1, 1, self.window), self.floor, dtype=self.dtype, device=self.device)
        row_bias[:, 0, 0, lo:hi] = torch.where(mask > 0, 0.0, self.floor).to(self.dtype)
        self.bias[index] = row_bias
        self.rope_pos[index] = lengths
        self.tokens[index, 0] = first_tokens
        for r, length in zip(rows, lengths.tolist()):
            self.used[r] = True
            self.first_col[r] = hi - int(length)
        return rows

    # ---------------------------------------------------------------------------------- decode
    def _fused_ok(self) -> bool:
        """The decode kernels of this library cover bf16 models of the architectures the fused training path covers,
        with head dimension 128 (every released OLMo model)."""
        from ..ops import enabled
        from ..ops import fused_block as fb

        cfg = self.config
        return (
            self.device.type == "cuda" and enabled() and self.dtype == torch.bfloat16 and fb.config_supported(cfg)
            and cfg.d_model // cfg.n_heads == 128 and not cfg.embedding_layer_norm
        )

    def _forward_fused(self, length: int) -> None:
        """The step as a short chain of kernels per block: projection, one kernel for QK-norm + rotary + cache write,
        one attention kernel over the window, projection, norm(+residual), projection, SwiGLU, projection,
        norm(+residual).  The projections go through the block's own modules, so dense and 4-bit weights both work."""
        from ..ops import fused_block as fb
        from ..ops import kernels as k

        cfg, t = self.config, self.model.transformer
        spec = fb.spec_from_config(cfg)
        cos, sin = fb.rope_tables(cfg.max_sequence_length, spec.head_dim, float(cfg.rope_theta), self.device)
        scale = 1.0 / (spec.head_dim ** 0.5)
        bias = self.bias.view(self.rows, self.window)

        def w(norm):
            return None if norm is None else norm.weight

        # Dense bf16 projections of a handful of rows are a stream of the weight matrix.  This library's weight-streaming
        # GEMM (csrc/gemm_smallm.cu) was measured against the library GEMM at 32 rows on one B200: 5.5 vs 5.2 TB/s on the
        # vocabulary projection (100352 x 4096), but 1.6-3.5 vs 2.0-3.8 TB/s on the block projections, whose 20-50 us
        # are dominated by start-up and by the second launch that adds the K splits.  OLMO_B200_DECODE_GEMM=auto (default)
        # therefore takes it for projections of at least 32768 features, `native` for all, `library` for none.
        mode = os.environ.get("OLMO_B200_DECODE_GEMM", "auto").strip().lower()
        own_gemm = self.rows <= 256 and mode != "library" and k.gemm_small_m_available()
        min_features = 0 if mode == "native" else 32768

        def proj(linear, h):
            if (own_gemm and type(linear) is torch.nn.Linear and linear.out_features >= min_features
                    and linear.weight.dtype == torch.bfloat16 and h.dtype == torch.bfloat16):
                y = k.gemm_small_m(h.contiguous(), linear.weight)
                return y if linear.bias is None else y + linear.bias
            return linear(h)

        x = t.wte(self.tokens).view(self.rows, cfg.d_model)
        for layer, block in enumerate(t.blocks):
            h = x if spec.norm_after else k.norm_fwd(x, w(block.attn_norm), None, spec.eps, spec.rms, save_stats=False)[0]
            qkv = proj(block.att_proj, h)
            q = k.decode_qkv(qkv, w(block.q_norm), w(block.k_norm), cos, sin, self.rope_pos, self.pos, self.k[layer], self.v[layer],
                             spec.Wq, spec.Wk, spec.head_dim, spec.eps, spec.clip_qkv, spec.qk_norm, spec.rope)
            o = k.decode_attention(q, self.k[layer], self.v[layer], bias, length, scale, spec.n_heads)
            a = proj(block.attn_out, o)
            if spec.norm_after:
                x1 = k.norm_fwd(a, w(block.attn_norm), None, spec.eps, spec.rms, residual=x, save_stats=False)[0]
                f = proj(block.ff_out, k.swiglu_fwd(proj(block.ff_proj, x1)))
                x = k.norm_fwd(f, w(block.ff_norm), None, spec.eps, spec.rms, residual=x1, save_stats=False)[0]
            else:
                x1 = x + a
                h2 = k.norm_fwd(x1, w(block.ff_norm), None, spec.eps, spec.rms, save_stats=False)[0]
                x = x1 + proj(block.ff_out, k.swiglu_fwd(proj(block.ff_proj, h2)))
        x = k.norm_fwd(x, w(t.ln_f), None, spec.eps, spec.rms, save_stats=False)[0]
        head = getattr(t, "ff_out", None)
        if head is not None and not cfg.scale_logits:
            self.logits.copy_(proj(head, x))
        else:
            self.logits.copy_(self.model.output_projection(x))

    def _forward(self, length: int) -> None:
        if self.fused:
            return self._forward_fused(length)
        t = self.model.transformer
        x = t.wte(self.tokens)
        if self.config.embedding_layer_norm:
            x = t.emb_norm(x)
        for layer, block in enumerate(t.blocks):
            x, _ = block(x, attention_bias=self.bias, layer_past=StaticKV(self.k[layer], self.v[layer], self.pos, length, self.rope_pos))
        x = t.ln_f(x)
        self.logits.copy_(self.model.output_projection(x)[:, 0])

    def _capture(self, length: int) -> "torch.cuda.CUDAGraph":
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):  # warm-up off the capture: library handles, workspaces, lazy module loads
            for _ in range(2):
                self._forward(length)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(graph, pool=self._pool):
            self._forward(length)
        return graph

    @torch.no_grad()
    def decode(self, active_rows: torch.Tensor) -> torch.Tensor:
        """One token for every row; returns the ``[rows, vocab]`` logits buffer (idle rows hold noise).  The caller
        samples, writes the chosen tokens into ``tokens`` and calls :meth:`advance`."""
        if self.cur >= self.window:
            self.compact(force=True)
            if self.cur >= self.window:
                raise RuntimeError("the key/value window is full: a row reached the window length without finishing")
        self.bias[active_rows, 0, 0, self.cur] = 0.0
        self.pos.fill_(self.cur)
        length = min(self.window, -(-(self.cur + 1) // self.bucket) * self.bucket)
        if self.cuda_graphs:
            graph = self._graphs.get(length)
            if graph is None:
                graph = self._graphs[length] = self._capture(length)
            graph.replay()
            self.graph_replays += 1
        else:
            self._forward(length)
        return self.logits

    def advance(self, active_rows: torch.Tensor, tokens: torch.Tensor) -> None:
        self.tokens[active_rows, 0] = tokens
        self.rope_pos.add_(1).clamp_(max=self.config.max_sequence_length - 1)
        self.cur += 1
