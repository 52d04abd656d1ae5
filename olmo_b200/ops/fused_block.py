"""
One transformer block as two explicit kernel sequences (forward, backward) with a hand-picked list of
saved activations — the unit of work of the sm_100a training path.

Forward of the OLMo-2 block (``norm_after``), M = B·T token rows, d = model width, H = SwiGLU width:

    qkv = x · Wqkvᵀ                       tcgen05 GEMM
    q,k = rope(rmsnorm(q)·wq, rmsnorm(k)·wk)   one kernel (csrc/rope.cu)
    o   = flash_attention(q, k, v)
    a   = o · Woᵀ                          GEMM
    x1  = x + rmsnorm(a)·w₁                one kernel (csrc/norm.cu)
    h   = x1 · Wffᵀ                        GEMM
    act = silu(h[:, H:]) · h[:, :H]
    f   = act · Woutᵀ                      GEMM
    y   = x1 + rmsnorm(f)·w₂

Saved for backward: x, qkv, (rstd of q and k), o, lse, a, x1, h, f and the norm statistics.  The rotated
q/k and the SwiGLU output are recomputed in the backward pass (two bandwidth-bound kernels) instead of being
stored, which is what lets a 7B model train on one 180 GB device without activation checkpointing.
Weight gradients go straight from the GEMM epilogue into the owner-supplied gradient buffers
(fp32 accumulate, or bf16 overwrite when a reduce-scatter follows).

The pre-norm OLMo-1 block (``norm_after=False``, optional ``clip_qkv``, non-parametric LayerNorm) is the
second variant; residual additions are folded into the GEMM epilogue there.

Reference semantics: ``olmo/model.py:728-823`` (block), ``:588-656`` (attention).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Optional, Tuple

import torch

from ..config import ActivationType, BlockType, LayerNormType
from . import attention as attn
from . import enabled
from . import kernels as k

__all__ = ["BlockSpec", "GradSink", "block_forward", "block_backward", "eligible", "run_block", "rope_tables", "spec_from_config"]


@dataclass(frozen=True)
class BlockSpec:
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    hidden: int  # SwiGLU output width (= ff_proj width / 2)
    eps: float
    rms: bool
    norm_after: bool
    qk_norm: bool
    rope: bool
    clip_qkv: float  # 0 = off

    @property
    def Wq(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def Wk(self) -> int:
        return self.n_kv_heads * self.head_dim


def spec_from_config(cfg) -> BlockSpec:
    return BlockSpec(
        d_model=cfg.d_model,
        n_heads=cfg.n_heads,
        n_kv_heads=cfg.effective_n_kv_heads,
        head_dim=cfg.d_model // cfg.n_heads,
        hidden=cfg.ff_proj_width // 2,
        eps=cfg.layer_norm_eps,
        rms=cfg.layer_norm_type == LayerNormType.rms,
        norm_after=cfg.norm_after,
        qk_norm=cfg.attention_layer_norm,
        rope=cfg.rope,
        clip_qkv=float(cfg.clip_qkv or 0.0),
    )


def config_supported(cfg) -> bool:
    """Static part of eligibility: what the fused kernels implement."""
    hd = cfg.d_model // cfg.n_heads
    return (
        cfg.block_type == BlockType.sequential
        and cfg.activation_type == ActivationType.swiglu
        and not cfg.include_bias
        and not (cfg.bias_for_layer_norm or False)
        and cfg.layer_norm_type in (LayerNormType.rms, LayerNormType.default)
        and (not cfg.attention_layer_norm or cfg.layer_norm_type == LayerNormType.rms)
        and not cfg.alibi
        and cfg.rope
        and cfg.rope_full_precision
        and cfg.attention_dropout == 0.0
        and cfg.residual_dropout == 0.0
        and hd % 16 == 0
        and cfg.d_model % 8 == 0
        and cfg.d_model <= 8192
        and (cfg.ff_proj_width // 2) % 8 == 0
    )


def eligible(block, x: torch.Tensor, attention_bias, layer_past, use_cache: bool, doc_masking: bool = False) -> bool:
    """True when this call can run on the fused path (training/eval forward without cache or explicit bias).  With
    intra-document masking the native attention kernel must cover the shape (head dim up to 128)."""
    if not (x.is_cuda and enabled()) or attention_bias is not None or layer_past is not None or use_cache:
        return False
    if doc_masking and block.config.d_model // block.config.n_heads > 128:
        return False
    if x.dtype != torch.bfloat16 and not (torch.is_autocast_enabled() and torch.get_autocast_dtype("cuda") == torch.bfloat16):
        return False
    if block._activation_checkpoint_fn is not None:  # fine-grained checkpointing is a portable-path feature
        return False
    if getattr(block, "_fused_ok", None) is None:
        block._fused_ok = config_supported(block.config)
    return bool(block._fused_ok)


_ROPE_CACHE: Dict[Tuple[int, int, float, int], Tuple[torch.Tensor, torch.Tensor]] = {}


def rope_tables(seq_len: int, head_dim: int, theta: float, device: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``cos``/``sin`` of shape ``[seq_len, head_dim/2]``, computed exactly like the portable model."""
    key = (seq_len, head_dim, float(theta), device.index or 0)
    hit = _ROPE_CACHE.get(key)
    if hit is None:
        inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float) / head_dim))
        ang = torch.outer(torch.arange(seq_len, device=device, dtype=torch.float), inv)
        hit = (ang.cos().contiguous(), ang.sin().contiguous())
        _ROPE_CACHE[key] = hit
    return hit


class GradSink:
    """Where parameter gradients go.

    The default sink allocates bf16 gradients and returns them (used by the autograd wrapper).  The
    flat-shard engine substitutes a sink that points each name at a slice of its gradient buffers.
    """

    def __init__(self) -> None:
        self.grads: Dict[str, torch.Tensor] = {}

    def matrix(self, name: str, dy: torch.Tensor, x: torch.Tensor) -> None:
        """``grad[name] (+)= dyᵀ · x`` for a Linear weight ``[out, in]``."""
        self.grads[name] = k.gemm(dy, x, a_trans=True, b_trans=True)

    def vector(self, name: str, like: torch.Tensor) -> torch.Tensor:
        """An fp32 accumulator for a norm weight; the kernel adds into it."""
        g = torch.zeros(like.shape, dtype=torch.float32, device=like.device)
        self.grads[name] = g
        return g


def _split_heads(buf: torch.Tensor, col0: int, width: int, B: int, T: int, hd: int) -> torch.Tensor:
    """View columns ``[col0, col0+width)`` of a ``[B·T, ld]`` buffer as ``(B, T, heads, hd)`` without copying."""
    ld = buf.stride(0)
    return buf.as_strided((B, T, width // hd, hd), (T * ld, ld, hd, 1), buf.storage_offset() + col0)


def _norm_w(w: Dict[str, Optional[torch.Tensor]], name: str) -> Optional[torch.Tensor]:
    return w.get(name)


def block_forward(
    spec: BlockSpec,
    w: Dict[str, Optional[torch.Tensor]],
    x: torch.Tensor,
    B: int,
    T: int,
    cos: torch.Tensor,
    sin: torch.Tensor,
    save: bool = True,
    gemm_kwargs: Optional[Dict[str, Dict[str, Any]]] = None,
    doc_start: Optional[torch.Tensor] = None,
    keep_recomputable: bool = False,
) -> Tuple[torch.Tensor, Optional[Dict[str, Any]]]:
    """``x`` is ``[B·T, d]`` bf16.  ``w`` maps ``att_proj, attn_out, ff_proj, ff_out`` to weights and
    ``attn_norm, ff_norm, q_norm, k_norm`` to norm weights or ``None``.  ``gemm_kwargs[name]`` may carry the
    readiness-flag arguments of a weight that is still arriving from peers.  ``keep_recomputable`` also saves the
    rotated q/k and the SwiGLU output, which the backward pass otherwise recomputes (two bandwidth-bound kernels per
    block traded for ``(Wq + Wk + hidden/2)·2`` bytes per token)."""
    gk = gemm_kwargs or {}
    Wq, Wk, hd = spec.Wq, spec.Wk, spec.head_dim
    saved: Dict[str, Any] = {}

    if spec.norm_after:
        h_in = x
    else:
        h_in, rstd1, mean1 = k.norm_fwd(x, _norm_w(w, "attn_norm"), None, spec.eps, spec.rms, save_stats=save)
        saved.update(rstd1=rstd1, mean1=mean1)
    qkv = k.gemm(h_in, w["att_proj"], **gk.get("att_proj", {}))
    qk, rstd_q, rstd_k = k.qk_norm_rope_fwd(
        qkv, _norm_w(w, "q_norm"), _norm_w(w, "k_norm"), cos, sin, T, Wq, Wk, hd, spec.eps, spec.clip_qkv,
        spec.qk_norm, spec.rope,
    )
    q = _split_heads(qk, 0, Wq, B, T, hd)
    kk = _split_heads(qk, Wq, Wk, B, T, hd)
    v = _split_heads(qk, Wq + Wk, Wk, B, T, hd) if spec.clip_qkv > 0 else _split_heads(qkv, Wq + Wk, Wk, B, T, hd)
    o, lse, backend = attn.attention_forward(q, kk, v, causal=True, doc_start=doc_start)
    o2 = o.view(B * T, Wq)
    qk_keep = qk if (save and keep_recomputable) else None
    del qk, q, kk

    if spec.norm_after:
        a = k.gemm(o2, w["attn_out"], **gk.get("attn_out", {}))
        x1, rstd_a, _ = k.norm_fwd(a, _norm_w(w, "attn_norm"), None, spec.eps, spec.rms, residual=x, save_stats=save)
        h = k.gemm(x1, w["ff_proj"], **gk.get("ff_proj", {}))
        act = k.swiglu_fwd(h)
        f = k.gemm(act, w["ff_out"], **gk.get("ff_out", {}))
        y, rstd_f, _ = k.norm_fwd(f, _norm_w(w, "ff_norm"), None, spec.eps, spec.rms, residual=x1, save_stats=save)
        if save:
            saved.update(a=a, rstd_a=rstd_a, f=f, rstd_f=rstd_f)
    else:
        x1 = k.gemm(o2, w["attn_out"], epilogue=k.EPI_BF16_ADD, residual=x, **gk.get("attn_out", {}))
        h2, rstd2, mean2 = k.norm_fwd(x1, _norm_w(w, "ff_norm"), None, spec.eps, spec.rms, save_stats=save)
        h = k.gemm(h2, w["ff_proj"], **gk.get("ff_proj", {}))
        act = k.swiglu_fwd(h)
        y = k.gemm(act, w["ff_out"], epilogue=k.EPI_BF16_ADD, residual=x1, **gk.get("ff_out", {}))
        if save:
            saved.update(rstd2=rstd2, mean2=mean2)
    if not save:
        return y, None
    saved.update(x=x, qkv=qkv, rstd_q=rstd_q, rstd_k=rstd_k, o=o, lse=lse, x1=x1, h=h, B=B, T=T, attn_backend=backend, doc_start=doc_start)
    if keep_recomputable:
        saved.update(qk=qk_keep, act=act)
        if not spec.norm_after:  # pre-norm blocks also recompute the two normalised GEMM inputs
            saved.update(h1=h_in, h2=h2)
    return y, saved


def block_backward(
    spec: BlockSpec,
    w: Dict[str, Optional[torch.Tensor]],
    saved: Dict[str, Any],
    dy: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    sink: GradSink,
    need_dx: bool = True,
    gemm_kwargs: Optional[Dict[str, Dict[str, Any]]] = None,
) -> Optional[torch.Tensor]:
    """Gradient w.r.t. the block input; parameter gradients are delivered to ``sink``.  ``gemm_kwargs`` may attach a
    communication task to the two largest input-gradient GEMMs (keys ``ff_out_dgrad`` and ``attn_out_dgrad``)."""
    gk = gemm_kwargs or {}
    Wq, Wk, hd = spec.Wq, spec.Wk, spec.head_dim
    B, T = saved["B"], saved["T"]
    M = B * T
    x, qkv, x1, h = saved["x"], saved["qkv"], saved["x1"], saved["h"]
    o2 = saved["o"].view(M, Wq)

    def vec(name: str) -> Optional[torch.Tensor]:
        p = _norm_w(w, name)
        return None if p is None else sink.vector(name, p)

    # ---- feed-forward half
    if spec.norm_after:
        d_f = k.norm_bwd(dy, saved["f"], _norm_w(w, "ff_norm"), saved["rstd_f"], None, spec.rms, dweight=vec("ff_norm"))
        dx1_res = dy
    else:
        d_f = dy
        dx1_res = dy
    act = saved.pop("act", None)
    if act is None:
        act = k.swiglu_fwd(h)  # recomputed
    sink.matrix("ff_out", d_f, act)
    d_act = k.gemm(d_f, w["ff_out"], b_trans=True, **gk.get("ff_out_dgrad", {}))
    del act
    d_h = k.swiglu_bwd(d_act, h)
    del d_act
    if spec.norm_after:
        sink.matrix("ff_proj", d_h, x1)
        dx1 = k.gemm(d_h, w["ff_proj"], b_trans=True, epilogue=k.EPI_BF16_ADD, residual=dx1_res, **gk.get("ff_proj_dgrad", {}))
    else:
        h2 = saved.pop("h2", None)
        if h2 is None:
            h2, _, _ = k.norm_fwd(x1, _norm_w(w, "ff_norm"), None, spec.eps, spec.rms, save_stats=False)  # recomputed
        sink.matrix("ff_proj", d_h, h2)
        del h2
        d_h2 = k.gemm(d_h, w["ff_proj"], b_trans=True, **gk.get("ff_proj_dgrad", {}))
        dx1 = k.norm_bwd(d_h2, x1, _norm_w(w, "ff_norm"), saved["rstd2"], saved["mean2"], spec.rms, dres=dx1_res, dweight=vec("ff_norm"))
    del d_h

    # ---- attention half
    if spec.norm_after:
        d_a = k.norm_bwd(dx1, saved["a"], _norm_w(w, "attn_norm"), saved["rstd_a"], None, spec.rms, dweight=vec("attn_norm"))
    else:
        d_a = dx1
    sink.matrix("attn_out", d_a, o2)
    d_o = k.gemm(d_a, w["attn_out"], b_trans=True, **gk.get("attn_out_dgrad", {}))

    qk = saved.pop("qk", None)
    if qk is None:
        qk, _, _ = k.qk_norm_rope_fwd(  # recomputed rotated q/k
            qkv, _norm_w(w, "q_norm"), _norm_w(w, "k_norm"), cos, sin, T, Wq, Wk, hd, spec.eps, spec.clip_qkv, spec.qk_norm, spec.rope
        )
    q = _split_heads(qk, 0, Wq, B, T, hd)
    kk = _split_heads(qk, Wq, Wk, B, T, hd)
    v = _split_heads(qk, Wq + Wk, Wk, B, T, hd) if spec.clip_qkv > 0 else _split_heads(qkv, Wq + Wk, Wk, B, T, hd)
    dqkv = torch.empty_like(qkv)
    attn.attention_backward(
        d_o.view(B, T, spec.n_heads, hd), q, kk, v, saved["o"], saved["lse"],
        _split_heads(dqkv, 0, Wq, B, T, hd), _split_heads(dqkv, Wq, Wk, B, T, hd), _split_heads(dqkv, Wq + Wk, Wk, B, T, hd),
        causal=True, backend=saved["attn_backend"], doc_start=saved.get("doc_start"),
    )
    del qk, q, kk, d_o
    k.qk_norm_rope_bwd(
        qkv, dqkv, _norm_w(w, "q_norm"), _norm_w(w, "k_norm"), cos, sin, saved["rstd_q"], saved["rstd_k"], T, Wq, Wk, hd,
        spec.clip_qkv, spec.qk_norm, spec.rope, dwq=vec("q_norm") if spec.qk_norm else None, dwk=vec("k_norm") if spec.qk_norm else None,
    )
    if spec.norm_after:
        sink.matrix("att_proj", dqkv, x)
        if not need_dx:
            assert "att_proj_dgrad" not in gk, "a collective was attached to a GEMM that is skipped"
            return None
        return k.gemm(dqkv, w["att_proj"], b_trans=True, epilogue=k.EPI_BF16_ADD, residual=dx1, **gk.get("att_proj_dgrad", {}))
    h1 = saved.pop("h1", None)
    if h1 is None:
        h1, _, _ = k.norm_fwd(x, _norm_w(w, "attn_norm"), None, spec.eps, spec.rms, save_stats=False)  # recomputed
    sink.matrix("att_proj", dqkv, h1)
    del h1
    d_h1 = k.gemm(dqkv, w["att_proj"], b_trans=True, **gk.get("att_proj_dgrad", {}))
    return k.norm_bwd(d_h1, x, _norm_w(w, "attn_norm"), saved["rstd1"], saved["mean1"], spec.rms, dres=dx1, dweight=vec("attn_norm"))


# ------------------------------------------------------------------------------ autograd wrapper

_PARAM_ORDER = ("att_proj", "attn_out", "ff_proj", "ff_out", "attn_norm", "ff_norm", "q_norm", "k_norm")


def _block_weights(block, dtype=torch.bfloat16) -> Dict[str, Optional[torch.Tensor]]:
    def cast(p):
        return None if p is None else (p if p.dtype == dtype else p.to(dtype))

    return {
        "att_proj": cast(block.att_proj.weight),
        "attn_out": cast(block.attn_out.weight),
        "ff_proj": cast(block.ff_proj.weight),
        "ff_out": cast(block.ff_out.weight),
        "attn_norm": cast(block.attn_norm.weight),
        "ff_norm": cast(block.ff_norm.weight),
        "q_norm": cast(block.q_norm.weight) if block.q_norm is not None else None,
        "k_norm": cast(block.k_norm.weight) if block.k_norm is not None else None,
    }


class _FusedBlock(torch.autograd.Function):
    @staticmethod
    def forward(ctx, spec, B, T, cos, sin, doc_start, x, *params):
        w = dict(zip(_PARAM_ORDER, params))
        need_grad = torch.is_grad_enabled() and (x.requires_grad or any(p is not None and p.requires_grad for p in params))
        y, saved = block_forward(spec, w, x, B, T, cos, sin, save=need_grad, doc_start=doc_start)
        ctx.spec, ctx.saved, ctx.w, ctx.cos, ctx.sin = spec, saved, w, cos, sin
        return y

    @staticmethod
    def backward(ctx, dy):
        sink = GradSink()
        dx = block_backward(ctx.spec, ctx.w, ctx.saved, dy.contiguous(), ctx.cos, ctx.sin, sink)
        ctx.saved = None
        grads = []
        for name in _PARAM_ORDER:
            g = sink.grads.get(name)
            p = ctx.w[name]
            grads.append(None if (g is None or p is None) else g.to(p.dtype))
        return (None, None, None, None, None, None, dx, *grads)


def run_block(block, x: torch.Tensor, max_doc_len=None, cu_doc_lens=None) -> torch.Tensor:
    """Autograd-visible fused block for ``(B, T, d)`` input.  Parameters held in fp32 are cast to bf16 on the
    way in (the engine avoids this by keeping bf16 compute copies)."""
    B, T, D = x.shape
    doc_start = None
    if cu_doc_lens is not None:  # intra-document masking: the kernels take per-token document starts
        from .attention_native import doc_start_from_cu

        doc_start = doc_start_from_cu(cu_doc_lens, B, T)
    spec = getattr(block, "_fused_spec", None)
    if spec is None:
        spec = block._fused_spec = spec_from_config(block.config)
    cos, sin = rope_tables(T, spec.head_dim, float(block.config.rope_theta), x.device)
    w = _block_weights(block)
    x2 = x.reshape(B * T, D)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    y = _FusedBlock.apply(spec, B, T, cos, sin, doc_start, x2.contiguous(), *[w[n] for n in _PARAM_ORDER])
    return y.view(B, T, D)
