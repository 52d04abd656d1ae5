"""
Attention entry points used by the model.

Layouts follow the flash-attention convention: ``q`` is ``(B, Tq, H, D)``, ``k``/``v`` are
``(B, Tk, Hkv, D)`` (grouped-query when ``Hkv < H``); the last dimension is contiguous and the others
may be strided views into a fused QKV buffer.

Three back ends implement the same ``forward -> (out, lse)`` / ``backward -> (dq, dk, dv)`` pair:

``native``   the tcgen05 kernels of ``csrc/attention.cu`` (head dim 128, bf16, causal or full);
``library``  the ``flash_attn`` package's kernels (counted as a library call, like cuBLAS);
``math``     an explicit fp32 softmax in PyTorch ops — any device, any mask; the numerical oracle.

``OLMO_B200_ATTENTION`` selects ``native`` (default, falls back to ``library`` for shapes the native
kernel does not cover), ``library`` or ``math``.
"""
from __future__ import annotations

import math
import os
from typing import Callable, Optional, Tuple

import torch

__all__ = [
    "flash_attention",
    "varlen_attention",
    "attention_forward",
    "attention_backward",
    "math_attention_forward",
    "backend_for",
]


def _requested_backend() -> str:
    return os.environ.get("OLMO_B200_ATTENTION", "native").strip().lower()


def _library():
    try:
        import flash_attn.flash_attn_interface as fai  # type: ignore

        return fai
    except Exception:
        return None


def _native_supports(q: torch.Tensor, k: torch.Tensor, causal: bool, dropout_p: float, varlen: bool) -> bool:
    from . import attention_native

    return attention_native.supports(q, k, causal, dropout_p, varlen)


def backend_for(q: torch.Tensor, k: torch.Tensor, causal: bool, dropout_p: float = 0.0, varlen: bool = False) -> str:
    """Pick the back end for these operands."""
    want = _requested_backend()
    if not q.is_cuda or q.dtype not in (torch.bfloat16, torch.float16) or want == "math":
        return "math"
    if want == "native" and _native_supports(q, k, causal, dropout_p, varlen):
        return "native"
    if _library() is not None:
        return "library"
    return "math"


# ------------------------------------------------------------------------------------------- math


def _expand_kv(k: torch.Tensor, H: int) -> torch.Tensor:
    Hkv = k.shape[2]
    return k if Hkv == H else k.repeat_interleave(H // Hkv, dim=2)


def _doc_mask(doc_start: torch.Tensor) -> torch.Tensor:
    """``[B, T]`` document starts -> boolean ``[B, 1, T, T]`` of pairs (query, key) with ``doc_start[query] <= key``."""
    T = doc_start.shape[1]
    keys = torch.arange(T, device=doc_start.device)
    return (keys.view(1, 1, 1, T) >= doc_start.view(doc_start.shape[0], 1, T, 1).to(torch.int64))


def _mask(Tq: int, Tk: int, causal: bool, device, cu: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """Boolean ``(Tq, Tk)`` mask of allowed pairs (bottom-right aligned causal, like flash-attention)."""
    allowed = None
    if causal:
        i = torch.arange(Tq, device=device)[:, None] + (Tk - Tq)
        j = torch.arange(Tk, device=device)[None, :]
        allowed = j <= i
    if cu is not None:
        doc = torch.bucketize(torch.arange(Tq, device=device), cu[1:].to(device), right=True)
        same = doc[:, None] == doc[None, :]
        allowed = same if allowed is None else (allowed & same)
    return allowed


def math_attention_forward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool, scale: Optional[float] = None,
    cu_seqlens: Optional[torch.Tensor] = None, doc_start: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 softmax attention; returns ``out (B,Tq,H,D)`` in the input dtype and ``lse (B,H,Tq)`` fp32."""
    B, Tq, H, D = q.shape
    Tk = k.shape[1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qf = q.float().transpose(1, 2)
    kf = _expand_kv(k, H).float().transpose(1, 2)
    vf = _expand_kv(v, H).float().transpose(1, 2)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    allowed = _mask(Tq, Tk, causal, q.device, cu_seqlens)
    if allowed is not None:
        s = s.masked_fill(~allowed, float("-inf"))
    if doc_start is not None:
        s = s.masked_fill(~_doc_mask(doc_start), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse.unsqueeze(-1))
    out = torch.matmul(p, vf).transpose(1, 2).to(q.dtype)
    return out, lse


def _math_attention_backward(do, q, k, v, out, lse, causal, scale, cu_seqlens=None, doc_start=None):
    B, Tq, H, D = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qf = q.float().transpose(1, 2)
    kf = _expand_kv(k, H).float().transpose(1, 2)
    vf = _expand_kv(v, H).float().transpose(1, 2)
    dof = do.float().transpose(1, 2)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    allowed = _mask(Tq, Tk, causal, q.device, cu_seqlens)
    if allowed is not None:
        s = s.masked_fill(~allowed, float("-inf"))
    if doc_start is not None:
        s = s.masked_fill(~_doc_mask(doc_start), float("-inf"))
    p = torch.exp(s - lse.unsqueeze(-1))
    dv = torch.matmul(p.transpose(-1, -2), dof)
    dp = torch.matmul(dof, vf.transpose(-1, -2))
    delta = (dof * out.float().transpose(1, 2)).sum(-1, keepdim=True)
    ds = p * (dp - delta) * scale
    dq = torch.matmul(ds, kf).transpose(1, 2)
    dk = torch.matmul(ds.transpose(-1, -2), qf)
    if Hkv != H:
        g = H // Hkv
        dk = dk.view(B, Hkv, g, Tk, D).sum(2)
        dv = dv.view(B, Hkv, g, Tk, D).sum(2)
    return dq.to(q.dtype), dk.transpose(1, 2).to(k.dtype), dv.transpose(1, 2).to(v.dtype)


# --------------------------------------------------------------------------- explicit fwd / bwd


def attention_forward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True, scale: Optional[float] = None,
    out: Optional[torch.Tensor] = None, doc_start: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, str]:
    """Forward without autograd bookkeeping: returns ``(out, lse, backend)``.  ``doc_start`` (int32 ``[B, T]``, causal
    only) restricts every query to the keys of its own document; the native kernel and the math path implement it."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    be = backend_for(q, k, causal)
    if doc_start is not None and be == "library":
        be = "math"  # the library expresses document masking through packed variable-length calls only
    if be == "native":
        from . import attention_native

        o, lse = attention_native.forward(q, k, v, causal, scale, out=out, doc_start=doc_start)
        return o, lse, be
    if be == "library":
        fai = _library()
        o, lse, _, _ = fai._flash_attn_forward(q, k, v, 0.0, scale, causal, -1, -1, 0.0, None, False)
        return o, lse, be
    o, lse = math_attention_forward(q, k, v, causal, scale, doc_start=doc_start)
    return o, lse, be


def attention_backward(
    do: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, lse: torch.Tensor,
    dq: torch.Tensor, dk: torch.Tensor, dv: torch.Tensor, causal: bool = True, scale: Optional[float] = None,
    backend: Optional[str] = None, doc_start: Optional[torch.Tensor] = None,
) -> None:
    """Backward into caller-provided (possibly strided) ``dq``, ``dk``, ``dv``."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    be = backend or backend_for(q, k, causal)
    if be == "native":
        from . import attention_native

        if attention_native.supports_backward(q, k, causal):
            attention_native.backward(do, q, k, v, out, lse, dq, dk, dv, causal, scale, doc_start=doc_start)
            return
        be = "library" if (_library() is not None and doc_start is None) else "math"
    if doc_start is not None and be == "library":
        be = "math"
    if be == "library":
        fai = _library()
        fai._flash_attn_backward(do, q, k, v, out, lse, dq, dk, dv, 0.0, scale, causal, -1, -1, 0.0, None, False)
        return
    g = _math_attention_backward(do, q, k, v, out, lse, causal, scale, doc_start=doc_start)
    dq.copy_(g[0])
    dk.copy_(g[1])
    dv.copy_(g[2])


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        o, lse, be = attention_forward(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale, ctx.backend = causal, scale, be
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        attention_backward(do.contiguous(), q, k, v, o, lse, dq, dk, dv, ctx.causal, ctx.scale, ctx.backend)
        return dq, dk, dv, None, None


def flash_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    dropout_p: float = 0.0,
    causal: bool = True,
    scale: Optional[float] = None,
    library_fn: Optional[Callable] = None,
) -> torch.Tensor:
    """Differentiable attention in ``(B, T, H, D)`` layout."""
    if dropout_p > 0.0:
        if library_fn is not None and q.is_cuda:
            return library_fn(q, k, v, dropout_p=dropout_p, softmax_scale=scale, causal=causal)
        H = q.shape[2]
        out = torch.nn.functional.scaled_dot_product_attention(
            q.transpose(1, 2), _expand_kv(k, H).transpose(1, 2), _expand_kv(v, H).transpose(1, 2),
            dropout_p=dropout_p, is_causal=causal, scale=scale,
        )
        return out.transpose(1, 2)
    return _Attention.apply(q, k, v, causal, scale)


class _VarlenMath(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cu, causal, scale):
        o, lse = math_attention_forward(q[None], k[None], v[None], causal, scale, cu_seqlens=cu)
        ctx.save_for_backward(q, k, v, o, lse, cu)
        ctx.causal, ctx.scale = causal, scale
        return o[0]

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, cu = ctx.saved_tensors
        dq, dk, dv = _math_attention_backward(do[None], q[None], k[None], v[None], o, lse, ctx.causal, ctx.scale, cu)
        return dq[0], dk[0], dv[0], None, None, None


def varlen_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    dropout_p: float = 0.0,
    causal: bool = True,
    scale: Optional[float] = None,
    library_fn: Optional[Callable] = None,
) -> torch.Tensor:
    """Intra-document attention over packed sequences: ``q``/``k``/``v`` are ``(total_tokens, H, D)`` and
    ``cu_seqlens`` the int32 cumulative document lengths with a leading 0."""
    if q.is_cuda and q.dtype in (torch.bfloat16, torch.float16) and _requested_backend() != "math":
        from . import attention_native

        if _requested_backend() != "library" and attention_native.supports_varlen(q, k, causal, dropout_p):
            return attention_native.varlen(q, k, v, cu_seqlens, max_seqlen, causal, scale)
        fn = library_fn
        if fn is None and _library() is not None:
            fn = _library().flash_attn_varlen_func
        if fn is not None:
            return fn(q, k, v, cu_seqlens, cu_seqlens, max_seqlen, max_seqlen, dropout_p=dropout_p, softmax_scale=scale, causal=causal)
    assert dropout_p == 0.0, "dropout with document masking needs the flash-attn package"
    return _VarlenMath.apply(q, k, v, cu_seqlens, causal, scale)
