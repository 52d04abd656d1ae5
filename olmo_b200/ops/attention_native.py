"""
Python side of the tcgen05 flash-attention kernels (``csrc/attention.cu``).

``supports`` reports whether the native kernel covers a call; callers fall back to the library or the
math back end otherwise (see :mod:`olmo_b200.ops.attention`).
"""
from __future__ import annotations

from ctypes import c_float, c_int
from typing import Optional, Tuple

import torch

from . import check, lib, ptr, status_tensor, stream_ptr


def _have_symbol(name: str) -> bool:
    try:
        return hasattr(lib(), name)
    except Exception:
        return False


TILE = 128  # the kernels work on 128-row tiles of 128-wide heads


def _needs_padding(q: torch.Tensor) -> bool:
    return q.shape[-1] != TILE or q.shape[1] % TILE != 0


def supports(q: torch.Tensor, k: torch.Tensor, causal: bool, dropout_p: float, varlen: bool) -> bool:
    """Kernel coverage: bf16, no dropout, self-attention (Tq == Tk), query heads a multiple of key heads, and either the
    kernels' own tile shape (head dim 128, T a multiple of 128) or a shape that zero padding brings to it: a head
    dimension below 128 that is a multiple of 8 (the extra columns add nothing to a score and produce zero outputs), and,
    for causal attention, any sequence length (padded keys come after every real query, so the causal mask hides them).
    ``varlen`` means packed sequences described by cumulative lengths; document masking inside fixed-length sequences
    is expressed with ``doc_start`` instead (see :func:`doc_start_from_lengths`) and is covered when ``causal``."""
    if varlen or dropout_p != 0.0 or q.dtype != torch.bfloat16 or not q.is_cuda:
        return False
    if q.dim() != 4 or q.shape[1] != k.shape[1] or q.shape[2] % k.shape[2] != 0:
        return False
    D, T = q.shape[-1], q.shape[1]
    if D > TILE or D % 8 != 0 or k.shape[-1] != D:
        return False
    if T % TILE != 0 and not causal:
        return False
    return _have_symbol("ob_attention_fwd")


def supports_backward(q: torch.Tensor, k: torch.Tensor, causal: bool) -> bool:
    return supports(q, k, causal, 0.0, False) and _have_symbol("ob_attention_bwd")


def _strides(t: torch.Tensor) -> Tuple[int, int, int]:
    assert t.stride(-1) == 1
    return t.stride(0), t.stride(1), t.stride(2)


def doc_start_from_lengths(doc_lens: torch.Tensor, seq_len: int) -> torch.Tensor:
    """``[B, max_docs]`` document lengths (zero padded, each row summing to ``seq_len``) -> int32 ``[B, seq_len]`` with, for
    every token, the position of the first token of its document."""
    lens = doc_lens.to(torch.int64)
    ends = lens.cumsum(dim=1)
    starts = ends - lens
    pos = torch.arange(seq_len, device=doc_lens.device).unsqueeze(0).expand(lens.shape[0], -1)
    doc_of = torch.searchsorted(ends, pos.contiguous(), right=True).clamp_(max=lens.shape[1] - 1)
    return starts.gather(1, doc_of).to(torch.int32).contiguous()


def doc_start_from_cu(cu_doc_lens: torch.Tensor, batch: int, seq_len: int) -> torch.Tensor:
    """Cumulative document boundaries over the flattened ``batch * seq_len`` token axis -> int32 ``[batch, seq_len]``."""
    cu = cu_doc_lens.to(torch.int64)
    pos = torch.arange(batch * seq_len, device=cu.device)
    doc_of = torch.searchsorted(cu, pos, right=True) - 1
    start = cu[doc_of.clamp_(min=0)]
    return (start - (pos // seq_len) * seq_len).clamp_(min=0).view(batch, seq_len).to(torch.int32).contiguous()


def _pad(t: torch.Tensor, T_pad: int) -> torch.Tensor:
    """``(B, T, H, D)`` -> contiguous ``(B, T_pad, H, 128)`` with zeros in the new rows and columns."""
    B, T, H, D = t.shape
    out = t.new_zeros((B, T_pad, H, TILE))
    out[:, :T, :, :D].copy_(t)
    return out


def _pad_doc_start(doc_start: Optional[torch.Tensor], T_pad: int) -> Optional[torch.Tensor]:
    if doc_start is None or doc_start.shape[1] == T_pad:
        return doc_start
    B, T = doc_start.shape
    tail = torch.arange(T, T_pad, device=doc_start.device, dtype=torch.int32).expand(B, -1)  # each padded token is its own document
    return torch.cat([doc_start, tail], dim=1).contiguous()


def forward(q, k, v, causal: bool, scale: float, out: Optional[torch.Tensor] = None, doc_start: Optional[torch.Tensor] = None):
    if _needs_padding(q):
        B, T, H, D = q.shape
        T_pad = -(-T // TILE) * TILE
        o_p, lse_p = forward(_pad(q, T_pad), _pad(k, T_pad), _pad(v, T_pad), causal, scale, doc_start=_pad_doc_start(doc_start, T_pad))
        o = o_p[:, :T, :, :D]
        if out is not None:
            out.copy_(o)
            o = out
        else:
            o = o.contiguous()
        return o, lse_p[:, :, :T].contiguous()
    B, T, H, D = q.shape
    if doc_start is not None:
        assert causal and doc_start.dtype == torch.int32 and doc_start.shape == (B, T) and doc_start.is_contiguous()
    Hkv = k.shape[2]
    o = torch.empty((B, T, H, D), dtype=q.dtype, device=q.device) if out is None else out
    lse = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    rc = lib().ob_attention_fwd(
        ptr(q), ptr(k), ptr(v), ptr(o), ptr(lse), c_int(B), c_int(T), c_int(H), c_int(Hkv),
        *(c_int(s) for s in _strides(q)), *(c_int(s) for s in _strides(k)), *(c_int(s) for s in _strides(v)),
        *(c_int(s) for s in _strides(o)), c_float(scale), c_int(int(causal)), ptr(status_tensor(q.device)), ptr(doc_start), stream_ptr(),
    )
    check(rc, "ob_attention_fwd")
    return o, lse


def backward(do, q, k, v, o, lse, dq, dk, dv, causal: bool, scale: float, doc_start: Optional[torch.Tensor] = None) -> None:
    """Gradients into caller-provided (possibly strided) ``dq``, ``dk``, ``dv``.  Scratch: ``delta`` (B·H·T floats) and
    an fp32 ``dq`` accumulator (B·T·H·128 floats) that key tiles add into with vector reductions."""
    if _needs_padding(q):
        B, T, H, D = q.shape
        T_pad = -(-T // TILE) * TILE
        qp, kp, vp = _pad(q, T_pad), _pad(k, T_pad), _pad(v, T_pad)
        lse_p = lse.new_zeros((B, H, T_pad))  # padded query rows have zero dO, so any finite statistic gives zero gradients
        lse_p[:, :, :T].copy_(lse)
        dqp, dkp, dvp = torch.empty_like(qp), torch.empty_like(kp), torch.empty_like(vp)
        backward(_pad(do, T_pad), qp, kp, vp, _pad(o, T_pad), lse_p, dqp, dkp, dvp, causal, scale, doc_start=_pad_doc_start(doc_start, T_pad))
        dq.copy_(dqp[:, :T, :, :D])
        dk.copy_(dkp[:, :T, :, :D])
        dv.copy_(dvp[:, :T, :, :D])
        return
    B, T, H, D = q.shape
    Hkv = k.shape[2]
    delta = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    dq_acc = torch.empty((B, T, H, D), dtype=torch.float32, device=q.device)
    rc = lib().ob_attention_bwd(
        ptr(do), ptr(q), ptr(k), ptr(v), ptr(o), ptr(lse), ptr(dq), ptr(dk), ptr(dv), ptr(delta), ptr(dq_acc),
        c_int(B), c_int(T), c_int(H), c_int(Hkv),
        *(c_int(s) for s in _strides(do)), *(c_int(s) for s in _strides(q)), *(c_int(s) for s in _strides(k)),
        *(c_int(s) for s in _strides(v)), *(c_int(s) for s in _strides(o)), *(c_int(s) for s in _strides(dq)),
        *(c_int(s) for s in _strides(dk)), *(c_int(s) for s in _strides(dv)),
        c_float(scale), c_int(int(causal)), ptr(status_tensor(q.device)), ptr(doc_start), stream_ptr(),
    )
    check(rc, "ob_attention_bwd", kernels=3)


def supports_varlen(q: torch.Tensor, k: torch.Tensor, causal: bool, dropout_p: float) -> bool:
    """Packed sequences ``(total_tokens, H, D)``: covered (through the document-masking kernels) when the single long
    row they form meets the kernel's shape rules and attention is causal."""
    return causal and q.dim() == 3 and supports(q[None], k[None], causal, dropout_p, False) and supports_backward(q[None], k[None], causal)


class _PackedAttention(torch.autograd.Function):
    """Causal attention over one packed row with per-token document starts."""

    @staticmethod
    def forward(ctx, q, k, v, doc_start, scale):
        o, lse = forward(q, k, v, True, scale, doc_start=doc_start)
        ctx.save_for_backward(q, k, v, o, lse, doc_start)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, doc_start = ctx.saved_tensors
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        backward(do.contiguous(), q, k, v, o, lse, dq, dk, dv, True, ctx.scale, doc_start=doc_start)
        return dq, dk, dv, None, None


def varlen(q, k, v, cu_seqlens, max_seqlen, causal, scale):
    """Intra-document causal attention over packed ``(total_tokens, H, D)`` tensors described by cumulative lengths:
    the pack is one row of ``total_tokens`` positions whose queries see the keys of their own document only (the
    kernels skip key tiles that lie wholly before a query tile's first document)."""
    assert causal, "packed sequences are covered for causal attention"
    total = q.shape[0]
    scale = scale if scale is not None else 1.0 / (q.shape[-1] ** 0.5)
    doc_start = doc_start_from_cu(cu_seqlens, 1, total)
    return _PackedAttention.apply(q[None].contiguous(), k[None].contiguous(), v[None].contiguous(), doc_start, scale)[0]
