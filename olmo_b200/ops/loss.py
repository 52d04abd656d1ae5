"""
Loss operators.

* :func:`cross_entropy_loss` — portable CE + optional z-loss (reference ``olmo/train.py:124-145``).
* :func:`fused_cross_entropy` — the same through the sm_100a kernel with an autograd wrapper
  (replaces the Triton CE the reference takes from flash-attn, ``olmo/train.py:148-205``).
* :func:`lm_head_loss` — LM-head GEMM, CE/z-loss and both head gradients in row chunks, so that
  neither fp32 logits nor the full bf16 logits tensor ever exist (used by the manual training path).
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.nn.functional as F

from . import kernels as k

__all__ = ["cross_entropy_loss", "fused_cross_entropy", "lm_head_loss"]


def cross_entropy_loss(
    logits: torch.Tensor,
    labels: torch.Tensor,
    ignore_index: int = -100,
    reduction: str = "mean",
    compute_z_loss: bool = False,
    z_loss_multiplier: float = 1e-4,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """CE over ``(N, V)`` logits; the z-loss is ``multiplier · logsumexp(logits)²`` over non-ignored rows,
    reduced the same way as the CE."""
    loss = F.cross_entropy(logits, labels, ignore_index=ignore_index, reduction=reduction)
    if not compute_z_loss:
        return loss, None
    z_sq = logits.logsumexp(-1).pow(2)
    mask = labels != ignore_index
    if reduction == "mean":
        z_sq = (z_sq * mask).sum() / mask.sum()
    elif reduction == "sum":
        z_sq = (z_sq * mask).sum()
    return loss, z_loss_multiplier * z_sq


class _FusedCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, ignore_index, z_mult, want_z):
        # gradient is produced in the same pass, into a private copy when the caller still needs the logits
        work = logits if not logits.requires_grad else logits.detach().clone()
        ce, z = k.cross_entropy_(work, labels, ignore_index, z_mult if want_z else 0.0, 1.0, write_grad=logits.requires_grad, want_z=want_z)
        ctx.save_for_backward(work if logits.requires_grad else None)
        ctx.mark_non_differentiable(labels)
        return ce, (z if want_z else ce.new_zeros(()))

    @staticmethod
    def backward(ctx, d_ce, d_z):
        (dlogits,) = ctx.saved_tensors
        # callers reduce with a plain sum / mean, so d_ce is one scalar broadcast over rows
        scale = d_ce.reshape(-1)[:1].to(dlogits.dtype) if d_ce.numel() > 0 else None
        if d_ce.numel() > 1 and not torch.all(d_ce == d_ce.reshape(-1)[0]):
            dlogits = dlogits * d_ce.unsqueeze(-1).to(dlogits.dtype)
        elif scale is not None:
            dlogits = dlogits * scale
        return dlogits, None, None, None, None


def fused_cross_entropy(
    logits: torch.Tensor,
    labels: torch.Tensor,
    ignore_index: int = -100,
    reduction: str = "mean",
    compute_z_loss: bool = False,
    z_loss_multiplier: float = 1e-4,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Kernel-backed CE (+ z-loss) for bf16 CUDA logits; same contract as :func:`cross_entropy_loss`.

    The z-loss gradient is folded into the CE gradient inside the kernel, so the returned z term is detached.
    """
    if not (logits.is_cuda and logits.dtype == torch.bfloat16):
        return cross_entropy_loss(logits, labels, ignore_index, reduction, compute_z_loss, z_loss_multiplier)
    ce, zsq = _FusedCE.apply(logits.contiguous(), labels, ignore_index, z_loss_multiplier, compute_z_loss)
    n_valid = (labels != ignore_index).sum().clamp(min=1)
    if reduction == "mean":
        loss, z = ce.sum() / n_valid, (zsq.sum() / n_valid if compute_z_loss else None)
    elif reduction == "sum":
        loss, z = ce.sum(), (zsq.sum() if compute_z_loss else None)
    else:
        loss, z = ce, (zsq if compute_z_loss else None)
    return loss, (z_loss_multiplier * z.detach() if z is not None else None)


def lm_head_loss(
    xn: torch.Tensor,
    weight: torch.Tensor,
    labels: torch.Tensor,
    *,
    ignore_index: int = -100,
    z_mult: float = 0.0,
    grad_scale: float = 1.0,
    logit_scale: float = 1.0,
    chunk_rows: int = 4096,
    wgrad: Optional[Callable[[torch.Tensor, torch.Tensor], None]] = None,
    need_grad: bool = True,
    gemm_kwargs: Optional[dict] = None,
) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """
    ``xn`` ``[M, d]`` bf16 (final-norm output), ``weight`` ``[V, d]`` bf16, ``labels`` ``[M]``.

    Returns ``(Σ CE, Σ lse², d xn)``; the gradient of ``grad_scale · (ΣCE + z_mult·Σlse²)`` w.r.t. the weight is
    handed to ``wgrad(dlogits_chunk, xn_chunk)`` chunk by chunk.
    """
    M, d = xn.shape
    ce_sum = torch.zeros((), dtype=torch.float32, device=xn.device)
    z_sum = torch.zeros((), dtype=torch.float32, device=xn.device)
    dxn = torch.empty_like(xn) if need_grad else None
    gk = gemm_kwargs or {}
    for r0 in range(0, M, chunk_rows):
        r1 = min(M, r0 + chunk_rows)
        xc = xn[r0:r1]
        logits = k.gemm(xc, weight, **gk)
        if logit_scale != 1.0:
            logits.mul_(logit_scale)
        ce, z = k.cross_entropy_(logits, labels[r0:r1], ignore_index, z_mult, grad_scale * 1.0, write_grad=need_grad, want_z=True)
        ce_sum += ce.sum()
        z_sum += z.sum()
        if need_grad:
            if logit_scale != 1.0:
                logits.mul_(logit_scale)
            k.gemm(logits, weight, b_trans=True, out=dxn[r0:r1])
            if wgrad is not None:
                wgrad(logits, xc)
        del logits
    return ce_sum, z_sum, dxn
