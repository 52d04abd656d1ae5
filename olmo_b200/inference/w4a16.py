"""
4-bit weight / 16-bit activation linear layer.

Storage (see ``csrc/w4a16.cu``): ``qweight [N, K/8] int32``, ``scales [N, K/G] bf16``, ``zeros [N, K/G] uint8`` and an
optional activation-order permutation ``perm [K] int32``.  On a CUDA device up to 8 tokens go through the dequantising
GEMV kernel (decode); larger batches reconstruct the bf16 matrix into a scratch buffer and run the tcgen05 GEMM (prefill).
On the CPU the C++ reference computes in fp32.  Reference counterpart: the ``QuantLinear`` modules of the vendored
AutoGPTQ under ``inference/compression/dependencies``.
"""
from __future__ import annotations

import ctypes

from typing import Optional, Tuple

import torch
import torch.nn as nn

__all__ = ["pack_int4", "unpack_int4", "quantize_groups", "QuantLinear"]

_SHIFTS = torch.arange(0, 32, 4, dtype=torch.int64)


def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """``[N, K]`` integers in 0..15 -> ``[N, K/8] int32`` (entry i of a word in bits 4i..4i+3)."""
    n, k = q.shape
    assert k % 8 == 0
    words = (q.to(torch.int64).reshape(n, k // 8, 8) << _SHIFTS.to(q.device)).sum(dim=-1)
    words = torch.where(words >= 2**31, words - 2**32, words)  # two's complement into int32
    return words.to(torch.int32)


def unpack_int4(qweight: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`pack_int4`: ``[N, K/8] int32`` -> ``[N, K] uint8``."""
    w = qweight.to(torch.int64) & 0xFFFFFFFF
    return ((w.unsqueeze(-1) >> _SHIFTS.to(qweight.device)) & 0xF).reshape(qweight.shape[0], -1).to(torch.uint8)


def quantize_groups(w: torch.Tensor, group: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Asymmetric 4-bit grid per group of ``group`` columns: returns ``(scales [N, K/G], zeros [N, K/G])`` in fp32."""
    n, k = w.shape
    g = w.float().reshape(n, k // group, group)
    lo = g.amin(dim=-1).clamp(max=0.0)
    hi = g.amax(dim=-1).clamp(min=0.0)
    flat = hi == lo
    scales = torch.where(flat, torch.ones_like(hi), (hi - lo) / 15.0)
    zeros = torch.round(-lo / scales).clamp(0, 15)
    return scales, zeros


class _QuantMatmul(torch.autograd.Function):
    """``x · Wᵀ`` through the quantised kernels with a gradient for ``x`` (the packed weights are constants)."""

    @staticmethod
    def forward(ctx, x2: torch.Tensor, layer: "QuantLinear") -> torch.Tensor:  # type: ignore[override]
        ctx.layer = layer
        return layer._matmul(x2)

    @staticmethod
    def backward(ctx, dy: torch.Tensor):  # type: ignore[override]
        return ctx.layer._input_gradient(dy).to(dy.dtype), None


class QuantLinear(nn.Module):
    """Drop-in replacement of a bias-free or biased ``nn.Linear`` holding 4-bit weights."""

    def __init__(self, in_features: int, out_features: int, group: int = 128, bias: bool = False, act_order: bool = False):
        super().__init__()
        assert in_features % group == 0 and group % 32 == 0, "K must be a multiple of the group size and the group of 32"
        self.in_features, self.out_features, self.group = in_features, out_features, group
        self.register_buffer("qweight", torch.zeros(out_features, in_features // 8, dtype=torch.int32))
        self.register_buffer("scales", torch.ones(out_features, in_features // group, dtype=torch.bfloat16))
        self.register_buffer("zeros", torch.zeros(out_features, in_features // group, dtype=torch.uint8))
        self.register_buffer("perm", torch.arange(in_features, dtype=torch.int32) if act_order else None)
        self.register_buffer("bias", torch.zeros(out_features, dtype=torch.bfloat16) if bias else None)
        self._scratch: Optional[torch.Tensor] = None

    # -- construction ----------------------------------------------------------------------------

    @classmethod
    def from_quantized(
        cls, q: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, group: int, perm: Optional[torch.Tensor] = None,
        bias: Optional[torch.Tensor] = None,
    ) -> "QuantLinear":
        """``q [N, K]`` integer codes in *stored* (permuted) column order."""
        n, k = q.shape
        layer = cls(k, n, group=group, bias=bias is not None, act_order=perm is not None)
        layer.qweight.copy_(pack_int4(q))
        layer.scales.copy_(scales.to(torch.bfloat16))
        layer.zeros.copy_(zeros.to(torch.uint8))
        if perm is not None:
            layer.perm.copy_(perm.to(torch.int32))
        if bias is not None:
            layer.bias.copy_(bias.to(torch.bfloat16))
        return layer

    @classmethod
    def from_linear_rtn(cls, linear: nn.Linear, group: int = 128) -> "QuantLinear":
        """Round-to-nearest quantisation of an existing layer (no calibration data)."""
        w = linear.weight.detach().float()
        scales, zeros = quantize_groups(w, group)
        # the kernels use bf16 scales: round the codes against the scales that will actually be applied
        s_used = scales.to(torch.bfloat16).float()
        q = torch.round(w.reshape(w.shape[0], -1, group) / s_used.unsqueeze(-1) + zeros.unsqueeze(-1)).clamp(0, 15).reshape_as(w)
        return cls.from_quantized(q, s_used, zeros, group, bias=None if linear.bias is None else linear.bias.detach())

    # -- maths -----------------------------------------------------------------------------------

    def dequantize(self) -> torch.Tensor:
        """Reconstructed weights ``[N, K]`` in the layer's stored column order (bf16 on CUDA, fp32 on CPU)."""
        if self.qweight.is_cuda:
            from ..ops import check, lib, ptr, stream_ptr

            out = torch.empty(self.out_features, self.in_features, dtype=torch.bfloat16, device=self.qweight.device)
            check(lib().ob_w4a16_dequant(ptr(self.qweight), ptr(self.scales), ptr(self.zeros), ptr(out), self.out_features, self.in_features,
                                         self.group, stream_ptr()), "ob_w4a16_dequant")
            return out
        from . import cpu_ref

        return cpu_ref.dequant(self.qweight, self.scales.float(), self.zeros, self.group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        # the kernels know nothing of autograd: when the input needs a gradient (adapters or prompts trained on top of a
        # quantised model) the product runs inside a Function whose backward multiplies by the reconstructed weights
        y = _QuantMatmul.apply(x2, self) if x2.requires_grad and torch.is_grad_enabled() else self._matmul(x2)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.reshape(*lead, self.out_features)

    def _input_gradient(self, dy: torch.Tensor) -> torch.Tensor:
        """``dy[M, N] · W`` in the input's own column order (``transpose_quant_matmul`` of the reference's Triton kernels,
        ``auto_gptq/nn_modules/triton_utils/kernels.py:186-278``): reconstruct once, one GEMM, undo the activation order."""
        w = self.dequantize()
        if dy.is_cuda and self.in_features % 8 == 0 and self.out_features % 8 == 0:
            from ..ops import kernels as k

            dx = k.gemm(dy.to(torch.bfloat16).contiguous(), w, b_trans=True)
        else:
            dx = dy.to(w.dtype) @ w
        if self.perm is not None:  # forward read column perm[j] of the input as stored column j
            dx = torch.empty_like(dx).index_copy_(1, self.perm.long(), dx)
        return dx

    def _matmul(self, x2: torch.Tensor) -> torch.Tensor:
        x = x2
        if not x2.is_cuda:
            from . import cpu_ref

            y = cpu_ref.matmul(x2, self.qweight, self.scales.float(), self.zeros, self.group, self.perm).to(x.dtype)
        else:
            from ..ops import check, lib, ptr, stream_ptr
            from ..ops import kernels as k

            xb = x2.to(torch.bfloat16).contiguous()
            if self.perm is not None:
                gathered = torch.empty_like(xb)
                check(lib().ob_gather_columns_bf16(ptr(xb), ptr(self.perm), ptr(gathered), xb.shape[0], self.in_features, stream_ptr()),
                      "ob_gather_columns_bf16")
                xb = gathered
            m = xb.shape[0]
            fused_ok = 8 < m <= 256 and lib().ob_w4a16_gemm_small_supported(m, self.out_features, self.in_features, self.group)
            if fused_ok:
                # decode batches: dequantisation fused into the operand staging of a tcgen05 GEMM; the packed weights
                # are read once and no bf16 copy of the matrix is written
                from ..ops import status_tensor

                y = torch.empty(m, self.out_features, dtype=torch.bfloat16, device=x.device)
                # layers with few 128-feature tiles split K over several CTAs, which add into a zeroed fp32 buffer
                splits = lib().ob_w4a16_gemm_small_splits(self.out_features, self.in_features)
                partial = torch.zeros(m, self.out_features, dtype=torch.float32, device=x.device) if splits > 1 else None
                check(lib().ob_w4a16_gemm_small(ptr(xb), ptr(self.qweight), ptr(self.scales), ptr(self.zeros), ptr(y), ptr(partial), m,
                                                self.out_features, self.in_features, self.group, splits, ptr(status_tensor(x.device)),
                                                stream_ptr()), "ob_w4a16_gemm_small")
                if partial is not None:
                    check(lib().ob_cast_f32_to_bf16(ptr(partial), ptr(y), ctypes.c_longlong(partial.numel()), stream_ptr()), "ob_cast_f32_to_bf16")
            elif m <= 64:
                # the matrix-vector kernel takes up to 8 rows per launch and reads the packed weights once per launch
                # (0.5 byte per weight), so up to 64 rows cost less traffic than reconstructing the matrix (2.5 bytes
                # per weight) and multiplying it (2 more)
                y = torch.empty(m, self.out_features, dtype=torch.bfloat16, device=x.device)
                for lo in range(0, m, 8):
                    rows = min(8, m - lo)
                    check(lib().ob_w4a16_gemv(ptr(xb[lo:]), ptr(self.qweight), ptr(self.scales), ptr(self.zeros), ptr(y[lo:]), rows,
                                              self.out_features, self.in_features, self.group, stream_ptr()), "ob_w4a16_gemv")
            else:
                y = k.gemm(xb, self.dequantize())
            y = y.to(x.dtype)
        return y

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, group={self.group}, act_order={self.perm is not None}"
