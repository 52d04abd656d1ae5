"""
Weight-only quantised linear layers with 2-, 3-, 4- or 8-bit weights and 16-bit activations (``csrc/wna16.cu``).

The 4-bit layer with its tensor-core paths is :class:`olmo_b200.inference.w4a16.QuantLinear`; this module covers the other
widths of the reference's vendored AutoGPTQ kernels (``autogptq_cuda_kernel_256.cu``: vector-matrix products for 2, 3, 4
and 8 bits).  Storage: a row of ``K`` weights is a little-endian bit stream (weight ``k`` in bits ``[k*B, (k+1)*B)``) in
int32 words, ``qweight [N, K*B/32]``; ``scales [N, K/G]`` bf16 and ``zeros [N, K/G]`` uint8 per group of ``G`` columns.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn

__all__ = ["pack_bits", "unpack_bits", "quantize_groups_bits", "BitsLinear", "SUPPORTED_BITS"]

SUPPORTED_BITS = (2, 3, 4, 8)


def pack_bits(q: torch.Tensor, bits: int) -> torch.Tensor:
    """``[N, K]`` integers in ``0 .. 2**bits - 1`` -> ``[N, K*bits/32] int32`` bit stream (``K`` a multiple of 32)."""
    assert bits in SUPPORTED_BITS and q.shape[1] % 32 == 0
    n, k = q.shape
    # expand every weight into its bits (least significant first), then fold 32 bits into a word
    shifts = torch.arange(bits, device=q.device, dtype=torch.int64)
    stream = ((q.to(torch.int64).unsqueeze(-1) >> shifts) & 1).reshape(n, k * bits // 32, 32)
    words = (stream << torch.arange(32, device=q.device, dtype=torch.int64)).sum(dim=-1)
    words = torch.where(words >= 2**31, words - 2**32, words)  # two's complement into int32
    return words.to(torch.int32)


def unpack_bits(qweight: torch.Tensor, bits: int) -> torch.Tensor:
    """Inverse of :func:`pack_bits`: ``[N, K*bits/32] int32`` -> ``[N, K] uint8``."""
    assert bits in SUPPORTED_BITS
    n = qweight.shape[0]
    w = qweight.to(torch.int64) & 0xFFFFFFFF
    stream = ((w.unsqueeze(-1) >> torch.arange(32, device=qweight.device, dtype=torch.int64)) & 1).reshape(n, -1, bits)
    vals = (stream << torch.arange(bits, device=qweight.device, dtype=torch.int64)).sum(dim=-1)
    return vals.to(torch.uint8)


def quantize_groups_bits(w: torch.Tensor, group: int, bits: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Round-to-nearest asymmetric grid per group of ``group`` columns: ``(q [N, K] uint8, scales [N, K/G], zeros [N, K/G])``."""
    n, k = w.shape
    top = float(2**bits - 1)
    g = w.float().reshape(n, k // group, group)
    lo = g.amin(dim=-1).clamp(max=0.0)
    hi = g.amax(dim=-1).clamp(min=0.0)
    scales = torch.where(hi == lo, torch.ones_like(hi), (hi - lo) / top)
    zeros = torch.round(-lo / scales).clamp(0, top)
    q = torch.round(g / scales.unsqueeze(-1) + zeros.unsqueeze(-1)).clamp(0, top).reshape(n, k).to(torch.uint8)
    return q, scales, zeros


class BitsLinear(nn.Module):
    """``nn.Linear`` replacement holding ``bits``-wide weights (2, 3, 4 or 8)."""

    def __init__(self, in_features: int, out_features: int, bits: int, group: int = 128, bias: bool = False):
        super().__init__()
        assert bits in SUPPORTED_BITS and group % 32 == 0 and in_features % group == 0
        self.in_features, self.out_features, self.bits, self.group = in_features, out_features, bits, group
        self.register_buffer("qweight", torch.zeros(out_features, in_features * bits // 32, dtype=torch.int32))
        self.register_buffer("scales", torch.ones(out_features, in_features // group, dtype=torch.bfloat16))
        self.register_buffer("zeros", torch.zeros(out_features, in_features // group, dtype=torch.uint8))
        self.bias = nn.Parameter(torch.zeros(out_features), requires_grad=False) if bias else None

    @classmethod
    def from_linear_rtn(cls, linear: nn.Linear, bits: int, group: int = 128) -> "BitsLinear":
        out = cls(linear.in_features, linear.out_features, bits, group, bias=linear.bias is not None)
        q, scales, zeros = quantize_groups_bits(linear.weight.detach(), group, bits)
        out.qweight.copy_(pack_bits(q, bits))
        out.scales.copy_(scales.to(torch.bfloat16))
        out.zeros.copy_(zeros.to(torch.uint8))
        if linear.bias is not None:
            out.bias.data.copy_(linear.bias.detach())
        return out.to(linear.weight.device)

    def dequantize(self) -> torch.Tensor:
        """Reconstructed ``[N, K]`` weights: bf16 from the kernel on CUDA, fp32 from plain tensor ops on the CPU."""
        if self.qweight.is_cuda:
            from ..ops import check, lib, ptr, stream_ptr

            out = torch.empty(self.out_features, self.in_features, dtype=torch.bfloat16, device=self.qweight.device)
            check(lib().ob_wna16_dequant(ptr(self.qweight), ptr(self.scales), ptr(self.zeros), ptr(out), self.out_features,
                                         self.in_features, self.group, self.bits, stream_ptr()), "ob_wna16_dequant")
            return out
        q = unpack_bits(self.qweight, self.bits).float().reshape(self.out_features, -1, self.group)
        return ((q - self.zeros.float().unsqueeze(-1)) * self.scales.float().unsqueeze(-1)).reshape(self.out_features, self.in_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        if not x2.is_cuda:
            y = (x2.float() @ self.dequantize().t()).to(x.dtype)
        else:
            from ..ops import check, lib, ptr, stream_ptr
            from ..ops import kernels as k

            xb = x2.to(torch.bfloat16).contiguous()
            m = xb.shape[0]
            if m <= 64:  # decode: the packed weights are streamed once per group of up to eight rows
                y = torch.empty(m, self.out_features, dtype=torch.bfloat16, device=x.device)
                for lo in range(0, m, 8):
                    rows = min(8, m - lo)
                    check(lib().ob_wna16_gemv(ptr(xb[lo:]), ptr(self.qweight), ptr(self.scales), ptr(self.zeros), ptr(y[lo:]), rows,
                                              self.out_features, self.in_features, self.group, self.bits, stream_ptr()), "ob_wna16_gemv")
            else:  # prefill: reconstruct once, then the tcgen05 GEMM
                y = k.gemm(xb, self.dequantize())
            y = y.to(x.dtype)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.reshape(*lead, self.out_features)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bits={self.bits}, group={self.group}"
