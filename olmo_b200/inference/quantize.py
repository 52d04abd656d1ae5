"""
Post-training 4-bit quantisation of an OLMo model (weights only; activations stay bf16).

``quantize_model`` walks the blocks in order.  For every block it records the inputs of its four linear layers
(``att_proj``, ``attn_out``, ``ff_proj``, ``ff_out``) on calibration text, quantises them — round-to-nearest, or GPTQ
(Frantar et al., 2022: column-by-column rounding with second-order error feedback, optional activation ordering) — swaps
in :class:`QuantLinear` modules and recomputes the block output so that later blocks calibrate on what they will really
see.  Reference counterpart: ``inference/compression/run_quantization.py`` + ``olmo_gptq_class.py`` (4 bit, group 128,
128 calibration samples) on top of the vendored AutoGPTQ.
"""
from __future__ import annotations

import logging
from typing import Any, Dict, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from .w4a16 import QuantLinear, quantize_groups

__all__ = ["BLOCK_LINEARS", "gptq_quantize_weight", "quantize_linear", "quantize_model", "quantized_state_summary"]

log = logging.getLogger(__name__)

#: the linears inside a block, in execution order
BLOCK_LINEARS = ("att_proj", "attn_out", "ff_proj", "ff_out")


def _grid(w: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    return torch.round(w / scale + zero).clamp(0, 15)


@torch.no_grad()
def gptq_quantize_weight(
    weight: torch.Tensor, hessian: torch.Tensor, group: int = 128, act_order: bool = True, percdamp: float = 0.01, blocksize: int = 128,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """
    GPTQ for one ``[N, K]`` matrix given ``H = Σ xᵀx`` (``[K, K]``).  Returns ``(codes [N, K], scales, zeros, perm)`` with
    codes in stored column order (``perm`` maps stored column j to original column ``perm[j]``; ``None`` without act-order).
    """
    W = weight.detach().float().clone()
    H = hessian.detach().float().clone()
    n, k = W.shape
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    perm = None
    if act_order:
        perm = torch.argsort(torch.diag(H), descending=True)
        W, H = W[:, perm], H[perm][:, perm]
    damp = percdamp * torch.mean(torch.diag(H))
    H.diagonal().add_(damp)
    L = torch.linalg.cholesky(H)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(L), upper=True)

    Q = torch.zeros_like(W)
    scales = torch.zeros(n, k // group, device=W.device)
    zeros = torch.zeros(n, k // group, device=W.device)
    for start in range(0, k, blocksize):
        end = min(start + blocksize, k)
        Wb = W[:, start:end].clone()
        Err = torch.zeros_like(Wb)
        Hb = Hinv[start:end, start:end]
        for i in range(end - start):
            col = start + i
            if col % group == 0:
                s, z = quantize_groups(W[:, col : col + group], group)
                s = s.to(torch.bfloat16).float()  # the kernels hold bf16 scales
                scales[:, col // group], zeros[:, col // group] = s[:, 0], z[:, 0]
            s, z = scales[:, col // group], zeros[:, col // group]
            w = Wb[:, i]
            q = _grid(w, s, z)
            Q[:, col] = q
            err = (w - (q - z) * s) / Hb[i, i]
            Wb[:, i:] -= err.unsqueeze(1) * Hb[i, i:].unsqueeze(0)
            Err[:, i] = err
        W[:, start:end] = Wb
        W[:, end:] -= Err @ Hinv[start:end, end:]
    return Q, scales, zeros, perm


@torch.no_grad()
def quantize_linear(linear: nn.Linear, hessian: Optional[torch.Tensor], group: int = 128, act_order: bool = True, method: str = "gptq") -> QuantLinear:
    if method == "rtn" or hessian is None:
        return QuantLinear.from_linear_rtn(linear, group).to(linear.weight.device)
    q, s, z, perm = gptq_quantize_weight(linear.weight, hessian, group=group, act_order=act_order)
    layer = QuantLinear.from_quantized(q, s, z, group, perm=perm, bias=None if linear.bias is None else linear.bias.detach())
    return layer.to(linear.weight.device)


class _Stop(Exception):
    pass


@torch.no_grad()
def quantize_model(
    model: nn.Module, calibration: Sequence[torch.Tensor], *, group: int = 128, act_order: bool = True, method: str = "gptq",
    linears: Iterable[str] = BLOCK_LINEARS,
) -> Dict[str, float]:
    """
    Quantise every block of an :class:`olmo_b200.models.olmo.OLMo` in place.  ``calibration`` is a list of ``[B, T]`` token
    tensors.  Returns the relative output error ``‖y_q − y‖ / ‖y‖`` of every replaced layer on the calibration inputs.
    """
    blocks: List[nn.Module] = list(model.all_blocks()) if hasattr(model, "all_blocks") else list(model.transformer.blocks)
    device = next(model.parameters()).device
    was_training = model.training
    model.eval()

    # 1. inputs (and keyword arguments) of the first block
    captured: List[Tuple[torch.Tensor, Dict[str, Any]]] = []

    def grab(_module, args, kwargs):
        captured.append((args[0].detach(), {k: v for k, v in kwargs.items() if k not in ("layer_past", "use_cache")}))
        raise _Stop

    handle = blocks[0].register_forward_pre_hook(grab, with_kwargs=True)
    for ids in calibration:
        try:
            model(ids.to(device))
        except _Stop:
            pass
    handle.remove()

    report: Dict[str, float] = {}
    states = captured
    for index, block in enumerate(blocks):
        names = [n for n in linears if isinstance(getattr(block, n, None), nn.Linear)]
        sums: Dict[str, torch.Tensor] = {}
        kept_in: Dict[str, List[torch.Tensor]] = {n: [] for n in names}

        def make_hook(name: str):
            def hook(_m, args):
                x = args[0].detach().reshape(-1, args[0].shape[-1]).float()
                sums[name] = sums.get(name, 0) + x.t() @ x
                if len(kept_in[name]) < 2:
                    kept_in[name].append(x[:256].clone())
            return hook

        # a block with packed 4-bit linears runs through its modules, never through the fused training kernels
        # (which read dense weights), and the statistics hooks below only fire on the module path
        block._fused_ok = False
        hooks = [getattr(block, n).register_forward_pre_hook(make_hook(n)) for n in names]
        for x, kw in states:
            block(x, **kw)
        for h in hooks:
            h.remove()
        for name in names:
            old = getattr(block, name)
            new = quantize_linear(old, sums.get(name), group=group, act_order=act_order, method=method)
            if kept_in[name]:
                probe = torch.cat(kept_in[name]).to(old.weight.dtype)
            else:  # no calibration inputs (round-to-nearest needs none): report the error on unit-variance noise
                probe = torch.randn(64, old.in_features, device=old.weight.device, dtype=old.weight.dtype,
                                    generator=torch.Generator(device=old.weight.device).manual_seed(index))
            want = old(probe).float()
            got = new(probe).float()
            report[f"blocks.{index}.{name}"] = float((got - want).norm() / want.norm().clamp_min(1e-12))
            setattr(block, name, new)
            if hasattr(block, "fused_dims") and name == "att_proj":
                pass  # the split of the fused projection depends on output widths only, which did not change
        # 2. outputs of the quantised block feed the next one
        next_states = []
        for x, kw in states:
            out = block(x, **kw)
            next_states.append(((out[0] if isinstance(out, tuple) else out).detach(), kw))
        states = next_states
        log.info("block %d quantised: %s", index, {n: round(report[f'blocks.{index}.{n}'], 4) for n in names})
    model.train(was_training)
    return report


def quantized_state_summary(model: nn.Module) -> Dict[str, float]:
    """Bytes held by quantised vs. full-precision parameters and buffers (for a before/after size report)."""
    q_bytes = fp_bytes = 0
    for module in model.modules():
        if isinstance(module, QuantLinear):
            q_bytes += sum(b.numel() * b.element_size() for b in module.buffers(recurse=False))
        else:
            fp_bytes += sum(p.numel() * p.element_size() for p in module.parameters(recurse=False))
    return {"quantized_bytes": q_bytes, "full_precision_bytes": fp_bytes, "total_gib": (q_bytes + fp_bytes) / 2**30}
