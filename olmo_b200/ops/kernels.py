"""
Thin Python wrappers over the C interface of ``_kernels.so`` (one function per exported symbol).

Each wrapper validates dtypes / contiguity, allocates outputs with torch's caching allocator, and
launches on the current stream.  Shapes use M for token rows, D for the model width.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_longlong
from typing import Optional, Tuple

import torch

from . import check, launch_count, lib, ptr, status_tensor, stream_ptr  # noqa: F401

EPI_BF16, EPI_F32_ACCUM, EPI_BF16_ADD, EPI_F32_STORE = 0, 1, 2, 3

_NUM_SMS = {}


def num_sms() -> int:
    d = torch.cuda.current_device()
    if d not in _NUM_SMS:
        _NUM_SMS[d] = torch.cuda.get_device_properties(d).multi_processor_count
    return _NUM_SMS[d]


def _bf16(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.bfloat16 or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA bf16 tensor, got {t.dtype} on {t.device}")


# ----------------------------------------------------------------------------------------- GEMM


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    *,
    a_trans: bool = False,
    b_trans: bool = False,
    out: Optional[torch.Tensor] = None,
    epilogue: int = EPI_BF16,
    residual: Optional[torch.Tensor] = None,
    b_ready: Optional[torch.Tensor] = None,
    rows_per_flag: int = 0,
    ready_value: int = 0,
    sms: int = 0,
    comm=None,
) -> torch.Tensor:
    """
    ``out[M, N] = op(a) @ op(b)ᵀ`` with fp32 accumulation on tcgen05 tensor cores.

    * ``a_trans=False``: ``a`` is ``[M, K]`` (K contiguous); ``a_trans=True``: ``a`` is ``[K, M]``.
    * ``b_trans=False``: ``b`` is ``[N, K]`` (a Linear weight);  ``b_trans=True``: ``b`` is ``[K, N]``.

    So a Linear forward is ``gemm(x, W)``, its input gradient ``gemm(dy, W, b_trans=True)`` and its weight
    gradient ``gemm(dy, x, a_trans=True, b_trans=True, epilogue=EPI_F32_ACCUM, out=grad)``.
    Operands may be row-strided views (last dimension contiguous, pitch a multiple of 8 elements).
    ``comm=(task, n_ctas)`` makes the first ``n_ctas`` blocks of the launch execute a peer-memory collective
    (:class:`olmo_b200.parallel.peer.CommTask`) while the others compute.
    """
    _bf16(a, "a")
    _bf16(b, "b")
    assert a.dim() == 2 and b.dim() == 2 and a.stride(1) == 1 and b.stride(1) == 1
    if a_trans:
        K, M = a.shape
    else:
        M, K = a.shape
    if b_trans:
        Kb, N = b.shape
    else:
        N, Kb = b.shape
    assert K == Kb, f"contraction mismatch {K} vs {Kb}"
    out_dtype = torch.bfloat16 if epilogue in (EPI_BF16, EPI_BF16_ADD) else torch.float32
    if out is None:
        assert epilogue != EPI_F32_ACCUM, "accumulating epilogue needs an existing output"
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    assert out.dtype == out_dtype and out.shape == (M, N) and out.stride(1) == 1
    if epilogue == EPI_BF16_ADD:
        assert residual is not None and residual.shape == out.shape and residual.stride() == out.stride()
        _bf16(residual, "residual")
    if comm is not None:
        task, n_ctas = comm
        rc = lib().ob_gemm_bf16_comm(
            ptr(a), ptr(b), ptr(out), ptr(residual),
            c_int(M), c_int(N), c_int(K), c_int(a.stride(0)), c_int(b.stride(0)), c_int(out.stride(0)),
            c_int(int(a_trans)), c_int(int(b_trans)), c_int(epilogue), ptr(status_tensor(a.device)), c_int(sms or num_sms()),
            ctypes.byref(task), c_int(n_ctas), stream_ptr(),
        )
        check(rc, "ob_gemm_bf16_comm")
        return out
    rc = lib().ob_gemm_bf16(
        ptr(a), ptr(b), ptr(out), ptr(residual),
        c_int(M), c_int(N), c_int(K), c_int(a.stride(0)), c_int(b.stride(0)), c_int(out.stride(0)),
        c_int(int(a_trans)), c_int(int(b_trans)), c_int(epilogue),
        ptr(b_ready), c_int(rows_per_flag), c_int(ready_value),
        ptr(status_tensor(a.device)), c_int(sms or num_sms()), stream_ptr(),
    )
    check(rc, "ob_gemm_bf16")
    return out


def gemm_small_m_available() -> bool:
    try:
        return hasattr(lib(), "ob_gemm_smallm")
    except Exception:
        return False


def gemm_small_m(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x[M, K] · w[N, K]ᵀ`` for a decode-sized batch (``1 <= M <= 256``): the weights are streamed once as the
    128-row tensor-core operand and the batch is the narrow one (``csrc/gemm_smallm.cu``).  Returns ``[M, N]`` bf16."""
    _bf16(x, "x")
    _bf16(w, "w")
    assert x.dim() == 2 and w.dim() == 2 and x.stride(1) == 1 and w.stride(1) == 1 and x.shape[1] == w.shape[1]
    M, K = x.shape
    N = w.shape[0]
    assert 1 <= M <= 256
    splits = lib().ob_gemm_smallm_splits(c_int(N), c_int(K), c_int(num_sms()))
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    partial = torch.empty(splits * M * N, dtype=torch.float32, device=x.device) if splits > 1 else None
    rc = lib().ob_gemm_smallm(
        ptr(x), ptr(w), ptr(y), ptr(partial), c_int(M), c_int(N), c_int(K), c_int(x.stride(0)), c_int(w.stride(0)), c_int(splits),
        ptr(status_tensor(x.device)), stream_ptr(),
    )
    check(rc, "ob_gemm_smallm", kernels=2 if splits > 1 else 1)
    return y


# ---------------------------------------------------------------------------------------- norms


def norm_fwd(
    x: torch.Tensor,
    weight: Optional[torch.Tensor],
    bias: Optional[torch.Tensor],
    eps: float,
    rms: bool,
    residual: Optional[torch.Tensor] = None,
    save_stats: bool = True,
) -> Tuple[torch.Tensor, Optional[torch.Tensor], Optional[torch.Tensor]]:
    """``out = [residual +] norm(x) [* weight] [+ bias]`` over the last dimension; returns ``(out, rstd, mean)``."""
    _bf16(x, "x")
    D = x.shape[-1]
    x2 = x.reshape(-1, D)
    assert x2.stride(1) == 1
    M = x2.shape[0]
    out = torch.empty((M, D), dtype=torch.bfloat16, device=x.device)
    rstd = torch.empty(M, dtype=torch.float32, device=x.device) if save_stats else None
    mean = torch.empty(M, dtype=torch.float32, device=x.device) if (save_stats and not rms) else None
    res2 = None
    if residual is not None:
        res2 = residual.reshape(-1, D)
        assert res2.is_contiguous()
    rc = lib().ob_norm_fwd(
        ptr(x2), ptr(res2), ptr(weight), ptr(bias), ptr(out), ptr(rstd), ptr(mean),
        c_int(M), c_int(D), c_int(x2.stride(0)), c_float(eps), c_int(int(rms)), stream_ptr(),
    )
    check(rc, "ob_norm_fwd")
    return out.view(x.shape), rstd, mean


def norm_bwd(
    dy: torch.Tensor,
    x: torch.Tensor,
    weight: Optional[torch.Tensor],
    rstd: torch.Tensor,
    mean: Optional[torch.Tensor],
    rms: bool,
    dres: Optional[torch.Tensor] = None,
    dweight: Optional[torch.Tensor] = None,
    dbias: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Input gradient of :func:`norm_fwd`; accumulates the weight / bias gradients into fp32 ``dweight`` / ``dbias``."""
    D = x.shape[-1]
    dy2, x2 = dy.reshape(-1, D), x.reshape(-1, D)
    assert dy2.is_contiguous() and x2.stride(1) == 1
    M = x2.shape[0]
    dx = torch.empty((M, D), dtype=torch.bfloat16, device=x.device) if out is None else out
    nparts = lib().ob_norm_rows_per_launch(c_int(M))
    dw_part = torch.empty((nparts, D), dtype=torch.float32, device=x.device) if dweight is not None else None
    db_part = torch.empty((nparts, D), dtype=torch.float32, device=x.device) if dbias is not None else None
    dres2 = None if dres is None else dres.reshape(-1, D)
    rc = lib().ob_norm_bwd(
        ptr(dy2), ptr(x2), ptr(weight), ptr(rstd), ptr(mean), ptr(dres2), ptr(dx), ptr(dw_part), ptr(db_part),
        c_int(M), c_int(D), c_int(x2.stride(0)), c_int(dx.stride(0)), c_int(int(rms)), stream_ptr(),
    )
    check(rc, "ob_norm_bwd")
    if dweight is not None:
        check(lib().ob_reduce_rows_f32(ptr(dw_part), c_int(rc), c_int(D), ptr(dweight), c_int(1), stream_ptr()), "reduce")
    if dbias is not None:
        check(lib().ob_reduce_rows_f32(ptr(db_part), c_int(rc), c_int(D), ptr(dbias), c_int(1), stream_ptr()), "reduce")
    return dx


# ------------------------------------------------------------------------------- QK-norm + RoPE


def qk_norm_rope_fwd(
    qkv: torch.Tensor,
    wq: Optional[torch.Tensor],
    wk: Optional[torch.Tensor],
    cos: Optional[torch.Tensor],
    sin: Optional[torch.Tensor],
    seq_len: int,
    Wq: int,
    Wk: int,
    head_dim: int,
    eps: float,
    clip: float,
    do_norm: bool,
    do_rope: bool,
    pos_offset: int = 0,
):
    """See ``csrc/rope.cu``.  ``qkv`` is ``[M, Wq+2Wk]``; returns ``(out, rstd_q, rstd_k)`` where ``out`` is
    ``[M, Wq+Wk]`` (q | k), or ``[M, Wq+2Wk]`` (q | k | clamped v) when ``clip > 0``."""
    _bf16(qkv, "qkv")
    M = qkv.shape[0]
    assert qkv.dim() == 2 and qkv.stride(1) == 1
    qk = torch.empty((M, Wq + Wk + (Wk if clip > 0 else 0)), dtype=torch.bfloat16, device=qkv.device)
    rq = torch.empty(M, dtype=torch.float32, device=qkv.device) if do_norm else None
    rk = torch.empty(M, dtype=torch.float32, device=qkv.device) if do_norm else None
    rc = lib().ob_qk_norm_rope_fwd(
        ptr(qkv), ptr(qk), ptr(wq), ptr(wk), ptr(cos), ptr(sin), ptr(rq), ptr(rk),
        c_int(M), c_int(seq_len), c_int(pos_offset), c_int(Wq), c_int(Wk), c_int(head_dim), c_int(qkv.stride(0)),
        c_int(qk.stride(0)), c_float(eps), c_float(clip), c_int(int(do_norm)), c_int(int(do_rope)), stream_ptr(),
    )
    check(rc, "ob_qk_norm_rope_fwd")
    return qk, rq, rk


def qk_norm_rope_bwd(
    qkv: torch.Tensor,
    dqkv: torch.Tensor,
    wq, wk, cos, sin, rstd_q, rstd_k,
    seq_len: int, Wq: int, Wk: int, head_dim: int, clip: float, do_norm: bool, do_rope: bool,
    dwq: Optional[torch.Tensor] = None,
    dwk: Optional[torch.Tensor] = None,
    pos_offset: int = 0,
) -> torch.Tensor:
    """In place on ``dqkv`` (same layout as ``qkv``); accumulates fp32 ``dwq`` / ``dwk``."""
    M = qkv.shape[0]
    assert dqkv.shape == qkv.shape and dqkv.stride() == qkv.stride()
    nparts = lib().ob_qk_rows_per_launch(c_int(M))
    need_w = do_norm and dwq is not None
    pq = torch.empty((nparts, Wq), dtype=torch.float32, device=qkv.device) if need_w else None
    pk = torch.empty((nparts, Wk), dtype=torch.float32, device=qkv.device) if need_w else None
    rc = lib().ob_qk_norm_rope_bwd(
        ptr(qkv), ptr(dqkv), ptr(wq), ptr(wk), ptr(cos), ptr(sin), ptr(rstd_q), ptr(rstd_k), ptr(pq), ptr(pk),
        c_int(M), c_int(seq_len), c_int(pos_offset), c_int(Wq), c_int(Wk), c_int(head_dim), c_int(qkv.stride(0)),
        c_float(clip), c_int(int(do_norm)), c_int(int(do_rope)), stream_ptr(),
    )
    check(rc, "ob_qk_norm_rope_bwd")
    if need_w:
        check(lib().ob_reduce_rows_f32(ptr(pq), c_int(rc), c_int(Wq), ptr(dwq), c_int(1), stream_ptr()), "reduce")
        check(lib().ob_reduce_rows_f32(ptr(pk), c_int(rc), c_int(Wk), ptr(dwk), c_int(1), stream_ptr()), "reduce")
    return dqkv


# ------------------------------------------------------------------------------------- pointwise


def swiglu_fwd(h: torch.Tensor) -> torch.Tensor:
    _bf16(h, "h")
    H = h.shape[-1] // 2
    h2 = h.reshape(-1, 2 * H)
    assert h2.is_contiguous()
    out = torch.empty((h2.shape[0], H), dtype=torch.bfloat16, device=h.device)
    check(lib().ob_swiglu_fwd(ptr(h2), ptr(out), c_int(h2.shape[0]), c_int(H), stream_ptr()), "ob_swiglu_fwd")
    return out.view(*h.shape[:-1], H)


def swiglu_bwd(dout: torch.Tensor, h: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    H = h.shape[-1] // 2
    h2, d2 = h.reshape(-1, 2 * H), dout.reshape(-1, H)
    assert h2.is_contiguous() and d2.is_contiguous()
    dh = torch.empty_like(h2) if out is None else out
    check(lib().ob_swiglu_bwd(ptr(d2), ptr(h2), ptr(dh), c_int(h2.shape[0]), c_int(H), stream_ptr()), "ob_swiglu_bwd")
    return dh.view(h.shape)


def embedding_fwd(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    _bf16(table, "table")
    assert ids.dtype == torch.int64 and table.is_contiguous()
    flat = ids.reshape(-1).contiguous()
    V, D = table.shape
    out = torch.empty((flat.numel(), D), dtype=torch.bfloat16, device=table.device)
    check(lib().ob_embedding_fwd(ptr(flat), ptr(table), ptr(out), c_int(flat.numel()), c_int(D), c_int(V), stream_ptr()), "ob_embedding_fwd")
    return out.view(*ids.shape, D)


def embedding_bwd(ids: torch.Tensor, dout: torch.Tensor, grad: torch.Tensor) -> None:
    """``grad[ids] += dout`` with ``grad`` an fp32 ``[V, D]`` accumulator."""
    assert grad.dtype == torch.float32 and grad.is_contiguous()
    flat = ids.reshape(-1).contiguous()
    V, D = grad.shape
    d2 = dout.reshape(-1, D)
    assert d2.is_contiguous() and d2.dtype == torch.bfloat16
    check(lib().ob_embedding_bwd(ptr(flat), ptr(d2), ptr(grad), c_int(flat.numel()), c_int(D), c_int(V), stream_ptr()), "ob_embedding_bwd")


def accum_bf16_to_f32(src: torch.Tensor, acc: torch.Tensor) -> None:
    assert src.numel() == acc.numel() and src.is_contiguous() and acc.is_contiguous()
    check(lib().ob_accum_bf16_to_f32(ptr(src), ptr(acc), c_longlong(src.numel()), stream_ptr()), "ob_accum_bf16_to_f32")


def cast_f32_to_bf16(src: torch.Tensor, dst: torch.Tensor) -> None:
    assert src.numel() == dst.numel() and src.is_contiguous() and dst.is_contiguous()
    check(lib().ob_cast_f32_to_bf16(ptr(src), ptr(dst), c_longlong(src.numel()), stream_ptr()), "ob_cast_f32_to_bf16")


# ------------------------------------------------------------------------------- loss / optimizer


def cross_entropy_(
    logits: torch.Tensor,
    labels: torch.Tensor,
    ignore_index: int = -100,
    z_mult: float = 0.0,
    grad_scale: float = 1.0,
    write_grad: bool = True,
    want_z: bool = True,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Per-row CE (and ``lse²``) of bf16 ``logits [R, V]``; with ``write_grad`` the logits are overwritten by
    ``grad_scale · d(CE + z_mult·lse²)/dlogits``."""
    _bf16(logits, "logits")
    assert logits.dim() == 2 and logits.stride(1) == 1 and labels.dtype == torch.int64
    R, V = logits.shape
    labels = labels.reshape(-1).contiguous()
    ce = torch.empty(R, dtype=torch.float32, device=logits.device)
    z = torch.empty(R, dtype=torch.float32, device=logits.device) if want_z else None
    rc = lib().ob_cross_entropy(
        ptr(logits), ptr(labels), ptr(ce), ptr(z), c_int(R), c_int(V), c_int(logits.stride(0)),
        c_longlong(ignore_index), c_float(z_mult), c_float(grad_scale), c_int(int(write_grad)), stream_ptr(),
    )
    check(rc, "ob_cross_entropy")
    return ce, z


def adamw_flat(p, g, m, v, p_lowp, seg_end, seg_wd, seg_lr, beta1, beta2, eps, step, gscale=None) -> None:
    n = p.numel()
    check(lib().ob_adamw(
        ptr(p), ptr(g), ptr(m), ptr(v), ptr(p_lowp), c_longlong(n), ptr(seg_end), ptr(seg_wd), ptr(seg_lr),
        c_int(seg_end.numel()), c_float(beta1), c_float(beta2), c_float(eps), c_int(step), ptr(gscale), stream_ptr(),
    ), "ob_adamw")


def lionw_flat(p, g, m, p_lowp, seg_end, seg_wd, seg_lr, beta1, beta2, gscale=None) -> None:
    n = p.numel()
    check(lib().ob_lionw(
        ptr(p), ptr(g), ptr(m), ptr(p_lowp), c_longlong(n), ptr(seg_end), ptr(seg_wd), ptr(seg_lr),
        c_int(seg_end.numel()), c_float(beta1), c_float(beta2), ptr(gscale), stream_ptr(),
    ), "ob_lionw")


def sumsq(g: torch.Tensor, out: torch.Tensor, accumulate: bool = False) -> torch.Tensor:
    """``out[0] (+)= Σ g²`` for a flat fp32 tensor (two-stage reduction through a scratch vector)."""
    assert g.dtype == torch.float32 and g.is_contiguous() and out.dtype == torch.float32
    n = g.numel()
    nparts = lib().ob_sumsq_num_partials(c_longlong(n))
    partials = torch.empty(nparts, dtype=torch.float32, device=g.device)
    check(lib().ob_sumsq_f32(ptr(g), c_longlong(n), ptr(partials), ptr(out), c_int(int(accumulate)), stream_ptr()), "ob_sumsq_f32", kernels=2)
    return out


def clip_coef(sumsq_t: torch.Tensor, max_norm: float, coef: torch.Tensor, norm_out: Optional[torch.Tensor] = None) -> None:
    check(lib().ob_clip_coef(ptr(sumsq_t), c_float(max_norm), ptr(coef), ptr(norm_out), stream_ptr()), "ob_clip_coef")


# ------------------------------------------------------------------------------- decode (serving)


def decode_qkv(
    qkv: torch.Tensor, wq: Optional[torch.Tensor], wk: Optional[torch.Tensor], cos: torch.Tensor, sin: torch.Tensor,
    rope_pos: torch.Tensor, write_col: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, Wq: int, Wk: int, hd: int,
    eps: float, clip: float, qk_norm: bool, rope: bool, q_out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One decode step's q/k/v post-processing: ``qkv [R, Wq + 2·Wk]`` -> rotated (and normalised) ``q [R, Wq]``; the new
    key and value rows are written into ``k_cache`` / ``v_cache`` (``[R, Hkv, window, hd]``) at column ``write_col[0]``.
    ``rope_pos [R]`` (int64) is each sequence's token index, ``cos`` / ``sin`` are fp32 ``[table_len, hd/2]``."""
    _bf16(qkv, "qkv")
    R = qkv.shape[0]
    assert qkv.is_contiguous() and qkv.shape[1] == Wq + 2 * Wk and k_cache.is_contiguous() and v_cache.is_contiguous()
    assert rope_pos.dtype == torch.int64 and write_col.dtype == torch.int64 and cos.dtype == torch.float32
    q = torch.empty((R, Wq), dtype=torch.bfloat16, device=qkv.device) if q_out is None else q_out
    check(lib().ob_decode_qkv(
        ptr(qkv), ptr(wq), ptr(wk), ptr(cos), ptr(sin), ptr(rope_pos), ptr(write_col), ptr(q), ptr(k_cache), ptr(v_cache),
        c_int(R), c_int(Wq), c_int(Wk), c_int(hd), c_int(k_cache.shape[2]), c_int(cos.shape[0]), c_float(eps), c_float(clip),
        c_int(int(qk_norm)), c_int(int(rope)), stream_ptr(),
    ), "ob_decode_qkv")
    return q


def decode_attention(
    q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, bias: torch.Tensor, length: int, scale: float, n_heads: int,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``softmax(q·Kᵀ·scale + bias)·V`` of one query per sequence over the first ``length`` columns of the windows.
    ``q [R, H·128]``, caches ``[R, Hkv, window, 128]``, ``bias`` bf16 with ``R·window`` elements (additive)."""
    _bf16(q, "q")
    R, Hkv, window, hd = k_cache.shape
    assert q.is_contiguous() and bias.dtype == torch.bfloat16 and bias.is_contiguous() and bias.numel() == R * window
    o = torch.empty_like(q) if out is None else out
    check(lib().ob_decode_attention(
        ptr(q), ptr(k_cache), ptr(v_cache), ptr(bias), ptr(o), c_int(R), c_int(n_heads), c_int(Hkv), c_int(hd), c_int(window),
        c_int(length), c_float(scale), stream_ptr(),
    ), "ob_decode_attention")
    return o
