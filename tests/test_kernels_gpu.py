"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _seed_and_status():
    torch.manual_seed(0)
    yield
    from olmo_b200 import ops

    ops.check_status()


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda", dtype=torch.float32) * scale).to(torch.bfloat16)


def _close(got, want, rtol=2e-2, atol=2e-2):
    got, want = got.float(), want.float()
    err = (got - want).abs().max().item()
    ref = want.abs().max().item()
    assert torch.allclose(got, want, rtol=rtol, atol=atol * max(ref, 1e-6)), f"max err {err} (ref max {ref})"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (200, 300, 72), (1024, 1024, 1024), (384, 11008, 4096)])
def test_gemm_nt(M, N, K):
    from olmo_b200.ops import kernels as k

    a, b = _rand(M, K), _rand(N, K)
    _close(k.gemm(a, b), a.float() @ b.float().t())


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (200, 264, 328), (512, 4096, 1024)])
def test_gemm_nn_dgrad(M, N, K):
    from olmo_b200.ops import kernels as k

    a, b = _rand(M, K), _rand(K, N)  # b is [K, N]: MN-major B operand
    _close(k.gemm(a, b, b_trans=True), a.float() @ b.float())


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (136, 264, 200), (4096, 1024, 2048)])
def test_gemm_tn_wgrad(M, N, K):
    from olmo_b200.ops import kernels as k

    a, b = _rand(K, M), _rand(K, N)  # both MN-major
    want = a.float().t() @ b.float()
    _close(k.gemm(a, b, a_trans=True, b_trans=True), want)
    acc = torch.ones(M, N, device="cuda", dtype=torch.float32)
    k.gemm(a, b, a_trans=True, b_trans=True, epilogue=k.EPI_F32_ACCUM, out=acc)
    _close(acc, want + 1.0, rtol=1e-2, atol=1e-2)
    st = k.gemm(a, b, a_trans=True, b_trans=True, epilogue=k.EPI_F32_STORE)
    _close(st, want, rtol=1e-2, atol=1e-2)


def test_gemm_residual_epilogue_and_strided_operands():
    from olmo_b200.ops import kernels as k

    M, N, K = 256, 512, 256
    big = _rand(M, 3 * K)
    a = big[:, K : 2 * K]  # row-strided view
    b, r = _rand(N, K), _rand(M, N)
    want = a.float() @ b.float().t() + r.float()
    _close(k.gemm(a, b, epilogue=k.EPI_BF16_ADD, residual=r), want)
    out = r.clone()
    k.gemm(a, b, epilogue=k.EPI_BF16_ADD, residual=out, out=out)  # in place
    _close(out, want)


@pytest.mark.parametrize("rms", [True, False])
@pytest.mark.parametrize("affine", [True, False])
def test_norm_fwd_bwd(rms, affine):
    from olmo_b200.ops import kernels as k

    M, D, eps = 300, 1024, 1e-5
    x, res, dy = _rand(M, D), _rand(M, D), _rand(M, D)
    w = (1 + 0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16) if affine else None
    b = (0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16) if (affine and not rms) else None

    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True) if affine else None
    bf = b.float().requires_grad_(True) if b is not None else None
    if rms:
        ref = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)
        if affine:
            ref = ref * wf
    else:
        ref = F.layer_norm(xf, (D,), wf, bf, eps)
    (ref * dy.float()).sum().backward()

    out, rstd, mean = k.norm_fwd(x, w, b, eps, rms, residual=res)
    _close(out, ref.detach() + res.float())
    dw = torch.zeros(D, device="cuda") if affine else None
    db = torch.zeros(D, device="cuda") if b is not None else None
    dx = k.norm_bwd(dy, x, w, rstd, mean, rms, dweight=dw, dbias=db)
    _close(dx, xf.grad)
    if affine:
        _close(dw, wf.grad, rtol=3e-2, atol=3e-2)
    if db is not None:
        _close(db, bf.grad, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("do_norm,clip,n_kv", [(True, 0.0, 8), (True, 0.0, 2), (False, 0.5, 8), (False, 0.0, 8)])
def test_qk_norm_rope(do_norm, clip, n_kv):
    from olmo_b200.ops import kernels as k

    B, T, H, hd, eps, theta = 2, 96, 8, 64, 1e-6, 500000.0
    Wq, Wk = H * hd, n_kv * hd
    M = B * T
    qkv = _rand(M, Wq + 2 * Wk)
    wq = (1 + 0.1 * torch.randn(Wq, device="cuda")).to(torch.bfloat16) if do_norm else None
    wk = (1 + 0.1 * torch.randn(Wk, device="cuda")).to(torch.bfloat16) if do_norm else None
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device="cuda", dtype=torch.float) / hd))
    ang = torch.outer(torch.arange(T, device="cuda", dtype=torch.float), inv)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()

    def reference(qkv_f, wq_f, wk_f):
        x = qkv_f.clamp(-clip, clip) if clip > 0 else qkv_f
        q, kk, v = x.split((Wq, Wk, Wk), dim=-1)

        def norm(t, w):
            if not do_norm:
                return t
            return t * torch.rsqrt(t.square().mean(-1, keepdim=True) + eps) * w

        def rope(t, nh):
            t = t.view(B, T, nh, hd)
            c = torch.cat((cos, cos), -1)[None, :, None, :]
            s = torch.cat((sin, sin), -1)[None, :, None, :]
            a, b_ = t.chunk(2, -1)
            return (t * c + torch.cat((-b_, a), -1) * s).reshape(M, nh * hd)

        return rope(norm(q, wq_f), H), rope(norm(kk, wk_f), n_kv), v

    qkv_f = qkv.float().requires_grad_(True)
    wq_f = wq.float().requires_grad_(True) if do_norm else None
    wk_f = wk.float().requires_grad_(True) if do_norm else None
    rq, rk, rv = reference(qkv_f, wq_f, wk_f)
    dq, dk, dv = _rand(M, Wq), _rand(M, Wk), _rand(M, Wk)
    ((rq * dq.float()).sum() + (rk * dk.float()).sum() + (rv * dv.float()).sum()).backward()

    qk, rstd_q, rstd_k = k.qk_norm_rope_fwd(qkv, wq, wk, cos, sin, T, Wq, Wk, hd, eps, clip, do_norm, True)
    _close(qk[:, :Wq], rq.detach())
    _close(qk[:, Wq : Wq + Wk], rk.detach())
    if clip > 0:
        _close(qk[:, Wq + Wk :], rv.detach())
    dqkv = torch.cat((dq, dk, dv), dim=-1).contiguous()
    dwq = torch.zeros(Wq, device="cuda") if do_norm else None
    dwk = torch.zeros(Wk, device="cuda") if do_norm else None
    k.qk_norm_rope_bwd(qkv, dqkv, wq, wk, cos, sin, rstd_q, rstd_k, T, Wq, Wk, hd, clip, do_norm, True, dwq, dwk)
    _close(dqkv, qkv_f.grad, rtol=3e-2, atol=3e-2)
    if do_norm:
        _close(dwq, wq_f.grad, rtol=3e-2, atol=3e-2)
        _close(dwk, wk_f.grad, rtol=3e-2, atol=3e-2)


def test_swiglu():
    from olmo_b200.ops import kernels as k

    M, H = 333, 1024
    h, d = _rand(M, 2 * H), _rand(M, H)
    hf = h.float().requires_grad_(True)
    v, g = hf.chunk(2, -1)
    ref = F.silu(g) * v
    (ref * d.float()).sum().backward()
    _close(k.swiglu_fwd(h), ref.detach())
    _close(k.swiglu_bwd(d, h), hf.grad)


def test_embedding():
    from olmo_b200.ops import kernels as k

    V, D = 1000, 256
    table = _rand(V, D)
    ids = torch.randint(0, V, (4, 37), device="cuda")
    out = k.embedding_fwd(ids, table)
    assert torch.equal(out, table[ids])
    d = _rand(4, 37, D)
    grad = torch.zeros(V, D, device="cuda")
    k.embedding_bwd(ids, d, grad)
    ref = torch.zeros(V, D, device="cuda").index_add_(0, ids.reshape(-1), d.reshape(-1, D).float())
    _close(grad, ref, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("z_mult", [0.0, 1e-4])
def test_cross_entropy(z_mult):
    from olmo_b200.ops import kernels as k

    R, V = 70, 100352
    logits = _rand(R, V, scale=2.0)
    labels = torch.randint(0, V, (R,), device="cuda")
    labels[::7] = -100
    lf = logits.float().requires_grad_(True)
    ce = F.cross_entropy(lf, labels, ignore_index=-100, reduction="none")
    z = torch.logsumexp(lf, -1).square() * (labels != -100)
    scale = 1.0 / 4096
    ((ce.sum() + z_mult * z.sum()) * scale).backward()
    work = logits.clone()
    got_ce, got_z = k.cross_entropy_(work, labels, -100, z_mult, scale, True)
    _close(got_ce, ce.detach(), rtol=1e-2, atol=1e-3)
    _close(got_z, z.detach(), rtol=1e-2, atol=1e-3)
    got, want = work.float(), lf.grad
    assert (got - want).abs().max().item() <= 2e-2 * want.abs().max().item() + 1e-7


def test_adamw_and_sumsq():
    from olmo_b200.ops import kernels as k

    n = 100_003
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    ref_p = torch.nn.Parameter(p.clone())
    opt = torch.optim.AdamW([ref_p], lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    lowp = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    seg_end = torch.tensor([n], device="cuda", dtype=torch.int64)
    seg_wd = torch.tensor([0.1], device="cuda")
    seg_lr = torch.tensor([3e-4], device="cuda")
    scale = torch.tensor([0.5], device="cuda")
    for step in range(1, 4):
        ref_p.grad = g * 0.5
        opt.step()
        k.adamw_flat(p, g, m, v, lowp, seg_end, seg_wd, seg_lr, 0.9, 0.95, 1e-8, step, scale)
    assert torch.allclose(p, ref_p.detach(), rtol=1e-5, atol=1e-6)
    assert torch.allclose(lowp.float(), p, rtol=1e-2, atol=1e-3)
    out = torch.zeros(1, device="cuda")
    k.sumsq(g, out)
    assert math.isclose(out.item(), g.double().square().sum().item(), rel_tol=1e-4)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("H,Hkv,T", [(4, 4, 512), (4, 2, 256), (2, 1, 1024)])
def test_native_attention_forward(causal, H, Hkv, T):
    from olmo_b200.ops import attention as A
    from olmo_b200.ops import attention_native as N

    B, D = 2, 128
    # operands are strided views into one fused buffer, as in the model
    fused = _rand(B * T, (H + 2 * Hkv) * D)
    q = fused[:, : H * D].view(B, T, H, D)
    k = fused[:, H * D : (H + Hkv) * D].view(B, T, Hkv, D)
    v = fused[:, (H + Hkv) * D :].view(B, T, Hkv, D)
    assert N.supports(q, k, causal, 0.0, False)
    scale = 1.0 / math.sqrt(D)
    o, lse = N.forward(q, k, v, causal, scale)
    ro, rlse = A.math_attention_forward(q, k, v, causal, scale)
    _close(o, ro, rtol=2e-2, atol=2e-2)
    assert torch.allclose(lse, rlse, rtol=1e-3, atol=2e-3), (lse - rlse).abs().max().item()


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("H,Hkv,T", [(4, 4, 512), (4, 2, 256)])
def test_native_attention_backward(causal, H, Hkv, T):
    from olmo_b200.ops import attention as A
    from olmo_b200.ops import attention_native as N

    B, D = 2, 128
    fused = _rand(B * T, (H + 2 * Hkv) * D)
    q = fused[:, : H * D].view(B, T, H, D)
    k = fused[:, H * D : (H + Hkv) * D].view(B, T, Hkv, D)
    v = fused[:, (H + Hkv) * D :].view(B, T, Hkv, D)
    assert N.supports_backward(q, k, causal)
    scale = 1.0 / math.sqrt(D)
    o, lse = N.forward(q, k, v, causal, scale)
    do = _rand(B, T, H, D)
    dfused = torch.zeros_like(fused)
    dq = dfused[:, : H * D].view(B, T, H, D)
    dk = dfused[:, H * D : (H + Hkv) * D].view(B, T, Hkv, D)
    dv = dfused[:, (H + Hkv) * D :].view(B, T, Hkv, D)
    N.backward(do, q, k, v, o, lse, dq, dk, dv, causal, scale)
    ro, rlse = A.math_attention_forward(q, k, v, causal, scale)
    rdq, rdk, rdv = A._math_attention_backward(do, q, k, v, ro, rlse, causal, scale)
    _close(dv, rdv, rtol=3e-2, atol=3e-2)
    _close(dk, rdk, rtol=3e-2, atol=3e-2)
    _close(dq, rdq, rtol=3e-2, atol=3e-2)


def _autograd_attention(q, k, v, do, causal, scale, doc_start=None):
    """fp32 attention written with differentiable torch ops; gradients come from autograd, not from hand-derived formulas."""
    B, T, H, D = q.shape
    Hkv = k.shape[2]
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ke = kf.repeat_interleave(H // Hkv, dim=2) if Hkv != H else kf
    ve = vf.repeat_interleave(H // Hkv, dim=2) if Hkv != H else vf
    s_ = torch.einsum("bthd,bshd->bhts", qf, ke) * scale
    allowed = torch.ones(T, T, dtype=torch.bool, device=q.device)
    if causal:
        allowed = torch.tril(allowed)
    allowed = allowed.view(1, 1, T, T)
    if doc_start is not None:
        keys = torch.arange(T, device=q.device).view(1, 1, 1, T)
        allowed = allowed & (keys >= doc_start.view(B, 1, T, 1).long())
    s_ = s_.masked_fill(~allowed, float("-inf"))
    out = torch.einsum("bhts,bshd->bthd", torch.softmax(s_, dim=-1), ve)
    out.backward(do.float())
    return out.detach(), qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("causal,H,Hkv,T,D", [
    (True, 4, 4, 512, 128), (False, 4, 2, 256, 128),   # the kernels' own tile shape
    (True, 4, 4, 200, 64), (True, 2, 1, 384, 96), (False, 2, 2, 256, 32), (True, 3, 3, 77, 128),  # reached by zero padding
])
def test_native_attention_against_fp32_autograd(causal, H, Hkv, T, D):
    from olmo_b200.ops import attention_native as N

    B = 2
    fused = _rand(B * T, (H + 2 * Hkv) * D)
    q = fused[:, : H * D].view(B, T, H, D)
    k = fused[:, H * D : (H + Hkv) * D].view(B, T, Hkv, D)
    v = fused[:, (H + Hkv) * D :].view(B, T, Hkv, D)
    assert N.supports_backward(q, k, causal)
    scale = 1.0 / math.sqrt(D)
    o, lse = N.forward(q, k, v, causal, scale)
    assert o.shape == (B, T, H, D) and lse.shape == (B, H, T)
    do = _rand(B, T, H, D)
    dfused = torch.zeros_like(fused)
    dq = dfused[:, : H * D].view(B, T, H, D)
    dk = dfused[:, H * D : (H + Hkv) * D].view(B, T, Hkv, D)
    dv = dfused[:, (H + Hkv) * D :].view(B, T, Hkv, D)
    N.backward(do, q, k, v, o, lse, dq, dk, dv, causal, scale)
    ro, rdq, rdk, rdv = _autograd_attention(q, k, v, do, causal, scale)
    _close(o, ro, rtol=2e-2, atol=2e-2)
    _close(dv, rdv, rtol=3e-2, atol=3e-2)
    _close(dk, rdk, rtol=3e-2, atol=3e-2)
    _close(dq, rdq, rtol=3e-2, atol=3e-2)


def test_native_attention_document_masking_with_padding_against_autograd():
    from olmo_b200.ops import attention_native as N

    B, T, H, D = 2, 300, 2, 64
    q, k, v, do = _rand(B, T, H, D), _rand(B, T, H, D), _rand(B, T, H, D), _rand(B, T, H, D)
    doc_lens = torch.tensor([[100, 150, 50], [300, 0, 0]], device="cuda")
    doc_start = N.doc_start_from_lengths(doc_lens, T)
    scale = 1.0 / math.sqrt(D)
    o, lse = N.forward(q, k, v, True, scale, doc_start=doc_start)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    N.backward(do, q, k, v, o, lse, dq, dk, dv, True, scale, doc_start=doc_start)
    ro, rdq, rdk, rdv = _autograd_attention(q, k, v, do, True, scale, doc_start=doc_start)
    _close(o, ro, rtol=2e-2, atol=2e-2)
    for got, want in ((dq, rdq), (dk, rdk), (dv, rdv)):
        _close(got, want, rtol=3e-2, atol=3e-2)


def _gemm_close(got, want, K):
    """Inputs are bf16 and accumulation is fp32, so the error of an output element is that of its final rounding (bf16
    outputs: 2^-8 relative) plus accumulation-order noise that grows like sqrt(K) times fp32 epsilon."""
    got, want = got.float(), want.float()
    ref = want.abs().max().item()
    out_eps = 2.0 ** -8
    tol = (out_eps + 4.0 * math.sqrt(K) * 2.0 ** -23) * max(ref, 1e-6)
    err = (got - want).abs().max().item()
    assert err <= tol, f"max err {err} > {tol} (ref max {ref}, K={K})"


@pytest.mark.parametrize("tma_store", [1, 0])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (300, 296, 72), (1000, 520, 4096), (8192, 4096, 11008), (257, 264, 128)])
def test_gemm_pair_epilogues_with_and_without_tma_stores(tma_store, M, N, K):
    """All four epilogues of the two-CTA kernel, output tiles leaving through shared memory + TMA (store or reduce-add) or
    through per-thread stores, ragged M and N included; tolerance scaled with sqrt(K)."""
    import ctypes

    from olmo_b200 import ops
    from olmo_b200.ops import kernels as k

    lib = ops.lib()
    lib.ob_set_gemm_pair_mode(ctypes.c_int(1))
    lib.ob_set_gemm_tma_store(ctypes.c_int(tma_store))
    try:
        a, b = _rand(M, K), _rand(N, K)
        ref = a.float() @ b.float().t()
        _gemm_close(k.gemm(a, b), ref, K)
        res = _rand(M, N)
        _gemm_close(k.gemm(a, b, epilogue=k.EPI_BF16_ADD, residual=res), ref + res.float(), K)
        dy = _rand(M, N)
        wref = dy.float().t() @ a.float()  # [N, K]: contraction over M
        acc = torch.full((N, K), 1.0, device="cuda")
        k.gemm(dy, a, a_trans=True, b_trans=True, epilogue=k.EPI_F32_ACCUM, out=acc)
        k.gemm(dy, a, a_trans=True, b_trans=True, epilogue=k.EPI_F32_ACCUM, out=acc)
        got, want = acc, 2 * wref + 1.0
        assert (got - want).abs().max().item() <= 8.0 * math.sqrt(M) * 2.0 ** -23 * want.abs().max().item() + 1e-5
        st = torch.full((N, K), 7.0, device="cuda")
        k.gemm(dy, a, a_trans=True, b_trans=True, epilogue=k.EPI_F32_STORE, out=st)
        assert (st - wref).abs().max().item() <= 8.0 * math.sqrt(M) * 2.0 ** -23 * wref.abs().max().item() + 1e-5
    finally:
        lib.ob_set_gemm_tma_store(ctypes.c_int(1))


@pytest.mark.parametrize("M", [1, 5, 16, 33, 64, 200])
@pytest.mark.parametrize("N,K", [(4096, 4096), (1000, 512), (384, 11008), (12288, 4096)])
def test_gemm_small_m_streams_weights(M, N, K):
    """Decode-sized products (weights as the 128-row operand, batch as the narrow one, K split over CTAs for layers with
    few feature tiles) against fp32; rows beyond the batch and features beyond N must not be written."""
    from olmo_b200 import ops
    from olmo_b200.ops import kernels as k

    assert k.gemm_small_m_available()
    x, w = _rand(M, K), _rand(N, K)
    y = k.gemm_small_m(x, w)
    ops.check_status()
    assert y.shape == (M, N)
    _gemm_close(y, x.float() @ w.float().t(), K)
    again = k.gemm_small_m(x, w)
    assert torch.equal(y, again)  # split sums are added in split order: bit-identical from run to run
    xs = _rand(M, K + 64)[:, :K]  # a strided activation view
    _gemm_close(k.gemm_small_m(xs, w), xs.float() @ w.float().t(), K)


@pytest.fixture
def pair_mode():
    """Route GEMMs through the two-CTA (cta_group::2) kernel for the duration of a test."""
    import ctypes

    from olmo_b200 import ops

    lib = ops.lib()
    before = lib.ob_get_gemm_pair_mode()
    lib.ob_set_gemm_pair_mode(ctypes.c_int(1))
    yield
    lib.ob_set_gemm_pair_mode(ctypes.c_int(before))


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (256, 512, 128), (300, 300, 72), (1024, 1024, 1024), (384, 11008, 4096)])
def test_gemm_pair_nt(pair_mode, M, N, K):
    from olmo_b200.ops import kernels as k

    a, b = _rand(M, K), _rand(N, K)
    _close(k.gemm(a, b), a.float() @ b.float().t())


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (264, 264, 328), (512, 4096, 1024)])
def test_gemm_pair_dgrad_wgrad(pair_mode, M, N, K):
    from olmo_b200.ops import kernels as k

    a, b = _rand(M, K), _rand(K, N)
    _close(k.gemm(a, b, b_trans=True), a.float() @ b.float())
    at, bt = _rand(K, M), _rand(K, N)
    want = at.float().t() @ bt.float()
    acc = torch.ones(M, N, device="cuda", dtype=torch.float32)
    k.gemm(at, bt, a_trans=True, b_trans=True, epilogue=k.EPI_F32_ACCUM, out=acc)
    _close(acc, want + 1.0, rtol=1e-2, atol=1e-2)
    r = _rand(M, N)
    _close(k.gemm(a, b, b_trans=True, epilogue=k.EPI_BF16_ADD, residual=r), a.float() @ b.float() + r.float())


@pytest.mark.parametrize("H,Hkv", [(4, 4), (4, 2)])
def test_native_attention_document_masking(H, Hkv):
    """Intra-document masking: forward and backward of the native kernels against the fp32 math path, with documents
    that start and end inside tiles, span several tiles, and coincide with tile borders."""
    from olmo_b200.ops import attention as A
    from olmo_b200.ops import attention_native as N

    B, T, D = 2, 1024, 128
    doc_lens = torch.tensor([[100, 156, 512, 7, 249, 0], [128, 128, 300, 400, 68, 0]], device="cuda")
    assert int(doc_lens.sum(1)[0]) == T and int(doc_lens.sum(1)[1]) == T
    ds = N.doc_start_from_lengths(doc_lens, T)
    fused = _rand(B * T, (H + 2 * Hkv) * D)
    q = fused[:, : H * D].view(B, T, H, D)
    k = fused[:, H * D : (H + Hkv) * D].view(B, T, Hkv, D)
    v = fused[:, (H + Hkv) * D :].view(B, T, Hkv, D)
    scale = 1.0 / math.sqrt(D)
    o, lse = N.forward(q, k, v, True, scale, doc_start=ds)
    ro, rlse = A.math_attention_forward(q, k, v, True, scale, doc_start=ds)
    _close(o, ro, rtol=2e-2, atol=2e-2)
    assert torch.allclose(lse, rlse, rtol=1e-3, atol=2e-3), (lse - rlse).abs().max().item()
    # the mask matters: unmasked attention differs
    o_plain, _ = N.forward(q, k, v, True, scale)
    assert (o_plain.float() - ro.float()).abs().max() > 0.05

    do = _rand(B, T, H, D)
    dfused = torch.zeros_like(fused)
    dq = dfused[:, : H * D].view(B, T, H, D)
    dk = dfused[:, H * D : (H + Hkv) * D].view(B, T, Hkv, D)
    dv = dfused[:, (H + Hkv) * D :].view(B, T, Hkv, D)
    N.backward(do, q, k, v, o, lse, dq, dk, dv, True, scale, doc_start=ds)
    rdq, rdk, rdv = A._math_attention_backward(do, q, k, v, ro, rlse, True, scale, doc_start=ds)
    _close(dv, rdv, rtol=3e-2, atol=3e-2)
    _close(dk, rdk, rtol=3e-2, atol=3e-2)
    _close(dq, rdq, rtol=3e-2, atol=3e-2)
    from olmo_b200 import ops

    ops.check_status()


@pytest.mark.parametrize("H,Hkv", [(2, 2), (4, 1)])
def test_native_attention_packed_sequences(H, Hkv):
    """Packed variable-length attention (cumulative document lengths over one token axis) through the public entry
    point: the native document-masking kernels against the fp32 math path, forward and backward."""
    from olmo_b200.ops import attention as A
    from olmo_b200.ops import attention_native as N

    total, D = 2048, 128
    cu = torch.tensor([0, 300, 301, 1024, 1500, 2048], device="cuda", dtype=torch.int32)
    q0, k0, v0 = _rand(total, H, D), _rand(total, Hkv, D), _rand(total, Hkv, D)
    assert N.supports_varlen(q0, k0, True, 0.0)

    def run(fn):
        q, k, v = (t.clone().requires_grad_(True) for t in (q0, k0, v0))
        out = fn(q, k, v)
        out.backward(torch.ones_like(out) * 0.01)
        return out, q.grad, k.grad, v.grad

    got = run(lambda q, k, v: A.varlen_attention(q, k, v, cu, 724, causal=True))
    want = run(lambda q, k, v: A._VarlenMath.apply(q, k, v, cu, True, 1.0 / math.sqrt(D)))
    for g, w in zip(got, want):
        _close(g, w, rtol=3e-2, atol=3e-2)
    # a query never sees the previous document: changing document 0 leaves the outputs of document 2 untouched
    q1, k1, v1 = q0.clone(), k0.clone(), v0.clone()
    k1[:300] += 1.0
    v1[:300] -= 1.0
    out1 = A.varlen_attention(q1, k1, v1, cu, 724, causal=True)
    assert torch.equal(out1[301:1024], got[0][301:1024].detach())


@pytest.mark.parametrize("qk_norm,clip,Hkv", [(True, 0.0, 4), (False, 1.5, 4), (True, 0.0, 2)])
def test_decode_qkv_kernel(qk_norm, clip, Hkv):
    """QK-norm + rotary + cache write of one decode step against the same arithmetic in fp32 PyTorch."""
    from olmo_b200.ops import kernels as k
    from olmo_b200.ops.fused_block import rope_tables

    R, H, hd, window, T = 5, 4, 128, 40, 64
    Wq, Wk = H * hd, Hkv * hd
    qkv = _rand(R, Wq + 2 * Wk)
    wq, wk = (_rand(Wq) * 0.1 + 1.0), (_rand(Wk) * 0.1 + 1.0)
    cos, sin = rope_tables(T, hd, 10000.0, torch.device("cuda"))
    rope_pos = torch.tensor([0, 3, 17, 63, 200], device="cuda")  # the last one is clamped to the table
    col = torch.tensor([7], device="cuda")
    kc = torch.full((R, Hkv, window, hd), 9.0, device="cuda", dtype=torch.bfloat16)
    vc = torch.full((R, Hkv, window, hd), 9.0, device="cuda", dtype=torch.bfloat16)
    q = k.decode_qkv(qkv, wq if qk_norm else None, wk if qk_norm else None, cos, sin, rope_pos, col, kc, vc, Wq, Wk, hd, 1e-6, clip, qk_norm, True)

    x = qkv.float()
    if clip > 0:
        x = x.clamp(-clip, clip)
    qf, kf, vf = x[:, :Wq], x[:, Wq : Wq + Wk], x[:, Wq + Wk :]
    if qk_norm:
        qf = qf * torch.rsqrt(qf.pow(2).mean(-1, keepdim=True) + 1e-6) * wq.float()
        kf = kf * torch.rsqrt(kf.pow(2).mean(-1, keepdim=True) + 1e-6) * wk.float()
    tok = rope_pos.clamp(max=T - 1)
    c = torch.cat((cos[tok], cos[tok]), -1)[:, None, :]
    s = torch.cat((sin[tok], sin[tok]), -1)[:, None, :]

    def rot(t, heads):
        t = t.view(R, heads, hd)
        a, b = t.chunk(2, dim=-1)
        return (t * c + torch.cat((-b, a), -1) * s).reshape(R, heads * hd)

    _close(q, rot(qf, H), rtol=2e-2, atol=2e-2)
    _close(kc[:, :, 7, :].reshape(R, Wk), rot(kf, Hkv), rtol=2e-2, atol=2e-2)
    _close(vc[:, :, 7, :].reshape(R, Wk), vf, rtol=1e-2, atol=1e-2)
    untouched = torch.ones(window, dtype=torch.bool, device="cuda")
    untouched[7] = False
    assert bool((kc[:, :, untouched] == 9.0).all()) and bool((vc[:, :, untouched] == 9.0).all())


@pytest.mark.parametrize("H,Hkv,length", [(4, 4, 128), (8, 2, 37), (2, 1, 3)])
def test_decode_attention_kernel(H, Hkv, length):
    """One query per sequence over a masked key/value window against softmax attention in fp32."""
    from olmo_b200.ops import kernels as k

    R, hd, window = 6, 128, 160
    q = _rand(R, H * hd)
    kc, vc = _rand(R, Hkv, window, hd), _rand(R, Hkv, window, hd)
    floor = torch.finfo(torch.bfloat16).min
    bias = torch.full((R, window), floor, device="cuda", dtype=torch.bfloat16)
    for r in range(R - 1):  # row r sees a right-aligned stretch of the first `length` columns; the last row is idle
        first = (r * 7) % length
        bias[r, first:length] = 0.0
    out = k.decode_attention(q, kc, vc, bias, length, 1.0 / math.sqrt(hd), H)
    assert torch.isfinite(out.float()).all()
    g = H // Hkv
    kf = kc[:, :, :length].float().repeat_interleave(g, dim=1)
    vf = vc[:, :, :length].float().repeat_interleave(g, dim=1)
    scores = torch.einsum("rhd,rhjd->rhj", q.float().view(R, H, hd), kf) / math.sqrt(hd) + bias[:, None, :length].float()
    want = torch.einsum("rhj,rhjd->rhd", torch.softmax(scores, dim=-1), vf).reshape(R, H * hd)
    _close(out[: R - 1], want[: R - 1], rtol=2e-2, atol=2e-2)
