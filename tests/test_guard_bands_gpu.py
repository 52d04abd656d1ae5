"""Out-of-bounds writes: every kernel that writes into a caller-supplied buffer runs with that buffer placed between
two guard bands of a sentinel pattern, on shapes that do not divide the kernels' tiles; the bands must be untouched
afterwards and the payload must have been written.  (A memory checker cannot be run on the test machines, so the
kernels are checked by their effects.)"""
import pytest
import torch

pytestmark = pytest.mark.gpu

GUARD = 4096  # elements on either side


class Guarded:
    """A tensor view of ``shape`` inside a larger allocation whose head and tail hold a sentinel."""

    def __init__(self, shape, dtype, fill=None):
        n = 1
        for s in shape:
            n *= s
        self.n = n
        self.sentinel = {torch.bfloat16: -12352.0, torch.float32: -1.2345678e30, torch.int64: -(1 << 40)}[dtype]
        self.raw = torch.full((n + 2 * GUARD,), self.sentinel, dtype=dtype, device="cuda")
        self.view = self.raw[GUARD : GUARD + n].view(*shape)
        if fill is not None:
            self.view.copy_(fill)

    def check(self, what: str, expect_written: bool = True) -> None:
        head, tail = self.raw[:GUARD], self.raw[GUARD + self.n :]
        assert bool((head == self.sentinel).all()), f"{what}: wrote before the buffer"
        assert bool((tail == self.sentinel).all()), f"{what}: wrote past the buffer"
        if expect_written:
            assert not bool((self.view == self.sentinel).any()), f"{what}: left part of the buffer unwritten"


def _rand(*shape):
    return torch.randn(*shape, device="cuda").to(torch.bfloat16)


@pytest.fixture(autouse=True)
def _status():
    torch.manual_seed(0)
    yield
    from olmo_b200 import ops

    ops.check_status()


@pytest.mark.parametrize("M,N,K", [(200, 304, 72), (129, 136, 264), (1000, 520, 136), (8, 4096, 128)])
def test_gemm_outputs_stay_inside(M, N, K):
    from olmo_b200.ops import kernels as k

    a, b = _rand(M, K), _rand(N, K)
    out = Guarded((M, N), torch.bfloat16)
    k.gemm(a, b, out=out.view)
    out.check(f"gemm NT {M}x{N}x{K}")
    torch.testing.assert_close(out.view.float(), a.float() @ b.float().t(), rtol=3e-2, atol=3e-1)

    Mt = (M + 7) // 8 * 8  # the transposed operand is M-major: its row pitch must be a multiple of 16 bytes
    at, bt = _rand(K, Mt), _rand(K, N)
    acc = Guarded((Mt, N), torch.float32, fill=torch.zeros(Mt, N, device="cuda"))
    k.gemm(at, bt, a_trans=True, b_trans=True, epilogue=k.EPI_F32_ACCUM, out=acc.view)
    acc.check(f"gemm TN accumulate {Mt}x{N}x{K}")
    torch.testing.assert_close(acc.view, at.float().t() @ bt.float(), rtol=3e-2, atol=3e-1)


@pytest.mark.parametrize("M,D", [(37, 256), (1000, 4096), (593, 2048)])
def test_row_kernels_stay_inside(M, D):
    from olmo_b200.ops import kernels as k

    x, dy, w = _rand(M, D), _rand(M, D), _rand(D)
    _, rstd, _ = k.norm_fwd(x, w, None, 1e-6, True)
    dx = Guarded((M, D), torch.bfloat16)
    dw = Guarded((D,), torch.float32, fill=torch.zeros(D, device="cuda"))
    k.norm_bwd(dy, x, w, rstd, None, True, dweight=dw.view, out=dx.view)
    dx.check(f"norm_bwd {M}x{D}")
    dw.check(f"norm_bwd weight gradient {M}x{D}")

    h, dact = _rand(M, 2 * D), _rand(M, D)
    dh = Guarded((M, 2 * D), torch.bfloat16)
    k.swiglu_bwd(dact, h, out=dh.view)
    dh.check(f"swiglu_bwd {M}x{D}")


@pytest.mark.parametrize("R,V", [(33, 1000), (130, 50304), (7, 100352)])
def test_cross_entropy_stays_inside(R, V):
    from olmo_b200.ops import kernels as k

    logits = Guarded((R, V), torch.bfloat16, fill=_rand(R, V))
    labels = torch.randint(0, V, (R,), device="cuda")
    labels[0] = -100
    want = torch.nn.functional.cross_entropy(logits.view.float(), labels, ignore_index=-100, reduction="none")
    ce, _ = k.cross_entropy_(logits.view, labels, -100, 1e-4, 1.0 / R, True)
    logits.check(f"cross entropy {R}x{V}")
    torch.testing.assert_close(ce, want, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("n", [8, 1000, 1 << 20, (1 << 20) + 8])
def test_flat_kernels_stay_inside(n):
    from olmo_b200.ops import kernels as k

    p = Guarded((n,), torch.float32, fill=torch.randn(n, device="cuda"))
    g = Guarded((n,), torch.float32, fill=torch.randn(n, device="cuda"))
    m = Guarded((n,), torch.float32, fill=torch.zeros(n, device="cuda"))
    v = Guarded((n,), torch.float32, fill=torch.zeros(n, device="cuda"))
    low = Guarded((n,), torch.bfloat16)
    seg_end = torch.tensor([n // 2 // 8 * 8, n], device="cuda", dtype=torch.int64)
    seg_wd, seg_lr = torch.tensor([0.1, 0.0], device="cuda"), torch.tensor([1e-3, 1e-3], device="cuda")
    k.adamw_flat(p.view, g.view, m.view, v.view, low.view, seg_end, seg_wd, seg_lr, 0.9, 0.95, 1e-8, 1, None)
    for name, t in (("p", p), ("g", g), ("m", m), ("v", v), ("low precision copy", low)):
        t.check(f"adamw {name} n={n}")
    torch.testing.assert_close(low.view.float(), p.view, rtol=1e-2, atol=1e-2)

    dst = Guarded((n,), torch.bfloat16)
    k.cast_f32_to_bf16(p.view, dst.view)
    dst.check(f"cast n={n}")
    acc = Guarded((n,), torch.float32, fill=torch.zeros(n, device="cuda"))
    k.accum_bf16_to_f32(dst.view, acc.view)
    acc.check(f"accumulate n={n}")
    total = torch.zeros(1, device="cuda")
    k.sumsq(g.view, total)
    g.check(f"sumsq input n={n}")
    torch.testing.assert_close(total[0], (g.view.double() ** 2).sum().float(), rtol=1e-4, atol=1e-4)


def test_embedding_gradient_stays_inside_and_ignores_bad_ids():
    from olmo_b200.ops import kernels as k

    V, D, M = 1000, 512, 300
    grad = Guarded((V, D), torch.float32, fill=torch.zeros(V, D, device="cuda"))
    ids = torch.randint(0, V, (M,), device="cuda")
    ids[5], ids[6] = V + 3, -1  # out-of-range ids are skipped, not dereferenced
    dout = _rand(M, D)
    k.embedding_bwd(ids, dout, grad.view)
    grad.check("embedding_bwd")
    ok = (ids >= 0) & (ids < V)
    want = torch.zeros(V, D, device="cuda").index_add_(0, ids[ok], dout[ok].float())
    torch.testing.assert_close(grad.view, want, rtol=1e-3, atol=1e-3)
    table = _rand(V, D)
    out = k.embedding_fwd(ids, table)
    assert torch.equal(out[ok], table[ids[ok]]) and torch.equal(out[5], table[0])
