"""Device-side failure detection without faulting the GPU: a collective kernel waits on a flag that nothing ever sets,
its bounded wait runs out after a short budget, the kernel returns, the status word reports it to the host, and the
context stays usable (the same stream runs a GEMM correctly afterwards)."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_through_status_word():
    from olmo_b200 import ops
    from olmo_b200.exceptions import OLMoKernelError
    from olmo_b200.ops import kernels as k
    from olmo_b200.parallel.peer import COMM_ALL_GATHER, CommTask

    dev = torch.device("cuda", 0)
    ops.check_status(dev)  # start clean
    n = 1 << 16
    src = torch.ones(2 * n, dtype=torch.bfloat16, device=dev)
    dst = torch.zeros(2 * n, dtype=torch.bfloat16, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)  # the "peer" never publishes: stays 0

    t = CommTask()
    t.kind, t.world, t.rank = COMM_ALL_GATHER, 2, 0
    t.elems, t.dst_peer_stride = n, n
    t.src[0], t.src[1] = src.data_ptr(), src.data_ptr() + 2 * n
    t.wait_flags[0], t.wait_flags[1] = None, flag.data_ptr()
    t.wait_value = 1
    t.dst = dst.data_ptr()
    t.status = ops.status_tensor(dev).data_ptr()
    t.wait_cycles = int(0.2 * 1.9e9)  # about 0.2 s of SM clocks
    t.sumsq_partials = None

    t0 = time.perf_counter()
    ops.check(ops.lib().ob_comm_launch(ctypes.byref(t), ctypes.c_int(4), ops.stream_ptr()), "ob_comm_launch")
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 0.05 < waited < 5.0, waited  # gave up after its budget instead of spinning forever
    with pytest.raises(OLMoKernelError, match="bounded wait"):
        ops.check_status(dev)
    ops.check_status(dev)  # the word was cleared by the failed check
    assert float(dst.float().abs().sum()) == 0.0  # nothing was copied from the silent peer

    # once the flag is set the same task completes, and the context is as usable as before
    flag.fill_(1)
    ops.check(ops.lib().ob_comm_launch(ctypes.byref(t), ctypes.c_int(4), ops.stream_ptr()), "ob_comm_launch")
    torch.cuda.synchronize()
    ops.check_status(dev)
    assert float(dst[n:].float().sum()) == n
    a = torch.randn(256, 128, device=dev, dtype=torch.bfloat16)
    b = torch.randn(384, 128, device=dev, dtype=torch.bfloat16)
    torch.testing.assert_close(k.gemm(a, b).float(), a.float() @ b.float().t(), rtol=2e-2, atol=2e-1)
