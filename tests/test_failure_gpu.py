"""The device-side bounded-wait failure path, exercised without a fault.

Every mbarrier spin in the library's pipelined kernels (GEMM, conv backward,
RMSNorm backward) is bounded: past its limit the waiting role sets
ERR_WAIT_TIMEOUT in the device error word, the CTA's other roles stop waiting,
the TMEM-owning warp frees its columns and the kernel returns. The self-test
kernel has that role structure around a barrier that nothing arrives on, with
a wait limit of a few milliseconds, so the wait runs out on purpose: no trap,
no hang, and the context stays usable for the next launch.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ERR_WAIT_TIMEOUT = 1


def _run(rnet, arrive, timeout_us, n_ctas):
    out = ctypes.c_uint(0)
    rnet.check(rnet.lib().rnet_selftest_bounded_wait(arrive, timeout_us, n_ctas,
                                                     ctypes.byref(out)))
    return out.value


def test_wait_runs_out_sets_error_and_returns(rnet, cuda):
    rnet.device_error(clear=True)
    # control: the barrier completes, nothing is flagged
    assert _run(rnet, 1, 5000, 4) == 0
    assert rnet.device_error(clear=True) == 0
    # nothing arrives: every CTA gives up after ~5 ms and returns
    n = 296  # two CTAs per SM: every SM frees TMEM on the abort path
    assert _run(rnet, 0, 5000, n) == n
    assert rnet.device_error(clear=True) & ERR_WAIT_TIMEOUT
    # the context is intact and TMEM was released: the control case and a
    # tcgen05 GEMM still run and are correct
    assert _run(rnet, 1, 5000, 296) == 0
    assert rnet.device_error(clear=True) == 0
    torch = cuda
    g = torch.Generator().manual_seed(3)
    a = torch.randn(256, 128, generator=g).cuda()
    b = torch.randn(192, 128, generator=g).cuda()
    c = torch.empty(256, 192, device="cuda")
    rnet.call("rnet_gemm_f32", 256, 192, 128, a.data_ptr(), 128, 0, b.data_ptr(), 128, 0,
              c.data_ptr(), 192, None, 0, 0, 1.0, None)
    torch.cuda.synchronize()
    ref = (a.double() @ b.double().T).float()
    assert torch.allclose(c, ref, rtol=1e-4, atol=1e-4)
    assert rnet.device_error(clear=True) == 0


def test_selftest_rejects_bad_arguments(rnet):
    out = ctypes.c_uint(0)
    assert rnet.lib().rnet_selftest_bounded_wait(0, 0, 1, ctypes.byref(out)) != 0
    assert rnet.lib().rnet_selftest_bounded_wait(0, 1000, 0, ctypes.byref(out)) != 0
    assert rnet.lib().rnet_selftest_bounded_wait(0, 1000, 1, None) != 0
