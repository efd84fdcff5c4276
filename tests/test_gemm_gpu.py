"""tcgen05 3xTF32 GEMM engine vs an fp64 torch reference of the same product,
through the C ABI (rnet_gemm_f32): all four operand majors, ragged shapes
(M, N, K not multiples of the tile), store / accumulate (split-K) / residual
epilogues, and long K (weight-gradient shape).

Every case runs on both tile shapes of the engine: single-CTA 128-row tiles
(cta_group 1) and CTA-pair 256-row tiles over two SMs (cta_group 2), and with
the automatic choice, which splits K over a workspace for short M.

Tolerance: max |err| / max |ref| <= 2e-5 (fp32-class; plain TF32 would give
~1e-3), tighter than the 1e-4 the layer parity tests use.
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5


@pytest.fixture(params=[0, 1, 2], ids=["auto", "cg1", "cg2"])
def cta_group(request, rnet):
    rnet.call("rnet_gemm_set_cta_group", request.param)
    yield request.param
    rnet.call("rnet_gemm_set_cta_group", 0)


def _run(rnet, torch, M, N, K, amn, bmn, op, bf16=False):
    g = torch.Generator(device="cuda").manual_seed(M * 131 + N * 7 + K + amn * 3 + bmn)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = torch.randn(N, K, device="cuda", generator=g)
    A = a.t().contiguous() if amn else a
    B = b.t().contiguous() if bmn else b
    C = torch.randn(M, N, device="cuda", generator=g) if op else torch.zeros(M, N, device="cuda")
    C0 = C.clone()
    rnet.call("rnet_gemm_set_precision", 1 if bf16 else 0)
    try:
        rnet.call("rnet_gemm_f32", M, N, K, rnet.ptr(A), M if amn else K, amn, rnet.ptr(B),
                  N if bmn else K, bmn, rnet.ptr(C), N, rnet.ptr(C0), N, op, ctypes.c_float(1.0),
                  None)
        torch.cuda.synchronize()
    finally:
        rnet.call("rnet_gemm_set_precision", 0)
    ref = a.double() @ b.double().t()
    if op:
        ref = ref + C0.double()
    return ((C.double() - ref).abs().max() / ref.abs().max()).item()


@pytest.mark.parametrize("amn", [0, 1])
@pytest.mark.parametrize("bmn", [0, 1])
@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (200, 300, 96), (64, 64, 64), (256, 512, 512),
                                   (1000, 1024, 520), (384, 640, 48), (132, 96, 40)])
def test_layouts_store(rnet, cuda, cta_group, M, N, K, amn, bmn):
    assert _run(rnet, cuda, M, N, K, amn, bmn, 0) <= TOL


@pytest.mark.parametrize("op", [1, 2])
def test_accumulate_and_residual(rnet, cuda, cta_group, op):
    assert _run(rnet, cuda, 512, 512, 1024, 0, 0, op) <= TOL


def test_long_k_split(rnet, cuda, cta_group):
    # weight-gradient shape: K = tokens, both operands MN-major, split-K red.add
    assert _run(rnet, cuda, 512, 1024, 16384, 1, 1, 1) <= TOL


BF16_TOL = 1e-2


@pytest.mark.parametrize("amn", [0, 1])
@pytest.mark.parametrize("bmn", [0, 1])
@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (200, 300, 96), (1000, 1024, 520),
                                   (384, 640, 48)])
def test_bf16_layouts(rnet, cuda, cta_group, M, N, K, amn, bmn):
    """bf16 operands, fp32 accumulation: within 1e-2 of max |ref| (inputs
    rounded to 8 significant bits), and clearly less exact than 3xTF32."""
    err = _run(rnet, cuda, M, N, K, amn, bmn, 0, bf16=True)
    assert err <= BF16_TOL
    assert err > 1e-5, f"error {err:.1e}: bf16 rounding not in effect"


def test_bf16_accumulate_long_k(rnet, cuda, cta_group):
    err = _run(rnet, cuda, 512, 1024, 16384, 1, 1, 1, bf16=True)
    assert 1e-6 < err <= BF16_TOL
