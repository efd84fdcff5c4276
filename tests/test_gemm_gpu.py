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


# ------------------------------------------------------------------ bf16 storage
ST16_TOL = 1e-5  # vs an fp64 product of the SAME bf16 inputs: only fp32 accumulation error


def _run_bf16(rnet, torch, M, N, K, amn, bmn, op, c16=False):
    g = torch.Generator(device="cuda").manual_seed(M * 17 + N * 5 + K + amn * 3 + bmn)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    A = a.t().contiguous() if amn else a
    B = b.t().contiguous() if bmn else b
    C = torch.randn(M, N, device="cuda", generator=g) if op else torch.zeros(M, N, device="cuda")
    C0 = C.clone()
    C16 = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16) if c16 else None
    rnet.call("rnet_gemm_bf16", M, N, K, rnet.ptr(A), M if amn else K, amn, rnet.ptr(B),
              N if bmn else K, bmn, rnet.ptr(C), N, rnet.ptr(C0), N, op, ctypes.c_float(1.0),
              rnet.ptr(C16), None)
    torch.cuda.synchronize()
    ref = a.double() @ b.double().t()
    if op:
        ref = ref + C0.double()
    err = ((C.double() - ref).abs().max() / ref.abs().max()).item()
    if c16:
        assert torch.equal(C16, C.bfloat16()), "bf16 copy is not the rounded fp32 result"
    return err


@pytest.mark.parametrize("amn", [0, 1])
@pytest.mark.parametrize("bmn", [0, 1])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (200, 304, 96), (256, 512, 512),
                                   (1000, 1024, 520), (384, 640, 48), (136, 96, 40),
                                   (2048, 1024, 4096)])
def test_bf16_storage_layouts(rnet, cuda, cta_group, M, N, K, amn, bmn):
    assert _run_bf16(rnet, cuda, M, N, K, amn, bmn, 0) <= ST16_TOL


@pytest.mark.parametrize("op,c16", [(1, False), (2, False), (0, True), (2, True)])
def test_bf16_storage_epilogues(rnet, cuda, cta_group, op, c16):
    for amn, bmn in ((0, 0), (1, 1)):
        assert _run_bf16(rnet, cuda, 512, 768, 1024, amn, bmn, op, c16) <= ST16_TOL


def test_bf16_storage_rejects_bad_pitch(rnet, cuda):
    torch = cuda
    a = torch.zeros(64, 68, device="cuda", dtype=torch.bfloat16)  # pitch 136 B
    b = torch.zeros(64, 68, device="cuda", dtype=torch.bfloat16)
    c = torch.zeros(64, 64, device="cuda")
    rc = rnet.lib().rnet_gemm_bf16(64, 64, 64, rnet.ptr(a), 68, 0, rnet.ptr(b), 68, 0,
                                  rnet.ptr(c), 64, None, 0, 0, ctypes.c_float(1.0), None, None)
    assert rc != 0
