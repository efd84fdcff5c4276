"""The allocation-free cross-entropy entry point.

Some callers cannot allocate device memory while they run (a framework that
owns all device memory through its own pool, or code running where a
cudaMalloc would be an unwanted synchronisation or is forbidden). For them
rnet_cross_entropy_forward_noalloc takes its scratch from a fixed array inside
the library instead of cudaMallocAsync. This checks, through the C ABI, that it
gives the same loss and dlogits as rnet_cross_entropy_forward on two calls in
a row (the second call reuses the array the first one left behind) and that an
oversized batch is refused with an error instead of overrunning the array.

This file is named to be collected last so a run that stops at the first
failure has already run every other test; it also passes on its own.
Tolerance: fp32 1e-4 relative (tests/helpers.py).
"""
import ctypes

import numpy as np
import pytest

from helpers import assert_close

pytestmark = pytest.mark.gpu


def _ce(rnet, name, logits, tgt, N, V, torch):
    loss = torch.full((1,), -1.0, device="cuda")
    dl = torch.full((N, V), 7.0, device="cuda")
    rnet.call(name, rnet.ptr(logits), rnet.ptr(tgt), rnet.ptr(loss), rnet.ptr(dl), N, V, None)
    torch.cuda.synchronize()
    return float(loss.item()), dl.cpu().numpy()


def test_noalloc_cross_entropy_matches_regular(rnet, cuda):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(3)
    for N, V in ((16384, 256), (1000, 256)):  # large then smaller: stale scratch is reused
        logits = torch.randn(N, V, device="cuda", generator=g) * 3
        tgt = torch.randint(0, V, (N,), device="cuda", generator=g, dtype=torch.int32)
        l_ref, d_ref = _ce(rnet, "rnet_cross_entropy_forward", logits, tgt, N, V, torch)
        l_new, d_new = _ce(rnet, "rnet_cross_entropy_forward_noalloc", logits, tgt, N, V, torch)
        assert abs(l_new - l_ref) <= 1e-4 * abs(l_ref), (N, l_new, l_ref)
        assert_close(d_new, d_ref, what=f"dlogits N={N}")


def test_noalloc_cross_entropy_rejects_oversize(rnet, cuda):
    torch = cuda
    N, V = 8 * 65536, 4  # one partial more than the fixed array holds
    logits = torch.zeros(N, V, device="cuda")
    tgt = torch.zeros(N, dtype=torch.int32, device="cuda")
    loss = torch.zeros(1, device="cuda")
    dl = torch.zeros(N, V, device="cuda")
    rc = rnet.lib().rnet_cross_entropy_forward_noalloc(
        rnet.ptr(logits), rnet.ptr(tgt), rnet.ptr(loss), rnet.ptr(dl), N, V, None)
    assert rc == -1  # RNET_ERR_ARG
    assert b"scratch limit" in rnet.lib().rnet_last_error()
