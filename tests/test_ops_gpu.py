"""Per-operation parity on the GPU: every C-ABI layer op (the reference's
include/layers.h surface) against the CPU oracle on the same seeded inputs.
Includes ragged shapes (T not a multiple of the 32-step scan chunk, slot
counts not a multiple of the 128-wide tile, tiny batches).

Tolerance: fp32, 1e-4 relative (tests/helpers.py); top-k bit-exact as sets
except selection margins < 1e-6.
"""
import ctypes

import numpy as np
import pytest

from helpers import assert_close

pytestmark = pytest.mark.gpu

F32 = ctypes.c_float


def _rng(seed):
    return np.random.default_rng(seed)


def _t(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _np(t):
    return t.detach().cpu().numpy()


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


@pytest.fixture(params=[0, 1], ids=["auto", "cg1"])
def cta_group(request, rnet):
    """GEMM tile shape: automatic (CTA pairs once M > 128) or single-CTA."""
    rnet.call("rnet_gemm_set_cta_group", request.param)
    yield request.param
    rnet.call("rnet_gemm_set_cta_group", 0)


# (1003, 256) and (13, 512): staged backward with a last 8-row group of 3 and 5 rows
@pytest.mark.parametrize("N,D", [(64, 64), (1000, 512), (7, 2048), (1003, 256), (13, 512),
                                 (3000, 2048), (999, 1024)])
def test_rms_norm(rnet, orc, cuda, N, D):
    torch = cuda
    r = _rng(N + D)
    x = r.normal(size=(N, D)).astype(np.float32)
    w = (1 + 0.1 * r.normal(size=D)).astype(np.float32)
    dy = r.normal(size=(N, D)).astype(np.float32)
    y0 = np.zeros_like(x); ri0 = np.zeros(N, np.float32)
    orc.lib().orc_rms_norm_fwd(_p(x), _p(w), _p(y0), _p(ri0), N, D, F32(1e-6))
    dx0 = np.zeros_like(x); dw0 = np.full(D, 0.5, np.float32)
    orc.lib().orc_rms_norm_bwd(_p(dy), _p(x), _p(w), _p(ri0), _p(dx0), _p(dw0), N, D)
    X, W, DY = _t(torch, x), _t(torch, w), _t(torch, dy)
    Y = torch.zeros_like(X); RI = torch.zeros(N, device="cuda")
    rnet.call("rnet_rms_norm_forward", rnet.ptr(X), rnet.ptr(W), rnet.ptr(Y), rnet.ptr(RI), N, D,
              F32(1e-6), None)
    DX = torch.zeros_like(X); DW = torch.full((D,), 0.5, device="cuda")
    rnet.call("rnet_rms_norm_backward", rnet.ptr(DY), rnet.ptr(X), rnet.ptr(W), rnet.ptr(RI),
              rnet.ptr(DX), rnet.ptr(DW), N, D, None)
    torch.cuda.synchronize()
    assert_close(_np(Y), y0, what="rms y")
    assert_close(_np(RI), ri0, what="rms rinv")
    assert_close(_np(DX), dx0, what="rms dx")
    assert_close(_np(DW), dw0, what="rms dw")


# (1, 300, 100): channel tail and ragged last segment; (1, 5, 1024): fewer
# tiles than SMs; (32, 256, 512): CTA tile ranges that straddle channel groups.
@pytest.mark.parametrize("B,T,D", [(2, 32, 64), (3, 100, 64), (4, 256, 512), (1, 5, 128),
                                   (1, 300, 100), (1, 5, 1024), (32, 256, 512)])
@pytest.mark.parametrize("quirk", [1, 0])
def test_causal_conv(rnet, orc, cuda, B, T, D, quirk):
    torch = cuda
    r = _rng(B * T + D + quirk)
    N = B * T
    x = r.normal(size=(N, D)).astype(np.float32)
    w3, w7, w15 = (r.normal(scale=0.3, size=(k, D)).astype(np.float32) for k in (3, 7, 15))
    mix = r.normal(scale=D ** -0.5, size=(D, D)).astype(np.float32)
    dy = r.normal(size=(N, D)).astype(np.float32)
    y0 = np.zeros_like(x); cb0 = np.zeros((3, N, D), np.float32)
    orc.lib().orc_conv_fwd(_p(x), _p(y0), _p(w3), _p(w7), _p(w15), _p(mix), _p(cb0), B, T, D)
    dx0 = np.full_like(x, 0.25)
    g3, g7, g15 = (np.full((k, D), 0.1, np.float32) for k in (3, 7, 15))
    gm = np.full((D, D), 0.1, np.float32)
    orc.lib().orc_conv_bwd(_p(dy), _p(x), _p(w3), _p(w7), _p(w15), _p(mix), _p(cb0), _p(dx0),
                           _p(g3), _p(g7), _p(g15), _p(gm), B, T, D, quirk)
    X, Y, CB = _t(torch, x), torch.zeros(N, D, device="cuda"), torch.zeros(3, N, D, device="cuda")
    W3, W7, W15, MX = (_t(torch, a) for a in (w3, w7, w15, mix))
    rnet.call("rnet_causal_conv_forward", *(rnet.ptr(a) for a in (X, Y, W3, W7, W15, MX, CB)), B,
              T, D, None)
    DX = torch.full((N, D), 0.25, device="cuda")
    G3, G7, G15 = (torch.full((k, D), 0.1, device="cuda") for k in (3, 7, 15))
    GM = torch.full((D, D), 0.1, device="cuda")
    rnet.call("rnet_causal_conv_backward",
              *(rnet.ptr(a) for a in (_t(torch, dy), X, W3, W7, W15, MX, CB, DX, G3, G7, G15, GM)),
              B, T, D, quirk, None)
    torch.cuda.synchronize()
    assert_close(_np(Y), y0, what="conv y")
    assert_close(_np(CB), cb0, what="conv_buf")
    assert_close(_np(DX), dx0, what="conv dx")
    for a, b, n in ((G3, g3, "dw3"), (G7, g7, "dw7"), (G15, g15, "dw15"), (GM, gm, "dmix")):
        assert_close(_np(a), b, what=n)


@pytest.mark.parametrize("B,T,D", [(2, 32, 64), (3, 100, 64), (2, 600, 128), (64, 256, 512)])
def test_min_gru(rnet, orc, cuda, B, T, D):
    torch = cuda
    r = _rng(B + T + D)
    N = B * T
    x = r.normal(size=(N, D)).astype(np.float32)
    Wz, Wh = (r.normal(scale=D ** -0.5, size=(D, D)).astype(np.float32) for _ in range(2))
    bz, bh = (r.normal(scale=0.5, size=D).astype(np.float32) for _ in range(2))
    dy = r.normal(size=(N, D)).astype(np.float32)
    y0, z0, h0 = (np.zeros_like(x) for _ in range(3))
    orc.lib().orc_gru_fwd(_p(x), _p(y0), _p(Wz), _p(Wh), _p(bz), _p(bh), _p(z0), _p(h0), B, T, D)
    dx0 = np.zeros_like(x)
    gz, gh = np.zeros((D, D), np.float32), np.zeros((D, D), np.float32)
    gbz, gbh = np.zeros(D, np.float32), np.zeros(D, np.float32)
    orc.lib().orc_gru_bwd(_p(dy), _p(x), _p(Wz), _p(Wh), _p(bz), _p(bh), _p(z0), _p(h0), _p(dx0),
                          _p(gz), _p(gh), _p(gbz), _p(gbh), B, T, D)
    X = _t(torch, x)
    T_ = [_t(torch, a) for a in (Wz, Wh, bz, bh)]
    Y, Z, H = (torch.zeros(N, D, device="cuda") for _ in range(3))
    rnet.call("rnet_min_gru_forward", rnet.ptr(X), rnet.ptr(Y), *(rnet.ptr(a) for a in T_),
              rnet.ptr(Z), rnet.ptr(H), B, T, D, None)
    DX = torch.zeros(N, D, device="cuda")
    GZ, GH = torch.zeros(D, D, device="cuda"), torch.zeros(D, D, device="cuda")
    GBZ, GBH = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
    rnet.call("rnet_min_gru_backward", rnet.ptr(_t(torch, dy)), rnet.ptr(X),
              *(rnet.ptr(a) for a in T_), rnet.ptr(Z), rnet.ptr(H), rnet.ptr(DX), rnet.ptr(GZ),
              rnet.ptr(GH), rnet.ptr(GBZ), rnet.ptr(GBH), B, T, D, None)
    torch.cuda.synchronize()
    assert_close(_np(Y), y0, what="gru y")
    assert_close(_np(Z), z0, what="gru z")
    assert_close(_np(H), h0, what="gru h")
    assert_close(_np(DX), dx0, what="gru dx")
    for a, b, n in ((GZ, gz, "dWz"), (GH, gh, "dWh"), (GBZ, gbz, "dbz"), (GBH, gbh, "dbh")):
        assert_close(_np(a), b, what=n)


@pytest.mark.parametrize("B,T,D,S", [(2, 32, 64, 64), (3, 100, 64, 160), (4, 128, 512, 1024)])
def test_slot_memory(rnet, orc, cuda, cta_group, B, T, D, S):
    torch = cuda
    r = _rng(B * T + S)
    N, k = B * T, 2
    x = r.normal(size=(N, D)).astype(np.float32)
    keys, vals = (r.normal(scale=D ** -0.5, size=(D, S)).astype(np.float32) for _ in range(2))
    pq, po = (r.normal(scale=D ** -0.5, size=(D, D)).astype(np.float32) for _ in range(2))
    dy = r.normal(size=(N, D)).astype(np.float32)
    y0, q0 = np.zeros_like(x), np.zeros_like(x)
    sc0 = np.zeros((N, S), np.float32)
    i0 = np.zeros((N, k), np.int32); w0 = np.zeros((N, k), np.float32)
    orc.lib().orc_slot_fwd(_p(x), _p(y0), _p(keys), _p(vals), _p(pq), _p(po), _p(q0), _p(sc0),
                           _p(i0), _p(w0), B, T, D, S, k)
    X = _t(torch, x)
    KV = [_t(torch, a) for a in (keys, vals, pq, po)]
    Y, Q = torch.zeros(N, D, device="cuda"), torch.zeros(N, D, device="cuda")
    SC = torch.zeros(N, S, device="cuda")
    I = torch.zeros(N, k, dtype=torch.int32, device="cuda")
    W = torch.zeros(N, k, device="cuda")
    rnet.call("rnet_slot_memory_forward", rnet.ptr(X), rnet.ptr(Y), *(rnet.ptr(a) for a in KV),
              rnet.ptr(Q), rnet.ptr(SC), rnet.ptr(I), rnet.ptr(W), B, T, D, S, k, None)
    torch.cuda.synchronize()
    assert_close(_np(Q), q0, what="slot q")
    assert_close(_np(SC), sc0, what="slot scores")
    # selection margins from the oracle's scores
    srt = np.sort(sc0, axis=1)
    margin = np.minimum(srt[:, -2] - srt[:, -3], srt[:, -1] - srt[:, -2])
    ours_i = np.sort(_np(I), axis=1)
    ref_i = np.sort(i0, axis=1)
    bad = np.any(ours_i != ref_i, axis=1) & (margin >= 1e-6)
    assert not bad.any(), f"top-2 mismatch on {bad.sum()} tokens"
    assert_close(_np(Y), y0, what="slot y")
    # backward from the SAME cached top-k on both sides
    I_np, W_np = _np(I).copy(), _np(W).copy()
    dx0 = np.zeros_like(x)
    gk, gv = np.zeros((D, S), np.float32), np.zeros((D, S), np.float32)
    gq, go = np.zeros((D, D), np.float32), np.zeros((D, D), np.float32)
    qn = _np(Q).copy()
    orc.lib().orc_slot_bwd(_p(dy), _p(x), _p(keys), _p(vals), _p(pq), _p(po), _p(qn), _p(I_np),
                           _p(W_np), _p(dx0), _p(gk), _p(gv), _p(gq), _p(go), B, T, D, S, k)
    DX = torch.zeros(N, D, device="cuda")
    G = [torch.zeros(D, S, device="cuda"), torch.zeros(D, S, device="cuda"),
         torch.zeros(D, D, device="cuda"), torch.zeros(D, D, device="cuda")]
    rnet.call("rnet_slot_memory_backward", rnet.ptr(_t(torch, dy)), rnet.ptr(X),
              *(rnet.ptr(a) for a in KV), rnet.ptr(Q), rnet.ptr(SC), rnet.ptr(I), rnet.ptr(W),
              rnet.ptr(DX), *(rnet.ptr(a) for a in G), B, T, D, S, k, None)
    torch.cuda.synchronize()
    assert_close(_np(DX), dx0, what="slot dx")
    for a, b, n in zip(G, (gk, gv, gq, go), ("dkeys", "dvalues", "dproj_q", "dproj_out")):
        assert_close(_np(a), b, what=n)


@pytest.mark.parametrize("N,D,F", [(64, 64, 128), (300, 64, 192), (2048, 512, 1024)])
@pytest.mark.parametrize("contiguous", [True, False])
def test_swiglu(rnet, orc, cuda, cta_group, N, D, F, contiguous):
    torch = cuda
    r = _rng(N + D + F + contiguous)
    x = r.normal(size=(N, D)).astype(np.float32)
    gu = r.normal(scale=D ** -0.5, size=(2 * F, D)).astype(np.float32)
    gate, up = gu[:F].copy(), gu[F:].copy()
    down = r.normal(scale=F ** -0.5, size=(D, F)).astype(np.float32)
    dy = r.normal(size=(N, D)).astype(np.float32)
    y0 = np.zeros_like(x); gc0 = np.zeros((N, F), np.float32); uc0 = np.zeros((N, F), np.float32)
    orc.lib().orc_swiglu_fwd(_p(x), _p(y0), _p(gate), _p(up), _p(down), _p(gc0), _p(uc0), N, D, F)
    dx0 = np.zeros_like(x)
    gg, gup, gd = np.zeros((F, D), np.float32), np.zeros((F, D), np.float32), np.zeros((D, F), np.float32)
    orc.lib().orc_swiglu_bwd(_p(dy), _p(x), _p(gate), _p(up), _p(down), _p(gc0), _p(uc0), _p(dx0),
                             _p(gg), _p(gup), _p(gd), N, D, F)
    X = _t(torch, x)
    if contiguous:
        GU = _t(torch, gu)
        GATE, UP = GU[:F], GU[F:]
    else:
        GATE, UP = _t(torch, gate), _t(torch, up)
    DOWN = _t(torch, down)
    Y = torch.zeros(N, D, device="cuda")
    GC, UC = torch.zeros(N, F, device="cuda"), torch.zeros(N, F, device="cuda")
    rnet.call("rnet_swiglu_forward", rnet.ptr(X), rnet.ptr(Y), rnet.ptr(GATE), rnet.ptr(UP),
              rnet.ptr(DOWN), rnet.ptr(GC), rnet.ptr(UC), N, D, F, None)
    DX = torch.zeros(N, D, device="cuda")
    DG, DU, DD = torch.zeros(F, D, device="cuda"), torch.zeros(F, D, device="cuda"), torch.zeros(D, F, device="cuda")
    rnet.call("rnet_swiglu_backward", rnet.ptr(_t(torch, dy)), rnet.ptr(X), rnet.ptr(GATE),
              rnet.ptr(UP), rnet.ptr(DOWN), rnet.ptr(GC), rnet.ptr(UC), rnet.ptr(DX), rnet.ptr(DG),
              rnet.ptr(DU), rnet.ptr(DD), N, D, F, None)
    torch.cuda.synchronize()
    assert_close(_np(Y), y0, what="ffn y")
    assert_close(_np(GC), gc0, what="gate cache")
    assert_close(_np(UC), uc0, what="up cache")
    assert_close(_np(DX), dx0, what="ffn dx")
    for a, b, n in ((DG, gg, "dgate"), (DU, gup, "dup"), (DD, gd, "ddown")):
        assert_close(_np(a), b, what=n)


@pytest.mark.parametrize("N,V,D", [(64, 256, 64), (4096, 256, 512)])
def test_embed_ce_linear(rnet, orc, cuda, N, V, D):
    torch = cuda
    r = _rng(N + V)
    tok = r.integers(0, V, N).astype(np.int32)
    tgt = r.integers(0, V, N).astype(np.int32)
    table = r.normal(size=(V, D)).astype(np.float32)
    W = r.normal(scale=D ** -0.5, size=(V, D)).astype(np.float32)
    e0 = np.zeros((N, D), np.float32)
    orc.lib().orc_embed_fwd(_p(tok), _p(table), _p(e0), N, D)
    lg0 = np.zeros((N, V), np.float32)
    orc.lib().orc_linear(_p(e0), _p(W), _p(lg0), N, V, D)
    loss0 = F32(0); dl0 = np.zeros_like(lg0)
    orc.lib().orc_cross_entropy(_p(lg0), _p(tgt), ctypes.byref(loss0), _p(dl0), N, V)
    dt0 = np.full((V, D), 0.5, np.float32)
    dout = r.normal(size=(N, D)).astype(np.float32)
    orc.lib().orc_embed_bwd(_p(dout), _p(tok), _p(dt0), N, V, D)
    TOK, TGT, TAB, WW = _t(torch, tok), _t(torch, tgt), _t(torch, table), _t(torch, W)
    E = torch.zeros(N, D, device="cuda"); LG = torch.zeros(N, V, device="cuda")
    rnet.call("rnet_embed_forward", rnet.ptr(TOK), rnet.ptr(TAB), rnet.ptr(E), N, V, D, None)
    rnet.call("rnet_linear_forward", rnet.ptr(E), rnet.ptr(WW), rnet.ptr(LG), N, V, D, None)
    L = torch.full((1,), 7.0, device="cuda"); DL = torch.zeros(N, V, device="cuda")
    rnet.call("rnet_cross_entropy_forward", rnet.ptr(LG), rnet.ptr(TGT), rnet.ptr(L), rnet.ptr(DL),
              N, V, None)
    DT = torch.full((V, D), 0.5, device="cuda")
    rnet.call("rnet_embed_backward", rnet.ptr(_t(torch, dout)), rnet.ptr(TOK),
              rnet.ptr(DT), N, V, D, None)
    torch.cuda.synchronize()
    assert_close(_np(E), e0, what="embed")
    assert_close(_np(LG), lg0, what="logits")
    assert abs(L.item() - loss0.value) <= 1e-4 * abs(loss0.value)
    assert_close(_np(DL), dl0, what="dlogits")
    assert_close(_np(DT), dt0, what="dtable")
