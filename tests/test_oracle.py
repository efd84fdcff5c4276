"""CPU checks of the oracle itself (no GPU):

* known-answer tests from the reference's algorithm (scan limits, conv delta
  response, top-k tie and order rules, CE on uniform logits);
* finite-difference check of the oracle's whole-model gradients (exact
  gradient mode, conv_dmix quirk off);
* the quirk mode differs from the exact gradient exactly in the mix weights;
* the oracle against the golden fixtures recorded from the reference's own
  CUDA build (tests/golden/make_golden.py).
"""
import ctypes
import math
import os

import numpy as np
import pytest

from helpers import FP32_TOL, assert_close, assert_grads_close, rel_err, topk_sets_match

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_topk_reference_order_and_ties(orc):
    # Hand-worked from the reference rule (replace the first minimum of the
    # held pair when strictly greater; held starts at (-1e30, idx 0) x 2):
    rows = np.array([
        [1, 3, 3, 2],      # -> held slot0=idx2, slot1=idx1 (tie 3/3 keeps first-seen in slot1)
        [5, 5, 5, 5],      # -> idx 0 then 1; later equal values never replace
        [4, 3, 2, 1],      # -> (0, 1) in positional order
        [1, 2, 3, 4],      # -> slot0 gets 2 then 3... final (2, 3)? worked below
    ], np.float32)
    N, S, k = rows.shape[0], rows.shape[1], 2
    idx = np.zeros((N, k), np.int32)
    w = np.zeros((N, k), np.float32)
    orc.lib().orc_topk_rows(_p(rows), N, S, k, _p(idx), _p(w))
    # row 3: i0: held=(1,-1e30)->m=1? held1<held0 -> m=1: held1=... step through:
    #   v=1: held=(-1e30,-1e30) m=0 -> held0=1(i0)
    #   v=2: held1<held0 -> m=1 -> held1=2(i1)
    #   v=3: held0(1)<held1? m = (held1 < held0) ? 1 : 0 = 0 -> held0=3(i2)
    #   v=4: held1(2) < held0(3) -> m=1 -> held1=4(i3)
    np.testing.assert_array_equal(idx, [[2, 1], [0, 1], [0, 1], [2, 3]])
    e = math.exp(-1.0)
    np.testing.assert_allclose(w[3], [e / (1 + e), 1 / (1 + e)], rtol=1e-6)
    np.testing.assert_allclose(w[1], [0.5, 0.5], rtol=1e-6)


def test_cross_entropy_uniform_logits(orc):
    N, V = 5, 256
    lg = np.zeros((N, V), np.float32)
    tgt = np.arange(N, dtype=np.int32)
    loss = ctypes.c_float(0)
    dl = np.zeros_like(lg)
    orc.lib().orc_cross_entropy(_p(lg), _p(tgt), ctypes.byref(loss), _p(dl), N, V)
    assert abs(loss.value - N * math.log(V)) < 1e-4
    assert abs(dl[0, 0] - (1 / V - 1)) < 1e-7 and abs(dl[0, 1] - 1 / V) < 1e-7


def test_scan_limits(orc):
    B, T, D = 2, 37, 8
    r = np.random.default_rng(0)
    x = r.normal(size=(B * T, D)).astype(np.float32)
    Wz = np.zeros((D, D), np.float32)
    Wh = r.normal(size=(D, D)).astype(np.float32)
    bh = r.normal(size=D).astype(np.float32)
    y, z, h = (np.zeros((B * T, D), np.float32) for _ in range(3))
    # z == 1 (bz large): h_t = h~_t
    bz = np.full(D, 60.0, np.float32)
    orc.lib().orc_gru_fwd(_p(x), _p(y), _p(Wz), _p(Wh), _p(bz), _p(bh), _p(z), _p(h), B, T, D)
    np.testing.assert_allclose(h, x @ Wh.T + bh, rtol=1e-5, atol=1e-5)
    # z == 0 (bz very negative): h stays 0
    bz = np.full(D, -60.0, np.float32)
    orc.lib().orc_gru_fwd(_p(x), _p(y), _p(Wz), _p(Wh), _p(bz), _p(bh), _p(z), _p(h), B, T, D)
    assert np.abs(h).max() < 1e-20


def test_conv_delta_returns_taps(orc):
    B, T, D = 1, 20, 4
    x = np.zeros((T, D), np.float32)
    x[0, :] = 1.0  # unit impulse at t = 0 in every channel
    r = np.random.default_rng(1)
    w3, w7, w15 = (r.normal(size=(k, D)).astype(np.float32) for k in (3, 7, 15))
    mix = np.eye(D, dtype=np.float32)
    y = np.zeros_like(x)
    cb = np.zeros((3, T, D), np.float32)
    orc.lib().orc_conv_fwd(_p(x), _p(y), _p(w3), _p(w7), _p(w15), _p(mix), _p(cb), B, T, D)
    # c_K[t] = w_K[K-1-t] for t < K: the impulse response is the reversed taps
    np.testing.assert_allclose(cb[1][:7], w7[::-1], rtol=1e-6)
    np.testing.assert_allclose(cb[2][:15], w15[::-1], rtol=1e-6)
    S = np.zeros((T, D), np.float32)
    S[:3] += w3[::-1]
    S[:7] += w7[::-1]
    S[:15] += w15[::-1]
    np.testing.assert_allclose(y, S, rtol=1e-5, atol=1e-6)


def _tiny(orc, rdata, std):
    cfg = orc.make_config(d_model=16, n_layers=2, d_ff=24, n_slots=8, top_k=2, vocab=16,
                          seq_len=9)
    params = rdata.init_params_normal(cfg, seed=3, std=std)
    r = np.random.default_rng(2)
    tok = r.integers(0, 16, size=(2, 9)).astype(np.int32)
    tgt = r.integers(0, 16, size=(2, 9)).astype(np.int32)
    return cfg, params, tok, tgt


def _loss(orc, cfg, params, tok, tgt):
    g = np.zeros_like(params)
    l = ctypes.c_float(0)
    orc.lib().orc_grads(ctypes.byref(cfg), _p(params), _p(g), _p(tok), _p(tgt), 2, 9, 0,
                        ctypes.byref(l))
    return l.value / 18.0, g


def test_finite_difference_gradients(orc, rdata):
    cfg, params, tok, tgt = _tiny(orc, rdata, std=0.3)
    params64 = params.astype(np.float64)
    _, g = _loss(orc, cfg, params, tok, tgt)
    r = np.random.default_rng(11)
    layout = rdata.tensor_layout(cfg)
    offs = np.cumsum([0] + [n for _, n in layout])
    checked = 0
    for ti, (name, n) in enumerate(layout):
        for j in r.choice(n, size=min(n, 3), replace=False):
            i = offs[ti] + j
            eps = 3e-3 * max(1.0, abs(params64[i]))
            pp, pm = params.copy(), params.copy()
            pp[i] += eps
            pm[i] -= eps
            lp, _ = _loss(orc, cfg, pp, tok, tgt)
            lm, _ = _loss(orc, cfg, pm, tok, tgt)
            fd = (lp - lm) / (2 * eps)
            # fp32 storage inside the forward bounds the FD accuracy
            assert abs(fd - g[i]) <= 2e-2 * max(abs(fd), abs(g[i])) + 2e-5, \
                f"{name}[{j}]: fd {fd:.6e} vs analytic {g[i]:.6e}"
            checked += 1
    assert checked > 50


def test_conv_quirk_only_changes_mix_gradient(orc, rdata):
    cfg, params, tok, tgt = _tiny(orc, rdata, std=0.3)
    outs = {}
    for q in (0, 1):
        g = np.zeros_like(params)
        l = ctypes.c_float(0)
        orc.lib().orc_grads(ctypes.byref(cfg), _p(params), _p(g), _p(tok), _p(tgt), 2, 9, q,
                            ctypes.byref(l))
        outs[q] = g
    parts0 = rdata.split(cfg, outs[0])
    parts1 = rdata.split(cfg, outs[1])
    # the quirk only changes which buffer the mix-weight gradient reads
    # (src/causal_conv.cu:155-168); no other gradient depends on it
    for name in parts0:
        same = np.array_equal(parts0[name], parts1[name])
        assert same != name.endswith(".mix"), name


@pytest.mark.parametrize("case", ["cfg_tiny", "cfg_small"])
def test_oracle_matches_reference_golden(case, orc, rdata):
    path = os.path.join(GOLDEN, f"{case}.npz")
    if not os.path.exists(path):
        pytest.skip("golden fixture not generated")
    g = np.load(path)
    c = g["config"]
    cfg = orc.make_config(int(c[0]), int(c[1]), int(c[2]), int(c[5]), int(c[6]), int(c[7]),
                          seq_len=int(c[8]))
    B, T = int(g["B"]), int(g["T"])
    out = orc.train_step(cfg, g["params"], g["tokens"], g["targets"], B, T, float(g["lr"]),
                         float(g["clip"]), quirk=1)
    assert abs(out["loss_sum"] - float(g["loss_sum"])) <= FP32_TOL * abs(float(g["loss_sum"]))
    assert_close(out["logits"], g["logits"], what="logits")
    margins = orc.topk_margins(cfg, g["params"], g["tokens"], B, T)
    assert topk_sets_match(out["topk_idx"], g["topk_idx"], margins).all()
    assert_grads_close(cfg, out["grads"], g["grads"], rdata.tensor_layout, what="oracle grads")
    d0 = out["params"].astype(np.float64) - g["params"]
    d1 = g["params_after"].astype(np.float64) - g["params"]
    assert rel_err(d0, d1) <= FP32_TOL


def test_forced_selection_hook(orc, rdata):
    """train_step(forced=...) overrides only rows inside the tie band whose
    selected set differs; with its own choices nothing changes."""
    cfg = orc.make_config(64, 1, 128, 64, 2, 256, seq_len=32)
    params = rdata.init_params_normal(cfg, seed=1234)
    tok, tgt = rdata.uniform_tokens(2, 32, seed=1)
    a = orc.train_step(cfg, params, tok, tgt, 2, 32)
    b = orc.train_step(cfg, params, tok, tgt, 2, 32, forced=a["topk_idx"], tau=1e30)
    assert b["n_forced"] == 0
    np.testing.assert_array_equal(a["grads"], b["grads"])
    f = a["topk_idx"].copy()
    f[0, 5] = [(f[0, 5, 0] + 1) % 64 if (f[0, 5, 0] + 1) % 64 != f[0, 5, 1] else
               (f[0, 5, 0] + 2) % 64, f[0, 5, 1]]
    c = orc.train_step(cfg, params, tok, tgt, 2, 32, forced=f, tau=0.0)
    assert c["n_forced"] == 0  # outside the band: not overridden
    d = orc.train_step(cfg, params, tok, tgt, 2, 32, forced=f, tau=1e30)
    assert d["n_forced"] == 1
    np.testing.assert_array_equal(d["topk_idx"][0, 5], f[0, 5])
    assert not np.array_equal(d["grads"], a["grads"])
