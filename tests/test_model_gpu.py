"""Whole-model parity on the GPU: one full training step of the CUDA engine
(through the C ABI) against the CPU oracle and against the golden fixtures
recorded from the reference's own CUDA build.

Tolerance: fp32, 1e-4 relative (per tensor, see tests/helpers.py); top-2
indices bit-exact as sets except tokens whose selection margin is < 1e-6.
"""
import os

import numpy as np
import pytest

from helpers import (FP32_TOL, assert_close, assert_grads_close, rel_err, topk_sets_match,
                     update_rel_err)

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

CASES = {
    "cfg_tiny": dict(d_model=64, n_layers=1, d_ff=128, n_slots=64, top_k=2, vocab=256, B=2, T=32,
                     pseed=1234, tseed=1),
    "cfg_small": dict(d_model=64, n_layers=2, d_ff=128, n_slots=160, top_k=2, vocab=256, B=3,
                      T=100, pseed=99, tseed=5),
}


def _run_engine(rnet, cuda, cfg, params, tok, tgt, B, T, lr=3e-4, clip=1.0, bf16=False):
    torch = cuda
    m = rnet.Model(cfg, device=0, reference_init=False)
    m.set_params(params)
    m.set_precision(bf16)
    d_in = torch.from_numpy(tok.reshape(-1)).cuda()
    d_tgt = torch.from_numpy(tgt.reshape(-1)).cuda()
    loss = torch.zeros(1, device="cuda")
    m.train_step(d_in, d_tgt, B, T, lr, clip, loss)
    m.synchronize()
    N = B * T
    tk = [m.topk_host(l, N) for l in range(cfg.n_layers)]
    out = dict(loss_sum=float(loss.item()), grads=m.get_grads(), params_after=m.get_params(),
               topk_idx=np.stack([t[0] for t in tk]), topk_w=np.stack([t[1] for t in tk]))
    m.close()
    return out


def _make(orc, rdata, c):
    cfg = orc.make_config(c["d_model"], c["n_layers"], c["d_ff"], c["n_slots"], c["top_k"],
                          c["vocab"], seq_len=c["T"])
    params = rdata.init_params_normal(cfg, seed=c["pseed"])
    tok, tgt = rdata.uniform_tokens(c["B"], c["T"], seed=c["tseed"])
    return cfg, params, tok, tgt


def _rcfg(rnet, cfg):
    return rnet.ModelConfig(cfg.d_model, cfg.n_layers, cfg.d_ff, cfg.n_heads, cfg.gru_dim,
                            cfg.n_slots, cfg.slot_top_k, cfg.vocab_size, cfg.seq_len, cfg.rms_eps)


def _compare(cfg, rdata, ours, ref, params, margins, what):
    assert abs(ours["loss_sum"] - ref["loss_sum"]) <= FP32_TOL * abs(ref["loss_sum"]), \
        f"{what}: loss {ours['loss_sum']} vs {ref['loss_sum']}"
    ok = topk_sets_match(ours["topk_idx"], ref["topk_idx"], margins)
    assert ok.all(), f"{what}: top-k index sets differ on {(~ok).sum()} tokens"
    assert_grads_close(cfg, ours["grads"], ref["grads"], rdata.tensor_layout, what=what + " grads")
    d_ours = ours["params_after"].astype(np.float64) - params
    d_ref = ref["params_after"].astype(np.float64) - params
    assert rel_err(d_ours, d_ref) <= FP32_TOL, f"{what}: SGD update rel {rel_err(d_ours, d_ref):.3e}"


@pytest.mark.parametrize("case", list(CASES))
def test_train_step_vs_oracle(case, rnet, rdata, orc, cuda):
    c = CASES[case]
    cfg, params, tok, tgt = _make(orc, rdata, c)
    ours = _run_engine(rnet, cuda, _rcfg(rnet, cfg), params, tok, tgt, c["B"], c["T"])
    ref = orc.train_step(cfg, params, tok, tgt, c["B"], c["T"], 3e-4, 1.0, quirk=1)
    margins = orc.topk_margins(cfg, params, tok, c["B"], c["T"])
    _compare(cfg, rdata, ours, ref, params.astype(np.float64), margins, f"{case} vs oracle")


@pytest.mark.parametrize("case", list(CASES))
def test_train_step_vs_reference_golden(case, rnet, rdata, orc, cuda):
    path = os.path.join(GOLDEN, f"{case}.npz")
    if not os.path.exists(path):
        pytest.skip("golden fixture not generated")
    g = np.load(path)
    c = CASES[case]
    cfg, params, tok, tgt = _make(orc, rdata, c)
    np.testing.assert_array_equal(params, g["params"])
    np.testing.assert_array_equal(tok, g["tokens"])
    ours = _run_engine(rnet, cuda, _rcfg(rnet, cfg), params, tok, tgt, c["B"], c["T"])
    ref = {k: g[k] for k in ("grads", "params_after", "topk_idx", "topk_w")}
    ref["loss_sum"] = float(g["loss_sum"])
    margins = orc.topk_margins(cfg, params, tok, c["B"], c["T"])
    _compare(cfg, rdata, ours, ref, params.astype(np.float64), margins, f"{case} vs reference")


BF16_TOL = 2e-2


@pytest.mark.parametrize("case", list(CASES))
def test_train_step_bf16_vs_oracle(case, rnet, rdata, orc, cuda):
    """bf16 GEMM arithmetic (fp32 accumulation) against the fp64-accumulating
    oracle: loss, the whole gradient vector and the SGD update within 2e-2
    (norm-relative). Per-tensor and top-2 comparisons are not made: bf16
    score rounding flips slot choices on near-tie tokens, which moves the
    gradients of those slots' keys and values as a whole."""
    c = CASES[case]
    cfg, params, tok, tgt = _make(orc, rdata, c)
    ours = _run_engine(rnet, cuda, _rcfg(rnet, cfg), params, tok, tgt, c["B"], c["T"], bf16=True)
    ref = orc.train_step(cfg, params, tok, tgt, c["B"], c["T"], 3e-4, 1.0, quirk=1)
    assert abs(ours["loss_sum"] - ref["loss_sum"]) <= BF16_TOL * abs(ref["loss_sum"])
    g = rel_err(ours["grads"].astype(np.float64), ref["grads"])
    assert g <= BF16_TOL, f"{case}: bf16 gradient rel {g:.3e}"
    p64 = params.astype(np.float64)
    u = rel_err(ours["params_after"].astype(np.float64) - p64, ref["params_after"] - p64)
    assert u <= BF16_TOL, f"{case}: bf16 SGD update rel {u:.3e}"
    # the bf16 path really ran: its error is far above the fp32 path's
    assert g > 1e-5, f"{case}: gradient matches to {g:.1e}: bf16 arithmetic not in effect"


def test_train_step_host_matches_device_step(rnet, rdata, orc, cuda):
    """rnet_model_train_step_host (pinned host tokens in, loss out: the e2e
    path bench.py times) against rnet_model_train_step on device buffers:
    same kernels in the same order. The first step gives the same loss bit
    for bit; parameters agree up to the summation order of the atomically
    accumulated gradients (embedding and slot-table scatter), so updates
    agree within 1e-5 and later losses within 1e-6. The first step also
    matches the oracle."""
    torch = cuda
    c = dict(CASES["cfg_small"])
    cfg, params, tok, tgt = _make(orc, rdata, c)
    rcfg = _rcfg(rnet, cfg)
    B, T = c["B"], c["T"]
    a = rnet.Model(rcfg, device=0, reference_init=False)
    b = rnet.Model(rcfg, device=0, reference_init=False)
    a.set_params(params)
    b.set_params(params)
    d_in = torch.from_numpy(tok.reshape(-1)).cuda()
    d_tgt = torch.from_numpy(tgt.reshape(-1)).cuda()
    h_in = torch.from_numpy(tok.reshape(-1).copy()).pin_memory()
    h_tgt = torch.from_numpy(tgt.reshape(-1).copy()).pin_memory()
    loss = torch.zeros(1, device="cuda")
    for i in range(3):
        a.train_step(d_in, d_tgt, B, T, 3e-4, 1.0, loss)
        a.synchronize()
        lb = b.train_step_host(h_in, h_tgt, B, T, 3e-4, 1.0)
        if i == 0:  # same parameters in: the same loss bit for bit
            assert float(loss.item()) == lb, f"step {i}: loss {loss.item()} vs host {lb}"
        else:
            assert abs(float(loss.item()) - lb) <= 1e-6 * abs(lb), f"step {i}"
        pa, pb = a.get_params(), b.get_params()
        assert update_rel_err(params, pb, pa) <= 1e-5, f"step {i}"
        if i == 0:
            ref = orc.train_step(cfg, params, tok, tgt, B, T, 3e-4, 1.0, quirk=1)
            assert abs(lb - ref["loss_sum"]) <= FP32_TOL * abs(ref["loss_sum"])
            d = b.get_params().astype(np.float64) - params
            assert rel_err(d, ref["params_after"] - params) <= FP32_TOL
    # pageable (non-pinned) host buffers take the same path
    lp = b.train_step_host(tok.reshape(-1).copy(), tgt.reshape(-1).copy(), B, T, 3e-4, 1.0)
    a.train_step(d_in, d_tgt, B, T, 3e-4, 1.0, loss)
    a.synchronize()
    assert abs(float(loss.item()) - lp) <= 1e-6 * abs(lp)
    a.close()
    b.close()


def test_graph_replayed_step_matches_eager(rnet, rdata, orc, cuda, monkeypatch):
    """Single-GPU train steps replay a captured CUDA graph once the same
    (B, T, lr, clip, configuration) repeats; the inputs are copied into the
    engine's own buffers first. Against a model built with RNET_TRAIN_GRAPH=0
    (every step eager), over steps that alternate two batches and switch
    precision midway (a new key: one eager step, then a new capture), the
    losses agree within 1e-6 and the cumulative updates within 1e-5 (the
    atomically accumulated gradients differ only in summation order)."""
    torch = cuda
    c = dict(CASES["cfg_small"])
    cfg, params, tok, tgt = _make(orc, rdata, c)
    rcfg = _rcfg(rnet, cfg)
    B, T = c["B"], c["T"]
    a = rnet.Model(rcfg, device=0, reference_init=False)
    monkeypatch.setenv("RNET_TRAIN_GRAPH", "0")
    b = rnet.Model(rcfg, device=0, reference_init=False)
    monkeypatch.delenv("RNET_TRAIN_GRAPH")
    a.set_params(params)
    b.set_params(params)
    tok2, tgt2 = rdata.uniform_tokens(B, T, seed=17)
    batches = [(torch.from_numpy(x.reshape(-1)).cuda(), torch.from_numpy(y.reshape(-1)).cuda())
               for x, y in ((tok, tgt), (tok2, tgt2))]
    la, lb = torch.zeros(1, device="cuda"), torch.zeros(1, device="cuda")
    for i in range(8):
        if i == 5:
            a.set_precision(True)
            b.set_precision(True)
        d_in, d_tgt = batches[i % 2]
        a.train_step(d_in, d_tgt, B, T, 3e-4, 1.0, la)
        b.train_step(d_in, d_tgt, B, T, 3e-4, 1.0, lb)
        a.synchronize()
        b.synchronize()
        x, y = float(la.item()), float(lb.item())
        assert abs(x - y) <= 1e-6 * abs(y), f"step {i}: graph loss {x} vs eager {y}"
        pa, pb = a.get_params(), b.get_params()
        assert update_rel_err(params, pa, pb) <= 1e-5, f"step {i}: cumulative update"
    a.close()
    b.close()


@pytest.mark.parametrize("bf16", [False, True])
def test_recompute_matches_cached_step(rnet, rdata, orc, cuda, bf16):
    """Activation recompute (only layer inputs kept; each layer's caches
    rebuilt before its backward) gives the same step as full caches: same
    loss bit for bit, parameters within the atomic-order noise (1e-6)."""
    torch = cuda
    c = dict(CASES["cfg_small"])
    cfg, params, tok, tgt = _make(orc, rdata, c)
    rcfg = _rcfg(rnet, cfg)
    B, T = c["B"], c["T"]
    d_in = torch.from_numpy(tok.reshape(-1)).cuda()
    d_tgt = torch.from_numpy(tgt.reshape(-1)).cuda()
    outs = []
    for rec in (False, True):
        m = rnet.Model(rcfg, device=0, reference_init=False)
        m.set_params(params)
        m.set_precision(bf16)
        m.set_recompute(rec)
        loss = torch.zeros(1, device="cuda")
        for _ in range(2):
            m.train_step(d_in, d_tgt, B, T, 3e-4, 1.0, loss)
        m.synchronize()
        outs.append((float(loss.item()), m.get_grads(), m.get_params()))
        if rec:
            with pytest.raises(rnet.RnetError):
                m.topk_host(0, B * T)
        m.close()
    assert abs(outs[0][0] - outs[1][0]) <= 1e-6 * abs(outs[0][0])
    assert rel_err(outs[1][1], outs[0][1]) <= 1e-6
    assert update_rel_err(params, outs[1][2], outs[0][2]) <= 1e-5


def test_optimizer_extensions(rnet, rdata, orc, cuda):
    """Momentum, weight decay and linear warmup (rnet_model_set_optimizer)
    against a numpy restatement of the rule, step by step, using the step's
    own gradients (still in the gradient buffer after the step): clip on the
    raw gradient norm, lr_t = lr * min(1, (t+1)/warmup) * min(1, clip/||g||),
    v = mu v + g + wd p, p -= lr_t v. With all three off the step is the
    reference's SGD (checked against the oracle elsewhere)."""
    torch = cuda
    c = dict(CASES["cfg_tiny"])
    cfg, params, tok, tgt = _make(orc, rdata, c)
    rcfg = _rcfg(rnet, cfg)
    B, T = c["B"], c["T"]
    m = rnet.Model(rcfg, device=0, reference_init=False)
    m.set_params(params)
    mu, wd, warm, lr, clip = 0.9, 0.01, 3, 3e-3, 1.0
    m.set_optimizer(mu, wd, warm)
    d_in = torch.from_numpy(tok.reshape(-1)).cuda()
    d_tgt = torch.from_numpy(tgt.reshape(-1)).cuda()
    p = params.astype(np.float64)
    v = np.zeros_like(p)
    for t in range(5):
        m.train_step(d_in, d_tgt, B, T, lr, clip)
        g = m.get_grads().astype(np.float64)
        norm = np.linalg.norm(g)
        lr_t = lr * min(1.0, (t + 1) / warm) * (min(1.0, clip / norm) if norm > 0 else 1.0)
        v = mu * v + g + wd * p
        want = p - lr_t * v
        got = m.get_params().astype(np.float64)
        # one-ulp differences of the fp32 parameters are rounding, not the rule
        assert update_rel_err(p, got, want) <= 1e-4, f"step {t}"
        p = got  # continue from the library's fp32 parameters
    with pytest.raises(rnet.RnetError):
        m.set_optimizer(1.5, 0.0, 0)
    m.close()
