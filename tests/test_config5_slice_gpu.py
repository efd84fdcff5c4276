"""Parity on a reduced slice of config 5: the scaled model's layer shapes
(d_model 2048, d_ff 5632, 8192 slots, top-2, vocab 256) with one layer and
one 2048-token sequence, N(0,0.02) weights (seed 4321), Zipf bytes (seed 9).

  * bf16 mode (config 5's arithmetic) against the reference's own CUDA build
    (fp32) and the fp64 oracle: loss, whole gradient, every gradient tensor
    off the slot path, and the SGD update within 2e-2; top-2 sets agree on
    >= 99.9 % of tokens whose margin exceeds 2e-2 of the row's largest score.
  * fp32 mode against the oracle at 1e-4 (loss, every gradient tensor, the
    update), with the oracle taking the engine's slot on rows inside the
    2e-6 tie band, as in the config-2 test.
  * recompute on/off give the same step at this size.

The full config 5 (24 layers, B16 x T2048 per GPU) is not runnable on the
reference (its layer cache is sized from free memory,
src/resonance_net.cpp:91-101, yet used whenever N <= 64*seq_len,
src/resonance_net.cpp:245); it is measured by bench.py --model c5.
"""
import numpy as np
import pytest

from helpers import FP32_TOL, rel_err, topk_sets_match, update_rel_err
from test_config2_parity_gpu import SLOT_PATH, TIE, _engine_step, _print_worst, _tensor_errs

pytestmark = pytest.mark.gpu

C5 = dict(d_model=2048, n_layers=1, d_ff=5632, n_slots=8192, top_k=2, vocab=256)
B, T = 1, 2048
BF16_TOL = 2e-2


@pytest.fixture(scope="module")
def setup(rnet, rdata, orc, cuda):
    assert orc.ref_available(), "oracle/_ref/libref.so (the reference build) is missing"
    ocfg = orc.make_config(**C5, seq_len=T)
    rcfg = rnet.ModelConfig.make(**C5, seq_len=T)
    params = rdata.init_params_normal(rcfg, seed=4321)
    tok, tgt = rdata.zipf_tokens(B, T, seed=9)
    return ocfg, rcfg, params, tok, tgt


@pytest.fixture(scope="module")
def reference(setup, rdata, orc, tmp_path_factory):
    ocfg, rcfg, params, tok, tgt = setup
    path = str(tmp_path_factory.mktemp("c5") / "init.bin")
    rdata.write_checkpoint(path, rcfg, params)
    ref = orc.RefModel.from_checkpoint(path)
    N = B * T
    loss = ref.train_step(tok, tgt, B, T, 3e-4, 1.0)
    idx, w = ref.topk(ocfg.n_layers, N, ocfg.slot_top_k)
    sc = ref.scores(0, N, ocfg.n_slots)
    out = dict(loss_sum=loss, grads=ref.grads(), params_after=ref.params(), topk_idx=idx,
               margins=orc.margins_from_scores(sc, 2)[None], score_scale=np.abs(sc).max(1)[None])
    ref.close()
    return out


@pytest.fixture(scope="module")
def ours_fp32(setup, rnet, cuda):
    ocfg, rcfg, params, tok, tgt = setup
    return _engine_step(rnet, cuda, rcfg, params, tok, tgt, B, T)


@pytest.fixture(scope="module")
def oracle_step(setup, orc, ours_fp32):
    ocfg, rcfg, params, tok, tgt = setup
    return orc.train_step(ocfg, params, tok, tgt, B, T, 3e-4, 1.0, quirk=1,
                          forced=ours_fp32["topk_idx"], tau=TIE)


def test_config5_slice_fp32_vs_oracle(setup, ours_fp32, oracle_step, rdata):
    ocfg, rcfg, params, tok, tgt = setup
    ours, orc_ = ours_fp32, oracle_step
    print(f"\n[config5 slice fp32] loss ours {ours['loss_sum']:.4f} oracle {orc_['loss_sum']:.4f};"
          f" in-band rows with the engine's slots: {orc_['n_forced']}")
    assert orc_["n_forced"] <= max(2, 1e-3 * B * T)
    assert topk_sets_match(ours["topk_idx"], orc_["topk_idx"]).all()
    assert abs(ours["loss_sum"] - orc_["loss_sum"]) <= FP32_TOL * abs(orc_["loss_sum"])
    errs = _tensor_errs(rcfg, rdata, ours["grads"], orc_["grads"])
    _print_worst("config5 slice fp32 vs oracle", errs)
    assert not {n: e for n, e in errs.items() if e > FP32_TOL}
    assert update_rel_err(params, ours["params_after"], orc_["params_after"]) <= FP32_TOL


def test_config5_slice_bf16(setup, reference, oracle_step, rnet, rdata, cuda):
    ocfg, rcfg, params, tok, tgt = setup
    ours = _engine_step(rnet, cuda, rcfg, params, tok, tgt, B, T, bf16=True)
    for name, other in (("reference", reference), ("oracle", oracle_step)):
        assert abs(ours["loss_sum"] - other["loss_sum"]) <= BF16_TOL * abs(other["loss_sum"])
        g = rel_err(ours["grads"], other["grads"])
        errs = _tensor_errs(rcfg, rdata, ours["grads"], other["grads"])
        _print_worst(f"config5 slice bf16 vs {name} (whole gradient {g:.2e})", errs)
        assert 1e-5 < g <= BF16_TOL
        bad = {n: e for n, e in errs.items()
               if e > BF16_TOL and n.split(".")[-1] not in SLOT_PATH}
        assert not bad, f"tensors over 2e-2 vs {name}: {bad}"
        u = rel_err(ours["params_after"].astype(np.float64) - params,
                    other["params_after"].astype(np.float64) - params)
        assert u <= BF16_TOL, f"update rel {u:.3e} vs {name}"
    ok = topk_sets_match(ours["topk_idx"], reference["topk_idx"]).reshape(
        reference["margins"].shape)
    keep = reference["margins"] >= BF16_TOL * reference["score_scale"]
    print(f"[config5 slice bf16] top-2 agreement outside near-ties {ok[keep].mean():.5f} "
          f"({keep.sum()} tokens)")
    assert ok[keep].mean() >= 0.999


def test_config5_slice_recompute(setup, ours_fp32, rnet, cuda):
    """bf16 + recompute (the config-5 bench settings) at two layers of the
    config-5 shapes gives the step of bf16 with full caches."""
    torch = cuda
    ocfg, rcfg, params, tok, tgt = setup
    rdata = __import__("importlib").import_module("resonance-net_b200.data")
    cfg2 = rnet.ModelConfig.make(**{**C5, "n_layers": 2}, seq_len=T)
    p2 = rdata.init_params_normal(cfg2, seed=77)
    d_in = torch.from_numpy(tok.reshape(-1)).cuda()
    d_tgt = torch.from_numpy(tgt.reshape(-1)).cuda()
    outs = []
    for rec in (False, True):
        m = rnet.Model(cfg2, device=0, reference_init=False)
        m.set_params(p2)
        m.set_precision(True)
        m.set_recompute(rec)
        loss = torch.zeros(1, device="cuda")
        m.train_step(d_in, d_tgt, B, T, 3e-4, 1.0, loss)
        m.synchronize()
        outs.append((float(loss.item()), m.get_grads()))
        m.close()
    assert outs[0][0] == outs[1][0]
    assert rel_err(outs[1][1], outs[0][1]) <= 1e-6
