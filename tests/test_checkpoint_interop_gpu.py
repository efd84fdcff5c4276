"""Drop-in interoperability with the reference itself (GPU):

  * a checkpoint the library writes loads into the reference's ResonanceNet
    (oracle/_ref/libref.so, src/resonance_net.cpp:784-824) with bit-equal
    parameters, and the file is byte-identical to the one the reference's
    own save() writes for the same weights (src/resonance_net.cpp:743-782);
  * a checkpoint the reference writes loads into the library bit-equal;
  * rnet_model_create(..., reference_init=1) gives exactly the weights of the
    reference's init_weights() (src/resonance_net.cpp:180-216);
  * the reference's own command-line program (src/main.cpp, unmodified),
    linked once against the reference library and once against
    librnet_b200.so through include/, trains the same model on the same data
    file with the same printed per-step losses.

The reference build (oracle/_ref) must be present on a GPU box: these tests
fail rather than skip when it is missing.
"""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(d_model=64, n_layers=2, d_ff=128, n_slots=96, top_k=2, vocab=256)
CFG2 = dict(d_model=512, n_layers=8, d_ff=1024, n_slots=1024, top_k=2, vocab=256)


@pytest.fixture(scope="module")
def ref_ok(orc, cuda):
    assert orc.ref_available(), "oracle/_ref/libref.so (the reference build) is missing"
    return True


@pytest.mark.parametrize("shape", ["small", "config2"])
def test_library_checkpoint_loads_into_reference(shape, ref_ok, rnet, rdata, orc, tmp_path):
    c = SMALL if shape == "small" else CFG2
    cfg = rnet.ModelConfig.make(**c, seq_len=64)
    params = rdata.init_params_normal(cfg, seed=11)
    m = rnet.Model(cfg, device=0, reference_init=False)
    m.set_params(params)
    ours_path = str(tmp_path / "ours.bin")
    m.save(ours_path)
    m.close()
    ref = orc.RefModel.from_checkpoint(ours_path)
    got = ref.params()
    np.testing.assert_array_equal(got.view(np.uint32), params.view(np.uint32))
    ref_path = str(tmp_path / "ref.bin")
    ref.save(ref_path)
    ref.close()
    with open(ours_path, "rb") as a, open(ref_path, "rb") as b:
        assert a.read() == b.read(), "library and reference checkpoints differ byte-wise"


@pytest.mark.parametrize("shape", ["small", "config2"])
def test_reference_checkpoint_loads_into_library(shape, ref_ok, rnet, orc, tmp_path):
    c = SMALL if shape == "small" else CFG2
    ocfg = orc.make_config(**c, seq_len=64)
    ref = orc.RefModel.init(ocfg)
    ref_params = ref.params()
    path = str(tmp_path / "ref.bin")
    ref.save(path)
    ref.close()
    m = rnet.Model.from_checkpoint(path, device=0)
    got = m.get_params()
    assert (m.cfg.d_model, m.cfg.n_layers, m.cfg.n_slots) == (c["d_model"], c["n_layers"],
                                                              c["n_slots"])
    m.close()
    np.testing.assert_array_equal(got.view(np.uint32), ref_params.view(np.uint32))
    # and into an existing model through load_weights
    m = rnet.Model(rnet.ModelConfig.make(**c, seq_len=64), device=0, reference_init=False)
    m.load_weights(path)
    np.testing.assert_array_equal(m.get_params().view(np.uint32), ref_params.view(np.uint32))
    m.close()


@pytest.mark.parametrize("shape", ["small", "config2"])
def test_reference_init_bit_identical(shape, ref_ok, rnet, orc):
    c = SMALL if shape == "small" else CFG2
    ocfg = orc.make_config(**c, seq_len=64)
    ref = orc.RefModel.init(ocfg)
    want = ref.params()
    ref.close()
    m = rnet.Model(rnet.ModelConfig.make(**c, seq_len=64), device=0, reference_init=True)
    got = m.get_params()
    m.close()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


_STEP = re.compile(r"^step\s+(\d+)\s+\|\s+loss\s+([0-9.]+)", re.M)


def _run_main(exe, data, steps, workdir):
    args = [exe, "train", "--data", data, "--d_model", "64", "--n_layers", "2", "--d_ff", "128",
            "--n_slots", "96", "--seq_len", "64", "--batch", "8", "--steps", str(steps),
            "--log", "1", "--save", workdir]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    r = subprocess.run(args, capture_output=True, text=True, timeout=300, env=env, cwd=workdir)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return [(int(s), float(l)) for s, l in _STEP.findall(r.stdout)]


def test_reference_main_program_drop_in(ref_ok, orc, rdata, tmp_path):
    """src/main.cpp unchanged, linked to either library: same losses."""
    for exe in (orc.REFMAIN_REF, orc.REFMAIN_RNET):
        assert os.path.exists(exe), f"{exe} not built (make -C oracle refmain)"
    data = str(tmp_path / "zipf.bin")
    rdata.zipf_bytes(1 << 20, seed=7).tofile(data)
    steps = 30
    a = _run_main(orc.REFMAIN_REF, data, steps, str(tmp_path))
    b = _run_main(orc.REFMAIN_RNET, data, steps, str(tmp_path))
    assert len(a) == steps and len(b) == steps, (a, b)
    print("\nstep  reference  librnet_b200")
    for (s, la), (_, lb) in zip(a, b):
        print(f"{s:4d}  {la:.4f}  {lb:.4f}")
    # losses are printed with 4 decimals (per token, ~5.5): allow one unit of
    # the last digit plus fp32 drift over the steps
    for (s, la), (_, lb) in zip(a, b):
        assert abs(la - lb) <= 2e-4, f"step {s}: reference {la} vs library {lb}"
    assert a[-1][1] < a[0][1], "the loss did not fall: the run is not training"


def test_async_save_snapshots_params_at_call(rnet, rdata, cuda, tmp_path):
    """rnet_model_save_async writes the parameters as they were when it was
    called, although training steps run while the file is written; the file
    is the synchronous save() of those parameters byte for byte."""
    torch = cuda
    cfg = rnet.ModelConfig.make(d_model=64, n_layers=2, d_ff=128, n_slots=64, seq_len=32)
    m = rnet.Model(cfg, device=0, reference_init=False)
    m.set_params(rdata.init_params_normal(cfg, seed=2))
    tok, tgt = rdata.uniform_tokens(2, 32, seed=4)
    d_in = torch.from_numpy(tok.reshape(-1)).cuda()
    d_tg = torch.from_numpy(tgt.reshape(-1)).cuda()
    m.train_step(d_in, d_tg, 2, 32)
    sync_path = str(tmp_path / "sync.bin")
    m.save(sync_path)
    at_call = m.get_params()
    async_path = str(tmp_path / "async.bin")
    m.save_async(async_path)
    for _ in range(5):  # training goes on while the file is written
        m.train_step(d_in, d_tg, 2, 32)
    m.save_wait()
    assert not np.array_equal(m.get_params(), at_call)
    with open(sync_path, "rb") as a, open(async_path, "rb") as b:
        assert a.read() == b.read()
    m.close()
