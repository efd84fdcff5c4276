"""Device-resident training batches (rnet_data_*) against the reference's own
DataLoader (src/data_loader.cpp:31-52, compiled unmodified into the oracle
harness): for the same corpus and seed every batch is identical, for a byte
corpus (window starts drawn on the host, windows gathered on the GPU) and
for the reference's synthetic tokens. Feeding the model from the loader
gives the same losses as feeding it the reference loader's host batches."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,T,steps", [(8, 64, 5), (3, 257, 4)])
def test_corpus_batches_match_reference_loader(rnet, rdata, orc, cuda, tmp_path, B, T, steps):
    torch = cuda
    assert orc.ref_available()
    corpus = rdata.zipf_bytes(1 << 20, seed=5).tobytes()
    path = tmp_path / "corpus.bin"
    path.write_bytes(corpus)
    want_in, want_tgt = orc.ref_loader_batches(str(path), 42, B, T, steps)
    dl = rnet.DataLoader(corpus, device=0, seed=42)
    for s in range(steps):
        d_in = torch.empty(B * T, dtype=torch.int32, device="cuda")
        d_tg = torch.empty(B * T, dtype=torch.int32, device="cuda")
        dl.batch(B, T, d_in, d_tg)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(d_in.cpu().numpy(), want_in[s])
        np.testing.assert_array_equal(d_tg.cpu().numpy(), want_tgt[s])
    dl.close()


def test_synthetic_batches_match_reference_loader(rnet, orc, cuda):
    torch = cuda
    B, T, steps = 4, 32, 3
    want_in, want_tgt = orc.ref_loader_batches("", 7, B, T, steps)
    dl = rnet.DataLoader(None, device=0, seed=7)
    for s in range(steps):
        d_in = torch.empty(B * T, dtype=torch.int32, device="cuda")
        d_tg = torch.empty(B * T, dtype=torch.int32, device="cuda")
        dl.batch(B, T, d_in, d_tg)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(d_in.cpu().numpy(), want_in[s])
        np.testing.assert_array_equal(d_tg.cpu().numpy(), want_tgt[s])
    dl.close()


def test_training_from_device_loader(rnet, rdata, orc, cuda, tmp_path):
    """Three steps fed by the device loader equal three steps fed with the
    reference loader's batches through the host-buffer API."""
    torch = cuda
    B, T = 4, 64
    cfg = rnet.ModelConfig.make(d_model=64, n_layers=2, d_ff=128, n_slots=64, seq_len=T)
    params = rdata.init_params_normal(cfg, seed=3)
    corpus = rdata.zipf_bytes(1 << 18, seed=6).tobytes()
    path = tmp_path / "c.bin"
    path.write_bytes(corpus)
    want_in, want_tgt = orc.ref_loader_batches(str(path), 42, B, T, 3)
    a = rnet.Model(cfg, device=0, reference_init=False)
    b = rnet.Model(cfg, device=0, reference_init=False)
    a.set_params(params)
    b.set_params(params)
    dl = rnet.DataLoader(corpus, device=0, seed=42)
    d_in = torch.empty(B * T, dtype=torch.int32, device="cuda")
    d_tg = torch.empty(B * T, dtype=torch.int32, device="cuda")
    loss = torch.zeros(1, device="cuda")
    for s in range(3):
        dl.batch(B, T, d_in, d_tg, stream=a.stream())
        a.train_step(d_in, d_tg, B, T, 3e-4, 1.0, loss)
        a.synchronize()
        lb = b.train_step_host(want_in[s].copy(), want_tgt[s].copy(), B, T, 3e-4, 1.0)
        assert abs(float(loss.item()) - lb) <= 1e-6 * abs(lb)
    dl.close()
    a.close()
    b.close()
