"""Recurrent decode parity on the GPU.

The decode path carries the O(1) state (conv tails + MinGRU h). Its logits
for every generated position must equal the oracle's full-sequence forward on
the same tokens (teacher forcing with the tokens the decoder produced), and
its greedy tokens must be the argmax of those logits (positions whose top-2
logit gap is below the tolerance are not judged on the token). The CUDA-graph
replay must be bit-identical to eager stepping.

Tolerance: fp32 1e-4 relative (tests/helpers.py).
"""
import numpy as np
import pytest

from helpers import assert_close

pytestmark = pytest.mark.gpu


def _setup(rnet, rdata, orc, M, T, d=64, L=2, F=128, S=160, std=0.05, seed=21):
    cfg = rnet.ModelConfig.make(d_model=d, n_layers=L, d_ff=F, n_slots=S, top_k=2, vocab=256,
                                seq_len=T)
    ocfg = orc.make_config(d, L, F, S, 2, 256, seq_len=T)
    params = rdata.init_params_normal(cfg, seed=seed, std=std)
    r = np.random.default_rng(seed)
    prompt = r.integers(0, 256, size=(M, T)).astype(np.int32)
    return cfg, ocfg, params, prompt


@pytest.mark.parametrize("M,T,steps", [(3, 37, 12), (8, 96, 20)])
def test_decode_matches_full_forward(rnet, rdata, orc, cuda, M, T, steps):
    torch = cuda
    cfg, ocfg, params, prompt = _setup(rnet, rdata, orc, M, T)
    m = rnet.Model(cfg, device=0, reference_init=False)
    m.set_params(params)
    dec = rnet.Decoder(m, M)
    dec.prefill(torch.from_numpy(prompt.reshape(-1)).cuda(), T)
    logits, toks = [], []
    lg, nx = dec.outputs_host()
    logits.append(lg)
    toks.append(nx)
    for _ in range(steps):
        dec.step(None)
        lg, nx = dec.outputs_host()
        logits.append(lg)
        toks.append(nx)
    m.synchronize()
    gen = np.stack(toks[:-1], axis=1)  # tokens fed at positions T..T+steps-1
    seq = np.ascontiguousarray(np.concatenate([prompt, gen], axis=1))
    full, _, _ = orc.forward(ocfg, params, seq, M, T + steps)
    full = full.reshape(M, T + steps, -1)
    for i in range(steps + 1):
        ref = full[:, T - 1 + i]
        assert_close(logits[i], ref, what=f"decode logits at step {i}")
        srt = np.sort(ref, axis=1)
        clear = (srt[:, -1] - srt[:, -2]) > 1e-4 * np.abs(ref).max()
        np.testing.assert_array_equal(toks[i][clear], np.argmax(ref, axis=1)[clear])
    dec.close()
    m.close()


def test_graph_replay_equals_eager(rnet, rdata, orc, cuda):
    torch = cuda
    M, T, steps = 4, 40, 16
    cfg, _, params, prompt = _setup(rnet, rdata, orc, M, T, seed=5)
    outs = []
    for graph in (False, True):
        m = rnet.Model(cfg, device=0, reference_init=False)
        m.set_params(params)
        dec = rnet.Decoder(m, M)
        dec.prefill(torch.from_numpy(prompt.reshape(-1)).cuda(), T)
        out = torch.zeros(steps, M, dtype=torch.int32, device="cuda")
        dec.generate(steps, out, use_graph=graph)
        lg, _ = dec.outputs_host()
        outs.append((out.cpu().numpy(), lg))
        dec.close()
        m.close()
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
