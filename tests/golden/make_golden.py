"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own CUDA
implementation (oracle/_ref/libref.so: the reference sources compiled
unmodified + oracle/ref_capi.cpp). Must run on a machine with a GPU:

    python tests/golden/make_golden.py tests/golden

Each fixture is one full training step exactly as the reference's `train`
loop performs it (zero_grad, forward, cross-entropy, scale by 1/N, backward,
clipped SGD; src/main.cpp:136-152): seeded N(0, 0.02) weights written through
the reference checkpoint format, seeded uniform byte tokens with next-byte
targets. Stored: inputs, the summed loss, every gradient (flat, checkpoint
order), logits, per-layer top-k indices and weights, and the updated weights.
"""
from __future__ import annotations

import ctypes
import importlib
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

data = importlib.import_module("resonance-net_b200.data")

CASES = {
    # BASELINE config 0 ("tiny plumbing step")
    "cfg_tiny": dict(d_model=64, n_layers=1, d_ff=128, n_slots=64, top_k=2, vocab=256, B=2, T=32,
                     pseed=1234, tseed=1),
    # two layers, wider, longer sequences (exercises several scan segments / tiles)
    "cfg_small": dict(d_model=64, n_layers=2, d_ff=128, n_slots=160, top_k=2, vocab=256, B=3,
                      T=100, pseed=99, tseed=5),
}


def run_case(name: str, c: dict, outdir: str) -> None:
    cfg = oracle.make_config(c["d_model"], c["n_layers"], c["d_ff"], c["n_slots"], c["top_k"],
                             c["vocab"], seq_len=c["T"])
    B, T = c["B"], c["T"]
    params = data.init_params_normal(cfg, seed=c["pseed"])
    tok, tgt = data.uniform_tokens(B, T, seed=c["tseed"])
    R = oracle.ref_lib()
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "w.bin")
        data.write_checkpoint(path, cfg, params)
        h = R.ref_model_load(path.encode())
        assert h, "reference failed to load checkpoint"
    n = int(R.ref_model_param_count(h))
    assert n == params.size, (n, params.size)
    tokc = np.ascontiguousarray(tok.reshape(-1), np.int32)
    tgtc = np.ascontiguousarray(tgt.reshape(-1), np.int32)
    loss = R.ref_train_step(h, tokc.ctypes.data_as(ctypes.c_void_p),
                            tgtc.ctypes.data_as(ctypes.c_void_p), B, T, 3e-4, 1.0)
    N = B * T
    grads = np.zeros(n, np.float32)
    after = np.zeros(n, np.float32)
    logits = np.zeros((N, cfg.vocab_size), np.float32)
    idx = np.zeros((cfg.n_layers, N, cfg.slot_top_k), np.int32)
    w = np.zeros((cfg.n_layers, N, cfg.slot_top_k), np.float32)
    R.ref_model_get_grads(h, grads.ctypes.data_as(ctypes.c_void_p))
    R.ref_model_get_params(h, after.ctypes.data_as(ctypes.c_void_p))
    R.ref_get_logits(h, logits.ctypes.data_as(ctypes.c_void_p), N)
    R.ref_get_topk(h, idx.ctypes.data_as(ctypes.c_void_p), w.ctypes.data_as(ctypes.c_void_p), N)
    R.ref_model_destroy(h)
    np.savez_compressed(
        os.path.join(outdir, f"{name}.npz"),
        config=np.array([cfg.d_model, cfg.n_layers, cfg.d_ff, cfg.n_heads, cfg.gru_dim,
                         cfg.n_slots, cfg.slot_top_k, cfg.vocab_size, cfg.seq_len], np.int32),
        B=B, T=T, lr=3e-4, clip=1.0, param_seed=c["pseed"], token_seed=c["tseed"],
        params=params, tokens=tok, targets=tgt, loss_sum=np.float32(loss), grads=grads,
        params_after=after,
        logits=logits, topk_idx=idx, topk_w=w)
    print(f"{name}: loss_sum={loss:.6f} |g|={np.linalg.norm(grads):.6e}")


if __name__ == "__main__":
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__))
    os.makedirs(out, exist_ok=True)
    for k, v in CASES.items():
        run_case(k, v, out)
