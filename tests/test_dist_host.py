"""Host-side multi-process paths, world size 2 over gloo on the CPU (no GPU):
the communicator-id rendezvous of dist_init_from_env (id file written by rank 0,
awaited by the others with a timeout), detection of a rank that leaves, and
the data-parallel step semantics the engine implements on the device (sum of
shard gradients, lr / world, clip against ||g|| / world) checked against the
single-process oracle step on the whole batch (fp32 tolerance)."""
import os
import socket
import time

import numpy as np
import pytest

import dist_workers

mp = pytest.importorskip("torch.multiprocessing")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn(fn, *args):
    mp.spawn(fn, args=(2, _port()) + args, nprocs=2, join=True)


def test_uid_rendezvous(tmp_path):
    path = str(tmp_path / "nccl.uid")
    _spawn(dist_workers.uid_rendezvous, path, str(tmp_path))
    a = (tmp_path / "uid0.bin").read_bytes()
    b = (tmp_path / "uid1.bin").read_bytes()
    assert len(a) == 128 and a == b
    assert not os.path.exists(path + ".tmp")  # published by rename, never half-written


def test_uid_read_times_out(rnet, tmp_path):
    import ctypes
    buf = ctypes.create_string_buffer(128)
    t0 = time.time()
    rc = rnet.lib().rnet_dist_uid_file_read(str(tmp_path / "missing").encode(), 300, buf)
    assert rc != 0
    assert "timeout" in rnet.lib().rnet_last_error().decode()
    assert 0.25 <= time.time() - t0 < 5


def test_dead_rank_detected(tmp_path):
    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=dist_workers.dead_rank, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert all(not p.is_alive() for p in procs)
    status = (tmp_path / "dead_rank.txt").read_text()
    assert status.startswith("error"), status


def test_dp_step_matches_full_batch(orc, rdata, tmp_path):
    case = dict(d_model=64, n_layers=1, d_ff=128, n_slots=64, top_k=2, vocab=256, B=4, T=32,
                pseed=1234, tseed=3, lr=3e-4, clip=1.0)
    _spawn(dist_workers.dp_step, str(tmp_path), case)
    dp = np.load(tmp_path / "dp_params.npy")
    cfg = orc.make_config(case["d_model"], case["n_layers"], case["d_ff"], case["n_slots"],
                          case["top_k"], case["vocab"], seq_len=case["T"])
    params = rdata.init_params_normal(cfg, seed=case["pseed"])
    tok, tgt = rdata.uniform_tokens(case["B"], case["T"], seed=case["tseed"])
    full = orc.train_step(cfg, params, tok, tgt, case["B"], case["T"], case["lr"], case["clip"])
    # the full-batch update in float64 from the oracle's gradient (the updated
    # fp32 parameters would round a 1e-6-sized update to ~1e-3 relative)
    g = full["grads"].astype(np.float64)
    lr = case["lr"]
    norm = float(np.sqrt(np.sum(g * g)))
    if norm > case["clip"]:
        lr *= case["clip"] / norm
    d_full = -lr * g
    d_dp = dp - params.astype(np.float64)
    rel = np.linalg.norm(d_dp - d_full) / np.linalg.norm(d_full)
    assert rel <= 1e-4, f"data-parallel step differs from the full-batch step: {rel:.2e}"
