"""Worker functions of the multi-process host tests (tests/test_dist_host.py).

They run as spawned processes in a world of size 2 over the gloo backend
(127.0.0.1), so they live in an importable module of their own."""
import ctypes
import datetime
import importlib
import os

import numpy as np


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def uid_rendezvous(rank, world, port, path, out_dir):
    """Rank 0 publishes a 128-byte communicator id through the library's id
    file (rnet_dist_uid_file_write); rank 1 waits for it
    (rnet_dist_uid_file_read). Every rank reports the bytes it holds."""
    dist = _init(rank, world, port)
    rnet = importlib.import_module("resonance-net_b200")
    buf = ctypes.create_string_buffer(128)
    if rank == 0:
        blob = np.random.default_rng(7).integers(0, 256, 128, dtype=np.uint8).tobytes()
        ctypes.memmove(buf, blob, 128)
        rnet.call("rnet_dist_uid_file_write", path.encode(), buf)
    else:
        rnet.call("rnet_dist_uid_file_read", path.encode(), 20000, buf)
    with open(os.path.join(out_dir, f"uid{rank}.bin"), "wb") as f:
        f.write(buf.raw)
    dist.barrier()
    dist.destroy_process_group()


def dead_rank(rank, world, port, out_dir):
    """Rank 1 leaves before the collective; rank 0's collective must fail
    within the group timeout instead of hanging."""
    import torch
    dist = _init(rank, world, port, timeout_s=3)
    if rank == 1:
        os._exit(0)
    status = "no error"
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
    except Exception as e:  # noqa: BLE001 - any collective failure is the signal
        status = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "dead_rank.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def dp_step(rank, world, port, out_dir, case):
    """Data-parallel semantics of the engine's step (and the reference's
    src/resonance_net.cpp:551-663): every rank computes the gradient of its
    shard (dlogits scaled by 1 / its own token count), the gradients are
    summed across ranks, the learning rate is divided by the world size and
    the clip is tested against ||g|| / world. Rank 0 writes the resulting
    parameters."""
    import torch
    import sys
    dist = _init(rank, world, port)
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import oracle
    rdata = importlib.import_module("resonance-net_b200.data")
    oracle.set_threads(1)
    cfg = oracle.make_config(case["d_model"], case["n_layers"], case["d_ff"], case["n_slots"],
                             case["top_k"], case["vocab"], seq_len=case["T"])
    params = rdata.init_params_normal(cfg, seed=case["pseed"])
    tok, tgt = rdata.uniform_tokens(case["B"], case["T"], seed=case["tseed"])
    per = case["B"] // world
    shard = slice(rank * per, (rank + 1) * per)
    out = oracle.train_step(cfg, params, tok[shard], tgt[shard], per, case["T"], case["lr"],
                            case["clip"])
    g = torch.from_numpy(out["grads"].astype(np.float64))
    dist.all_reduce(g)  # sum over ranks
    g = g.numpy()
    lr = case["lr"] / world
    norm = float(np.sqrt(np.sum(g * g)))
    if case["clip"] > 0 and norm / world > case["clip"]:
        lr *= case["clip"] / (norm / world)
    new = params.astype(np.float64) - lr * g
    if rank == 0:
        np.save(os.path.join(out_dir, "dp_params.npy"), new)
    dist.barrier()
    dist.destroy_process_group()


def dp_engine(rank, world, port, out_dir, case):
    """Data-parallel engine step on `world` GPUs: each rank trains its shard of
    the batch with the NCCL gradient all-reduce (rnet.Dist); rank 0 writes the
    updated parameters."""
    import torch
    if case.get("bucket_mb"):
        os.environ["RNET_DP_BUCKET_MB"] = str(case["bucket_mb"])
    dist = _init(rank, world, port)
    rnet = importlib.import_module("resonance-net_b200")
    rdata = importlib.import_module("resonance-net_b200.data")
    torch.cuda.set_device(rank)
    cfg = rnet.ModelConfig.make(d_model=case["d_model"], n_layers=case["n_layers"],
                                d_ff=case["d_ff"], n_slots=case["n_slots"], top_k=case["top_k"],
                                vocab=case["vocab"], seq_len=case["T"])
    m = rnet.Model(cfg, device=rank, reference_init=False)
    m.set_params(rdata.init_params_normal(cfg, seed=case["pseed"]))
    m.set_precision(case.get("bf16", False))  # bf16 mode: bf16 gradient all-reduce
    uid = [rnet.Dist.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    d = rnet.Dist(rank, world, rank, uid[0])
    m.set_dist(d)
    tok, tgt = rdata.uniform_tokens(case["B"], case["T"], seed=case["tseed"])
    per = case["B"] // world
    sl = slice(rank * per, (rank + 1) * per)
    d_in = torch.from_numpy(np.ascontiguousarray(tok[sl]).reshape(-1)).cuda()
    d_tg = torch.from_numpy(np.ascontiguousarray(tgt[sl]).reshape(-1)).cuda()
    loss = torch.zeros(1, device="cuda")
    m.train_step(d_in, d_tg, per, case["T"], case["lr"], case["clip"], loss)
    m.synchronize()
    if rank == 0:
        np.save(os.path.join(out_dir, "dp_engine_params.npy"), m.get_params())
    dist.barrier()
    m.set_dist(None)
    d.close()
    m.close()
    dist.destroy_process_group()
