"""The C++ drop-in boundary: a program written against the reference's C++
API compiles against include/ and links librnet_b200.so (CPU), and runs a
reference-style train loop + checkpoint round trip + generate (GPU).

Also the host side of the distributed init (file-based ncclUniqueId exchange,
reference src/dist.cpp:53-93) with real processes: a rank that never appears
makes the waiter return a timeout status instead of hanging, and a file
shorter than an id is never accepted (no GPU, no NCCL needed)."""
import ctypes
import importlib
import multiprocessing as mp
import os
import subprocess
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "dropin_main.cpp")


def _build(tmp_path, rnet):
    exe = str(tmp_path / "dropin_main")
    libdir = os.path.dirname(rnet.LIB_PATH)
    cmd = ["g++", "-std=c++20", "-O1", "-I", os.path.join(ROOT, "include"),
           "-I", "/usr/local/cuda/include", SRC, "-L", libdir, "-lrnet_b200",
           "-L", "/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{libdir}",
           "-Wl,-rpath,/usr/local/cuda/lib64", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_dropin_compiles_and_links(tmp_path, rnet):
    rnet.lib()
    assert os.path.exists(_build(tmp_path, rnet))


@pytest.mark.gpu
def test_dropin_runs_reference_style_loop(tmp_path, rnet, cuda):
    exe = _build(tmp_path, rnet)
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    r = subprocess.run([exe, str(tmp_path / "ckpt.bin")], capture_output=True, text=True,
                       timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "DROPIN OK" in r.stdout
    rdata = importlib.import_module("resonance-net_b200.data")
    cfg = rnet.ModelConfig.make(d_model=64, n_layers=2, d_ff=128, n_slots=64, seq_len=32)
    assert os.path.getsize(tmp_path / "ckpt.bin") == 40 + 4 * rdata.param_count(cfg)


def _reader(path, timeout_ms, q):
    rnet = importlib.import_module("resonance-net_b200")
    buf = ctypes.create_string_buffer(128)
    t0 = time.time()
    rc = rnet.lib().rnet_dist_uid_file_read(path.encode(), timeout_ms, buf)
    q.put((rc, buf.raw, time.time() - t0, rnet.lib().rnet_last_error().decode()))


def test_uid_rendezvous_between_processes(tmp_path, rnet):
    path = str(tmp_path / "uid")
    uid = bytes(range(128))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_reader, args=(path, 20000, q))
    p.start()
    time.sleep(0.5)
    assert rnet.lib().rnet_dist_uid_file_write(path.encode(), uid) == 0
    rc, got, _, _ = q.get(timeout=60)
    p.join(10)
    assert rc == 0 and got == uid
    assert not os.path.exists(path + ".tmp")


def test_uid_rendezvous_missing_rank_times_out(tmp_path, rnet):
    path = str(tmp_path / "never")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_reader, args=(path, 400, q))
    p.start()
    rc, _, dt, msg = q.get(timeout=60)
    p.join(10)
    assert rc == -4 and "timeout" in msg  # RNET_ERR_TIMEOUT
    assert 0.3 < dt < 10


def test_uid_rendezvous_truncated_file(tmp_path, rnet):
    path = tmp_path / "short"
    path.write_bytes(b"x" * 10)
    buf = ctypes.create_string_buffer(128)
    rc = rnet.lib().rnet_dist_uid_file_read(str(path).encode(), 300, buf)
    assert rc == -4  # a partial id never satisfies the reader
