"""CPU checks of the drop-in boundary (no GPU, no compute calls):
the shared library loads, exports every entry point include/rnet_capi.h
declares, the Python binding covers exactly that set, the config struct is the
40-byte checkpoint header, and the parameter layout matches the reference's
ModelConfig::param_count (include/config.h:27-49)."""
import ctypes
import os
import re
import struct
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "rnet_capi.h")


def declared_symbols():
    src = open(HDR).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rnet_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(rnet):
    lib = rnet.lib()
    names = declared_symbols()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", rnet.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (rnet_[a-z0-9_]+)$", out, flags=re.M))
    assert set(names) <= exported
    assert lib.rnet_abi_version() == 100


def test_binding_covers_header(rnet):
    assert sorted(rnet.exported_symbols()) == declared_symbols()


def test_config_struct_is_checkpoint_header(rnet, rdata):
    assert ctypes.sizeof(rnet.ModelConfig) == 40
    c = rnet.ModelConfig.make()
    raw = bytes(c)
    fields = struct.unpack(rdata.HEADER_FMT, raw)
    assert fields[:9] == (512, 8, 1024, 8, 512, 1024, 2, 256, 256)
    assert abs(fields[9] - 1e-6) < 1e-12


def reference_param_count(d, L, f, s, v):
    # include/config.h:27-49 restated
    p = v * d * 2 + d
    p += L * (4 * d + 25 * d + d * d + 2 * d * d + 2 * d + 2 * d * s + 2 * d * d + 3 * d * f)
    return p


def test_layout_matches_reference_param_count(rnet, rdata, orc):
    for (d, L, f, s, v) in [(64, 1, 128, 64, 256), (512, 8, 1024, 1024, 256),
                            (2048, 24, 5632, 8192, 256)]:
        cfg = rnet.ModelConfig.make(d_model=d, n_layers=L, d_ff=f, n_slots=s, vocab=v)
        assert rdata.param_count(cfg) == reference_param_count(d, L, f, s, v)
    assert rdata.param_count(rnet.ModelConfig.make()) == 31_846_912
    oc = orc.make_config(512, 8, 1024, 1024, 2, 256, 256)
    assert orc.param_count(oc) == 31_846_912


def test_checkpoint_roundtrip(tmp_path, rnet, rdata):
    cfg = rnet.ModelConfig.make(d_model=32, n_layers=2, d_ff=64, n_slots=32, vocab=256)
    p = rdata.init_params_normal(cfg, seed=5)
    path = str(tmp_path / "c.bin")
    rdata.write_checkpoint(path, cfg, p)
    assert os.path.getsize(path) == 40 + 4 * p.size
    hdr, q = rdata.read_checkpoint(path)
    assert hdr[:9] == (32, 2, 64, 8, 32, 32, 2, 256, 256)
    np.testing.assert_array_equal(p, q)
    # gains 1, biases 0, weights ~N(0, 0.02)
    parts = rdata.split(cfg, p)
    assert np.all(parts["L1.norm3"] == 1) and np.all(parts["L0.bz"] == 0)
    assert abs(parts["L0.mix"].std() - 0.02) < 0.003


def test_zipf_bytes_distribution(rdata):
    b = rdata.zipf_bytes(200_000, seed=7)
    counts = np.bincount(b, minlength=256)
    top = np.sort(counts)[::-1]
    # Zipf(1.1): rank-1 / rank-2 frequency ratio ~ 2^1.1
    assert 1.9 < top[0] / top[1] < 2.4
    assert counts.sum() == 200_000
    assert np.array_equal(rdata.zipf_bytes(1000, seed=7), rdata.zipf_bytes(1000, seed=7))


def test_rms_norm_rejects_unaligned_pointers_without_launch(rnet):
    """The RMSNorm kernels move rows as float4 / bulk copies: an offset view
    (a slice starting at an odd element) is refused with RNET_ERR_ARG before
    anything is launched, instead of faulting on the GPU."""
    lib = rnet.lib()
    buf = np.zeros(4 * 64 + 8, np.float32)
    base = buf.ctypes.data + (-buf.ctypes.data) % 16  # 16-byte aligned address
    n0 = rnet.kernel_launches()
    ok = ctypes.c_void_p(base)
    odd = ctypes.c_void_p(base + 4)
    rc = lib.rnet_rms_norm_forward(odd, ok, ok, ok, 4, 64, ctypes.c_float(1e-6), None)
    assert rc == -1 and "16-byte aligned" in lib.rnet_last_error().decode()
    rc = lib.rnet_rms_norm_backward(ok, odd, ok, ok, ok, ok, 4, 64, None)
    assert rc == -1 and "16-byte aligned" in lib.rnet_last_error().decode()
    rc = lib.rnet_rms_norm_backward(ok, ok, ok, ok, odd, ok, 4, 64, None)
    assert rc == -1
    rc = lib.rnet_rms_norm_forward(ok, ok, ok, ok, 4, 62, ctypes.c_float(1e-6), None)
    assert rc == -1 and "multiple of 4" in lib.rnet_last_error().decode()
    assert rnet.kernel_launches() == n0
