"""ORACLE — test infrastructure only.

ctypes bindings of
  * liboracle.so  — scalar C++/OpenMP restatement of the reference math
                    (oracle/oracle.cpp, every function cites the reference
                    file:line it follows);
  * _ref/libref.so — the reference's own CUDA sources compiled unmodified
                    plus a small C-ABI harness (oracle/ref_capi.cpp).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this package, and only as the checker or the timed baseline —
never as the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_ORACLE = os.path.join(HERE, "liboracle.so")
LIB_REF = os.path.join(HERE, "_ref", "libref.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


class OrcConfig(ctypes.Structure):
    """Byte-identical to the reference ModelConfig (include/config.h:7-18)."""
    _fields_ = [("d_model", _I), ("n_layers", _I), ("d_ff", _I), ("n_heads", _I),
                ("gru_dim", _I), ("n_slots", _I), ("slot_top_k", _I), ("vocab_size", _I),
                ("seq_len", _I), ("rms_eps", _F)]


def make_config(d_model=512, n_layers=8, d_ff=1024, n_slots=1024, top_k=2, vocab=256,
                seq_len=256, eps=1e-6) -> OrcConfig:
    return OrcConfig(d_model, n_layers, d_ff, 8, d_model, n_slots, top_k, vocab, seq_len, eps)


def build() -> None:
    """Compile liboracle.so (and the reference harness when the reference
    sources are present in this container)."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    # skipped by the Makefile when the reference sources are absent
    subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True,
                   stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_ORACLE):
            build()
        _lib = ctypes.CDLL(LIB_ORACLE)
        _lib.orc_param_count.restype = ctypes.c_size_t
        _lib.orc_param_count.argtypes = [ctypes.POINTER(OrcConfig)]
    return _lib


def ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_P)


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


def param_count(cfg: OrcConfig) -> int:
    return int(lib().orc_param_count(ctypes.byref(cfg)))


def train_step(cfg, params, tokens, targets, B, T, lr=3e-4, clip=1.0, quirk=1, forced=None,
               tau=0.0):
    """One reference training step. Returns dict(loss_sum, grads, params (updated),
    topk_idx [L,N,k], topk_w [L,N,k], logits [N,V], n_forced).

    forced [L,N,k] (optional): on rows whose selection margin is below `tau`
    and whose selected slot set differs from forced's, use forced's slots
    (n_forced counts those rows) — the same discrete choices as the
    implementation under test on near-ties, so the rest compares continuously."""
    params = np.array(params, dtype=np.float32, copy=True)
    n = param_count(cfg)
    grads = np.zeros(n, np.float32)
    N = B * T
    k = cfg.slot_top_k
    idx = np.zeros((cfg.n_layers, N, k), np.int32)
    w = np.zeros((cfg.n_layers, N, k), np.float32)
    logits = np.zeros((N, cfg.vocab_size), np.float32)
    loss = _F(0)
    tok = np.ascontiguousarray(tokens, np.int32)
    tgt = np.ascontiguousarray(targets, np.int32)
    nf = _I(0)
    fz = None if forced is None else np.ascontiguousarray(forced, np.int32)
    if fz is not None:
        assert fz.shape == idx.shape
    lib().orc_train_step_forced(ctypes.byref(cfg), ptr(params), ptr(grads), ptr(tok), ptr(tgt),
                                B, T, _F(lr), _F(clip), quirk, ctypes.byref(loss), ptr(idx),
                                ptr(w), ptr(logits), ptr(fz), _F(tau), ctypes.byref(nf))
    return dict(loss_sum=loss.value, grads=grads, params=params, params_after=params,
                topk_idx=idx, topk_w=w, logits=logits, n_forced=nf.value)


def forward(cfg, params, tokens, B, T):
    N = B * T
    logits = np.zeros((N, cfg.vocab_size), np.float32)
    idx = np.zeros((cfg.n_layers, N, cfg.slot_top_k), np.int32)
    w = np.zeros((cfg.n_layers, N, cfg.slot_top_k), np.float32)
    tok = np.ascontiguousarray(tokens, np.int32)
    lib().orc_model_forward(ctypes.byref(cfg), ptr(np.ascontiguousarray(params, np.float32)),
                            ptr(tok), B, T, ptr(logits), ptr(idx), ptr(w))
    return logits, idx, w


def topk_margins(cfg, params, tokens, B, T):
    """Per-layer top-k selection margins [L, B*T] (see oracle.cpp topk_row)."""
    m = np.zeros((cfg.n_layers, B * T), np.float32)
    tok = np.ascontiguousarray(tokens, np.int32)
    lib().orc_topk_margins(ctypes.byref(cfg), ptr(np.ascontiguousarray(params, np.float32)),
                           ptr(tok), B, T, ptr(m))
    return m


def sgd_step(cfg, params, grads, lr, clip, world=1):
    p = np.array(params, np.float32, copy=True)
    lib().orc_sgd_step(ctypes.byref(cfg), ptr(p), ptr(np.ascontiguousarray(grads, np.float32)),
                       _F(lr), _F(clip), int(world))
    return p


# ------------------------------------------------------------------ reference harness
_ref = None


def ref_available() -> bool:
    return os.path.exists(LIB_REF)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        _ref = ctypes.CDLL(LIB_REF)
        _ref.ref_model_load.restype = _P
        _ref.ref_model_load.argtypes = [ctypes.c_char_p]
        _ref.ref_model_param_count.restype = ctypes.c_size_t
        _ref.ref_model_param_count.argtypes = [_P]
        _ref.ref_train_step.restype = _F
        _ref.ref_train_step.argtypes = [_P, _P, _P, _I, _I, _F, _F]
        _ref.ref_train_step_device.argtypes = [_P, _P, _P, _I, _I, _F, _F]
        _ref.ref_forward.argtypes = [_P, _P, _I, _I, _P]
        _ref.ref_forward_device.argtypes = [_P, _P, _I, _I]
        for f in ("ref_model_get_params", "ref_model_get_grads"):
            getattr(_ref, f).argtypes = [_P, _P]
        _ref.ref_get_logits.argtypes = [_P, _P, _I]
        _ref.ref_get_topk.argtypes = [_P, _P, _P, _I]
        _ref.ref_model_destroy.argtypes = [_P]
        _ref.ref_model_init.restype = _P
        _ref.ref_model_init.argtypes = [ctypes.POINTER(OrcConfig)]
        _ref.ref_model_save.argtypes = [_P, ctypes.c_char_p]
        _ref.ref_model_load_into.argtypes = [_P, ctypes.c_char_p]
        _ref.ref_get_scores.argtypes = [_P, _I, _P, _I]
        _ref.ref_loader_batches.argtypes = [ctypes.c_char_p, ctypes.c_uint, _I, _I, _I, _P, _P]
    return _ref


REFMAIN_REF = os.path.join(HERE, "_ref", "refmain_ref")
REFMAIN_RNET = os.path.join(HERE, "_ref", "refmain_rnet")


class RefModel:
    """The reference's own ResonanceNet (oracle/_ref/libref.so) on the GPU."""

    def __init__(self, handle):
        if not handle:
            raise RuntimeError("reference model creation failed")
        self.h = handle
        self.lib = ref_lib()

    @classmethod
    def from_checkpoint(cls, path: str) -> "RefModel":
        return cls(ref_lib().ref_model_load(path.encode()))

    @classmethod
    def init(cls, cfg: OrcConfig) -> "RefModel":
        """Weights from the reference's own init_weights()."""
        return cls(ref_lib().ref_model_init(ctypes.byref(cfg)))

    def param_count(self) -> int:
        return int(self.lib.ref_model_param_count(self.h))

    def params(self) -> np.ndarray:
        out = np.empty(self.param_count(), np.float32)
        self.lib.ref_model_get_params(self.h, ptr(out))
        return out

    def grads(self) -> np.ndarray:
        out = np.empty(self.param_count(), np.float32)
        self.lib.ref_model_get_grads(self.h, ptr(out))
        return out

    def save(self, path: str) -> None:
        assert self.lib.ref_model_save(self.h, path.encode()) == 1

    def load(self, path: str) -> None:
        assert self.lib.ref_model_load_into(self.h, path.encode()) == 1

    def train_step(self, tok, tgt, B, T, lr=3e-4, clip=1.0) -> float:
        tok = np.ascontiguousarray(tok, np.int32)
        tgt = np.ascontiguousarray(tgt, np.int32)
        return float(self.lib.ref_train_step(self.h, ptr(tok), ptr(tgt), B, T, lr, clip))

    def topk(self, n_layers, N, k):
        idx = np.zeros((n_layers, N, k), np.int32)
        w = np.zeros((n_layers, N, k), np.float32)
        self.lib.ref_get_topk(self.h, ptr(idx), ptr(w), N)
        return idx, w

    def scores(self, layer, N, S) -> np.ndarray:
        out = np.empty((N, S), np.float32)
        self.lib.ref_get_scores(self.h, layer, ptr(out), N)
        return out

    def logits(self, N, V) -> np.ndarray:
        out = np.empty((N, V), np.float32)
        self.lib.ref_get_logits(self.h, ptr(out), N)
        return out

    def close(self) -> None:
        if self.h:
            self.lib.ref_model_destroy(self.h)
            self.h = None


def ref_loader_batches(path: str, seed: int, B: int, T: int, steps: int):
    """Batches of the reference's own DataLoader ([steps, B*T] inputs, targets)."""
    inp = np.zeros((steps, B * T), np.int32)
    tgt = np.zeros((steps, B * T), np.int32)
    assert ref_lib().ref_loader_batches((path or "").encode(), seed, B, T, steps, ptr(inp),
                                        ptr(tgt)) == 1
    return inp, tgt


def margins_from_scores(scores: np.ndarray, k: int = 2) -> np.ndarray:
    """Selection margin per row, as topk_row in oracle.cpp defines it: the
    smaller of (k-th minus (k+1)-th largest score) and the smallest gap among
    the k selected."""
    top = -np.partition(-scores, k, axis=1)[:, :k + 1]
    top = -np.sort(-top, axis=1)
    m = top[:, k - 1] - top[:, k]
    for a in range(k - 1):
        m = np.minimum(m, top[:, a] - top[:, a + 1])
    return m
