"""Python binding of librnet_b200.so (the B200 / sm_100a ResonanceNet library).

Only the C ABI declared in include/rnet_capi.h is used. There is no Python or
CPU fallback: if the shared library is missing or cannot be loaded this module
raises, and every call that fails raises RnetError with the library's message.

The package directory name contains a hyphen, so import it with
``importlib.import_module("resonance-net_b200")`` (see ``load()`` below).
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librnet_b200.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t


class RnetError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"rnet error {code}: {msg}")
        self.code = code


class ModelConfig(ctypes.Structure):
    """rnet_model_config — byte-identical to the reference ModelConfig /
    the 40-byte checkpoint header."""
    _fields_ = [("d_model", _I), ("n_layers", _I), ("d_ff", _I), ("n_heads", _I),
                ("gru_dim", _I), ("n_slots", _I), ("slot_top_k", _I), ("vocab_size", _I),
                ("seq_len", _I), ("rms_eps", _F)]

    @classmethod
    def make(cls, d_model=512, n_layers=8, d_ff=1024, n_slots=1024, top_k=2, vocab=256,
             seq_len=256, eps=1e-6, n_heads=8):
        return cls(d_model, n_layers, d_ff, n_heads, d_model, n_slots, top_k, vocab, seq_len, eps)


# name -> argtypes (all return int status)
_SIGS = {
    "rnet_abi_version": [],
    "rnet_device_error": [ctypes.POINTER(ctypes.c_uint), _I],
    "rnet_selftest_bounded_wait": [_I, ctypes.c_uint, _I, ctypes.POINTER(ctypes.c_uint)],
    "rnet_gemm_f32": [_I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _I, _P, _I, _I, _F, _P],
    "rnet_gemm_bf16": [_I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _I, _P, _I, _I, _F, _P, _P],
    "rnet_gemm_set_cta_group": [_I],
    "rnet_gemm_set_precision": [_I],
    "rnet_rms_norm_forward": [_P, _P, _P, _P, _I, _I, _F, _P],
    "rnet_rms_norm_backward": [_P, _P, _P, _P, _P, _P, _I, _I, _P],
    "rnet_embed_forward": [_P, _P, _P, _I, _I, _I, _P],
    "rnet_embed_backward": [_P, _P, _P, _I, _I, _I, _P],
    "rnet_linear_forward": [_P, _P, _P, _I, _I, _I, _P],
    "rnet_causal_conv_forward": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "rnet_causal_conv_backward": [_P] * 12 + [_I, _I, _I, _I, _P],
    "rnet_min_gru_forward": [_P] * 8 + [_I, _I, _I, _P],
    "rnet_min_gru_backward": [_P] * 13 + [_I, _I, _I, _P],
    "rnet_slot_memory_forward": [_P] * 10 + [_I, _I, _I, _I, _I, _P],
    "rnet_slot_memory_backward": [_P] * 15 + [_I, _I, _I, _I, _I, _P],
    "rnet_swiglu_forward": [_P] * 7 + [_I, _I, _I, _P],
    "rnet_swiglu_backward": [_P] * 11 + [_I, _I, _I, _P],
    "rnet_cross_entropy_forward": [_P, _P, _P, _P, _I, _I, _P],
    "rnet_cross_entropy_forward_noalloc": [_P, _P, _P, _P, _I, _I, _P],
    "rnet_residual_add": [_P, _P, _SZ, _P],
    "rnet_scale_grads": [_P, _F, _SZ, _P],
    "rnet_model_create": [ctypes.POINTER(ModelConfig), _I, _I, ctypes.POINTER(_P)],
    "rnet_model_create_from_checkpoint": [ctypes.c_char_p, _I, ctypes.POINTER(_P)],
    "rnet_model_destroy": [_P],
    "rnet_model_get_config": [_P, ctypes.POINTER(ModelConfig)],
    "rnet_model_param_count": [_P, ctypes.POINTER(_SZ)],
    "rnet_model_device_buffers": [_P, ctypes.POINTER(_P), ctypes.POINTER(_P)],
    "rnet_model_stream": [_P, ctypes.POINTER(_P)],
    "rnet_model_set_params": [_P, _P, _SZ],
    "rnet_model_get_params": [_P, _P, _SZ],
    "rnet_model_set_params_device": [_P, _P, _SZ],
    "rnet_model_get_grads": [_P, _P, _SZ],
    "rnet_model_params_updated": [_P],
    "rnet_model_set_conv_quirk": [_P, _I],
    "rnet_model_set_precision": [_P, _I],
    "rnet_model_set_recompute": [_P, _I],
    "rnet_model_set_optimizer": [_P, _F, _F, _I],
    "rnet_model_forward": [_P, _P, _P, _I, _I],
    "rnet_model_backward": [_P, _P, _P, _I, _I],
    "rnet_model_zero_grad": [_P],
    "rnet_model_step": [_P, _F, _F],
    "rnet_model_train_step": [_P, _P, _P, _I, _I, _F, _F, _P],
    "rnet_model_train_step_host": [_P, _P, _P, _I, _I, _F, _F, ctypes.POINTER(_F)],
    "rnet_model_topk": [_P, _I, ctypes.POINTER(_P), ctypes.POINTER(_P)],
    "rnet_model_topk_host": [_P, _I, _P, _P, _SZ],
    "rnet_model_save": [_P, ctypes.c_char_p],
    "rnet_model_load_weights": [_P, ctypes.c_char_p],
    "rnet_model_save_async": [_P, ctypes.c_char_p],
    "rnet_model_save_wait": [_P],
    "rnet_model_synchronize": [_P],
    "rnet_model_profile_enable": [_P, _I],
    "rnet_model_profile_read": [_P, _P, _P, _P, _P, _I, _I],
    "rnet_kernel_launches": [ctypes.POINTER(ctypes.c_ulonglong)],
    "rnet_decoder_create": [_P, _I, ctypes.POINTER(_P)],
    "rnet_decoder_destroy": [_P],
    "rnet_decoder_prefill": [_P, _P, _I],
    "rnet_decoder_step": [_P, _P],
    "rnet_decoder_generate": [_P, _I, _P, _I],
    "rnet_decoder_set_sampling": [_P, _F, _F, ctypes.c_ulonglong],
    "rnet_decoder_outputs": [_P, ctypes.POINTER(_P), ctypes.POINTER(_P)],
    "rnet_decoder_state": [_P, ctypes.POINTER(_P), ctypes.POINTER(_SZ)],
    "rnet_decoder_outputs_host": [_P, _P, _P],
    "rnet_dist_unique_id": [ctypes.c_char_p],
    "rnet_dist_create": [_I, _I, _I, ctypes.c_char_p, _I, ctypes.POINTER(_P)],
    "rnet_dist_destroy": [_P],
    "rnet_dist_allreduce_sum": [_P, _P, _SZ, _P],
    "rnet_dist_group_start": [_P],
    "rnet_dist_group_end": [_P],
    "rnet_dist_uid_file_write": [ctypes.c_char_p, ctypes.c_char_p],
    "rnet_dist_uid_file_read": [ctypes.c_char_p, _I, ctypes.c_char_p],
    "rnet_model_set_dist": [_P, _P],
    "rnet_data_create": [_P, _SZ, _I, ctypes.c_uint, ctypes.POINTER(_P)],
    "rnet_data_destroy": [_P],
    "rnet_data_batch": [_P, _I, _I, _P, _P, _P],
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load librnet_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} not found: build it with "
                               "`python -c 'import __graft_entry__ as g; g.build()'`")
        L = ctypes.CDLL(LIB_PATH)
        L.rnet_last_error.restype = ctypes.c_char_p
        L.rnet_last_error.argtypes = []
        for name, args in _SIGS.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = _I
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return ["rnet_last_error", *_SIGS.keys()]


def check(rc: int) -> None:
    if rc != 0:
        raise RnetError(rc, lib().rnet_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def _ptr(x) -> _P:
    """Device/host address of a torch tensor, numpy array or raw int."""
    if x is None:
        return _P(0)
    if isinstance(x, int):
        return _P(x)
    if hasattr(x, "data_ptr"):
        return _P(x.data_ptr())
    if hasattr(x, "ctypes"):
        return x.ctypes.data_as(_P)
    raise TypeError(type(x))


ptr = _ptr


class Model:
    """Owning handle over an rnet_model (the reference's ResonanceNet)."""

    def __init__(self, cfg: ModelConfig, device: int = 0, reference_init: bool = True,
                 _handle: Optional[int] = None):
        self._h = _P()
        if _handle is not None:
            self._h = _P(_handle)
        else:
            check(lib().rnet_model_create(ctypes.byref(cfg), device, int(reference_init),
                                          ctypes.byref(self._h)))
        c = ModelConfig()
        check(lib().rnet_model_get_config(self._h, ctypes.byref(c)))
        self.cfg = c
        n = _SZ()
        check(lib().rnet_model_param_count(self._h, ctypes.byref(n)))
        self.num_params = n.value

    @classmethod
    def from_checkpoint(cls, path: str, device: int = 0) -> "Model":
        h = _P()
        check(lib().rnet_model_create_from_checkpoint(path.encode(), device, ctypes.byref(h)))
        return cls(None, _handle=h.value)

    def close(self) -> None:
        if self._h:
            lib().rnet_model_destroy(self._h)
            self._h = _P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # raw handle for C calls
    @property
    def handle(self) -> _P:
        return self._h

    def device_buffers(self) -> tuple[int, int]:
        p, g = _P(), _P()
        check(lib().rnet_model_device_buffers(self._h, ctypes.byref(p), ctypes.byref(g)))
        return p.value, g.value

    def stream(self) -> int:
        s = _P()
        check(lib().rnet_model_stream(self._h, ctypes.byref(s)))
        return s.value or 0

    def set_params(self, host) -> None:
        check(lib().rnet_model_set_params(self._h, _ptr(host), host.size))

    def set_params_device(self, d_params) -> None:
        check(lib().rnet_model_set_params_device(self._h, _ptr(d_params), self.num_params))

    def get_params(self):
        import numpy as np
        out = np.empty(self.num_params, np.float32)
        check(lib().rnet_model_get_params(self._h, _ptr(out), out.size))
        return out

    def get_grads(self):
        import numpy as np
        out = np.empty(self.num_params, np.float32)
        check(lib().rnet_model_get_grads(self._h, _ptr(out), out.size))
        return out

    def set_conv_quirk(self, on: bool) -> None:
        check(lib().rnet_model_set_conv_quirk(self._h, int(on)))

    def set_precision(self, bf16: bool) -> None:
        """GEMM arithmetic: fp32-accurate (default) or bf16 operands / fp32 accumulation."""
        check(lib().rnet_model_set_precision(self._h, int(bool(bf16))))

    def set_optimizer(self, momentum: float = 0.0, weight_decay: float = 0.0,
                      warmup_steps: int = 0) -> None:
        check(lib().rnet_model_set_optimizer(self._h, momentum, weight_decay, warmup_steps))

    def set_recompute(self, on: bool) -> None:
        """Keep only layer inputs and recompute each layer's caches in backward."""
        check(lib().rnet_model_set_recompute(self._h, int(bool(on))))

    def forward(self, d_tokens, d_logits, batch: int, seq_len: int) -> None:
        check(lib().rnet_model_forward(self._h, _ptr(d_tokens), _ptr(d_logits), batch, seq_len))

    def backward(self, d_dlogits, d_tokens, batch: int, seq_len: int) -> None:
        check(lib().rnet_model_backward(self._h, _ptr(d_dlogits), _ptr(d_tokens), batch, seq_len))

    def zero_grad(self) -> None:
        check(lib().rnet_model_zero_grad(self._h))

    def step(self, lr: float, clip: float) -> None:
        check(lib().rnet_model_step(self._h, lr, clip))

    def train_step(self, d_in, d_tgt, batch: int, seq_len: int, lr: float = 3e-4,
                   clip: float = 1.0, d_loss_sum=None) -> None:
        check(lib().rnet_model_train_step(self._h, _ptr(d_in), _ptr(d_tgt), batch, seq_len, lr,
                                          clip, _ptr(d_loss_sum)))

    def train_step_host(self, h_in, h_tgt, batch: int, seq_len: int, lr: float = 3e-4,
                        clip: float = 1.0) -> float:
        loss = _F()
        check(lib().rnet_model_train_step_host(self._h, _ptr(h_in), _ptr(h_tgt), batch, seq_len,
                                               lr, clip, ctypes.byref(loss)))
        return loss.value

    def topk(self, layer: int) -> tuple[int, int]:
        i, w = _P(), _P()
        check(lib().rnet_model_topk(self._h, layer, ctypes.byref(i), ctypes.byref(w)))
        return i.value, w.value

    def topk_host(self, layer: int, n_tokens: int):
        import numpy as np
        k = self.cfg.slot_top_k
        idx = np.empty(n_tokens * k, np.int32)
        w = np.empty(n_tokens * k, np.float32)
        check(lib().rnet_model_topk_host(self._h, layer, _ptr(idx), _ptr(w), idx.size))
        return idx.reshape(n_tokens, k), w.reshape(n_tokens, k)

    def save(self, path: str) -> None:
        check(lib().rnet_model_save(self._h, path.encode()))

    def save_async(self, path: str) -> None:
        check(lib().rnet_model_save_async(self._h, path.encode()))

    def save_wait(self) -> None:
        check(lib().rnet_model_save_wait(self._h))

    def load_weights(self, path: str) -> None:
        check(lib().rnet_model_load_weights(self._h, path.encode()))

    def synchronize(self) -> None:
        check(lib().rnet_model_synchronize(self._h))

    def profile_enable(self, on: bool = True) -> None:
        check(lib().rnet_model_profile_enable(self._h, int(on)))

    def profile_read(self, reset: bool = True) -> dict:
        """{kind: {ms, flops, bytes, launches}} of the timed launch groups."""
        import numpy as np
        n = len(PROFILE_KINDS)
        ms, fl, by = (np.zeros(n, np.float64) for _ in range(3))
        la = np.zeros(n, np.int64)
        check(lib().rnet_model_profile_read(self._h, _ptr(ms), _ptr(fl), _ptr(by), _ptr(la), n,
                                            int(reset)))
        return {k: dict(ms=float(ms[i]), flops=float(fl[i]), bytes=float(by[i]),
                        launches=int(la[i])) for i, k in enumerate(PROFILE_KINDS)}

    def set_dist(self, dist: Optional["Dist"]) -> None:
        check(lib().rnet_model_set_dist(self._h, dist.handle if dist else _P(0)))


class Decoder:
    """Batched recurrent decoder over a Model (n_streams in lock step)."""

    def __init__(self, model: Model, n_streams: int):
        self.model = model
        self.M = n_streams
        self.handle = _P()
        check(lib().rnet_decoder_create(model.handle, n_streams, ctypes.byref(self.handle)))

    def prefill(self, d_tokens, seq_len: int) -> None:
        check(lib().rnet_decoder_prefill(self.handle, _ptr(d_tokens), seq_len))

    def step(self, d_tokens=None) -> None:
        check(lib().rnet_decoder_step(self.handle, _ptr(d_tokens)))

    def set_sampling(self, temperature: float = 0.0, top_p: float = 1.0, seed: int = 0) -> None:
        """Greedy (temperature 0) or temperature + top-p sampling on the device."""
        check(lib().rnet_decoder_set_sampling(self.handle, temperature, top_p, seed))

    def generate(self, n_steps: int, d_out=None, use_graph: bool = True) -> None:
        check(lib().rnet_decoder_generate(self.handle, n_steps, _ptr(d_out), int(use_graph)))

    def outputs(self) -> tuple[int, int]:
        lg, nx = _P(), _P()
        check(lib().rnet_decoder_outputs(self.handle, ctypes.byref(lg), ctypes.byref(nx)))
        return lg.value, nx.value

    def outputs_host(self):
        """(logits [M, V], next tokens [M]) as numpy arrays."""
        import numpy as np
        lg = np.empty((self.M, self.model.cfg.vocab_size), np.float32)
        nx = np.empty(self.M, np.int32)
        check(lib().rnet_decoder_outputs_host(self.handle, _ptr(lg), _ptr(nx)))
        return lg, nx

    def state(self) -> tuple[int, int]:
        p, n = _P(), _SZ()
        check(lib().rnet_decoder_state(self.handle, ctypes.byref(p), ctypes.byref(n)))
        return p.value, n.value

    def close(self) -> None:
        if self.handle:
            lib().rnet_decoder_destroy(self.handle)
            self.handle = _P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Dist:
    """NCCL communicator (the reference's DistState)."""

    def __init__(self, rank: int, world: int, local_rank: int, uid: bytes,
                 timeout_ms: int = 120000):
        assert len(uid) == 128
        self.handle = _P()
        check(lib().rnet_dist_create(rank, world, local_rank, uid, timeout_ms,
                                     ctypes.byref(self.handle)))
        self.rank, self.world = rank, world

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().rnet_dist_unique_id(buf))
        return buf.raw

    def allreduce_sum(self, d_buf, count: int, stream: int = 0) -> None:
        check(lib().rnet_dist_allreduce_sum(self.handle, _ptr(d_buf), count, _P(stream)))

    def close(self) -> None:
        if self.handle:
            lib().rnet_dist_destroy(self.handle)
            self.handle = _P()


class DataLoader:
    """The reference's batch sampler with the corpus resident on the GPU
    (rnet_data_*): same batches as src/data_loader.cpp for the same seed."""

    def __init__(self, corpus: Optional[bytes], device: int = 0, seed: int = 42):
        self.handle = _P()
        buf = corpus or b""
        check(lib().rnet_data_create(buf if buf else None, len(buf), device, seed,
                                     ctypes.byref(self.handle)))

    def batch(self, batch: int, seq_len: int, d_inputs, d_targets, stream=None) -> None:
        check(lib().rnet_data_batch(self.handle, batch, seq_len, _ptr(d_inputs), _ptr(d_targets),
                                    _ptr(stream)))

    def close(self) -> None:
        if self.handle:
            lib().rnet_data_destroy(self.handle)
            self.handle = _P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


PROFILE_KINDS = ("gemm", "scan_fwd", "scan_bwd", "conv_fwd", "conv_bwd", "rms_fwd", "rms_bwd",
                 "slot_gather", "slot_sparse_bwd", "embed", "cross_entropy", "sgd", "other",
                 "comm_wait")


def kernel_launches() -> int:
    n = ctypes.c_ulonglong(0)
    check(lib().rnet_kernel_launches(ctypes.byref(n)))
    return n.value


def device_error(clear: bool = True) -> int:
    w = ctypes.c_uint(0)
    check(lib().rnet_device_error(ctypes.byref(w), int(clear)))
    return w.value
