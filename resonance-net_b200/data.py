"""Synthetic inputs, parameter layouts and checkpoint files (host side).

Checkpoint layout follows the reference (src/resonance_net.cpp:743-782): the
40-byte ModelConfig header, then every parameter tensor as raw fp32 in a fixed
order. `tensor_layout()` names that order; the library's flat parameter and
gradient buffers use the same order.
"""
from __future__ import annotations

import struct

import numpy as np

HEADER_FMT = "<9if"  # 9 x int32 + float32 rms_eps = 40 bytes


def tensor_layout(cfg) -> list[tuple[str, int]]:
    D, V, F, S = cfg.d_model, cfg.vocab_size, cfg.d_ff, cfg.n_slots
    out = [("embed", V * D), ("output", V * D), ("final_norm", D)]
    for l in range(cfg.n_layers):
        p = f"L{l}."
        out += [(p + "norm1", D), (p + "norm2", D), (p + "norm3", D), (p + "norm4", D),
                (p + "conv3", 3 * D), (p + "conv7", 7 * D), (p + "conv15", 15 * D),
                (p + "mix", D * D), (p + "Wz", D * D), (p + "Wh", D * D), (p + "bz", D),
                (p + "bh", D), (p + "slot_keys", D * S), (p + "slot_values", D * S),
                (p + "proj_q", D * D), (p + "proj_out", D * D), (p + "gate", F * D),
                (p + "up", F * D), (p + "down", D * F)]
    return out


def param_count(cfg) -> int:
    return sum(n for _, n in tensor_layout(cfg))


def split(cfg, flat: np.ndarray) -> dict[str, np.ndarray]:
    out, off = {}, 0
    for name, n in tensor_layout(cfg):
        out[name] = flat[off:off + n]
        off += n
    return out


def init_params_normal(cfg, seed: int = 1234, std: float = 0.02) -> np.ndarray:
    """N(0, std) weights drawn in checkpoint order with one PCG64 stream;
    RMSNorm gains 1, MinGRU biases 0."""
    rng = np.random.default_rng(seed)
    parts = []
    for name, n in tensor_layout(cfg):
        base = name.split(".")[-1]
        if base.startswith("norm") or base == "final_norm":
            parts.append(np.ones(n, np.float32))
        elif base in ("bz", "bh"):
            parts.append(np.zeros(n, np.float32))
        else:
            parts.append(rng.normal(0.0, std, n).astype(np.float32))
    return np.concatenate(parts)


def uniform_tokens(B: int, T: int, seed: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """i.i.d. uniform bytes; targets are the following byte of the same row."""
    rng = np.random.default_rng(seed)
    seq = rng.integers(0, 256, size=(B, T + 1), dtype=np.int64).astype(np.int32)
    return np.ascontiguousarray(seq[:, :T]), np.ascontiguousarray(seq[:, 1:])


def zipf_bytes(n: int, seed: int = 7, s: float = 1.1) -> np.ndarray:
    """n bytes drawn i.i.d. from Zipf(s) over ranks 1..256, mapped to byte
    values through a permutation seeded by `seed`."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(256)
    p = 1.0 / np.arange(1, 257, dtype=np.float64) ** s
    p /= p.sum()
    ranks = rng.choice(256, size=n, p=p)
    return perm[ranks].astype(np.uint8)


def zipf_tokens(B: int, T: int, seed: int = 7, s: float = 1.1) -> tuple[np.ndarray, np.ndarray]:
    seq = zipf_bytes(B * (T + 1), seed=seed, s=s).astype(np.int32).reshape(B, T + 1)
    return np.ascontiguousarray(seq[:, :T]), np.ascontiguousarray(seq[:, 1:])


def write_checkpoint(path: str, cfg, params: np.ndarray) -> None:
    hdr = struct.pack(HEADER_FMT, cfg.d_model, cfg.n_layers, cfg.d_ff, cfg.n_heads, cfg.gru_dim,
                      cfg.n_slots, cfg.slot_top_k, cfg.vocab_size, cfg.seq_len, cfg.rms_eps)
    assert len(hdr) == 40
    with open(path, "wb") as f:
        f.write(hdr)
        f.write(np.ascontiguousarray(params, np.float32).tobytes())


def read_checkpoint(path: str) -> tuple[tuple, np.ndarray]:
    with open(path, "rb") as f:
        hdr = struct.unpack(HEADER_FMT, f.read(40))
        params = np.frombuffer(f.read(), np.float32).copy()
    return hdr, params
