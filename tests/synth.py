"""Seeded synthetic inputs with the BASELINE configs' distributions
(weights N(0, 0.02), activations N(0, 1)); used by tests and smoke."""
from __future__ import annotations

import json
import struct

import numpy as np

import oracle


def rng(seed: int):
    return np.random.default_rng(seed)


def weights(seed: int, n: int, k: int, std: float = 0.02) -> np.ndarray:
    return rng(seed).normal(0.0, std, size=(n, k)).astype(np.float32)


def activation(seed: int, k: int) -> np.ndarray:
    return rng(seed).normal(0.0, 1.0, size=k).astype(np.float32)


def q4_0(seed: int, n: int, k: int) -> np.ndarray:
    return oracle.encode_q4_0(weights(seed, n, k))


def q8_0(seed: int, n: int, k: int) -> np.ndarray:
    return oracle.encode_q8_0(weights(seed, n, k))


def nf4(seed: int, n: int, k: int, group: int = 64):
    return oracle.quantize_nf4(weights(seed, n, k), group)


def k_quant(kind: int, seed: int, n: int, k: int) -> np.ndarray:
    """n rows of k values as random Q4_K / Q6_K super-blocks: random code,
    scale and min bytes (every pattern is a valid block) with small positive
    fp16 super-block scales, the magnitudes GGUF files carry."""
    g = np.random.default_rng(seed)
    bb = oracle.K_BLOCK_BYTES[kind]
    blocks = g.integers(0, 256, size=(n * (k // 256), bb), dtype=np.uint8)
    f16 = lambda v: np.array([oracle.f32_to_f16_bits(float(t)) for t in v], dtype=np.uint16).view(np.uint8).reshape(-1, 2)
    nb = blocks.shape[0]
    if kind == oracle.Q4_K:
        blocks[:, 0:2] = f16(g.uniform(2e-4, 1e-3, nb))
        blocks[:, 2:4] = f16(g.uniform(1e-4, 5e-4, nb))
    else:
        blocks[:, 208:210] = f16(g.uniform(5e-5, 3e-4, nb))
    return blocks.reshape(-1)


def max_rel_err(got, ref) -> float:
    """max_i |got_i - ref_i| / max(|ref_i|, 1e-3 * max|ref|): the north-star
    metric (element-wise relative error, guarded where ref_i is near zero)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    floor = 1e-3 * max(np.abs(ref).max(), 1e-30)
    return float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), floor)))


def normwise_rel_err(got, ref) -> float:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


_ST_TAGS = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.uint8): "U8",
            np.dtype(np.int8): "I8", np.dtype(np.int32): "I32", np.dtype(np.uint32): "U32",
            np.dtype(np.int64): "I64", np.dtype(np.float64): "F64"}


def write_safetensors(path: str, tensors: dict, align: int = 8) -> None:
    """Minimal safetensors writer (test fixture): name -> numpy array, or
    name -> ("BF16", uint16 array).  Header padded with spaces to `align`."""
    header, blobs, off = {}, [], 0
    for name, v in tensors.items():
        tag, arr = v if isinstance(v, tuple) else (_ST_TAGS[np.asarray(v).dtype], v)
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": tag, "shape": list(np.asarray(arr).shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((-(8 + len(hb))) % align)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)
