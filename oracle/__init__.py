"""TEST INFRASTRUCTURE ONLY: ctypes wrapper over the C restatement of the
reference's CPU arithmetic (``oracle/aljabr_oracle.c``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs use this package, and only as the checker or the timed CPU baseline.
The product path (``aljabr_b200``) never imports it.

Parity status: Q4_0 (raw and prepared-cache order) / Q8_0 / Q4_K / Q6_K /
fp16 / attention restatements are pinned by the reference's known-answer
tests (``tests/golden/``).  The NF4 fp32 GEMV (Apple
Accelerate ``cblas_sgemv`` in the reference) and the NF4 quantizer (external
project) are "parity unpinned"; NF4 dequantisation is pinned by its table and
nibble order.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "aljabr_oracle.c")
_HDR = os.path.join(_HERE, "aljabr_oracle.h")
_LIB = os.path.join(_HERE, "liboracle.so")

CFLAGS = ["-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math", "-pthread"]

Q4_0, Q8_0, Q4_K, Q6_K, NF4 = 2, 8, 12, 14, 100
K_BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}   # per 256-value super-block


def build(force: bool = False) -> str:
    """Compile the restatement into ``oracle/liboracle.so`` (gcc)."""
    stale = (not os.path.exists(_LIB)) or any(
        os.path.getmtime(p) > os.path.getmtime(_LIB) for p in (_SRC, _HDR))
    if force or stale:
        subprocess.check_call(["gcc", *CFLAGS, _SRC, "-o", _LIB, "-lm"])
    return _LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()   # compiles only when the library is missing or older than the sources
        _lib = ctypes.CDLL(_LIB)
        _declare(_lib)
    return _lib


_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float


def _declare(L):
    L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.orc_f16_to_f32.restype = _f
    L.orc_f32_to_f16_bits.argtypes = [_f]
    L.orc_f32_to_f16_bits.restype = ctypes.c_uint16
    L.orc_java_round.argtypes = [_f]
    L.orc_java_round.restype = _i
    L.orc_f32_to_bf16_rne.argtypes = [_f]
    L.orc_f32_to_bf16_rne.restype = ctypes.c_uint16
    for name in ("orc_encode_q4_0", "orc_encode_q8_0"):
        getattr(L, name).argtypes = [_p, _i64, _p]
    L.orc_quantize_nf4.argtypes = [_p, _i64, _i, _p, _p]
    L.orc_dequantize_nf4.argtypes = [_p, _p, _p, _i64, _i]
    L.orc_dequantize_q4_0.argtypes = [_p, _p, _i64]
    L.orc_dequantize_q8_0.argtypes = [_p, _p, _i64]
    for name in ("orc_dot_row_q4_0", "orc_dot_row_q8_0_scalar", "orc_dot_row_q8_0_vector"):
        getattr(L, name).argtypes = [_p, _i, _p]
        getattr(L, name).restype = _f
    L.orc_matvec_q4_0.argtypes = [_p, _p, _p, _i, _i, _i]
    L.orc_matvec_q4_0_prepared.argtypes = [_p, _p, _p, _i, _i, _i]
    L.orc_dot_row_q4_0_prepared.argtypes = [_p, _i, _p]
    L.orc_dot_row_q4_0_prepared.restype = _f
    L.orc_set_decode_threads.argtypes = [_i]
    L.orc_rmsnorm_binding.argtypes = [_p, _p, _p, _i, _f]
    L.orc_silu_ffn_binding.argtypes = [_p, _p, _p, _i]
    L.orc_matvec_q8_0.argtypes = [_p, _p, _p, _i, _i, _i, _i]
    for name in ("orc_dot_row_q4_k", "orc_dot_row_q6_k"):
        getattr(L, name).argtypes = [_p, _i, _p]
        getattr(L, name).restype = _f
    L.orc_dequantize_k_row.argtypes = [_i, _p, _i, _p]
    L.orc_matvec_k.argtypes = [_i, _p, _p, _p, _i, _i, _i]
    L.orc_matvec_nf4.argtypes = [_p, _p, _p, _p, _i, _i, _i, _p, _i]
    L.orc_matvec_f64.argtypes = [_i, _p, _p, _p, _p, _i, _i, _i, _i]
    L.orc_gqa_decode_attention.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _f]
    L.orc_prefill_attention.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i]
    L.orc_fa4_attention.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _f, _i, _f]
    L.orc_vec_dot.argtypes = [_p, _p, _i]
    L.orc_vec_dot.restype = _f
    L.orc_rms_norm.argtypes = [_p, _p, _p, _i, _f]
    L.orc_rope.argtypes = [_p, _i, _i, _i, _i, _f]
    L.orc_swiglu.argtypes = [_p, _p, _p, _i]
    L.orc_softmax.argtypes = [_p, _i]
    L.orc_decode_step_nf4.argtypes = [_p, _p, _p, _p, _p, _p, _i, _i, _i, _p, _p]
    L.orc_decode_step_typed.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _p, _p]
    L.orc_dequantize_row_ref.argtypes = [_i, _p, _i, _p]


def _ptr(a):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------- scalars
def f16_to_f32(bits: int) -> float:
    return lib().orc_f16_to_f32(bits)


def f16_to_f32_array(bits) -> np.ndarray:
    """Vector form of RT/GgufQuantTables.f16ToF32 (via the 64K table)."""
    table = _f16_table()
    return table[np.asarray(bits, dtype=np.uint16)]


_F16 = None


def _f16_table():
    global _F16
    if _F16 is None:
        L = lib()
        _F16 = np.array([L.orc_f16_to_f32(i) for i in range(65536)], dtype=np.float32)
    return _F16


def f32_to_f16_bits(v: float) -> int:
    return lib().orc_f32_to_f16_bits(v)


def java_round(v: float) -> int:
    return lib().orc_java_round(v)


def f32_to_bf16_bits(a) -> np.ndarray:
    """bf16 round-to-nearest-even bit patterns of a float32 array."""
    a = _c(a, np.float32)
    b = a.view(np.uint32).astype(np.uint64)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- encoders
def encode_q4_0(values) -> np.ndarray:
    v = _c(values, np.float32).ravel()
    assert v.size % 32 == 0
    out = np.empty(v.size // 32 * 18, dtype=np.uint8)
    lib().orc_encode_q4_0(_ptr(v), v.size, _ptr(out))
    return out


def encode_q8_0(values) -> np.ndarray:
    v = _c(values, np.float32).ravel()
    assert v.size % 32 == 0
    out = np.empty(v.size // 32 * 34, dtype=np.uint8)
    lib().orc_encode_q8_0(_ptr(v), v.size, _ptr(out))
    return out


def quantize_nf4(values, group_size: int):
    v = _c(values, np.float32).ravel()
    codes = np.zeros((v.size + 1) // 2, dtype=np.uint8)
    absmax = np.zeros((v.size + group_size - 1) // group_size, dtype=np.float32)
    lib().orc_quantize_nf4(_ptr(v), v.size, group_size, _ptr(codes), _ptr(absmax))
    return codes, absmax


# ---------------------------------------------------------------- dequant
def dequantize_nf4(codes, absmax, numel: int, group_size: int) -> np.ndarray:
    codes = _c(codes, np.uint8)
    absmax = _c(absmax, np.float32)
    out = np.empty(numel, dtype=np.float32)
    lib().orc_dequantize_nf4(_ptr(codes), _ptr(out), _ptr(absmax), numel, group_size)
    return out


def dequantize_q4_0(blocks, numel: int) -> np.ndarray:
    blocks = _c(blocks, np.uint8)
    out = np.empty(numel, dtype=np.float32)
    lib().orc_dequantize_q4_0(_ptr(blocks), _ptr(out), numel)
    return out


def dequantize_q8_0(blocks, numel: int) -> np.ndarray:
    blocks = _c(blocks, np.uint8)
    out = np.empty(numel, dtype=np.float32)
    lib().orc_dequantize_q8_0(_ptr(blocks), _ptr(out), numel)
    return out


# ---------------------------------------------------------------- dots / matvec
def dot_row_q4_0(row, x) -> float:
    row, x = _c(row, np.uint8), _c(x, np.float32)
    return lib().orc_dot_row_q4_0(_ptr(row), x.size, _ptr(x))


def dot_row_q4_0_prepared(row, x) -> float:
    row, x = _c(row, np.uint8), _c(x, np.float32)
    return lib().orc_dot_row_q4_0_prepared(_ptr(row), x.size, _ptr(x))


def dot_row_q8_0(row, x, vector_order: bool = True) -> float:
    row, x = _c(row, np.uint8), _c(x, np.float32)
    fn = lib().orc_dot_row_q8_0_vector if vector_order else lib().orc_dot_row_q8_0_scalar
    return fn(_ptr(row), x.size, _ptr(x))


def matvec_q4_0(w, x, N: int, threads: int = 1) -> np.ndarray:
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty(N, dtype=np.float32)
    lib().orc_matvec_q4_0(_ptr(w), _ptr(x), _ptr(y), x.size, N, threads)
    return y


def matvec_q4_0_prepared(w, x, N: int, threads: int = 1) -> np.ndarray:
    """Q4_0 in the prepared-cache order, the reference's default for >= 32 rows."""
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty(N, dtype=np.float32)
    lib().orc_matvec_q4_0_prepared(_ptr(w), _ptr(x), _ptr(y), x.size, N, threads)
    return y


def matvec_q8_0(w, x, N: int, vector_order: bool = True, threads: int = 1) -> np.ndarray:
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty(N, dtype=np.float32)
    lib().orc_matvec_q8_0(_ptr(w), _ptr(x), _ptr(y), x.size, N, int(vector_order), threads)
    return y


def dot_row_k(kind: int, row, x) -> float:
    """One Q4_K / Q6_K row dot in the reference's float order."""
    row, x = _c(row, np.uint8), _c(x, np.float32)
    fn = lib().orc_dot_row_q4_k if kind == Q4_K else lib().orc_dot_row_q6_k
    return fn(_ptr(row), x.size, _ptr(x))


def dequantize_k_row(kind: int, row, columns: int) -> np.ndarray:
    """The values of one Q4_K / Q6_K row (fp64, from the element formulas)."""
    row = _c(row, np.uint8)
    out = np.empty(columns, dtype=np.float64)
    lib().orc_dequantize_k_row(kind, _ptr(row), columns, _ptr(out))
    return out


def dequantize_row_ref(kind: int, row, columns: int) -> np.ndarray:
    """One GGUF row as float32 in the reference's dequantiser order
    (GgufBlockDequantizer / GgufKBlockDequantizer), as the typed decode
    step's embedding lookup uses it."""
    row = _c(row, np.uint8)
    out = np.empty(columns, dtype=np.float32)
    lib().orc_dequantize_row_ref(kind, _ptr(row), columns, _ptr(out))
    return out


def matvec_k(kind: int, w, x, N: int, threads: int = 1) -> np.ndarray:
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty(N, dtype=np.float32)
    lib().orc_matvec_k(kind, _ptr(w), _ptr(x), _ptr(y), x.size, N, threads)
    return y


def matvec_nf4(codes, absmax, x, N: int, group_size: int, bias=None, threads: int = 1) -> np.ndarray:
    codes, absmax, x = _c(codes, np.uint8), _c(absmax, np.float32), _c(x, np.float32)
    bias = None if bias is None else _c(bias, np.float32)
    y = np.empty(N, dtype=np.float32)
    lib().orc_matvec_nf4(_ptr(codes), _ptr(absmax), _ptr(x), _ptr(y), x.size, N, group_size,
                         _ptr(bias), threads)
    return y


def matvec_f64(kind: int, w, x, N: int, absmax=None, group_size: int = 64, threads: int = 1) -> np.ndarray:
    w, x = _c(w, np.uint8), _c(x, np.float32)
    absmax = None if absmax is None else _c(absmax, np.float32)
    y = np.empty(N, dtype=np.float64)
    lib().orc_matvec_f64(kind, _ptr(w), _ptr(absmax), _ptr(x), _ptr(y), x.size, N, group_size, threads)
    return y


# ---------------------------------------------------------------- attention / glue
def gqa_decode_attention(q, k_cache, v_cache, stride: int, kv_heads: int, q_heads: int,
                         head_dim: int, seq_len: int, start_pos: int, scale: float) -> np.ndarray:
    q = _c(q, np.float32)
    k_cache, v_cache = _c(k_cache, np.float32), _c(v_cache, np.float32)
    out = np.empty(q_heads * head_dim, dtype=np.float32)
    scores = np.empty(max(seq_len - start_pos, 1), dtype=np.float32)
    lib().orc_gqa_decode_attention(_ptr(q), _ptr(out), _ptr(scores), _ptr(k_cache), _ptr(v_cache),
                                   stride, kv_heads, q_heads, head_dim, seq_len, start_pos, scale)
    return out


def prefill_attention(q, k, v, tokens: int, q_heads: int, kv_heads: int, head_dim: int, scale: float,
                      window: int = 0, kv_stride: int = 0) -> np.ndarray:
    """GgufPrefillAttentionExecution's Java loop: q [tokens][q_heads*head_dim],
    k / v [tokens][kv_stride] (kv_stride 0: kv_heads*head_dim); returns
    [tokens][q_heads*head_dim]."""
    kv_stride = kv_stride or kv_heads * head_dim
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.empty(tokens * q_heads * head_dim, dtype=np.float32)
    scores = np.empty(max(tokens, 1), dtype=np.float32)
    lib().orc_prefill_attention(_ptr(out), _ptr(q), _ptr(k), _ptr(v), _ptr(scores), tokens, q_heads, kv_heads,
                                head_dim, scale, window, kv_stride)
    return out.reshape(tokens, q_heads * head_dim)


def fa4_attention(q, k, v, B: int, T: int, S: int, H: int, H_kv: int, D: int, scale: float,
                  causal: bool = True, soft_cap: float = 0.0) -> np.ndarray:
    """The FlashAttention-4 seam's CPU contract (MetalFlashAttentionCpuFallback):
    q [B][T][H][D], k / v [B][S][H_kv][D]; returns [B][T][H][D] flat."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.empty(B * T * H * D, dtype=np.float32)
    scores = np.empty(max(S, 1), dtype=np.float32)
    lib().orc_fa4_attention(_ptr(out), _ptr(q), _ptr(k), _ptr(v), _ptr(scores), B, T, S, H, H_kv, D, scale,
                            1 if causal else 0, soft_cap)
    return out


def rms_norm(x, w, eps: float) -> np.ndarray:
    x, w = _c(x, np.float32), _c(w, np.float32)
    out = np.empty_like(x)
    lib().orc_rms_norm(_ptr(x), _ptr(w), _ptr(out), x.size, eps)
    return out


def rmsnorm_binding(x, w, eps: float) -> np.ndarray:
    """BlackwellCpuFallback.rmsNorm: the FFM binding's RMSNorm contract."""
    x, w = _c(x, np.float32), _c(w, np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm_binding(_ptr(x), _ptr(w), _ptr(out), x.size, eps)
    return out


def silu_ffn_binding(gate, up) -> np.ndarray:
    """BlackwellCpuFallback.siluFfn: out = silu(gate) * up."""
    gate, up = _c(gate, np.float32), _c(up, np.float32)
    out = np.empty_like(gate)
    lib().orc_silu_ffn_binding(_ptr(gate), _ptr(up), _ptr(out), gate.size)
    return out


def rope(x, n_heads: int, head_dim: int, pos: int, freq_base: float) -> np.ndarray:
    x = _c(x, np.float32).copy()
    lib().orc_rope(_ptr(x), n_heads, head_dim, head_dim, pos, freq_base)
    return x


def swiglu(gate, up) -> np.ndarray:
    gate, up = _c(gate, np.float32), _c(up, np.float32)
    out = np.empty_like(gate)
    lib().orc_swiglu(_ptr(gate), _ptr(up), _ptr(out), gate.size)
    return out


class LlamaCfg(ctypes.Structure):
    _fields_ = [("layers", _i), ("hidden", _i), ("q_heads", _i), ("kv_heads", _i),
                ("head_dim", _i), ("ffn", _i), ("vocab", _i), ("max_ctx", _i), ("group", _i),
                ("eps", _f), ("rope_theta", _f)]


def set_decode_threads(threads: int) -> None:
    """Host threads for the decode-step restatements' matvecs (speed only)."""
    lib().orc_set_decode_threads(int(threads))


def decode_step_nf4(cfg: LlamaCfg, codes: list, absmax: list, norms, k_cache, v_cache,
                    token: int, pos: int, want_logits: bool = True):
    """One decode step (DP:297-545); k_cache/v_cache ([layers][max_ctx][Hkv*D],
    float32 or uint16 bf16 bits) are updated in place at `pos`.
    Returns (x, logits)."""
    codes = [_c(c, np.uint8) for c in codes]
    absmax = [_c(a, np.float32) for a in absmax]
    cp = (ctypes.c_void_p * len(codes))(*[c.ctypes.data for c in codes])
    ap = (ctypes.c_void_p * len(absmax))(*[a.ctypes.data for a in absmax])
    norms = _c(norms, np.float32)
    assert k_cache.dtype in (np.uint16, np.float32) and k_cache.flags.c_contiguous
    assert v_cache.dtype == k_cache.dtype and v_cache.flags.c_contiguous
    kv_bf16 = int(k_cache.dtype == np.uint16)
    x = np.empty(cfg.hidden, dtype=np.float32)
    logits = np.empty(cfg.vocab, dtype=np.float32) if want_logits else None
    lib().orc_decode_step_nf4(ctypes.byref(cfg), cp, ap, _ptr(norms), _ptr(k_cache), _ptr(v_cache),
                              kv_bf16, token, pos, _ptr(x), _ptr(logits))
    return x, logits


def decode_step_typed(cfg: LlamaCfg, weights: list, types: list, absmax: list, norms, k_cache, v_cache,
                      token: int, pos: int, want_logits: bool = True):
    """decode_step_nf4 with one GGUF type per tensor (Q4_0 / Q8_0 / Q4_K /
    Q6_K / NF4; absmax[i] is used only for NF4 tensors and may be None)."""
    weights = [_c(w, np.uint8) for w in weights]
    absmax = [None if a is None else _c(a, np.float32) for a in absmax]
    wp = (ctypes.c_void_p * len(weights))(*[w.ctypes.data for w in weights])
    ap = (ctypes.c_void_p * len(absmax))(*[None if a is None else a.ctypes.data for a in absmax])
    tp = (ctypes.c_int * len(types))(*types)
    norms = _c(norms, np.float32)
    assert k_cache.dtype in (np.uint16, np.float32) and k_cache.flags.c_contiguous
    assert v_cache.dtype == k_cache.dtype and v_cache.flags.c_contiguous
    kv_bf16 = int(k_cache.dtype == np.uint16)
    x = np.empty(cfg.hidden, dtype=np.float32)
    logits = np.empty(cfg.vocab, dtype=np.float32) if want_logits else None
    lib().orc_decode_step_typed(ctypes.byref(cfg), wp, tp, ap, _ptr(norms), _ptr(k_cache), _ptr(v_cache),
                                kv_bf16, token, pos, _ptr(x), _ptr(logits))
    return x, logits
