"""ctypes binding of libaljabr_blackwell.so (include/aljabr_blackwell.h).

This is the same surface a Java FFM binding (BlackwellBinding) downcalls; the
Python side exists so the parity tests and the benchmark drive exactly the
C-ABI a JVM would.  There is no CPU fallback: if the library is missing or a
call fails, an exception says why.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libaljabr_blackwell.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "aljabr_blackwell.h")

ALJ_OK = 0
ALJ_ERR_NOT_INITIALIZED = -1
ALJ_ERR_BAD_DIMS = -2
ALJ_ERR_UNSUPPORTED = -3
ALJ_ERR_NOT_REGISTERED = -4
ALJ_ERR_CUDA = -5
ALJ_ERR_TIMEOUT = -6
ALJ_ERR_BAD_ARG = -7
ALJ_ERR_NO_MEMORY = -8

TYPE_Q4_0 = 2
TYPE_Q8_0 = 8
TYPE_NF4 = 100
TYPE_Q4_K = 12
TYPE_Q6_K = 14
KV_F32 = 0
KV_BF16 = 1


class ProviderError(RuntimeError):
    """A non-zero status from the native provider (mirrors ProviderException)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"aljabr_blackwell error {code}: {message}")
        self.code = code


class UnsupportedOperation(ProviderError):
    """ALJ_ERR_UNSUPPORTED (mirrors UnsupportedOperationException)."""


_p = ctypes.c_void_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol declared in the header is listed.
SIGNATURES = {
    "aljabr_blackwell_init": (_i, [_i]),
    "aljabr_blackwell_device_count": (_i, []),
    "aljabr_blackwell_device_get": (_i, [_i]),
    "aljabr_blackwell_device_name": (_i, [ctypes.c_char_p, _i, _i]),
    "aljabr_blackwell_compute_capability": (_i, [_i]),
    "aljabr_blackwell_tmem_size": (_ll, [_i]),
    "aljabr_blackwell_free_memory": (_ll, []),
    "aljabr_blackwell_last_error": (ctypes.c_char_p, []),
    "aljabr_blackwell_set_verbose": (None, [_i]),
    "aljabr_blackwell_device_status": (_i, [ctypes.POINTER(ctypes.c_uint)]),
    "aljabr_blackwell_shutdown": (_i, []),
    "aljabr_blackwell_set_pdl": (_i, [_i]),
    "aljabr_blackwell_prefetch_hint": (_i, [_p, _sz]),
    "aljabr_blackwell_register_model_buffer": (_i, [_p, _sz]),
    "aljabr_blackwell_unregister_model_buffer": (_i, [_p]),
    "aljabr_blackwell_device_address": (_p, [_p]),
    "aljabr_blackwell_matvec_tb_q4_0": (_i, [_p, _p, _p, _i, _i]),
    "aljabr_blackwell_matvec_tb_q8_0": (_i, [_p, _p, _p, _i, _i]),
    "aljabr_blackwell_matvec_tb_q4_k": (_i, [_p, _p, _p, _i, _i]),
    "aljabr_blackwell_matvec_tb_q6_k": (_i, [_p, _p, _p, _i, _i]),
    "aljabr_blackwell_matvec_tb_nf4": (_i, [_p, _p, _p, _p, _i, _i, _i]),
    "aljabr_blackwell_linear_nf4": (_i, [_p, _p, _p, _p, _p, _i, _i, _i]),
    "aljabr_blackwell_matvec_tb_pair": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i]),
    "aljabr_blackwell_matvec_tb_triple": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i]),
    "aljabr_blackwell_matvec_tb_batch": (_i, [_p, _p, _p, _i, _i, _i, _i]),
    "aljabr_blackwell_matvec_tb_triple_batch": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _i]),
    "aljabr_blackwell_dequantize_nf4": (_i, [_p, _p, _p, _ll, _i]),
    "aljabr_blackwell_dequantize_q4_0": (_i, [_p, _p, _ll]),
    "aljabr_blackwell_dequantize_q8_0": (_i, [_p, _p, _ll]),
    "aljabr_blackwell_rmsnorm": (_i, [_p, _p, _p, _i, _f]),
    "aljabr_blackwell_silu_ffn": (_i, [_p, _p, _p, _i]),
    "aljabr_blackwell_decode_attention": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f]),
    "aljabr_blackwell_matvec_dev": (_i, [_i, _p, _p, _p, _p, _i, _i, _i, _p, _p]),
    "aljabr_blackwell_dequantize_dev": (_i, [_i, _p, _p, _p, _ll, _i, _p]),
    "aljabr_blackwell_decode_attention_dev": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _p]),
    "aljabr_blackwell_decode_attention_noalloc": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _p]),
    "aljabr_blackwell_prefill_attention": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i]),
    "aljabr_blackwell_fa4_attention": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _f, _i, _i, _f]),
    "aljabr_blackwell_fa4_sdpa_available": (_i, []),
    "aljabr_blackwell_fa4_bf16_available": (_i, []),
    "aljabr_blackwell_prefill_attention_dev": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _i, _i, _f, _p]),
    "aljabr_blackwell_gemm_nf4_workspace_size": (_ll, [_i, _i, _i, _p]),
    "aljabr_blackwell_gemm_nf4_packed_size": (_ll, [_i, _i, _i]),
    "aljabr_blackwell_gemm_nf4_pack": (_i, [_p, _p, _p, _i, _i, _i, _p]),
    "aljabr_blackwell_gemm_nf4_dev": (_i, [_i, _p, _p, _p, _p, _p, _i, _i, _i, _p, _ll, _p]),
    "aljabr_blackwell_gemm_q_packed_size": (_ll, [_i, _i, _i]),
    "aljabr_blackwell_gemm_q_pack": (_i, [_i, _p, _p, _i, _i, _p]),
    "aljabr_blackwell_gemm_q_workspace_size": (_ll, [_i, _i]),
    "aljabr_blackwell_gemm_q_dev": (_i, [_i, _i, _p, _p, _p, _p, _p, _i, _i, _p, _ll, _p]),
    "aljabr_blackwell_nccl_unique_id": (_i, [_p, _i]),
    "aljabr_blackwell_decode_model_create": (_i, [ctypes.POINTER(_i), _f, _f, _i, _i, _p,
                                                  ctypes.POINTER(ctypes.c_ulonglong)]),
    "aljabr_blackwell_register_decode_layer": (_i, [ctypes.c_ulonglong, _i, _p, _p, _p, _p]),
    "aljabr_blackwell_register_output": (_i, [ctypes.c_ulonglong, _p, _p, _p, _p, _p]),
    "aljabr_blackwell_register_decode_layer_typed": (_i, [ctypes.c_ulonglong, _i, _p, _p, _p, _p, _p]),
    "aljabr_blackwell_register_output_typed": (_i, [ctypes.c_ulonglong, _p, _i, _p, _p, _i, _p, _p]),
    "aljabr_blackwell_decode_step_token": (_i, [ctypes.c_ulonglong, _i, _i, _p, _p]),
    "aljabr_blackwell_decode_run": (_i, [ctypes.c_ulonglong, _i, _i, _i, _p]),
    "aljabr_blackwell_sync_kv_cache": (_i, [ctypes.c_ulonglong, _i, _i, _p, _p]),
    "aljabr_blackwell_decode_read_state": (_i, [ctypes.c_ulonglong, _p, _p, _p]),
    "aljabr_blackwell_decode_model_destroy": (_i, [ctypes.c_ulonglong]),
}


def header_symbols() -> list[str]:
    """Every function the public header declares (parsed from the header text)."""
    with open(HEADER_PATH) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(aljabr_blackwell_\w+)\s*\(", text)))


_lib = None


def lib() -> ctypes.CDLL:
    """Load the native library (built in-tree by aljabr_b200.build)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ProviderError(ALJ_ERR_NOT_INITIALIZED,
                                f"{LIB_PATH} is missing: run `python -m aljabr_b200.build` (nvcc, sm_100a)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    msg = lib().aljabr_blackwell_last_error()
    return msg.decode() if msg else ""


def check(rc: int) -> int:
    if rc != ALJ_OK:
        cls = UnsupportedOperation if rc == ALJ_ERR_UNSUPPORTED else ProviderError
        raise cls(rc, last_error())
    return rc


def call(name: str, *args) -> int:
    return check(getattr(lib(), name)(*args))


def gemm_nf4_workspace_size(M: int, K: int, rows) -> int:
    """Bytes of device workspace aljabr_blackwell_gemm_nf4_dev needs."""
    n = len(rows)
    v = lib().aljabr_blackwell_gemm_nf4_workspace_size(M, K, n, (ctypes.c_int * n)(*rows))
    if v < 0:
        check(int(v))
    return int(v)


def gemm_nf4_packed_size(rows: int, K: int, group: int) -> int:
    """Bytes of the packed form of one NF4 matrix [rows][K]."""
    v = lib().aljabr_blackwell_gemm_nf4_packed_size(rows, K, group)
    if v < 0:
        check(int(v))
    return int(v)


def gemm_nf4_pack(packed: int, codes: int, absmax: int, rows: int, K: int, group: int, stream=None) -> int:
    """Repack an NF4 matrix (device codes + absmax) for gemm_nf4_dev."""
    return call("aljabr_blackwell_gemm_nf4_pack", ctypes.c_void_p(packed), ctypes.c_void_p(codes),
                ctypes.c_void_p(absmax), rows, K, group, None if stream is None else ctypes.c_void_p(stream))


def gemm_nf4_dev(y, ldy, packed, rows, x_bf16: int, M: int, K: int, group: int,
                 workspace: int, workspace_bytes: int, stream=None) -> int:
    """Batched NF4 linear on device pointers: y[s][m * ldy[s] + n] = sum_k x[m][k] W_s[n][k],
    W_s packed by gemm_nf4_pack."""
    n = len(y)
    P = ctypes.c_void_p * n
    I = ctypes.c_int * n
    return call("aljabr_blackwell_gemm_nf4_dev", n, P(*y), I(*ldy), P(*packed), I(*rows),
                ctypes.c_void_p(x_bf16), M, K, group, ctypes.c_void_p(workspace), workspace_bytes,
                None if stream is None else ctypes.c_void_p(stream))


def gemm_q_packed_size(type_id: int, rows: int, K: int) -> int:
    """Bytes of the packed form of one Q4_0 / Q8_0 matrix [rows][K]."""
    v = lib().aljabr_blackwell_gemm_q_packed_size(type_id, rows, K)
    if v < 0:
        check(int(v))
    return int(v)


def gemm_q_workspace_size(M: int, K: int) -> int:
    """Workspace bytes of one gemm_q_dev call with M tokens."""
    v = lib().aljabr_blackwell_gemm_q_workspace_size(M, K)
    if v < 0:
        check(int(v))
    return int(v)


def gemm_q_pack(type_id: int, packed: int, weights: int, rows: int, K: int, stream=None) -> int:
    """Repack a Q4_0 / Q8_0 matrix (device GGUF blocks) for gemm_q_dev."""
    return call("aljabr_blackwell_gemm_q_pack", type_id, ctypes.c_void_p(packed), ctypes.c_void_p(weights), rows, K,
                None if stream is None else ctypes.c_void_p(stream))


def gemm_q_dev(type_id: int, y, ldy, packed, rows, x: int, M: int, K: int, workspace: int, workspace_bytes: int,
               stream=None) -> int:
    """Batched Q4_0 / Q8_0 linear on device pointers: y[s][m * ldy[s] + n] = sum_k x[m][k] W_s[n][k]
    for fp32 x, W_s packed by gemm_q_pack."""
    n = len(y)
    P = ctypes.c_void_p * n
    I = ctypes.c_int * n
    return call("aljabr_blackwell_gemm_q_dev", type_id, n, P(*y), I(*ldy), P(*packed), I(*rows), ctypes.c_void_p(x),
                M, K, ctypes.c_void_p(workspace), workspace_bytes, None if stream is None else ctypes.c_void_p(stream))
