"""Host-side mirror of the reference's GGUF dispatch seam and NF4 linear, on
top of the C-ABI.

Reference interfaces mirrored (paths relative to the reference project):
  * GgufMetalBridge.matVec / matVecPair / matVecTriple / matVecBatch and
    ensureModelRegistered -- engine/gguf/aljabr-gguf-java/.../javabackend/
    GgufMetalBridge.java:590-602,701-759; here `GgufBlackwellBridge`.
  * GgufExecutionDispatcher.dispatchMatVec* -- GgufExecutionDispatcher.java:24-72;
    here `GgufExecutionDispatcher`, minus the CPU fallback: an unsupported
    type or shape raises UnsupportedOperation instead.
  * GgufDecodeAttentionExecution.execute -- GgufDecodeAttentionExecution.java:70-106.
  * AccelOps.linear for NF4 weights (M == 1) and DequantizationKernel.dequantizeNf4
    -- engine/safetensor/aljabr-safetensor-core/.../tensor/AccelOps.java:392-470,
    DequantizationKernel.java:84-102.

A "model" here is the bytes of a GGUF file held in host memory (numpy uint8,
standing for the reference's mmap'd MemorySegment); tensors are offsets into
it.  Registration copies the whole buffer to HBM once, as
aljabr_metal_register_model_buffer does for the Metal provider.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import native
from .native import TYPE_NF4, TYPE_Q4_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, UnsupportedOperation

BLOCK_BYTES = {TYPE_Q4_0: 18, TYPE_Q8_0: 34}
# Types whose matvec the bridge routes, as GgufMetalBridge.matVec routes Q4_K,
# Q6_K and Q8_0 (GgufMetalBridge.java:701-716) -- plus Q4_0, which this
# provider serves natively where the Metal bridge leaves it to the CPU.
MATVEC_ENTRY = {
    TYPE_Q4_0: "aljabr_blackwell_matvec_tb_q4_0",
    TYPE_Q8_0: "aljabr_blackwell_matvec_tb_q8_0",
    TYPE_Q4_K: "aljabr_blackwell_matvec_tb_q4_k",
    TYPE_Q6_K: "aljabr_blackwell_matvec_tb_q6_k",
}


@dataclass(frozen=True)
class GgufTensor:
    """GGUFTensorInfo: name, ggml shape [columns, rows], type id, byte offset."""
    name: str
    shape: tuple
    type_id: int
    offset: int

    @property
    def columns(self) -> int:
        return int(self.shape[0])

    @property
    def rows(self) -> int:
        return int(self.shape[1]) if len(self.shape) > 1 else 1


class GgufModel:
    """GGUFModel: a host byte buffer (the mmap) plus its tensors."""

    def __init__(self, data: np.ndarray, tensors: list | None = None):
        assert data.dtype == np.uint8 and data.flags.c_contiguous
        self.data = data
        self.tensors = {t.name: t for t in (tensors or [])}

    def address(self, tensor: GgufTensor) -> int:
        return self.data.ctypes.data + tensor.offset

    @staticmethod
    def pack(named_blocks: list) -> "GgufModel":
        """Build a model buffer from (name, type_id, columns, rows, bytes) entries,
        each tensor 32-byte aligned as GGUF files align tensor data."""
        size = 0
        layout = []
        for name, type_id, cols, rows, blob in named_blocks:
            size = (size + 31) // 32 * 32
            layout.append((name, type_id, cols, rows, size, blob))
            size += len(blob)
        data = np.zeros(max(size, 32), dtype=np.uint8)
        tensors = []
        for name, type_id, cols, rows, off, blob in layout:
            data[off:off + len(blob)] = np.frombuffer(np.ascontiguousarray(blob).tobytes(), dtype=np.uint8)
            tensors.append(GgufTensor(name, (cols, rows), type_id, off))
        return GgufModel(data, tensors)


def _fptr(a: np.ndarray) -> int:
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data


class GgufBlackwellBridge:
    """Boolean-returning bridge with the shapes of GgufMetalBridge's matVec*."""

    _registered: dict = {}

    @classmethod
    def ensure_model_registered(cls, model: GgufModel) -> None:
        key = model.data.ctypes.data
        if cls._registered.get(key) is not model:
            native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(key), model.data.nbytes)
            cls._registered[key] = model

    @classmethod
    def release_model(cls, model: GgufModel) -> None:
        key = model.data.ctypes.data
        if cls._registered.pop(key, None) is not None:
            native.call("aljabr_blackwell_unregister_model_buffer", ctypes.c_void_p(key))

    @staticmethod
    def is_type_supported(type_id: int) -> bool:
        """GgufMetalBridge.isTypeSupported (GgufMetalBridge.java:604-606) for the
        types this provider has kernels for."""
        return type_id in MATVEC_ENTRY

    @classmethod
    def mat_vec(cls, model: GgufModel, tensor: GgufTensor, vector: np.ndarray, output: np.ndarray) -> bool:
        cls.ensure_model_registered(model)
        K, N = tensor.columns, tensor.rows
        if vector.size < K or output.size < N:
            raise ValueError("vector/output shorter than the tensor's columns/rows")
        fn = MATVEC_ENTRY.get(tensor.type_id)
        if fn is None:
            raise UnsupportedOperation(native.ALJ_ERR_UNSUPPORTED, f"GGUF type {tensor.type_id} ({tensor.name})")
        native.call(fn, _fptr(output), _fptr(vector), ctypes.c_void_p(model.address(tensor)), K, N)
        return True

    @classmethod
    def mat_vec_pair(cls, model, t0, out0, t1, out1, vector) -> bool:
        cls.ensure_model_registered(model)
        if t0.columns != t1.columns:
            raise ValueError("pair tensors must share their column count")
        native.call("aljabr_blackwell_matvec_tb_pair", _fptr(out0), _fptr(out1), _fptr(vector),
                    ctypes.c_void_p(model.address(t0)), ctypes.c_void_p(model.address(t1)),
                    t0.columns, t0.rows, t1.rows, t0.type_id, t1.type_id)
        return True

    @classmethod
    def mat_vec_triple(cls, model, t0, out0, t1, out1, t2, out2, vector) -> bool:
        cls.ensure_model_registered(model)
        if not (t0.columns == t1.columns == t2.columns):
            raise ValueError("triple tensors must share their column count")
        native.call("aljabr_blackwell_matvec_tb_triple", _fptr(out0), _fptr(out1), _fptr(out2), _fptr(vector),
                    ctypes.c_void_p(model.address(t0)), ctypes.c_void_p(model.address(t1)),
                    ctypes.c_void_p(model.address(t2)), t0.columns, t0.rows, t1.rows, t2.rows,
                    t0.type_id, t1.type_id, t2.type_id)
        return True

    @classmethod
    def mat_vec_batch(cls, model, tensor, input_batch, output_batch, batch_size) -> bool:
        cls.ensure_model_registered(model)
        native.call("aljabr_blackwell_matvec_tb_batch", _fptr(output_batch), _fptr(input_batch),
                    ctypes.c_void_p(model.address(tensor)), tensor.columns, tensor.rows, tensor.type_id, batch_size)
        return True


class GgufExecutionDispatcher:
    """GgufExecutionDispatcher with the Blackwell bridge as its only provider."""

    def __init__(self, model: GgufModel):
        self.model = model
        self.count_gpu = 0

    def dispatch_mat_vec(self, tensor, input_vec, output):
        GgufBlackwellBridge.mat_vec(self.model, tensor, input_vec, output)
        self.count_gpu += 1

    def dispatch_mat_vec_pair(self, t0, out0, t1, out1, input_vec):
        GgufBlackwellBridge.mat_vec_pair(self.model, t0, out0, t1, out1, input_vec)
        self.count_gpu += 2

    def dispatch_mat_vec_triple(self, t0, out0, t1, out1, t2, out2, input_vec):
        GgufBlackwellBridge.mat_vec_triple(self.model, t0, out0, t1, out1, t2, out2, input_vec)
        self.count_gpu += 3

    def dispatch_mat_vec_batch(self, tensor, input_batch, output_batch, batch_size):
        GgufBlackwellBridge.mat_vec_batch(self.model, tensor, input_batch, output_batch, batch_size)
        self.count_gpu += batch_size


def dequantize_row_block(type_id: int, blob: np.ndarray, numel: int) -> np.ndarray:
    """GgufBlockDequantizer over device-resident or host bytes (host bytes are
    registered for the duration of the call)."""
    out = np.empty(numel, dtype=np.float32)
    fn = {TYPE_Q4_0: "aljabr_blackwell_dequantize_q4_0", TYPE_Q8_0: "aljabr_blackwell_dequantize_q8_0"}[type_id]
    with _registered(blob):
        native.call(fn, _fptr(out), ctypes.c_void_p(blob.ctypes.data), numel)
    return out


def dequantize_nf4(src: np.ndarray, scales: np.ndarray, numel: int, group_size: int) -> np.ndarray:
    """DequantizationKernel.dequantizeNf4(src, dst, scales, numel, groupSize)."""
    out = np.empty(numel, dtype=np.float32)
    with _registered(src), _registered(scales):
        native.call("aljabr_blackwell_dequantize_nf4", _fptr(out), ctypes.c_void_p(src.ctypes.data),
                    ctypes.c_void_p(scales.ctypes.data), numel, group_size)
    return out


class AccelNf4Linear:
    """AccelOps.linear(input, weight, bias) for an NF4 weight and M == 1:
    y = dequant(W) x + bias, computed without materialising dequant(W)."""

    def __init__(self, codes: np.ndarray, absmax: np.ndarray, out_features: int, in_features: int,
                 group_size: int = 64, bias: np.ndarray | None = None):
        self.codes = np.ascontiguousarray(codes, dtype=np.uint8)
        self.absmax = np.ascontiguousarray(absmax, dtype=np.float32)
        self.N, self.K, self.group = out_features, in_features, group_size
        self.bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(self.codes.ctypes.data), self.codes.nbytes)
        native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(self.absmax.ctypes.data), self.absmax.nbytes)

    def __call__(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(self.N, dtype=np.float32)
        native.call("aljabr_blackwell_linear_nf4", _fptr(y), _fptr(x), ctypes.c_void_p(self.codes.ctypes.data),
                    ctypes.c_void_p(self.absmax.ctypes.data),
                    None if self.bias is None else ctypes.c_void_p(self.bias.ctypes.data), self.K, self.N, self.group)
        return y

    def close(self):
        for a in (self.codes, self.absmax):
            native.lib().aljabr_blackwell_unregister_model_buffer(ctypes.c_void_p(a.ctypes.data))


def decode_attention(query: np.ndarray, key_cache_ptr: int, value_cache_ptr: int, kv_dtype: int,
                     cache_head_stride: int, kv_heads: int, query_heads: int, head_dim: int,
                     sequence_length: int, start_position: int, scale: float) -> np.ndarray:
    """GgufDecodeAttentionExecution.execute with the caches in device memory."""
    q = np.ascontiguousarray(query, dtype=np.float32)
    out = np.empty(query_heads * head_dim, dtype=np.float32)
    native.call("aljabr_blackwell_decode_attention", _fptr(out), _fptr(q), ctypes.c_void_p(key_cache_ptr),
                ctypes.c_void_p(value_cache_ptr), kv_dtype, cache_head_stride, kv_heads, query_heads, head_dim,
                sequence_length, start_position, ctypes.c_float(scale))
    return out


class _registered:
    """Register a host array as a model buffer for the duration of a block."""

    def __init__(self, a: np.ndarray):
        self.a = a

    def __enter__(self):
        native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(self.a.ctypes.data), self.a.nbytes)
        return self

    def __exit__(self, *exc):
        native.lib().aljabr_blackwell_unregister_model_buffer(ctypes.c_void_p(self.a.ctypes.data))
        return False
