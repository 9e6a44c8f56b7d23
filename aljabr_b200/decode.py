"""Host wrapper of the device-resident decode step (aljabr_blackwell_decode_*).

Mirrors the reference's decode-step registration seam (the Metal bridge's
registerDecodeLayer / registerOutput / decodeStepToken,
engine/gguf/aljabr-gguf-java/.../javabackend/GgufMetalBridge.java:1879-2053)
for a Llama-shaped model whose linear weights are NF4 or, through
register_layer_typed / register_output_typed, GGUF Q4_0 / Q8_0 / Q4_K / Q6_K
with one type per tensor (registerDecodeLayer's typeQ .. typeDown).

Weights may be given as numpy arrays (registered as model buffers: copied to
HBM once, kept alive by this object) or as device addresses (ints, e.g.
torch tensors' data_ptr()), which the model references without copying.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import native

WEIGHT_ORDER = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass(frozen=True)
class LlamaShape:
    layers: int
    hidden: int
    q_heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    max_ctx: int
    group: int = 64
    kv_dtype: int = native.KV_BF16
    eps: float = 1e-5
    rope_theta: float = 500000.0

    def rows(self, name: str) -> int:
        """Rows of each full (unsharded) matrix, row-major [rows][cols]."""
        return {"q": self.q_heads * self.head_dim, "k": self.kv_heads * self.head_dim,
                "v": self.kv_heads * self.head_dim, "o": self.hidden, "gate": self.ffn, "up": self.ffn,
                "down": self.hidden, "embd": self.vocab, "head": self.vocab}[name]

    def cols(self, name: str) -> int:
        return {"o": self.q_heads * self.head_dim, "down": self.ffn}.get(name, self.hidden)


LLAMA3_8B = LlamaShape(layers=32, hidden=4096, q_heads=32, kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
                       max_ctx=4096)


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    native.call("aljabr_blackwell_nccl_unique_id", buf, 128)
    return buf.raw


class LlamaNf4Decoder:
    def __init__(self, shape: LlamaShape, tp_world: int = 1, tp_rank: int = 0, nccl_id: bytes | None = None):
        self.shape = shape
        self.tp_world, self.tp_rank = tp_world, tp_rank
        dims = (ctypes.c_int * 10)(shape.layers, shape.hidden, shape.q_heads, shape.kv_heads, shape.head_dim,
                                   shape.ffn, shape.vocab, shape.max_ctx, shape.group, shape.kv_dtype)
        h = ctypes.c_ulonglong(0)
        idbuf = None if nccl_id is None else ctypes.create_string_buffer(nccl_id, 128)
        native.call("aljabr_blackwell_decode_model_create", dims, ctypes.c_float(shape.eps),
                    ctypes.c_float(shape.rope_theta), tp_world, tp_rank, idbuf, ctypes.byref(h))
        self.handle = h.value
        self._keep = []          # host arrays registered as model buffers

    # -- weights ---------------------------------------------------------------
    def _addr(self, a) -> int:
        if isinstance(a, (int, np.integer)):
            return int(a)
        if hasattr(a, "data_ptr"):
            return int(a.data_ptr())
        a = np.ascontiguousarray(a)
        native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(a.ctypes.data), a.nbytes)
        self._keep.append(a)
        return a.ctypes.data

    def register_layer(self, layer: int, codes: list, absmax: list, attn_norm, ffn_norm):
        c = (ctypes.c_void_p * 7)(*[self._addr(x) for x in codes])
        a = (ctypes.c_void_p * 7)(*[self._addr(x) for x in absmax])
        an = np.ascontiguousarray(attn_norm, dtype=np.float32)
        fn = np.ascontiguousarray(ffn_norm, dtype=np.float32)
        native.call("aljabr_blackwell_register_decode_layer", ctypes.c_ulonglong(self.handle), layer, c, a,
                    an.ctypes.data, fn.ctypes.data)

    def register_output(self, embd_codes, embd_absmax, head_codes, head_absmax, output_norm):
        on = np.ascontiguousarray(output_norm, dtype=np.float32)
        native.call("aljabr_blackwell_register_output", ctypes.c_ulonglong(self.handle),
                    ctypes.c_void_p(self._addr(embd_codes)), ctypes.c_void_p(self._addr(embd_absmax)),
                    ctypes.c_void_p(self._addr(head_codes)), ctypes.c_void_p(self._addr(head_absmax)), on.ctypes.data)

    def register_layer_typed(self, layer: int, weights: list, types: list, attn_norm, ffn_norm, absmax=None):
        """One GGUF type per tensor (native.TYPE_Q4_0 / Q8_0 / Q4_K / Q6_K / NF4),
        as registerDecodeLayer's typeQ .. typeDown; absmax[i] only for NF4."""
        w = (ctypes.c_void_p * 7)(*[self._addr(x) for x in weights])
        t = (ctypes.c_int * 7)(*types)
        a = None if absmax is None else (ctypes.c_void_p * 7)(*[None if x is None else self._addr(x) for x in absmax])
        an = np.ascontiguousarray(attn_norm, dtype=np.float32)
        fn = np.ascontiguousarray(ffn_norm, dtype=np.float32)
        native.call("aljabr_blackwell_register_decode_layer_typed", ctypes.c_ulonglong(self.handle), layer, w, t, a,
                    an.ctypes.data, fn.ctypes.data)

    def register_output_typed(self, embd, embd_type: int, head, head_type: int, output_norm, embd_absmax=None,
                              head_absmax=None):
        on = np.ascontiguousarray(output_norm, dtype=np.float32)
        ptr = (lambda a: None if a is None else ctypes.c_void_p(self._addr(a)))
        native.call("aljabr_blackwell_register_output_typed", ctypes.c_ulonglong(self.handle),
                    ctypes.c_void_p(self._addr(embd)), embd_type, ptr(embd_absmax), ctypes.c_void_p(self._addr(head)),
                    head_type, ptr(head_absmax), on.ctypes.data)

    def sync_kv_cache(self, layer: int, seq_len: int, k, v):
        native.call("aljabr_blackwell_sync_kv_cache", ctypes.c_ulonglong(self.handle), layer, seq_len,
                    ctypes.c_void_p(self._ptr_any(k)), ctypes.c_void_p(self._ptr_any(v)))

    @staticmethod
    def _ptr_any(a) -> int:
        if isinstance(a, (int, np.integer)):
            return int(a)
        if hasattr(a, "data_ptr"):
            return int(a.data_ptr())
        return np.ascontiguousarray(a).ctypes.data

    # -- decoding --------------------------------------------------------------
    def step(self, token: int, pos: int, want_logits: bool = False):
        logits = np.empty(self.shape.vocab, np.float32) if want_logits else None
        nxt = ctypes.c_int(-1)
        native.call("aljabr_blackwell_decode_step_token", ctypes.c_ulonglong(self.handle), token, pos,
                    None if logits is None else logits.ctypes.data, ctypes.byref(nxt))
        return nxt.value, logits

    def run(self, token: int, pos: int, n_tokens: int) -> np.ndarray:
        """Greedy decode of n_tokens starting at `pos`, entirely on the device."""
        out = np.empty(n_tokens, np.int32)
        native.call("aljabr_blackwell_decode_run", ctypes.c_ulonglong(self.handle), token, pos, n_tokens,
                    out.ctypes.data)
        return out

    def read_state(self):
        s = self.shape
        kv_heads = s.kv_heads // self.tp_world
        dt = np.uint16 if s.kv_dtype == native.KV_BF16 else np.float32
        x = np.empty(s.hidden, np.float32)
        k = np.empty((s.layers, s.max_ctx, kv_heads * s.head_dim), dt)
        v = np.empty_like(k)
        native.call("aljabr_blackwell_decode_read_state", ctypes.c_ulonglong(self.handle), x.ctypes.data,
                    k.ctypes.data, v.ctypes.data)
        return x, k, v

    def close(self):
        if self.handle:
            native.call("aljabr_blackwell_decode_model_destroy", ctypes.c_ulonglong(self.handle))
            self.handle = 0
        for a in self._keep:
            native.lib().aljabr_blackwell_unregister_model_buffer(ctypes.c_void_p(a.ctypes.data))
        self._keep = []


def shard_rows(a: np.ndarray, rows: int, cols: int, world: int, rank: int, packed_per_row: int | None = None):
    """Row block `rank` of a row-major matrix stored flat (codes or absmax)."""
    per_row = a.size // rows if packed_per_row is None else packed_per_row
    r = rows // world
    return np.ascontiguousarray(a.reshape(rows, per_row)[rank * r:(rank + 1) * r]).ravel()
