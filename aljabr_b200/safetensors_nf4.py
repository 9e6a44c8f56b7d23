"""Safetensors NF4 adapter: the on-disk format in front of the NF4 kernels.

Mirrors how the reference's safetensors bridge attaches quantization to a
weight (engine/safetensor/aljabr-safetensor-bridge/src/main/java/tech/kayys/
aljabr/safetensor/bridge/AccelWeightBridge.java:164-222,
`attachQuantizationMetadata`):
  * a tensor whose name ends in `.qweight` or `.weight` is a weight, and
    `<base>.scales` / `.qzeros` / `.g_idx` are its metadata (`:164-170`);
  * BF16 / F16 weights of rank >= 2 stay unquantized (`:176-182`);
  * with `<base>.scales` present, a U8 `.qweight` is NF4, an I32 / U32 (or an
    I8 `.qweight`) is INT4, anything else INT8 (`:184-197`);
  * NF4 and INT4 widen the last dimension of the logical shape (x2 for bytes,
    x8 for 32-bit words, `:199-209`), and the group size is 128 (`:215`).
The NF4 codes are two per byte with the high nibble first and the scales are
fp32, one per 128 consecutive elements of the flattened weight
(AccelTensor.java:1025, DequantizationKernel.dequantizeNf4) -- the layout the
library's NF4 matvec, linear and decode-step kernels take.

The file is read through one read-only memory map and registered with the
library once (`aljabr_blackwell_register_model_buffer`: copied to HBM in
chunks); every tensor is then addressed by its host address inside the map,
which the library resolves to the device copy, as the reference passes
MemorySegments of the mapped file.  Only NF4 weights run on the GPU here;
INT4 / INT8 weights are classified but not supported (their operations
return UNSUPPORTED)."""
from __future__ import annotations

import ctypes
import json
import struct
from dataclasses import dataclass

import numpy as np

from . import native

# safetensors dtype tags -> numpy dtypes (BF16 as its raw 16-bit pattern)
_NP = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I64": np.int64,
       "I32": np.int32, "I16": np.int16, "I8": np.int8, "U64": np.uint64, "U32": np.uint32, "U16": np.uint16,
       "U8": np.uint8, "BOOL": np.uint8}

NF4_GROUP = 128


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple
    begin: int          # byte offset from the start of the file
    end: int


class SafetensorShard:
    """One .safetensors file: 8-byte little-endian header length, the JSON
    header, then the tensor data; mapped read-only."""

    def __init__(self, path: str):
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
        data0 = 8 + n
        self.path = path
        self.metadata = header.pop("__metadata__", {})
        self.tensors = {}
        for name, e in header.items():
            b, en = e["data_offsets"]
            self.tensors[name] = TensorInfo(name, e["dtype"], tuple(e["shape"]), data0 + b, data0 + en)
        self.map = np.memmap(path, dtype=np.uint8, mode="r")
        self.registered = False

    def find(self, name: str) -> TensorInfo | None:
        return self.tensors.get(name)

    def array(self, name: str) -> np.ndarray:
        """The tensor as a numpy view into the map (BF16 as uint16 bits)."""
        t = self.tensors[name]
        dt = np.dtype(_NP[t.dtype])
        return self.map[t.begin:t.end].view(dt).reshape(t.shape)

    def address(self, name: str) -> int:
        """Host address of the tensor's first byte inside the map."""
        return int(self.map.ctypes.data) + self.tensors[name].begin

    # -- registration with the library ---------------------------------------
    def register(self) -> None:
        """Copy the whole file to HBM once; tensors are then addressed inside it."""
        if not self.registered:
            native.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(int(self.map.ctypes.data)),
                        int(self.map.nbytes))
            self.registered = True

    def unregister(self) -> None:
        if self.registered:
            native.call("aljabr_blackwell_unregister_model_buffer", ctypes.c_void_p(int(self.map.ctypes.data)))
            self.registered = False


def is_weight_tensor(name: str) -> bool:
    return name.endswith(".weight") or name.endswith(".qweight")


def is_metadata_tensor(name: str) -> bool:
    return name.endswith(".scales") or name.endswith(".qzeros") or name.endswith(".g_idx")


def quant_type(shard: SafetensorShard, weight_name: str) -> str | None:
    """The reference's classification of one weight tensor: "BF16", "F16",
    "NF4", "INT4", "INT8", or None (no scales: plain floats)."""
    t = shard.tensors[weight_name]
    if t.dtype == "BF16" and len(t.shape) >= 2:
        return "BF16"
    if t.dtype == "F16" and len(t.shape) >= 2:
        return "F16"
    base = weight_name[:weight_name.rindex(".")]
    if shard.find(base + ".scales") is None:
        return None
    if t.dtype in ("I32", "U32") or (t.dtype == "I8" and weight_name.endswith(".qweight")):
        return "INT4"
    if t.dtype == "U8" and weight_name.endswith(".qweight"):
        return "NF4"
    return "INT8"


def logical_shape(shard: SafetensorShard, weight_name: str) -> tuple:
    """Stored shape with the last dimension widened for packed 4-bit codes."""
    t = shard.tensors[weight_name]
    shape = list(t.shape)
    if quant_type(shard, weight_name) in ("NF4", "INT4"):
        if t.dtype in ("U8", "I8"):
            shape[-1] *= 2
        elif t.dtype in ("I32", "U32"):
            shape[-1] *= 8
    return tuple(shape)


@dataclass(frozen=True)
class Nf4Weight:
    """An NF4 linear weight [rows][cols] inside a shard."""
    name: str            # the `.qweight` tensor
    rows: int
    cols: int
    group: int
    codes_addr: int      # host addresses inside the map
    scales_addr: int


def nf4_weights(shard: SafetensorShard) -> dict:
    """Every weight the reference would classify as NF4, by base name."""
    out = {}
    for name in shard.tensors:
        if not is_weight_tensor(name) or quant_type(shard, name) != "NF4":
            continue
        shape = logical_shape(shard, name)
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        cols = int(shape[-1])
        base = name[:name.rindex(".")]
        scales = shard.tensors[base + ".scales"]
        numel = rows * cols
        if scales.dtype != "F32" or (scales.end - scales.begin) // 4 < (numel + NF4_GROUP - 1) // NF4_GROUP:
            raise ValueError(f"{base}.scales: expected fp32, one per {NF4_GROUP} elements of {name}")
        out[base] = Nf4Weight(name, rows, cols, NF4_GROUP, shard.address(name), shard.address(base + ".scales"))
    return out


class SafetensorNf4Linear:
    """AccelOps.linear (M == 1) for an NF4 weight of a registered shard."""

    def __init__(self, shard: SafetensorShard, weight: Nf4Weight, bias: np.ndarray | None = None):
        shard.register()
        self.shard, self.w = shard, weight
        self.bias = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)

    def __call__(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.size != self.w.cols:
            raise ValueError(f"input of {x.size} elements for a weight with {self.w.cols} columns")
        y = np.empty(self.w.rows, dtype=np.float32)
        native.call("aljabr_blackwell_linear_nf4", ctypes.c_void_p(y.ctypes.data), ctypes.c_void_p(x.ctypes.data),
                    ctypes.c_void_p(self.w.codes_addr), ctypes.c_void_p(self.w.scales_addr),
                    None if self.bias is None else ctypes.c_void_p(self.bias.ctypes.data), self.w.cols,
                    self.w.rows, self.w.group)
        return y


# Hugging Face Llama tensor names of one decoder layer, in the library's order.
LLAMA_LAYER = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def register_llama_decoder(decoder, shard: SafetensorShard, prefix: str = "model.") -> None:
    """Register a Llama-shaped NF4 checkpoint (Hugging Face tensor names,
    `.qweight` + `.scales` at group 128, fp32 or bf16 norm weights) with a
    LlamaNf4Decoder whose shape has group == 128."""
    if decoder.shape.group != NF4_GROUP:
        raise ValueError(f"the decoder's NF4 group is {decoder.shape.group}; safetensors NF4 uses {NF4_GROUP}")
    shard.register()
    w = nf4_weights(shard)

    def norm(name):
        a = shard.array(name)
        if shard.tensors[name].dtype == "BF16":
            return (a.astype(np.uint32) << 16).view(np.float32)
        return np.asarray(a, dtype=np.float32)

    for layer in range(decoder.shape.layers):
        base = f"{prefix}layers.{layer}."
        ws = [w[base + t] for t in LLAMA_LAYER]
        decoder.register_layer(layer, [x.codes_addr for x in ws], [x.scales_addr for x in ws],
                               norm(base + "input_layernorm.weight"), norm(base + "post_attention_layernorm.weight"))
    emb, head = w[prefix + "embed_tokens"], w["lm_head"]
    decoder.register_output(emb.codes_addr, emb.scales_addr, head.codes_addr, head.scales_addr,
                            norm(prefix + "norm.weight"))
