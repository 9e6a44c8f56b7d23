"""The safetensors NF4 adapter's host logic (no GPU): header parsing, the
reference's quantization classification (AccelWeightBridge.java:164-222:
U8 `.qweight` + `.scales` -> NF4 with the last dimension doubled, I32 / U32
or I8 `.qweight` -> INT4, other scaled weights INT8, BF16 / F16 matrices
unquantized, group size 128), and views / addresses into the file map."""
import numpy as np

from aljabr_b200 import safetensors_nf4 as st
from tests import synth


def test_classification_follows_the_reference(tmp_path):
    p = str(tmp_path / "m.safetensors")
    r = synth.rng(0)
    synth.write_safetensors(p, {
        "a.qweight": r.integers(0, 256, size=(8, 64), dtype=np.uint8),
        "a.scales": np.ones(8 * 128 // 128, np.float32),
        "b.qweight": r.integers(0, 2 ** 31, size=(8, 16), dtype=np.int64).astype(np.int32),
        "b.scales": np.ones(8, np.float32),
        "b.qzeros": np.zeros(8, np.int32),
        "c.qweight": r.integers(-128, 128, size=(8, 32), dtype=np.int8),
        "c.scales": np.ones(8, np.float32),
        "d.weight": r.integers(0, 256, size=(8, 32), dtype=np.uint8),
        "d.scales": np.ones(8, np.float32),
        "e.weight": ("BF16", np.zeros((4, 4), np.uint16)),
        "f.weight": np.zeros((4, 4), np.float16),
        "g.weight": np.zeros((4, 4), np.float32),
    })
    sh = st.SafetensorShard(p)
    assert st.quant_type(sh, "a.qweight") == "NF4" and st.logical_shape(sh, "a.qweight") == (8, 128)
    assert st.quant_type(sh, "b.qweight") == "INT4" and st.logical_shape(sh, "b.qweight") == (8, 128)
    assert st.quant_type(sh, "c.qweight") == "INT4" and st.logical_shape(sh, "c.qweight") == (8, 64)
    assert st.quant_type(sh, "d.weight") == "INT8" and st.logical_shape(sh, "d.weight") == (8, 32)
    assert st.quant_type(sh, "e.weight") == "BF16"
    assert st.quant_type(sh, "f.weight") == "F16"
    assert st.quant_type(sh, "g.weight") is None
    assert st.is_metadata_tensor("b.qzeros") and st.is_metadata_tensor("a.scales")
    assert not st.is_weight_tensor("a.scales")
    w = st.nf4_weights(sh)
    assert list(w) == ["a"]
    a = w["a"]
    assert (a.rows, a.cols, a.group) == (8, 128, 128)


def test_views_and_addresses(tmp_path):
    p = str(tmp_path / "m.safetensors")
    r = synth.rng(1)
    codes = r.integers(0, 256, size=(16, 128), dtype=np.uint8)
    scales = r.random(16 * 256 // 128).astype(np.float32)
    synth.write_safetensors(p, {"x.qweight": codes, "x.scales": scales, "n.weight": np.arange(5, dtype=np.float32)})
    sh = st.SafetensorShard(p)
    np.testing.assert_array_equal(sh.array("x.qweight"), codes)
    np.testing.assert_array_equal(sh.array("x.scales"), scales)
    w = st.nf4_weights(sh)["x"]
    base = int(sh.map.ctypes.data)
    assert w.codes_addr == base + sh.tensors["x.qweight"].begin
    assert w.scales_addr == base + sh.tensors["x.scales"].begin
    got = np.ctypeslib.as_array((np.ctypeslib.ctypes.c_uint8 * codes.size).from_address(w.codes_addr))
    np.testing.assert_array_equal(got.reshape(codes.shape), codes)


def test_short_scales_are_rejected(tmp_path):
    p = str(tmp_path / "m.safetensors")
    synth.write_safetensors(p, {"x.qweight": np.zeros((4, 128), np.uint8), "x.scales": np.ones(3, np.float32)})
    sh = st.SafetensorShard(p)
    try:
        st.nf4_weights(sh)
    except ValueError as e:
        assert "scales" in str(e)
    else:
        raise AssertionError("expected a ValueError for too few scales")
