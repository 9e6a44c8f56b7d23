"""Host-side provider logic (no GPU): operation support answers and the
GGUF model buffer packing used by the bridge."""
import numpy as np

from aljabr_b200 import provider
from aljabr_b200.bridge import GgufModel


def test_operation_support_native_only_for_implemented_kernels():
    assert provider.operation_support("matvec", {"type": "q4_0"}).support == "NATIVE"
    assert provider.operation_support("matvec", {"type": "nf4"}).support == "NATIVE"
    assert provider.operation_support("matvec", {"type": "q4_k"}).support == "NATIVE"
    assert provider.operation_support("matvec", {"type": "q6_k"}).support == "NATIVE"
    assert provider.operation_support("matvec", {"type": "q5_k"}).support == "UNSUPPORTED"
    assert provider.operation_support("attention.gqa.decode", {"dtype": "bf16"}).support == "NATIVE"
    assert provider.operation_support("softmax", {}).support == "UNSUPPORTED"


def test_bridge_routes_the_types_the_metal_seam_routes():
    # GgufMetalBridge.matVec routes Q4_K (12), Q6_K (14) and Q8_0 (8)
    from aljabr_b200.bridge import GgufBlackwellBridge
    for t in (2, 8, 12, 14):
        assert GgufBlackwellBridge.is_type_supported(t)
    for t in (0, 1, 3, 13, 30):
        assert not GgufBlackwellBridge.is_type_supported(t)


def test_operation_support_requires_constraints():
    import pytest
    with pytest.raises(TypeError):
        provider.operation_support("matvec", None)


def test_gguf_model_pack_aligns_tensors_to_32_bytes():
    a = np.arange(18 * 3, dtype=np.uint8)
    b = np.arange(34 * 2, dtype=np.uint8)
    m = GgufModel.pack([("a", 2, 32, 3, a), ("b", 8, 32, 2, b)])
    ta, tb = m.tensors["a"], m.tensors["b"]
    assert ta.offset % 32 == 0 and tb.offset % 32 == 0
    assert (ta.columns, ta.rows) == (32, 3)
    np.testing.assert_array_equal(m.data[tb.offset:tb.offset + b.size], b)
