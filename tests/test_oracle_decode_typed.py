"""CPU: the oracle's typed decode step is the NF4 step when every tensor is
NF4 (bit-identical), and its GGUF routes use the pinned row dots."""
import numpy as np

import oracle


def _cfg():
    return oracle.LlamaCfg(1, 256, 4, 2, 64, 512, 64, 4, 64, 1e-5, 10000.0)


def test_typed_step_with_nf4_types_is_the_nf4_step():
    cfg = _cfg()
    g = np.random.default_rng(3)
    shapes = [(256, 256), (128, 256), (128, 256), (256, 256), (512, 256), (512, 256), (256, 512), (64, 256), (64, 256)]
    codes, absmax = [], []
    for i, (r, c) in enumerate(shapes):
        cd, am = oracle.quantize_nf4(g.normal(0, 1.0 if i == 7 else 0.02, size=(r, c)).astype(np.float32), 64)
        codes.append(cd)
        absmax.append(am)
    norms = (1.0 + 0.1 * g.normal(size=3 * 256)).astype(np.float32)
    k1 = np.zeros((1, 4, 128), np.float32)
    v1 = np.zeros_like(k1)
    k2, v2 = k1.copy(), v1.copy()
    for pos, tok in enumerate([3, 60, 0]):
        x1, l1 = oracle.decode_step_nf4(cfg, codes, absmax, norms, k1, v1, tok, pos)
        x2, l2 = oracle.decode_step_typed(cfg, codes, [oracle.NF4] * 9, absmax, norms, k2, v2, tok, pos)
        np.testing.assert_array_equal(x1.view(np.uint32), x2.view(np.uint32))
        np.testing.assert_array_equal(l1.view(np.uint32), l2.view(np.uint32))
    np.testing.assert_array_equal(k1, k2)


def test_typed_step_logits_use_the_row_dots():
    """With one layer whose projections are Q8_0, the lm_head (Q4_0) logits
    are orc_dot_row_q4_0 of the output-normed residual stream."""
    cfg = _cfg()
    g = np.random.default_rng(4)
    shapes = [(256, 256), (128, 256), (128, 256), (256, 256), (512, 256), (512, 256), (256, 512), (64, 256), (64, 256)]
    types = [oracle.Q8_0] * 7 + [oracle.Q8_0, oracle.Q4_0]
    weights = []
    for i, (r, c) in enumerate(shapes):
        vals = g.normal(0, 1.0 if i == 7 else 0.02, size=(r, c)).astype(np.float32)
        weights.append(oracle.encode_q4_0(vals) if types[i] == oracle.Q4_0 else oracle.encode_q8_0(vals))
    norms = (1.0 + 0.1 * g.normal(size=3 * 256)).astype(np.float32)
    kc = np.zeros((1, 4, 128), np.float32)
    vc = np.zeros_like(kc)
    x, logits = oracle.decode_step_typed(cfg, weights, types, [None] * 9, norms, kc, vc, 5, 0)
    xn = np.empty(256, np.float32)
    out_norm = np.ascontiguousarray(norms[512:])
    oracle.lib().orc_rms_norm(oracle._ptr(x), oracle._ptr(out_norm), oracle._ptr(xn), 256, np.float32(1e-5))
    head = weights[8].reshape(64, -1)
    ref = np.array([oracle.dot_row_q4_0(head[r], xn) for r in range(64)], np.float32)
    np.testing.assert_array_equal(logits.view(np.uint32), ref.view(np.uint32))


def test_row_dequantiser_known_answers(golden):
    """orc_dequantize_row_ref (the typed step's embedding lookup) reproduces the
    reference's GgufQ4KTest / GgufQ6KTest dequantised rows exactly."""
    seen = set()
    for fx in golden.values():
        if fx["kind"] != "k_dequant":
            continue
        seen.add(fx["type"])
        got = oracle.dequantize_row_ref(fx["type"], np.array(fx["weights"], np.uint8), fx["K"])
        np.testing.assert_array_equal(got, np.array(fx["expected"], np.float32), err_msg=fx["name"])
    assert seen == {oracle.Q4_K, oracle.Q6_K}


def test_row_dequantiser_matches_element_formulas():
    """Random K-quant rows: the float-order dequantiser is within float
    rounding of the fp64 element formulas; Q4_0 / Q8_0 are the block
    dequantisers themselves."""
    from tests import synth
    for kind in (oracle.Q4_K, oracle.Q6_K):
        row = synth.k_quant(kind, 17 + kind, 1, 1024)
        got = oracle.dequantize_row_ref(kind, row, 1024).astype(np.float64)
        ref = oracle.dequantize_k_row(kind, row, 1024)
        assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-6)) < 1e-6
    vals = np.random.default_rng(2).normal(0, 1, 256).astype(np.float32)
    w4, w8 = oracle.encode_q4_0(vals), oracle.encode_q8_0(vals)
    np.testing.assert_array_equal(oracle.dequantize_row_ref(oracle.Q4_0, w4, 256), oracle.dequantize_q4_0(w4, 256))
    np.testing.assert_array_equal(oracle.dequantize_row_ref(oracle.Q8_0, w8, 256), oracle.dequantize_q8_0(w8, 256))
