"""The oracle checked against the reference's own known-answer tests
(restated in tests/golden/known_answers.json by make_golden.py)."""
import math

import numpy as np
import pytest

import oracle


def _fixtures(golden, kind):
    return [fx for fx in golden.values() if fx["kind"] == kind]


def test_fixture_set_present(golden):
    kinds = {fx["kind"] for fx in golden.values()}
    assert {"q4_0_matvec", "q4_0_dequant", "q8_0_matvec", "f16", "attention", "nf4_dequant"} <= kinds


def test_q4_0_matvec_known_answers(golden):
    for fx in _fixtures(golden, "q4_0_matvec"):
        w = np.array(fx["weights"], dtype=np.uint8)
        x = np.array(fx["x"], dtype=np.float32)
        y = oracle.matvec_q4_0(w, x, fx["N"])
        np.testing.assert_allclose(y, fx["expected"], rtol=0, atol=fx["tol"] * max(1.0, np.abs(fx["expected"]).max()),
                                   err_msg=fx["name"])
        for threads in (2, 3):
            np.testing.assert_array_equal(oracle.matvec_q4_0(w, x, fx["N"], threads=threads), y)


def test_q4_0_prepared_order_known_answers(golden):
    # The prepared-cache order (GgufQ32Dot.dotRowQ32PreparedNoBiasScalar) is
    # the reference's default for >= 32 rows; the same known answers hold
    # (GgufQ32Test.java:18-42 asserts 16 / 48 through matVecRows, whichever
    # order the cache policy picks).
    for fx in _fixtures(golden, "q4_0_matvec"):
        w = np.array(fx["weights"], dtype=np.uint8)
        x = np.array(fx["x"], dtype=np.float32)
        y = oracle.matvec_q4_0_prepared(w, x, fx["N"])
        np.testing.assert_allclose(y, fx["expected"], rtol=0, atol=fx["tol"] * max(1.0, np.abs(fx["expected"]).max()),
                                   err_msg=fx["name"])
        for threads in (2, 3):
            np.testing.assert_array_equal(oracle.matvec_q4_0_prepared(w, x, fx["N"], threads=threads), y)


def test_q4_0_prepared_and_raw_orders_agree_with_fp64():
    rng = np.random.default_rng(13)
    for K, N in ((4096, 64), (14336, 32), (4128, 40)):   # 4128: 129 blocks, exercises the fma tail
        w = oracle.encode_q4_0(rng.normal(0, 0.02, size=K * N).astype(np.float32))
        x = rng.normal(0, 1, size=K).astype(np.float32)
        raw = oracle.matvec_q4_0(w, x, N)
        prep = oracle.matvec_q4_0_prepared(w, x, N)
        g = oracle.matvec_f64(oracle.Q4_0, w, x, N)
        scale = np.abs(g).max()
        assert np.max(np.abs(raw - g)) / scale < 1e-5
        assert np.max(np.abs(prep - g)) / scale < 1e-5
        # the orders differ (fma vs separate rounding), so they are close but not equal
        assert np.max(np.abs(prep - raw)) / scale < 1e-5
        row = w[:(K // 32) * 18]
        assert oracle.dot_row_q4_0_prepared(row, x) == prep[0]


def test_binding_glue_restatement():
    rng = np.random.default_rng(14)
    x = rng.normal(0, 1, size=4096).astype(np.float32)
    w = rng.normal(1, 0.1, size=4096).astype(np.float32)
    out = oracle.rmsnorm_binding(x, w, 1e-6)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt(np.mean(x64 * x64) + 1e-6) * w
    assert np.max(np.abs(out - ref)) < 1e-5
    g = rng.normal(0, 2, size=1000).astype(np.float32)
    u = rng.normal(0, 1, size=1000).astype(np.float32)
    s = oracle.silu_ffn_binding(g, u)
    g64 = g.astype(np.float64)
    np.testing.assert_allclose(s, g64 / (1 + np.exp(-g64)) * u, rtol=1e-6, atol=1e-7)


def test_q4_0_dequant_known_answers(golden):
    for fx in _fixtures(golden, "q4_0_dequant"):
        y = oracle.dequantize_q4_0(np.array(fx["weights"], dtype=np.uint8), fx["numel"])
        np.testing.assert_array_equal(y, np.array(fx["expected"], dtype=np.float32), err_msg=fx["name"])


def test_q8_0_matvec_known_answers(golden):
    for fx in _fixtures(golden, "q8_0_matvec"):
        w = np.array(fx["weights"], dtype=np.uint8)
        x = np.array(fx["x"], dtype=np.float32)
        for vector_order in (True, False):
            y = oracle.matvec_q8_0(w, x, fx["N"], vector_order=vector_order)
            np.testing.assert_allclose(y, fx["expected"], rtol=fx["tol"], atol=fx["tol"], err_msg=fx["name"])


def test_f16_special_values(golden):
    fx = golden["f16_special_values"]
    for bits, exp in zip(fx["bits"], fx["expected_bits"]):
        v = np.float32(oracle.f16_to_f32(bits))
        if exp == "nan":
            assert math.isnan(v)
            assert int(v.view(np.uint32)) == 0x7FC00000          # Float.NaN, canonical
        else:
            assert int(v.view(np.uint32)) == exp


def test_f16_table_matches_ieee_for_finite_values():
    bits = np.arange(65536, dtype=np.uint16)
    table = oracle.f16_to_f32_array(bits)
    ieee = bits.view(np.float16).astype(np.float32)
    finite = np.isfinite(ieee)
    np.testing.assert_array_equal(table[finite].view(np.uint32), ieee[finite].view(np.uint32))
    assert np.all(np.isnan(table[np.isnan(ieee)]))


def test_attention_known_answers(golden):
    for fx in _fixtures(golden, "attention"):
        out = oracle.gqa_decode_attention(np.array(fx["q"]), np.array(fx["k"]), np.array(fx["v"]),
                                          fx["stride"], fx["kv_heads"], fx["q_heads"], fx["head_dim"],
                                          fx["seq_len"], fx["start"], fx["scale"])
        np.testing.assert_allclose(out, fx["expected"], atol=fx["tol"], rtol=0, err_msg=fx["name"])


def test_nf4_table_and_nibble_order(golden):
    fx = golden["nf4_table_high_nibble_first"]
    y = oracle.dequantize_nf4(np.array(fx["codes"], np.uint8), np.array(fx["absmax"], np.float32),
                              fx["numel"], fx["group"])
    np.testing.assert_array_equal(y, np.array(fx["expected"], dtype=np.float32))


def test_q4_0_encoder_round_trip():
    rng = np.random.default_rng(7)
    w = rng.normal(0, 0.02, size=32 * 64).astype(np.float32)
    blocks = oracle.encode_q4_0(w)
    deq = oracle.dequantize_q4_0(blocks, w.size)
    # half a quantisation step, plus |code| times the fp16 rounding of the scale
    scale = np.abs(w.reshape(-1, 32)).max(axis=1) / 7.0
    err = np.abs(deq - w).reshape(-1, 32).max(axis=1)
    assert np.all(err <= scale * (0.5 + 8 * 2.0 ** -11) + 1e-7)
    codes = blocks.reshape(-1, 18)[:, 2:]
    assert codes.min() >= 0x00 and (codes & 0x0F).max() <= 15


def test_q8_0_encoder_round_trip():
    rng = np.random.default_rng(8)
    w = rng.normal(0, 0.02, size=32 * 64).astype(np.float32)
    blocks = oracle.encode_q8_0(w)
    deq = oracle.dequantize_q8_0(blocks, w.size)
    scale = np.abs(w.reshape(-1, 32)).max(axis=1) / 127.0
    err = np.abs(deq - w).reshape(-1, 32).max(axis=1)
    assert np.all(err <= scale * (0.5 + 127 * 2.0 ** -11) + 1e-7)


def test_f32_to_f16_encoder_matches_numpy_for_normals():
    rng = np.random.default_rng(9)
    v = rng.uniform(1e-3, 100, size=2000).astype(np.float32)
    ours = np.array([oracle.f32_to_f16_bits(float(a)) for a in v], dtype=np.uint16)
    ref = v.astype(np.float16).view(np.uint16)
    # GGUFWriter rounds half up rather than to even: allow 1-ulp differences only at ties
    assert np.max(np.abs(ours.astype(np.int32) - ref.astype(np.int32))) <= 1


def test_java_round_semantics():
    assert oracle.java_round(2.5) == 3
    assert oracle.java_round(-2.5) == -2
    assert oracle.java_round(0.49999997) == 0
    assert oracle.java_round(float("nan")) == 0


def test_nf4_quantizer_round_trip():
    rng = np.random.default_rng(10)
    w = rng.normal(0, 0.02, size=64 * 32).astype(np.float32)
    codes, absmax = oracle.quantize_nf4(w, 64)
    deq = oracle.dequantize_nf4(codes, absmax, w.size, 64)
    rel = np.linalg.norm(deq - w) / np.linalg.norm(w)
    assert rel < 0.12


def test_q8_vector_and_scalar_orders_agree():
    rng = np.random.default_rng(11)
    K, N = 4096, 64
    w = oracle.encode_q8_0(rng.normal(0, 0.02, size=K * N).astype(np.float32))
    x = rng.normal(0, 1, size=K).astype(np.float32)
    a = oracle.matvec_q8_0(w, x, N, vector_order=True)
    b = oracle.matvec_q8_0(w, x, N, vector_order=False)
    g = oracle.matvec_f64(oracle.Q8_0, w, x, N)
    scale = np.abs(g).max()
    assert np.max(np.abs(a - g)) / scale < 1e-5
    assert np.max(np.abs(b - g)) / scale < 1e-5


def test_rope_rotation_preserves_pair_norm():
    rng = np.random.default_rng(12)
    x = rng.normal(size=4 * 128).astype(np.float32)
    y = oracle.rope(x, 4, 128, 77, 500000.0)
    xr = x.reshape(4, 2, 64)
    yr = y.reshape(4, 2, 64)
    np.testing.assert_allclose(np.hypot(xr[:, 0], xr[:, 1]), np.hypot(yr[:, 0], yr[:, 1]), rtol=1e-5)
    np.testing.assert_array_equal(oracle.rope(x, 4, 128, 0, 500000.0), x)


def test_k_quant_matvec_known_answers(golden):
    """Q4_K / Q6_K row dots (GgufQ4RawDot.dotRowQ4K, GgufQ6RawDot.dotRowQ6K
    restated) against the values the reference's raw K-quant tests assert."""
    fxs = _fixtures(golden, "k_matvec")
    assert {fx["type"] for fx in fxs} == {oracle.Q4_K, oracle.Q6_K}
    for fx in fxs:
        w = np.array(fx["weights"], dtype=np.uint8)
        x = np.array(fx["x"], dtype=np.float32)
        y = oracle.matvec_k(fx["type"], w, x, fx["N"])
        np.testing.assert_array_equal(y, np.array(fx["expected"], dtype=np.float32), err_msg=fx["name"])
        # the fp64 element formulas give the same value on these exact cases
        y64 = oracle.matvec_f64(fx["type"], w, x, fx["N"])
        np.testing.assert_allclose(y64, fx["expected"], rtol=0, atol=0, err_msg=fx["name"])


def test_k_quant_dot_matches_fp64_on_random_rows():
    """The float-order restatement stays within float rounding of the fp64
    element sums on random super-blocks (every byte pattern is a valid block)."""
    from tests import synth
    for kind in (oracle.Q4_K, oracle.Q6_K):
        w = synth.k_quant(kind, 11 + kind, 4, 2048)
        x = np.random.default_rng(kind).normal(0, 1, 2048).astype(np.float32)
        y = oracle.matvec_k(kind, w, x, 4, threads=2)
        y64 = oracle.matvec_f64(kind, w, x, 4)
        assert synth.normwise_rel_err(y, y64) < 1e-6
