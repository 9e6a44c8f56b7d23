"""The prefill-attention oracles (restatements of GgufPrefillAttentionExecution
.java:44-82 and MetalFlashAttentionCpuFallback.java:46-104) checked against
the decode-attention oracle, which the reference's own known answers pin
(tests/golden/known_answers.json, GgufDecodeAttentionExecutionTest): token t
of a causal prefill is decode attention over positions [0, t] (or, with a
sliding window W, [t - W + 1, t]), and the FlashAttention-4 contract at S = T
is the Java loop.  The two dot orders differ (sequential vs 8-lane), so rows
agree to rounding, not bit for bit."""
import numpy as np

import oracle
from tests import synth


def _data(T, Hq, Hkv, D, seed):
    r = synth.rng(seed)
    q = r.normal(size=(T, Hq * D)).astype(np.float32)
    k = r.normal(size=(T, Hkv * D)).astype(np.float32)
    v = r.normal(size=(T, Hkv * D)).astype(np.float32)
    return q, k, v


def test_prefill_rows_are_decode_attention():
    T, Hq, Hkv, D, scale = 23, 8, 2, 32, 0.2
    q, k, v = _data(T, Hq, Hkv, D, 1)
    out = oracle.prefill_attention(q, k, v, T, Hq, Hkv, D, scale)
    for t in (0, 1, 11, T - 1):
        dec = oracle.gqa_decode_attention(q[t], k, v, Hkv * D, Hkv, Hq, D, t + 1, 0, scale)
        np.testing.assert_allclose(out[t], dec, rtol=1e-5, atol=1e-6)


def test_prefill_window_rows_are_decode_windows():
    T, Hq, Hkv, D, scale, W = 30, 4, 4, 16, 0.3, 7
    q, k, v = _data(T, Hq, Hkv, D, 2)
    out = oracle.prefill_attention(q, k, v, T, Hq, Hkv, D, scale, window=W)
    for t in (0, 5, 6, 29):
        dec = oracle.gqa_decode_attention(q[t], k, v, Hkv * D, Hkv, Hq, D, t + 1, max(0, t - W + 1), scale)
        np.testing.assert_allclose(out[t], dec, rtol=1e-5, atol=1e-6)


def test_fa4_contract_is_the_java_loop_at_s_eq_t():
    T, Hq, Hkv, D, scale = 17, 6, 3, 32, 0.25
    q, k, v = _data(T, Hq, Hkv, D, 3)
    java = oracle.prefill_attention(q, k, v, T, Hq, Hkv, D, scale)
    fa4 = oracle.fa4_attention(q, k, v, 1, T, T, Hq, Hkv, D, scale, causal=True)
    np.testing.assert_allclose(fa4.reshape(T, -1), java, rtol=1e-5, atol=1e-6)


def test_fa4_causal_offset_and_soft_cap():
    """S > T: query t sees keys [0, S - T + t]; a soft cap bounds every logit."""
    B, T, S, H, Hkv, D = 1, 3, 8, 2, 1, 16
    r = synth.rng(4)
    q = r.normal(size=(B, T, H, D)).astype(np.float32) * 4
    k = r.normal(size=(B, S, Hkv, D)).astype(np.float32)
    v = r.normal(size=(B, S, Hkv, D)).astype(np.float32)
    out = oracle.fa4_attention(q, k, v, B, T, S, H, Hkv, D, 1.0, causal=True).reshape(T, H, D)
    for t in range(T):
        dec = oracle.gqa_decode_attention(q[0, t].ravel(), k[0].reshape(S, -1), v[0].reshape(S, -1), Hkv * D, Hkv, H,
                                          D, S - T + t + 1, 0, 1.0)
        np.testing.assert_allclose(out[t].ravel(), dec, rtol=1e-5, atol=1e-6)
    capped = oracle.fa4_attention(q, k, v, B, T, S, H, Hkv, D, 1.0, causal=False, soft_cap=2.0)
    assert np.all(np.isfinite(capped))
