"""GPU parity of the full decode step (NF4 Llama-shaped model, one CUDA graph
per token) against the oracle's restatement of GgufDecodePass's layer loop.

Per step we compare the residual stream after the last layer and the
logits.  With an fp32 KV cache the two implementations store identical
k/v, so the only differences are summation orders (tolerance 1e-3 max
relative error, as for the single kernels).  With a bf16 cache both sides
round k/v to bf16; a k/v value that lands within ~1e-7 of a bf16 rounding
boundary can round differently on the two sides (one bf16 ulp, 2^-8), so the
bf16 case is held to a normwise bound instead."""
import numpy as np
import pytest

import oracle
from tests import synth

pytestmark = pytest.mark.gpu


def _model(seed, shape):
    """Random NF4 weights in the oracle's tensor order + fp32 norms."""
    g = np.random.default_rng(seed)
    names = ["q", "k", "v", "o", "gate", "up", "down"]
    codes, absmax = [], []
    for _ in range(shape.layers):
        for n in names:
            c, a = oracle.quantize_nf4(g.normal(0, 0.02, size=(shape.rows(n), shape.cols(n))).astype(np.float32),
                                       shape.group)
            codes.append(c)
            absmax.append(a)
    for n in ("embd", "head"):
        std = 1.0 if n == "embd" else 0.02
        c, a = oracle.quantize_nf4(g.normal(0, std, size=(shape.rows(n), shape.cols(n))).astype(np.float32),
                                   shape.group)
        codes.append(c)
        absmax.append(a)
    norms = (1.0 + 0.1 * g.normal(size=(shape.layers * 2 + 1) * shape.hidden)).astype(np.float32)
    return codes, absmax, norms


def _build(shape, codes, absmax, norms):
    from aljabr_b200.decode import LlamaNf4Decoder
    dec = LlamaNf4Decoder(shape)
    H = shape.hidden
    for l in range(shape.layers):
        dec.register_layer(l, codes[7 * l:7 * l + 7], absmax[7 * l:7 * l + 7], norms[2 * l * H:(2 * l + 1) * H],
                           norms[(2 * l + 1) * H:(2 * l + 2) * H])
    dec.register_output(codes[7 * shape.layers], absmax[7 * shape.layers], codes[7 * shape.layers + 1],
                        absmax[7 * shape.layers + 1], norms[2 * shape.layers * H:])
    return dec


def _cfg(shape):
    return oracle.LlamaCfg(shape.layers, shape.hidden, shape.q_heads, shape.kv_heads, shape.head_dim, shape.ffn,
                           shape.vocab, shape.max_ctx, shape.group, shape.eps, shape.rope_theta)


# "small" runs the plain-kernel fallbacks (K below 2048); "wide" has every K a
# multiple of 2048, so the projections run the TMA table kernel with its fused
# epilogues (q/k/v segments, residual + RMSNorm, SwiGLU pair, lm_head).
SHAPES = {
    "small": dict(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1024, max_ctx=32),
    "wide": dict(layers=2, hidden=2048, q_heads=16, kv_heads=4, head_dim=128, ffn=4096, vocab=2048, max_ctx=16),
}


@pytest.mark.parametrize("kv_dtype", [0, 1])
@pytest.mark.parametrize("which", ["small", "wide"])
def test_decode_step_matches_oracle(kv_dtype, which):
    from aljabr_b200 import native
    from aljabr_b200.decode import LlamaShape
    native.call("aljabr_blackwell_init", 0)
    shape = LlamaShape(**SHAPES[which], kv_dtype=kv_dtype)
    codes, absmax, norms = _model(123, shape)
    dec = _build(shape, codes, absmax, norms)
    cdt = np.uint16 if kv_dtype else np.float32
    kc = np.zeros((shape.layers, shape.max_ctx, shape.kv_heads * shape.head_dim), cdt)
    vc = np.zeros_like(kc)
    cfg = _cfg(shape)
    tokens = [7, 300, 5, 1023, 64, 64, 0, 811, 2, 999] if which == "small" else [7, 1300, 5, 2047, 64]
    try:
        for pos, tok in enumerate(tokens):
            nxt, logits = dec.step(tok, pos, want_logits=True)
            x_ref, logits_ref = oracle.decode_step_nf4(cfg, codes, absmax, norms, kc, vc, tok, pos)
            x_gpu, _, _ = dec.read_state()
            if kv_dtype == 0:
                assert synth.max_rel_err(x_gpu, x_ref) < 1e-3, pos
                assert synth.max_rel_err(logits, logits_ref) < 1e-3, pos
                assert nxt == int(np.argmax(logits_ref)), pos
            else:
                assert synth.normwise_rel_err(x_gpu, x_ref) < 1e-3, pos
                assert synth.normwise_rel_err(logits, logits_ref) < 1e-3, pos
            assert nxt == int(np.argmax(logits))
        _, k_gpu, v_gpu = dec.read_state()
        n = len(tokens)
        if kv_dtype == 0:
            assert synth.max_rel_err(k_gpu[:, :n], kc[:, :n]) < 1e-3
            assert synth.max_rel_err(v_gpu[:, :n], vc[:, :n]) < 1e-3
        else:
            kg = oracle.bf16_bits_to_f32(k_gpu[:, :n])
            kr = oracle.bf16_bits_to_f32(kc[:, :n])
            assert synth.normwise_rel_err(kg, kr) < 1e-3
    finally:
        dec.close()


def test_decode_run_greedy_matches_stepwise():
    """decode_run (argmax fed back on the device) == host-driven steps."""
    from aljabr_b200 import native
    from aljabr_b200.decode import LlamaShape
    native.call("aljabr_blackwell_init", 0)
    shape = LlamaShape(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1024, max_ctx=32,
                       kv_dtype=0)
    codes, absmax, norms = _model(77, shape)
    a = _build(shape, codes, absmax, norms)
    b = _build(shape, codes, absmax, norms)
    try:
        run = a.run(11, 0, 12)
        tok, seq = 11, []
        for pos in range(12):
            tok, _ = b.step(tok, pos)
            seq.append(tok)
        np.testing.assert_array_equal(run, np.array(seq, np.int32))
    finally:
        a.close()
        b.close()


def test_decode_rejects_bad_arguments():
    from aljabr_b200 import native
    from aljabr_b200.decode import LlamaNf4Decoder, LlamaShape
    native.call("aljabr_blackwell_init", 0)
    with pytest.raises(native.ProviderError):
        LlamaNf4Decoder(LlamaShape(layers=1, hidden=200, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=64,
                                   max_ctx=8))
    shape = LlamaShape(layers=1, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=64, max_ctx=8)
    dec = LlamaNf4Decoder(shape)
    try:
        with pytest.raises(native.ProviderError):     # layers not registered yet
            dec.step(0, 0)
        with pytest.raises(native.ProviderError):
            dec.step(0, 8)
    finally:
        dec.close()
