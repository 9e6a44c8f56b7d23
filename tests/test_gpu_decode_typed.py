"""GPU parity of the decode step with GGUF-typed weights, one type per tensor
(registerDecodeLayer's typeQ .. typeDown), against the oracle's typed
restatement of GgufDecodePass's layer loop.

Mixes the formats the way llama.cpp's Q4_K_M files do (Q4_K projections with
Q6_K v / down), plus Q4_0 / Q8_0 tensors and a Q8_0 embedding.  With an fp32
KV cache the two sides differ only in summation order: 1e-3 max relative
error on the residual stream and the logits, as for the single kernels."""
import numpy as np
import pytest

import oracle
from tests import synth

pytestmark = pytest.mark.gpu

NAMES = ["q", "k", "v", "o", "gate", "up", "down"]
# per layer, q k v o gate up down
LAYER_TYPES = [
    [oracle.Q4_K, oracle.Q4_K, oracle.Q6_K, oracle.Q4_0, oracle.Q4_K, oracle.Q4_K, oracle.Q6_K],
    [oracle.Q8_0, oracle.Q8_0, oracle.Q8_0, oracle.Q6_K, oracle.Q4_0, oracle.Q4_0, oracle.Q8_0],
]


def _f16_bytes(v):
    return np.array([oracle.f32_to_f16_bits(float(t)) for t in v], dtype=np.uint16).view(np.uint8).reshape(-1, 2)


def _tensor(kind, g, rows, cols, std=0.02):
    """Random GGUF blocks with weights of roughly `std` magnitude."""
    if kind == oracle.Q4_0:
        return oracle.encode_q4_0(g.normal(0, std, size=(rows, cols)).astype(np.float32))
    if kind == oracle.Q8_0:
        return oracle.encode_q8_0(g.normal(0, std, size=(rows, cols)).astype(np.float32))
    w = synth.k_quant(kind, int(g.integers(1 << 30)), rows, cols)
    blocks = w.reshape(-1, oracle.K_BLOCK_BYTES[kind])
    nb = blocks.shape[0]
    if kind == oracle.Q4_K:   # d * scale * q ~ 240 d on average
        blocks[:, 0:2] = _f16_bytes(g.uniform(0.5, 2.0, nb) * std / 240)
        blocks[:, 2:4] = _f16_bytes(g.uniform(0.5, 2.0, nb) * std / 60)
    else:                     # d * |scale| * |q - 32| ~ 1000 d
        blocks[:, 208:210] = _f16_bytes(g.uniform(0.5, 2.0, nb) * std / 1000)
    return w


def _model(seed, shape, layer_types, embd_type, head_type):
    g = np.random.default_rng(seed)
    weights, types = [], []
    for l in range(shape.layers):
        for n, t in zip(NAMES, layer_types[l % len(layer_types)]):
            weights.append(_tensor(t, g, shape.rows(n), shape.cols(n)))
            types.append(t)
    weights.append(_tensor(embd_type, g, shape.rows("embd"), shape.cols("embd"), std=1.0))
    types.append(embd_type)
    weights.append(_tensor(head_type, g, shape.rows("head"), shape.cols("head")))
    types.append(head_type)
    norms = (1.0 + 0.1 * g.normal(size=(shape.layers * 2 + 1) * shape.hidden)).astype(np.float32)
    return weights, types, norms


def _build(shape, weights, types, norms):
    from aljabr_b200.decode import LlamaNf4Decoder
    dec = LlamaNf4Decoder(shape)
    H, L = shape.hidden, shape.layers
    for l in range(L):
        dec.register_layer_typed(l, weights[7 * l:7 * l + 7], types[7 * l:7 * l + 7],
                                 norms[2 * l * H:(2 * l + 1) * H], norms[(2 * l + 1) * H:(2 * l + 2) * H])
    dec.register_output_typed(weights[7 * L], types[7 * L], weights[7 * L + 1], types[7 * L + 1], norms[2 * L * H:])
    return dec


# "small": every K below 2048 (generic Q4_0 / Q8_0 kernels); "wide": K a
# multiple of 2048, so Q4_0 / Q8_0 run the tensor-core kernel.
SHAPES = {
    "small": dict(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1024, max_ctx=32),
    "wide": dict(layers=2, hidden=2048, q_heads=16, kv_heads=4, head_dim=128, ffn=4096, vocab=2048, max_ctx=16),
}


@pytest.mark.parametrize("which,embd_type,head_type", [("small", oracle.Q8_0, oracle.Q6_K),
                                                       ("small", oracle.Q4_K, oracle.Q4_0),
                                                       ("wide", oracle.Q6_K, oracle.Q8_0)])
def test_typed_decode_step_matches_oracle(which, embd_type, head_type):
    from aljabr_b200 import native
    from aljabr_b200.decode import LlamaShape
    native.call("aljabr_blackwell_init", 0)
    shape = LlamaShape(**SHAPES[which], kv_dtype=0)
    weights, types, norms = _model(321, shape, LAYER_TYPES, embd_type, head_type)
    dec = _build(shape, weights, types, norms)
    kc = np.zeros((shape.layers, shape.max_ctx, shape.kv_heads * shape.head_dim), np.float32)
    vc = np.zeros_like(kc)
    cfg = oracle.LlamaCfg(shape.layers, shape.hidden, shape.q_heads, shape.kv_heads, shape.head_dim, shape.ffn,
                          shape.vocab, shape.max_ctx, shape.group, shape.eps, shape.rope_theta)
    absmax = [None] * len(weights)
    tokens = [7, 300, 5, 1023, 64, 0, 811, 2] if which == "small" else [7, 1300, 2047, 64]
    try:
        for pos, tok in enumerate(tokens):
            nxt, logits = dec.step(tok, pos, want_logits=True)
            x_ref, logits_ref = oracle.decode_step_typed(cfg, weights, types, absmax, norms, kc, vc, tok, pos)
            x_gpu, _, _ = dec.read_state()
            assert synth.max_rel_err(x_gpu, x_ref) < 1e-3, pos
            assert synth.max_rel_err(logits, logits_ref) < 1e-3, pos
            assert nxt == int(np.argmax(logits_ref)), pos
        _, k_gpu, v_gpu = dec.read_state()
        n = len(tokens)
        assert synth.max_rel_err(k_gpu[:, :n], kc[:, :n]) < 1e-3
        assert synth.max_rel_err(v_gpu[:, :n], vc[:, :n]) < 1e-3
    finally:
        dec.close()


def test_typed_decode_run_greedy_matches_stepwise():
    """decode_run (argmax fed back on the device) == host-driven steps, for a
    GGUF-typed model with a bf16 KV cache."""
    from aljabr_b200 import native
    from aljabr_b200.decode import LlamaShape
    native.call("aljabr_blackwell_init", 0)
    shape = LlamaShape(**SHAPES["small"], kv_dtype=1)
    weights, types, norms = _model(99, shape, LAYER_TYPES, oracle.Q4_K, oracle.Q6_K)
    a = _build(shape, weights, types, norms)
    b = _build(shape, weights, types, norms)
    try:
        run = a.run(11, 0, 10)
        tok, seq = 11, []
        for pos in range(10):
            tok, _ = b.step(tok, pos)
            seq.append(tok)
        np.testing.assert_array_equal(run, np.array(seq, np.int32))
    finally:
        a.close()
        b.close()


def test_typed_decode_rejects_unknown_types():
    from aljabr_b200 import native
    from aljabr_b200.decode import LlamaNf4Decoder, LlamaShape
    native.call("aljabr_blackwell_init", 0)
    shape = LlamaShape(**SHAPES["small"], kv_dtype=0)
    weights, types, norms = _model(5, shape, LAYER_TYPES, oracle.Q8_0, oracle.Q8_0)
    dec = LlamaNf4Decoder(shape)
    H = shape.hidden
    try:
        with pytest.raises(native.ProviderError):
            dec.register_layer_typed(0, weights[:7], [13] + types[1:7], norms[:H], norms[H:2 * H])
        with pytest.raises(native.ProviderError):   # NF4 needs its absmax
            dec.register_layer_typed(0, weights[:7], [native.TYPE_NF4] + types[1:7], norms[:H], norms[H:2 * H])
    finally:
        dec.close()
