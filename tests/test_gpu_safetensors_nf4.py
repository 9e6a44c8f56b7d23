"""GPU parity of the safetensors NF4 adapter (AccelWeightBridge.java:164-222:
U8 `.qweight` + fp32 `.scales`, group size 128) end to end:
  * AccelOps.linear (M = 1) on a weight read from a .safetensors file, group
    128, with and without bias, against the oracle and fp64;
  * the chunked model upload (register_model_buffer: 32 MB chunks through
    pinned bounce buffers): a ~200 MB buffer, checked bit-exact across the
    chunk boundaries through the device dequantiser;
  * the Llama decode step built from a Hugging Face-named NF4 checkpoint at
    group 128 (the plain-kernel shape and the table-kernel shape) against
    the oracle's decode step."""
import ctypes
import os
import time

import numpy as np
import pytest

import oracle
from tests import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from aljabr_b200 import native
    native.call("aljabr_blackwell_init", 0)
    return native


def test_linear_group128_from_file(lib, tmp_path):
    from aljabr_b200 import safetensors_nf4 as st
    N, K = 2048, 4096
    w = synth.weights(3, N, K)
    codes, absmax = oracle.quantize_nf4(w, 128)
    bias = synth.activation(4, N) * np.float32(0.1)
    p = str(tmp_path / "lin.safetensors")
    synth.write_safetensors(p, {"proj.qweight": codes.reshape(N, K // 2), "proj.scales": absmax})
    sh = st.SafetensorShard(p)
    try:
        wt = st.nf4_weights(sh)["proj"]
        assert (wt.rows, wt.cols, wt.group) == (N, K, 128)
        x = synth.activation(5, K)
        for b in (None, bias):
            y = st.SafetensorNf4Linear(sh, wt, bias=b)(x)
            ref = oracle.matvec_nf4(codes, absmax, x, N, 128, bias=b, threads=8)
            assert synth.max_rel_err(y, ref) < 1e-3
            f64 = oracle.matvec_f64(oracle.NF4, codes, x, N, absmax=absmax, group_size=128, threads=8)
            if b is not None:
                f64 = f64 + b
            assert synth.max_rel_err(y, f64) < 1e-3
    finally:
        sh.unregister()


def test_chunked_upload_bit_exact(lib):
    """A ~200 MB registered buffer of Q8_0 blocks, dequantised on the device
    around the 32 MB chunk boundaries and at the end."""
    import torch
    nblocks = 200 * 2 ** 20 // 34
    r = synth.rng(7)
    blob = r.integers(0, 256, size=nblocks * 34, dtype=np.uint8)
    d = (r.random(nblocks).astype(np.float32) * 0.01 + 1e-3).astype(np.float16)
    blob.reshape(nblocks, 34)[:, 0:2] = d.view(np.uint8).reshape(nblocks, 2)
    t0 = time.perf_counter()
    lib.call("aljabr_blackwell_register_model_buffer", ctypes.c_void_p(blob.ctypes.data), blob.nbytes)
    dt = time.perf_counter() - t0
    print(f"upload {blob.nbytes / dt / 1e9:.1f} GB/s ({blob.nbytes / 2 ** 20:.0f} MB in {dt * 1e3:.1f} ms)")
    try:
        dev = lib.lib().aljabr_blackwell_device_address(ctypes.c_void_p(blob.ctypes.data))
        assert dev
        chunk_blocks = (32 << 20) // 34
        for b0 in (0, chunk_blocks - 100, 2 * chunk_blocks - 100, 3 * chunk_blocks - 3, nblocks - 600):
            nb = 600
            out = torch.empty(nb * 32, device="cuda")
            torch.cuda.synchronize()
            lib.call("aljabr_blackwell_dequantize_dev", lib.TYPE_Q8_0, ctypes.c_void_p(out.data_ptr()),
                     ctypes.c_void_p(dev + b0 * 34), None, nb * 32, 0, None)
            torch.cuda.synchronize()
            ref = oracle.dequantize_q8_0(blob[b0 * 34:(b0 + nb) * 34], nb * 32)
            np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    finally:
        lib.call("aljabr_blackwell_unregister_model_buffer", ctypes.c_void_p(blob.ctypes.data))


SHAPES = {
    # group 128 needs every K a multiple of 512 in the decode step's NF4 kernels
    "small": dict(layers=2, hidden=512, q_heads=8, kv_heads=2, head_dim=64, ffn=1024, vocab=1024, max_ctx=16),
    "wide": dict(layers=2, hidden=2048, q_heads=16, kv_heads=4, head_dim=128, ffn=4096, vocab=2048, max_ctx=8),
}


@pytest.mark.parametrize("which", ["small", "wide"])
def test_decode_from_hf_checkpoint_group128(lib, tmp_path, which):
    from aljabr_b200 import safetensors_nf4 as st
    from aljabr_b200.decode import LlamaNf4Decoder, LlamaShape
    shape = LlamaShape(**SHAPES[which], group=128, kv_dtype=0)
    g = np.random.default_rng(11)
    H = shape.hidden
    tensors, codes, absmax = {}, [], []
    names = dict(zip(("q", "k", "v", "o", "gate", "up", "down"), st.LLAMA_LAYER))

    def add(name, kind, std=0.02):
        c, a = oracle.quantize_nf4(g.normal(0, std, size=(shape.rows(kind), shape.cols(kind))).astype(np.float32),
                                   128)
        tensors[name + ".qweight"] = c.reshape(shape.rows(kind), shape.cols(kind) // 2)
        tensors[name + ".scales"] = a
        codes.append(c)
        absmax.append(a)

    norms = (1.0 + 0.1 * g.normal(size=(shape.layers * 2 + 1) * H)).astype(np.float32)
    for layer in range(shape.layers):
        for kind, hf in names.items():
            add(f"model.layers.{layer}.{hf}", kind)
        tensors[f"model.layers.{layer}.input_layernorm.weight"] = norms[2 * layer * H:(2 * layer + 1) * H]
        tensors[f"model.layers.{layer}.post_attention_layernorm.weight"] = norms[(2 * layer + 1) * H:(2 * layer + 2) * H]
    add("model.embed_tokens", "embd", std=1.0)
    add("lm_head", "head")
    tensors["model.norm.weight"] = norms[2 * shape.layers * H:]
    p = str(tmp_path / "llama.safetensors")
    synth.write_safetensors(p, tensors)

    sh = st.SafetensorShard(p)
    dec = LlamaNf4Decoder(shape)
    try:
        st.register_llama_decoder(dec, sh)
        cfg = oracle.LlamaCfg(shape.layers, H, shape.q_heads, shape.kv_heads, shape.head_dim, shape.ffn, shape.vocab,
                              shape.max_ctx, 128, shape.eps, shape.rope_theta)
        kc = np.zeros((shape.layers, shape.max_ctx, shape.kv_heads * shape.head_dim), np.float32)
        vc = np.zeros_like(kc)
        for pos, tok in enumerate([3, 1000 % shape.vocab, 17, 5]):
            nxt, logits = dec.step(tok, pos, want_logits=True)
            x_ref, logits_ref = oracle.decode_step_nf4(cfg, codes, absmax, norms, kc, vc, tok, pos)
            x_gpu, _, _ = dec.read_state()
            assert synth.max_rel_err(x_gpu, x_ref) < 1e-3, pos
            assert synth.max_rel_err(logits, logits_ref) < 1e-3, pos
            assert nxt == int(np.argmax(logits_ref)), pos
    finally:
        dec.close()
        sh.unregister()
