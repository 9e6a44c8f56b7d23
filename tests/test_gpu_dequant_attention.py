"""GPU parity: bit-exact dequantisation (the north star's bar for dequantised
weights) and GQA decode attention against the oracle."""
import math

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


def _same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) | np.isnan(b)
    assert np.array_equal(np.isnan(a), np.isnan(b))
    np.testing.assert_array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


def test_golden_dequant(lib, golden):
    from aljabr_b200.bridge import dequantize_nf4, dequantize_row_block
    for fx in golden.values():
        if fx["kind"] == "q4_0_dequant":
            y = dequantize_row_block(lib.TYPE_Q4_0, np.array(fx["weights"], np.uint8), fx["numel"])
            _same_bits(y, np.array(fx["expected"], np.float32))
        elif fx["kind"] == "nf4_dequant":
            y = dequantize_nf4(np.array(fx["codes"], np.uint8), np.array(fx["absmax"], np.float32),
                               fx["numel"], fx["group"])
            _same_bits(y, np.array(fx["expected"], np.float32))


def test_f16_scale_special_values_through_q4_0_dequant(lib, golden):
    """GgufF16SpecialTest's fp16 patterns used as Q4_0 block scales."""
    from aljabr_b200.bridge import dequantize_row_block
    bits = golden["f16_special_values"]["bits"] + [0x3C00, 0xBC00, 0x0400, 0x7BFF]
    blocks = []
    for i, b in enumerate(bits):
        codes = [(j * 7 + i) & 0xFF for j in range(16)]
        blocks += [b & 0xFF, b >> 8] + codes
    w = np.array(blocks, np.uint8)
    y = dequantize_row_block(lib.TYPE_Q4_0, w, 32 * len(bits))
    _same_bits(y, oracle.dequantize_q4_0(w, 32 * len(bits)))


@pytest.mark.parametrize("n,k", [(4096, 4096), (1024, 4096), (33, 96)])
def test_q4_0_q8_0_dequant_bit_exact(lib, n, k):
    from aljabr_b200.bridge import dequantize_row_block
    w4 = synth.q4_0(50 + n, n, k)
    # include blocks with negative scales and zero codes (the -0.0 -> +0.0 case)
    w4.reshape(-1, 18)[::7, 1] |= 0x80
    _same_bits(dequantize_row_block(lib.TYPE_Q4_0, w4, n * k), oracle.dequantize_q4_0(w4, n * k))
    w8 = synth.q8_0(60 + n, n, k)
    w8.reshape(-1, 34)[::5, 1] |= 0x80
    _same_bits(dequantize_row_block(lib.TYPE_Q8_0, w8, n * k), oracle.dequantize_q8_0(w8, n * k))


@pytest.mark.parametrize("n,k,group", [(4096, 4096, 64), (512, 4096, 128), (7, 100, 64), (3, 33, 8)])
def test_nf4_dequant_bit_exact(lib, n, k, group):
    from aljabr_b200.bridge import dequantize_nf4
    codes, absmax = synth.nf4(70 + n, n, k, group)
    absmax[::3] *= -1.0
    numel = n * k
    _same_bits(dequantize_nf4(codes, absmax, numel, group), oracle.dequantize_nf4(codes, absmax, numel, group))


def _attention_case(lib, kv_dtype, Hq, Hkv, D, ctx, start, seed, use_fallback_stride=False):
    import torch
    from aljabr_b200.bridge import decode_attention
    stride = Hkv * D + (4 if use_fallback_stride else 0)
    g = np.random.default_rng(seed)
    kf = g.normal(0, 1, size=(ctx, stride)).astype(np.float32)
    vf = g.normal(0, 1, size=(ctx, stride)).astype(np.float32)
    q = g.normal(0, 1, size=Hq * D).astype(np.float32)
    if kv_dtype == lib.KV_BF16:
        kb, vb = oracle.f32_to_bf16_bits(kf), oracle.f32_to_bf16_bits(vf)
        kf, vf = oracle.bf16_bits_to_f32(kb), oracle.bf16_bits_to_f32(vb)
        dk = torch.from_numpy(kb.view(np.int16)).cuda()
        dv = torch.from_numpy(vb.view(np.int16)).cuda()
    else:
        dk, dv = torch.from_numpy(kf).cuda(), torch.from_numpy(vf).cuda()
    scale = float(np.float32(1.0 / math.sqrt(D)))
    torch.cuda.synchronize()   # caches written on torch's stream; the library's stream is non-blocking
    out = decode_attention(q, dk.data_ptr(), dv.data_ptr(), kv_dtype, stride, Hkv, Hq, D, ctx, start, scale)
    ref = oracle.gqa_decode_attention(q, kf.ravel(), vf.ravel(), stride, Hkv, Hq, D, ctx, start, scale)
    return out, ref


@pytest.mark.parametrize("kv_dtype", [1, 0])
@pytest.mark.parametrize("Hq,Hkv,D,ctx,start", [(32, 8, 128, 4096, 0), (32, 8, 128, 4096, 3000), (32, 8, 128, 1, 0),
                                                 (32, 8, 128, 77, 0), (64, 8, 128, 2048, 0), (16, 16, 64, 300, 5),
                                                 (8, 2, 64, 1000, 0), (4, 1, 256, 513, 0)])
def test_gqa_decode_attention_parity(lib, kv_dtype, Hq, Hkv, D, ctx, start):
    out, ref = _attention_case(lib, kv_dtype, Hq, Hkv, D, ctx, start, seed=Hq * 1000 + ctx)
    assert synth.max_rel_err(out, ref) < 1e-3
    assert synth.normwise_rel_err(out, ref) < 1e-5


@pytest.mark.parametrize("kv_dtype,Hq,Hkv,D,ctx,start,pad", [
    (1, 32, 8, 128, 32768, 0, 0),   # long cache: 171 splits of <= 192 rows, merged through global memory
    (1, 16, 2, 128, 4096, 0, 0),    # 2 kv heads: 64 splits merged through global memory
    (1, 32, 8, 128, 4096, 0, 0),    # one cluster per kv head, merged over distributed shared memory
    (1, 32, 8, 128, 4090, 0, 0),    # clusters with a partial last box
    (1, 32, 8, 128, 130, 0, 0),     # two splits of 65 rows: partial TMA box and partial 16-row chunk
    (1, 24, 8, 128, 999, 7, 0),     # 3 query heads per kv head, ragged start
    (1, 64, 8, 64, 2049, 0, 0),     # 8 query heads per kv head, head_dim 64
    (1, 8, 8, 128, 5000, 4000, 0),  # one query head per kv head, window past the start
    (1, 32, 8, 128, 1000, 0, 4),    # rows 8-byte but not 16-byte aligned: shuffle kernel
    (0, 16, 4, 64, 2500, 0, 0),     # f32 cache: shuffle kernel
])
def test_gqa_decode_attention_kernel_paths(lib, kv_dtype, Hq, Hkv, D, ctx, start, pad):
    out, ref = _attention_case(lib, kv_dtype, Hq, Hkv, D, ctx, start, seed=ctx + pad, use_fallback_stride=pad > 0)
    assert synth.max_rel_err(out, ref) < 1e-3
    assert synth.normwise_rel_err(out, ref) < 1e-5


@pytest.mark.parametrize("Hq,Hkv,D,ctx", [(6, 3, 40, 129), (32, 8, 128, 333)])
def test_gqa_decode_attention_generic_layouts(lib, Hq, Hkv, D, ctx):
    out, ref = _attention_case(lib, 0, Hq, Hkv, D, ctx, 0, seed=ctx, use_fallback_stride=True)
    assert synth.max_rel_err(out, ref) < 1e-3


def test_attention_golden_known_answers(lib, golden):
    import torch
    from aljabr_b200.bridge import decode_attention
    for fx in golden.values():
        if fx["kind"] != "attention":
            continue
        dk = torch.tensor(fx["k"], dtype=torch.float32, device="cuda")
        dv = torch.tensor(fx["v"], dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        out = decode_attention(np.array(fx["q"], np.float32), dk.data_ptr(), dv.data_ptr(), lib.KV_F32, fx["stride"],
                               fx["kv_heads"], fx["q_heads"], fx["head_dim"], fx["seq_len"], fx["start"], fx["scale"])
        np.testing.assert_allclose(out, fx["expected"], atol=fx["tol"], rtol=0, err_msg=fx["name"])


def test_attention_rejects_bad_geometry(lib):
    import torch
    from aljabr_b200.bridge import decode_attention
    from aljabr_b200.native import ProviderError
    dk = torch.zeros(64, device="cuda")
    with pytest.raises(ProviderError):
        decode_attention(np.zeros(6, np.float32), dk.data_ptr(), dk.data_ptr(), 0, 4, 4, 6, 1, 4, 0, 1.0)
    with pytest.raises(ProviderError):
        decode_attention(np.zeros(4, np.float32), dk.data_ptr(), dk.data_ptr(), 0, 4, 4, 4, 1, 4, 4, 1.0)
