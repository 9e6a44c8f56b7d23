"""GPU parity of the prefill attention kernel against the oracle's restatements
of both reference contracts:
  * GgufPrefillAttentionExecution.execute's Java loop (engine/gguf/aljabr-gguf-
    java/.../javabackend/GgufPrefillAttentionExecution.java:44-82) through
    aljabr_blackwell_prefill_attention: causal and sliding-window, a KV row
    stride wider than the KV heads, GQA group sizes 1 / 3 / 4 / 8, head
    dimensions 64 / 96 / 128 / 256, 1 to 200 tokens;
  * the FlashAttention-4 seam's CPU contract (backend/metal/aljabr-backend-
    metal/.../binding/MetalFlashAttentionCpuFallback.java:46-104) through
    aljabr_blackwell_fa4_attention: batches, S > T (causal offset S - T),
    non-causal, soft cap;
  * the device-pointer entry at the Llama-3-8B attention shape, T = 512.
Tolerance: max element-wise relative error 1e-3, denominator guarded by
1e-3 * max|ref|."""
import ctypes

import numpy as np
import pytest

import oracle
from tests import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(scope="module")
def lib():
    from aljabr_b200 import native
    native.call("aljabr_blackwell_init", 0)
    return native


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def _rand(seed, *shape, scale=1.0):
    return (synth.rng(seed).normal(size=shape) * scale).astype(np.float32)


def _java(lib, T, Hq, Hkv, D, window=0, kv_stride=0, seed=0, qscale=1.0):
    kv_stride = kv_stride or Hkv * D
    q = _rand(seed, T, Hq * D, scale=qscale)
    k = _rand(seed + 1, T, kv_stride)
    v = _rand(seed + 2, T, kv_stride)
    scale = float(1.0 / np.sqrt(D))
    out = np.full((T, Hq * D), np.nan, np.float32)
    lib.call("aljabr_blackwell_prefill_attention", _p(out), _p(q), _p(k), _p(v), T, Hq, Hkv, D, scale, window,
             kv_stride)
    ref = oracle.prefill_attention(q, k, v, T, Hq, Hkv, D, scale, window=window, kv_stride=kv_stride)
    err = synth.max_rel_err(out, ref)
    assert err < TOL, (T, Hq, Hkv, D, window, err)


@pytest.mark.parametrize("T", [1, 7, 64, 65, 200])
def test_java_causal_lengths(lib, T):
    _java(lib, T, 8, 2, 128, seed=T)


@pytest.mark.parametrize("window", [1, 5, 16, 300])
def test_java_sliding_window(lib, window):
    _java(lib, 150, 8, 2, 128, window=window, seed=window)


def test_java_wide_kv_stride(lib):
    _java(lib, 33, 4, 2, 64, kv_stride=2 * 64 + 24, seed=11)


@pytest.mark.parametrize("Hq,Hkv", [(4, 4), (6, 2), (16, 4), (16, 2)])
def test_java_gqa_groups(lib, Hq, Hkv):
    _java(lib, 40, Hq, Hkv, 64, seed=Hq * 10 + Hkv)


@pytest.mark.parametrize("D", [64, 96, 256])
def test_java_head_dims(lib, D):
    _java(lib, 45, 4, 2, D, seed=D)


def _f64_prefill(q, k, v, T, Hq, Hkv, D, scale):
    q64, k64, v64 = (a.astype(np.float64) for a in (q, k, v))
    out = np.zeros((T, Hq * D))
    g = Hq // Hkv
    for h in range(Hq):
        kh = h // g
        s = q64[:, h * D:(h + 1) * D] @ k64[:, kh * D:(kh + 1) * D].T * scale
        s[np.triu_indices(T, 1)] = -np.inf
        w = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h * D:(h + 1) * D] = (w / w.sum(axis=1, keepdims=True)) @ v64[:, kh * D:(kh + 1) * D]
    return out


def test_java_peaked_scores(lib):
    """Large logits (std ~8, a sharp softmax).  There the fp32 dot's own
    rounding (~1e-5 on the scores, in the reference's order as in any other)
    reaches ~1e-3 of the smallest outputs, so both fp32 results are held to
    fp64: the GPU's error within 1e-3 or twice the reference-order oracle's."""
    T, Hq, Hkv, D = 70, 4, 1, 128
    q = _rand(99, T, Hq * D, scale=8.0)
    k = _rand(100, T, Hkv * D)
    v = _rand(101, T, Hkv * D)
    scale = float(1.0 / np.sqrt(D))
    out = np.full((T, Hq * D), np.nan, np.float32)
    lib.call("aljabr_blackwell_prefill_attention", _p(out), _p(q), _p(k), _p(v), T, Hq, Hkv, D, scale, 0, Hkv * D)
    ref = oracle.prefill_attention(q, k, v, T, Hq, Hkv, D, scale)
    exact = _f64_prefill(q, k, v, T, Hq, Hkv, D, scale)
    e_gpu, e_ref = synth.max_rel_err(out, exact), synth.max_rel_err(ref, exact)
    assert e_gpu < max(TOL, 2 * e_ref), (e_gpu, e_ref)


@pytest.mark.parametrize("B,T,S,causal,cap", [(1, 9, 9, 1, 0.0), (2, 5, 9, 1, 0.0), (2, 6, 6, 0, 0.0),
                                              (1, 12, 20, 1, 30.0), (3, 4, 4, 0, 5.0)])
def test_fa4_contract(lib, B, T, S, causal, cap):
    H, Hkv, D = 4, 2, 64
    q = _rand(B * 100 + T, B, T, H, D)
    k = _rand(B * 100 + T + 1, B, S, Hkv, D)
    v = _rand(B * 100 + T + 2, B, S, Hkv, D)
    out = np.full(B * T * H * D, np.nan, np.float32)
    rc = lib.lib().aljabr_blackwell_fa4_attention(_p(out), _p(q), _p(k), _p(v), B, T, S, H, Hkv, D, 0.125, causal, 0,
                                                  cap)
    assert rc == 0, lib.lib().aljabr_blackwell_last_error()
    ref = oracle.fa4_attention(q, k, v, B, T, S, H, Hkv, D, 0.125, causal=bool(causal), soft_cap=cap)
    assert synth.max_rel_err(out, ref) < TOL


def test_fa4_availability(lib):
    assert lib.lib().aljabr_blackwell_fa4_sdpa_available() == 1
    assert lib.lib().aljabr_blackwell_fa4_bf16_available() == 0


def test_dev_llama_shape(lib):
    """Llama-3-8B attention (32 / 8 heads, head_dim 128) over a 512-token prompt."""
    import torch
    T, Hq, Hkv, D = 512, 32, 8, 128
    q = _rand(5, T, Hq * D)
    k = _rand(6, T, Hkv * D)
    v = _rand(7, T, Hkv * D)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    dout = torch.full((T, Hq * D), float("nan"), device="cuda")
    torch.cuda.synchronize()
    lib.call("aljabr_blackwell_prefill_attention_dev", ctypes.c_void_p(dout.data_ptr()),
             ctypes.c_void_p(dq.data_ptr()), ctypes.c_void_p(dk.data_ptr()), ctypes.c_void_p(dv.data_ptr()), 1, T, T,
             Hq, Hkv, D, Hkv * D, float(1 / np.sqrt(D)), 1, 0, 0.0, None)
    torch.cuda.synchronize()
    ref = oracle.prefill_attention(q, k, v, T, Hq, Hkv, D, float(1 / np.sqrt(D)))
    assert synth.max_rel_err(dout.cpu().numpy(), ref) < TOL
