"""GPU: aljabr_blackwell_decode_attention_noalloc (split scratch in a static
device array) against aljabr_blackwell_decode_attention_dev (scratch from
cudaMalloc), called back to back through the C-ABI.  Named so pytest
collects it last; it also passes when run alone."""
import ctypes
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_FLOATS = 1 << 20


@pytest.fixture(scope="module")
def lib():
    import torch
    from aljabr_b200 import native
    native.call("aljabr_blackwell_init", 0)
    torch.cuda.set_device(0)
    return native


def _caches(kv_dtype, ctx, stride, seed):
    import torch
    g = np.random.default_rng(seed)
    k = torch.from_numpy(g.normal(0, 1, size=(ctx, stride)).astype(np.float32)).cuda()
    v = torch.from_numpy(g.normal(0, 1, size=(ctx, stride)).astype(np.float32)).cuda()
    if kv_dtype == 1:
        k, v = k.to(torch.bfloat16), v.to(torch.bfloat16)
    return k, v


def _run(native, name, q, k, v, kv_dtype, stride, Hkv, Hq, D, ctx, start, scale, stream):
    import torch
    out = torch.full((Hq * D,), float("nan"), device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()   # the _dev entry's NULL stream is the library's own, not torch's
    rc = getattr(native.lib(), name)(
        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), kv_dtype, stride, Hkv, Hq, D, ctx, start, ctypes.c_float(scale),
        ctypes.c_void_p(stream))
    return rc, out


@pytest.mark.parametrize("kv_dtype", [1, 0])
@pytest.mark.parametrize("Hq,Hkv,D,ctx,start", [(32, 8, 128, 4096, 0), (32, 8, 128, 2500, 700),
                                                 (8, 2, 64, 1000, 0), (32, 8, 128, 40, 0)])
def test_noalloc_matches_dev_entry_twice(lib, kv_dtype, Hq, Hkv, D, ctx, start):
    import torch
    stride = Hkv * D
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream().cuda_stream
    k, v = _caches(kv_dtype, ctx, stride, seed=ctx + Hq)
    g = np.random.default_rng(ctx)
    for call in range(2):   # two calls in a row, different queries
        q = torch.from_numpy(g.normal(0, 1, size=Hq * D).astype(np.float32)).cuda()
        rc0, want = _run(lib, "aljabr_blackwell_decode_attention_dev", q, k, v, kv_dtype, stride, Hkv, Hq, D, ctx,
                         start, scale, stream)
        rc1, got = _run(lib, "aljabr_blackwell_decode_attention_noalloc", q, k, v, kv_dtype, stride, Hkv, Hq, D,
                        ctx, start, scale, stream)
        torch.cuda.synchronize()
        assert rc0 == 0 and rc1 == 0, (call, rc0, rc1)
        w, o = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(o).all()
        floor = 1e-3 * np.abs(w).max()
        rel = (np.abs(o - w) / np.maximum(np.abs(w), floor)).max()
        assert rel < 1e-3, (call, rel)
        if ctx == 4096:   # and on its own against the CPU restatement of the reference
            import oracle
            kf, vf = k.float().cpu().numpy(), v.float().cpu().numpy()
            ref = oracle.gqa_decode_attention(q.cpu().numpy(), kf.ravel(), vf.ravel(), stride, Hkv, Hq, D, ctx,
                                              start, scale)
            rel = (np.abs(o - ref) / np.maximum(np.abs(ref), 1e-3 * np.abs(ref).max())).max()
            assert rel < 1e-3, (call, rel)


def test_noalloc_rejects_scratch_beyond_static_array(lib):
    import torch
    # 1 KV head, 128 query heads of 256: 256 splits need 128*256*258 floats.
    Hq, Hkv, D, ctx = 128, 1, 256, 16384
    assert Hq * 256 * (D + 2) > NOALLOC_SCRATCH_FLOATS
    k, v = _caches(1, ctx, Hkv * D, seed=5)
    q = torch.zeros(Hq * D, device="cuda", dtype=torch.float32)
    rc, out = _run(lib, "aljabr_blackwell_decode_attention_noalloc", q, k, v, 1, Hkv * D, Hkv, Hq, D, ctx, 0,
                   1.0 / 16.0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == lib.ALJ_ERR_BAD_DIMS
    assert torch.isnan(out).all()   # nothing was launched
