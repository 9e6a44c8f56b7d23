"""GPU checks of the entry points the reference's FFM class binds beside the
hot path (BlackwellBinding.java:456-583): device selection, name, TMEM size,
and the RMSNorm / SiLU-FFN glue against the oracle's restatement of the
binding's own contract (BlackwellCpuFallback.java:50-79).

Tolerance: the glue is elementwise fp32 with one reduction; the GPU's sum of
squares is a fixed-order tree, the restatement's a sequential loop, so the
bound is 1e-5 relative (far inside the north star's 1e-3)."""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from aljabr_b200 import native
    native.call("aljabr_blackwell_init", 0)
    return native


def test_device_queries(lib):
    L = lib.lib()
    assert L.aljabr_blackwell_device_get(0) == 0
    buf = ctypes.create_string_buffer(256)
    assert L.aljabr_blackwell_device_name(buf, 256, 0) == 0
    assert b"B200" in buf.value or len(buf.value) > 0
    short = ctypes.create_string_buffer(4)
    assert L.aljabr_blackwell_device_name(short, 4, 0) == 0
    assert len(short.value) == 3
    assert L.aljabr_blackwell_device_name(buf, 256, 999) == lib.ALJ_ERR_BAD_ARG
    assert L.aljabr_blackwell_device_get(-1) == lib.ALJ_ERR_BAD_ARG
    sms = __import__("torch").cuda.get_device_properties(0).multi_processor_count
    assert L.aljabr_blackwell_tmem_size(0) == sms * 256 * 1024
    assert L.aljabr_blackwell_compute_capability(0) == 100


@pytest.mark.parametrize("n", [1, 4096, 8192, 14336, 100003])
def test_rmsnorm_host_buffers(lib, n):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 1, size=n).astype(np.float32)
    w = rng.normal(1, 0.2, size=n).astype(np.float32)
    out = np.full(n, np.nan, np.float32)
    lib.call("aljabr_blackwell_rmsnorm", out.ctypes.data, x.ctypes.data, w.ctypes.data, n, ctypes.c_float(1e-6))
    ref = oracle.rmsnorm_binding(x, w, 1e-6)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-6)


def test_rmsnorm_device_buffers_in_place(lib):
    import torch
    n = 4096
    rng = np.random.default_rng(5)
    x = rng.normal(0, 3, size=n).astype(np.float32)
    w = rng.normal(1, 0.2, size=n).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    dw = torch.from_numpy(w).cuda()
    torch.cuda.synchronize()
    lib.call("aljabr_blackwell_rmsnorm", dx.data_ptr(), dx.data_ptr(), dw.data_ptr(), n, ctypes.c_float(1e-5))
    np.testing.assert_allclose(dx.cpu().numpy(), oracle.rmsnorm_binding(x, w, 1e-5), rtol=1e-5, atol=1e-6)


def test_silu_ffn_aliased_as_the_runner_calls_it(lib):
    # BlackwellRunner.java:586 passes one buffer as out, gate and up
    import torch
    n = 14336
    rng = np.random.default_rng(6)
    g = rng.normal(0, 3, size=n).astype(np.float32)
    u = rng.normal(0, 1, size=n).astype(np.float32)
    out = np.full(n, np.nan, np.float32)
    lib.call("aljabr_blackwell_silu_ffn", out.ctypes.data, g.ctypes.data, u.ctypes.data, n)
    np.testing.assert_allclose(out, oracle.silu_ffn_binding(g, u), rtol=1e-5, atol=1e-7)
    d = torch.from_numpy(g).cuda()
    torch.cuda.synchronize()
    lib.call("aljabr_blackwell_silu_ffn", d.data_ptr(), d.data_ptr(), d.data_ptr(), n)
    np.testing.assert_allclose(d.cpu().numpy(), oracle.silu_ffn_binding(g, g), rtol=1e-5, atol=1e-7)


def test_glue_rejects_bad_sizes(lib):
    L = lib.lib()
    x = np.zeros(4, np.float32)
    assert L.aljabr_blackwell_rmsnorm(x.ctypes.data, x.ctypes.data, x.ctypes.data, 0, ctypes.c_float(1e-6)) \
        == lib.ALJ_ERR_BAD_DIMS
    assert L.aljabr_blackwell_silu_ffn(None, x.ctypes.data, x.ctypes.data, 4) == lib.ALJ_ERR_BAD_ARG
