"""GPU parity of the dequantise-and-matvec kernels against the oracle (the
reference's summation order) and the fp64 ground truth, through the C-ABI.

Tolerance (north star): max element-wise relative error 1e-3, with the
denominator guarded by 1e-3 * max|ref| where ref_i is near zero."""
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


def _host_matvec(lib, type_id, w, x, K, N, absmax=None, group=64, bias=None):
    """Drive the host-buffer entry point with w registered as a model buffer."""
    from aljabr_b200.bridge import _registered
    y = np.full(N, np.nan, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    with _registered(w):
        if type_id == lib.TYPE_Q4_0:
            lib.call("aljabr_blackwell_matvec_tb_q4_0", y.ctypes.data, x.ctypes.data, w.ctypes.data, K, N)
        elif type_id == lib.TYPE_Q8_0:
            lib.call("aljabr_blackwell_matvec_tb_q8_0", y.ctypes.data, x.ctypes.data, w.ctypes.data, K, N)
        else:
            with _registered(absmax):
                b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
                lib.call("aljabr_blackwell_linear_nf4", y.ctypes.data, x.ctypes.data, w.ctypes.data,
                         absmax.ctypes.data, None if b is None else b.ctypes.data, K, N, group)
    return y


def test_golden_known_answers_q4_0_q8_0(lib, golden):
    for fx in golden.values():
        if fx["kind"] not in ("q4_0_matvec", "q8_0_matvec"):
            continue
        t = lib.TYPE_Q4_0 if fx["kind"] == "q4_0_matvec" else lib.TYPE_Q8_0
        w = np.array(fx["weights"], dtype=np.uint8)
        y = _host_matvec(lib, t, w, np.array(fx["x"], np.float32), fx["K"], fx["N"])
        exp = np.array(fx["expected"], dtype=np.float32)
        if fx["tol"] == 0.0:
            np.testing.assert_array_equal(y, exp, err_msg=fx["name"])
        else:
            np.testing.assert_allclose(y, exp, rtol=fx["tol"], atol=fx["tol"], err_msg=fx["name"])


@pytest.mark.parametrize("N,K", [(7, 256), (33, 512), (300, 2048), (1024, 4096), (4096, 4096),
                                 (14336, 4096), (4096, 14336), (5, 160), (3, 96), (36, 256), (64, 2304),
                                 (148 * 4 + 4, 6144)])
def test_q4_0_matvec_parity(lib, N, K):
    w = synth.q4_0(1000 + N, N, K)
    x = synth.activation(2000 + K, K)
    y = _host_matvec(lib, lib.TYPE_Q4_0, w, x, K, N)
    ref = oracle.matvec_q4_0(w, x, N, threads=8)
    g = oracle.matvec_f64(oracle.Q4_0, w, x, N, threads=8)
    assert synth.max_rel_err(y, ref) < TOL
    assert synth.max_rel_err(y, g) < TOL
    assert synth.normwise_rel_err(y, g) < 1e-5
    if N >= 32:
        # the reference's default order at >= 32 rows: the prepared cache
        # (GgufPreparedCachePolicy.java:66-75, GgufQ32Dot.java:627-670)
        prep = oracle.matvec_q4_0_prepared(w, x, N, threads=8)
        assert synth.max_rel_err(y, prep) < TOL


@pytest.mark.parametrize("N,K", [(7, 256), (1024, 4096), (4096, 4096), (14336, 4096), (4096, 14336), (5, 160),
                                 (64, 1280), (36, 256)])
def test_q8_0_matvec_parity(lib, N, K):
    w = synth.q8_0(3000 + N, N, K)
    x = synth.activation(4000 + K, K)
    y = _host_matvec(lib, lib.TYPE_Q8_0, w, x, K, N)
    for vector_order in (True, False):
        ref = oracle.matvec_q8_0(w, x, N, vector_order=vector_order, threads=8)
        assert synth.max_rel_err(y, ref) < TOL
    g = oracle.matvec_f64(oracle.Q8_0, w, x, N, threads=8)
    assert synth.max_rel_err(y, g) < TOL
    assert synth.normwise_rel_err(y, g) < 1e-5


@pytest.mark.parametrize("N,K,group", [(7, 256, 64), (4096, 4096, 64), (1024, 4096, 128), (14336, 4096, 64),
                                       (4096, 14336, 64), (9, 200, 64), (6, 384, 96), (64, 1280, 64),
                                       (8, 1536, 128), (128256 // 16, 4096, 64)])
def test_nf4_matvec_parity(lib, N, K, group):
    codes, absmax = synth.nf4(5000 + N, N, K, group)
    x = synth.activation(6000 + K, K)
    y = _host_matvec(lib, lib.TYPE_NF4, codes, x, K, N, absmax=absmax, group=group)
    ref = oracle.matvec_nf4(codes, absmax, x, N, group, threads=8)
    g = oracle.matvec_f64(oracle.NF4, codes, x, N, absmax=absmax, group_size=group, threads=8)
    assert synth.max_rel_err(y, ref) < TOL
    assert synth.max_rel_err(y, g) < TOL
    assert synth.normwise_rel_err(y, g) < 1e-5


def test_nf4_linear_bias(lib):
    N, K = 512, 4096
    codes, absmax = synth.nf4(7, N, K)
    x = synth.activation(8, K)
    bias = synth.activation(9, N)
    y = _host_matvec(lib, lib.TYPE_NF4, codes, x, K, N, absmax=absmax, bias=bias)
    ref = oracle.matvec_nf4(codes, absmax, x, N, 64, bias=bias, threads=8)
    assert synth.max_rel_err(y, ref) < TOL


def test_bridge_pair_triple_batch(lib):
    from aljabr_b200.bridge import GgufBlackwellBridge, GgufExecutionDispatcher, GgufModel
    K = 4096
    wq, wk, wv = synth.q4_0(11, 4096, K), synth.q4_0(12, 1024, K), synth.q8_0(13, 1024, K)
    model = GgufModel.pack([("q", 2, K, 4096, wq), ("k", 2, K, 1024, wk), ("v", 8, K, 1024, wv)])
    t = model.tensors
    x = synth.activation(14, K)
    d = GgufExecutionDispatcher(model)
    q, k, v = (np.zeros(n, np.float32) for n in (4096, 1024, 1024))
    d.dispatch_mat_vec_triple(t["q"], q, t["k"], k, t["v"], v, x)
    assert synth.max_rel_err(q, oracle.matvec_q4_0(wq, x, 4096, threads=8)) < TOL
    assert synth.max_rel_err(k, oracle.matvec_q4_0(wk, x, 1024, threads=8)) < TOL
    assert synth.max_rel_err(v, oracle.matvec_q8_0(wv, x, 1024, threads=8)) < TOL
    q2, k2 = np.zeros(4096, np.float32), np.zeros(1024, np.float32)
    d.dispatch_mat_vec_pair(t["q"], q2, t["k"], k2, x)
    np.testing.assert_array_equal(q2, q)
    np.testing.assert_array_equal(k2, k)
    xb = np.stack([synth.activation(20 + b, K) for b in range(3)])
    yb = np.zeros((3, 1024), np.float32)
    d.dispatch_mat_vec_batch(t["k"], xb, yb, 3)
    for b in range(3):
        assert synth.max_rel_err(yb[b], oracle.matvec_q4_0(wk, xb[b], 1024, threads=8)) < TOL
    # batches of Q4_0 run on the tensor-core GEMM, single rows on the matvec:
    # the two agree to the tolerance, not bit for bit
    y1 = np.zeros(1024, np.float32)
    d.dispatch_mat_vec(t["k"], xb[1], y1)
    assert synth.max_rel_err(yb[1], y1) < TOL
    GgufBlackwellBridge.release_model(model)


def test_device_pointer_api_matches_host_api(lib):
    import torch
    N, K = 4096, 4096
    w = synth.q4_0(30, N, K)
    x = synth.activation(31, K)
    host = _host_matvec(lib, lib.TYPE_Q4_0, w, x, K, N)
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty(N, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()   # inputs prepared on torch's stream; the library's stream is non-blocking
    lib.call("aljabr_blackwell_matvec_dev", lib.TYPE_Q4_0, dy.data_ptr(), dx.data_ptr(), dw.data_ptr(), None,
             K, N, 0, None, None)
    torch.cuda.synchronize()   # device-wide: the library's own stream ran the kernel
    np.testing.assert_array_equal(dy.cpu().numpy(), host)


def test_errors_are_reported_not_fallen_back(lib):
    from aljabr_b200.native import ProviderError, UnsupportedOperation
    w = synth.q4_0(40, 4, 256)
    x = synth.activation(41, 256)
    y = np.zeros(4, np.float32)
    # an unregistered host pointer is not silently read on the CPU
    with pytest.raises(ProviderError) as e:
        lib.call("aljabr_blackwell_matvec_tb_q4_0", y.ctypes.data, x.ctypes.data, w.ctypes.data, 256, 4)
    assert e.value.code == lib.ALJ_ERR_NOT_REGISTERED
    with pytest.raises(ProviderError) as e:
        lib.call("aljabr_blackwell_matvec_tb_q4_0", y.ctypes.data, x.ctypes.data, w.ctypes.data, 250, 4)
    assert e.value.code == lib.ALJ_ERR_BAD_DIMS
    with pytest.raises(UnsupportedOperation):
        lib.call("aljabr_blackwell_matvec_tb_batch", y.ctypes.data, x.ctypes.data, w.ctypes.data, 256, 4, 13, 1)
    bits = ctypes.c_uint(0)
    lib.call("aljabr_blackwell_device_status", ctypes.byref(bits))
    assert bits.value == 0
