"""GPU parity of the GGUF K-quant matvecs (Q4_K, Q6_K) against the oracle
(the reference's GgufQ4RawDot.dotRowQ4K / GgufQ6RawDot.dotRowQ6K float order),
the fp64 element sums and the reference's own known answers, through the C-ABI.

Tolerance (north star): max element-wise relative error 1e-3, with the
denominator guarded by 1e-3 * max|ref| where ref_i is near zero."""
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


def _dev_matvec(lib, type_id, w, x, K, N, bias=None, w_offset=0):
    """aljabr_blackwell_matvec_dev on device copies; w_offset shifts the weight base."""
    import torch
    dw = torch.zeros(w.size + 16, dtype=torch.uint8, device="cuda")
    dw[w_offset:w_offset + w.size] = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    dy = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    db = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, np.float32)).cuda()
    torch.cuda.synchronize()   # inputs prepared on torch's stream; the library's stream is non-blocking
    lib.call("aljabr_blackwell_matvec_dev", type_id, dy.data_ptr(), dx.data_ptr(), dw.data_ptr() + w_offset, None,
             K, N, 0, None if db is None else db.data_ptr(), None)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


def _host_matvec(lib, type_id, w, x, K, N):
    from aljabr_b200.bridge import _registered
    y = np.full(N, np.nan, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    name = "aljabr_blackwell_matvec_tb_q4_k" if type_id == lib.TYPE_Q4_K else "aljabr_blackwell_matvec_tb_q6_k"
    with _registered(w):
        lib.call(name, y.ctypes.data, x.ctypes.data, w.ctypes.data, K, N)
    return y


def test_golden_known_answers(lib, golden):
    seen = set()
    for fx in golden.values():
        if fx["kind"] != "k_matvec":
            continue
        seen.add(fx["type"])
        w = np.array(fx["weights"], dtype=np.uint8)
        x = np.array(fx["x"], np.float32)
        for y in (_host_matvec(lib, fx["type"], w, x, fx["K"], fx["N"]),
                  _dev_matvec(lib, fx["type"], w, x, fx["K"], fx["N"])):
            np.testing.assert_array_equal(y, np.array(fx["expected"], np.float32), err_msg=fx["name"])
    assert seen == {lib.TYPE_Q4_K, lib.TYPE_Q6_K}


@pytest.mark.parametrize("kind", [oracle.Q4_K, oracle.Q6_K])
@pytest.mark.parametrize("N,K", [(1, 256), (7, 512), (37, 2816), (300, 2048), (4096, 4096), (1024, 14336),
                                 (14336, 4096), (33, 5120), (40, 11264),
                                 # Q4_K on integer tensor cores (K a multiple of 2048, rows in 4s):
                                 # ragged 16-row tiles and a 36-row slab
                                 (100, 2048), (516, 6144)])
def test_matches_oracle_and_fp64(lib, kind, N, K):
    w = synth.k_quant(kind, 100 + N + kind, N, K)
    x = synth.activation(200 + K, K)
    y = _dev_matvec(lib, kind, w, x, K, N)
    ref = oracle.matvec_k(kind, w, x, N, threads=8)
    ref64 = oracle.matvec_f64(kind, w, x, N, threads=8)
    assert synth.max_rel_err(y, ref) < TOL
    assert synth.max_rel_err(y, ref64) < TOL
    assert synth.normwise_rel_err(y, ref64) < 1e-5


@pytest.mark.parametrize("kind", [oracle.Q4_K, oracle.Q6_K])
def test_host_entry_and_bias(lib, kind):
    N, K = 515, 2304
    w = synth.k_quant(kind, 7 + kind, N, K)
    x = synth.activation(8, K)
    bias = synth.activation(9, N)
    ref = oracle.matvec_k(kind, w, x, N, threads=8)
    np.testing.assert_array_equal(_host_matvec(lib, kind, w, x, K, N), _dev_matvec(lib, kind, w, x, K, N))
    yb = _dev_matvec(lib, kind, w, x, K, N, bias=bias)
    assert synth.max_rel_err(yb, ref + bias) < TOL


def test_q6_k_rows_need_only_two_byte_alignment(lib):
    """Q6_K super-blocks are 210 bytes, so rows start on 2-byte boundaries."""
    N, K = 33, 768
    w = synth.k_quant(oracle.Q6_K, 5, N, K)
    x = synth.activation(6, K)
    y = _dev_matvec(lib, oracle.Q6_K, w, x, K, N, w_offset=2)
    assert synth.max_rel_err(y, oracle.matvec_k(oracle.Q6_K, w, x, N)) < TOL


def test_k_quant_errors(lib):
    from aljabr_b200.native import ProviderError, UnsupportedOperation
    w = synth.k_quant(oracle.Q4_K, 1, 4, 512)
    x = synth.activation(2, 512)
    with pytest.raises(ProviderError) as e:
        _dev_matvec(lib, oracle.Q4_K, w, x, 500, 4)
    assert e.value.code == lib.ALJ_ERR_BAD_DIMS
    # a Q4_K base that is not 16-byte aligned is refused, not read misaligned
    with pytest.raises(UnsupportedOperation):
        _dev_matvec(lib, oracle.Q4_K, w, x, 512, 4, w_offset=8)
