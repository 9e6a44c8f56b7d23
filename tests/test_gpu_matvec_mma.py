"""GPU parity of the tensor-core Q4_0 path (K a multiple of 2048) against the
oracle: ragged row counts (4-row units, 8/4-row TMA boxes), weight segments
that split slabs, activations with outliers and extreme scales (the per-block
exponent and exact hi/lo split of x), and bit-identical repeat calls (the
fixed-order partial reduction).  Tolerance: max element-wise relative error
1e-3 with the denominator guarded by 1e-3 * max|ref|."""
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


def _dev_matvec(lib, w, x, K, N):
    import torch
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    dy = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()   # inputs from torch's stream; the library's own stream is non-blocking
    lib.call("aljabr_blackwell_matvec_dev", lib.TYPE_Q4_0, dy.data_ptr(), dx.data_ptr(), dw.data_ptr(), None,
             K, N, 0, None, None)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("N", [4, 8, 12, 20, 28, 36, 100, 596, 1028, 148 * 16 + 12])
@pytest.mark.parametrize("K", [2048, 4096])
def test_ragged_rows(lib, N, K):
    w = synth.q4_0(300 + N, N, K)
    x = synth.activation(400 + K, K)
    y = _dev_matvec(lib, w, x, K, N)
    assert synth.max_rel_err(y, oracle.matvec_q4_0(w, x, N, threads=8)) < TOL


@pytest.mark.parametrize("scale", [1.0, 3e4, 1e-6])
def test_activation_outliers_and_scales(lib, scale):
    N, K = 2048, 8192
    w = synth.q4_0(7, N, K)
    x = synth.activation(8, K) * np.float32(scale)
    x[5::97] *= 50.0          # outliers dominate their 32-element blocks
    x[7::131] = 0.0
    x[:32] = 0.0              # an all-zero block
    y = _dev_matvec(lib, w, x, K, N)
    assert synth.max_rel_err(y, oracle.matvec_q4_0(w, x, N, threads=8)) < TOL
    assert synth.max_rel_err(y, oracle.matvec_f64(oracle.Q4_0, w, x, N, threads=8)) < TOL


def test_repeat_calls_are_bit_identical(lib):
    N, K = 4096, 14336
    w = synth.q4_0(9, N, K)
    x = synth.activation(10, K)
    a = _dev_matvec(lib, w, x, K, N)
    b = _dev_matvec(lib, w, x, K, N)
    np.testing.assert_array_equal(a, b)


def test_segments_split_slabs(lib):
    """Three Q4_0 segments whose boundaries fall inside 16-row slabs."""
    from aljabr_b200.bridge import GgufExecutionDispatcher, GgufModel
    K = 4096
    rows = (1028, 516, 1020)
    ws = [synth.q4_0(50 + i, n, K) for i, n in enumerate(rows)]
    model = GgufModel.pack([(f"s{i}", 2, K, n, w) for i, (n, w) in enumerate(zip(rows, ws))])
    t = model.tensors
    x = synth.activation(60, K)
    outs = [np.zeros(n, np.float32) for n in rows]
    d = GgufExecutionDispatcher(model)
    d.dispatch_mat_vec_triple(t["s0"], outs[0], t["s1"], outs[1], t["s2"], outs[2], x)
    for w, n, y in zip(ws, rows, outs):
        assert synth.max_rel_err(y, oracle.matvec_q4_0(w, x, n, threads=8)) < TOL


def test_prefetch_hint_changes_nothing_but_timing(lib):
    """The one-shot L2 prefetch hint is consumed by the next launch and does not
    change its result; a host pointer that is neither registered nor device
    memory is refused."""
    import torch
    from aljabr_b200.native import ProviderError
    N, K = 4096, 4096
    w = synth.q4_0(70, N, K)
    x = synth.activation(71, K)
    plain = _dev_matvec(lib, w, x, K, N)
    nxt = torch.from_numpy(synth.q4_0(72, 14336, K)).cuda()
    torch.cuda.synchronize()
    lib.call("aljabr_blackwell_prefetch_hint", nxt.data_ptr(), nxt.numel())
    hinted = _dev_matvec(lib, w, x, K, N)
    np.testing.assert_array_equal(hinted, plain)
    host = np.zeros(1024, np.uint8)
    with pytest.raises(ProviderError):
        lib.call("aljabr_blackwell_prefetch_hint", host.ctypes.data, host.nbytes)
    lib.call("aljabr_blackwell_prefetch_hint", None, 0)


def _dev_matvec_q8(lib, w, x, K, N):
    import torch
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    dy = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()   # inputs from torch's stream; the library's own stream is non-blocking
    lib.call("aljabr_blackwell_matvec_dev", lib.TYPE_Q8_0, dy.data_ptr(), dx.data_ptr(), dw.data_ptr(), None,
             K, N, 0, None, None)
    torch.cuda.synchronize()
    return dy.cpu().numpy()


@pytest.mark.parametrize("N", [4, 12, 36, 596, 2380])
@pytest.mark.parametrize("K", [2048, 6144])
def test_q8_0_ragged_rows(lib, N, K):
    w = synth.q8_0(500 + N, N, K)
    x = synth.activation(600 + K, K)
    y = _dev_matvec_q8(lib, w, x, K, N)
    assert synth.max_rel_err(y, oracle.matvec_q8_0(w, x, N, threads=8)) < TOL
    assert synth.max_rel_err(y, oracle.matvec_f64(oracle.Q8_0, w, x, N, threads=8)) < TOL


@pytest.mark.parametrize("scale", [1.0, 3e4, 1e-6])
def test_q8_0_activation_outliers_and_scales(lib, scale):
    N, K = 1024, 8192
    w = synth.q8_0(17, N, K)
    x = synth.activation(18, K) * np.float32(scale)
    x[5::97] *= 50.0
    x[:32] = 0.0
    y = _dev_matvec_q8(lib, w, x, K, N)
    assert synth.max_rel_err(y, oracle.matvec_q8_0(w, x, N, threads=8)) < TOL
