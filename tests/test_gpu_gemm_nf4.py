"""GPU parity of the tcgen05 batched NF4 linear (AccelOps.linear for M > 1,
engine/safetensor/.../tensor/AccelOps.java:453-456) against the oracle: each
output row m is the reference's fp32 NF4 matvec of token m's bf16
activations.  Covers token counts on and off the 16/32/64/128 token tiles,
several token tiles, ragged weight rows, group 64 and 128, three segments
sharing one input (q/k/v), an output stride wider than the rows, activations
with outliers and extreme scales (the per-token power-of-two scaling), the
stream-K split of long K (partials summed by the last CTA), and bit-identical
repeats.  Tolerance: max element-wise relative error 1e-3 with the
denominator guarded by 1e-3 * max|ref| (also checked against fp64)."""
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


def _bf16(x):
    """Round fp32 to bf16 (nearest-even); returns (bits uint16, values fp32)."""
    bits = oracle.f32_to_bf16_bits(np.ascontiguousarray(x, np.float32))
    return bits, oracle.bf16_bits_to_f32(bits).reshape(x.shape)


def _pack(lib, codes, absmax, rows, K, group):
    import torch
    dc = torch.from_numpy(np.ascontiguousarray(codes)).cuda()
    da = torch.from_numpy(np.ascontiguousarray(absmax, np.float32)).cuda()
    pk = torch.empty(lib.gemm_nf4_packed_size(rows, K, group), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    lib.gemm_nf4_pack(pk.data_ptr(), dc.data_ptr(), da.data_ptr(), rows, K, group)
    torch.cuda.synchronize()
    return pk


def _run(lib, segs, xbits, M, K, group, ldy=None, repeat=1):
    import torch
    rows = [s[2] for s in segs]
    ldy = ldy or rows
    dx = torch.from_numpy(xbits.view(np.int16).reshape(M, K)).cuda()
    pks = [_pack(lib, c, a, r, K, group) for c, a, r in segs]
    dy = [torch.full((M * l,), float("nan"), dtype=torch.float32, device="cuda") for l in ldy]
    ws_bytes = lib.gemm_nf4_workspace_size(M, K, rows)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(repeat):
        torch.cuda.synchronize()
        lib.gemm_nf4_dev([y.data_ptr() for y in dy], ldy, [p.data_ptr() for p in pks],
                         rows, dx.data_ptr(), M, K, group, ws.data_ptr(), ws_bytes)
        torch.cuda.synchronize()
        outs.append([y.cpu().numpy().reshape(M, l)[:, :r].copy() for y, l, r in zip(dy, ldy, rows)])
    st = __import__("ctypes").c_uint(0)
    lib.call("aljabr_blackwell_device_status", __import__("ctypes").byref(st))
    assert st.value == 0, f"device fault word {st.value:#x}"
    return outs if repeat > 1 else outs[0]


def _check(y, ref, tol=TOL):
    """Element-wise bound; on failure name the offending (token, row) pairs."""
    err = synth.max_rel_err(y, ref)
    if not err < tol:
        y64, r64 = np.asarray(y, np.float64), np.asarray(ref, np.float64)
        rel = np.abs(y64 - r64) / np.maximum(np.abs(r64), 1e-3 * np.abs(r64).max())
        bad = np.argwhere(~(rel < tol))
        pts = ", ".join(f"({t},{n}) {y64[t, n]:.4g}/{r64[t, n]:.4g}" for t, n in bad[:8])
        raise AssertionError(f"max rel err {err:.3g}: {len(bad)} bad of {y64.size}, tokens "
                             f"{sorted(set(bad[:, 0].tolist()))[:12]}, row tiles "
                             f"{sorted(set((bad[:, 1] // 128).tolist()))[:12]}; first: {pts}")


def _ref(codes, absmax, xv, n, group):
    return np.stack([oracle.matvec_nf4(codes, absmax, xv[m], n, group, threads=8) for m in range(xv.shape[0])])


def _ref64(codes, absmax, xv, n, group):
    return np.stack([oracle.matvec_f64(oracle.NF4, codes, xv[m], n, absmax=absmax, group_size=group, threads=8)
                     for m in range(xv.shape[0])])


@pytest.mark.parametrize("M", [2, 16, 17, 31, 64, 65, 128, 130, 300])
def test_token_counts(lib, M):
    N, K, g = 256, 2048, 64
    codes, absmax = synth.nf4(11, N, K, g)
    xbits, xv = _bf16(np.random.default_rng(M).normal(0, 1, (M, K)).astype(np.float32))
    (y,) = _run(lib, [(codes, absmax, N)], xbits, M, K, g)
    _check(y, _ref(codes, absmax, xv, N, g))


@pytest.mark.parametrize("N", [1, 100, 129, 1000])
@pytest.mark.parametrize("group", [64, 128])
def test_ragged_rows_and_groups(lib, N, group):
    M, K = 16, 4096
    codes, absmax = synth.nf4(20 + N, N, K, group)
    xbits, xv = _bf16(np.random.default_rng(N).normal(0, 1, (M, K)).astype(np.float32))
    (y,) = _run(lib, [(codes, absmax, N)], xbits, M, K, group)
    _check(y, _ref(codes, absmax, xv, N, group))


def test_three_segments_and_stride(lib):
    M, K, g = 64, 4096, 64
    rows = (512, 128, 128)
    segs = [(*synth.nf4(30 + i, r, K, g), r) for i, r in enumerate(rows)]
    xbits, xv = _bf16(np.random.default_rng(3).normal(0, 1, (M, K)).astype(np.float32))
    ys = _run(lib, segs, xbits, M, K, g, ldy=[r + 64 for r in rows])
    for (c, a, r), y in zip(segs, ys):
        _check(y, _ref(c, a, xv, r, g))


def test_long_k_split_between_ctas(lib):
    """K = 28672 (the 70B down projection) over few tiles: every tile's K
    range is split between CTAs and finished from partials."""
    M, N, K, g = 16, 256, 28672, 64
    codes, absmax = synth.nf4(40, N, K, g)
    xbits, xv = _bf16(np.random.default_rng(4).normal(0, 1, (M, K)).astype(np.float32))
    (y,) = _run(lib, [(codes, absmax, N)], xbits, M, K, g)
    _check(y, _ref(codes, absmax, xv, N, g))
    _check(y, _ref64(codes, absmax, xv, N, g))


@pytest.mark.parametrize("scale", [1.0, 3e4, 1e-6])
def test_activation_outliers_and_scales(lib, scale):
    M, N, K, g = 32, 512, 4096, 64
    codes, absmax = synth.nf4(50, N, K, g)
    x = np.random.default_rng(5).normal(0, 1, (M, K)).astype(np.float32) * np.float32(scale)
    x[:, 5::97] *= 50.0
    x[1] = 0.0                      # an all-zero token
    x[2, :64] = 0.0
    xbits, xv = _bf16(x)
    (y,) = _run(lib, [(codes, absmax, N)], xbits, M, K, g)
    _check(y, _ref(codes, absmax, xv, N, g))
    _check(y, _ref64(codes, absmax, xv, N, g))
    assert np.all(y[1] == 0.0)


def test_negative_scales(lib):
    M, N, K, g = 16, 256, 2048, 64
    codes, absmax = synth.nf4(60, N, K, g)
    absmax = absmax.copy()
    absmax[::3] *= -1.0
    xbits, xv = _bf16(np.random.default_rng(6).normal(0, 1, (M, K)).astype(np.float32))
    (y,) = _run(lib, [(codes, absmax, N)], xbits, M, K, g)
    _check(y, _ref(codes, absmax, xv, N, g))


def test_repeat_calls_are_bit_identical(lib):
    M, N, K, g = 64, 1024, 8192, 64
    codes, absmax = synth.nf4(70, N, K, g)
    xbits, xv = _bf16(np.random.default_rng(7).normal(0, 1, (M, K)).astype(np.float32))
    a, b = _run(lib, [(codes, absmax, N)], xbits, M, K, g, repeat=2)
    np.testing.assert_array_equal(a[0], b[0])
    _check(a[0], _ref(codes, absmax, xv, N, g))


def _pack_ref(codes, absmax, rows, K, group):
    """numpy restatement of the packed layout: per 128-row tile, per 256-column
    unit, 128 rows x 128 code bytes; then per tile, per 16-group slot, 128 rows
    x 16 absmax (zero past the matrix)."""
    tiles, units, ncols = -(-rows // 128), K // 256, K // group
    slots = -(-ncols // 16)
    c = np.zeros((tiles * 128, K // 2), np.uint8)
    c[:rows] = codes.reshape(rows, K // 2)
    pc = c.reshape(tiles, 128, units, 128).transpose(0, 2, 1, 3).ravel()
    a = np.zeros((tiles * 128, slots * 16), np.float32)
    a[:rows, :ncols] = absmax.reshape(rows, ncols)
    pa = a.reshape(tiles, 128, slots, 16).transpose(0, 2, 1, 3).ravel()
    return np.concatenate([pc, pa.view(np.uint8)])


@pytest.mark.parametrize("rows,K,group", [(128, 256, 64), (200, 4096, 64), (77, 2304, 128), (1000, 28672, 64)])
def test_pack_layout(lib, rows, K, group):
    codes, absmax = synth.nf4(80 + rows, rows, K, group)
    pk = _pack(lib, codes, absmax, rows, K, group)
    np.testing.assert_array_equal(pk.cpu().numpy(), _pack_ref(codes, absmax, rows, K, group))


def test_unsupported_shapes_are_refused(lib):
    import torch
    from aljabr_b200.native import UnsupportedOperation, ProviderError
    M, N, K = 4, 128, 200
    z = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    with pytest.raises(UnsupportedOperation):
        lib.gemm_nf4_dev([z.data_ptr()], [N], [z.data_ptr()], [N], z.data_ptr(), M, K, 64,
                         z.data_ptr(), z.numel())
    with pytest.raises(UnsupportedOperation):
        lib.gemm_nf4_packed_size(N, K, 64)
    with pytest.raises(ProviderError):      # workspace too small
        lib.gemm_nf4_dev([z.data_ptr()], [N], [z.data_ptr()], [N], z.data_ptr(), M, 256, 64,
                         z.data_ptr(), 256)


# one rank's TP8 row shard of a Llama-3-70B layer (hidden
# 8192, 64 query heads, 8 KV heads, head_dim 128, FFN 28672): q/k/v = 1024 +
# 128 + 128 rows (one launch, three segments), o = 1024 rows, gate/up = 3584
# + 3584 rows, down = 1024 rows of K = 28672.
C5_SHARDS = {"qkv": ((1024, 128, 128), 8192), "o": ((1024,), 8192), "gate_up": ((3584, 3584), 8192),
             "down": ((1024,), 28672)}


def _ref64_dense(codes, absmax, xv, n, K, group):
    """fp64 X W^T on the bit-exact dequantised weight (DequantizationKernel order)."""
    w = oracle.dequantize_nf4(codes, absmax, n * K, group).reshape(n, K).astype(np.float64)
    return xv.astype(np.float64) @ w.T


@pytest.mark.parametrize("M", [16, 64, 512])
@pytest.mark.parametrize("shard", sorted(C5_SHARDS))
def test_c5_tp8_shard_shapes(lib, shard, M):
    rows, K = C5_SHARDS[shard]
    g = 64
    segs = [(*synth.nf4(900 + 17 * i + K // 1024, r, K, g), r) for i, r in enumerate(rows)]
    xbits, xv = _bf16(np.random.default_rng(M + K).normal(0, 1, (M, K)).astype(np.float32))
    ys = _run(lib, segs, xbits, M, K, g)
    pick = np.unique(np.linspace(0, M - 1, min(M, 8)).astype(int))   # tokens checked in the reference order
    for (c, a, r), y in zip(segs, ys):
        _check(y, _ref64_dense(c, a, xv, r, K, g))
        _check(y[pick], _ref(c, a, xv[pick], r, g))
