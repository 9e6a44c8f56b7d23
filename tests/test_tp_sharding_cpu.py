"""Host-side tensor-parallel logic on CPU (gloo, world size 2).

The decode step's TP mode row-shards every matrix (each rank holds a
contiguous row block, codes and absmax alike), computes its slice of each
matvec, and joins the slices with an all-gather in rank order.  These tests
run that data flow with the oracle as the per-rank compute and gloo as the
collective, and check it reproduces the unsharded result -- i.e. that
`shard_rows` cuts the packed NF4 / Q4_0 layouts on the right boundaries and
that rank-order concatenation is the right join."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from aljabr_b200.decode import shard_rows
        g = np.random.default_rng(5)
        N, K, G = 96, 512, 64
        w = g.normal(0, 0.02, size=(N, K)).astype(np.float32)
        x = g.normal(size=K).astype(np.float32)
        codes, absmax = oracle.quantize_nf4(w, G)
        c_r = shard_rows(codes, N, K, world, rank)
        a_r = shard_rows(absmax, N, K, world, rank)
        y_r = oracle.matvec_nf4(c_r, a_r, x, N // world, G)
        parts = [torch.zeros(N // world) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(y_r))
        y_tp = torch.cat(parts).numpy()
        y_full = oracle.matvec_nf4(codes, absmax, x, N, G)

        q4 = oracle.encode_q4_0(w)
        q_r = shard_rows(q4, N, K, world, rank)
        yq_r = oracle.matvec_q4_0(q_r, x, N // world)
        partsq = [torch.zeros(N // world) for _ in range(world)]
        dist.all_gather(partsq, torch.from_numpy(yq_r))
        yq_tp = torch.cat(partsq).numpy()
        yq_full = oracle.matvec_q4_0(q4, x, N)
        if rank == 0:
            result_q.put((y_tp, y_full, yq_tp, yq_full))
    finally:
        dist.destroy_process_group()


def test_row_sharded_matvec_allgather_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        y_tp, y_full, yq_tp, yq_full = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
    for p in procs:
        assert p.exitcode == 0
    np.testing.assert_array_equal(y_tp, y_full)
    np.testing.assert_array_equal(yq_tp, yq_full)


def test_shard_rows_respects_head_blocks():
    from aljabr_b200.decode import LLAMA3_8B, shard_rows
    s = LLAMA3_8B
    world = 8
    rows, cols = s.rows("k"), s.cols("k")
    codes = np.arange(rows * cols // 2, dtype=np.int64).astype(np.uint8)
    # rank r of 8 holds exactly kv head r: rows [r*128, (r+1)*128)
    for r in (0, 3, 7):
        sh = shard_rows(codes, rows, cols, world, r)
        assert sh.size == rows // world * cols // 2
        np.testing.assert_array_equal(sh[:16], codes.reshape(rows, -1)[r * 128, :16])


def test_shard_sizes_cover_every_row():
    from aljabr_b200.decode import shard_rows
    a = np.arange(40 * 6, dtype=np.float32)
    parts = [shard_rows(a, 40, 6, 4, r) for r in range(4)]
    np.testing.assert_array_equal(np.concatenate(parts), a)
    with pytest.raises(ValueError):
        a.reshape(7, -1)


def _gemm_worker(rank, world, port, result_q):
    """Batched NF4 linear row-sharded over `world` gloo ranks: each rank's
    oracle outputs for its row block, joined by tp_gemm.gather_token_rows,
    equal the unsharded outputs for every token."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from aljabr_b200.decode import shard_rows
        from aljabr_b200.tp_gemm import gather_token_rows, shard_extent
        g = np.random.default_rng(9)
        N, K, G, M = 128, 512, 64, 5
        w = g.normal(0, 0.02, size=(N, K)).astype(np.float32)
        x = g.normal(size=(M, K)).astype(np.float32)
        codes, absmax = oracle.quantize_nf4(w, G)
        row0, rows = shard_extent(N, world, rank)
        c_r = shard_rows(codes, N, K, world, rank)
        a_r = shard_rows(absmax, N, K, world, rank)
        y_r = np.stack([oracle.matvec_nf4(c_r, a_r, x[m], rows, G) for m in range(M)])
        y_tp = gather_token_rows(torch.from_numpy(y_r), world).numpy()
        y_full = np.stack([oracle.matvec_nf4(codes, absmax, x[m], N, G) for m in range(M)])
        ok = y_tp.shape == (M, N) and np.array_equal(y_tp, y_full) and row0 == rank * (N // world)
        result_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_batched_gather_reproduces_unsharded_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29640 + os.getpid() % 200
    procs = [ctx.Process(target=_gemm_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
