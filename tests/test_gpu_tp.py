"""Tensor-parallel decode step on 2 GPUs (one process per GPU, NCCL
all-gather inside the captured graph) against the oracle's unsharded decode
step.  Skipped when fewer than 2 GPUs are visible."""
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _rank_main(rank, world, nccl_id, q, which, exchange):
    os.environ["ALJ_TP_EXCHANGE"] = exchange
    import torch
    torch.cuda.set_device(rank)
    from aljabr_b200 import native
    from aljabr_b200.decode import LlamaNf4Decoder, shard_rows
    from tests.test_gpu_decode import _model
    native.call("aljabr_blackwell_init", rank)
    shape = _shape(which)
    codes, absmax, norms = _model(321, shape)
    dec = LlamaNf4Decoder(shape, tp_world=world, tp_rank=rank, nccl_id=nccl_id)
    H = shape.hidden
    names = ["q", "k", "v", "o", "gate", "up", "down"]
    try:
        for l in range(shape.layers):
            cs, As = [], []
            for i, n in enumerate(names):
                rows, cols = shape.rows(n), shape.cols(n)
                cs.append(shard_rows(codes[7 * l + i], rows, cols, world, rank))
                As.append(shard_rows(absmax[7 * l + i], rows, cols, world, rank))
            dec.register_layer(l, cs, As, norms[2 * l * H:(2 * l + 1) * H], norms[(2 * l + 1) * H:(2 * l + 2) * H])
        L = shape.layers
        dec.register_output(codes[7 * L], absmax[7 * L],
                            shard_rows(codes[7 * L + 1], shape.vocab, H, world, rank),
                            shard_rows(absmax[7 * L + 1], shape.vocab, H, world, rank), norms[2 * L * H:])
        out = []
        for pos, tok in enumerate([3, 77, 900, 5, 5]):
            nxt, logits = dec.step(tok, pos, want_logits=True)
            out.append((nxt, logits))
        q.put((rank, out))
    finally:
        dec.close()


def _shape(which):
    """"small" runs the plain-kernel fallbacks; "wide" has K a multiple of 2048
    everywhere, so each rank's shards run the TMA table kernel."""
    from aljabr_b200.decode import LlamaShape
    if which == "small":
        return LlamaShape(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1024, max_ctx=16,
                          kv_dtype=0)
    return LlamaShape(layers=2, hidden=2048, q_heads=16, kv_heads=4, head_dim=128, ffn=4096, vocab=2048, max_ctx=16,
                      kv_dtype=0)


@pytest.mark.skipif(int(os.environ.get("ALJ_TEST_GPUS", "0")) < 2, reason="needs 2 GPUs (set ALJ_TEST_GPUS=2)")
@pytest.mark.parametrize("which,exchange", [("small", "nccl"), ("wide", "nccl"), ("wide", "p2p")])
def test_tp2_decode_matches_oracle(which, exchange):
    """exchange "p2p" joins the slices with NVLink peer stores from the
    producing kernels (the wide shape runs the table kernel that carries the
    push); "nccl" with ncclAllGather."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("fewer than 2 GPUs")
    from aljabr_b200.decode import nccl_unique_id
    from tests.test_gpu_decode import _cfg, _model
    nid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, nid, q, which, exchange)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    shape = _shape(which)
    codes, absmax, norms = _model(321, shape)
    kc = np.zeros((shape.layers, shape.max_ctx, shape.kv_heads * shape.head_dim), np.float32)
    vc = np.zeros_like(kc)
    for pos, tok in enumerate([3, 77, 900, 5, 5]):
        _, ref = oracle.decode_step_nf4(_cfg(shape), codes, absmax, norms, kc, vc, tok, pos)
        for r in range(2):
            nxt, logits = results[r][pos]
            from tests import synth
            assert synth.max_rel_err(logits, ref) < 1e-3, (r, pos)
            assert nxt == int(np.argmax(ref))
