"""The tensor-parallel decoder (mxq_decoder_create_sharded): each rank holds
its heads (q/k/v rows, K/V cache, attention) and FFN units (gate/up rows),
and the O and down columns of both; two peer exchanges a layer bring every
rank's partial sums into every mailbox, added in rank order by the residual.

- one rank (the sharded code path on one GPU, exchanging through its own
  mailbox): prompt logits, decode steps (batch 2 and batch 1, both
  graph-replayed) and scored log-probs bit-identical to the unsharded
  decoder of the same seed, at a small shape and at the 7B layer shape;
- every rank's weights are exactly the unsharded weights' bytes for that
  rank (heads' q/k/v rows, gate and up rows, O and down columns); the head
  is whole;
- bad groups are refused, and a pass before connect() is refused;
- two ranks on two GPUs (skipped with fewer): both ranks return the same
  logits, within 1e-5 of the unsharded decoder on one GPU (the block sums
  of O and down are added in another fp32 order).
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch

from cpu_model_b200 import mx

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import shard_workers  # noqa: E402

pytestmark = pytest.mark.gpu
REL_TOL = 1e-5
CFG = dict(n_layers=2, d_model=256, n_heads=2, ffn=512, vocab=1000, fmt=4, max_batch=2, max_ctx=64, max_rows=128)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def toks(rng, vocab, *shape):
    return torch.from_numpy(rng.integers(0, vocab, shape, dtype=np.int32)).cuda()


def passes(dec, vocab, b, steps=4, seed=17):
    rng = np.random.default_rng(seed)
    out = [dec.prefill(toks(rng, vocab, b, 5)).cpu().numpy()]
    for _ in range(steps):
        out.append(dec.decode(toks(rng, vocab, b)).cpu().numpy())
    dec.reset()
    one = [dec.prefill(toks(rng, vocab, 1, 3)).cpu().numpy()]
    for _ in range(steps):
        one.append(dec.decode(toks(rng, vocab, 1)).cpu().numpy())
    dec.reset()
    logp, _ = dec.score(toks(rng, vocab, b, 8))
    return out, one, logp.cpu().numpy()


def one_rank(ctx, cfg, seed):
    d = mx.Decoder(seed=seed, ctx=ctx, rank=0, world=1, **cfg)
    d.connect([d.handle()])
    return d


@pytest.mark.parametrize("fmt", [4, 8])
def test_one_rank_sharded_decoder_is_bit_identical(ctx, fmt):
    cfg = dict(CFG, fmt=fmt)
    plain = mx.Decoder(seed=5, ctx=ctx, **cfg)
    tp = one_rank(ctx, cfg, 5)
    try:
        a, b = passes(plain, cfg["vocab"], 2), passes(tp, cfg["vocab"], 2)
        for x, y in zip(a[0] + a[1], b[0] + b[1]):
            assert np.array_equal(x, y)
        assert np.array_equal(a[2], b[2])
        assert all(np.isfinite(x).all() for x in b[0] + b[1])
    finally:
        tp.close()
        plain.close()


def test_one_rank_sharded_decoder_7b_layer_shape(ctx):
    cfg = dict(n_layers=1, d_model=4096, n_heads=32, ffn=11008, vocab=32000, fmt=4, max_batch=1, max_ctx=16,
               max_rows=16)
    plain = mx.Decoder(seed=3, ctx=ctx, **cfg)
    tp = one_rank(ctx, cfg, 3)
    try:
        rng = np.random.default_rng(2)
        prompt = toks(rng, 32000, 1, 4)
        assert np.array_equal(plain.prefill(prompt).cpu().numpy(), tp.prefill(prompt).cpu().numpy())
        for _ in range(3):
            t = toks(rng, 32000, 1)
            assert np.array_equal(plain.decode(t).cpu().numpy(), tp.decode(t).cpu().numpy())
    finally:
        tp.close()
        plain.close()


@pytest.mark.parametrize("world,cfg", [(2, CFG), (4, dict(CFG, d_model=512, n_heads=4, ffn=1024))])
def test_rank_weights_are_rows_of_the_unsharded_weights(ctx, world, cfg):
    plain = mx.Decoder(seed=9, ctx=ctx, **cfg)
    d, f = cfg["d_model"], cfg["ffn"]
    dl, fl = d // world, f // world
    try:
        for rank in range(world):
            sh = mx.Decoder(seed=9, ctx=ctx, rank=rank, world=world, **cfg)
            try:
                per = 2 if cfg["fmt"] == 4 else 1          # elements a data byte
                for layer in range(cfg["n_layers"]):
                    for which, rows in [
                        (mx.DEC_QKV, [np.arange(rank * dl, (rank + 1) * dl) + j * d for j in range(3)]),
                        (mx.DEC_GATE_UP, [np.arange(rank * fl, (rank + 1) * fl) + j * f for j in range(2)]),
                    ]:
                        full_d, full_s = plain.download(layer, which)
                        got_d, got_s = sh.download(layer, which)
                        idx = np.concatenate(rows)
                        assert np.array_equal(got_d, full_d[idx]) and np.array_equal(got_s, full_s[idx])
                    for which, c0, n in [(mx.DEC_O, rank * dl, dl), (mx.DEC_DOWN, rank * fl, fl)]:
                        full_d, full_s = plain.download(layer, which)
                        got_d, got_s = sh.download(layer, which)
                        assert np.array_equal(got_d, full_d[:, c0 // per:(c0 + n) // per])
                        assert np.array_equal(got_s, full_s[:, c0 // 32:(c0 + n) // 32])
                hd, hs = plain.download(0, mx.DEC_LM_HEAD)
                gd, gs = sh.download(0, mx.DEC_LM_HEAD)
                assert np.array_equal(gd, hd) and np.array_equal(gs, hs)
                # a pass before connect() is refused (no kernel runs)
                with pytest.raises(ValueError, match="not connected"):
                    sh.prefill(torch.zeros((1, 2), dtype=torch.int32, device="cuda"))
            finally:
                sh.close()
    finally:
        plain.close()


@pytest.mark.parametrize("world", [4, 8])
def test_7b_rank_shard_shapes_in_every_regime(ctx, world):
    """The linears a rank of a 4- or 8-GPU 7B decoder runs -- QKV and gate|up
    rows, O and down columns (K = 4096 / world and 11008 / world, the
    latter an odd number of 32-blocks at 8 GPUs) -- through the batch-1,
    small-batch and tensor-core paths, against the oracle."""
    from oracle import oracle
    from cpu_model_b200 import synth
    d, f = 4096, 11008
    shapes = [(3 * d // world, d), (d, d // world), (2 * f // world, d), (d, f // world)]
    for i, (n, k) in enumerate(shapes):
        w, ws = synth.weights(4, n, k, -8, -3, 60 + i)
        W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), 4, n, k, ctx)
        try:
            for b in (1, 8, 32, 130):
                x = synth.normal((b, k), 70 + b)
                xq, xs = oracle.quantize_x(x)
                ref = oracle.gemv(4, xq, xs, w, ws, n, k)
                y = mx.mx_linear(torch.from_numpy(x).cuda(), W, ctx).cpu().numpy()
                assert rel_l2(y, ref) <= REL_TOL, (n, k, b)
                if b == 1:      # the MX-input GEMV the batch-1 down projection runs
                    a = mx.mx_quantize_x(torch.from_numpy(x).cuda(), ctx)
                    y = mx.mx_gemv(a, W, ctx).cpu().numpy()
                    assert rel_l2(y, ref) <= REL_TOL, (n, k, "mx")
        finally:
            W.close()


@pytest.mark.parametrize("rank,world,cfg", [
    (0, 3, CFG),                                                # 3 does not divide 2 heads
    (2, 2, CFG),                                                # rank out of range
    (0, 9, dict(CFG, d_model=1152, n_heads=9, ffn=2304)),       # more than 8 ranks
    (0, 4, dict(CFG, d_model=512, n_heads=4, ffn=576)),         # 144 FFN columns a rank: not whole 32-blocks
])
def test_bad_groups_are_refused(ctx, rank, world, cfg):
    with pytest.raises(ValueError):
        mx.Decoder(seed=1, ctx=ctx, rank=rank, world=world, **cfg)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fmt", [4, 8])
def test_two_rank_decoder(tmp_path, fmt):
    world, steps = 2, 4
    cfg = dict(CFG, fmt=fmt)
    mpc = torch.multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [mpc.Process(target=shard_workers.decoder_tp_worker,
                         args=(r, world, port, cfg, 11, steps, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0, p.exitcode
    res = [np.load(os.path.join(tmp_path, "dec_%d.npz" % r)) for r in range(world)]
    for r in range(world):
        for key in ("outs", "one", "logp"):
            assert np.array_equal(res[r][key], res[0][key])          # every rank returns the same
            assert rel_l2(res[r][key], res[r]["ref_" + key]) <= REL_TOL, key
            assert np.isfinite(res[r][key]).all()
