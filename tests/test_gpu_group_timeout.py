"""The bounded waits of the expert-parallel MoE group and of the
tensor-parallel decoder run out when a rank never calls, and are reported.

Rank 1 of each two-rank group lives in a child process on the same GPU: it
creates its group, hands over its mailbox handle and then launches nothing.
Rank 0 (this process) runs a call with a 20 ms wait limit; its exchange
waits on rank 1's flag, which nothing sets, gives up, and the call's
mxq_synchronize reports MXQ_ERR_TIMEOUT.  Only rank 0's kernel ever waits,
and on a flag no kernel sets; the context stays usable afterwards.
"""
import os
import sys

import numpy as np
import pytest
import torch

from cpu_model_b200 import _lib, mx, synth

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import shard_workers  # noqa: E402

pytestmark = pytest.mark.gpu
DEC = dict(n_layers=2, d_model=256, n_heads=2, ffn=512, vocab=1000, fmt=4, max_batch=2, max_ctx=64, max_rows=128)


def idle_peer(kind, args):
    mpc = torch.multiprocessing.get_context("spawn")
    q, done = mpc.Queue(), mpc.Event()
    p = mpc.Process(target=shard_workers.idle_rank_worker, args=(kind, args, q, done))
    p.start()
    return p, q.get(timeout=180), done


def finish(p, done):
    done.set()
    p.join(timeout=60)
    if p.is_alive():
        p.kill()


def test_moe_group_wait_runs_out_and_context_recovers(ctx):
    t, d, f, e, k = 64, 256, 512, 4, 2
    p, peer_handle, done = idle_peer("moe", (t, k, d))
    experts = shard_workers.moe_experts_dev(ctx, 4, e, d, f, 0.25, 1300)
    g, u, dn = ([m[i] for m in experts] for i in range(3))
    G = mx.MoEGroup(0, 2, t, k, d, ctx)
    try:
        G.connect([G.handle(), peer_handle])
        G.set_wait_limit(20000)
        x = torch.from_numpy(synth.normal((t, d), 3)).cuda()
        logits = torch.from_numpy(synth.normal((t, e), 4)).cuda()
        G.moe_swiglu(x, logits, g[:2], u[:2], dn[:2], k)
        with pytest.raises(_lib.MXError) as err:
            ctx.synchronize()
        assert err.value.code == _lib.MXQ_ERR_TIMEOUT
        # the context still computes correctly
        y1 = mx.moe_swiglu(x, logits, g, u, dn, k, ctx).cpu().numpy()
        y2 = mx.moe_swiglu(x, logits, g, u, dn, k, ctx).cpu().numpy()
        ctx.synchronize()
        assert np.array_equal(y1, y2) and np.linalg.norm(y1) > 0
    finally:
        G.close()
        finish(p, done)
        for m in experts:
            for W in m:
                W.close()


def test_sharded_decoder_wait_runs_out_and_context_recovers(ctx):
    p, peer_handle, done = idle_peer("decoder", DEC)
    D = mx.Decoder(seed=5, ctx=ctx, rank=0, world=2, **DEC)
    try:
        D.connect([D.handle(), peer_handle])
        D.set_wait_limit(20000)
        D.prefill(torch.zeros((1, 3), dtype=torch.int32, device="cuda"))
        with pytest.raises(_lib.MXError) as err:
            ctx.synchronize()
        assert err.value.code == _lib.MXQ_ERR_TIMEOUT
        plain = mx.Decoder(seed=5, ctx=ctx, **DEC)
        try:
            a = plain.prefill(torch.ones((1, 3), dtype=torch.int32, device="cuda")).cpu().numpy()
            ctx.synchronize()
            assert np.isfinite(a).all()
        finally:
            plain.close()
    finally:
        D.close()
        finish(p, done)
