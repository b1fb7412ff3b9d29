"""The expert-parallel MoE layer (mxq_moe_group_*, mxq_moe_swiglu_sharded):
each rank runs its own experts on the tokens routed to them, writes the
expert outputs into its mailbox, and one exchange copies them to every other
rank's mailbox over NVLink before the combine.

- one rank (runs on one GPU, the exchange through its own mailbox):
  bit-identical to mxq_moe_swiglu over the same experts, int4 and int8,
  over repeated calls (the mailbox halves alternate), idle experts included;
- bad groups and calls are refused;
- two ranks on two GPUs (skipped with fewer): each rank holding half the
  experts returns y bit-identical to mxq_moe_swiglu over all experts on one
  GPU, on both ranks.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch

from cpu_model_b200 import mx, synth

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import shard_workers  # noqa: E402

pytestmark = pytest.mark.gpu


def one_rank(ctx, t, k, d):
    G = mx.MoEGroup(0, 1, t, k, d, ctx)
    G.connect([G.handle()])
    return G


@pytest.mark.parametrize("fmt", [4, 8])
@pytest.mark.parametrize("t,d,f,e,k", [(48, 256, 512, 4, 2), (130, 128, 256, 8, 2), (300, 512, 1024, 8, 2)])
def test_one_rank_group_matches_moe(ctx, fmt, t, d, f, e, k):
    experts = shard_workers.moe_experts_dev(ctx, fmt, e, d, f, 0.25, 100 + t)
    g, u, dn = ([m[i] for m in experts] for i in range(3))
    G = one_rank(ctx, t, k, d)
    try:
        for i in range(3):
            x = torch.from_numpy(synth.normal((t, d), 7 + i)).cuda()
            logits = torch.from_numpy(synth.normal((t, e), 8 + i)).cuda()
            if i == 2:
                logits[:, 1] -= 100.0            # an idle expert
            ref = mx.moe_swiglu(x, logits, g, u, dn, k, ctx).cpu().numpy()
            y = G.moe_swiglu(x, logits, g, u, dn, k).cpu().numpy()
            assert np.array_equal(y, ref)
            assert np.linalg.norm(ref) > 0
    finally:
        G.close()
        for m in experts:
            for W in m:
                W.close()


def test_bad_groups_and_calls_are_refused(ctx):
    with pytest.raises(ValueError):
        mx.MoEGroup(2, 2, 16, 2, 128, ctx)            # rank out of range
    with pytest.raises(ValueError):
        mx.MoEGroup(0, 9, 16, 2, 128, ctx)            # more than 8 ranks
    with pytest.raises(ValueError):
        mx.MoEGroup(0, 1, 16, 2, 130, ctx)            # d_model not a multiple of 4
    experts = shard_workers.moe_experts_dev(ctx, 4, 2, 128, 256, 0.5, 900)
    g, u, dn = ([m[i] for m in experts] for i in range(3))
    G = one_rank(ctx, 16, 1, 128)
    G2 = mx.MoEGroup(0, 2, 16, 1, 128, ctx)
    try:
        x = torch.from_numpy(synth.normal((32, 128), 1)).cuda()
        logits = torch.from_numpy(synth.normal((32, 2), 2)).cuda()
        with pytest.raises(ValueError, match="routes"):
            G.moe_swiglu(x, logits, g, u, dn, 1)        # 32 tokens x top-1 > 16 routes
        with pytest.raises(ValueError, match="not connected"):
            G2.moe_swiglu(x[:16], logits[:16], g[:1], u[:1], dn[:1], 1)
        ctx.synchronize()
    finally:
        G2.close()
        G.close()
        for m in experts:
            for W in m:
                W.close()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fmt", [4, 8])
def test_two_rank_moe(tmp_path, fmt):
    world, calls = 2, 3
    mpc = torch.multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [mpc.Process(target=shard_workers.moe_ep_worker,
                         args=(r, world, port, fmt, 300, 512, 1024, 8, 2, calls, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0, p.exitcode
    res = [np.load(os.path.join(tmp_path, "moe_%d.npz" % r)) for r in range(world)]
    for r in range(world):
        assert np.array_equal(res[r]["outs"], res[r]["refs"])
        assert np.array_equal(res[r]["outs"], res[0]["outs"])
        assert np.linalg.norm(res[r]["outs"]) > 0
