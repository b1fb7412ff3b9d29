"""Rank bodies for the multi-process (gloo, CPU) tests of
cpu_model_b200.shard: the exchange logic runs for real over
torch.distributed, the per-rank compute is the CPU oracle."""
import os

import numpy as np
import torch
import torch.distributed as dist

from oracle import oracle
from cpu_model_b200 import shard, synth


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def oracle_linear(fmt, k):
    def linear(x, w):
        data, scales, n = w
        xq, xs = oracle.quantize_x(x.numpy())
        return torch.from_numpy(oracle.gemv(fmt, xq, xs, data, scales, n, k))
    return linear


def row_slice(fmt, data, scales):
    def fn(lo, hi):
        return (np.ascontiguousarray(data[lo:hi]), np.ascontiguousarray(scales[lo:hi]), hi - lo)
    return fn


def pair_worker(rank, world, port, fmt, b, d, f, outdir):
    _init(rank, world, port)
    wu, su = synth.weights(fmt, f, d, -7, -3, 1)
    wd, sd = synth.weights(fmt, d, f, -7, -3, 2)
    up = shard.ColumnShardedLinear(f, row_slice(fmt, wu, su), oracle_linear(fmt, d))
    down = shard.ColumnShardedLinear(d, row_slice(fmt, wd, sd), oracle_linear(fmt, f))
    x = torch.from_numpy(synth.normal((b, d), 3))
    y = shard.sharded_pair(x, up, down)
    np.save(os.path.join(outdir, "pair_%d.npy" % rank), y.numpy())
    dist.barrier()
    dist.destroy_process_group()


def moe_experts(fmt, e, d, f):
    out = []
    for j in range(e):
        wg, sg = synth.weights(fmt, f, d, -7, -3, 10 + j)
        wu, su = synth.weights(fmt, f, d, -7, -3, 20 + j)
        wd, sd = synth.weights(fmt, d, f, -7, -3, 30 + j)
        mg, md = synth.block_mask(f, d, 0.5, 40 + j), synth.block_mask(d, f, 0.5, 50 + j)
        out.append((synth.apply_block_mask(fmt, wg, mg), sg, synth.apply_block_mask(fmt, wu, mg), su,
                    synth.apply_block_mask(fmt, wd, md), sd))
    return out


def moe_worker(rank, world, port, fmt, t, d, f, e, k, outdir):
    _init(rank, world, port)
    experts = moe_experts(fmt, e, d, f)
    x = synth.normal((t, d), 100 + rank)
    logits = synth.normal((t, e), 200 + rank)
    idx, gate = oracle.route_topk(logits, k)

    def expert_mlp(j, rows):
        wg, sg, wu, su, wd, sd = experts[j]
        return torch.from_numpy(oracle.mlp_swiglu(fmt, rows.numpy(), d, f, wg, sg, wu, su, wd, sd)[0])

    y = shard.moe_expert_parallel(torch.from_numpy(x), torch.from_numpy(idx), torch.from_numpy(gate), e,
                                  expert_mlp)
    np.save(os.path.join(outdir, "moe_%d.npy" % rank), y.numpy())
    dist.barrier()
    dist.destroy_process_group()


def peer_pair_worker(rank, world, port, fmt, k, m, n, steps, outdir):
    """One GPU rank of mxq_linear_pair_sharded: the handles travel over a
    gloo group; the result (every step) and a local re-computation from the
    plain linears on every rank's shard are saved for the parent."""
    from cpu_model_b200 import mx
    _init(rank, world, port)
    torch.cuda.set_device(rank)
    ctx = mx.MXContext(rank)
    w1, s1 = synth.weights(fmt, m, k, -8, -3, 91)
    w2, s2 = synth.weights(fmt, n, m, -8, -3, 92)
    m_s, n_s = m // world, n // world
    W1 = [mx.MXWeight(torch.from_numpy(np.ascontiguousarray(w1[r * m_s:(r + 1) * m_s])),
                      torch.from_numpy(np.ascontiguousarray(s1[r * m_s:(r + 1) * m_s])), fmt, m_s, k, ctx)
          for r in range(world)]
    W2 = [mx.MXWeight(torch.from_numpy(np.ascontiguousarray(w2[r * n_s:(r + 1) * n_s])),
                      torch.from_numpy(np.ascontiguousarray(s2[r * n_s:(r + 1) * n_s])), fmt, n_s, m, ctx)
          for r in range(world)]
    P = mx.PeerGroup(rank, world, m, n, ctx)
    handles = [None] * world
    dist.all_gather_object(handles, P.handle())
    P.connect(handles)
    dist.barrier()
    outs = []
    for i in range(steps):
        x = torch.from_numpy(synth.normal((1, k), 93 + i)).cuda()
        outs.append(P.linear_pair(x, W1[rank], W2[rank]).cpu().numpy())
    # CUDA-graph capture of two calls, replayed twice
    xg = torch.from_numpy(synth.normal((1, k), 99)).cuda()
    yg = torch.empty((1, n), dtype=torch.float32, device="cuda")
    ctx.synchronize()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        P.linear_pair(xg, W1[rank], W2[rank], out=yg)       # warm (sizes workspaces)
        ctx.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            P.linear_pair(xg, W1[rank], W2[rank], out=yg)
            P.linear_pair(xg, W1[rank], W2[rank], out=yg)
    torch.cuda.synchronize()
    graph_outs = []
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        graph_outs.append(yg.cpu().numpy())
    ctx.synchronize()
    del g
    # the same values from the plain linears on every shard
    refs = []
    for i in list(range(steps)) + [None]:
        x = torch.from_numpy(synth.normal((1, k), 93 + i if i is not None else 99)).cuda()
        y1 = torch.cat([mx.mx_linear(x, W1[r], ctx) for r in range(world)], dim=1)
        refs.append(torch.cat([mx.mx_linear(y1, W2[r], ctx) for r in range(world)], dim=1).cpu().numpy())
    ctx.synchronize()
    np.savez(os.path.join(outdir, "peer_%d.npz" % rank), outs=np.stack(outs), graph=np.stack(graph_outs),
             refs=np.stack(refs))
    dist.barrier()
    P.close()
    for w in W1 + W2:
        w.close()
    ctx.close()
    dist.destroy_process_group()


def decoder_tp_worker(rank, world, port, cfg, seed, steps, outdir):
    """One GPU rank of the tensor-parallel decoder: handles over a gloo group;
    a prompt, `steps` decode steps (graph-replayed after the first) and a
    scoring pass, then the same calls on an unsharded decoder of the same
    seed on this GPU; everything saved for the parent."""
    from cpu_model_b200 import mx
    _init(rank, world, port)
    torch.cuda.set_device(rank)
    ctx = mx.MXContext(rank)
    b, vocab = cfg["max_batch"], cfg["vocab"]

    def run(dec):
        rng = np.random.default_rng(17)       # the same tokens on every rank
        outs = [dec.prefill(torch.from_numpy(rng.integers(0, vocab, (b, 5), dtype=np.int32)).cuda()).cpu().numpy()]
        for _ in range(steps):
            tok = torch.from_numpy(rng.integers(0, vocab, (b,), dtype=np.int32)).cuda()
            outs.append(dec.decode(tok).cpu().numpy())
        dec.reset()
        one = [dec.prefill(torch.from_numpy(rng.integers(0, vocab, (1, 3), dtype=np.int32)).cuda()).cpu().numpy()]
        for _ in range(steps):
            one.append(dec.decode(torch.from_numpy(rng.integers(0, vocab, (1,), dtype=np.int32)).cuda()).cpu().numpy())
        dec.reset()
        logp, _ = dec.score(torch.from_numpy(rng.integers(0, vocab, (b, 8), dtype=np.int32)).cuda())
        return np.stack(outs), np.stack(one), logp.cpu().numpy()

    dec = mx.Decoder(seed=seed, ctx=ctx, rank=rank, world=world, **cfg)
    handles = [None] * world
    dist.all_gather_object(handles, dec.handle())
    dec.connect(handles)
    dist.barrier()
    tp = run(dec)
    ctx.synchronize()
    dist.barrier()
    dec.close()
    ref = run(mx.Decoder(seed=seed, ctx=ctx, **cfg))
    np.savez(os.path.join(outdir, "dec_%d.npz" % rank), outs=tp[0], one=tp[1], logp=tp[2],
             ref_outs=ref[0], ref_one=ref[1], ref_logp=ref[2])
    dist.barrier()
    dist.destroy_process_group()


def moe_experts_dev(ctx, fmt, e, d, f, density, seed):
    """E experts (gate [F][D], up [F][D], down [D][F]) of block-sparse MX
    weights from per-expert seeds, as device handles."""
    from cpu_model_b200 import mx
    out = []
    for j in range(e):
        mats = []
        for i, (n, k) in enumerate(((f, d), (f, d), (d, f))):
            w, ws = synth.weights(fmt, n, k, -8, -3, seed + 10 * j + i)
            mask = synth.block_mask(n, k, density, seed + 10 * j + i + 500)
            mats.append(mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx, block_mask=mask))
        out.append(mats)
    return out


def moe_ep_worker(rank, world, port, fmt, t, d, f, e, k, calls, outdir):
    """One GPU rank of mxq_moe_swiglu_sharded: handles over a gloo group; the
    same tokens and logits on every rank; `calls` calls (the mailbox halves
    alternate), then mxq_moe_swiglu over all experts on this GPU."""
    from cpu_model_b200 import mx
    _init(rank, world, port)
    torch.cuda.set_device(rank)
    ctx = mx.MXContext(rank)
    experts = moe_experts_dev(ctx, fmt, e, d, f, 0.25, 700)
    el = e // world
    mine = experts[rank * el:(rank + 1) * el]
    G = mx.MoEGroup(rank, world, t, k, d, ctx)
    handles = [None] * world
    dist.all_gather_object(handles, G.handle())
    G.connect(handles)
    dist.barrier()
    outs = []
    for i in range(calls):
        x = torch.from_numpy(synth.normal((t, d), 31 + i)).cuda()
        logits = torch.from_numpy(synth.normal((t, e), 41 + i)).cuda()
        outs.append(G.moe_swiglu(x, logits, [m[0] for m in mine], [m[1] for m in mine], [m[2] for m in mine],
                                 k).cpu().numpy())
    ctx.synchronize()
    dist.barrier()
    G.close()
    refs = []
    for i in range(calls):
        x = torch.from_numpy(synth.normal((t, d), 31 + i)).cuda()
        logits = torch.from_numpy(synth.normal((t, e), 41 + i)).cuda()
        refs.append(mx.moe_swiglu(x, logits, [m[0] for m in experts], [m[1] for m in experts],
                                  [m[2] for m in experts], k, ctx).cpu().numpy())
    np.savez(os.path.join(outdir, "moe_%d.npz" % rank), outs=np.stack(outs), refs=np.stack(refs))
    dist.barrier()
    dist.destroy_process_group()


def idle_rank_worker(kind, args, q, done):
    """Rank 1 of a two-rank group on this GPU that never calls: it creates
    its group (a MoE group or a sharded decoder), hands its mailbox handle
    to the parent and waits, launching nothing, until the parent is done."""
    from cpu_model_b200 import mx
    ctx = mx.MXContext(0)
    if kind == "moe":
        g = mx.MoEGroup(1, 2, *args, ctx=ctx)
    else:
        g = mx.Decoder(seed=5, ctx=ctx, rank=1, world=2, **args)
    q.put(g.handle())
    done.wait(120)
    g.close()
    ctx.close()
