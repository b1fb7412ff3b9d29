"""GPU parity of the dense decoder on the MX linears (mxq_decoder_*), through
libmxq.so's C-ABI, stage by stage against the oracle on the GPU's own
intermediates (mxq_decoder_set_trace):

  RMSNorm             rel-L2 <= 1e-6 against float64;
  every MX linear     rel-L2 <= 1e-5 against the oracle's exactly rounded
                      gemv on the GPU's quantised input;
  rotary embedding    bit-exact (the same float32 operations, the same table);
  K/V cache           bf16 of the rotated k / v, bit-exact;
  attention           rel-L2 <= 1e-5 against float64 softmax attention over
                      the bf16 cache (prompt and one-token paths);
  logits / log-probs  rel-L2 <= 1e-5 on the GPU's final hidden state.

Plus: decode steps replayed from a CUDA graph are bit-identical to a fresh
run, and the reference's error contract (invalid sizes -> invalid argument).
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from cpu_model_b200 import mx

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, d_model=256, n_heads=2, ffn=512, vocab=1000, fmt=4, max_batch=2, max_ctx=64, max_rows=128)
HD = 128


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return np.linalg.norm(a - b) / (den if den > 0 else 1.0)


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def lin(dec, layer, which, x):
    """The oracle's MX linear on the GPU's fp32 input (quantised bit-exactly)."""
    data, scales = dec.download(layer, which)
    n, k = scales.shape[0], scales.shape[1] * 32
    xq, xs = oracle.quantize_x(x)
    return oracle.gemv(dec.cfg.fmt, xq, xs, data, scales, n, k)


def tokens(b, t, seed, vocab=1000):
    return np.random.default_rng(seed).integers(0, vocab, size=(b, t), dtype=np.int32)


@pytest.fixture(scope="module")
def dec(ctx):
    d = mx.Decoder(seed=5, ctx=ctx, **CFG)
    yield d
    d.close()


def check_layer(dec, layer, tr, B, T, pos0, cos, sin, kv):
    """Stage-wise check of one traced layer; kv = (k, v) bf16 of every cached
    position before this pass, [B][P][H][hd] (P = pos0)."""
    d, H, F = dec.cfg.d_model, dec.cfg.n_heads, dec.cfg.ffn
    R = B * T
    assert rel_l2(tr["norm1"], oracle.rmsnorm(tr["in"], np.ones(d), dec.cfg.norm_eps)) <= 1e-6
    assert rel_l2(tr["qkv"], lin(dec, layer, mx.DEC_QKV, tr["norm1"])) <= 1e-5
    qkv = tr["qkv"].reshape(B, T, 3, H, HD)
    pos = pos0 + np.arange(T)
    qrot = oracle.rope_rotate(qkv[:, :, 0], np.broadcast_to(pos, (B, T)), cos, sin)
    assert np.array_equal(tr["rope"].reshape(B, T, 3, H, HD)[:, :, 0], qrot)
    krot = oracle.bf16_round(oracle.rope_rotate(qkv[:, :, 1], np.broadcast_to(pos, (B, T)), cos, sin))
    vb = oracle.bf16_round(qkv[:, :, 2])
    att = np.concatenate([oracle.attention(qrot[b], np.concatenate([kv[0][b], krot[b]]),
                                           np.concatenate([kv[1][b], vb[b]]), pos) for b in range(B)])
    assert rel_l2(tr["att"], att) <= 1e-5
    assert rel_l2(tr["h1"], tr["in"] + lin(dec, layer, mx.DEC_O, tr["att"])) <= 1e-5
    assert rel_l2(tr["norm2"], oracle.rmsnorm(tr["h1"], np.ones(d), dec.cfg.norm_eps)) <= 1e-6
    assert rel_l2(tr["gu"], lin(dec, layer, mx.DEC_GATE_UP, tr["norm2"])) <= 1e-5
    hq, hs = oracle.swiglu_quantize(tr["gu"][:, :F], tr["gu"][:, F:])
    data, scales = dec.download(layer, mx.DEC_DOWN)
    down = oracle.gemv(dec.cfg.fmt, hq, hs, data, scales, d, F)
    assert rel_l2(tr["out"], tr["h1"] + down) <= 1e-5
    return krot, vb


def traces(dec, R):
    d, F = dec.cfg.d_model, dec.cfg.ffn
    shapes = {"in": (R, d), "norm1": (R, d), "qkv": (R, 3 * d), "rope": (R, 3 * d), "att": (R, d), "h1": (R, d),
              "norm2": (R, d), "gu": (R, 2 * F), "out": (R, d)}
    return {k: dec.get_trace(k, s) for k, s in shapes.items()}


def test_prefill_stagewise_and_logits(dec):
    B, T = 2, 40
    tok = tokens(B, T, 1)
    cos, sin = oracle.rope_table(CFG["max_ctx"], 10000.0)
    for layer in range(CFG["n_layers"]):
        dec.reset()
        dec.set_trace(layer)
        dec.prefill(cuda(tok))
        empty = np.zeros((B, 0, CFG["n_heads"], HD), np.float32)
        check_layer(dec, layer, traces(dec, B * T), B, T, 0, cos, sin, (empty, empty))
    # the head on the GPU's final hidden state (last token of each sequence)
    dec.reset()
    dec.set_trace(CFG["n_layers"])
    logits = host(dec.prefill(cuda(tok)))
    dec.set_trace(-1)
    h = dec.get_trace("in", (B * T, CFG["d_model"]))[T - 1::T]
    hn = oracle.rmsnorm(h, np.ones(CFG["d_model"]), 1e-5)
    assert rel_l2(logits, lin(dec, 0, mx.DEC_LM_HEAD, hn)) <= 1e-5
    assert dec.length() == T


def test_decode_stagewise_attention(dec):
    """One-token attention over the cache (the prompt's keys plus its own)."""
    B, T = 2, 50
    tok = tokens(B, T + 1, 2)
    cos, sin = oracle.rope_table(CFG["max_ctx"], 10000.0)
    d, H = CFG["d_model"], CFG["n_heads"]
    dec.reset()
    dec.set_trace(0)
    dec.prefill(cuda(tok[:, :T]))
    qkv = dec.get_trace("qkv", (B * T, 3 * d)).reshape(B, T, 3, H, HD)
    pos = np.broadcast_to(np.arange(T), (B, T))
    kc = oracle.bf16_round(oracle.rope_rotate(qkv[:, :, 1], pos, cos, sin))
    vc = oracle.bf16_round(qkv[:, :, 2])
    dec.decode(cuda(tok[:, T].copy()))
    check_layer(dec, 0, traces(dec, B), B, 1, T, cos, sin, (kc, vc))
    dec.set_trace(-1)
    assert dec.length() == T + 1


def test_decode_graph_replay_is_deterministic(dec):
    B, T, steps = 2, 20, 6
    tok = tokens(B, T + steps, 3)
    runs = []
    for _ in range(2):
        dec.reset()
        dec.prefill(cuda(tok[:, :T]))
        outs = [host(dec.decode(cuda(tok[:, T + i].copy()))) for i in range(steps)]
        runs.append(np.stack(outs))
    assert np.all(np.isfinite(runs[0]))
    assert np.array_equal(runs[0], runs[1])


def test_decode_agrees_with_longer_prefill(dec):
    """The next-token logits from the one-token path and from a prompt one
    token longer: different kernels (GEMV vs GEMM sums, the two attention
    paths), so close but not bit-identical."""
    B, T = 2, 30
    tok = tokens(B, T + 1, 4)
    dec.reset()
    dec.prefill(cuda(tok[:, :T]))
    a = host(dec.decode(cuda(tok[:, T].copy())))
    dec.reset()
    b = host(dec.prefill(cuda(tok)))
    assert rel_l2(a, b) <= 2e-2


def test_score_logprobs_and_values(ctx):
    D = mx.Decoder(seed=9, ctx=ctx, value_head=True, **CFG)
    B, T = 2, 48
    tok = tokens(B, T, 5)
    D.set_trace(CFG["n_layers"])
    logp, values = D.score(cuda(tok))
    logp, values = host(logp), host(values)
    D.set_trace(-1)
    h = D.get_trace("in", (B * T, CFG["d_model"]))
    hn = oracle.rmsnorm(h, np.ones(CFG["d_model"]), 1e-5)
    logits = lin(D, 0, mx.DEC_LM_HEAD, hn)                      # [B*T][vocab + 1]
    assert logits.shape[1] == CFG["vocab"] + 1
    tgt = np.concatenate([tok[:, 1:], np.zeros((B, 1), np.int32)], axis=1).ravel()
    ref = oracle.log_softmax_at(logits[:, :CFG["vocab"]], tgt).reshape(B, T)[:, :T - 1]
    assert rel_l2(logp, ref) <= 1e-5
    assert rel_l2(values, logits[:, CFG["vocab"]].reshape(B, T)) <= 1e-5
    # more sequences than one pass holds: shapes and finiteness
    lp3, v3 = D.score(cuda(tokens(5, T, 6)))
    assert host(lp3).shape == (5, T - 1) and np.all(np.isfinite(host(lp3))) and np.all(np.isfinite(host(v3)))
    D.close()


def test_decoder_errors(dec, ctx):
    dec.reset()
    with pytest.raises(ValueError):                  # batch above max_batch
        dec.prefill(cuda(tokens(3, 4, 7)))
    with pytest.raises(ValueError):                  # prompt longer than the context
        dec.prefill(cuda(tokens(1, CFG["max_ctx"] + 1, 7)))
    dec.prefill(cuda(tokens(1, CFG["max_ctx"], 8)))
    with pytest.raises(ValueError):                  # the context is full
        dec.decode(cuda(np.zeros(1, np.int32)))
    with pytest.raises(ValueError):                  # head dim must be 128
        mx.Decoder(ctx=ctx, **dict(CFG, n_heads=4))
    dec.reset()
    ctx.synchronize()


def test_weight_download_roundtrip(ctx):
    from cpu_model_b200 import synth
    for fmt, n, k in ((4, 300, 448), (8, 129, 96)):
        w, ws = synth.weights(fmt, n, k, -9, -2, 31)
        W = mx.MXWeight(torch.from_numpy(w), torch.from_numpy(ws), fmt, n, k, ctx)
        data = np.empty_like(w)
        sc = np.empty_like(ws)
        mx.check(ctx.lib.mxq_weight_download(W.h, data.ctypes.data_as(mx.ctypes.c_void_p),
                                             sc.ctypes.data_as(mx.ctypes.c_void_p)), ctx.h)
        assert np.array_equal(data, w) and np.array_equal(sc, ws)
        W.close()
