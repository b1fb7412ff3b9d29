"""GPU parity for the PPO rollout forward drop-in (training/ppo_trainer.cpp
:57-66, :77): the policy head kernel and the three-linear MX forward through
libmxq.so, against the CPU oracle on the same seeded inputs (relative L2
<= 1e-5)."""
import numpy as np
import pytest
import torch

from oracle import oracle
from cpu_model_b200 import mx, synth

pytestmark = pytest.mark.gpu

REL_TOL = 1e-5


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


@pytest.mark.parametrize("rows,cols", [(1000, 80), (5, 3), (7, 1000), (1, 1)])
def test_policy_head_matches_oracle(ctx, rows, cols):
    g = synth.rng(rows + cols)
    logits = (g.standard_normal((rows, cols)) * 4).astype(np.float32)
    actions = g.random((rows, cols)).astype(np.float32)
    lp0, alp0, ent0 = oracle.policy_head(logits, actions)
    lp, alp, ent = mx.policy_head(cuda(logits), cuda(actions), ctx)
    assert rel_l2(host(lp), lp0) <= REL_TOL
    assert rel_l2(host(alp), alp0) <= REL_TOL
    assert rel_l2(host(ent), ent0) <= REL_TOL or np.abs(host(ent) - ent0).max() < 1e-5


def test_ppo_rollout_forward_reference_shapes(ctx):
    """States [R][1616] -> latent 2048 -> 80 logits and a value, MX-int8
    weights (the 1616-feature states are zero-padded to K = 1632)."""
    r, s, d, a = 64, 1616, 2048, 80
    kp = 1632
    wp, sp = synth.weights(8, d, kp, -9, -5, 1)
    wpi, spi = synth.weights(8, a, d, -9, -5, 2)
    wv, sv = synth.weights(8, 1, d, -9, -5, 3)
    Wp = mx.MXWeight(torch.from_numpy(wp), torch.from_numpy(sp), 8, d, kp, ctx)
    Wpi = mx.MXWeight(torch.from_numpy(wpi), torch.from_numpy(spi), 8, a, d, ctx)
    Wv = mx.MXWeight(torch.from_numpy(wv), torch.from_numpy(sv), 8, 1, d, ctx)
    states = synth.normal((r, s), 4)
    actions = np.eye(a, dtype=np.float32)[synth.rng(5).integers(0, a, r)]
    lp, alp, ent, val = mx.ppo_rollout_forward(cuda(states), cuda(actions), Wp, Wpi, Wv, ctx)
    # oracle: the same chain on the host
    sq, ss = oracle.quantize_x(np.pad(states, ((0, 0), (0, kp - s))))
    latent = oracle.gemv(8, sq, ss, wp, sp, d, kp)
    # the GPU's latent feeds the next linears: compare stage by stage on it
    lat_gpu = host(mx.mx_linear(torch.nn.functional.pad(cuda(states), (0, kp - s)), Wp, ctx))
    assert rel_l2(lat_gpu, latent) <= REL_TOL
    lq, ls = oracle.quantize_x(lat_gpu)
    logits = oracle.gemv(8, lq, ls, wpi, spi, a, d)
    values = oracle.gemv(8, lq, ls, wv, sv, 1, d)[:, 0]
    lp0, alp0, ent0 = oracle.policy_head(logits, actions)
    assert rel_l2(host(val), values) <= REL_TOL
    assert rel_l2(host(lp), lp0) <= REL_TOL
    assert rel_l2(host(alp), alp0) <= REL_TOL
    assert rel_l2(host(ent), ent0) <= REL_TOL
    # one combined [81][2048] head: the latent quantised once, same results
    Wh = mx.MXWeight(torch.from_numpy(np.concatenate([wpi, wv])), torch.from_numpy(np.concatenate([spi, sv])),
                     8, a + 1, d, ctx)
    lp2, alp2, ent2, val2 = mx.ppo_rollout_forward(cuda(states), cuda(actions), Wp, Wh, None, ctx)
    assert rel_l2(host(lp2), host(lp)) <= 1e-6 and rel_l2(host(val2), host(val)) <= 1e-6
    assert rel_l2(host(alp2), host(alp)) <= 1e-6 and rel_l2(host(ent2), host(ent)) <= 1e-6
    for w in (Wp, Wpi, Wv, Wh):
        w.close()
