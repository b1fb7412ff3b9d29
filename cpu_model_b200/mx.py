"""Host-side mirror of the reference's nca::linalg MX operator interface.

The reference's removed core/linalg/mx_linear.hpp exposed free functions over
MXUINT8Tensor (activations) and MXINT8Tensor (weights) containers
(nn/tests/autotest.hpp:93-136; names in nn/tests/test_auto_generated.cpp:
41-56).  The same names are provided here over torch CUDA tensors, each one a
thin call into libmxq.so (include/mxq.h).  Shape errors raise ValueError, the
Python counterpart of the reference's std::invalid_argument.

torch is used only as the device-memory and stream carrier; all arithmetic
runs in the library's sm_100a kernels.
"""
import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import ACT_NONE, ACT_SILU, FMT_INT4, FMT_INT8, PATH_AUTO, PATH_GEMM, PATH_GEMV, check

__all__ = [
    "MXContext", "MXWeight", "MXActivation", "context",
    "mx_quantize_x", "mx_fused_silu_quantize_x", "fused_gated_silu_quantize",
    "mx_gemv", "mx_dot", "mx_dual_dot", "mx_quad_dot", "mx_rank16_dot",
    "mx_rank16_dot_ptrs", "mx_block_dots", "mx_linear", "mx_linear_pair",
    "gated_mlp_step", "route_topk", "HashedRouter", "HaltingState", "halting_step", "mx_quantize_w",
    "fused_compute_gae", "fused_compute_gae_ring",
    "FMT_INT4", "FMT_INT8", "PATH_AUTO", "PATH_GEMV", "PATH_GEMM",
]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _need_cuda(t, dtype, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError("%s must be a CUDA tensor" % name)
    if t.dtype != dtype:
        raise ValueError("%s must be %s, got %s" % (name, dtype, t.dtype))
    if not t.is_contiguous():
        raise ValueError("%s must be contiguous" % name)


class MXContext:
    """One library context per device; work goes to torch's current stream."""

    def __init__(self, device=0):
        self.lib = _lib.load()
        self.device = device
        h = ctypes.c_void_p()
        check(self.lib.mxq_create(device, ctypes.byref(h)))
        self.h = h

    def _bind(self):
        s = torch.cuda.current_stream(self.device).cuda_stream
        check(self.lib.mxq_set_stream(self.h, ctypes.c_void_p(s)), self.h)

    def set_path(self, path):
        check(self.lib.mxq_set_path(self.h, path), self.h)

    def reserve(self, max_batch, max_k):
        check(self.lib.mxq_reserve(self.h, max_batch, max_k), self.h)

    def synchronize(self):
        self._bind()
        check(self.lib.mxq_synchronize(self.h), self.h)

    def launch_count(self):
        v = ctypes.c_uint64()
        check(self.lib.mxq_launch_count(self.h, ctypes.byref(v)), self.h)
        return v.value

    def close(self):
        if getattr(self, "h", None):
            self.lib.mxq_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_contexts = {}


def context(device=None):
    """The default per-device context (created on first use)."""
    if device is None:
        device = torch.cuda.current_device()
    if device not in _contexts:
        _contexts[device] = MXContext(device)
    return _contexts[device]


@dataclass
class MXActivation:
    """MXUINT8Tensor: q = u8 (value + 128) [B][K], s = E8M0 [B][K/32]."""
    q: torch.Tensor
    s: torch.Tensor

    @property
    def batch(self):
        return self.q.shape[0]

    @property
    def k(self):
        return self.q.shape[1]


class MXWeight:
    """MXINT8Tensor (int8 [N][K] or int4 packed [N][K/2]) + E8M0 scales
    [N][K/32], uploaded once into the library's tiled device layout."""

    def __init__(self, data, scales, fmt, n, k, ctx=None, block_mask=None):
        """block_mask (optional): host uint8 [ceil(n/64)][k/64], nonzero =
        64x64 block present; the weight is then stored block-sparse
        (mxq_weight_create_bsr) and masked-out blocks read as zero."""
        self.ctx = ctx or context()
        self.fmt, self.n, self.k = fmt, n, k
        self.block_sparse = block_mask is not None
        data = torch.as_tensor(data)
        scales = torch.as_tensor(scales)
        exp_bytes = n * k // (2 if fmt == FMT_INT4 else 1)
        if data.numel() * data.element_size() != exp_bytes:
            raise ValueError("weight data has %d bytes, expected %d" % (data.numel() * data.element_size(), exp_bytes))
        if scales.numel() != n * k // 32:
            raise ValueError("weight scales have %d entries, expected %d" % (scales.numel(), n * k // 32))
        data = data.contiguous()
        scales = scales.contiguous()
        on_dev = 1 if data.is_cuda else 0
        if data.is_cuda != scales.is_cuda:
            raise ValueError("data and scales must both be host or both be device tensors")
        h = ctypes.c_void_p()
        self.ctx._bind()
        if block_mask is None:
            check(self.ctx.lib.mxq_weight_create(self.ctx.h, fmt, n, k, _ptr(data), _ptr(scales), on_dev,
                                                 ctypes.byref(h)), self.ctx.h)
        else:
            mask = torch.as_tensor(block_mask).to(torch.uint8).contiguous().cpu()
            if mask.numel() != ((n + 63) // 64) * (k // 64):
                raise ValueError("block mask has %d entries, expected %d" % (mask.numel(), ((n + 63) // 64) * (k // 64)))
            check(self.ctx.lib.mxq_weight_create_bsr(self.ctx.h, fmt, n, k, _ptr(data), _ptr(scales), _ptr(mask),
                                                     on_dev, ctypes.byref(h)), self.ctx.h)
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.mxq_weight_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def download(self):
        """(data, scales) in the MXINT8Tensor layout (numpy); dense only."""
        import numpy as np
        data = np.empty((self.n, self.k // 2), np.uint8) if self.fmt == FMT_INT4 else \
            np.empty((self.n, self.k), np.int8)
        scales = np.empty((self.n, self.k // 32), np.uint8)
        check(self.ctx.lib.mxq_weight_download(self.h, data.ctypes.data_as(ctypes.c_void_p),
                                               scales.ctypes.data_as(ctypes.c_void_p)), self.ctx.h)
        return data, scales

    def save(self, path):
        """Write the weight as an MXQW file (mxq_weight_save)."""
        check(self.ctx.lib.mxq_weight_save(self.h, str(path).encode()), self.ctx.h)

    @classmethod
    def load(cls, path, ctx=None):
        """Read an MXQW file into a new weight (mxq_weight_load)."""
        ctx = ctx or context()
        h = ctypes.c_void_p()
        ctx._bind()
        check(ctx.lib.mxq_weight_load(ctx.h, str(path).encode(), ctypes.byref(h)), ctx.h)
        obj = cls.__new__(cls)
        obj.ctx, obj.h, obj.block_sparse = ctx, h, False
        fmt, n, k = ctypes.c_int(), ctypes.c_size_t(), ctypes.c_size_t()
        check(ctx.lib.mxq_weight_shape(h, ctypes.byref(fmt), ctypes.byref(n), ctypes.byref(k)), ctx.h)
        obj.fmt, obj.n, obj.k = fmt.value, n.value, k.value
        return obj

    @classmethod
    def from_float(cls, w, fmt, ctx=None):
        """fp32 rows (a CUDA tensor [N][K], K a multiple of 32) quantised on
        the device (mx_quantize_w) into a new weight."""
        ctx = ctx or context()
        data, scales, _ = mx_quantize_w(w.contiguous(), fmt, ctx, with_sums=False)
        return cls(data, scales, fmt, w.shape[0], w.shape[1], ctx)


def _quant(x, act, ctx):
    ctx = ctx or context()
    _need_cuda(x, torch.float32, "x")
    if x.dim() == 1:
        x = x.unsqueeze(0)
    b, k = x.shape
    q = torch.empty((b, k), dtype=torch.uint8, device=x.device)
    s = torch.empty((b, k // 32), dtype=torch.uint8, device=x.device)
    ctx._bind()
    check(ctx.lib.mxq_quantize_x(ctx.h, _ptr(x), b, k, act, _ptr(q), _ptr(s)), ctx.h)
    return MXActivation(q, s)


def mx_quantize_x(x, ctx=None):
    """nca::linalg::mx_quantize_x: fp32 [B][K] -> MXActivation."""
    return _quant(x, ACT_NONE, ctx)


def mx_fused_silu_quantize_x(x, ctx=None):
    """nca::linalg::mx_fused_silu_quantize_x: silu(x) -> MXActivation."""
    return _quant(x, ACT_SILU, ctx)


def fused_gated_silu_quantize(gate, up, ctx=None):
    """nca::layers::fused_gated_silu_quantize: silu(gate) * up -> MX."""
    ctx = ctx or context()
    _need_cuda(gate, torch.float32, "gate")
    _need_cuda(up, torch.float32, "up")
    if gate.shape != up.shape:
        raise ValueError("gate and up shapes differ")
    if gate.dim() == 1:
        gate, up = gate.unsqueeze(0), up.unsqueeze(0)
    b, k = gate.shape
    q = torch.empty((b, k), dtype=torch.uint8, device=gate.device)
    s = torch.empty((b, k // 32), dtype=torch.uint8, device=gate.device)
    ctx._bind()
    check(ctx.lib.mxq_swiglu_quantize(ctx.h, _ptr(gate), _ptr(up), b, k, _ptr(q), _ptr(s)), ctx.h)
    return MXActivation(q, s)


def _check_act(x, w):
    _need_cuda(x.q, torch.uint8, "activation q")
    _need_cuda(x.s, torch.uint8, "activation scales")
    if x.k != w.k:
        raise ValueError("activation K=%d does not match weight K=%d" % (x.k, w.k))


def mx_gemv(x, w, ctx=None):
    """nca::linalg::mx_gemv: y[b][n] = sum_blocks 2^(e_x+e_w) * dot, fp32."""
    ctx = ctx or w.ctx
    _check_act(x, w)
    y = torch.empty((x.batch, w.n), dtype=torch.float32, device=x.q.device)
    ctx._bind()
    check(ctx.lib.mxq_gemv(ctx.h, w.h, _ptr(x.q), _ptr(x.s), x.batch, _ptr(y)), ctx.h)
    return y


def _rows(w, n, name):
    if w.n != n:
        raise ValueError("%s needs a %d-row weight, got %d rows" % (name, n, w.n))


def mx_dot(x, w, ctx=None):
    """nca::linalg::mx_dot: one weight row."""
    _rows(w, 1, "mx_dot")
    return mx_gemv(x, w, ctx)


def mx_dual_dot(x, w, ctx=None):
    _rows(w, 2, "mx_dual_dot")
    return mx_gemv(x, w, ctx)


def mx_quad_dot(x, w, ctx=None):
    _rows(w, 4, "mx_quad_dot")
    return mx_gemv(x, w, ctx)


def mx_rank16_dot(x, w, ctx=None):
    _rows(w, 16, "mx_rank16_dot")
    return mx_gemv(x, w, ctx)


def mx_rank16_dot_ptrs(x, w, rows=None, ctx=None):
    """nca::linalg::mx_rank16_dot_ptrs.  Two forms:
    - the reference's pointer-array form (nn/tests/autotest.hpp:126-136):
      `w` a list of one-row MXWeight (16 in the reference, up to 64 here),
      rows None -> y [B][len(w)] (mxq_rank16_dot_ptrs);
    - rows gathered by id from one expert-pool weight: `w` an MXWeight and
      `rows` an int32 device tensor of row ids (mxq_gather_dot)."""
    if isinstance(w, (list, tuple)):
        ctx = ctx or w[0].ctx
        if rows is not None:
            raise ValueError("mx_rank16_dot_ptrs: the pointer form takes no row ids")
        for wj in w:
            _check_act(x, wj)
            if wj.n != 1:
                raise ValueError("mx_rank16_dot_ptrs: each weight must have one row, got %d" % wj.n)
        arr = (ctypes.c_void_p * len(w))(*[wj.h.value for wj in w])
        y = torch.empty((x.batch, len(w)), dtype=torch.float32, device=x.q.device)
        ctx._bind()
        check(ctx.lib.mxq_rank16_dot_ptrs(ctx.h, ctypes.cast(arr, ctypes.c_void_p), len(w), _ptr(x.q), _ptr(x.s),
                                          x.batch, _ptr(y)), ctx.h)
        return y
    ctx = ctx or w.ctx
    _check_act(x, w)
    _need_cuda(rows, torch.int32, "rows")
    y = torch.empty((x.batch, rows.numel()), dtype=torch.float32, device=x.q.device)
    ctx._bind()
    check(ctx.lib.mxq_gather_dot(ctx.h, w.h, _ptr(x.q), _ptr(x.s), x.batch, _ptr(rows), rows.numel(),
                                 _ptr(y)), ctx.h)
    return y


def mx_block_dots(x, w, ctx=None):
    """Per-block int32 dots [B][N][K/32] (the dpbusd - 128*w_sum values)."""
    ctx = ctx or w.ctx
    _check_act(x, w)
    d = torch.empty((x.batch, w.n, w.k // 32), dtype=torch.int32, device=x.q.device)
    ctx._bind()
    check(ctx.lib.mxq_block_dots(ctx.h, w.h, _ptr(x.q), x.batch, _ptr(d)), ctx.h)
    return d


def mx_linear(x, w, ctx=None):
    """fp32 [B][K] -> quantise -> MX linear -> fp32 [B][N]."""
    ctx = ctx or w.ctx
    _need_cuda(x, torch.float32, "x")
    if x.dim() == 1:
        x = x.unsqueeze(0)
    if x.shape[1] != w.k:
        raise ValueError("x K=%d does not match weight K=%d" % (x.shape[1], w.k))
    y = torch.empty((x.shape[0], w.n), dtype=torch.float32, device=x.device)
    ctx._bind()
    check(ctx.lib.mxq_linear(ctx.h, w.h, _ptr(x), x.shape[0], _ptr(y)), ctx.h)
    return y


def mx_linear_pair(x, w1, w2, ctx=None):
    ctx = ctx or w1.ctx
    _need_cuda(x, torch.float32, "x")
    if x.dim() == 1:
        x = x.unsqueeze(0)
    y = torch.empty((x.shape[0], w2.n), dtype=torch.float32, device=x.device)
    ctx._bind()
    check(ctx.lib.mxq_linear_pair(ctx.h, w1.h, w2.h, _ptr(x), x.shape[0], _ptr(y)), ctx.h)
    return y


class PeerGroup:
    """One rank of a batch-1 linear pair column-sharded over `world` GPUs
    (mxq_peers_*): the first linear's rows of the MX intermediate and the
    second's fp32 rows go straight into every rank's mailbox over NVLink.

    handle() gives this rank's 64-byte mailbox handle; the caller gathers
    every rank's (e.g. torch.distributed.all_gather_object) and passes the
    list, in rank order, to connect()."""

    def __init__(self, rank, world, n1, n2, ctx=None):
        self.ctx = ctx or context()
        self.rank, self.world, self.n1, self.n2 = rank, world, n1, n2
        h = ctypes.c_void_p()
        self._handle = ctypes.create_string_buffer(_lib.PEER_HANDLE_BYTES)
        self.ctx._bind()
        check(self.ctx.lib.mxq_peers_create(self.ctx.h, rank, world, n1, n2, ctypes.byref(h),
                                            ctypes.cast(self._handle, ctypes.c_void_p)), self.ctx.h)
        self.h = h

    def handle(self):
        return bytes(self._handle.raw)

    def connect(self, handles):
        assert len(handles) == self.world and all(len(b) == _lib.PEER_HANDLE_BYTES for b in handles)
        buf = ctypes.create_string_buffer(b"".join(handles), _lib.PEER_HANDLE_BYTES * self.world)
        check(self.ctx.lib.mxq_peers_connect(self.h, ctypes.cast(buf, ctypes.c_void_p)), self.ctx.h)

    def set_wait_limit(self, us):
        check(self.ctx.lib.mxq_peers_set_wait_limit(self.h, int(us)), self.ctx.h)

    def linear_pair(self, x, w1, w2, out=None):
        """x [K] or [1, K] fp32 on this rank's GPU; w1 / w2 this rank's
        shards; returns the full [1, n2] output (the same on every rank)."""
        _need_cuda(x, torch.float32, "x")
        y = out if out is not None else torch.empty((1, self.n2), dtype=torch.float32, device=x.device)
        self.ctx._bind()
        check(self.ctx.lib.mxq_linear_pair_sharded(self.ctx.h, self.h, w1.h, w2.h, _ptr(x), _ptr(y)), self.ctx.h)
        return y

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.mxq_peers_destroy(self.h)
            self.h = None


def gated_mlp_step(x, w_gate, w_up, w_down, ctx=None):
    """nca::layers::gated_mlp_step: down(quant(silu(gate x) * up x))."""
    ctx = ctx or w_gate.ctx
    _need_cuda(x, torch.float32, "x")
    if x.dim() == 1:
        x = x.unsqueeze(0)
    y = torch.empty((x.shape[0], w_down.n), dtype=torch.float32, device=x.device)
    ctx._bind()
    check(ctx.lib.mxq_mlp_swiglu(ctx.h, w_gate.h, w_up.h, w_down.h, _ptr(x), x.shape[0], _ptr(y)), ctx.h)
    return y


def route_topk(logits, k, ctx=None):
    """Top-k experts per token: (idx int32 [T][k], gate fp32 [T][k])."""
    ctx = ctx or context()
    _need_cuda(logits, torch.float32, "logits")
    t, e = logits.shape
    if k == 0 or k > e:
        raise ValueError("Top-K (%d) must be in [1, n_experts=%d]" % (k, e))
    idx = torch.empty((t, k), dtype=torch.int32, device=logits.device)
    gate = torch.empty((t, k), dtype=torch.float32, device=logits.device)
    ctx._bind()
    check(ctx.lib.mxq_route_topk(ctx.h, _ptr(logits), t, e, k, _ptr(idx), _ptr(gate)), ctx.h)
    return idx, gate


class HashedRouter:
    """linalg::HashedRouter{Config{d, n_experts, top_k, n_hashes}}
    (nn/tests/test_robustness.cpp:13-35): top_k > n_experts raises ValueError
    at construction (the reference's invalid_argument).

    route(x): the LSH router (mxq_hashed_route) -- sign-of-projection codes of
    the MX-quantised input over n_hashes seeded +-1 hyperplanes, experts
    ranked by Hamming similarity of seeded expert codes, ties to the lower id;
    returns (idx int32 [T][top_k], score int32 [T][top_k]).
    route_logits(logits): softmax top-k over caller-supplied logits
    (mxq_route_topk), the MoE layer's router."""

    def __init__(self, d, n_experts, top_k, n_hashes=8, seed=0):
        if top_k > n_experts or top_k == 0:
            raise ValueError("HashedRouter: top_k (%d) exceeds n_experts (%d)" % (top_k, n_experts))
        if not 1 <= n_hashes <= 32 or d % 32:
            raise ValueError("HashedRouter: n_hashes in [1, 32] and d a multiple of 32")
        self.d, self.n_experts, self.top_k, self.n_hashes, self.seed = d, n_experts, top_k, n_hashes, seed

    def route(self, x, ctx=None):
        ctx = ctx or context()
        _need_cuda(x, torch.float32, "x")
        x2 = x.reshape(-1, x.shape[-1])
        if x2.shape[1] != self.d:
            raise ValueError("x has %d features, router d is %d" % (x2.shape[1], self.d))
        t = x2.shape[0]
        idx = torch.empty((t, self.top_k), dtype=torch.int32, device=x.device)
        score = torch.empty((t, self.top_k), dtype=torch.int32, device=x.device)
        ctx._bind()
        check(ctx.lib.mxq_hashed_route(ctx.h, _ptr(x2), t, self.d, self.n_experts, self.top_k, self.n_hashes,
                                       self.seed, _ptr(idx), _ptr(score)), ctx.h)
        return idx, score

    def route_logits(self, logits, ctx=None):
        if logits.shape[-1] != self.n_experts:
            raise ValueError("logits last dim %d != n_experts %d" % (logits.shape[-1], self.n_experts))
        return route_topk(logits.reshape(-1, self.n_experts), self.top_k, ctx)


class HaltingState:
    """nca::layers::HaltingState (nn/core/layers/halting.hpp:16-20) for B
    tokens on the device: 16 bytes per token {float p_sum, float remainder,
    uint64 steps} (mxq_halting_state)."""

    def __init__(self, batch, device=None):
        self.raw = torch.zeros((batch, 4), dtype=torch.float32,
                               device=device if device is not None else torch.cuda.current_device())

    @property
    def p_sum(self):
        return self.raw[:, 0]

    @property
    def remainder(self):
        return self.raw[:, 1]

    @property
    def steps(self):
        return self.raw[:, 2:4].contiguous().view(torch.int64).reshape(-1)


def halting_step(x, w_halt, bias, state, ctx=None):
    """nca::layers::halting_step (nn/core/layers/halting.hpp:24-30), batched
    over the tokens of an MXActivation: p = sigmoid(w_halt . x + bias), ACT
    update of `state` (HaltingState) in place.  Returns (p [B], should_halt
    uint8 [B])."""
    ctx = ctx or w_halt.ctx
    _check_act(x, w_halt)
    if w_halt.n != 1:
        raise ValueError("halting_step: w_halt must have one row, got %d" % w_halt.n)
    if state.raw.shape[0] != x.batch:
        raise ValueError("halting_step: state holds %d tokens, activation %d" % (state.raw.shape[0], x.batch))
    p = torch.empty(x.batch, dtype=torch.float32, device=x.q.device)
    h = torch.empty(x.batch, dtype=torch.uint8, device=x.q.device)
    ctx._bind()
    check(ctx.lib.mxq_halting_step(ctx.h, w_halt.h, _ptr(x.q), _ptr(x.s), x.batch, float(bias), _ptr(state.raw),
                                   _ptr(p), _ptr(h)), ctx.h)
    return p, h


def mx_update_gaussian_moment(w, g, x, step, ctx=None):
    """nca::linalg::mx_update_gaussian_moment: in place, w += step * g x^T in
    the weight's own E8M0 grid, re-clamped to the int8 / int4 range
    (mxq_update_gaussian_moment).  g [N], x [K] fp32 CUDA tensors."""
    ctx = ctx or w.ctx
    _need_cuda(g, torch.float32, "g")
    _need_cuda(x, torch.float32, "x")
    if g.numel() != w.n or x.numel() != w.k:
        raise ValueError("update: g needs %d values and x %d" % (w.n, w.k))
    ctx._bind()
    check(ctx.lib.mxq_update_gaussian_moment(ctx.h, w.h, _ptr(g), _ptr(x), float(step)), ctx.h)


def micro_moe(x, w_gate, w_up, w_down, n_routed, n_shared, idx, gate=None, ctx=None):
    """The micro-expert pool layer (mxq_micro_moe): x [T][D], 16-row experts
    in the gate/up pools [(n_routed + n_shared) * 16][D] and the down pool
    [D][(n_routed + n_shared) * 16]; idx/gate [T][k] from a router (gate None
    = weight 1); shared experts always active.  Returns y [T][D]."""
    ctx = ctx or w_gate.ctx
    _need_cuda(x, torch.float32, "x")
    t, d = x.shape
    k = 0 if idx is None else idx.shape[1]
    if idx is not None:
        _need_cuda(idx, torch.int32, "idx")
    if gate is not None:
        _need_cuda(gate, torch.float32, "gate")
    y = torch.empty((t, w_down.n), dtype=torch.float32, device=x.device)
    ctx._bind()
    check(ctx.lib.mxq_micro_moe(ctx.h, w_gate.h, w_up.h, w_down.h, n_routed, n_shared, _ptr(x), _ptr(idx),
                                _ptr(gate), t, k, _ptr(y)), ctx.h)
    return y


def mx_compute_activation_norm(x, ctx=None):
    """nca::linalg::mx_compute_activation_norm: L2 norm per MX activation row."""
    ctx = ctx or context()
    _need_cuda(x.q, torch.uint8, "activation q")
    out = torch.empty(x.batch, dtype=torch.float32, device=x.q.device)
    ctx._bind()
    check(ctx.lib.mxq_activation_norm(ctx.h, _ptr(x.q), _ptr(x.s), x.batch, x.k, _ptr(out)), ctx.h)
    return out


def mx_quantize_w(w, fmt, ctx=None, with_sums=True):
    """nca::linalg::mx_quantize_w on the device: fp32 [N][K] -> (data int8
    [N][K] or packed int4 uint8 [N][K/2], E8M0 scales [N][K/32], w_sums int32
    [N][K/32] or None)."""
    ctx = ctx or context()
    _need_cuda(w, torch.float32, "w")
    n, k = w.shape
    if fmt not in (FMT_INT4, FMT_INT8):
        raise ValueError("unknown weight format %d" % fmt)
    data = torch.empty((n, k // 2), dtype=torch.uint8, device=w.device) if fmt == FMT_INT4 else \
        torch.empty((n, k), dtype=torch.int8, device=w.device)
    scales = torch.empty((n, k // 32), dtype=torch.uint8, device=w.device)
    sums = torch.empty((n, k // 32), dtype=torch.int32, device=w.device) if with_sums else None
    ctx._bind()
    check(ctx.lib.mxq_quantize_w(ctx.h, fmt, _ptr(w), n, k, _ptr(data), _ptr(scales), _ptr(sums)), ctx.h)
    return data, scales, sums


def fused_compute_gae(rewards, values, dones, next_values, gamma=0.99, lam=0.95, ctx=None):
    """nca::env::ReplayMemory::fused_compute_gae on [T][E] interleaved data.
    Returns (advantages, returns)."""
    ctx = ctx or context()
    _need_cuda(rewards, torch.float32, "rewards")
    _need_cuda(values, torch.float32, "values")
    _need_cuda(dones, torch.uint8, "dones")
    _need_cuda(next_values, torch.float32, "next_values")
    t, e = rewards.shape
    if values.shape != (t, e) or dones.shape != (t, e) or next_values.numel() != e:
        raise ValueError("GAE input shapes disagree")
    adv = torch.empty_like(rewards)
    ret = torch.empty_like(rewards)
    ctx._bind()
    check(ctx.lib.mxq_gae(ctx.h, _ptr(rewards), _ptr(values), _ptr(dones), _ptr(next_values), t, e,
                          float(gamma), float(lam), _ptr(adv), _ptr(ret)), ctx.h)
    return adv, ret


def fused_compute_gae_ring(rewards, values, dones, next_values, size, cursor, t, e, adv, ret, gamma=0.99,
                           lam=0.95, ctx=None):
    """ReplayMemory::fused_compute_gae on the ring buffer itself
    (mxq_gae_ring): 1-D device ring arrays of the capacity, `size` items
    stored, next write at `cursor`; the latest t*e items are swept and only
    the first 1024 environments written, as in the reference.  adv/ret are
    updated in place and returned."""
    ctx = ctx or context()
    for name, tns, dt in (("rewards", rewards, torch.float32), ("values", values, torch.float32),
                          ("dones", dones, torch.uint8), ("next_values", next_values, torch.float32),
                          ("adv", adv, torch.float32), ("ret", ret, torch.float32)):
        _need_cuda(tns, dt, name)
    cap = rewards.numel()
    if values.numel() != cap or dones.numel() != cap or adv.numel() != cap or ret.numel() != cap:
        raise ValueError("GAE ring arrays must all hold the capacity")
    if next_values.numel() < min(e, 1024):
        raise ValueError("next_values needs one value per environment")
    ctx._bind()
    check(ctx.lib.mxq_gae_ring(ctx.h, _ptr(rewards), _ptr(values), _ptr(dones), _ptr(next_values), cap, size,
                               cursor, t, e, float(gamma), float(lam), _ptr(adv), _ptr(ret)), ctx.h)
    return adv, ret


def moe_swiglu(x, logits, gate_w, up_w, down_w, k, ctx=None):
    """Top-k SwiGLU mixture-of-experts layer (mxq_moe_swiglu): x fp32 [T][D]
    and router logits [T][E] on the device; gate_w/up_w/down_w lists of E
    MXWeight ([F][D], [F][D], [D][F], dense or block-sparse).  Returns y
    [T][D].  k > E raises ValueError (the HashedRouter contract)."""
    ctx = ctx or context()
    _need_cuda(x, torch.float32, "x")
    _need_cuda(logits, torch.float32, "logits")
    t, d = x.shape
    e = len(gate_w)
    if logits.shape != (t, e) or len(up_w) != e or len(down_w) != e:
        raise ValueError("moe: logits must be [T][E] with E gate/up/down weights")
    arr = lambda ws: (ctypes.c_void_p * e)(*[w.h.value for w in ws])
    g, u, dn = arr(gate_w), arr(up_w), arr(down_w)
    y = torch.empty((t, d), dtype=torch.float32, device=x.device)
    ctx._bind()
    check(ctx.lib.mxq_moe_swiglu(ctx.h, ctypes.cast(g, ctypes.c_void_p), ctypes.cast(u, ctypes.c_void_p),
                                 ctypes.cast(dn, ctypes.c_void_p), e, _ptr(x), _ptr(logits), t, k, _ptr(y)),
          ctx.h)
    return y


class MoEGroup:
    """One rank of the expert-parallel MoE layer over `world` GPUs
    (mxq_moe_group_*, mxq_moe_swiglu_sharded): rank r owns experts
    [r E/world, (r+1) E/world); every rank passes all T tokens and gets the
    full y, bit-identical to moe_swiglu over all experts on one GPU.

    handle() gives this rank's 64-byte mailbox handle; the caller gathers
    every rank's (e.g. torch.distributed.all_gather_object) and passes the
    list, in rank order, to connect()."""

    def __init__(self, rank, world, max_tokens, top_k, d_model, ctx=None):
        self.ctx = ctx or context()
        self.rank, self.world = rank, world
        h = ctypes.c_void_p()
        self._handle = ctypes.create_string_buffer(_lib.PEER_HANDLE_BYTES)
        self.ctx._bind()
        check(self.ctx.lib.mxq_moe_group_create(self.ctx.h, rank, world, max_tokens, top_k, d_model, ctypes.byref(h),
                                                ctypes.cast(self._handle, ctypes.c_void_p)), self.ctx.h)
        self.h = h

    def handle(self):
        return bytes(self._handle.raw)

    def connect(self, handles):
        assert len(handles) == self.world and all(len(b) == _lib.PEER_HANDLE_BYTES for b in handles)
        buf = ctypes.create_string_buffer(b"".join(handles), _lib.PEER_HANDLE_BYTES * self.world)
        check(self.ctx.lib.mxq_moe_group_connect(self.h, ctypes.cast(buf, ctypes.c_void_p)), self.ctx.h)

    def set_wait_limit(self, us):
        check(self.ctx.lib.mxq_moe_group_set_wait_limit(self.h, int(us)), self.ctx.h)

    def moe_swiglu(self, x, logits, gate_w, up_w, down_w, k, out=None):
        """x [T][D], logits [T][E] (the same on every rank); gate_w/up_w/down_w
        this rank's E/world experts.  Returns y [T][D]."""
        _need_cuda(x, torch.float32, "x")
        _need_cuda(logits, torch.float32, "logits")
        t, d = x.shape
        e = logits.shape[1]
        n = len(gate_w)
        if n * self.world != e or len(up_w) != n or len(down_w) != n:
            raise ValueError("moe group: each rank passes E/world gate/up/down weights")
        arr = lambda ws: (ctypes.c_void_p * n)(*[w.h.value for w in ws])
        g, u, dn = arr(gate_w), arr(up_w), arr(down_w)
        y = out if out is not None else torch.empty((t, d), dtype=torch.float32, device=x.device)
        self.ctx._bind()
        check(self.ctx.lib.mxq_moe_swiglu_sharded(self.ctx.h, self.h, ctypes.cast(g, ctypes.c_void_p),
                                                  ctypes.cast(u, ctypes.c_void_p), ctypes.cast(dn, ctypes.c_void_p),
                                                  e, _ptr(x), _ptr(logits), t, k, _ptr(y)), self.ctx.h)
        return y

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.mxq_moe_group_destroy(self.h)
            self.h = None


def policy_head(logits, actions, ctx=None):
    """PPO rollout head (mxq_policy_head): (log_probs [R][C], action_logp [R],
    entropy [R]) from logits and action weights [R][C]."""
    ctx = ctx or context()
    _need_cuda(logits, torch.float32, "logits")
    _need_cuda(actions, torch.float32, "actions")
    if logits.shape != actions.shape or logits.dim() != 2:
        raise ValueError("policy_head: logits and actions must both be [R][C]")
    r, c = logits.shape
    lp = torch.empty_like(logits)
    alp = torch.empty(r, dtype=torch.float32, device=logits.device)
    ent = torch.empty(r, dtype=torch.float32, device=logits.device)
    ctx._bind()
    check(ctx.lib.mxq_policy_head(ctx.h, _ptr(logits), _ptr(actions), r, c, _ptr(lp), _ptr(alp), _ptr(ent)),
          ctx.h)
    return lp, alp, ent


def ppo_rollout_forward(states, actions, w_proj, w_policy, w_value=None, ctx=None):
    """The rollout forward of PPOTrainer::update_step
    (training/ppo_trainer.cpp:57-66, :77) with its products as MX linears:
    latent = states . proj, logits = latent . policy^T, values = latent .
    value^T, then the policy head.  states [R][S] is zero-padded to the
    projection's K (S = 1616 -> 1632, the next multiple of 32).  With
    w_value None, w_policy holds A + 1 rows, the last being the value head,
    so the latent is quantised once for both.
    Returns (log_probs, action_logp, entropy, values [R])."""
    ctx = ctx or w_proj.ctx
    _need_cuda(states, torch.float32, "states")
    if states.shape[1] != w_proj.k:
        if states.shape[1] > w_proj.k:
            raise ValueError("states have %d features, projection K is %d" % (states.shape[1], w_proj.k))
        states = torch.nn.functional.pad(states, (0, w_proj.k - states.shape[1]))
    latent = mx_linear(states.contiguous(), w_proj, ctx)
    if w_value is None:
        head = mx_linear(latent, w_policy, ctx)
        a = head.shape[1] - 1
        logits, values = head[:, :a].contiguous(), head[:, a].contiguous()
    else:
        logits = mx_linear(latent, w_policy, ctx)
        values = mx_linear(latent, w_value, ctx)[:, 0]
    lp, alp, ent = policy_head(logits, actions, ctx)
    return lp, alp, ent, values


# ------------------------------------------------------------------ decoder ---
DEC_QKV, DEC_O, DEC_GATE_UP, DEC_DOWN, DEC_LM_HEAD = 0, 1, 2, 3, 4
TRACE = {"in": 0, "norm1": 1, "qkv": 2, "rope": 3, "att": 4, "h1": 5, "norm2": 6, "gu": 7, "out": 8}


class DecoderConfig(ctypes.Structure):
    """mxq_decoder_config (include/mxq.h)."""
    _fields_ = [("n_layers", ctypes.c_int), ("d_model", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("ffn", ctypes.c_int), ("vocab", ctypes.c_int), ("fmt", ctypes.c_int), ("max_batch", ctypes.c_int),
                ("max_ctx", ctypes.c_int), ("max_rows", ctypes.c_int), ("value_head", ctypes.c_int),
                ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float)]


class Decoder:
    """The dense decoder on the MX linears (mxq_decoder_*): prefill a prompt,
    decode one token per sequence per step (CUDA-graph replayed), or score
    whole sequences (per-token log-probs and values, the rollout forward).
    Weights are synthetic, generated from `seed` on the device.

    With `world` set, rank `rank` of a tensor-parallel decoder over `world`
    GPUs (mxq_decoder_create_sharded): handle() gives this rank's 64-byte
    mailbox handle; the caller gathers every rank's (e.g.
    torch.distributed.all_gather_object) and passes the list, in rank order,
    to connect() before the first pass."""

    def __init__(self, n_layers, d_model, n_heads, ffn, vocab, fmt=FMT_INT4, max_batch=1, max_ctx=2048,
                 max_rows=8192, value_head=False, rope_theta=10000.0, norm_eps=1e-5, seed=0, ctx=None,
                 rank=0, world=None):
        self.ctx = ctx or context()
        self.cfg = DecoderConfig(n_layers, d_model, n_heads, ffn, vocab, fmt, max_batch, max_ctx, max_rows,
                                 1 if value_head else 0, rope_theta, norm_eps)
        self.rank, self.world = rank, world
        h = ctypes.c_void_p()
        self.ctx._bind()
        if world is None:
            check(self.ctx.lib.mxq_decoder_create(self.ctx.h, ctypes.byref(self.cfg), seed, ctypes.byref(h)),
                  self.ctx.h)
        else:
            self._handle = ctypes.create_string_buffer(_lib.PEER_HANDLE_BYTES)
            check(self.ctx.lib.mxq_decoder_create_sharded(self.ctx.h, ctypes.byref(self.cfg), seed, rank, world,
                                                          ctypes.byref(h),
                                                          ctypes.cast(self._handle, ctypes.c_void_p)), self.ctx.h)
        self.h = h

    def handle(self):
        return bytes(self._handle.raw)

    def connect(self, handles):
        assert self.world is not None and len(handles) == self.world
        assert all(len(b) == _lib.PEER_HANDLE_BYTES for b in handles)
        buf = ctypes.create_string_buffer(b"".join(handles), _lib.PEER_HANDLE_BYTES * self.world)
        check(self.ctx.lib.mxq_decoder_connect(self.h, ctypes.cast(buf, ctypes.c_void_p)), self.ctx.h)

    def set_wait_limit(self, us):
        check(self.ctx.lib.mxq_decoder_set_wait_limit(self.h, int(us)), self.ctx.h)

    def _tokens(self, tokens):
        if not isinstance(tokens, torch.Tensor) or tokens.dtype != torch.int32 or not tokens.is_contiguous():
            raise ValueError("tokens must be a contiguous int32 tensor")
        return tokens

    def prefill(self, tokens):
        """tokens [B][T] -> logits of the last position [B][vocab]."""
        tokens = self._tokens(tokens)
        b, t = tokens.shape
        logits = torch.empty((b, self.cfg.vocab), dtype=torch.float32, device="cuda")
        self.ctx._bind()
        check(self.ctx.lib.mxq_decoder_prefill(self.h, _ptr(tokens), b, t, _ptr(logits)), self.ctx.h)
        return logits

    def decode(self, tokens):
        """tokens [B] (one per sequence) -> logits [B][vocab]."""
        tokens = self._tokens(tokens)
        b = tokens.numel()
        logits = torch.empty((b, self.cfg.vocab), dtype=torch.float32, device="cuda")
        self.ctx._bind()
        check(self.ctx.lib.mxq_decoder_decode(self.h, _ptr(tokens), b, _ptr(logits)), self.ctx.h)
        return logits

    def score(self, tokens):
        """tokens [B][T] -> (logp [B][T-1], values [B][T] or None)."""
        tokens = self._tokens(tokens)
        b, t = tokens.shape
        logp = torch.empty((b, t - 1), dtype=torch.float32, device="cuda")
        values = torch.empty((b, t), dtype=torch.float32, device="cuda") if self.cfg.value_head else None
        self.ctx._bind()
        check(self.ctx.lib.mxq_decoder_score(self.h, _ptr(tokens), b, t, _ptr(logp), _ptr(values)), self.ctx.h)
        return logp, values

    def reset(self):
        check(self.ctx.lib.mxq_decoder_reset(self.h), self.ctx.h)

    def length(self):
        v = ctypes.c_int()
        check(self.ctx.lib.mxq_decoder_length(self.h, ctypes.byref(v)), self.ctx.h)
        return v.value

    def weight_handle(self, layer, which):
        w = ctypes.c_void_p()
        check(self.ctx.lib.mxq_decoder_weight(self.h, layer, which, ctypes.byref(w)), self.ctx.h)
        return w

    def download(self, layer, which):
        """(data, scales) of one weight in the MXINT8Tensor layout (numpy)."""
        import numpy as np
        w = self.weight_handle(layer, which)
        fmt, n, k = ctypes.c_int(), ctypes.c_size_t(), ctypes.c_size_t()
        check(self.ctx.lib.mxq_weight_shape(w, ctypes.byref(fmt), ctypes.byref(n), ctypes.byref(k)), self.ctx.h)
        data = np.empty((n.value, k.value // 2), np.uint8) if fmt.value == FMT_INT4 else \
            np.empty((n.value, k.value), np.int8)
        scales = np.empty((n.value, k.value // 32), np.uint8)
        check(self.ctx.lib.mxq_weight_download(w, data.ctypes.data_as(ctypes.c_void_p),
                                               scales.ctypes.data_as(ctypes.c_void_p)), self.ctx.h)
        return data, scales

    def embedding_rows(self, row0, nrows):
        import numpy as np
        out = np.empty((nrows, self.cfg.d_model), np.float32)
        check(self.ctx.lib.mxq_decoder_embedding(self.h, row0, nrows, out.ctypes.data_as(ctypes.c_void_p)),
              self.ctx.h)
        return out

    def set_trace(self, layer):
        check(self.ctx.lib.mxq_decoder_set_trace(self.h, layer), self.ctx.h)

    def get_trace(self, name, shape):
        import numpy as np
        out = np.empty(shape, np.float32)
        check(self.ctx.lib.mxq_decoder_get_trace(self.h, TRACE[name], out.ctypes.data_as(ctypes.c_void_p),
                                                 out.size), self.ctx.h)
        return out

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.mxq_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
