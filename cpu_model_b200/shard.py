"""Multi-GPU plumbing for the MX linear and the MoE layer over
torch.distributed (one process per GPU; NCCL over NVLink on the GPUs, gloo
for the CPU tests).

Column sharding (output features) -- every rank owns a contiguous slice of
a weight's rows with the full K, so each output row is computed exactly as on
one GPU (same kernel, same K order); one all-gather of y per linear puts the
slices back together.  Used for the MLP pair: up is gathered before down
(down needs every up feature), down is gathered at the layer boundary.

Expert parallelism -- experts are partitioned over the ranks in contiguous
ranges; every rank routes its own tokens (top-k, the router contract of
nn/tests/test_robustness.cpp:13-35), sends each (token, expert) route to the
rank owning the expert with one all_to_all_single (counts exchanged first),
runs its experts on what it received, returns the outputs with a second
all_to_all_single and combines a token's k outputs in routing order.

The per-rank compute is passed in (a linear, an expert MLP), so the same
exchange logic runs on the GPU with libmxq.so and, in the gloo tests, with a
CPU stand-in.
"""
import torch
import torch.distributed as dist


def row_shards(n, world):
    """Contiguous, balanced row ranges [(lo, hi)] of an n-row weight."""
    return [(r * n // world, (r + 1) * n // world) for r in range(world)]


def gather_columns(y_local, n, group=None):
    """All-gather rank-local output columns [B][hi-lo] into [B][n] (ranks
    hold the balanced slices of row_shards; slices are padded to the largest
    one for the collective)."""
    world = dist.get_world_size(group)
    shards = row_shards(n, world)
    width = max(hi - lo for lo, hi in shards)
    b = y_local.shape[0]
    send = torch.zeros((b, width), dtype=y_local.dtype, device=y_local.device)
    send[:, :y_local.shape[1]] = y_local
    if y_local.is_cuda:
        recv = torch.empty((world, b, width), dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(recv, send, group=group)
        parts = list(recv.unbind(0))
    else:
        parts = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(parts, send, group=group)
    return torch.cat([parts[r][:, :hi - lo] for r, (lo, hi) in enumerate(shards)], dim=1)


class ColumnShardedLinear:
    """This rank's row slice of an MX weight.

    weight_fn(lo, hi) builds the slice (e.g. an MXWeight from rows lo..hi of
    the host data and scales); linear(x, w) computes x -> [B][hi-lo]."""

    def __init__(self, n, weight_fn, linear, group=None):
        self.n = n
        self.group = group
        self.rank = dist.get_rank(group)
        self.lo, self.hi = row_shards(n, dist.get_world_size(group))[self.rank]
        self.w = weight_fn(self.lo, self.hi)
        self.linear = linear

    def local(self, x):
        return self.linear(x, self.w)

    def __call__(self, x):
        return gather_columns(self.local(x), self.n, self.group)


def sharded_pair(x, up, down):
    """The 7B-MLP linear pair on column shards: up slice -> all-gather ->
    down slice -> all-gather.  Identical rows to the single-GPU pair."""
    return down(up(x))


def expert_owner(e, n_experts, world):
    """Rank owning expert e (contiguous balanced ranges)."""
    for r, (lo, hi) in enumerate(row_shards(n_experts, world)):
        if lo <= e < hi:
            return r
    raise ValueError("expert %d out of range" % e)


def _exchange(payload, send_counts, group):
    """all_to_all_single of row blocks: payload rows grouped by destination
    rank, send_counts[r] rows to rank r; returns (received rows,
    recv_counts)."""
    world = dist.get_world_size(group)
    dev = payload.device
    sc = torch.tensor(send_counts, dtype=torch.int64, device=dev)
    rc = torch.empty(world, dtype=torch.int64, device=dev)
    dist.all_to_all_single(rc, sc, group=group)
    recv_counts = [int(v) for v in rc.tolist()]
    flat_in = payload.reshape(payload.shape[0], -1)
    out = torch.empty((sum(recv_counts), flat_in.shape[1]), dtype=payload.dtype, device=dev)
    dist.all_to_all_single(out, flat_in.contiguous(), output_split_sizes=recv_counts,
                           input_split_sizes=list(send_counts), group=group)
    return out, recv_counts


def moe_expert_parallel(x, idx, gate, n_experts, expert_mlp, group=None):
    """One MoE layer with experts partitioned over the ranks.

    x [T][D] this rank's tokens; idx/gate [T][k] its routing (top-k ids and
    softmax gates); expert_mlp(e, rows [M][D]) -> [M][D] runs local expert e.
    Routes are sent in (destination rank, expert, token, slot) order, so the
    rows each expert sees arrive in a fixed order; the result is
    y[t] = sum_j gate[t][j] * expert_{idx[t][j]}(x[t]) summed in j order."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    t, k = idx.shape
    d = x.shape[1]
    dev = x.device
    idx_l = idx.to(torch.int64)
    owner = torch.tensor([expert_owner(e, n_experts, world) for e in range(n_experts)], device=dev)
    route_e = idx_l.reshape(-1)                                  # route r = t*k + j
    route_dst = owner[route_e]
    # stable order: destination rank, then expert, then route id
    key = (route_dst * n_experts + route_e) * (t * k) + torch.arange(t * k, device=dev)
    order = torch.argsort(key)
    send_counts = torch.bincount(route_dst, minlength=world).tolist()
    rows = x.repeat_interleave(k, dim=0)[order]                   # [T*k][D]
    tag = route_e[order].to(x.dtype).unsqueeze(1)                 # expert id travels with the row
    payload = torch.cat([rows, tag], dim=1)
    recv, recv_counts = _exchange(payload, send_counts, group)
    rx, re = recv[:, :d], recv[:, d].to(torch.int64)
    out = torch.empty_like(rx)
    lo, hi = row_shards(n_experts, world)[rank]
    for e in range(lo, hi):
        sel = (re == e).nonzero(as_tuple=True)[0]
        if sel.numel():
            out[sel] = expert_mlp(e, rx[sel].contiguous())
    back, _ = _exchange(out, recv_counts, group)                  # rows return in send order
    y_routes = torch.empty((t * k, d), dtype=x.dtype, device=dev)
    y_routes[order] = back
    y_routes = y_routes.reshape(t, k, d)
    y = torch.zeros((t, d), dtype=x.dtype, device=dev)
    for j in range(k):
        y = torch.addcmul(y, gate[:, j:j + 1].to(x.dtype), y_routes[:, j])
    return y
