"""Point-sharded slice/deslice coupling across the GPUs of one node.

The slice is a sum over points, the deslice and both backward passes are
per point given the token state, so the coupling shards over N with no
exchange of point data: each rank slices its own contiguous range of points,
the tiny per-rank partials (z_num, s) -- B*H*G*(DV+1) floats -- are summed
across ranks, and the deslice runs locally on the replicated tokens. In the
backward the per-rank token gradients are summed the same way (the slice's
upstream gradient needs all of them), and the parameter gradients (dW, db,
dtau) are summed once at the end (the point-sharded coupling the reference
plans in ROADMAP.md "Point-sharded slice": an all-reduce of (z_num, s) in
the forward and of dtokens in the backward).

Every cross-rank sum is an all-gather of the per-rank partials into a
(world, ...) buffer followed by a sum in rank order 0, 1, ..., so every rank
computes bitwise the same result and the result is bitwise reproducible
run to run for a fixed world size, whatever algorithm NCCL picks.
"""

import torch
import torch.distributed as dist


def shard_range(n, rank, world):
    """Contiguous point range [start, stop) of ``rank``: N // world points
    each, the remainder one point each to the last ranks."""
    base, rem = divmod(n, world)
    start = rank * base + max(0, rank - (world - rem))
    return start, start + base + (1 if rank >= world - rem else 0)


def _fold(buf):
    """Sum of the (world, n) rows of ``buf`` in rank order: one native launch
    (``fs_rank_sum``) for fp32 on the GPU, torch adds otherwise (CPU ranks)."""
    if buf.is_cuda and buf.dtype == torch.float32:
        from .kernels import _native as nat
        out = torch.empty(buf.shape[1:], dtype=buf.dtype, device=buf.device)
        stream = torch.cuda.current_stream(buf.device).cuda_stream
        nat.check(nat.load().fs_rank_sum(buf.data_ptr(), out.data_ptr(), buf.shape[0],
                                         out.numel(), stream))
        return out
    out = buf[0].clone()
    for r in range(1, buf.shape[0]):
        out += buf[r]
    return out


def ordered_sum_many(ts, group=None):
    """Each tensor of ``ts`` summed over the ranks of ``group`` in rank order
    (no autograd), through one all-gather of their concatenation."""
    world = dist.get_world_size(group)
    if world == 1:
        return [t.clone() for t in ts]
    dtype = ts[0].dtype
    if any(t.dtype != dtype for t in ts):
        return [ordered_sum(t, group) for t in ts]
    flat_in = torch.cat([t.reshape(-1) for t in ts]) if len(ts) > 1 else ts[0].reshape(-1)
    n = flat_in.numel()
    # a flat (world * n) output: the layout every backend accepts
    flat = torch.empty(world * n, dtype=dtype, device=flat_in.device)
    dist.all_gather_into_tensor(flat, flat_in.contiguous(), group=group)
    total = _fold(flat.view(world, n))
    out, off = [], 0
    for t in ts:
        out.append(total[off:off + t.numel()].view(t.shape))
        off += t.numel()
    return out


def ordered_sum(t, group=None):
    """Sum of ``t`` over the ranks of ``group`` in rank order (no autograd)."""
    return ordered_sum_many([t], group)[0]


class _RankSum(torch.autograd.Function):
    """y = sum over ranks of x, replicated on every rank; the gradient of a
    loss summed over ranks with respect to each rank's x is again the sum
    over ranks of the gradients at y."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return ordered_sum(x, group)

    @staticmethod
    def backward(ctx, g):
        return ordered_sum(g, ctx.group), None


def rank_sum(x, group=None):
    return _RankSum.apply(x, group)


class _RankSumMany(torch.autograd.Function):
    """Several tensors summed over the ranks through one all-gather, and
    their gradients likewise through one all-gather in the backward."""

    @staticmethod
    def forward(ctx, group, *xs):
        ctx.group = group
        ctx.like = [(x.shape, x.dtype, x.device) for x in xs]
        return tuple(ordered_sum_many(list(xs), group))

    @staticmethod
    def backward(ctx, *gs):
        # every rank takes the same collective, so a missing gradient is a zero one
        gs = [g if g is not None else torch.zeros(sh, dtype=dt, device=dv)
              for g, (sh, dt, dv) in zip(gs, ctx.like)]
        return (None,) + tuple(ordered_sum_many(gs, ctx.group))


def rank_sum_many(xs, group=None):
    """``rank_sum`` of each tensor of ``xs`` with one collective each way."""
    return _RankSumMany.apply(group, *xs)


def sharded_slice(x_mid, fx_mid, weight, bias, tau, group=None, slice_fn=None):
    """``fused_slice`` of this rank's points, summed over the ranks: returns
    the global z_num (B, H, G, DV) and s (B, H, G) on every rank.
    ``slice_fn`` replaces ``fused_slice`` (tests run the host logic on CPU
    ranks with the eager reference in its place)."""
    if slice_fn is None:
        from .kernels import fused_slice as slice_fn
    z_num, s = slice_fn(x_mid, fx_mid, weight, bias, tau)
    z_num, s = rank_sum_many([z_num, s], group)
    return z_num, s


def sharded_coupling(x_mid, fx_mid, weight, bias, tau, mix=None, eps=1e-5, group=None,
                     slice_fn=None, deslice_fn=None):
    """slice -> z_num / (s + eps) -> mix (None = identity) -> deslice over the
    rank's points; the output rows are this rank's points."""
    if deslice_fn is None:
        from .kernels import fused_deslice as deslice_fn
    z_num, s = sharded_slice(x_mid, fx_mid, weight, bias, tau, group, slice_fn)
    tokens = z_num / (s + eps)[..., None]
    if mix is not None:
        tokens = mix(tokens)
    return deslice_fn(x_mid, weight, bias, tau, tokens)


def reduce_grads(params, group=None):
    """Sum the gradients of replicated parameters over the ranks, in rank
    order, in place (the data-parallel gradient of the sharded coupling);
    one all-gather for all of them."""
    grads = [p.grad for p in params if p is not None and p.grad is not None]
    if not grads:
        return
    for g, tot in zip(grads, ordered_sum_many(grads, group)):
        g.copy_(tot)
