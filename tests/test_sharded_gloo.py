"""The point-sharded coupling's host logic on two CPU ranks (gloo): the point
ranges, the rank-ordered sums, the op-by-op sharded round and the tied round
(``fused_coupling(group=...)``) with eager stand-ins for the native ops,
against the same round on one process."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import eager_torch as E


class EagerOps:
    """float64 eager stand-ins for the three ops fused_coupling calls."""

    @staticmethod
    def flash_slice(x, fx, W, b, tau, dot):
        return E.slice_fwd(x, fx, W, b, tau)

    @staticmethod
    def flash_deslice(x, W, b, tau, tok, dot):
        return E.deslice_fwd(x, W, b, tau, tok)

    @staticmethod
    def coupled_bwd(x, fx, d_out, W, b, tau, tok, dz, ds, dot):
        L = [t.detach().clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
        with torch.enable_grad():
            z, s = E.slice_fwd(*L)
            out = E.deslice_fwd(L[0], L[2], L[3], L[4], tok)
            loss = (out * d_out).sum() + (z * dz).sum() + (s * ds).sum()
            return torch.autograd.grad(loss, L)


def _inputs(N=61, B=1, H=2, D=8, G=5, seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    return (r(B, N, H, D), r(B, N, H, D), r(H, G, D) / D ** 0.5, 0.1 * r(H, G),
            0.3 + 0.7 * torch.rand(H, generator=g, dtype=torch.float64), r(B, N, H, D),
            torch.eye(D, dtype=torch.float64) + 0.1 * r(D, D))


def _round(fn, x, fx, W, b, tau, r, M, tied=False, **kw):
    L = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
    Mp = M.clone().requires_grad_(True)
    if tied:  # the tied round returns gradients for the mix parameters it is given
        kw["mix_params"] = [Mp]
    out = fn(*L, mix=lambda t: t @ Mp, **kw)
    (out * r).sum().backward()
    return out.detach(), [t.grad for t in L] + [Mp.grad]


def _plain(v, back=False):
    """Tensors <-> numpy arrays, recursively: results cross the queue by value
    (a tensor is passed as a file descriptor that the parent fetches from the
    child, which may have exited by then)."""
    if isinstance(v, dict):
        return {k: _plain(u, back) for k, u in v.items()}
    if isinstance(v, (list, tuple)):
        return type(v)(_plain(u, back) for u in v)
    if back and isinstance(v, np.ndarray):
        return torch.from_numpy(v)
    if not back and isinstance(v, torch.Tensor):
        return v.detach().numpy().copy()
    return v


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from flashslice_b200 import sharded
        from flashslice_b200.kernels import fused_coupling
        x, fx, W, b, tau, r, M = _inputs()
        N = x.shape[1]
        lo, hi = sharded.shard_range(N, rank, world)
        xs, fs, rs = x[:, lo:hi], fx[:, lo:hi], r[:, lo:hi]
        res = {"range": (lo, hi)}
        # rank-ordered sum: identical on every rank
        res["osum"] = sharded.ordered_sum(torch.full((3,), float(rank + 1), dtype=torch.float64))
        # several tensors through one gather, shapes kept
        res["osum_many"] = sharded.ordered_sum_many(
            [torch.full((2, 3), float(rank + 1), dtype=torch.float64),
             torch.arange(4, dtype=torch.float64) * (rank + 1)])
        # op-by-op sharded round with eager ops
        out1, g1 = _round(lambda *a, mix, **k: sharded.sharded_coupling(
            *a, mix=mix, slice_fn=E.slice_fwd, deslice_fn=E.deslice_fwd), xs, fs, W, b, tau, rs, M)
        # tied round, sharded, with eager stand-ins for the native ops
        out2, g2 = _round(fused_coupling, xs, fs, W, b, tau, rs, M, tied=True,
                          group=dist.group.WORLD, _ops=EagerOps)
        for g in (g1, g2):  # the data-parallel sum of the replicated parameters' gradients
            for i in (2, 3, 4, 5):
                g[i] = sharded.ordered_sum(g[i])
        res.update(out1=out1, g1=g1, out2=out2, g2=g2)
        q.put((rank, _plain(res)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = {r: _plain(v, back=True) for r, v in (q.get(timeout=180) for _ in procs)}
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


@pytest.fixture(scope="module")
def two_ranks():
    # a second try with a fresh port: the port picked free can be taken by
    # another process before the ranks bind it
    try:
        res = _run_ranks()
        if any(isinstance(v, str) for v in res.values()):
            res = _run_ranks()
    except (EOFError, OSError):
        res = _run_ranks()
    for r, v in res.items():
        assert not isinstance(v, str), "rank %d failed: %s" % (r, v)
    return res


def test_shard_ranges_cover(two_ranks):
    (a0, b0), (a1, b1) = two_ranks[0]["range"], two_ranks[1]["range"]
    assert a0 == 0 and b0 == a1 and b1 == 61


def test_ordered_sum_replicated(two_ranks):
    assert torch.equal(two_ranks[0]["osum"], two_ranks[1]["osum"])
    assert torch.equal(two_ranks[0]["osum"], torch.full((3,), 3.0, dtype=torch.float64))
    a, b = two_ranks[0]["osum_many"], two_ranks[1]["osum_many"]
    assert all(torch.equal(u, v) for u, v in zip(a, b))
    assert torch.equal(a[0], torch.full((2, 3), 3.0, dtype=torch.float64))
    assert torch.equal(a[1], torch.arange(4, dtype=torch.float64) * 3)


@pytest.mark.parametrize("which", ["1", "2"])
def test_sharded_round_matches_single_process(two_ranks, which):
    from flashslice_b200.kernels import fused_coupling
    x, fx, W, b, tau, r, M = _inputs()
    out, g = _round(fused_coupling, x, fx, W, b, tau, r, M, tied=True, _ops=EagerOps)
    out_ref, g_ref = _round(lambda *a, mix: E.deslice_fwd(
        a[0], a[2], a[3], a[4], mix(E.slice_fwd(*a)[0] / (E.slice_fwd(*a)[1] + 1e-5)[..., None])),
        x, fx, W, b, tau, r, M)
    # the single-process tied round agrees with plain autograd of the eager round
    assert torch.allclose(out, out_ref, rtol=1e-12, atol=1e-12)
    for a, c in zip(g, g_ref):
        assert torch.allclose(a, c, rtol=1e-10, atol=1e-12)
    r0, r1 = two_ranks[0], two_ranks[1]
    cat = torch.cat([r0["out" + which], r1["out" + which]], dim=1)
    assert torch.allclose(cat, out, rtol=1e-12, atol=1e-12)
    gx = torch.cat([r0["g" + which][0], r1["g" + which][0]], dim=1)
    gf = torch.cat([r0["g" + which][1], r1["g" + which][1]], dim=1)
    assert torch.allclose(gx, g[0], rtol=1e-10, atol=1e-12)
    assert torch.allclose(gf, g[1], rtol=1e-10, atol=1e-12)
    for i in (2, 3, 4, 5):  # W, b, tau and the mix parameter, summed over the ranks
        assert torch.equal(r0["g" + which][i], r1["g" + which][i])
        assert torch.allclose(r0["g" + which][i], g[i], rtol=1e-10, atol=1e-12), i
