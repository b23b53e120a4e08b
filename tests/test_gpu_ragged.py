"""Ragged batches (samples of different N packed along the point axis, one
launch per op): every result against the dense ops applied sample by sample
and against the float64 eager math, gradients included; the tensor-core
kernels run once per op for all samples."""

import pytest
import torch

from parity import relerr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    import flashslice_b200.kernels as K
    from flashslice_b200.kernels import _native as nat
    from flashslice_b200.kernels import ragged as R
    lib = nat.load()
    lib.fs_device_status(1)
    return K, R, lib


def _inputs(lens, mode, H=4, D=32, seed=9):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    S, N = len(lens), sum(lens)
    x, fx, up = r(1, N, H, D), r(1, N, H, D), r(1, N, H, D)
    W = {"gd": r(32, D), "hgd": r(H, 32, D), "bhgd": r(S, H, 32, D)}[mode] / D ** 0.5
    b = {"gd": r(32), "hgd": r(H, 32), "bhgd": r(S, H, 32)}[mode] * 0.1
    tau = 0.3 + 0.7 * torch.rand(H, generator=g, dtype=torch.float64)
    splits = [0]
    for n in lens:
        splits.append(splits[-1] + n)
    return [t.cuda() for t in (x, fx, W, b, tau, up)], splits


def _eager_round(x, fx, W, b, tau, splits, mix=None):
    from oracle import eager_torch as E
    S = len(splits) - 1
    outs = []
    for i in range(S):
        a, e = splits[i], splits[i + 1]
        Wi = W[i:i + 1] if W.dim() == 4 else W
        bi = b[i:i + 1] if b.dim() == 3 else b
        z, s = E.slice_fwd(x[:, a:e], fx[:, a:e], Wi, bi, tau)
        tok = z / (s + 1e-5)[..., None]
        if mix is not None:
            tok = mix(tok)
        outs.append(E.deslice_fwd(x[:, a:e], Wi, bi, tau, tok))
    return torch.cat(outs, dim=1)


LENS = [77, 4097, 0, 128, 1, 20_000]


@pytest.mark.parametrize("mode", ["gd", "hgd", "bhgd"])
def test_ragged_coupling(env, mode):
    K, R, lib = env
    (x, fx, W, b, tau, up), splits = _inputs(LENS, mode)
    leaves = [t.float().clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
    n0 = lib.fs_tc_launch_count()
    out = R.ragged_coupling(*leaves, splits)
    (out * up.float()).sum().backward()
    torch.cuda.synchronize()
    # slice, deslice, the dtokens pass, the coupled backward: once each for all samples
    assert lib.fs_tc_launch_count() - n0 == 4
    ref_leaves = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
    ref = _eager_round(*ref_leaves, splits)
    (ref * up).sum().backward()
    assert relerr(out, ref) <= 1e-5
    for a, e, name in zip(leaves, ref_leaves, ("x", "fx", "W", "b", "tau")):
        assert relerr(a.grad, e.grad) <= 2e-5, (name, relerr(a.grad, e.grad))
    assert lib.fs_device_status(1) == 0


def test_ragged_ops_match_dense_per_sample(env):
    """ragged_slice / ragged_deslice (op by op, their own backward) against
    the dense ops on each sample: equal to rounding."""
    K, R, lib = env
    (x, fx, W, b, tau, up), splits = _inputs([300, 5000, 129], "bhgd", seed=4)
    x, fx, W, b, tau, up = (t.float() for t in (x, fx, W, b, tau, up))
    g = torch.Generator(device="cuda").manual_seed(1)
    tok = torch.randn(3, 4, 32, 32, device="cuda", generator=g)
    L = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau, tok)]
    z, s = R.ragged_slice(L[0], L[1], L[2], L[3], L[4], splits)
    out = R.ragged_deslice(L[0], L[2], L[3], L[4], L[5], splits)
    ((out * up).sum() + (z * tok).sum() + s.sum()).backward()
    D = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau, tok)]
    zs, ss, outs = [], [], []
    for i in range(3):
        a, e = splits[i], splits[i + 1]
        zi, si = K.fused_slice(D[0][:, a:e], D[1][:, a:e], D[2][i:i + 1], D[3][i:i + 1], D[4])
        zs.append(zi), ss.append(si)
        outs.append(K.fused_deslice(D[0][:, a:e], D[2][i:i + 1], D[3][i:i + 1], D[4],
                                    D[5][i:i + 1]))
    zd, sd, od = torch.cat(zs), torch.cat(ss), torch.cat(outs, dim=1)
    ((od * up).sum() + (zd * tok).sum() + sd.sum()).backward()
    for a, e in ((z, zd), (s, sd), (out, od)):
        assert relerr(a, e) <= 1e-6
    for a, e in zip(L, D):
        assert relerr(a.grad, e.grad) <= 1e-5


def test_ragged_with_mix_and_fallback(env):
    """A mix between the ops (per-sample token attention stand-in), and a
    shape the tensor cores do not serve (D = 64: the samples run one by one
    on the exact kernels) -- both against the eager math."""
    K, R, lib = env
    g = torch.Generator().manual_seed(21)
    M0 = (torch.eye(32, dtype=torch.float64) + 0.1 * torch.randn(32, 32, generator=g,
                                                                dtype=torch.float64)).cuda()
    for D in (32, 64):
        (x, fx, W, b, tau, up), splits = _inputs([1000, 3, 2500], "hgd", D=D, seed=D)
        if D == 64:
            fx = fx[..., :32].contiguous()
            up = up[..., :32].contiguous()
        M = M0.float().clone().requires_grad_(True)
        leaves = [t.float().clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
        out = R.ragged_coupling(*leaves, splits, mix=lambda t: t @ M, mix_params=[M])
        (out * up.float()).sum().backward()
        Md = M0.clone().requires_grad_(True)
        ref_leaves = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
        ref = _eager_round(*ref_leaves, splits, mix=lambda t: t @ Md)
        (ref * up).sum().backward()
        assert relerr(out, ref) <= 1e-5, (D, relerr(out, ref))
        for a, e in zip(leaves + [M], ref_leaves + [Md]):
            assert relerr(a.grad, e.grad) <= 5e-5, (D, relerr(a.grad, e.grad))


def test_ragged_coupling_bf16(env):
    """bf16 samples in one launch per op: against the dense bf16 rounds run
    sample by sample (the same kernels per sample)."""
    K, R, lib = env
    (x, fx, W, b, tau, up), splits = _inputs([333, 4000, 1], "hgd", seed=31)
    x, fx, up = x.bfloat16(), fx.bfloat16(), up.bfloat16()
    W, b, tau = W.float(), b.float(), tau.float()
    L = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
    n0 = lib.fs_tc_launch_count()
    out = R.ragged_coupling(*L, splits)
    (out.float() * up.float()).sum().backward()
    assert lib.fs_tc_launch_count() - n0 == 4 and out.dtype == torch.bfloat16
    D = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
    outs = [K.fused_coupling(D[0][:, a:e], D[1][:, a:e], D[2], D[3], D[4])
            for a, e in zip(splits[:-1], splits[1:])]
    od = torch.cat(outs, dim=1)
    (od.float() * up.float()).sum().backward()
    assert relerr(out, od) <= 1e-2
    for a, e in zip(L, D):
        assert relerr(a.grad, e.grad) <= (1e-2 if a.dtype == torch.bfloat16 else 1e-4)
