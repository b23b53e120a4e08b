"""fused_coupling: one slice -> tokens -> deslice round with the tied
backward (dtokens pass + one coupled kernel), against the float64 eager
round, the exact-fp32 FMA engine and the plain op-by-op composition."""

import pytest
import torch

from parity import relerr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    import flashslice_b200.kernels as K
    from flashslice_b200.kernels import _native as nat
    from flashslice_b200.kernels import _state
    lib = nat.load()
    lib.fs_device_status(1)
    return K, _state, lib


def _inputs(N, mode, B=1, H=4, D=32, seed=5):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    x, fx = r(B, N, H, D), r(B, N, H, D)
    W = {"gd": r(32, D), "hgd": r(H, 32, D), "bhgd": r(B, H, 32, D)}[mode] / D ** 0.5
    b = {"gd": r(32), "hgd": r(H, 32), "bhgd": r(B, H, 32)}[mode] * 0.1
    tau = 0.3 + 0.7 * torch.rand(H, generator=g, dtype=torch.float64)
    rr = r(B, N, H, D)
    return [t.cuda() for t in (x, fx, W, b, tau, rr)]


def _leaves(ts):
    return [t.detach().float().clone().requires_grad_(True) for t in ts]


def _grads(out, leaves, r, extra=()):
    out.backward(r.float())
    torch.cuda.synchronize()
    res = {"out": out.detach()}
    for k, v in zip(("x", "fx", "W", "b", "tau") + tuple("p%d" % i for i in range(len(extra))),
                    tuple(leaves) + tuple(extra)):
        res["grad:" + k] = v.grad
    return res


def _coupled(K, x, fx, W, b, tau, r, mix=None, params=()):
    L = _leaves((x, fx, W, b, tau))
    out = K.fused_coupling(*L, mix=mix, mix_params=list(params))
    return _grads(out, L, r, params)


def _composed(K, x, fx, W, b, tau, r, mix=None, params=()):
    L = _leaves((x, fx, W, b, tau))
    z, s = K.fused_slice(*L)
    tok = z / (s + 1e-5)[..., None]
    if mix is not None:
        tok = mix(tok)
    out = K.fused_deslice(L[0], L[2], L[3], L[4], tok)
    return _grads(out, L, r, params)


@pytest.mark.parametrize("N", [77, 4097, 100_003])
@pytest.mark.parametrize("mode", ["gd", "hgd", "bhgd"])
def test_coupling_matches_eager(env, N, mode):
    """Forward and every gradient of a round: the tied backward against the
    float64 eager round, gated like the op-by-op rounds (within 1e-5 of the
    exact FMA engine, or as close to the truth as it)."""
    K, st, lib = env
    x, fx, W, b, tau, r = _inputs(N, mode, B=2 if mode == "bhgd" else 1)
    n0 = lib.fs_tc_launch_count()
    tc = _coupled(K, x, fx, W, b, tau, r)
    # slice, deslice, the dtokens pass and the coupled backward
    assert lib.fs_tc_launch_count() - n0 == 4, "the tensor-core kernels did not run"
    st.set_engine("fma")
    try:
        ex = _composed(K, x, fx, W, b, tau, r)
    finally:
        st.set_engine("auto")
    from oracle import eager_torch as E
    ref = E.coupling_round(*[t.detach().clone().requires_grad_(True)
                             for t in (x, fx, W, b, tau)], r)
    for k in ("out", "grad:x", "grad:fx", "grad:W", "grad:b", "grad:tau"):
        et, ee = relerr(tc[k], ref[k]), relerr(ex[k], ref[k])
        assert relerr(tc[k], ex[k]) <= 1e-5 or et <= 1.25 * ee + 1e-6, (k, et, ee)
    assert lib.fs_device_status(1) == 0


def test_coupling_with_mix(env):
    """A mix with a parameter between the normalisation and the deslice: the
    tied round's gradients (the mix parameter's included) against the
    op-by-op composition through autograd."""
    K, st, lib = env
    x, fx, W, b, tau, r = _inputs(20_000, "hgd", B=2, H=8)
    g = torch.Generator().manual_seed(11)
    M0 = (torch.eye(32, dtype=torch.float64)
          + 0.1 * torch.randn(32, 32, generator=g, dtype=torch.float64)).cuda()
    res = []
    for fn in (_coupled, _composed):
        M = M0.float().clone().requires_grad_(True)
        res.append(fn(K, x, fx, W, b, tau, r, mix=lambda t, M=M: t @ M, params=(M,)))
    tc, ref = res
    for k in ref:
        assert relerr(tc[k], ref[k]) <= 1e-5, (k, relerr(tc[k], ref[k]))
    assert lib.fs_device_status(1) == 0


def test_coupling_unsupported_shape(env):
    """D = DV = 64 is outside the coupled kernel: the tied round forms
    dtokens with the slice forward and then runs the two backward ops and
    adds (the exact FMA kernels); it agrees with the op-by-op round to
    rounding."""
    K, st, lib = env
    x, fx, W, b, tau, r = _inputs(5000, "hgd", D=64)
    n0 = lib.fs_tc_launch_count()
    tc = _coupled(K, x, fx, W, b, tau, r)
    assert lib.fs_tc_launch_count() == n0
    ref = _composed(K, x, fx, W, b, tau, r)
    for k in ref:
        assert relerr(tc[k], ref[k]) <= 1e-5, (k, relerr(tc[k], ref[k]))


def test_coupling_strided_and_deterministic(env):
    K, st, lib = env
    x, fx, W, b, tau, r = _inputs(30_000, "gd", B=1, H=8)
    xs = x.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    a = _coupled(K, xs, fx, W, b, tau, r)
    c = _coupled(K, xs, fx, W, b, tau, r)
    for k in a:
        assert torch.equal(a[k], c[k]), k
    ref = _composed(K, x, fx, W, b, tau, r)
    for k in ref:
        assert relerr(a[k], ref[k]) <= 1e-5, (k, relerr(a[k], ref[k]))
    assert lib.fs_device_status(1) == 0


def test_coupled_bwd_abi_refuses_unsupported(env):
    """The C entry point reports shapes it does not serve instead of
    computing them (FS_ERR_UNSUPPORTED), and says which ones it serves."""
    K, st, lib = env
    import ctypes
    from flashslice_b200.kernels import _native as nat
    p = nat.Problem(1, 100, 2, 64, 64, 32, 0, 0, nat.FAMILY_SINGLE, 0, 1, 1, 1, 1, 0, 0)
    assert lib.fs_coupled_supported(ctypes.byref(p)) == 0
    p = nat.Problem(1, 100, 2, 32, 32, 32, 0, 0, nat.FAMILY_SINGLE, 0, 1, 1, 1, 1, 0, 0)
    assert lib.fs_coupled_supported(ctypes.byref(p)) == 1
    p.engine = nat.ENGINE_FMA
    assert lib.fs_coupled_supported(ctypes.byref(p)) == 0


def test_rank_sum_native(env):
    """fs_rank_sum: the rank-order sum of a gathered (world, n) buffer, bitwise
    the sequential fold (rank 0 + rank 1 + ...), one native launch."""
    K, st, lib = env
    from flashslice_b200 import sharded
    g = torch.Generator(device="cuda").manual_seed(3)
    for world, n in [(2, 1), (3, 1000), (8, 33_825)]:
        buf = torch.randn(world, n, device="cuda", generator=g)
        n0 = lib.fs_launch_count()
        got = sharded._fold(buf)
        assert lib.fs_launch_count() - n0 == 1
        ref = buf[0].clone()
        for r in range(1, world):
            ref += buf[r]
        assert torch.equal(got, ref)
