"""The blocked family's slot-owning slice forward on the tensor cores (bf16
point tensors, bf16 dot mode, D = 32, DV = 32 or 64, G a multiple of 128)
against the exact FMA kernels on the same inputs and statistics and against
the float64 math (the reference's bf16 gate, 2e-2)."""

import pytest
import torch

from parity import relerr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env(cuda_device):
    import flashslice_b200.kernels as K
    from flashslice_b200.kernels import _native as nat
    from flashslice_b200.kernels import _state
    lib = nat.load()
    lib.fs_device_status(1)
    K.set_dot_mode("bf16")
    yield K, _state, lib
    K.set_dot_mode("ieee")


def _inputs(B, N, H, DV, G, mode, bias, seed=3):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    x, fx = r(B, N, H, 32).bfloat16(), r(B, N, H, DV).bfloat16()
    W = {"gd": r(G, 32), "hgd": r(H, G, 32), "bhgd": r(B, H, G, 32)}[mode] / 32 ** 0.5
    b = {"gd": r(G), "hgd": r(H, G), "bhgd": r(B, H, G)}[mode] * 0.1 if bias else None
    tau = 0.3 + 0.7 * torch.rand(H, generator=g, dtype=torch.float64)
    return (x.cuda(), fx.cuda(), W.float().cuda(), None if b is None else b.float().cuda(),
            tau.float().cuda())


@pytest.mark.parametrize("case", [
    dict(B=1, N=5000, H=4, DV=64, G=128, mode="hgd", bias=True),
    dict(B=2, N=4097, H=2, DV=32, G=256, mode="bhgd", bias=False),
    dict(B=1, N=77, H=4, DV=64, G=1024, mode="gd", bias=True),
    dict(B=2, N=20_000, H=8, DV=64, G=1024, mode="bhgd", bias=False),
], ids=["g128-hgd", "g256-bhgd-dv32", "g1024-n77", "g1024-cfg3like"])
def test_blocked_slice_on_tensor_cores(env, case):
    K, st, lib = env
    x, fx, W, b, tau = _inputs(**case)
    n0 = lib.fs_tc_launch_count()
    z, s, stats = K.fused_slice(x, fx, W, b, tau, return_stats=True)
    torch.cuda.synchronize()
    assert lib.fs_tc_launch_count() - n0 == 1, "the tensor-core kernel did not run"
    st.set_engine("fma")
    try:
        ze, se = K.fused_slice(x, fx, W, b, tau, stats=stats)
    finally:
        st.set_engine("auto")
    # the weights w are rounded to bf16 for the value dot (the bf16 dot mode)
    assert relerr(z, ze) <= 1e-2 and relerr(s, se) <= 1e-2, (relerr(z, ze), relerr(s, se))
    from oracle import eager_torch as E
    bb = b if b is not None else torch.zeros(W.shape[-2], device="cuda")
    zt, sdt = E.slice_fwd(x.double(), fx.double(), W.double(), bb.double(), tau.double())
    assert relerr(z, zt) <= 2e-2 and relerr(s, sdt) <= 2e-2
    # statistics handed in take the same path
    n1 = lib.fs_tc_launch_count()
    z2, s2 = K.fused_slice(x, fx, W, b, tau, stats=stats)
    assert lib.fs_tc_launch_count() - n1 == 1
    assert torch.equal(z2, z) and torch.equal(s2, s)
    assert lib.fs_device_status(1) == 0


@pytest.mark.parametrize("case", [
    dict(B=1, N=5000, H=4, DV=64, G=128, mode="hgd", bias=True),
    dict(B=2, N=20_000, H=8, DV=64, G=1024, mode="bhgd", bias=False),
    dict(B=1, N=3001, H=2, DV=32, G=256, mode="gd", bias=True),
], ids=["g128", "g1024-cfg3like", "g256-dv32"])
def test_blocked_round_backward_on_tensor_cores(env, case):
    """A whole op-by-op round (slice, normalise, deslice) and its backward:
    the slot-owning backward kernels (dW, db, dtokens) run on the tensor
    cores; every gradient against the FMA engine and the float64 math."""
    K, st, lib = env
    x, fx, W, b, tau = _inputs(**case)
    g = torch.Generator().manual_seed(8)
    up = torch.randn(x.shape[:3] + (case["DV"],), generator=g).bfloat16().cuda()
    bb = b if b is not None else torch.zeros(W.shape[-2], device="cuda")

    def round_(engine):
        st.set_engine(engine)
        try:
            L = [t.clone().requires_grad_(True) for t in (x, fx, W, bb, tau)]
            z, s = K.fused_slice(*L)
            out = K.fused_deslice(L[0], L[2], L[3], L[4], z / (s + 1e-5)[..., None])
            (out.float() * up.float()).sum().backward()
            torch.cuda.synchronize()
            return [out] + [t.grad for t in L]
        finally:
            st.set_engine("auto")

    n0 = lib.fs_tc_launch_count()
    tc = round_("auto")
    # the slot-owning slice forward, and the slot-owning halves of both backward ops
    assert lib.fs_tc_launch_count() - n0 == 3
    ex = round_("fma")
    from oracle import eager_torch as E
    ref = E.coupling_round(*[t.detach().double().clone().requires_grad_(True)
                             for t in (x, fx, W, bb, tau)], up.double())
    for a, e, k in zip(tc, ex, ("out", "grad:x", "grad:fx", "grad:W", "grad:b", "grad:tau")):
        # the temperature gradient is a sum that cancels: the bf16 rounding of
        # the value dots moves it most (the reference's bf16 gate, 2e-2)
        assert relerr(a, e) <= (2e-2 if k == "grad:tau" else 1e-2), (k, relerr(a, e))
        assert relerr(a, ref[k]) <= 2e-2, (k, relerr(a, ref[k]))
    assert lib.fs_device_status(1) == 0
