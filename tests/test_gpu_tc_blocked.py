"""The blocked family on the tensor cores (bf16 point tensors, bf16 dot
mode, D = 32, DV = 32 or 64, G a multiple of 128): the slot-owning slice
forward and backward halves, the point-owning deslice forward and backward
halves, against the exact FMA kernels on the same inputs and statistics
and against the float64 math (the reference's bf16 gate, 2e-2)."""

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
    # the statistics (operand images, point-owning kernel), the slot-owning slice
    assert lib.fs_tc_launch_count() - n0 == 3, "the tensor-core kernels did not run"
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
    # the slice forward's statistics and slot-owning kernel; the deslice
    # forward, called here without statistics: its own (images, statistics)
    # and then its images and kernel; each backward op's images,
    # point-owning and slot-owning halves
    assert lib.fs_tc_launch_count() - n0 == 3 + 4 + 3 + 3
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


@pytest.mark.parametrize("case", [
    dict(B=1, N=5000, H=4, DV=64, G=128, mode="hgd", bias=True),
    dict(B=2, N=4097, H=2, DV=32, G=256, mode="bhgd", bias=False),
    dict(B=1, N=77, H=4, DV=64, G=1024, mode="gd", bias=True),
], ids=["g128-hgd", "g256-bhgd-dv32", "g1024-n77"])
def test_blocked_deslice_forward_on_tensor_cores(env, case):
    """The deslice forward with the slice's statistics handed in: the
    point-owning tensor-core kernel against the FMA kernel on the same
    statistics and the float64 math; repeated calls agree bitwise."""
    K, st, lib = env
    x, fx, W, b, tau = _inputs(**case)
    g = torch.Generator().manual_seed(5)
    tok = torch.randn(case["B"], case["H"], case["G"], case["DV"], generator=g).cuda()
    _, _, stats = K.fused_slice(x, fx, W, b, tau, return_stats=True)
    n0 = lib.fs_tc_launch_count()
    out = K.fused_deslice(x, W, b, tau, tok, stats=stats)
    torch.cuda.synchronize()
    assert lib.fs_tc_launch_count() - n0 == 2, "the tensor-core kernels did not run"
    assert out.dtype == torch.bfloat16
    # without statistics (the deslice -> slice order): formed on the tensor
    # cores first, then the same kernel; they match the slice's
    n1 = lib.fs_tc_launch_count()
    out_o, st_o = K.fused_deslice(x, W, b, tau, tok, return_stats=True)
    torch.cuda.synchronize()
    assert lib.fs_tc_launch_count() - n1 == 4
    assert torch.equal(st_o, stats) and torch.equal(out_o, out)
    out2 = K.fused_deslice(x, W, b, tau, tok, stats=stats)
    assert torch.equal(out, out2)
    st.set_engine("fma")
    try:
        oe = K.fused_deslice(x, W, b, tau, tok, stats=stats)
    finally:
        st.set_engine("auto")
    assert relerr(out, oe) <= 1e-2, relerr(out, oe)
    from oracle import eager_torch as E
    bb = b if b is not None else torch.zeros(W.shape[-2], device="cuda")
    ot = E.deslice_fwd(x.double(), W.double(), bb.double(), tau.double(), tok.double())
    assert relerr(out, ot) <= 2e-2, relerr(out, ot)
    assert lib.fs_device_status(1) == 0


@pytest.mark.parametrize("case", [
    dict(B=1, N=5000, H=4, DV=64, G=128, mode="hgd", bias=True),
    dict(B=2, N=4097, H=2, DV=32, G=1024, mode="bhgd", bias=False),
], ids=["g128", "g1024-dv32"])
def test_blocked_statistics_on_tensor_cores(env, case):
    """The per-point statistics on the tensor cores, online (one pass, the
    default stats mode) and two-pass (logits from W in two bf16 parts,
    within 2^-17 of each product), against the FMA engine's exact-fp32 ones:
    m and l to about 1e-5 relative, two to three orders below the bf16 dot
    mode's own rounding; the two modes' m bitwise equal (a max is exact)
    (``parity_ops.py:213-235``)."""
    from flashslice_b200.kernels.blocked import set_stats_mode
    K, st, lib = env
    x, fx, W, b, tau = _inputs(**case)
    got = {}
    try:
        for mode in ("online", "two-pass"):
            set_stats_mode(mode)
            n0 = lib.fs_tc_launch_count()
            _, _, got[mode] = K.fused_slice(x, fx, W, b, tau, return_stats=True)
            torch.cuda.synchronize()
            assert lib.fs_tc_launch_count() - n0 == 3
            st.set_engine("fma")
            try:
                _, _, s_fma = K.fused_slice(x, fx, W, b, tau, return_stats=True)
            finally:
                st.set_engine("auto")
            m, mf = got[mode][:, :, 0], s_fma[:, :, 0]
            dm = float((m - mf).abs().max())
            assert dm <= 1e-5 * (1 + float(mf.abs().max())), (mode, dm)
            l, lf = got[mode][:, :, 1], s_fma[:, :, 1]
            dl = float(((l - lf).abs() / lf).max())
            assert dl <= 1e-4, (mode, dl)
    finally:
        set_stats_mode("online")
    assert torch.equal(got["online"][:, :, 0], got["two-pass"][:, :, 0])
    lo, lt = got["online"][:, :, 1], got["two-pass"][:, :, 1]
    assert float(((lo - lt).abs() / lt).max()) <= 1e-5
    assert lib.fs_device_status(1) == 0


def test_blocked_coupling_round_on_tensor_cores(env):
    """fused_coupling on the blocked family hands the slice's statistics to
    the deslice (as the reference's layer does): every kernel of the round
    on the tensor cores; values against the FMA engine's round."""
    K, st, lib = env
    case = dict(B=2, N=20_000, H=8, DV=64, G=1024, mode="bhgd", bias=False)
    x, fx, W, b, tau = _inputs(**case)
    g = torch.Generator().manual_seed(9)
    up = torch.randn(x.shape[:3] + (64,), generator=g).bfloat16().cuda()
    bb = torch.zeros(W.shape[-2], device="cuda")

    def round_(engine):
        st.set_engine(engine)
        try:
            L = [t.clone().requires_grad_(True) for t in (x, fx, W, bb, tau)]
            out = K.fused_coupling(*L)
            (out.float() * up.float()).sum().backward()
            torch.cuda.synchronize()
            return [out] + [t.grad for t in L]
        finally:
            st.set_engine("auto")

    n0 = lib.fs_tc_launch_count()
    tc = round_("auto")
    # slice forward 3, deslice forward 2, the two backward ops 3 each
    assert lib.fs_tc_launch_count() - n0 == 3 + 2 + 3 + 3
    ex = round_("fma")
    for a, e, k in zip(tc, ex, ("out", "grad:x", "grad:fx", "grad:W", "grad:b", "grad:tau")):
        assert relerr(a, e) <= (2e-2 if k == "grad:tau" else 1e-2), (k, relerr(a, e))
    tc2 = round_("auto")
    for a, a2 in zip(tc, tc2):
        assert torch.equal(a, a2)
    assert lib.fs_device_status(1) == 0
