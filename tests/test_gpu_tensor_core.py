"""The tensor-core (tcgen05) kernels against the exact-fp32 FMA kernels and
the float64 truth, on the shapes they serve (fp32, D = DV = G = 32), with
ragged point counts, strided inputs and every weight layout; plus proof that
the tensor-core path actually ran and that no bounded device wait gave up."""

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


def _inputs(N, mode, B=1, H=4, seed=3, strided=False):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    x, fx = r(B, N, H, 32), r(B, N, H, 32)
    if strided:
        x = x.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    W = {"gd": r(32, 32), "hgd": r(H, 32, 32), "bhgd": r(B, H, 32, 32)}[mode] / 32 ** 0.5
    b = {"gd": r(32), "hgd": r(H, 32), "bhgd": r(B, H, 32)}[mode] * 0.1
    tau = 0.3 + 0.7 * torch.rand(H, generator=g, dtype=torch.float64)
    tok = r(B, H, 32, 32)
    return [t.cuda() for t in (x, fx, W, b, tau, tok)]


def _run(K, st, engine, x, fx, W, b, tau, tok):
    st.set_engine(engine)
    try:
        f = [t.float() for t in (x, fx, W, b, tau, tok)]  # .float() keeps x's strides
        z, s = K.fused_slice(f[0], f[1], f[2], f[3], f[4])
        out = K.fused_deslice(f[0], f[2], f[3], f[4], f[5])
        torch.cuda.synchronize()
        return z, s, out
    finally:
        st.set_engine("auto")


@pytest.mark.parametrize("N", [1, 77, 128, 129, 4097, 100_003])
@pytest.mark.parametrize("mode", ["gd", "hgd", "bhgd"])
def test_forward_matches_exact_engine(env, N, mode):
    K, st, lib = env
    x, fx, W, b, tau, tok = _inputs(N, mode, B=2 if mode == "bhgd" else 1)
    n0 = lib.fs_tc_launch_count()
    tc = _run(K, st, "auto", x, fx, W, b, tau, tok)
    assert lib.fs_tc_launch_count() - n0 == 2, "the tensor-core kernels did not run"
    n1 = lib.fs_tc_launch_count()
    ex = _run(K, st, "fma", x, fx, W, b, tau, tok)
    assert lib.fs_tc_launch_count() == n1
    from oracle import eager_torch as E
    z64, s64 = E.slice_fwd(x, fx, W, b, tau)
    o64 = E.deslice_fwd(x, W, b, tau, tok)
    for name, a, e, ref in (("z_num", tc[0], ex[0], z64), ("s", tc[1], ex[1], s64),
                            ("out", tc[2], ex[2], o64)):
        et, ee = relerr(a, ref), relerr(e, ref)
        # the tensor-core split products are at least as accurate as fp32 FMA
        assert et <= max(2.0 * ee, 1e-6), (name, et, ee)
        assert relerr(a, e) <= 1e-5, (name, relerr(a, e))
    assert lib.fs_device_status(1) == 0


def test_forward_strided_input(env):
    K, st, lib = env
    x, fx, W, b, tau, tok = _inputs(5000, "hgd", B=2, strided=True)
    assert not x.is_contiguous()
    n0 = lib.fs_tc_launch_count()
    tc = _run(K, st, "auto", x, fx, W, b, tau, tok)
    assert lib.fs_tc_launch_count() - n0 == 2
    ex = _run(K, st, "fma", x, fx, W, b, tau, tok)
    for a, e in zip(tc, ex):
        assert relerr(a, e) <= 1e-5
    assert lib.fs_device_status(1) == 0


def test_forward_deterministic(env):
    K, st, lib = env
    x, fx, W, b, tau, tok = _inputs(300_000, "hgd", B=1, H=8)
    a = _run(K, st, "auto", x, fx, W, b, tau, tok)
    c = _run(K, st, "auto", x, fx, W, b, tau, tok)
    for u, v in zip(a, c):
        assert torch.equal(u, v)


def _round(K, st, engine, leaves, r):
    """slice -> normalise -> deslice, forward and backward of sum(out * r)."""
    st.set_engine(engine)
    try:
        L = [t.detach().float().requires_grad_(True) for t in leaves]
        x, fx, W, b, tau = L
        z, s = K.fused_slice(x, fx, W, b, tau)
        out = K.fused_deslice(x, W, b, tau, z / (s + 1e-5)[..., None])
        out.backward(r.float())
        torch.cuda.synchronize()
        res = {"out": out.detach(), "z_num": z.detach(), "s": s.detach()}
        for k, v in zip(("x", "fx", "W", "b", "tau"), L):
            res["grad:" + k] = v.grad
        return res
    finally:
        st.set_engine("auto")


@pytest.mark.parametrize("N", [77, 4097, 100_003])
@pytest.mark.parametrize("mode", ["gd", "hgd", "bhgd"])
def test_round_matches_exact_engine(env, N, mode):
    """Forward and backward of a coupling round on the tensor-core kernels
    against the exact FMA kernels and the float64 eager reference."""
    K, st, lib = env
    x, fx, W, b, tau, _ = _inputs(N, mode, B=2 if mode == "bhgd" else 1)
    r = torch.randn(x.shape, generator=torch.Generator().manual_seed(9),
                    dtype=torch.float64).cuda()
    n0 = lib.fs_tc_launch_count()
    tc = _round(K, st, "auto", (x, fx, W, b, tau), r)
    assert lib.fs_tc_launch_count() - n0 == 4, "the tensor-core kernels did not run"
    ex = _round(K, st, "fma", (x, fx, W, b, tau), r)
    from oracle import eager_torch as E
    L = [t.detach().clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
    ref = E.coupling_round(*L, r)
    for k in ref:
        et, ee = relerr(tc[k], ref[k]), relerr(ex[k], ref[k])
        assert relerr(tc[k], ex[k]) <= 1e-5 or et <= 1.25 * ee + 1e-6, (k, et, ee)
    assert lib.fs_device_status(1) == 0


def test_round_deterministic(env):
    K, st, lib = env
    x, fx, W, b, tau, _ = _inputs(200_000, "hgd", B=1, H=8)
    r = torch.randn(x.shape, generator=torch.Generator().manual_seed(2),
                    dtype=torch.float64).cuda()
    a = _round(K, st, "auto", (x, fx, W, b, tau), r)
    c = _round(K, st, "auto", (x, fx, W, b, tau), r)
    for k in a:
        assert torch.equal(a[k], c[k]), k


def test_bounded_wait_reports_and_context_survives(env):
    """A device-side wait that runs out (an mbarrier nothing arrives at, 5 ms
    limit) sets the status word, its kernel returns, and the same context
    then runs the tensor-core kernels correctly: failure detection without a
    GPU fault."""
    import ctypes
    K, st, lib = env
    from flashslice_b200.kernels import _native as nat
    assert lib.fs_device_status(1) == 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nat.check(lib.fs_selftest_wait_timeout(5_000_000, stream))
    assert lib.fs_device_status(1) == 1
    assert lib.fs_device_status(0) == 0
    x, fx, W, b, tau, tok = _inputs(4097, "hgd")
    tc = _run(K, st, "auto", x, fx, W, b, tau, tok)
    ex = _run(K, st, "fma", x, fx, W, b, tau, tok)
    for a, e in zip(tc, ex):
        assert relerr(a, e) <= 1e-5
    assert lib.fs_device_status(1) == 0


def _tied(K, leaves, r):
    """fused_coupling forward and backward of sum(out * r)."""
    L = [t.detach().float().requires_grad_(True) for t in leaves]
    out = K.fused_coupling(*L, eps=1e-5)
    out.backward(r.float())
    torch.cuda.synchronize()
    res = {"out": out.detach()}
    for k, v in zip(("x", "fx", "W", "b", "tau"), L):
        res["grad:" + k] = v.grad
    return res


def test_real_kernels_waits_run_out_and_context_survives(env):
    """The failure path of the real tensor-core kernels, made on a healthy
    GPU: their device-side waits get a 100 ns limit (the TMA loads and MMAs
    take longer), so they give up. The status word is set, every later wait
    of a thread that gave up returns at once, the issuing thread stops issuing
    and lets what it issued land, and the kernels return within a bound; with
    the default limit back, the same context computes correctly. Covers the
    tied rounds at G = 32 and G = 64 (slice, deslice, dtokens pass, coupled
    backward)."""
    import time
    K, st, lib = env
    from flashslice_b200.kernels import _native as nat
    from oracle import eager_torch as E
    assert lib.fs_device_status(1) == 0
    x, fx, W, b, tau, tok = _inputs(200_000, "hgd", H=8)
    W64 = torch.cat([W, W.flip(1)], dim=1)
    b64 = torch.cat([b, -b], dim=1)
    r = torch.randn(x.shape, generator=torch.Generator().manual_seed(2),
                    dtype=torch.float64).cuda()
    torch.cuda.synchronize()
    nat.check(lib.fs_set_wait_limit_ns(100))
    try:
        t0 = time.monotonic()
        n0 = lib.fs_tc_launch_count()
        _tied(K, (x, fx, W, b, tau), r)
        _tied(K, (x, fx, W64, b64, tau), r)
        waited = time.monotonic() - t0
        assert lib.fs_tc_launch_count() - n0 == 8
    finally:
        nat.check(lib.fs_set_wait_limit_ns(0))
    assert lib.fs_device_status(1) == 1
    assert waited < 60, waited
    for WW, bb in ((W, b), (W64, b64)):
        tc = _tied(K, (x, fx, WW, bb, tau), r)
        st.set_engine("fma")
        try:
            ex = _round(K, st, "fma", (x, fx, WW, bb, tau), r)
        finally:
            st.set_engine("auto")
        ref = E.coupling_round(*[t.detach().clone().requires_grad_(True)
                                 for t in (x, fx, WW, bb, tau)], r)
        for k in tc:
            et, ee = relerr(tc[k], ref[k]), relerr(ex[k], ref[k])
            assert relerr(tc[k], ex[k]) <= 1e-5 or et <= 1.25 * ee + 1e-6, (k, et, ee)
    assert lib.fs_device_status(1) == 0
