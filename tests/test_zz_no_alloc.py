"""The allocation-free slice forward (``fs_slice_fwd_noalloc``) through the C ABI.

Some callers cannot allocate device memory at all -- a host that owns and
pre-plans every device buffer, or an FFI caller with no device allocator at
hand -- so they cannot hand the ordinary entry point its workspace. The
allocation-free variant keeps its partial sums in a static scratch array in
the library. This test checks it against the ordinary workspace entry point
on the same inputs, on two calls in a row (the scratch keeps the last call's
contents, which must not leak into the next), and that a problem whose
partials do not fit the scratch is refused with a clear error.

This file sorts last so that a run stopping at the first failure has run
every other test before it; it also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the fp32 tolerance of the parity tests


def _relerr(a, ref):
    n = ref.double().norm()
    return float((a.double() - ref.double()).norm() / n) if n > 0 else float(a.abs().max())


def _inputs(seed, B=1, N=50_000, H=4, D=32, DV=32, G=32):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)  # noqa: E731
    x, fx = rn(B, N, H, D), rn(B, N, H, DV)
    W, b = rn(H, G, D) / D ** 0.5, 0.02 * rn(H, G)
    tau = 0.3 + 0.7 * torch.rand(H, device="cuda", generator=g)
    return x, fx, W, b, tau


def _problem(nat, x, fx, W):
    B, N, H, D = x.shape
    G = W.shape[-2]
    return nat.Problem(B, N, H, D, fx.shape[3], G, 0, 0, nat.FAMILY_SINGLE, 0, 1, H, 1, H, 0, 0)


def test_noalloc_matches_workspace_entry_point(cuda_device):
    from flashslice_b200.kernels import _native as nat
    lib = nat.load()
    stream = nat.stream_of(torch.empty(1, device="cuda"))
    for seed in (11, 12):  # two calls in a row, different inputs
        x, fx, W, b, tau = _inputs(seed)
        B, N, H, D = x.shape
        G, DV = W.shape[-2], fx.shape[3]
        prob = _problem(nat, x, fx, W)
        nws = lib.fs_workspace_bytes(nat.OP_SLICE_FWD, ctypes.byref(prob))
        ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
        z_ref = torch.empty(B, H, G, DV, device="cuda")
        s_ref = torch.empty(B, H, G, device="cuda")
        nat.check(lib.fs_slice_fwd(ctypes.byref(prob), nat.t4(x), nat.t4(fx), nat.ptr(W),
                                   nat.ptr(b), nat.ptr(tau), None, None, nat.ptr(z_ref),
                                   nat.ptr(s_ref), nat.ptr(ws), nws, stream))
        z = torch.full((B, H, G, DV), float("nan"), device="cuda")
        s = torch.full((B, H, G), float("nan"), device="cuda")
        nat.check(lib.fs_slice_fwd_noalloc(ctypes.byref(prob), nat.t4(x), nat.t4(fx),
                                           nat.ptr(W), nat.ptr(b), nat.ptr(tau), nat.ptr(z),
                                           nat.ptr(s), stream))
        torch.cuda.synchronize()
        assert torch.isfinite(z).all() and torch.isfinite(s).all()
        assert _relerr(z, z_ref) <= TOL
        assert _relerr(s, s_ref) <= TOL
        # s sums the slice weights: its total over the slots is the point count
        assert abs(float(s.double().sum()) - B * N * H) <= 1e-4 * B * N * H


def test_noalloc_refuses_what_does_not_fit(cuda_device):
    from flashslice_b200.kernels import _native as nat
    lib = nat.load()
    # 4096 (b, h) pairs: the partial sums exceed the static scratch
    x = torch.empty(512, 64, 8, 32, device="cuda")
    W = torch.empty(8, 32, 32, device="cuda")
    prob = _problem(nat, x, x, W)
    out = torch.empty(512 * 8 * 32 * 32, device="cuda")
    one = nat.ptr(out)
    rc = lib.fs_slice_fwd_noalloc(ctypes.byref(prob), nat.t4(x), nat.t4(x), nat.ptr(W), one, one,
                                  one, one, nat.stream_of(x))
    assert rc == nat.FS_ERR_UNSUPPORTED
    assert b"scratch" in lib.fs_last_error()
    # shapes outside the single-tile family are refused, not served wrongly
    W64 = torch.empty(8, 64, 32, device="cuda")
    prob = _problem(nat, x[:1], x[:1], W64)
    rc = lib.fs_slice_fwd_noalloc(ctypes.byref(prob), nat.t4(x[:1]), nat.t4(x[:1]),
                                  nat.ptr(W64), one, one, one, one, nat.stream_of(x))
    assert rc == nat.FS_ERR_UNSUPPORTED
