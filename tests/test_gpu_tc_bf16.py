"""bf16 point tensors on the tensor-core engine (D = DV = G = 32): the point
tiles are read as bf16 (each value its own exact hi part), the weights and
tokens still split three ways, the outputs stored in bf16. Against the exact
FMA kernels on the same bf16 inputs (the same exact products, so agreement to
fp32 rounding, bf16 outputs to their rounding) and against the float64 math
on those inputs within the reference's bf16 gate (2e-2)."""

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


def _inputs(N, mode, B=1, H=4, seed=13):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    x, fx, up = (r(B, N, H, 32).bfloat16() for _ in range(3))
    W = {"gd": r(32, 32), "hgd": r(H, 32, 32), "bhgd": r(B, H, 32, 32)}[mode] / 32 ** 0.5
    b = {"gd": r(32), "hgd": r(H, 32), "bhgd": r(B, H, 32)}[mode] * 0.1
    tau = 0.3 + 0.7 * torch.rand(H, generator=g, dtype=torch.float64)
    return [t.cuda() for t in (x, fx, W.float(), b.float(), tau.float(), up)]


def _round(K, x, fx, W, b, tau, up, tied):
    L = [t.clone().requires_grad_(True) for t in (x, fx, W, b, tau)]
    if tied:
        out = K.fused_coupling(*L)
    else:
        z, s = K.fused_slice(*L)
        out = K.fused_deslice(L[0], L[2], L[3], L[4], z / (s + 1e-5)[..., None])
    (out.float() * up.float()).sum().backward()
    torch.cuda.synchronize()
    return [out] + [t.grad for t in L]


@pytest.mark.parametrize("N", [77, 4097, 100_003])
@pytest.mark.parametrize("mode", ["gd", "hgd", "bhgd"])
def test_bf16_round_matches_fma_and_truth(env, N, mode):
    K, st, lib = env
    x, fx, W, b, tau, up = _inputs(N, mode, B=2 if mode == "bhgd" else 1)
    n0 = lib.fs_tc_launch_count()
    tc = _round(K, x, fx, W, b, tau, up, tied=True)
    assert lib.fs_tc_launch_count() - n0 == 4, "the tensor-core kernels did not run"
    assert tc[0].dtype == torch.bfloat16 and tc[1].dtype == torch.bfloat16
    st.set_engine("fma")
    try:
        n1 = lib.fs_tc_launch_count()
        ex = _round(K, x, fx, W, b, tau, up, tied=False)
        assert lib.fs_tc_launch_count() == n1
    finally:
        st.set_engine("auto")
    from oracle import eager_torch as E
    ref = E.coupling_round(*[t.detach().double().clone().requires_grad_(True)
                             for t in (x, fx, W, b, tau)], up.double())
    names = ("out", "grad:x", "grad:fx", "grad:W", "grad:b", "grad:tau")
    for a, e, k in zip(tc, ex, names):
        et, ee = relerr(a, ref[k]), relerr(e, ref[k])
        if a.dtype == torch.bfloat16:
            # bf16 results round the same fp32 values: their own rounding apart
            assert relerr(a, e) <= 1e-2, (k, relerr(a, e))
        else:
            # the fp32 gate of the fp32 rounds: within 1e-5 of the exact FMA
            # kernels, or as close to the truth as they are (the tied and the
            # op-by-op rounds sum the temperature gradient differently)
            assert relerr(a, e) <= 1e-5 or et <= 1.25 * ee + 1e-6, (k, et, ee)
        assert et <= 2e-2, (k, et)
    assert lib.fs_device_status(1) == 0


def test_bf16_op_by_op_backward_on_tensor_cores(env):
    """The op-by-op round (slice and deslice backward kernels) in bf16."""
    K, st, lib = env
    x, fx, W, b, tau, up = _inputs(30_000, "hgd", H=8)
    n0 = lib.fs_tc_launch_count()
    tc = _round(K, x, fx, W, b, tau, up, tied=False)
    assert lib.fs_tc_launch_count() - n0 == 4  # slice, deslice, their backward kernels
    st.set_engine("fma")
    try:
        ex = _round(K, x, fx, W, b, tau, up, tied=False)
    finally:
        st.set_engine("auto")
    for a, e in zip(tc, ex):
        tol = 1e-2 if a.dtype == torch.bfloat16 else 1e-5
        assert relerr(a, e) <= tol
