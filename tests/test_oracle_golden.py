"""The CPU oracle is pinned to the reference's own outputs.

The fixtures come from the reference itself (``tests/golden/make_golden.py``):
its eager op math in float64 with autograd, and its Triton statistics and
online-deslice kernels interpreted on the CPU in float32. The oracle must
reproduce the float64 results to rounding, and the kernel outputs to float32
rounding, before it is trusted as the checker of the CUDA path.
"""

import numpy as np
import pytest
import torch

from oracle import coupling as C
from oracle import eager_torch as E

from golden_io import index, load, op_inputs, relerr

OPS = index()["ops"]


@pytest.mark.parametrize("case", OPS, ids=[c["name"] for c in OPS])
def test_oracle_ops_match_reference_fp64(case):
    a = load(case["file"])
    i = op_inputs(a)
    z, s = C.slice_fwd(i["x"], i["fx"], i["W"], i["b"], i["tau"])
    assert relerr(z, a["slice:z_num"]) < 1e-12
    assert relerr(s, a["slice:s"]) < 1e-12
    dx, dfx, dW, db, dt = C.slice_bwd(i["x"], i["fx"], i["W"], i["b"], i["tau"],
                                      i["dz"], i["ds"])
    got = {"x": dx, "fx": dfx, "W": dW, "b": db, "tau": dt}
    for k, v in got.items():
        key = "slice:grad:" + k
        if v is None:
            assert key not in a
            continue
        assert v.shape == a[key].shape, key
        # a vanishing reference (G=1: the softmax over one slot is constant)
        # is compared absolutely
        tol = 1e-10 if np.linalg.norm(a[key]) > 1e-12 else 1e-12
        assert relerr(v, a[key]) < tol, key
    out = C.deslice_fwd(i["x"], i["W"], i["b"], i["tau"], i["tok"])
    assert relerr(out, a["deslice:out"]) < 1e-12
    dx, dtok, dW, db, dt = C.deslice_bwd(i["x"], i["W"], i["b"], i["tau"], i["tok"],
                                         i["dout"])
    got = {"x": dx, "tok": dtok, "W": dW, "b": db, "tau": dt}
    for k, v in got.items():
        key = "deslice:grad:" + k
        if v is None:
            assert key not in a
            continue
        assert v.shape == a[key].shape, key
        tol = 1e-10 if np.linalg.norm(a[key]) > 1e-12 else 1e-12
        assert relerr(v, a[key]) < tol, key


KCASES = [c for c in OPS if "kern:stats_online" in load(c["file"])]


@pytest.mark.parametrize("case", KCASES, ids=[c["name"] for c in KCASES])
def test_oracle_stats_match_reference_kernels(case):
    """(m, l) in the reference kernels' (B, H, 2, N) layout: the float64
    oracle agrees with the float32 Triton kernels to float32 rounding, and
    the kernels' two statistics modes agree on m bitwise
    (``parity_ops.py:213-235``)."""
    a = load(case["file"])
    i = op_inputs(a)
    st = C.stats(i["x"], i["W"], i["b"], i["tau"])
    for key in ("kern:stats_online", "kern:stats_twopass", "kern:deslice_online_stats"):
        k = a[key]
        assert k.shape == st.shape
        assert np.max(np.abs(k[:, :, 0] - st[:, :, 0])) < 1e-5 * (1 + np.abs(st[:, :, 0]).max())
        assert np.max(np.abs(k[:, :, 1] - st[:, :, 1]) / st[:, :, 1]) < 1e-5
    assert np.array_equal(a["kern:stats_online"][:, :, 0], a["kern:stats_twopass"][:, :, 0])
    out = C.deslice_fwd(i["x"], i["W"], i["b"], i["tau"], i["tok"])
    assert relerr(out, a["kern:deslice_online_out"]) < 1e-5


def test_eager_torch_matches_numpy_coupling():
    """The torch restatement used as the fp32 reference and CPU baseline and
    the numpy oracle agree on one coupling round in float64."""
    rng = np.random.RandomState(3)
    B, N, H, D, G = 2, 37, 3, 16, 24
    x, fx = rng.standard_normal((B, N, H, D)), rng.standard_normal((B, N, H, D))
    W, b = rng.standard_normal((H, G, D)) / 4, 0.1 * rng.standard_normal((H, G))
    tau, r = 0.5 + rng.rand(H), rng.standard_normal((B, N, H, D))
    ref = C.coupling_round(x, fx, W, b, tau, r)
    T = lambda a: torch.tensor(a, dtype=torch.float64, requires_grad=True)  # noqa: E731
    got = E.coupling_round(T(x), T(fx), T(W), T(b), T(tau), torch.tensor(r))
    for k in ("out", "z_num", "s", "grad:x", "grad:fx", "grad:W", "grad:b", "grad:tau"):
        assert relerr(got[k].numpy(), ref[k]) < 1e-11, k


def test_reduce_param_shapes():
    g4 = np.arange(2 * 3 * 4 * 5, dtype=np.float64).reshape(2, 3, 4, 5)
    assert C._reduce_param(g4, (4, 5)).shape == (4, 5)
    np.testing.assert_allclose(C._reduce_param(g4, (4, 5)), g4.sum((0, 1)))
    np.testing.assert_allclose(C._reduce_param(g4, (3, 4, 5)), g4.sum(0))
    np.testing.assert_allclose(C._reduce_param(g4, (1, 3, 4, 5)), g4.sum(0, keepdims=True))
    np.testing.assert_allclose(C._reduce_param(g4, (2, 3, 4, 5)), g4)
