"""Off-mesh deslice (the tokens of one point set queried at another point
set, ROADMAP.md:74-79 of the reference) and 16-bit outputs: the slice runs
over the mesh points, the deslice over query points with their own N; values
and every gradient (query and mesh inputs, the shared weights) against the
float64 eager composition."""

import pytest
import torch

from parity import relerr

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    import flashslice_b200.kernels as K
    return K


def _round(K, x, fx, xq, W, b, tau, r, eager=False):
    if eager:
        from oracle import eager_torch as E
        z, s = E.slice_fwd(x, fx, W, b, tau)
        return E.deslice_fwd(xq, W, b, tau, z / (s + 1e-5)[..., None])
    z, s = K.fused_slice(x, fx, W, b, tau)
    return K.fused_deslice(xq, W, b, tau, z / (s + 1e-5)[..., None])


@pytest.mark.parametrize("Nq", [1, 300, 50_001])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_offmesh_deslice(K, Nq, dtype):
    g = torch.Generator().manual_seed(17)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    B, N, H = 1, 20_000, 4
    x, fx, xq = r(B, N, H, 32), r(B, N, H, 32), r(B, Nq, H, 32)
    W, b = r(H, 32, 32) / 32 ** 0.5, 0.1 * r(H, 32)
    tau = 0.3 + 0.7 * torch.rand(H, generator=g, dtype=torch.float64)
    up = r(B, Nq, H, 32)
    # the truth on the very inputs the op sees (points rounded to `dtype`)
    x, fx, xq = (t.to(dtype).double() for t in (x, fx, xq))
    ref_leaves = [t.cuda().requires_grad_(True) for t in (x, fx, xq, W, b, tau)]
    ref = _round(K, *ref_leaves, None, eager=True)
    (ref * up.cuda()).sum().backward()
    # points in `dtype`, parameters fp32 (as a layer under autocast holds them)
    leaves = [t.cuda().to(dtype).requires_grad_(True) for t in (x, fx, xq)] + \
             [t.cuda().float().requires_grad_(True) for t in (W, b, tau)]
    out = _round(K, *leaves, None)
    assert out.shape == (B, Nq, H, 32) and out.dtype == dtype
    (out.float() * up.cuda().float()).sum().backward()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert relerr(out.double(), ref) <= tol
    for a, e, name in zip(leaves, ref_leaves, ("x", "fx", "xq", "W", "b", "tau")):
        err = relerr(a.grad.double(), e.grad)
        # the reference's own gate for gradients through a round of fp32 ops
        assert err <= (2e-5 if dtype == torch.float32 else 3e-2), (name, err)
