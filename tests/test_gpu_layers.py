"""The layer and the model on their fused path (the tensor-core coupling
round with the tied backward) against the same modules on their eager path,
and torch.compile of the ops in one graph."""

import pytest
import torch

from parity import relerr

pytestmark = pytest.mark.gpu


def _layer_run(layer, x, up):
    x = x.clone().requires_grad_(True)
    y, _ = layer(x)
    (y * up).sum().backward()
    res = {"out": y.detach(), "grad:x": x.grad}
    for k, p in layer.named_parameters():
        if p.grad is not None:  # unused by a variant (to_q, to_k without token attention)
            res["grad:" + k] = p.grad.clone()
            p.grad = None
    return res


@pytest.mark.parametrize("kw", [{}, {"no_token_attention": True}, {"untied_deslice": True}],
                         ids=["tied", "notokattn", "untied"])
def test_layer_fused_matches_eager(cuda_device, kw):
    torch.backends.cuda.matmul.allow_tf32 = False
    from flashslice_b200 import Physics_Attention_Irregular_Mesh
    from flashslice_b200.kernels import _native as nat
    torch.manual_seed(0)
    eager = Physics_Attention_Irregular_Mesh(256, heads=8, dim_head=32, slice_num=32, **kw)
    fused = Physics_Attention_Irregular_Mesh(256, heads=8, dim_head=32, slice_num=32,
                                             use_fused_slice=True, **kw)
    fused.load_state_dict(eager.state_dict())
    assert fused.use_fused_slice
    truth = Physics_Attention_Irregular_Mesh(256, heads=8, dim_head=32, slice_num=32, **kw)
    truth.load_state_dict(eager.state_dict())
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 5000, 256, generator=g)
    up = torch.randn(2, 5000, 256, generator=g)
    lib = nat.load()
    n0 = lib.fs_tc_launch_count()
    rf = _layer_run(fused.cuda(), x.cuda(), up.cuda())
    ran = lib.fs_tc_launch_count() - n0
    # tied: slice, deslice, dtokens pass, coupled backward; untied: the four ops
    assert ran == 4, ran
    re = _layer_run(eager.cuda(), x.cuda(), up.cuda())
    rt = _layer_run(truth.double().cuda(), x.double().cuda(), up.double().cuda())
    for k in rt:
        ef, ee = relerr(rf[k], rt[k]), relerr(re[k], rt[k])
        assert ef <= max(2.0 * ee, 1e-5), (k, ef, ee)


def test_layer_bf16_autocast_on_tensor_cores(cuda_device):
    """The layer under bf16 autocast: its projections hand bf16 x_mid / fx_mid
    to the coupling round, which runs on the tensor cores; output and
    gradients against the float64 layer within the reference's bf16 gate
    (2e-2), as close as the eager path under the same autocast."""
    torch.backends.cuda.matmul.allow_tf32 = False
    from flashslice_b200 import Physics_Attention_Irregular_Mesh
    from flashslice_b200.kernels import _native as nat
    torch.manual_seed(5)
    kw = dict(heads=8, dim_head=32, slice_num=32)
    eager = Physics_Attention_Irregular_Mesh(256, **kw)
    fused = Physics_Attention_Irregular_Mesh(256, use_fused_slice=True, **kw)
    fused.load_state_dict(eager.state_dict())
    truth = Physics_Attention_Irregular_Mesh(256, **kw)
    truth.load_state_dict(eager.state_dict())
    g = torch.Generator().manual_seed(6)
    x = torch.randn(1, 8000, 256, generator=g)
    up = torch.randn(1, 8000, 256, generator=g)
    lib = nat.load()
    n0 = lib.fs_tc_launch_count()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        rf = _layer_run(fused.cuda(), x.cuda(), up.cuda())
    assert lib.fs_tc_launch_count() - n0 == 4
    with torch.autocast("cuda", dtype=torch.bfloat16):
        re = _layer_run(eager.cuda(), x.cuda(), up.cuda())
    rt = _layer_run(truth.double().cuda(), x.double().cuda(), up.double().cuda())
    for k in rt:
        ef, ee = relerr(rf[k].double(), rt[k]), relerr(re[k].double(), rt[k])
        assert ef <= max(1.25 * ee, 2e-2), (k, ef, ee)


def test_transolver_fused_trains(cuda_device):
    """A few optimiser steps of a small Transolver on the fused path track the
    eager model step for step."""
    torch.backends.cuda.matmul.allow_tf32 = False
    from flashslice_b200 import Transolver
    torch.manual_seed(3)
    kw = dict(space_dim=3, fun_dim=1, out_dim=4, n_hidden=256, n_heads=8, n_layers=2,
              slice_num=32)
    eager = Transolver(**kw).cuda()
    fused = Transolver(use_fused_slice=True, **kw).cuda()
    fused.load_state_dict(eager.state_dict())
    g = torch.Generator().manual_seed(4)
    xc = torch.rand(1, 4000, 3, generator=g).cuda()
    fv = torch.randn(1, 4000, 1, generator=g).cuda()
    y = torch.randn(1, 4000, 4, generator=g).cuda()
    opts = [torch.optim.Adam(m.parameters(), lr=1e-3) for m in (eager, fused)]
    for step in range(3):
        losses = []
        for m, opt in zip((eager, fused), opts):
            opt.zero_grad()
            loss = ((m(xc, fv) - y) ** 2).mean()
            loss.backward()
            opt.step()
            losses.append(loss.item())
        assert abs(losses[0] - losses[1]) <= 1e-4 * abs(losses[0]), (step, losses)


def test_ops_compile_fullgraph(cuda_device):
    """The custom ops are single opaque nodes: one round compiles with
    fullgraph=True and matches the eager call."""
    import flashslice_b200.kernels as K
    g = torch.Generator().manual_seed(6)
    x = torch.randn(1, 3000, 4, 32, generator=g).cuda()
    fx = torch.randn(1, 3000, 4, 32, generator=g).cuda()
    W = (torch.randn(4, 32, 32, generator=g) / 32 ** 0.5).cuda()
    b = (0.1 * torch.randn(4, 32, generator=g)).cuda()
    tau = torch.full((4,), 0.5).cuda()

    def round_(x, fx, W, b, tau):
        z, s = K.fused_slice(x, fx, W, b, tau)
        return K.fused_deslice(x, W, b, tau, z / (s + 1e-5)[..., None])

    ref = round_(x, fx, W, b, tau)
    out = torch.compile(round_, fullgraph=True)(x, fx, W, b, tau)
    assert relerr(out, ref) <= 1e-6
