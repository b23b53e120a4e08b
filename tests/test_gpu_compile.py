"""torch.compile of the layer and the model on the fused path: one graph,
forward and backward (``fullgraph=True``, no graph break), with outputs and
every gradient matching the same modules run eagerly. The custom ops are
opaque nodes with registered fakes and autograd (``slice_ops.py:787-954``,
``blocked.py:1472-1568`` in the reference); under compile the coupling round
is their plain composition, the token attention traced between them."""

import pytest
import torch

from parity import relerr

pytestmark = pytest.mark.gpu


def _run(fn, leaves, up):
    leaves = [t.detach().clone().requires_grad_(True) for t in leaves]
    out = fn(*leaves)
    out = out[0] if isinstance(out, tuple) else out
    (out * up).sum().backward()
    return [out.detach()] + [t.grad for t in leaves]


def _module_run(m, inputs, up):
    inputs = [t.detach().clone().requires_grad_(True) for t in inputs]
    out = m(*inputs)
    out = out[0] if isinstance(out, tuple) else out
    (out * up).sum().backward()
    res = {"out": out.detach()}
    for i, t in enumerate(inputs):
        res["grad:in%d" % i] = t.grad
    for k, p in m.named_parameters():
        if p.grad is not None:  # (a compiled module prefixes its names with _orig_mod.)
            res["grad:" + k.replace("_orig_mod.", "")] = p.grad.clone()
            p.grad = None
    return res


def _no_breaks(fn, *args):
    torch._dynamo.reset()
    exp = torch._dynamo.explain(fn)(*args)
    assert exp.graph_break_count == 0, exp.break_reasons
    assert exp.graph_count == 1, exp.graph_count


def _gate_vs_truth(got, ref_eager, truth, factor=2.0):
    """Compiled fused results against the float64 truth, at least nearly as
    close as the reference's fp32 eager path (the gate of the layer tests:
    the temperature gradients are cancellations, so a fixed relative bound
    between two fp32 evaluations says little about them)."""
    assert set(got) == set(truth), set(got) ^ set(truth)
    for k in truth:
        ef, ee = relerr(got[k], truth[k]), relerr(ref_eager[k], truth[k])
        assert ef <= max(factor * ee, 1e-5), (k, ef, ee)


@pytest.mark.parametrize("kw", [{}, {"no_token_attention": True}, {"untied_deslice": True}],
                         ids=["tied", "notokattn", "untied"])
def test_layer_compiles_into_one_graph_with_its_backward(cuda_device, kw):
    torch.backends.cuda.matmul.allow_tf32 = False
    from flashslice_b200 import Physics_Attention_Irregular_Mesh
    torch.manual_seed(0)
    mk = lambda fused: Physics_Attention_Irregular_Mesh(  # noqa: E731
        128, heads=4, dim_head=32, slice_num=32, use_fused_slice=fused, **kw)
    layer = mk(True)
    eager, truth = mk(False), mk(False)
    eager.load_state_dict(layer.state_dict())
    truth.load_state_dict(layer.state_dict())
    layer, eager, truth = layer.cuda(), eager.cuda(), truth.double().cuda()
    assert layer.use_fused_slice
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 3000, 128, generator=g).cuda()
    up = torch.randn(2, 3000, 128, generator=g).cuda()
    _no_breaks(layer, x)
    torch._dynamo.reset()
    got = _module_run(torch.compile(layer, fullgraph=True), [x], up)
    _gate_vs_truth(got, _module_run(eager, [x], up),
                   _module_run(truth, [x.double()], up.double()))


def test_transolver_compiles_into_one_graph_with_its_backward(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    from flashslice_b200 import Transolver
    torch.manual_seed(3)
    kw = dict(space_dim=3, fun_dim=1, out_dim=4, n_hidden=128, n_heads=4, n_layers=2,
              slice_num=32)
    model = Transolver(use_fused_slice=True, **kw)
    eager, truth = Transolver(**kw), Transolver(**kw)
    eager.load_state_dict(model.state_dict())
    truth.load_state_dict(model.state_dict())
    model, eager, truth = model.cuda(), eager.cuda(), truth.double().cuda()
    g = torch.Generator().manual_seed(4)
    xc = torch.rand(1, 3000, 3, generator=g).cuda()
    fv = torch.randn(1, 3000, 1, generator=g).cuda()
    up = torch.randn(1, 3000, 4, generator=g).cuda()
    _no_breaks(model, xc, fv)
    torch._dynamo.reset()
    got = _module_run(torch.compile(model, fullgraph=True), [xc, fv], up)
    # two layers: inductor reorders the sums of the layer norms and MLPs
    # around the ops, so the most sensitive gradients (the token attention's
    # q and k projections) may sit a few times eager's distance from the truth
    _gate_vs_truth(got, _module_run(eager, [xc, fv], up),
                   _module_run(truth, [xc.double(), fv.double()], up.double()), factor=4.0)


@pytest.mark.parametrize("G,dt", [(32, torch.float32), (64, torch.float32),
                                  (128, torch.bfloat16)],
                         ids=["single-tile", "blocked-fp32", "blocked-bf16"])
def test_round_with_permuted_per_sample_weight_compiles(cuda_device, G, dt):
    """A coupling round with the reference's per-sample weight -- a permuted
    view of tokens @ Wk -- forward and backward under fullgraph compile: the
    parameter gradients come back contiguous from both the fakes and the
    kernels, so the compiled graph's stride checks hold."""
    import flashslice_b200.kernels as K
    B, N, H, D = 2, 2500, 4, 32
    g = torch.Generator().manual_seed(7)
    x = torch.randn(B, N, H, D, generator=g).cuda().to(dt)
    fx = torch.randn(B, N, H, D, generator=g).cuda().to(dt)
    tok_k = torch.randn(B, G, 16, generator=g).cuda()
    Wk = (torch.randn(16, H * D, generator=g) / (16 * D) ** 0.5).cuda()
    b = (0.1 * torch.randn(G, generator=g)).cuda()
    tau = (0.3 + 0.7 * torch.rand(H, generator=g)).cuda()
    up = torch.randn(B, N, H, D, generator=g).cuda().to(dt)
    if dt == torch.bfloat16:
        K.set_dot_mode("bf16")

    def round_(x, fx, tk, Wk, b, tau):
        W = (tk @ Wk).view(B, G, H, D).permute(0, 2, 1, 3)  # not contiguous
        z, s = K.fused_slice(x, fx, W, b, tau)
        return K.fused_deslice(x, W, b, tau, z / (s + 1e-5)[..., None])

    try:
        leaves = [x, fx, tok_k, Wk, b, tau]
        _no_breaks(round_, *leaves)
        ref = _run(round_, leaves, up)
        torch._dynamo.reset()
        got = _run(torch.compile(round_, fullgraph=True), leaves, up)
    finally:
        K.set_dot_mode("ieee")
    tol = 1e-5 if dt == torch.float32 else 1e-2
    for i, (a, r) in enumerate(zip(got, ref)):
        assert relerr(a.float(), r.float()) <= tol, (i, relerr(a.float(), r.float()))
