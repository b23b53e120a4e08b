"""The custom ops' fake kernels on the CPU (no GPU needed): shapes and
dtypes of every output as the reference's fakes give them
(``slice_ops.py:894-919``, ``blocked.py:1502-1529``) -- z_num, s and the
statistics fp32, out and the point gradients in the point tensors' dtype,
the parameter gradients in the parameters' -- and the graph a blocked
coupling round traces to, which hands the slice's statistics to the deslice
(``physics_attention.py:95-136``)."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import flashslice_b200.kernels as K

ops = torch.ops.flashslice


def _leaves(B=2, N=300, H=4, D=32, DV=64, G=1024, dtype=torch.bfloat16):
    dev = "cuda"
    return dict(x=torch.empty(B, N, H, D, device=dev, dtype=dtype),
                fx=torch.empty(B, N, H, DV, device=dev, dtype=dtype),
                W=torch.empty(B, H, G, D, device=dev), b=torch.empty(G, device=dev),
                tau=torch.empty(H, device=dev), tok=torch.empty(B, H, G, DV, device=dev),
                dout=torch.empty(B, N, H, DV, device=dev, dtype=dtype))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_single_tile_fakes(dtype):
    with FakeTensorMode():
        L = _leaves(G=32, DV=32, dtype=dtype)
        x, fx, W, b, tau = L["x"], L["fx"], L["W"], L["b"], L["tau"]
        z, s = ops.flash_slice(x, fx, W, b, tau, 0)
        assert z.shape == (2, 4, 32, 32) and z.dtype == torch.float32
        assert s.shape == (2, 4, 32) and s.dtype == torch.float32
        out = ops.flash_deslice(x, W, b, tau, z, 0)
        assert out.shape == (2, 300, 4, 32) and out.dtype == dtype
        g = ops.flash_slice_bwd(x, fx, W, b, tau, z, s, 0)
        assert [t.shape for t in g] == [x.shape, fx.shape, W.shape, b.shape, tau.shape]
        assert g[0].dtype == dtype and g[2].dtype == torch.float32
        g = ops.flash_deslice_bwd(x, W, b, tau, z, out, 0)
        assert [t.shape for t in g] == [x.shape, z.shape, W.shape, b.shape, tau.shape]
        g = ops.coupled_bwd(x, fx, out, W, b, tau, z, z, s, 0)
        assert [t.shape for t in g] == [x.shape, fx.shape, W.shape, b.shape, tau.shape]


def test_blocked_fakes():
    with FakeTensorMode():
        L = _leaves()
        x, fx, W, b, tau, tok = L["x"], L["fx"], L["W"], L["b"], L["tau"], L["tok"]
        z, s, st = ops.slice_blk(x, fx, W, b, tau, None, 3)
        assert z.shape == (2, 4, 1024, 64) and z.dtype == torch.float32
        assert st.shape == (2, 4, 2, 300) and st.dtype == torch.float32
        out, st2 = ops.deslice_blk(x, W, b, tau, tok, st, 3)
        assert out.shape == (2, 300, 4, 64) and out.dtype == torch.bfloat16
        assert st2.shape == st.shape
        g = ops.slice_blk_bwd(x, fx, W, b, tau, st, z, s, 3)
        assert [t.shape for t in g] == [x.shape, fx.shape, W.shape, b.shape, tau.shape]
        assert g[0].dtype == torch.bfloat16 and g[1].dtype == torch.bfloat16
        g = ops.deslice_blk_bwd(x, W, b, tau, tok, st, L["dout"], 3)
        assert [t.shape for t in g] == [x.shape, tok.shape, W.shape, b.shape, tau.shape]


def test_blocked_coupling_hands_statistics_to_the_deslice():
    K.set_dot_mode("bf16")
    try:
        with FakeTensorMode():
            L = _leaves()
            g = make_fx(lambda x, fx, W, b, tau: K.fused_coupling(x, fx, W, b, tau))(
                L["x"], L["fx"], L["W"], L["b"], L["tau"])
    finally:
        K.set_dot_mode("ieee")
    calls = [n for n in g.graph.nodes if n.op == "call_function"]
    sl = [n for n in calls if "slice_blk" in str(n.target) and "deslice" not in str(n.target)]
    de = [n for n in calls if "deslice_blk" in str(n.target)]
    assert len(sl) == 1 and len(de) == 1
    # deslice_blk(x, W, b, tau, tokens, stats, dot): its stats are the slice's third output
    # (through the detach that fused_slice applies to them)
    node = de[0].args[5]
    for _ in range(8):
        assert node is not None and node.op == "call_function", node
        if node.args[0] is sl[0]:
            break
        node = node.args[0]
    assert node.args[0] is sl[0] and node.args[1] == 2


def test_fake_parameter_gradients_are_contiguous_for_a_permuted_weight():
    """The reference's per-sample weight is a permuted view (tokens @ Wk viewed
    (B, G, H, D) and permuted to (B, H, G, D)); the CUDA impls return its
    gradient contiguous, and so must the fakes, or a compiled graph's stride
    checks would fail on the real output."""
    with FakeTensorMode():
        L = _leaves(G=32, DV=32, dtype=torch.float32)
        x, fx, b, tau = L["x"], L["fx"], L["b"], L["tau"]
        Wp = torch.empty(2, 32, 4, 32, device="cuda").permute(0, 2, 1, 3)
        assert not Wp.is_contiguous()
        z, s = ops.flash_slice(x, fx, Wp, b, tau, 0)
        for g in (ops.flash_slice_bwd(x, fx, Wp, b, tau, z, s, 0),
                  ops.flash_deslice_bwd(x, Wp, b, tau, z, x, 0),
                  ops.coupled_bwd(x, fx, x, Wp, b, tau, z, z, s, 0)):
            assert g[2].shape == Wp.shape and g[2].is_contiguous()
        Lb = _leaves()
        Wb = torch.empty(2, 1024, 4, 32, device="cuda").permute(0, 2, 1, 3)
        z, s, st = ops.slice_blk(Lb["x"], Lb["fx"], Wb, Lb["b"], Lb["tau"], None, 3)
        g = ops.slice_blk_bwd(Lb["x"], Lb["fx"], Wb, Lb["b"], Lb["tau"], st, z, s, 3)
        assert g[2].is_contiguous()
        g = ops.deslice_blk_bwd(Lb["x"], Wb, Lb["b"], Lb["tau"], Lb["tok"], st, Lb["dout"], 3)
        assert g[2].is_contiguous()
