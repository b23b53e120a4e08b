"""GPU parity of the fused ops against the reference's own implementation.

Mirrors the reference's op-level gate (``bench/parity_ops.py``): weight
layouts gd / hgd / bhgd, a value width apart from the logits width, both call
orders of a tied coupling, the tiny-N / masked-G / single-slot corners, bf16
inputs, run-to-run bitwise determinism; plus strided inputs, fp16, N = 0 / 1,
the widest head and the golden fixtures made by the reference. Every call
goes through the custom ops into ``libflashslice_b200.so``.
"""

import numpy as np
import pytest
import torch

from golden_io import index, load, op_inputs
from parity import Case, assert_checks, gate_case, relerr

pytestmark = pytest.mark.gpu

N = 4097


@pytest.fixture(scope="module")
def K(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    import flashslice_b200.kernels as K
    return K


CASES = [
    # name, case kwargs, kernel mode, dot, order, dtau gate
    ("gd-single-g32", dict(B=2, N=N, H=4, D=32, G=32, mode="gd"), "auto", "", "slice-first"),
    ("gd-blk-g256", dict(B=2, N=N, H=4, D=32, G=256, mode="gd"), "auto", "", "slice-first"),
    ("gd-blk-g256-deslice-first", dict(B=2, N=N, H=4, D=32, G=256, mode="gd"), "auto", "",
     "deslice-first"),
    ("hgd-single-g32", dict(B=2, N=N, H=4, D=32, G=32, mode="hgd"), "auto", "", "slice-first"),
    ("hgd-blk-g48-d40-dv24", dict(B=2, N=N, H=4, D=40, G=48, DV=24, mode="hgd"), "auto", "",
     "slice-first"),
    ("bhgd-single-g64", dict(B=2, N=N, H=4, D=32, G=64), "auto", "", "slice-first"),
    ("bhgd-blk-g256-nobias", dict(B=2, N=N, H=4, D=32, G=256, bias=False), "auto", "",
     "slice-first"),
    ("bhgd-forced-blk-g32", dict(B=2, N=N, H=4, D=32, G=32), "blocked", "", "slice-first"),
    ("bhgd-forced-blk-g32-deslice-first", dict(B=2, N=N, H=4, D=32, G=32), "blocked", "",
     "deslice-first"),
    ("bhgd-blk-g2048-d56-dv32", dict(B=1, N=N, H=8, D=56, G=2048, DV=32, bias=False), "auto",
     "", "slice-first"),
    ("bhgd-blk-g2048-d56-dv32-deslice-first",
     dict(B=1, N=N, H=8, D=56, G=2048, DV=32, bias=False), "auto", "", "deslice-first"),
    ("bhgd-blk-g1024-d56-dv32-deslice-first-bias", dict(B=1, N=N, H=8, D=56, G=1024, DV=32),
     "auto", "", "deslice-first"),
    ("bhgd-blk-tinyN17-g256-d56-dv32", dict(B=2, N=17, H=4, D=56, G=256, DV=32, bias=False),
     "auto", "", "slice-first"),
    ("bhgd-blk-tinyN17-g256-d56-dv32-deslice-first",
     dict(B=2, N=17, H=4, D=56, G=256, DV=32, bias=False), "auto", "", "deslice-first"),
    ("gd-blk-tinyN17-g512-deslice-first", dict(B=2, N=17, H=4, D=32, G=512, mode="gd"), "auto",
     "", "deslice-first"),
    ("hgd-blk-g40-masked-deslice-first", dict(B=2, N=N, H=4, D=32, G=40, mode="hgd"), "auto",
     "", "deslice-first"),
    ("bhgd-blk-g1-d56-dv32", dict(B=1, N=N, H=2, D=56, G=1, DV=32, bias=False), "auto", "",
     "slice-first"),
    ("gd-single-g16-d16", dict(B=1, N=N, H=2, D=16, G=16, mode="gd"), "auto", "", "slice-first"),
    ("gd-single-g128-d128", dict(B=1, N=1000, H=2, D=128, G=128, mode="gd"), "auto", "",
     "slice-first"),
    ("gd-blk-d256-g32", dict(B=1, N=700, H=2, D=256, G=32, mode="gd"), "auto", "", "slice-first"),
    ("hgd-blk-d24-g8", dict(B=1, N=N, H=3, D=24, G=8, mode="hgd"), "auto", "", "slice-first"),
    ("hgd-single-g32-strided", dict(B=2, N=N, H=4, D=32, G=32, mode="hgd", strided=True),
     "auto", "", "slice-first"),
    ("hgd-blk-g64-strided-deslice-first",
     dict(B=2, N=N, H=4, D=32, G=64, mode="hgd", strided=True), "blocked", "", "deslice-first"),
    ("gd-single-n1", dict(B=1, N=1, H=2, D=32, G=32, mode="gd"), "auto", "", "slice-first"),
    ("gd-blk-n1-deslice-first", dict(B=1, N=1, H=2, D=32, G=64, mode="gd"), "auto", "",
     "deslice-first"),
    # bf16 activations and computed bf16 weights
    ("bhgd-bf16-single-g32", dict(B=2, N=N, H=4, D=32, G=32), "auto", "bf16", "slice-first"),
    ("bhgd-bf16-blk-g256-d56-dv32", dict(B=1, N=N, H=8, D=56, G=256, DV=32, bias=False), "auto",
     "bf16", "slice-first"),
    ("bhgd-bf16-blk-g1024-d56-dv32-deslice-first",
     dict(B=1, N=N, H=8, D=56, G=1024, DV=32, bias=False), "auto", "bf16", "deslice-first"),
    # every dot level on the exact path
    ("hgd-single-g32-tf32", dict(B=1, N=N, H=4, D=32, G=32, mode="hgd"), "auto", "tf32",
     "slice-first"),
    ("hgd-single-g32-tf32x3", dict(B=1, N=N, H=4, D=32, G=32, mode="hgd"), "auto", "tf32x3",
     "slice-first"),
]


@pytest.mark.parametrize("name,kw,kmode,dot,order", CASES, ids=[c[0] for c in CASES])
def test_parity_case(K, name, kw, kmode, dot, order):
    assert_checks(gate_case(Case(**kw), K, kernel_mode=kmode, dot=dot, order=order))


def test_empty_n(K):
    dev = torch.device("cuda")
    x = torch.randn(1, 0, 2, 32, device=dev)
    W = torch.randn(32, 32, device=dev)
    tau = torch.ones(2, device=dev)
    z, s = K.fused_slice(x, x, W, None, tau)
    assert z.shape == (1, 2, 32, 32) and float(z.abs().sum()) == 0 and float(s.abs().sum()) == 0
    out = K.fused_deslice(x, W, None, tau, torch.randn(1, 2, 32, 32, device=dev))
    assert out.shape == (1, 0, 2, 32)


def test_fp16_inputs(K):
    c = Case(B=1, N=2000, H=2, D=32, G=32, mode="hgd")
    L = {k: v.float() for k, v in c.leaves.items()}
    x16, fx16 = L["x"].half(), L["fx"].half()
    z, s = K.fused_slice(x16, fx16, L["w"], L["b"], L["tau"])
    from oracle import eager_torch as E
    zr, sr = E.slice_fwd(x16.float(), fx16.float(), L["w"], L["b"], L["tau"])
    assert relerr(z, zr) < 1e-5 and relerr(s, sr) < 1e-5
    out = K.fused_deslice(x16, L["w"], L["b"], L["tau"], L["tok"])
    assert out.dtype == torch.float16
    outr = E.deslice_fwd(x16.float(), L["w"], L["b"], L["tau"], L["tok"])
    assert relerr(out.float(), outr) < 2e-3


OPS = index()["ops"]


@pytest.mark.parametrize("case", OPS, ids=[c["name"] for c in OPS])
@pytest.mark.parametrize("kmode", ["auto", "blocked"])
def test_golden_fixtures(K, case, kmode):
    """Each op against the reference's own float64 results, per op."""
    a = load(case["file"])
    i = op_inputs(a)
    dev = torch.device("cuda")
    T = lambda k: None if i[k] is None else torch.tensor(i[k], dtype=torch.float32, device=dev)  # noqa
    x, fx, W, b, tau, tok = T("x"), T("fx"), T("W"), T("b"), T("tau"), T("tok")
    dz, ds, dout = T("dz"), T("ds"), T("dout")
    K.set_kernel_mode(kmode)
    try:
        leaves = [t.requires_grad_(True) for t in (x, fx, W, tau) + ((b,) if b is not None else ())]
        z, s = K.fused_slice(x, fx, W, b, tau)
        ((z * dz).sum() + (s * ds).sum()).backward()
        got = {"slice:z_num": z, "slice:s": s, "slice:grad:x": x.grad, "slice:grad:fx": fx.grad,
               "slice:grad:W": W.grad, "slice:grad:tau": tau.grad}
        if b is not None:
            got["slice:grad:b"] = b.grad
        for t in leaves:
            t.grad = None
        tok.requires_grad_(True)
        out = K.fused_deslice(x, W, b, tau, tok)
        (out * dout).sum().backward()
        got.update({"deslice:out": out, "deslice:grad:x": x.grad, "deslice:grad:W": W.grad,
                    "deslice:grad:tau": tau.grad, "deslice:grad:tok": tok.grad})
        if b is not None:
            got["deslice:grad:b"] = b.grad
    finally:
        K.set_kernel_mode("auto")
    for k, v in got.items():
        ref = torch.tensor(a[k])
        assert tuple(v.shape) == tuple(ref.shape), k
        if float(ref.norm()) < 1e-12:
            assert float(v.abs().max()) <= 1e-6, k
            continue
        tol = 1e-4 if "grad:tau" in k else 2e-5
        assert relerr(v.detach().cpu(), ref) < tol, (k, relerr(v.detach().cpu(), ref))


def test_stats_modes_agree(K):
    """The online and two-pass statistics and the online deslice's: m bitwise
    equal (a max is exact), l to rounding (``parity_ops.py:213-235``); and
    against the float64 oracle."""
    from oracle import coupling as C
    from flashslice_b200.kernels.blocked import compute_stats, set_stats_mode
    c = Case(B=1, N=N, H=8, D=56, G=1024, DV=32, bias=False)
    L = {k: v.float() for k, v in c.leaves.items()}
    x, fx, w, b, tau, tok = c.build(L, amp=False)
    w = w.contiguous()
    bb = w.new_zeros(w.shape[-2])
    try:
        set_stats_mode("online")
        _, st_online = K.fused_deslice(x, w, None, tau, tok, return_stats=True)
        st_stats = compute_stats(x, w, bb, tau)
        set_stats_mode("two-pass")
        st_two = compute_stats(x, w, bb, tau)
    finally:
        set_stats_mode("online")
    assert torch.equal(st_online[:, :, 0], st_two[:, :, 0])
    assert torch.equal(st_stats[:, :, 0], st_two[:, :, 0])
    for st in (st_online, st_stats):
        assert float(((st[:, :, 1] - st_two[:, :, 1]).abs() / st_two[:, :, 1]).max()) < 1e-5
    ref = C.stats(x.double().cpu().numpy(), w.double().cpu().numpy(), None,
                  tau.double().cpu().numpy())
    got = st_two.double().cpu().numpy()
    assert np.max(np.abs(got[:, :, 0] - ref[:, :, 0])) < 1e-4
    # l is an fp32 sum of G = 1024 exponentials whose arguments carry the
    # logits' own fp32 rounding: a few 1e-6 relative is the fp32 floor
    assert np.max(np.abs(got[:, :, 1] - ref[:, :, 1]) / ref[:, :, 1]) < 2e-5


def test_call_orders(K):
    """Every call order of the two ops builds a graph that survives a
    backward (``parity_ops.py:239-332``)."""
    def leaves(B=1, N=2049, H=4, D=56, DV=32, G=256, Ht=48, mode="bhgd"):
        g = torch.Generator().manual_seed(0)
        r = lambda *s: torch.randn(*s, generator=g).cuda()  # noqa: E731
        L = {"x": r(B, N, H, D), "fx": r(B, N, H, DV), "tau": torch.ones(H).cuda(),
             "tok": r(B, H, G, DV)}
        if mode == "bhgd":
            L["t"], L["Wk"] = r(B, G, Ht), r(Ht, H * D) / 8.0
        else:
            L["w"] = r(G, D) / 8.0
        for v in L.values():
            v.requires_grad_(True)
        return L

    def weight(L):
        if "w" in L:
            return L["w"]
        B, G, _ = L["t"].shape
        H, D = L["x"].shape[2], L["x"].shape[3]
        return (L["t"] @ L["Wk"]).view(B, G, H, D).permute(0, 2, 1, 3)

    def loss_of(*ts):
        return sum(t.float().sum() for t in ts)

    from flashslice_b200.kernels.blocked import compute_stats
    fs, fd = K.fused_slice, K.fused_deslice

    def v1(L):
        return loss_of(*fs(L["x"], L["fx"], weight(L), None, L["tau"]))

    def v2(L):
        return loss_of(fd(L["x"], weight(L), None, L["tau"], L["tok"]))

    def v3(L):
        w = weight(L)
        out = fd(L["x"], w, None, L["tau"], L["tok"])
        return loss_of(out, *fs(L["x"], L["fx"], w, None, L["tau"]))

    def v4(L):
        w = weight(L)
        out, st = fd(L["x"], w, None, L["tau"], L["tok"], return_stats=True)
        return loss_of(out, *fs(L["x"], L["fx"], w, None, L["tau"], stats=st))

    def v5(L):
        w = weight(L)
        z, s, st = fs(L["x"], L["fx"], w, None, L["tau"], return_stats=True)
        return loss_of(fd(L["x"], w, None, L["tau"], L["tok"], stats=st), z, s)

    def v6(L):
        out = fd(L["x"], weight(L), None, L["tau"], L["tok"])
        return loss_of(out, *fs(L["x"], L["fx"], weight(L), None, L["tau"]))

    def v7(L):
        w = weight(L)
        st = compute_stats(L["x"], w.contiguous(), w.new_zeros(w.shape[-2]), L["tau"]).detach()
        out = fd(L["x"], w, None, L["tau"], L["tok"], stats=st)
        return loss_of(out, *fs(L["x"], L["fx"], w, None, L["tau"], stats=st))

    def v8(L):
        w = weight(L)
        out, st = fd(L["x"], w, None, L["tau"], L["tok"], return_stats=True)
        z, s = fs(L["x"], L["fx"], w, None, L["tau"], stats=st)
        loss_of(out).backward(retain_graph=True)
        return loss_of(z, s)

    variants = [(v1, {}), (v2, {}), (v3, {}), (v4, {}), (v5, {}), (v6, {}), (v7, {}), (v8, {}),
                (v4, dict(D=32, DV=32, G=32)), (v4, dict(mode="gd"))]
    for fn, kw in variants:
        L = leaves(**kw)
        fn(L).backward()
        torch.cuda.synchronize()
        for k, v in L.items():
            if v.grad is not None:
                assert torch.isfinite(v.grad).all(), (fn.__name__, k)


def test_errors(K):
    dev = torch.device("cuda")
    x = torch.randn(1, 10, 2, 32, device=dev)
    tau = torch.ones(2, device=dev)
    with pytest.raises(ValueError):
        K.fused_slice(x, x, torch.randn(8, 31, device=dev), None, tau)  # D mismatch
    with pytest.raises(ValueError):
        K.fused_slice(x, x, torch.randn(3, 8, 32, device=dev), None, tau)  # heads 3 vs 2
    with pytest.raises(ValueError):
        K.fused_slice(torch.randn(1, 10, 2, 300, device=dev), torch.randn(1, 10, 2, 300, device=dev),
                      torch.randn(8, 300, device=dev), None, tau)  # D > 256
    with pytest.raises(RuntimeError):
        K.fused_slice(x.cpu(), x.cpu(), torch.randn(8, 32), None, tau.cpu())  # no CPU kernels
