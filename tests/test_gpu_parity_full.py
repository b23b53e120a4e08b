"""Parity at the benchmark configurations' full sizes.

The 1e-5 gate gets harder as N grows (the fp32 reference's own error grows
with the sums over points), so the configurations the bench times are gated
at their own sizes here, through every surface a reference user calls:

* config 2 (B=1, N=2^20, H=8, D=DV=G=32, per-head W, tau ~ U[0.3, 1], fp32
  ieee): the tied round ``fused_coupling`` (what ``bench.py`` times), the
  op-by-op round (``fused_slice`` -> normalise -> ``fused_deslice``) and the
  reverse call order (``fused_deslice`` with statistics out, then
  ``fused_slice`` with them in);
* config 5 at one GPU's share of eight (N=2^21, G=64, fp32 ieee): the same;
* config 3 (B=2, N=262,144, H=8, D=32, DV=64, G=1024, per-sample W, no bias,
  bf16 inputs in the bf16 dot mode): the slice-first round.

The checker is the reference's eager op math (``oracle/eager_torch.py``,
``bench/parity_ops.py:59-79`` in the reference) run on the device, one head
at a time (heads do not interact; this bounds its memory), in fp32 -- the
reference's own implementation -- and in fp64 as the truth. Gate, as in
``bench/parity_ops.py:159-208``: every output and gradient within 1e-5
relative of the fp32 reference, or at least as close to the fp64 truth as
the reference (1.25x its distance + 1e-6; the temperature gradient 2x on the
G-blocked family); bf16 within 2e-2 of the fp32 reference on the same bf16
inputs."""

import pytest
import torch

from oracle import eager_torch as E
from parity import BF16_TOL, FP32_TOL, relerr

pytestmark = pytest.mark.gpu

EPS = 1e-5


@pytest.fixture(scope="module")
def K(cuda_device):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    import flashslice_b200.kernels as K
    return K


def _config(name, seed=0):
    """float64 device leaves of a configuration, with the upstream gradients
    (r for out, rz for z_num, rs for s) and tokens for the reverse order."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    rn = lambda *s: torch.randn(*s, generator=g, device="cuda", dtype=torch.float64)  # noqa
    if name == "cfg2":
        B, N, H, D, DV, G = 1, 1 << 20, 8, 32, 32, 32
    elif name == "cfg5":
        B, N, H, D, DV, G = 1, 1 << 21, 8, 32, 32, 64
    else:
        B, N, H, D, DV, G = 2, 262144, 8, 32, 64, 1024
    L = {"x": rn(B, N, H, D), "fx": rn(B, N, H, DV)}
    if name == "cfg3":
        Ht = 64
        Wk = rn(Ht, H * D) / (Ht * D) ** 0.5
        L["W"] = (rn(B, G, Ht) @ Wk).view(B, G, H, D).permute(0, 2, 1, 3).contiguous()
        L["b"] = None
        L["tau"] = torch.full((H,), 0.5, device="cuda", dtype=torch.float64)
    else:
        L["W"] = rn(H, G, D) / D ** 0.5
        L["b"] = 0.02 * rn(H, G)
        L["tau"] = (0.3 + 0.7 * torch.rand(H, generator=g, device="cuda", dtype=torch.float64)
                    if name == "cfg2" else
                    torch.full((H,), 0.5, device="cuda", dtype=torch.float64))
    up = {"r": rn(B, N, H, DV), "rz": rn(B, H, G, DV), "rs": rn(B, H, G),
          "tok": rn(B, H, G, DV)}
    return L, up


def _head(t, h, axis):
    return None if t is None else t.narrow(axis, h, 1)


def _eager(L, up, dtype, order, amp=False, with_zs=True):
    """The reference's eager round, head by head, in ``dtype`` (inputs first
    rounded to bf16 when ``amp``). Returns outputs and leaf gradients."""
    H = L["x"].shape[2]
    wax = L["W"].dim() - 3  # the head axis of W: (H, G, D) or (B, H, G, D)
    res = {}
    parts = {}
    for h in range(H):
        def leaf(t, axis):
            t = _head(t, h, axis)
            if t is None:
                return None
            if amp:
                t = t.to(torch.bfloat16)
            return t.to(dtype).detach().requires_grad_(True)
        x, fx = leaf(L["x"], 2), leaf(L["fx"], 2)
        W = leaf(L["W"], wax)
        b = leaf(L["b"], L["b"].dim() - 2) if L["b"] is not None else None
        tau = L["tau"][h:h + 1].to(dtype).detach().requires_grad_(True)
        r = _head(up["r"], h, 2)
        r = (r.to(torch.bfloat16) if amp else r).to(dtype)  # as the fused side gets it
        rz, rs = _head(up["rz"], h, 1).to(dtype), _head(up["rs"], h, 1).to(dtype)
        tok = None
        if order == "slice-first":
            out, z, s = E.coupling_forward(x, fx, W, b, tau, EPS)
        else:
            tok = _head(up["tok"], h, 1).to(dtype).detach().requires_grad_(True)
            out = E.deslice_fwd(x, W, b, tau, tok)
            z, s = E.slice_fwd(x, fx, W, b, tau)
        loss = (out * r).sum()
        if with_zs:
            loss = loss + (z * rz).sum() + (s * rs).sum()
        loss.backward()
        got = {"out": (out, 2), "z_num": (z, 1), "s": (s, 1), "grad:x": (x.grad, 2),
               "grad:fx": (fx.grad, 2), "grad:W": (W.grad, wax), "grad:tau": (tau.grad, 0)}
        if b is not None:
            got["grad:b"] = (b.grad, L["b"].dim() - 2)
        if tok is not None:
            got["grad:tok"] = (tok.grad, 1)
        for k, (v, ax) in got.items():
            parts.setdefault(k, []).append((v.detach(), ax))
    for k, vs in parts.items():
        res[k] = torch.cat([v for v, _ in vs], dim=vs[0][1])
    return res


def _fused(K, L, up, surface, dt):
    """One round through the fused ops on the device, in point dtype dt."""
    x = L["x"].to(dt).detach().requires_grad_(True)
    fx = L["fx"].to(dt).detach().requires_grad_(True)
    pw = dt if dt == torch.bfloat16 else torch.float32  # bf16 runs round W as the inputs
    W = L["W"].to(pw).detach().requires_grad_(True)
    b = None if L["b"] is None else L["b"].to(pw).detach().requires_grad_(True)
    tau = L["tau"].float().detach().requires_grad_(True)
    r = up["r"].to(dt)
    tok = None
    if surface == "tied":
        out = K.fused_coupling(x, fx, W, b, tau, eps=EPS)
        out.backward(r)
        res = {"out": out.detach()}
    elif surface == "op-by-op":
        z, s = K.fused_slice(x, fx, W, b, tau)
        out = K.fused_deslice(x, W, b, tau, z / (s + EPS)[..., None])
        loss = (out.float() * r.float()).sum() + (z * up["rz"].float()).sum() + \
            (s * up["rs"].float()).sum()
        loss.backward()
        res = {"out": out.detach(), "z_num": z.detach(), "s": s.detach()}
    else:
        tok = up["tok"].float().detach().requires_grad_(True)
        out, st = K.fused_deslice(x, W, b, tau, tok, return_stats=True)
        z, s = K.fused_slice(x, fx, W, b, tau, stats=st)
        loss = (out.float() * r.float()).sum() + (z * up["rz"].float()).sum() + \
            (s * up["rs"].float()).sum()
        loss.backward()
        res = {"out": out.detach(), "z_num": z.detach(), "s": s.detach(),
               "grad:tok": tok.grad}
    res.update({"grad:x": x.grad, "grad:fx": fx.grad, "grad:W": W.grad, "grad:tau": tau.grad})
    if b is not None:
        res["grad:b"] = b.grad
    return res


def _gate(fu, e32, e64, blocked=False, bf16=False, skip=()):
    bad = []
    for k, ref in e32.items():
        if k in skip:
            continue
        assert k in fu, k
        fe = relerr(fu[k].float(), ref)
        if bf16:
            if not fe <= BF16_TOL:
                bad.append((k, "fused-vs-eager %.3e" % fe))
            continue
        ee, ef = relerr(ref, e64[k]), relerr(fu[k], e64[k])
        g = 2.0 if (blocked and k == "grad:tau") else 1.25
        if not (fe <= FP32_TOL or ef <= g * ee + 1e-6):
            bad.append((k, "fused-vs-eager %.3e fused-vs-fp64 %.3e eager-vs-fp64 %.3e"
                        % (fe, ef, ee)))
    assert not bad, bad


@pytest.mark.parametrize("cfg", ["cfg2", "cfg5"])
@pytest.mark.parametrize("surface", ["tied", "op-by-op", "deslice-first"])
def test_full_size_fp32(K, cfg, surface):
    L, up = _config(cfg)
    order = "deslice-first" if surface == "deslice-first" else "slice-first"
    zs = surface != "tied"  # the tied round returns out only
    fu = _fused(K, L, up, surface, torch.float32)
    e32 = _eager(L, up, torch.float32, order, with_zs=zs)
    e64 = _eager(L, up, torch.float64, order, with_zs=zs)
    # the tied round returns out only: z_num and s stay inside it
    _gate(fu, e32, e64, skip=() if zs else ("z_num", "s"))
    # bitwise the same on a second run
    fu2 = _fused(K, L, up, surface, torch.float32)
    for k in fu:
        assert torch.equal(fu[k], fu2[k]), k


def test_full_size_cfg3_bf16(K):
    L, up = _config("cfg3")
    K.set_dot_mode("bf16")
    try:
        fu = _fused(K, L, up, "op-by-op", torch.bfloat16)
    finally:
        K.set_dot_mode("ieee")
    e32 = _eager(L, up, torch.float32, "slice-first", amp=True)
    _gate(fu, e32, None, bf16=True)
