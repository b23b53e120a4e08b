"""The reference's eager op math on torch CPU tensors -- TEST INFRASTRUCTURE
and the timed CPU BASELINE only.

A restatement of ``bench/parity_ops.py:59-79`` (``_membership`` / ``eager``)
of the reference: the slice weights as an einsum + softmax, the slice and
deslice as einsums, the backward by torch autograd. In fp32 this is the
"reference's own implementation" the parity tolerances are quoted against;
``bench.py`` times it (all host threads) as the CPU baseline of the
slice -> normalise -> identity mix -> deslice coupling round.

The GPU parity tests also run it on device tensors, as their checker; it
never runs in the product path.
"""

import torch


def membership(x, w, b, tau):
    """(B, H, N, G) slice weights (``parity_ops.py:59-66``)."""
    B, N, H, D = x.shape
    w4 = w.reshape((1,) * (4 - w.dim()) + tuple(w.shape)).expand(B, H, -1, -1)
    lg = torch.einsum("bnhd,bhgd->bhng", x, w4)
    if b is not None:
        lg = lg + b.reshape((1,) * (3 - b.dim()) + tuple(b.shape))[:, :, None, :]
    return torch.softmax(lg / tau.view(1, H, 1, 1), dim=-1)


def slice_fwd(x, fx, w, b, tau):
    sw = membership(x, w, b, tau)
    return torch.einsum("bhng,bnhd->bhgd", sw, fx), sw.sum(2)


def deslice_fwd(x, w, b, tau, tok):
    sw = membership(x, w, b, tau)
    return torch.einsum("bhgd,bhng->bnhd", tok.to(sw.dtype), sw)


def coupling_forward(x, fx, w, b, tau, eps=1e-5, mix=None):
    """slice -> z_num / (s + eps) -> mix (None = identity) -> deslice, sharing
    one membership as the eager module does (``parity_ops.py:69-79``)."""
    sw = membership(x, w, b, tau)
    z = torch.einsum("bhng,bnhd->bhgd", sw, fx)
    s = sw.sum(2)
    tok = z / (s + eps)[..., None]
    if mix is not None:
        tok = tok @ mix
    out = torch.einsum("bhgd,bhng->bnhd", tok.to(sw.dtype), sw)
    return out, z, s


def coupling_round(x, fx, w, b, tau, r, eps=1e-5, mix=None, r_z=None, r_s=None):
    """Forward and backward of loss = sum(out * r) [+ sum(z * r_z) +
    sum(s * r_s)] with autograd; returns a dict of detached results and the
    gradients of the leaves that require them."""
    leaves = {"x": x, "fx": fx, "W": w, "b": b, "tau": tau}
    out, z, s = coupling_forward(x, fx, w, b, tau, eps, mix)
    loss = (out * r).sum()
    if r_z is not None:
        loss = loss + (z * r_z).sum()
    if r_s is not None:
        loss = loss + (s * r_s).sum()
    loss.backward()
    res = {"out": out.detach(), "z_num": z.detach(), "s": s.detach()}
    for k, v in leaves.items():
        if v is not None and v.grad is not None:
            res["grad:" + k] = v.grad.detach()
    return res


def eager_orders(x, fx, w, b, tau, tm, tok, order):
    """Both call orders of a tied coupling as ``parity_ops.eager`` forms them
    (``parity_ops.py:69-79``): slice-first normalises the slice output,
    applies ``tm`` and deslices it; deslice-first deslices the given tokens
    and slices independently."""
    sw = membership(x, w, b, tau)
    z = torch.einsum("bhng,bnhd->bhgd", sw, fx)
    s = sw.sum(2)
    if order == "slice-first":
        tok = (z / (s + 1e-5)[..., None]) @ tm
    out = torch.einsum("bhgd,bhng->bnhd", tok.to(sw.dtype), sw)
    return out, z, s
