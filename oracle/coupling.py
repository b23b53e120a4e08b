"""numpy restatement of the slice/deslice coupling -- TEST INFRASTRUCTURE ONLY.

The arithmetic follows the reference's specification of the ops
(``flashslice/kernels/slice_ops.py:5-13``, module docstring):

    logit[b,h,n,g] = (x_mid[b,n,h,:] . W[b,h,g,:] + bias[b,h,g]) / tau[h]
    w = softmax_g(logit)
    slice:   z_num[b,h,g,:] = sum_n w[b,h,n,g] fx_mid[b,n,h,:]
             s[b,h,g]       = sum_n w[b,h,n,g]
    deslice: out[b,n,h,:]   = sum_g w[b,h,n,g] tokens[b,h,g,:]

with the weight and bias broadcast from (G, D) | (H, G, D) | (B, H, G, D)
and None | (G,) | (H, G) | (B, H, G) (``slice_ops.py:503-526``), and the
backward of ``_slice_bwd_kernel`` / ``_deslice_bwd_kernel``
(``slice_ops.py:644-776``) written out analytically:

    dw  = fx . dz_num^T + ds            (slice)   | d_out . tokens^T (deslice)
    dl  = w * (dw - sum_g w dw)         softmax Jacobian, pre-division
    du  = dl / tau
    dx  = du @ W,  dW = du^T @ x,  db = sum_n du
    dtau = sum dl * (-logit / tau)      (``slice_ops.py:705``)
    dfx = w @ dz_num (slice),  dtokens = w^T @ d_out (deslice)

Gradients of a shared weight or bias are summed over the axes it is shared
along and returned in its own shape (``slice_ops.py:481-500``). The
per-point statistics are the row max and the sum of exponentials,
``stats[b,h,0,n] = m``, ``stats[b,h,1,n] = l`` (``blocked.py:293-346``).

Every function computes in the dtype of its inputs; pass float64 arrays for
the truth. Nothing here is used by the product path.
"""

import numpy as np


def _w4(W, B, H):
    """Weight broadcast to (B, H, G, D) (``parity_ops.py:60-61``)."""
    W = np.asarray(W)
    return np.broadcast_to(W.reshape((1,) * (4 - W.ndim) + W.shape),
                           (B, H) + W.shape[-2:])


def _b3(bias, B, H, G, dtype):
    if bias is None:
        return np.zeros((B, H, G), dtype=dtype)
    bias = np.asarray(bias)
    return np.broadcast_to(bias.reshape((1,) * (3 - bias.ndim) + bias.shape),
                           (B, H, G))


def logits(x, W, bias, tau):
    """(B, H, N, G) logits, bias added before the division by tau."""
    B, N, H, D = x.shape
    W4 = _w4(W, B, H)
    G = W4.shape[2]
    u = np.einsum("bnhd,bhgd->bhng", x, W4)
    u = u + _b3(bias, B, H, G, x.dtype)[:, :, None, :]
    return u / np.asarray(tau).reshape(1, H, 1, 1)


def membership(x, W, bias, tau):
    """(B, H, N, G) slice weights w = softmax over G of the logits."""
    L = logits(x, W, bias, tau)
    m = L.max(axis=-1, keepdims=True)
    e = np.exp(L - m)
    return e / e.sum(axis=-1, keepdims=True)


def stats(x, W, bias, tau):
    """(B, H, 2, N): row max m and sum of exponentials l of the logits."""
    L = logits(x, W, bias, tau)
    m = L.max(axis=-1)
    l = np.exp(L - m[..., None]).sum(axis=-1)
    return np.stack([m, l], axis=2)


def slice_fwd(x, fx, W, bias, tau):
    """z_num (B, H, G, DV), s (B, H, G)."""
    w = membership(x, W, bias, tau)
    z = np.einsum("bhng,bnhv->bhgv", w, fx)
    return z, w.sum(axis=2)


def deslice_fwd(x, W, bias, tau, tokens):
    """out (B, N, H, DV)."""
    w = membership(x, W, bias, tau)
    return np.einsum("bhng,bhgv->bnhv", w, tokens)


def _reduce_param(g4, shape):
    """Sum a (B, H, G, ...) gradient over the leading axes (batch, heads) the
    parameter is broadcast along -- absent or of extent 1 -- and return it
    in the parameter's own shape (``slice_ops.py:481-500``)."""
    trailing = g4.ndim - 2
    lead = tuple(shape[:len(shape) - trailing])
    lead = (1,) * (2 - len(lead)) + lead
    out = g4
    for axis in (0, 1):
        if lead[axis] == 1:
            out = out.sum(axis=axis, keepdims=True)
    return out.reshape(shape)


def _param_grads(x, W, bias, tau, L, dl):
    """dx, dW, db, dtau from the pre-division logit gradient dl."""
    B, N, H, D = x.shape
    t = np.asarray(tau).reshape(1, H, 1, 1)
    du = dl / t
    W4 = _w4(W, B, H)
    dx = np.einsum("bhng,bhgd->bnhd", du, W4)
    dW4 = np.einsum("bhng,bnhd->bhgd", du, x)
    db3 = du.sum(axis=2)
    dtau = (dl * (-L / t)).sum(axis=(0, 2, 3))
    dW = _reduce_param(dW4, np.shape(W))
    db = None if bias is None else _reduce_param(db3, np.shape(bias))
    return dx, dW, db, dtau


def _jacobian(w, dw):
    return w * (dw - (w * dw).sum(axis=-1, keepdims=True))


def slice_bwd(x, fx, W, bias, tau, dz, ds):
    """dx, dfx, dW, db, dtau of the slice for upstream dz (B, H, G, DV) and
    ds (B, H, G) (None = zeros). db is None when bias is None."""
    L = logits(x, W, bias, tau)
    w = membership(x, W, bias, tau)
    if ds is None:
        ds = np.zeros(dz.shape[:-1], dtype=dz.dtype)
    dfx = np.einsum("bhng,bhgv->bnhv", w, dz)
    dw = np.einsum("bnhv,bhgv->bhng", fx, dz) + ds[:, :, None, :]
    dx, dW, db, dtau = _param_grads(x, W, bias, tau, L, _jacobian(w, dw))
    return dx, dfx, dW, db, dtau


def deslice_bwd(x, W, bias, tau, tokens, dout):
    """dx, dtokens, dW, db, dtau of the deslice for upstream dout."""
    L = logits(x, W, bias, tau)
    w = membership(x, W, bias, tau)
    dtok = np.einsum("bhng,bnhv->bhgv", w, dout)
    dw = np.einsum("bnhv,bhgv->bhng", dout, tokens)
    dx, dW, db, dtau = _param_grads(x, W, bias, tau, L, _jacobian(w, dw))
    return dx, dtok, dW, db, dtau


def coupling_round(x, fx, W, bias, tau, r, eps=1e-5, mix=None):
    """One slice -> normalise -> mix -> deslice coupling, forward and the
    backward of loss = sum(out * r) (the benchmark's round). ``mix`` is a
    (DV, DV) matrix applied to the normalised tokens (None = identity).

    Returns a dict with out, z_num, s and the gradients of x, fx, W, bias
    (None without one) and tau."""
    z, s = slice_fwd(x, fx, W, bias, tau)
    den = (s + eps)[..., None]
    zn = z / den
    tok = zn if mix is None else zn @ mix
    out = deslice_fwd(x, W, bias, tau, tok)
    dx1, dtok, dW1, db1, dt1 = deslice_bwd(x, W, bias, tau, tok, r)
    dzn = dtok if mix is None else dtok @ np.asarray(mix).T
    dz = dzn / den
    ds = -(dzn * z).sum(axis=-1) / (s + eps) ** 2
    dx2, dfx, dW2, db2, dt2 = slice_bwd(x, fx, W, bias, tau, dz, ds)
    return {"out": out, "z_num": z, "s": s, "grad:x": dx1 + dx2,
            "grad:fx": dfx, "grad:W": dW1 + dW2,
            "grad:b": None if bias is None else db1 + db2,
            "grad:tau": dt1 + dt2}
