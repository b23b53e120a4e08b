"""The ``flashslice.kernels`` operator surface over the native B200 library.

Same public names, arguments, shapes, dtypes, custom-op schemas and error
behaviour as the reference (Shizheng-Wen/flashslice v0.3.0,
``flashslice/kernels/slice_ops.py``); every op runs in the sm_100a kernels of
``libflashslice_b200.so`` through its C ABI (``include/flashslice_b200.h``).

Math (``slice_ops.py:5-13``): per point n, head h and slot g,
``w = softmax_g((x_mid . W + b) / tau)``; the slice pools
``z_num[g] = sum_n w fx_mid``, ``s[g] = sum_n w``; the deslice scatters
``out[n] = sum_g w tokens[g]``. The (B, H, N, G) weights are never written to
memory; the backward recomputes them.

Two contracts, routed by shape exactly as the reference routes
(``slice_ops.py:387-444``): the single-tile family (D and G powers of two in
[16, 128], DV = D) forms the softmax whole per point and returns no
statistics; the G-blocked family (every other shape, or forced by
``set_kernel_mode``) works from per-point statistics (m, l) that either op
can hand to the other.

Dot levels (``set_dot_mode``): every level is accepted and computed with
fp32 products and fp32 accumulation, i.e. at least at the precision the
level asks for.
"""

import os

import ctypes

import torch

from . import _native as nat
from . import _state

# --------------------------------------------------------------------------- modes

# 0=ieee fp32, 1=tf32 value dots, 2=bf16 value dots, 3=all dots bf16,
# 4=tf32x3 (slice_ops.py:336-345)
_DOT_LEVELS = {"": 0, "ieee": 0, "tf32": 1, "bf16v": 2, "bf16": 3, "tf32x3": 4}
_DOT_ENV = os.environ.get("FLASHSLICE_DOT_MODE", "").lower()


def set_dot_mode(mode):
    """'ieee' (default), 'tf32', 'bf16v', 'bf16' or 'tf32x3' -- overrides
    FLASHSLICE_DOT_MODE (``slice_ops.py:346-352``)."""
    global _DOT_ENV
    mode = (mode or "").lower()
    if mode not in _DOT_LEVELS:
        raise ValueError("dot mode must be one of %s, got %r"
                         % (sorted(k for k in _DOT_LEVELS if k), mode))
    _DOT_ENV = mode


def _dot_mode(t):
    """The dot level for inputs of t's dtype: the bf16 levels fall back to
    tf32 on fp32 inputs (``slice_ops.py:355-359``)."""
    lvl = _DOT_LEVELS[_DOT_ENV]
    if lvl in (2, 3) and t.dtype == torch.float32:
        return 1
    return lvl


_D_MAX = 256
_KERNEL_MODES = ("auto", "single-tile", "blocked")
_KERNEL_MODE = os.environ.get("FLASHSLICE_KERNEL_MODE", "").lower() or "auto"


def set_kernel_mode(mode):
    """'auto' (default), 'single-tile' or 'blocked' -- overrides
    FLASHSLICE_KERNEL_MODE (``slice_ops.py:373-384``)."""
    global _KERNEL_MODE
    if mode not in _KERNEL_MODES:
        raise ValueError("kernel mode must be one of %s, got %r" % (_KERNEL_MODES, mode))
    _KERNEL_MODE = mode


def _pow2_in(v, lo, hi):
    return lo <= v <= hi and (v & (v - 1)) == 0


def single_tile_dims(d, g, dv=None):
    """True when the single-tile contract serves (D, G): both powers of two
    in [16, 128] and the value width equal to D (``slice_ops.py:387-393``)."""
    if dv is not None and dv != d:
        return False
    return _pow2_in(d, 16, 128) and _pow2_in(g, 16, 128)


def unsupported_dims(d, g, dv=None):
    """Why the fused ops cannot serve these dims, or None if they can
    (``slice_ops.py:396-420``): the logits width D and the value width DV
    must lie in [1, 256], the slot count G must be positive."""
    if not 1 <= d <= _D_MAX:
        return ("dim_head=%d is outside the fused kernels' supported range [1, %d]"
                % (d, _D_MAX))
    if dv is not None and not 1 <= dv <= _D_MAX:
        return ("value width %d is outside the fused kernels' supported range [1, %d]"
                % (dv, _D_MAX))
    if g < 1:
        return "slice_num=%d is not a positive slice count" % g
    return None


def _check_dims(d, g, dv=None):
    why = unsupported_dims(d, g, dv)
    if why:
        raise ValueError("fused_slice: " + why)


def _use_blocked(d, g, dv=None, dot=0, device=None):
    """Route a shape: False = the single-tile contract, True = G-blocked
    (``slice_ops.py:429-444``)."""
    if _KERNEL_MODE == "blocked":
        return True
    if _KERNEL_MODE == "single-tile":
        if not single_tile_dims(d, g, dv):
            raise ValueError("kernel mode 'single-tile' cannot serve dim_head=%d, "
                             "slice_num=%d, value width %s (powers of two in [16, 128], "
                             "equal widths)" % (d, g, dv))
        return False
    return not single_tile_dims(d, g, dv)


# The reference keeps Triton tile tables per GPU class (slice_ops.py:270-302).
# This build has one native implementation for sm_100a; the selector is kept
# so that code which sets or reads it runs unchanged.
_TILE_TABLES = ("hopper", "ada")
_TILE_TABLE = os.environ.get("FLASHSLICE_TILE_TABLE", "").lower() or "auto"
_HOPPER_SMEM = 200 * 1024


def set_tile_table(name):
    """'auto' (default), 'hopper' or 'ada'. Accepted for compatibility; the
    native kernels do not depend on it."""
    global _TILE_TABLE
    if name not in ("auto",) + _TILE_TABLES:
        raise ValueError("tile table must be 'auto', 'hopper' or 'ada', got %r" % (name,))
    _TILE_TABLE = name


def tile_table(device=None):
    """The tile-table class the reference would use on ``device``."""
    if _TILE_TABLE != "auto":
        return _TILE_TABLE
    idx = torch.cuda.current_device() if device is None else torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    smem = torch.cuda.get_device_properties(idx).shared_memory_per_block_optin
    return "hopper" if smem >= _HOPPER_SMEM else "ada"


# --------------------------------------------------------------------------- shapes

def _lead2(t, trailing):
    """(batch, heads) extents of a weight-like tensor's leading dims, 1 where
    absent (``slice_ops.py:455-458``)."""
    return ((1, 1) + tuple(t.shape[:-trailing]))[-2:]


def _prep_wb(x_mid, weight, bias):
    """Validate weight (G, D) | (H, G, D) | (B, H, G, D) and bias None | (G,)
    | (H, G) | (B, H, G) against x_mid (B, N, H, D); a None bias becomes
    zeros(G) (``slice_ops.py:503-526``). Returns (weight, bias, G)."""
    if x_mid.dim() != 4:
        raise ValueError("x_mid must be (B, N, H, D), got shape %s" % (tuple(x_mid.shape),))
    B, N, H, D = x_mid.shape
    if weight.dim() not in (2, 3, 4):
        raise ValueError("weight must be (G, D), (H, G, D) or (B, H, G, D), got shape %s"
                         % (tuple(weight.shape),))
    G = weight.shape[-2]
    if weight.shape[-1] != D:
        raise ValueError("weight's last dim is %d, x_mid's head width is %d"
                         % (weight.shape[-1], D))
    if bias is None:
        bias = weight.new_zeros(G)
    elif bias.dim() not in (1, 2, 3) or bias.shape[-1] != G:
        raise ValueError("bias must be (G,), (H, G) or (B, H, G) with G=%d, got shape %s"
                         % (G, tuple(bias.shape)))
    for name, t, trailing in (("weight", weight, 2), ("bias", bias, 1)):
        for got, want, axis in zip(tuple(t.shape[:-trailing])[::-1], (H, B), ("heads", "batch")):
            if got not in (1, want):
                raise ValueError("%s has %d along %s, x_mid has %d" % (name, got, axis, want))
    return weight, bias, G


def _extents(weight, bias, B, H):
    Bw, Hw = _lead2(weight, 2)
    Bb, Hb = _lead2(bias, 1)
    for name, got in (("weight", (Bw, Hw)), ("bias", (Bb, Hb))):
        if got[0] not in (1, B) or got[1] not in (1, H):
            raise ValueError("%s has (batch, heads) = %s, x_mid has (%d, %d)"
                             % (name, got, B, H))
    if bias.shape[-1] != weight.shape[-2]:
        raise ValueError("bias has %d slices, weight %d" % (bias.shape[-1], weight.shape[-2]))
    return Bw, Hw, Bb, Hb


# --------------------------------------------------------------------------- native calls

def _f32(t):
    return t.contiguous() if t.dtype == torch.float32 else t.float().contiguous()


def _point_dtype(*ts):
    """The one dtype the point tensors of a call travel in: their common
    dtype when the kernels read it natively, else fp32."""
    dts = {t.dtype for t in ts}
    if len(dts) == 1:
        dt = dts.pop()
        if dt in nat.DTYPE_CODE:
            return dt
    return torch.float32


def _check_device(*ts):
    dev = ts[0].device
    if dev.type != "cuda":
        raise RuntimeError("flashslice_b200 ops run on CUDA tensors only (got %s); there is "
                           "no CPU implementation" % dev)
    for t in ts[1:]:
        if t is not None and t.device != dev:
            raise ValueError("all inputs must be on %s, got %s" % (dev, t.device))


class _Call:
    """Arguments of one native call prepared from the op's tensors."""

    def __init__(self, x_mid, dv, weight, bias, tau, dot, family, flags, pdtype):
        B, N, H, D = x_mid.shape
        self.B, self.N, self.H, self.D, self.DV = B, N, H, D, dv
        self.G = weight.shape[-2]
        self.ext = _extents(weight, bias, B, H)
        self.w = _f32(weight)
        self.b = _f32(bias)
        self.tau = _f32(tau)
        if self.tau.numel() != H:
            raise ValueError("tau must have H=%d entries, got %d" % (H, self.tau.numel()))
        Bw, Hw, Bb, Hb = self.ext
        self.prob = nat.Problem(B, N, H, D, dv, self.G, nat.DTYPE_CODE[pdtype], int(dot), family,
                                1 if _state.stats_mode == "two-pass" else 0, Bw, Hw, Bb, Hb,
                                flags, nat.ENGINES[_state.engine])
        self.device = x_mid.device

    def workspace(self, op):
        return nat.workspace(op, self.prob, self.device)


def _pt(t, dtype):
    return t if t.dtype == dtype else t.to(dtype)


def native_slice(x_mid, fx_mid, weight, bias, tau, stats, dot, family, want_stats):
    """z_num, s and (blocked family) the statistics used."""
    _check_device(x_mid, fx_mid, weight, bias, tau, stats)
    B, N, H, _ = x_mid.shape
    G, DV = weight.shape[-2], fx_mid.shape[3]
    dev = x_mid.device
    z = torch.empty(B, H, G, DV, device=dev, dtype=torch.float32)
    s = torch.empty(B, H, G, device=dev, dtype=torch.float32)
    st_out = None
    if family == nat.FAMILY_BLOCKED and stats is None and want_stats:
        st_out = torch.empty(B, H, 2, N, device=dev, dtype=torch.float32)
    st_in = None if stats is None else _f32(stats)
    if N == 0:
        z.zero_()
        s.zero_()
        return z, s, (st_in if st_in is not None else st_out)
    pd = _point_dtype(x_mid, fx_mid)
    xm, fm = _pt(x_mid, pd), _pt(fx_mid, pd)
    flags = (nat.FLAG_STATS_IN if st_in is not None else 0) | \
        (nat.FLAG_STATS_OUT if st_out is not None else 0)
    c = _Call(xm, DV, weight, bias, tau, dot, family, flags, pd)
    ws, nws = c.workspace(nat.OP_SLICE_FWD)
    lib = nat.load()
    with torch.cuda.device(dev):
        nat.check(lib.fs_slice_fwd(
            c.prob, nat.t4(xm), nat.t4(fm), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau),
            nat.ptr(st_in), nat.ptr(st_out), nat.ptr(z), nat.ptr(s), nat.ptr(ws), nws,
            nat.stream_of(xm)))
    return z, s, (st_in if st_in is not None else st_out)


def native_deslice(x_mid, weight, bias, tau, tokens, stats, dot, family, want_stats):
    """out (B, N, H, DV) in x_mid's dtype and (blocked family) the statistics."""
    _check_device(x_mid, weight, bias, tau, tokens, stats)
    B, N, H, _ = x_mid.shape
    DV = tokens.shape[3]
    dev = x_mid.device
    out = torch.empty(B, N, H, DV, device=dev, dtype=x_mid.dtype)
    st_out = None
    if family == nat.FAMILY_BLOCKED and stats is None and want_stats:
        st_out = torch.empty(B, H, 2, N, device=dev, dtype=torch.float32)
    st_in = None if stats is None else _f32(stats)
    if N == 0:
        return out, (st_in if st_in is not None else st_out)
    pd = _point_dtype(x_mid)
    xm = _pt(x_mid, pd)
    o = out if out.dtype == pd else torch.empty(B, N, H, DV, device=dev, dtype=pd)
    flags = (nat.FLAG_STATS_IN if st_in is not None else 0) | \
        (nat.FLAG_STATS_OUT if st_out is not None else 0)
    c = _Call(xm, DV, weight, bias, tau, dot, family, flags, pd)
    tok = _f32(tokens)
    ws, nws = c.workspace(nat.OP_DESLICE_FWD)
    lib = nat.load()
    with torch.cuda.device(dev):
        nat.check(lib.fs_deslice_fwd(
            c.prob, nat.t4(xm), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau), nat.ptr(tok),
            nat.ptr(st_in), nat.ptr(st_out), nat.t4(o), nat.ptr(ws), nws, nat.stream_of(xm)))
    if o is not out:
        out.copy_(o)
    return out, (st_in if st_in is not None else st_out)


def _param_grads(c, weight, bias, tau, dW, db, dt):
    return (dW.reshape(weight.shape).to(weight.dtype), db.reshape(bias.shape).to(bias.dtype),
            dt.to(tau.dtype))


def native_slice_bwd(x_mid, fx_mid, weight, bias, tau, stats, dz_num, ds, dot, family):
    """dx_mid, dfx_mid, dW, db, dtau of the slice."""
    _check_device(x_mid, fx_mid, weight, bias, tau, stats, dz_num, ds)
    B, N, H, D = x_mid.shape
    DV = fx_mid.shape[3]
    dev = x_mid.device
    dxm = torch.empty_like(x_mid)
    dfx = torch.empty_like(fx_mid)
    Bw, Hw = _lead2(weight, 2)
    Bb, Hb = _lead2(bias, 1)
    G = weight.shape[-2]
    dW = torch.empty(Bw, Hw, G, D, device=dev, dtype=torch.float32)
    db = torch.empty(Bb, Hb, G, device=dev, dtype=torch.float32)
    dt = torch.empty(H, device=dev, dtype=torch.float32)
    if N == 0:
        dxm.zero_(), dfx.zero_(), dW.zero_(), db.zero_(), dt.zero_()
        return (dxm, dfx) + _param_grads(None, weight, bias, tau, dW, db, dt)
    pd = _point_dtype(x_mid, fx_mid)
    xm, fm = _pt(x_mid, pd), _pt(fx_mid, pd)
    dxo = dxm if dxm.dtype == pd else torch.empty_like(xm)
    dfo = dfx if dfx.dtype == pd else torch.empty_like(fm)
    st_in = None if stats is None else _f32(stats)
    c = _Call(xm, DV, weight, bias, tau, dot, family,
              nat.FLAG_STATS_IN if st_in is not None else 0, pd)
    dzn, dsf = _f32(dz_num), _f32(ds)
    ws, nws = c.workspace(nat.OP_SLICE_BWD)
    lib = nat.load()
    with torch.cuda.device(dev):
        nat.check(lib.fs_slice_bwd(
            c.prob, nat.t4(xm), nat.t4(fm), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau),
            nat.ptr(st_in), nat.ptr(dzn), nat.ptr(dsf), nat.t4(dxo), nat.t4(dfo), nat.ptr(dW),
            nat.ptr(db), nat.ptr(dt), nat.ptr(ws), nws, nat.stream_of(xm)))
    if dxo is not dxm:
        dxm.copy_(dxo)
    if dfo is not dfx:
        dfx.copy_(dfo)
    return (dxm, dfx) + _param_grads(c, weight, bias, tau, dW, db, dt)


def native_deslice_bwd(x_mid, weight, bias, tau, tokens, stats, d_out, dot, family):
    """dx_mid, dtokens, dW, db, dtau of the deslice."""
    _check_device(x_mid, weight, bias, tau, tokens, stats, d_out)
    B, N, H, D = x_mid.shape
    DV = tokens.shape[3]
    dev = x_mid.device
    dxm = torch.empty_like(x_mid)
    Bw, Hw = _lead2(weight, 2)
    Bb, Hb = _lead2(bias, 1)
    G = weight.shape[-2]
    dtok = torch.empty(B, H, G, DV, device=dev, dtype=torch.float32)
    dW = torch.empty(Bw, Hw, G, D, device=dev, dtype=torch.float32)
    db = torch.empty(Bb, Hb, G, device=dev, dtype=torch.float32)
    dt = torch.empty(H, device=dev, dtype=torch.float32)
    if N == 0:
        dxm.zero_(), dtok.zero_(), dW.zero_(), db.zero_(), dt.zero_()
        return (dxm, dtok.to(tokens.dtype)) + _param_grads(None, weight, bias, tau, dW, db, dt)
    pd = _point_dtype(x_mid, d_out)
    xm, dom = _pt(x_mid, pd), _pt(d_out, pd)
    dxo = dxm if dxm.dtype == pd else torch.empty_like(xm)
    st_in = None if stats is None else _f32(stats)
    c = _Call(xm, DV, weight, bias, tau, dot, family,
              nat.FLAG_STATS_IN if st_in is not None else 0, pd)
    tok = _f32(tokens)
    ws, nws = c.workspace(nat.OP_DESLICE_BWD)
    lib = nat.load()
    with torch.cuda.device(dev):
        nat.check(lib.fs_deslice_bwd(
            c.prob, nat.t4(xm), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau), nat.ptr(tok),
            nat.ptr(st_in), nat.t4(dom), nat.t4(dxo), nat.ptr(dtok), nat.ptr(dW), nat.ptr(db),
            nat.ptr(dt), nat.ptr(ws), nws, nat.stream_of(xm)))
    if dxo is not dxm:
        dxm.copy_(dxo)
    return (dxm, dtok.to(tokens.dtype)) + _param_grads(c, weight, bias, tau, dW, db, dt)


def _coupled_call(x_mid, fx_mid, weight, bias, tau, dot):
    """The native problem of a coupled backward, or None when the coupled
    kernel does not serve these inputs (shape, dtype, engine, layout)."""
    if fx_mid.shape[3] != x_mid.shape[3] or x_mid.dtype not in (torch.float32, torch.bfloat16) \
            or fx_mid.dtype != x_mid.dtype or not x_mid.is_cuda:
        return None
    c = _Call(x_mid, fx_mid.shape[3], weight, bias, tau, dot, nat.FAMILY_SINGLE, 0,
              x_mid.dtype)
    return c if nat.load().fs_coupled_supported(ctypes.byref(c.prob)) else None


def native_coupled_bwd(x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds, dot):
    """dx_mid, dfx_mid, dW, db, dtau of a whole coupling round (both ops'
    contributions summed), or None when the coupled kernel does not serve the
    inputs."""
    _check_device(x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds)
    B, N, H, D = x_mid.shape
    if N == 0:
        return None
    c = _coupled_call(x_mid, fx_mid, weight, bias, tau, dot)
    if c is None or d_out.dtype != x_mid.dtype:
        return None
    dev = x_mid.device
    dxm = torch.empty_like(x_mid)
    dfx = torch.empty_like(fx_mid)
    Bw, Hw = _lead2(weight, 2)
    Bb, Hb = _lead2(bias, 1)
    G = weight.shape[-2]
    dW = torch.empty(Bw, Hw, G, D, device=dev, dtype=torch.float32)
    db = torch.empty(Bb, Hb, G, device=dev, dtype=torch.float32)
    dt = torch.empty(H, device=dev, dtype=torch.float32)
    tok, dzn, dsf = _f32(tokens), _f32(dz_num), _f32(ds)
    ws, nws = c.workspace(nat.OP_SLICE_BWD)
    lib = nat.load()
    with torch.cuda.device(dev):
        rc = lib.fs_coupled_bwd(
            c.prob, nat.t4(x_mid), nat.t4(fx_mid), nat.t4(d_out), nat.ptr(c.w), nat.ptr(c.b),
            nat.ptr(c.tau), nat.ptr(tok), nat.ptr(dzn), nat.ptr(dsf), nat.t4(dxm), nat.t4(dfx),
            nat.ptr(dW), nat.ptr(db), nat.ptr(dt), nat.ptr(ws), nws, nat.stream_of(x_mid))
    if rc == nat.FS_ERR_UNSUPPORTED:
        return None
    nat.check(rc)
    return (dxm, dfx) + _param_grads(c, weight, bias, tau, dW, db, dt)


def native_stats(x_mid, weight, bias, tau, dot=0):
    """(B, H, 2, N) fp32 statistics of the slice logits."""
    _check_device(x_mid, weight, bias, tau)
    B, N, H, D = x_mid.shape
    st = torch.empty(B, H, 2, N, device=x_mid.device, dtype=torch.float32)
    if N == 0:
        return st
    pd = _point_dtype(x_mid)
    xm = _pt(x_mid, pd)
    c = _Call(xm, D, weight, bias, tau, dot, nat.FAMILY_BLOCKED, 0, pd)
    lib = nat.load()
    with torch.cuda.device(x_mid.device):
        nat.check(lib.fs_compute_stats(c.prob, nat.t4(xm), nat.ptr(c.w), nat.ptr(c.b),
                                       nat.ptr(c.tau), nat.ptr(st), nat.stream_of(xm)))
    return st


# --------------------------------------------------------------------------- custom ops
# Same schemas as the reference (slice_ops.py:787-801), so that torch.compile
# sees each op as one opaque node and the whole layer stays one graph.

_LIB = torch.library.Library("flashslice", "DEF")
_LIB.define("flash_slice(Tensor x_mid, Tensor fx_mid, Tensor weight, Tensor bias, "
            "Tensor tau, int dot) -> (Tensor, Tensor)")
_LIB.define("flash_slice_bwd(Tensor x_mid, Tensor fx_mid, Tensor weight, Tensor bias, "
            "Tensor tau, Tensor dz_num, Tensor ds, int dot) "
            "-> (Tensor, Tensor, Tensor, Tensor, Tensor)")
_LIB.define("flash_deslice(Tensor x_mid, Tensor weight, Tensor bias, Tensor tau, "
            "Tensor tokens, int dot) -> Tensor")
_LIB.define("flash_deslice_bwd(Tensor x_mid, Tensor weight, Tensor bias, Tensor tau, "
            "Tensor tokens, Tensor d_out, int dot) "
            "-> (Tensor, Tensor, Tensor, Tensor, Tensor)")
# No reference counterpart: the tied backward of a coupling round (below).
_LIB.define("coupled_bwd(Tensor x_mid, Tensor fx_mid, Tensor d_out, Tensor weight, "
            "Tensor bias, Tensor tau, Tensor tokens, Tensor dz_num, Tensor ds, int dot) "
            "-> (Tensor, Tensor, Tensor, Tensor, Tensor)")


def _slice_impl(x_mid, fx_mid, weight, bias, tau, dot):
    z, s, _ = native_slice(x_mid, fx_mid, weight, bias, tau, None, dot, nat.FAMILY_SINGLE,
                           False)
    return z, s


# The op-by-op backward ops at G = 64 run on the tensor cores through the
# coupled backward kernel with the other op's contribution zeroed: the slice
# backward is the coupled one with zero tokens (d_out tok^T vanishes; fx is
# passed in d_out's place), the deslice backward is the dtokens pass (a slice
# forward of d_out) and the coupled one with zero dz_num and ds (its dfx,
# w dz_num = 0, is discarded). Exact zeros: the split products of 0 are 0.
# Shapes the coupled kernel does not serve run the FMA backward kernels.

def _slice_bwd_impl(x_mid, fx_mid, weight, bias, tau, dz_num, ds, dot):
    if weight.shape[-2] == 64 and x_mid.shape[1] > 0:
        r = native_coupled_bwd(x_mid, fx_mid, fx_mid, weight, bias, tau,
                               torch.zeros_like(dz_num, dtype=torch.float32), dz_num, ds, dot)
        if r is not None:
            return r
    return native_slice_bwd(x_mid, fx_mid, weight, bias, tau, None, dz_num, ds, dot,
                            nat.FAMILY_SINGLE)


def _deslice_impl(x_mid, weight, bias, tau, tokens, dot):
    out, _ = native_deslice(x_mid, weight, bias, tau, tokens, None, dot, nat.FAMILY_SINGLE,
                            False)
    return out


def _deslice_bwd_impl(x_mid, weight, bias, tau, tokens, d_out, dot):
    if weight.shape[-2] == 64 and x_mid.shape[1] > 0 and \
            _coupled_call(x_mid, d_out, weight, bias, tau, dot) is not None:
        dtok, s = _slice_impl(x_mid, d_out, weight, bias, tau, dot)
        r = native_coupled_bwd(x_mid, d_out, d_out, weight, bias, tau, tokens,
                               torch.zeros_like(dtok), torch.zeros_like(s), dot)
        if r is not None:
            dxm, _, dw, db, dt = r
            return dxm, dtok.to(tokens.dtype), dw, db, dt
    return native_deslice_bwd(x_mid, weight, bias, tau, tokens, None, d_out, dot,
                              nat.FAMILY_SINGLE)


def _coupled_bwd_impl(x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds, dot):
    r = native_coupled_bwd(x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds, dot)
    if r is not None:
        return r
    # inputs the coupled kernel does not serve: the two backward ops, summed
    dxd, _, dwd, dbd, dtd = native_deslice_bwd(x_mid, weight, bias, tau, tokens, None, d_out,
                                               dot, nat.FAMILY_SINGLE)
    dxs, dfx, dws, dbs, dts = native_slice_bwd(x_mid, fx_mid, weight, bias, tau, None, dz_num,
                                               ds, dot, nat.FAMILY_SINGLE)
    return dxd + dxs, dfx, dwd + dws, dbd + dbs, dtd + dts


_LIB.impl("flash_slice", _slice_impl, "CUDA")
_LIB.impl("flash_slice_bwd", _slice_bwd_impl, "CUDA")
_LIB.impl("flash_deslice", _deslice_impl, "CUDA")
_LIB.impl("flash_deslice_bwd", _deslice_bwd_impl, "CUDA")
_LIB.impl("coupled_bwd", _coupled_bwd_impl, "CUDA")


@torch.library.register_fake("flashslice::flash_slice")
def _(x_mid, fx_mid, weight, bias, tau, dot):
    B, N, H, D = x_mid.shape
    G = weight.shape[-2]
    return (x_mid.new_empty((B, H, G, fx_mid.shape[3]), dtype=torch.float32),
            x_mid.new_empty((B, H, G), dtype=torch.float32))


def _fresh(t):
    """An output in t's shape, dtype and device with contiguous strides: the
    parameter and token gradients come back contiguous whatever the input's
    strides (a permuted per-sample weight included), as the CUDA impls make
    them, so that compiled graphs see the strides the kernels produce."""
    return t.new_empty(t.shape)


@torch.library.register_fake("flashslice::flash_slice_bwd")
def _(x_mid, fx_mid, weight, bias, tau, dz_num, ds, dot):
    return (torch.empty_like(x_mid), torch.empty_like(fx_mid), _fresh(weight), _fresh(bias),
            _fresh(tau))


@torch.library.register_fake("flashslice::flash_deslice")
def _(x_mid, weight, bias, tau, tokens, dot):
    B, N, H, D = x_mid.shape
    return x_mid.new_empty((B, N, H, tokens.shape[3]))


@torch.library.register_fake("flashslice::flash_deslice_bwd")
def _(x_mid, weight, bias, tau, tokens, d_out, dot):
    return (torch.empty_like(x_mid), _fresh(tokens), _fresh(weight), _fresh(bias),
            _fresh(tau))


@torch.library.register_fake("flashslice::coupled_bwd")
def _(x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds, dot):
    return (torch.empty_like(x_mid), torch.empty_like(fx_mid), _fresh(weight), _fresh(bias),
            _fresh(tau))


def _slice_setup(ctx, inputs, output):
    x_mid, fx_mid, weight, bias, tau, dot = inputs
    ctx.save_for_backward(x_mid, fx_mid, weight, bias, tau)
    ctx.dot = dot


def _slice_grad(ctx, dz_num, ds):
    x_mid, fx_mid, weight, bias, tau = ctx.saved_tensors
    if ds is None:
        ds = torch.zeros(dz_num.shape[:-1], device=dz_num.device, dtype=torch.float32)
    dxm, dfx, dw, db, dtau = torch.ops.flashslice.flash_slice_bwd(
        x_mid, fx_mid, weight, bias, tau, dz_num, ds, ctx.dot)
    return dxm, dfx, dw, db, dtau, None


def _deslice_setup(ctx, inputs, output):
    x_mid, weight, bias, tau, tokens, dot = inputs
    ctx.save_for_backward(x_mid, weight, bias, tau, tokens)
    ctx.dot = dot


def _deslice_grad(ctx, d_out):
    x_mid, weight, bias, tau, tokens = ctx.saved_tensors
    dxm, dtok, dw, db, dtau = torch.ops.flashslice.flash_deslice_bwd(
        x_mid, weight, bias, tau, tokens, d_out, ctx.dot)
    return dxm, dw, db, dtau, dtok, None


torch.library.register_autograd("flashslice::flash_slice", _slice_grad,
                                setup_context=_slice_setup)
torch.library.register_autograd("flashslice::flash_deslice", _deslice_grad,
                                setup_context=_deslice_setup)


# --------------------------------------------------------------------------- coupling round
# Forward: z_num, s = slice; tokens = mix(z_num / (s + eps)); out = deslice.
# Backward (tied; no reference counterpart as one op): the tokens' gradient
# dtokens = sum_n w^T d_out is a slice forward with d_out in place of fx;
# autograd through mix and the normalisation gives dz_num and ds; then one
# coupled kernel forms the slice's and the deslice's remaining gradients
# together (dx once, without summing two dx tensors). The reference runs the
# two backward ops (slice_ops.py:822-885) and autograd adds their dx.

def _tc_strides(t):
    """t, or a contiguous copy when its layout is not one the tensor-core
    kernels read (unit width stride, 16-byte aligned strides and base)."""
    per16 = 16 // t.element_size()
    ok = t.stride(3) == 1 and all(st % per16 == 0 for st in t.stride()[:3]) and \
        t.data_ptr() % 16 == 0
    return t if ok else t.contiguous()


def _rank_sum(t, group):
    if group is None:
        return t
    from ..sharded import ordered_sum
    return ordered_sum(t, group)


def _rank_sum_many(ts, group):
    if group is None:
        return ts
    from ..sharded import ordered_sum_many
    return ordered_sum_many(ts, group)


class _CouplingRound(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_mid, fx_mid, weight, bias, tau, eps, dot, mix, group, ops, *params):
        z, s = ops.flash_slice(x_mid, fx_mid, weight, bias, tau, dot)
        z, s = _rank_sum_many([z, s], group)
        den = s + eps
        tin = z / den[..., None]
        graph = None
        if mix is not None:
            leaf = tin.detach().requires_grad_(True)
            with torch.enable_grad():
                tok_graph = mix(leaf)
            graph = (leaf, tok_graph)
            tok = tok_graph.detach()
        else:
            tok = tin
        out = ops.flash_deslice(x_mid, weight, bias, tau, tok, dot)
        ctx.save_for_backward(x_mid, fx_mid, weight, bias, tau, z, den, tok)
        ctx.graph, ctx.params, ctx.dot, ctx.group, ctx.ops = graph, params, dot, group, ops
        return out

    @staticmethod
    def backward(ctx, d_out):
        x_mid, fx_mid, weight, bias, tau, z, den, tok = ctx.saved_tensors
        d_out = _tc_strides(d_out)
        # this rank's part of the tokens' gradient; back through mix it gives
        # this rank's part of the mix parameters' gradients (summed over the
        # ranks like W's), then the tokens-in gradient is summed over ranks
        dtok, _ = ctx.ops.flash_slice(x_mid, d_out, weight, bias, tau, ctx.dot)
        pgrads = (None,) * len(ctx.params)
        if ctx.graph is not None:
            leaf, tok_graph = ctx.graph
            g = torch.autograd.grad(tok_graph, (leaf,) + tuple(ctx.params), dtok,
                                    allow_unused=True)
            dtin = g[0] if g[0] is not None else torch.zeros_like(leaf)
            pgrads = g[1:]
            ctx.graph = None
        else:
            dtin = dtok
        dtin = _rank_sum(dtin, ctx.group)
        dz = dtin / den[..., None]
        ds = -(dtin * z).sum(-1) / (den * den)
        dx, dfx, dw, db, dtau = ctx.ops.coupled_bwd(
            x_mid, fx_mid, d_out, weight, bias, tau, tok, dz, ds, ctx.dot)
        need = ctx.needs_input_grad
        grads = tuple(g if n else None for g, n in zip((dx, dfx, dw, db, dtau), need[:5]))
        return grads + (None, None, None, None, None) + tuple(pgrads)


def fused_coupling(x_mid, fx_mid, weight, bias, tau, mix=None, mix_params=None, eps=1e-5,
                   group=None, _ops=None):
    """One coupling round: z_num, s = fused_slice(...); tokens =
    mix(z_num / (s + eps)[..., None]) (identity when mix is None); returns
    fused_deslice(x_mid, weight, bias, tau, tokens). Same values as that
    composition; its backward is tied: the two ops' point gradients are formed
    in one pass over the points. ``mix`` is any differentiable function of the
    (B, H, G, DV) tokens; the gradients of its parameters are returned only
    for those listed in ``mix_params`` (by default the parameters of ``mix``
    when it is a ``torch.nn.Module``). The blocked family, and calls with
    gradients disabled, run the plain composition.

    ``group``: a process group over which the points are sharded (each rank
    passes its own points): z_num and s, and in the backward the gradient of
    the normalised tokens, are summed over the ranks in rank order (bitwise
    the same on every rank); the returned gradients of W, b, tau and the mix
    parameters are this rank's part, to be summed over the ranks like those
    of the op-by-op sharded coupling (``flashslice_b200.sharded``).

    ``_ops`` replaces the three ops the round calls (``flash_slice``,
    ``flash_deslice``, ``coupled_bwd``; tests run the rank logic on CPU
    with eager stand-ins)."""
    weight, bias, G = _prep_wb(x_mid, weight, bias)
    D, DV = x_mid.shape[3], fx_mid.shape[3]
    _check_dims(D, G, DV)
    dot = _dot_mode(x_mid)
    if mix_params is None:
        mix_params = [q for q in mix.parameters()] if isinstance(mix, torch.nn.Module) else []
    params = tuple(q for q in mix_params if q.requires_grad)
    if group is not None and torch.distributed.get_world_size(group) == 1:
        group = None
    # Under torch.compile the round is the plain composition of the custom
    # ops (each with its registered autograd), which traces into one graph
    # with its backward; the tied backward's autograd.Function runs a Python
    # mix through torch.autograd.grad, which a compiled graph cannot hold.
    if _ops is None and (_use_blocked(D, G, DV, dot, x_mid.device) or
                         not torch.is_grad_enabled() or torch.compiler.is_compiling()):
        if group is not None:
            from ..sharded import sharded_coupling
            return sharded_coupling(x_mid, fx_mid, weight, bias, tau, mix, eps, group)
        # the slice's per-point statistics serve the deslice (blocked family;
        # None on the single-tile path), as physics_attention.py:95-136 hands
        # them over
        z, s, st = fused_slice(x_mid, fx_mid, weight, bias, tau, return_stats=True)
        tok = z / (s + eps)[..., None]
        if mix is not None:
            tok = mix(tok)
        return fused_deslice(x_mid, weight, bias, tau, tok, stats=st)
    return _CouplingRound.apply(x_mid, fx_mid, weight, bias, tau, eps, dot, mix, group,
                                _ops if _ops is not None else torch.ops.flashslice, *params)


# --------------------------------------------------------------------------- public API

def fused_slice(x_mid, fx_mid, weight, bias, tau, return_stats=False, stats=None):
    """x_mid: (B, N, H, D); fx_mid: (B, N, H, DV); weight: (G, D), (H, G, D)
    or (B, H, G, D); bias: None, (G,), (H, G) or (B, H, G); tau: (H,).
    Returns fp32 z_num (B, H, G, DV) and s (B, H, G); normalise outside as
    z = z_num / (s + eps)[..., None].

    ``stats``: the per-point statistics of these logits from a tied op that
    ran before (``fused_deslice(..., return_stats=True)``); the statistics
    pass is then skipped. With ``return_stats=True`` a third value is
    returned: the (B, H, 2, N) fp32 statistics on the blocked path, None on
    the single-tile path (``slice_ops.py:961-996``)."""
    weight, bias, G = _prep_wb(x_mid, weight, bias)
    D, DV = x_mid.shape[3], fx_mid.shape[3]
    _check_dims(D, G, DV)
    dot = _dot_mode(x_mid)
    if _use_blocked(D, G, DV, dot, x_mid.device):
        from . import blocked  # noqa: F401  (registers the blocked ops)
        z_num, s, st = torch.ops.flashslice.slice_blk(x_mid, fx_mid, weight, bias, tau, stats,
                                                      dot)
        return (z_num, s, st.detach()) if return_stats else (z_num, s)
    z_num, s = torch.ops.flashslice.flash_slice(x_mid, fx_mid, weight, bias, tau, dot)
    return (z_num, s, None) if return_stats else (z_num, s)


def fused_deslice(x_mid, weight, bias, tau, tokens, stats=None, return_stats=False):
    """tokens: (B, H, G, DV). Returns out (B, N, H, DV) in x_mid's dtype; with
    ``return_stats=True`` (out, stats), stats None on the single-tile path.
    ``stats`` is what ``fused_slice(..., return_stats=True)`` returned for the
    same x_mid, weight, bias and tau (``slice_ops.py:999-1022``)."""
    weight, bias, G = _prep_wb(x_mid, weight, bias)
    D, DV = x_mid.shape[3], tokens.shape[3]
    _check_dims(D, G, DV)
    dot = _dot_mode(x_mid)
    if _use_blocked(D, G, DV, dot, x_mid.device):
        from . import blocked  # noqa: F401
        out, st = torch.ops.flashslice.deslice_blk(x_mid, weight, bias, tau, tokens, stats, dot)
        return (out, st.detach()) if return_stats else out
    out = torch.ops.flashslice.flash_deslice(x_mid, weight, bias, tau, tokens, dot)
    return (out, None) if return_stats else out
