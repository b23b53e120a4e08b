"""Ragged batches: samples with different point counts, packed along the
point axis, in one launch per op.

The reference plans this ("Ragged batching", ``ROADMAP.md:66-68``: samples
of different N in one launch through row splits, so that small meshes fill
the GPU) and has no implementation; the functions here follow its operator
contract per sample:

* ``x_mid``, ``fx_mid`` are ``(1, N_total, H, D)``: sample b owns rows
  ``row_splits[b] .. row_splits[b + 1]`` (``row_splits``: S + 1
  non-decreasing ints from 0 to N_total);
* weight ``(G, D) | (H, G, D) | (S, H, G, D)``, bias likewise, tokens,
  ``z_num`` ``(S, H, G, DV)`` and ``s`` ``(S, H, G)`` are per sample;
* every result equals the dense op applied to each sample alone.

The tensor-core engine serves them in one launch per op (fp32 or bf16 point
tensors, D = DV = 32, at most ``FS_MAX_SPLITS`` samples; G = 32, and G = 64
for the tied round of ``ragged_coupling``): each (sample, head) gets its
CTAs and masks the rows past its sample. Other problems run the dense ops
sample by sample (still native, one launch per sample)."""

import ctypes

import torch

from . import _native as nat
from . import _state
from .slice_ops import (_CouplingRound, _check_device, _extents, _f32, _lead2, _param_grads,
                        _prep_wb, _tc_strides, fused_coupling, fused_deslice, fused_slice)

MAX_SPLITS = 128  # FS_MAX_SPLITS


class _Shape:
    """Shape-only stand-in for a (S, N, H, D) point tensor (weight checks)."""

    def __init__(self, *shape):
        self.shape = torch.Size(shape)

    def dim(self):
        return len(self.shape)


def _splits(row_splits, n):
    r = torch.as_tensor(row_splits, dtype=torch.int64).detach().cpu().contiguous().reshape(-1)
    if r.numel() < 2 or int(r[0]) != 0 or int(r[-1]) != n or bool((r[1:] < r[:-1]).any()):
        raise ValueError("row_splits must be S + 1 >= 2 non-decreasing offsets from 0 to "
                         "N=%d, got %s" % (n, r.tolist()))
    return r


def _check_points(x_mid, *others):
    if x_mid.dim() != 4 or x_mid.shape[0] != 1:
        raise ValueError("ragged point tensors are (1, N_total, H, D), got shape %s"
                         % (tuple(x_mid.shape),))
    for t in others:
        if t is not None and tuple(t.shape[:3]) != tuple(x_mid.shape[:3]):
            raise ValueError("point tensors disagree: %s vs %s"
                             % (tuple(t.shape), tuple(x_mid.shape)))


def _rows(t, splits, b):
    return t[:, int(splits[b]):int(splits[b + 1])]


def _of(t, b, S, trailing):
    """Sample b's weight-like tensor (keeps the leading batch axis)."""
    if t.dim() == trailing + 2 and t.shape[0] == S:
        return t[b:b + 1]
    return t


class _Native:
    """One ragged problem for the C ABI; None when the tensor-core engine
    cannot serve it (the callers then go sample by sample)."""

    def __init__(self, x_mid, dv, weight, bias, tau, dot, splits):
        _, N, H, D = x_mid.shape
        S = splits.numel() - 1
        self.S, self.N, self.H, self.D, self.DV = S, N, H, D, dv
        self.G = weight.shape[-2]
        Bw, Hw, Bb, Hb = _extents(weight, bias, S, H)
        self.w, self.b, self.tau = _f32(weight), _f32(bias), _f32(tau)
        self.splits = splits  # the ABI reads the host array during the call
        self.prob = nat.Problem(S, N, H, D, dv, self.G, nat.DTYPE_CODE[x_mid.dtype], int(dot),
                                nat.FAMILY_SINGLE, 0, Bw, Hw, Bb, Hb, 0,
                                nat.ENGINES[_state.engine], ctypes.c_void_p(splits.data_ptr()))
        self.device = x_mid.device

    @staticmethod
    def make(x_mid, dv, weight, bias, tau, dot, splits, tied=False):
        """``tied``: only the slice forward, deslice forward and coupled
        backward will run (a tied round), which the engine also serves at
        G = 64; the op-by-op backward entry points serve ragged rows at G = 32
        only."""
        S = splits.numel() - 1
        slots = (32, 64) if tied else (32,)
        if (x_mid.dtype not in (torch.float32, torch.bfloat16) or S > MAX_SPLITS or
                x_mid.shape[1] == 0 or x_mid.shape[3] != 32 or dv != 32 or
                weight.shape[-2] not in slots or not x_mid.is_cuda):
            return None
        c = _Native(x_mid, dv, weight, bias, tau, dot, splits)
        return c if nat.load().fs_coupled_supported(ctypes.byref(c.prob)) else None

    def workspace(self, op):
        return nat.workspace(op, self.prob, self.device)


def native_slice(x_mid, fx_mid, weight, bias, tau, splits, dot=0):
    """(z_num (S, H, G, DV), s (S, H, G)) in one launch, or None."""
    c = _Native.make(x_mid, fx_mid.shape[3], weight, bias, tau, dot, splits, tied=True)
    if c is None or fx_mid.dtype != x_mid.dtype:
        return None
    x_mid, fx_mid = _tc_strides(x_mid), _tc_strides(fx_mid)
    z = torch.empty(c.S, c.H, c.G, c.DV, device=c.device, dtype=torch.float32)
    s = torch.empty(c.S, c.H, c.G, device=c.device, dtype=torch.float32)
    ws, nws = c.workspace(nat.OP_SLICE_FWD)
    with torch.cuda.device(c.device):
        nat.check(nat.load().fs_slice_fwd(
            c.prob, nat.t4(x_mid), nat.t4(fx_mid), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau),
            None, None, nat.ptr(z), nat.ptr(s), nat.ptr(ws), nws, nat.stream_of(x_mid)))
    return z, s


def native_deslice(x_mid, weight, bias, tau, tokens, splits, dot=0):
    """out (1, N_total, H, DV) in one launch, or None."""
    c = _Native.make(x_mid, tokens.shape[3], weight, bias, tau, dot, splits, tied=True)
    if c is None:
        return None
    x_mid = _tc_strides(x_mid)
    out = torch.empty(1, c.N, c.H, c.DV, device=c.device, dtype=x_mid.dtype)
    tok = _f32(tokens)
    ws, nws = c.workspace(nat.OP_DESLICE_FWD)
    with torch.cuda.device(c.device):
        nat.check(nat.load().fs_deslice_fwd(
            c.prob, nat.t4(x_mid), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau), nat.ptr(tok),
            None, None, nat.t4(out), nat.ptr(ws), nws, nat.stream_of(x_mid)))
    return out


def _param_bufs(c, weight, bias):
    Bw, Hw = _lead2(weight, 2)
    Bb, Hb = _lead2(bias, 1)
    dev = c.device
    return (torch.empty(Bw, Hw, c.G, c.D, device=dev, dtype=torch.float32),
            torch.empty(Bb, Hb, c.G, device=dev, dtype=torch.float32),
            torch.empty(c.H, device=dev, dtype=torch.float32))


def native_slice_bwd(x_mid, fx_mid, weight, bias, tau, dz_num, ds, splits, dot=0):
    c = _Native.make(x_mid, fx_mid.shape[3], weight, bias, tau, dot, splits)
    x_mid, fx_mid = _tc_strides(x_mid), _tc_strides(fx_mid)
    dx, dfx = torch.empty_like(x_mid), torch.empty_like(fx_mid)
    dW, db, dt = _param_bufs(c, weight, bias)
    ws, nws = c.workspace(nat.OP_SLICE_BWD)
    with torch.cuda.device(c.device):
        nat.check(nat.load().fs_slice_bwd(
            c.prob, nat.t4(x_mid), nat.t4(fx_mid), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau),
            None, nat.ptr(_f32(dz_num)), nat.ptr(_f32(ds)), nat.t4(dx), nat.t4(dfx),
            nat.ptr(dW), nat.ptr(db), nat.ptr(dt), nat.ptr(ws), nws, nat.stream_of(x_mid)))
    return (dx, dfx) + _param_grads(c, weight, bias, tau, dW, db, dt)


def native_deslice_bwd(x_mid, weight, bias, tau, tokens, d_out, splits, dot=0):
    c = _Native.make(x_mid, tokens.shape[3], weight, bias, tau, dot, splits)
    x_mid, d_out = _tc_strides(x_mid), _tc_strides(d_out.to(x_mid.dtype))
    dx = torch.empty_like(x_mid)
    dtok = torch.empty(c.S, c.H, c.G, c.DV, device=c.device, dtype=torch.float32)
    dW, db, dt = _param_bufs(c, weight, bias)
    ws, nws = c.workspace(nat.OP_DESLICE_BWD)
    with torch.cuda.device(c.device):
        nat.check(nat.load().fs_deslice_bwd(
            c.prob, nat.t4(x_mid), nat.ptr(c.w), nat.ptr(c.b), nat.ptr(c.tau),
            nat.ptr(_f32(tokens)), None, nat.t4(d_out), nat.t4(dx), nat.ptr(dtok), nat.ptr(dW),
            nat.ptr(db), nat.ptr(dt), nat.ptr(ws), nws, nat.stream_of(x_mid)))
    return (dx, dtok.to(tokens.dtype)) + _param_grads(c, weight, bias, tau, dW, db, dt)


def native_coupled_bwd(x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds, splits,
                       dot=0):
    c = _Native.make(x_mid, fx_mid.shape[3], weight, bias, tau, dot, splits, tied=True)
    x_mid, fx_mid = _tc_strides(x_mid), _tc_strides(fx_mid)
    d_out = _tc_strides(d_out.to(x_mid.dtype))
    dx, dfx = torch.empty_like(x_mid), torch.empty_like(fx_mid)
    dW, db, dt = _param_bufs(c, weight, bias)
    ws, nws = c.workspace(nat.OP_SLICE_BWD)
    with torch.cuda.device(c.device):
        nat.check(nat.load().fs_coupled_bwd(
            c.prob, nat.t4(x_mid), nat.t4(fx_mid), nat.t4(d_out), nat.ptr(c.w), nat.ptr(c.b),
            nat.ptr(c.tau), nat.ptr(_f32(tokens)), nat.ptr(_f32(dz_num)), nat.ptr(_f32(ds)),
            nat.t4(dx), nat.t4(dfx), nat.ptr(dW), nat.ptr(db), nat.ptr(dt), nat.ptr(ws), nws,
            nat.stream_of(x_mid)))
    return (dx, dfx) + _param_grads(c, weight, bias, tau, dW, db, dt)


class _RaggedOps:
    """The three ops of a coupling round over ragged samples (the interface
    ``_CouplingRound`` calls)."""

    def __init__(self, splits):
        self.splits = splits

    def flash_slice(self, x_mid, fx_mid, weight, bias, tau, dot):
        return native_slice(x_mid, fx_mid, weight, bias, tau, self.splits, dot)

    def flash_deslice(self, x_mid, weight, bias, tau, tokens, dot):
        return native_deslice(x_mid, weight, bias, tau, tokens, self.splits, dot)

    def coupled_bwd(self, x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds, dot):
        return native_coupled_bwd(x_mid, fx_mid, d_out, weight, bias, tau, tokens, dz_num, ds,
                                  self.splits, dot)


class _RaggedSlice(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_mid, fx_mid, weight, bias, tau, splits):
        z, s = native_slice(x_mid, fx_mid, weight, bias, tau, splits)
        ctx.save_for_backward(x_mid, fx_mid, weight, bias, tau)
        ctx.splits = splits
        return z, s

    @staticmethod
    def backward(ctx, dz, ds):
        x_mid, fx_mid, weight, bias, tau = ctx.saved_tensors
        g = native_slice_bwd(x_mid, fx_mid, weight, bias, tau, dz, ds, ctx.splits)
        return g + (None,)


class _RaggedDeslice(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_mid, weight, bias, tau, tokens, splits):
        out = native_deslice(x_mid, weight, bias, tau, tokens, splits)
        ctx.save_for_backward(x_mid, weight, bias, tau, tokens)
        ctx.splits = splits
        return out

    @staticmethod
    def backward(ctx, d_out):
        x_mid, weight, bias, tau, tokens = ctx.saved_tensors
        dx, dtok, dW, db, dt = native_deslice_bwd(x_mid, weight, bias, tau, tokens, d_out,
                                                  ctx.splits)
        return dx, dW, db, dt, dtok, None


def _prep(x_mid, weight, bias, splits):
    S = splits.numel() - 1
    _, N, H, D = x_mid.shape
    return _prep_wb(_Shape(S, N, H, D), weight, bias)


def ragged_slice(x_mid, fx_mid, weight, bias, tau, row_splits):
    """``fused_slice`` of every sample: returns z_num (S, H, G, DV) and s
    (S, H, G)."""
    _check_points(x_mid, fx_mid)
    _check_device(x_mid, fx_mid, weight, bias, tau)
    splits = _splits(row_splits, x_mid.shape[1])
    weight, bias, G = _prep(x_mid, weight, bias, splits)
    if _Native.make(x_mid, fx_mid.shape[3], weight, bias, tau, 0, splits) is not None and \
            fx_mid.dtype == x_mid.dtype:
        return _RaggedSlice.apply(x_mid, fx_mid, weight, bias, tau, splits)
    S = splits.numel() - 1
    parts = [fused_slice(_rows(x_mid, splits, b), _rows(fx_mid, splits, b),
                         _of(weight, b, S, 2), _of(bias, b, S, 1), tau) for b in range(S)]
    return torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])


def ragged_deslice(x_mid, weight, bias, tau, tokens, row_splits):
    """``fused_deslice`` of every sample with its tokens (S, H, G, DV):
    returns out (1, N_total, H, DV)."""
    _check_points(x_mid)
    _check_device(x_mid, weight, bias, tau, tokens)
    splits = _splits(row_splits, x_mid.shape[1])
    weight, bias, G = _prep(x_mid, weight, bias, splits)
    if _Native.make(x_mid, tokens.shape[3], weight, bias, tau, 0, splits) is not None:
        return _RaggedDeslice.apply(x_mid, weight, bias, tau, tokens, splits)
    S = splits.numel() - 1
    outs = [fused_deslice(_rows(x_mid, splits, b), _of(weight, b, S, 2), _of(bias, b, S, 1),
                          tau, tokens[b:b + 1]) for b in range(S)]
    return torch.cat(outs, dim=1)


def ragged_coupling(x_mid, fx_mid, weight, bias, tau, row_splits, mix=None, mix_params=None,
                    eps=1e-5):
    """``fused_coupling`` of every sample (``mix`` maps the (S, H, G, DV)
    tokens, each sample's its own): one launch per op for all samples, with
    the tied backward. Returns out (1, N_total, H, DV)."""
    _check_points(x_mid, fx_mid)
    _check_device(x_mid, fx_mid, weight, bias, tau)
    splits = _splits(row_splits, x_mid.shape[1])
    weight, bias, G = _prep(x_mid, weight, bias, splits)
    if mix_params is None:
        mix_params = [q for q in mix.parameters()] if isinstance(mix, torch.nn.Module) else []
    params = tuple(q for q in mix_params if q.requires_grad)
    if _Native.make(x_mid, fx_mid.shape[3], weight, bias, tau, 0, splits,
                    tied=True) is not None and fx_mid.dtype == x_mid.dtype:
        return _CouplingRound.apply(x_mid, fx_mid, weight, bias, tau, eps, 0, mix, None,
                                    _RaggedOps(splits), *params)
    S = splits.numel() - 1

    outs = [fused_coupling(_rows(x_mid, splits, b), _rows(fx_mid, splits, b),
                           _of(weight, b, S, 2), _of(bias, b, S, 1), tau, mix=mix,
                           mix_params=list(params), eps=eps) for b in range(S)]
    return torch.cat(outs, dim=1)
