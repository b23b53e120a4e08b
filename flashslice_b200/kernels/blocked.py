"""The G-blocked contract of ``flashslice.kernels.blocked`` over the native
library: any slot count G and any head width up to 256, with the per-point
softmax statistics (m, l) formed once and handed between the ops.

Same custom-op schemas as the reference (``blocked.py:1472-1568``):
``slice_blk`` returns (z_num, s, stats), ``deslice_blk`` (out, stats), and
their backward ops take the statistics the forward saved. Without
statistics in hand the deslice forms its output and the statistics in one
online pass (stats mode "online", the default) or after a max-then-sum pass
("two-pass"), as ``set_stats_mode`` selects (``blocked.py:101-120``).

The native engine recomputes the weights 32 slots at a time: slot-owning
kernels form the sums over points (z_num, s, dW, db, dtokens), point-owning
kernels the per-point outputs and the temperature gradient row by row over
all of G, with delta = sum_g w dw handed from the latter to the former
(``blocked.py:577-888``).
"""

import torch

from . import _native as nat
from . import _state
from .slice_ops import (_fresh, native_deslice, native_deslice_bwd, native_slice,  # noqa: F401
                        native_slice_bwd, native_stats, set_tile_table, tile_table)


def set_block_g(gb):
    """Force the reference's Triton G-block size (a power of two >= 16), or
    None for automatic. Validated and recorded for compatibility; the native
    engine always recomputes the weights in blocks of 32 slots."""
    if gb is not None and (gb < 16 or (gb & (gb - 1)) != 0):
        raise ValueError("block size must be a power of two >= 16, got %r" % gb)
    _state.block_g = gb


def set_stats_mode(mode):
    """``"online"`` (default) or ``"two-pass"``: how the statistics are formed
    when none are handed in. Overrides FLASHSLICE_STATS_MODE."""
    if mode not in _state.STATS_MODES:
        raise ValueError("stats mode must be one of %s, got %r" % (_state.STATS_MODES, mode))
    _state.stats_mode = mode


def stats_mode():
    return _state.stats_mode


def compute_stats(x_mid, weight, bias, tau, dot=0):
    """(B, H, 2, N) fp32 softmax statistics of the slice logits per point:
    [..., 0, :] the row max, [..., 1, :] the sum of exponentials
    (``blocked.py:1329-1343``)."""
    return native_stats(x_mid, weight, bias, tau, dot)


torch.library.define(
    "flashslice::slice_blk",
    "(Tensor x_mid, Tensor fx_mid, Tensor weight, Tensor bias, Tensor tau, "
    "Tensor? stats, int dot) -> (Tensor, Tensor, Tensor)")
torch.library.define(
    "flashslice::slice_blk_bwd",
    "(Tensor x_mid, Tensor fx_mid, Tensor weight, Tensor bias, Tensor tau, "
    "Tensor stats, Tensor dz_num, Tensor ds, int dot) "
    "-> (Tensor, Tensor, Tensor, Tensor, Tensor)")
torch.library.define(
    "flashslice::deslice_blk",
    "(Tensor x_mid, Tensor weight, Tensor bias, Tensor tau, Tensor tokens, "
    "Tensor? stats, int dot) -> (Tensor, Tensor)")
torch.library.define(
    "flashslice::deslice_blk_bwd",
    "(Tensor x_mid, Tensor weight, Tensor bias, Tensor tau, Tensor tokens, "
    "Tensor stats, Tensor d_out, int dot) "
    "-> (Tensor, Tensor, Tensor, Tensor, Tensor)")


def _slice_blk_impl(x_mid, fx_mid, weight, bias, tau, stats, dot):
    z, s, st = native_slice(x_mid, fx_mid, weight, bias, tau, stats, dot, nat.FAMILY_BLOCKED,
                            True)
    # a custom op must not return one of its inputs: hand back a copy of
    # statistics that were passed in
    return z, s, (st.clone() if stats is not None and st is stats else st)


def _slice_blk_bwd_impl(x_mid, fx_mid, weight, bias, tau, stats, dz_num, ds, dot):
    return native_slice_bwd(x_mid, fx_mid, weight, bias, tau, stats, dz_num, ds, dot,
                            nat.FAMILY_BLOCKED)


def _deslice_blk_impl(x_mid, weight, bias, tau, tokens, stats, dot):
    out, st = native_deslice(x_mid, weight, bias, tau, tokens, stats, dot, nat.FAMILY_BLOCKED,
                             True)
    return out, (st.clone() if stats is not None and st is stats else st)


def _deslice_blk_bwd_impl(x_mid, weight, bias, tau, tokens, stats, d_out, dot):
    return native_deslice_bwd(x_mid, weight, bias, tau, tokens, stats, d_out, dot,
                              nat.FAMILY_BLOCKED)


torch.library.impl("flashslice::slice_blk", "CUDA", _slice_blk_impl)
torch.library.impl("flashslice::slice_blk_bwd", "CUDA", _slice_blk_bwd_impl)
torch.library.impl("flashslice::deslice_blk", "CUDA", _deslice_blk_impl)
torch.library.impl("flashslice::deslice_blk_bwd", "CUDA", _deslice_blk_bwd_impl)


@torch.library.register_fake("flashslice::slice_blk")
def _(x_mid, fx_mid, weight, bias, tau, stats, dot):
    B, N, H, D = x_mid.shape
    G = weight.shape[-2]
    return (x_mid.new_empty((B, H, G, fx_mid.shape[3]), dtype=torch.float32),
            x_mid.new_empty((B, H, G), dtype=torch.float32),
            x_mid.new_empty((B, H, 2, N), dtype=torch.float32))


@torch.library.register_fake("flashslice::slice_blk_bwd")
def _(x_mid, fx_mid, weight, bias, tau, stats, dz_num, ds, dot):
    return (torch.empty_like(x_mid), torch.empty_like(fx_mid), _fresh(weight), _fresh(bias),
            _fresh(tau))


@torch.library.register_fake("flashslice::deslice_blk")
def _(x_mid, weight, bias, tau, tokens, stats, dot):
    B, N, H, D = x_mid.shape
    return (x_mid.new_empty((B, N, H, tokens.shape[3])),
            x_mid.new_empty((B, H, 2, N), dtype=torch.float32))


@torch.library.register_fake("flashslice::deslice_blk_bwd")
def _(x_mid, weight, bias, tau, tokens, stats, d_out, dot):
    return (torch.empty_like(x_mid), _fresh(tokens), _fresh(weight), _fresh(bias),
            _fresh(tau))


def _slice_setup(ctx, inputs, output):
    x_mid, fx_mid, weight, bias, tau, stats, dot = inputs
    ctx.save_for_backward(x_mid, fx_mid, weight, bias, tau, output[2])
    ctx.dot = dot


def _slice_grad(ctx, dz_num, ds, dstats):
    # The statistics are saved intermediates, not a differentiable output;
    # a gradient on them is ignored (blocked.py:1539-1543).
    x_mid, fx_mid, weight, bias, tau, stats = ctx.saved_tensors
    if ds is None:
        ds = torch.zeros(dz_num.shape[:-1], device=dz_num.device, dtype=torch.float32)
    dxm, dfx, dw, db, dtau = torch.ops.flashslice.slice_blk_bwd(
        x_mid, fx_mid, weight, bias, tau, stats, dz_num, ds, ctx.dot)
    return dxm, dfx, dw, db, dtau, None, None


def _deslice_setup(ctx, inputs, output):
    x_mid, weight, bias, tau, tokens, stats, dot = inputs
    ctx.save_for_backward(x_mid, weight, bias, tau, tokens, output[1])
    ctx.dot = dot


def _deslice_grad(ctx, d_out, dstats):
    x_mid, weight, bias, tau, tokens, stats = ctx.saved_tensors
    dxm, dtok, dw, db, dtau = torch.ops.flashslice.deslice_blk_bwd(
        x_mid, weight, bias, tau, tokens, stats, d_out, ctx.dot)
    return dxm, dw, db, dtau, dtok, None, None


torch.library.register_autograd("flashslice::slice_blk", _slice_grad,
                                setup_context=_slice_setup)
torch.library.register_autograd("flashslice::deslice_blk", _deslice_grad,
                                setup_context=_deslice_setup)

__all__ = ["set_block_g", "compute_stats", "set_stats_mode", "stats_mode"]
