"""Fused slice/deslice ops on B200: the ``flashslice.kernels`` surface.

``fused_slice`` and ``fused_deslice`` are ``torch.library`` custom ops in the
``flashslice`` namespace, with autograd and fake (meta) kernels registered,
so that they compose with autograd and stay one torch.compile graph. They
run in hand-written sm_100a kernels reached through the C ABI of
``libflashslice_b200.so``; there is no Triton and no CPU fallback.

Exports mirror the reference (``flashslice/kernels/__init__.py:44-59``);
``fused_coupling`` (a whole slice -> tokens -> deslice round with a tied
backward) and the ragged-batch forms ``ragged_slice``, ``ragged_deslice``,
``ragged_coupling`` (samples of different N in one launch per op) have no
reference counterpart.
"""

from .slice_ops import (fused_slice, fused_deslice, fused_coupling, unsupported_dims,
                        single_tile_dims, set_dot_mode, set_kernel_mode, set_tile_table,
                        tile_table)
from . import blocked  # noqa: F401  -- registers the flashslice::*_blk ops
from .blocked import set_block_g, set_stats_mode, stats_mode
from ._state import set_engine
from .ragged import ragged_slice, ragged_deslice, ragged_coupling

__all__ = ["fused_slice", "fused_deslice", "fused_coupling", "unsupported_dims",
           "single_tile_dims",
           "set_dot_mode", "set_kernel_mode", "set_block_g", "set_stats_mode",
           "stats_mode", "set_tile_table", "tile_table", "set_engine", "ragged_slice",
           "ragged_deslice", "ragged_coupling"]
