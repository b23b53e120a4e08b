"""Dims contract, routing and the visible eager fallback (CPU).

Mirrors the reference's ``tests/test_dims.py``: the single-tile contract
serves D and G that are powers of two in [16, 128] with DV = D, the G-blocked
contract every other G and D up to 256; D beyond that makes a layer built
with ``use_fused_slice=True`` fall back to eager *visibly*, and the model
report the effective state. (The reference's tile-table and Triton block-size
tests are Triton tuning with no counterpart here.)
"""

import pytest
import torch

from flashslice_b200.kernels.slice_ops import (_use_blocked, set_kernel_mode, single_tile_dims,
                                               unsupported_dims)
from flashslice_b200.layers.physics_attention import Physics_Attention_Irregular_Mesh


@pytest.mark.parametrize("d,g", [(16, 16), (32, 32), (32, 64), (32, 128), (128, 32)])
def test_single_tile_dims(d, g):
    assert unsupported_dims(d, g) is None
    assert single_tile_dims(d, g)
    assert not _use_blocked(d, g)


@pytest.mark.parametrize("d,g", [(32, 8), (32, 256), (32, 48), (8, 32), (256, 32), (24, 40),
                                 (32, 1), (32, 1024)])
def test_blocked_dims(d, g):
    assert unsupported_dims(d, g) is None
    assert not single_tile_dims(d, g)
    assert _use_blocked(d, g)


@pytest.mark.parametrize("d,g", [(512, 32), (0, 32), (32, 0)])
def test_unsupported_dims(d, g):
    why = unsupported_dims(d, g)
    assert why and ("dim_head" in why or "slice_num" in why)


def test_kernel_mode_switch():
    try:
        set_kernel_mode("blocked")
        assert _use_blocked(32, 32)
        set_kernel_mode("single-tile")
        assert not _use_blocked(32, 32)
        with pytest.raises(ValueError, match="single-tile"):
            _use_blocked(32, 256)
        with pytest.raises(ValueError):
            set_kernel_mode("fast")
    finally:
        set_kernel_mode("auto")
    assert not _use_blocked(32, 32) and _use_blocked(32, 256)


@pytest.mark.parametrize("d,g,dv", [(32, 32, 24), (56, 1024, 32), (64, 64, 32)])
def test_value_width_routes_to_blocked(d, g, dv):
    assert unsupported_dims(d, g, dv) is None
    assert not single_tile_dims(d, g, dv)
    assert _use_blocked(d, g, dv)


def test_equal_value_width_keeps_single_tile():
    assert single_tile_dims(32, 32, 32)
    assert not _use_blocked(32, 32, 32)


def test_value_width_bounds():
    assert "value width" in unsupported_dims(32, 32, 512)
    assert "value width" in unsupported_dims(32, 32, 0)


def _layer(g, d=32, heads=8):
    return Physics_Attention_Irregular_Mesh(dim=heads * d, heads=heads, dim_head=d, slice_num=g,
                                            use_fused_slice=True)


@pytest.mark.parametrize("g", [32, 8, 256])
def test_layer_keeps_kernels_on_supported_dims(g):
    layer = _layer(g=g)
    assert layer.use_fused_slice is True
    assert layer.fused_slice_fallback is None


def test_layer_falls_back_visibly(caplog):
    with caplog.at_level("WARNING"):
        layer = _layer(g=32, d=512, heads=2)
    assert layer.use_fused_slice is False
    assert "dim_head=512" in layer.fused_slice_fallback
    assert any("falling back" in r.message for r in caplog.records)


def test_model_reports_effective_state():
    from flashslice_b200 import Transolver

    def build(dim_head):
        return Transolver(space_dim=3, fun_dim=3, out_dim=1, n_hidden=64, n_heads=2, n_layers=2,
                          slice_num=32, mlp_ratio=1, dim_head=dim_head, use_fused_slice=True)

    assert build(32).use_fused_slice is True
    assert build(512).use_fused_slice is False


def test_fused_rejects_incompatible_ablations():
    from flashslice_b200 import Transolver
    for flag in ("share_slice_across_layers", "slice_once"):
        with pytest.raises(ValueError, match="use_fused_slice"):
            Transolver(space_dim=3, fun_dim=3, out_dim=1, n_hidden=64, n_heads=2, n_layers=2,
                       slice_num=32, use_fused_slice=True, **{flag: True})
    with pytest.raises(ValueError, match="At most one"):
        Transolver(space_dim=3, fun_dim=3, out_dim=1, n_hidden=64, n_heads=2, n_layers=2,
                   no_token_attention=True, mlp_only=True)


def test_forward_matches_eager_on_unsupported_dims():
    torch.manual_seed(0)
    fused = _layer(g=8, d=512, heads=2)
    eager = Physics_Attention_Irregular_Mesh(dim=2 * 512, heads=2, dim_head=512, slice_num=8,
                                             use_fused_slice=False)
    eager.load_state_dict(fused.state_dict())
    x = torch.randn(1, 97, 1024)
    with torch.no_grad():
        assert torch.equal(fused(x)[0], eager(x)[0])


def test_modes_validate():
    from flashslice_b200.kernels import (set_block_g, set_dot_mode, set_stats_mode,
                                         set_tile_table, stats_mode, tile_table)
    with pytest.raises(ValueError):
        set_dot_mode("fp64")
    set_dot_mode("tf32x3")
    set_dot_mode("")
    with pytest.raises(ValueError):
        set_block_g(12)
    set_block_g(64)
    set_block_g(None)
    try:
        set_stats_mode("two-pass")
        assert stats_mode() == "two-pass"
        with pytest.raises(ValueError):
            set_stats_mode("streaming")
    finally:
        set_stats_mode("online")
    try:
        set_tile_table("ada")
        assert tile_table() == "ada"
        with pytest.raises(ValueError):
            set_tile_table("ampere")
    finally:
        set_tile_table("auto")


def test_dot_mode_levels():
    from flashslice_b200.kernels import set_dot_mode
    from flashslice_b200.kernels.slice_ops import _dot_mode
    f32, bf = torch.empty(1), torch.empty(1, dtype=torch.bfloat16)
    try:
        for mode, lf, lb in (("ieee", 0, 0), ("tf32", 1, 1), ("bf16v", 1, 2), ("bf16", 1, 3),
                             ("tf32x3", 4, 4)):
            set_dot_mode(mode)
            assert _dot_mode(f32) == lf and _dot_mode(bf) == lb
    finally:
        set_dot_mode("")


def test_prep_wb_errors():
    from flashslice_b200.kernels.slice_ops import _prep_wb
    x = torch.empty(2, 5, 4, 8)
    w, b, G = _prep_wb(x, torch.empty(6, 8), None)
    assert G == 6 and b.shape == (6,) and float(b.abs().sum()) == 0
    for bad_w, bad_b in ((torch.empty(6, 7), None), (torch.empty(3, 6, 8), None),
                         (torch.empty(6, 8), torch.empty(5)), (torch.empty(6), None),
                         (torch.empty(3, 4, 6, 8), None), (torch.empty(6, 8), torch.empty(3, 6))):
        with pytest.raises(ValueError):
            _prep_wb(x, bad_w, bad_b)


def test_no_cpu_kernels():
    """The ops have no CPU implementation: CPU tensors raise, nothing falls
    back to eager math."""
    from flashslice_b200.kernels import fused_slice
    x = torch.randn(1, 4, 2, 16)
    with pytest.raises((RuntimeError, NotImplementedError)):
        fused_slice(x, x, torch.randn(16, 16), None, torch.ones(2))
