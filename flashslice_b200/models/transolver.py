# Portions of this file restate code from flashslice (https://github.com/Shizheng-Wen/flashslice),
# Copyright 2026 Shizheng Wen, licensed under the Apache License 2.0, which in
# turn derives from Transolver (https://github.com/thuml/Transolver),
# Copyright (c) 2024 THUML @ Tsinghua University, used under the MIT License.

"""Transolver on unstructured point clouds over the B200 slice/deslice ops.

Module structure, parameter names, initialisation and the five ablation
flags follow the reference's ``flashslice/models/transolver.py:41-215``, so
that checkpoints interchange and ``use_fused_slice=True`` is an
implementation switch only. At most one ablation flag may be set; the two
that consume materialised slice weights (``share_slice_across_layers``,
``slice_once``) are refused with ``use_fused_slice``, and a model whose
layers fell back to the eager form reports ``use_fused_slice=False``.
"""

from typing import Optional

import torch
import torch.nn as nn
from torch.nn.init import trunc_normal_

from ..layers.basic import MLP
from ..layers.physics_attention import Physics_Attention_Irregular_Mesh


class TransolverBlock(nn.Module):
    """Physics-attention residual, then a pointwise MLP residual (pre-LN)."""

    def __init__(self, num_heads, hidden_dim, dropout, act="gelu", mlp_ratio=4, last_layer=False,
                 out_dim=1, slice_num=32, untied_deslice=False, no_token_attention=False,
                 mlp_only=False, dim_head=None, slice_dim_head=None, use_fused_slice=False):
        super().__init__()
        self.last_layer = last_layer
        self.mlp_only = mlp_only
        self.ln_1 = nn.LayerNorm(hidden_dim)
        if not mlp_only:
            self.Attn = Physics_Attention_Irregular_Mesh(
                hidden_dim, heads=num_heads,
                dim_head=dim_head if dim_head is not None else hidden_dim // num_heads,
                dropout=dropout, slice_num=slice_num, untied_deslice=untied_deslice,
                no_token_attention=no_token_attention, slice_dim_head=slice_dim_head,
                use_fused_slice=use_fused_slice)
        self.ln_2 = nn.LayerNorm(hidden_dim)
        self.mlp = MLP(hidden_dim, hidden_dim * mlp_ratio, hidden_dim, n_layers=0, res=False,
                       act=act)
        if last_layer:
            self.ln_3 = nn.LayerNorm(hidden_dim)
            self.mlp2 = nn.Linear(hidden_dim, out_dim)

    def forward(self, fx, slice_weights_in=None):
        w = None
        if not self.mlp_only:
            a, w = self.Attn(self.ln_1(fx), slice_weights_in=slice_weights_in)
            fx = fx + a
        fx = fx + self.mlp(self.ln_2(fx))
        if self.last_layer:
            return self.mlp2(self.ln_3(fx)), w
        return fx, w


class TokenTransformerBlock(nn.Module):
    """Pre-LN transformer block over slot tokens (``slice_once`` only)."""

    def __init__(self, num_heads, hidden_dim, dropout, act="gelu", mlp_ratio=4):
        super().__init__()
        self.ln_1 = nn.LayerNorm(hidden_dim)
        self.attn = nn.MultiheadAttention(hidden_dim, num_heads, dropout=dropout,
                                          batch_first=True)
        self.ln_2 = nn.LayerNorm(hidden_dim)
        self.mlp = MLP(hidden_dim, hidden_dim * mlp_ratio, hidden_dim, n_layers=0, res=False,
                       act=act)

    def forward(self, tokens):
        h = self.ln_1(tokens)
        tokens = tokens + self.attn(h, h, h, need_weights=False)[0]
        return tokens + self.mlp(self.ln_2(tokens))


class Transolver(nn.Module):
    """``model(x, fx)``: coordinates (B, N, space_dim) and features
    (B, N, fun_dim) or None -> (B, N, out_dim)."""

    def __init__(self, space_dim=3, fun_dim=1, out_dim=1, n_hidden=256, n_heads=8, n_layers=8,
                 slice_num=32, mlp_ratio=2, dropout=0.0, act="gelu",
                 dim_head: Optional[int] = None, slice_dim_head: Optional[int] = None,
                 untie_slice_weights=False, share_slice_across_layers=False, slice_once=False,
                 no_token_attention=False, mlp_only=False, use_fused_slice=False):
        super().__init__()
        self.n_hidden = n_hidden
        self.preprocess = MLP(fun_dim + space_dim, n_hidden * 2, n_hidden, n_layers=0, res=False,
                              act=act)
        self.untied_deslice = untie_slice_weights
        self.share_slice_across_layers = share_slice_across_layers
        self.slice_once = slice_once
        self.no_token_attention = no_token_attention
        self.mlp_only = mlp_only
        if sum([untie_slice_weights, share_slice_across_layers, slice_once, no_token_attention,
                mlp_only]) > 1:
            raise ValueError("At most one ablation flag may be enabled at a time.")
        self.use_fused_slice = use_fused_slice
        if use_fused_slice and (share_slice_across_layers or slice_once):
            raise ValueError("use_fused_slice is incompatible with share_slice_across_layers "
                             "and slice_once: both need the slice weights the kernel never "
                             "materializes.")
        if slice_once:
            self.slice_proj = nn.Linear(n_hidden, slice_num)
            self.slice_temperature = nn.Parameter(torch.tensor(0.5))
            self.token_blocks = nn.ModuleList([
                TokenTransformerBlock(n_heads, n_hidden, dropout, act=act, mlp_ratio=mlp_ratio)
                for _ in range(n_layers)])
            self.out_norm = nn.LayerNorm(n_hidden)
            self.out_head = nn.Linear(n_hidden, out_dim)
        else:
            self.blocks = nn.ModuleList([
                TransolverBlock(n_heads, n_hidden, dropout, act=act, mlp_ratio=mlp_ratio,
                                out_dim=out_dim, slice_num=slice_num,
                                last_layer=(i == n_layers - 1),
                                untied_deslice=untie_slice_weights,
                                no_token_attention=no_token_attention, mlp_only=mlp_only,
                                dim_head=dim_head, slice_dim_head=slice_dim_head,
                                use_fused_slice=use_fused_slice)
                for i in range(n_layers)])
            if use_fused_slice and any(
                    getattr(getattr(b, "Attn", None), "fused_slice_fallback", None)
                    for b in self.blocks):
                # a layer refused its dims and runs eager: report the effective state
                self.use_fused_slice = False
        self.placeholder = nn.Parameter((1 / n_hidden) * torch.rand(n_hidden, dtype=torch.float))
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(m):
        if isinstance(m, nn.Linear):
            trunc_normal_(m.weight, std=0.02)
            if m.bias is not None:
                nn.init.constant_(m.bias, 0)
        elif isinstance(m, (nn.LayerNorm, nn.BatchNorm1d)):
            nn.init.constant_(m.bias, 0)
            nn.init.constant_(m.weight, 1.0)

    def _slice_once_forward(self, fx):
        w = torch.softmax(self.slice_proj(fx) / self.slice_temperature, dim=-1)
        tokens = torch.einsum("bnc,bng->bgc", fx, w) / (w.sum(1) + 1e-5).unsqueeze(-1)
        for block in self.token_blocks:
            tokens = block(tokens)
        out = torch.einsum("bgc,bng->bnc", tokens, w) + fx
        return self.out_head(self.out_norm(out))

    def forward(self, x, fx=None):
        fx = self.preprocess(torch.cat((x, fx), dim=-1) if fx is not None else x)
        fx = fx + self.placeholder[None, None, :]
        if self.slice_once:
            return self._slice_once_forward(fx)
        shared = None
        for block in self.blocks:
            fx, w = block(fx, slice_weights_in=shared)
            if self.share_slice_across_layers and shared is None:
                shared = w
        return fx


__all__ = ["Transolver", "TransolverBlock", "TokenTransformerBlock"]
