# Portions of this file restate code from flashslice (https://github.com/Shizheng-Wen/flashslice),
# Copyright 2026 Shizheng Wen, licensed under the Apache License 2.0, which in
# turn derives from Transolver (https://github.com/thuml/Transolver),
# Copyright (c) 2024 THUML @ Tsinghua University, used under the MIT License.

"""Physics-attention for irregular meshes with the slice/deslice coupling on
the B200 ops.

The module and parameter names follow the reference's
``Physics_Attention_Irregular_Mesh`` (``flashslice/layers/physics_attention.py:
28-181``) so that state dicts interchange; ``use_fused_slice`` switches the
slice/deslice between the fused ops and the eager einsum form, with the same
outputs. Shapes the fused ops cannot serve (``unsupported_dims``) fall back
to the eager form visibly: a warning, ``use_fused_slice`` reads False and
``fused_slice_fallback`` holds the reason (``physics_attention.py:44-61``).
"""

import logging

import torch
import torch.nn as nn

logger = logging.getLogger(__name__)


class Physics_Attention_Irregular_Mesh(nn.Module):
    """Slice the N points into G soft slots per head, attend among the slot
    tokens, deslice back to the points.

    ``untied_deslice``: the deslice has its own projection and temperature.
    ``no_token_attention``: the tokens are mapped by ``to_v`` only.
    ``slice_dim_head``: width of the token attention (default ``dim_head``)."""

    def __init__(self, dim, heads=8, dim_head=64, dropout=0., slice_num=64, shapelist=None,
                 untied_deslice=False, no_token_attention=False, slice_dim_head=None,
                 use_fused_slice=False):
        super().__init__()
        self.use_fused_slice = use_fused_slice
        self.fused_slice_fallback = None
        if use_fused_slice:
            from ..kernels.slice_ops import unsupported_dims
            why = unsupported_dims(dim_head, slice_num)
            if why:
                logger.warning("use_fused_slice=True but %s; falling back to the eager "
                               "slice/deslice path (identical outputs, baseline speed and "
                               "memory).", why)
                self.use_fused_slice = False
                self.fused_slice_fallback = why
        inner = dim_head * heads
        self.dim_head = dim_head
        self.slice_dim_head = dim_head if slice_dim_head is None else slice_dim_head
        self.heads = heads
        self.scale = self.slice_dim_head ** -0.5
        self.softmax = nn.Softmax(dim=-1)
        self.dropout = nn.Dropout(dropout)
        self.temperature = nn.Parameter(torch.full([1, heads, 1, 1], 0.5))
        self.untied_deslice = untied_deslice
        self.no_token_attention = no_token_attention
        self.in_project_x = nn.Linear(dim, inner)
        self.in_project_fx = nn.Linear(dim, inner)
        self.in_project_slice = nn.Linear(dim_head, slice_num)
        nn.init.orthogonal_(self.in_project_slice.weight)
        if untied_deslice:
            self.deslice_temperature = nn.Parameter(torch.full([1, heads, 1, 1], 0.5))
            self.in_project_deslice = nn.Linear(dim_head, slice_num)
            nn.init.orthogonal_(self.in_project_deslice.weight)
        sdh = self.slice_dim_head
        self.to_q = nn.Linear(dim_head, sdh, bias=False)
        self.to_k = nn.Linear(dim_head, sdh, bias=False)
        self.to_v = nn.Linear(dim_head, sdh, bias=False)
        self.slice_down = nn.Identity() if sdh == dim_head else nn.Linear(sdh, dim_head,
                                                                          bias=False)
        self.to_out = nn.Sequential(nn.Linear(inner, dim), nn.Dropout(dropout))

    def _mix(self, tok):
        """Attention among the G slot tokens of each head (tiny)."""
        if self.no_token_attention:
            mixed = self.to_v(tok)
        else:
            q, k, v = self.to_q(tok), self.to_k(tok), self.to_v(tok)
            att = self.dropout(self.softmax(torch.matmul(q, k.transpose(-1, -2)) * self.scale))
            mixed = torch.matmul(att, v)
        return self.slice_down(mixed)

    def _forward_fused(self, x):
        from ..kernels.slice_ops import (_dot_mode, _use_blocked, fused_coupling, fused_deslice,
                                         fused_slice)
        B, N, _ = x.shape
        H, D = self.heads, self.dim_head
        # (B, N, H, D) views of the projections: the ops read them by strides
        fx_mid = self.in_project_fx(x).view(B, N, H, D)
        x_mid = self.in_project_x(x).view(B, N, H, D)
        tau = self.temperature.view(H)
        G = self.in_project_slice.weight.shape[0]
        if not self.untied_deslice and not _use_blocked(D, G, D, _dot_mode(x_mid), x.device):
            # one round with the tied backward; the token attention is its mix
            params = [q for m in (self.to_q, self.to_k, self.to_v, self.slice_down)
                      for q in m.parameters()]
            out = fused_coupling(x_mid, fx_mid, self.in_project_slice.weight,
                                 self.in_project_slice.bias, tau, mix=self._mix,
                                 mix_params=params, eps=1e-5)
            return self.to_out(out.reshape(B, N, H * D)), None
        z_num, s, stats = fused_slice(x_mid, fx_mid, self.in_project_slice.weight,
                                      self.in_project_slice.bias, tau, return_stats=True)
        tokens = self._mix(z_num / (s + 1e-5).unsqueeze(-1))
        if self.untied_deslice:
            out = fused_deslice(x_mid, self.in_project_deslice.weight,
                                self.in_project_deslice.bias, self.deslice_temperature.view(H),
                                tokens)
        else:
            out = fused_deslice(x_mid, self.in_project_slice.weight, self.in_project_slice.bias,
                                tau, tokens, stats=stats)
        return self.to_out(out.reshape(B, N, H * D)), None

    def _memberships(self, x_mid, proj, temperature):
        return self.softmax(proj(x_mid) / temperature)

    def forward(self, x, slice_weights_in=None):
        """x (B, N, C) -> (out (B, N, C), slice weights (B, H, N, G) or None)."""
        if self.use_fused_slice:
            if slice_weights_in is not None:
                raise ValueError("use_fused_slice cannot consume externally provided slice "
                                 "weights.")
            return self._forward_fused(x)
        B, N, _ = x.shape
        H, D = self.heads, self.dim_head
        fx_mid = self.in_project_fx(x).reshape(B, N, H, D).permute(0, 2, 1, 3).contiguous()
        x_mid = None
        if slice_weights_in is None or self.untied_deslice:
            x_mid = self.in_project_x(x).reshape(B, N, H, D).permute(0, 2, 1, 3).contiguous()
        if slice_weights_in is None:
            w = self._memberships(x_mid, self.in_project_slice, self.temperature)
        else:
            w = slice_weights_in
        norm = w.sum(2)
        tok = torch.einsum("bhnc,bhng->bhgc", fx_mid, w)
        tok = tok / (norm + 1e-5)[:, :, :, None]
        tokens = self._mix(tok)
        wd = (self._memberships(x_mid, self.in_project_deslice, self.deslice_temperature)
              if self.untied_deslice else w)
        out = torch.einsum("bhgc,bhng->bhnc", tokens, wd)
        out = out.permute(0, 2, 1, 3).reshape(B, N, H * D)
        return self.to_out(out), w
