# Portions of this file restate code from flashslice (https://github.com/Shizheng-Wen/flashslice),
# Copyright 2026 Shizheng Wen, licensed under the Apache License 2.0, which in
# turn derives from Transolver (https://github.com/thuml/Transolver),
# Copyright (c) 2024 THUML @ Tsinghua University, used under the MIT License.

"""The pointwise MLP of every Transolver block (parameter names as the
reference's ``flashslice/layers/basic.py:28-53``: linear_pre, linears,
linear_post)."""

import torch.nn as nn

ACTIVATION = {"gelu": nn.GELU, "tanh": nn.Tanh, "sigmoid": nn.Sigmoid, "relu": nn.ReLU,
              "leaky_relu": lambda: nn.LeakyReLU(0.1), "softplus": nn.Softplus, "ELU": nn.ELU,
              "silu": nn.SiLU}


class MLP(nn.Module):
    """n_input -> n_hidden (act) -> [n_layers x (n_hidden -> n_hidden, act),
    residual when ``res``] -> n_output."""

    def __init__(self, n_input, n_hidden, n_output, n_layers=1, act="gelu", res=True):
        super().__init__()
        if act not in ACTIVATION:
            raise NotImplementedError(act)
        act = ACTIVATION[act]
        self.n_input, self.n_hidden, self.n_output = n_input, n_hidden, n_output
        self.n_layers, self.res = n_layers, res
        self.linear_pre = nn.Sequential(nn.Linear(n_input, n_hidden), act())
        self.linear_post = nn.Linear(n_hidden, n_output)
        self.linears = nn.ModuleList([nn.Sequential(nn.Linear(n_hidden, n_hidden), act())
                                      for _ in range(n_layers)])

    def forward(self, x):
        x = self.linear_pre(x)
        for layer in self.linears:
            x = layer(x) + x if self.res else layer(x)
        return self.linear_post(x)
