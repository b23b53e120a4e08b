"""The physics-attention layer (three variants) and a tiny Transolver against
the reference's own eager modules: fixtures written by
``tests/golden/make_golden.py`` from the reference in float64 (state dict,
input, output, input and parameter gradients). The eager path runs on CPU;
it is the form the layers fall back to, and the definition the fused path is
held to on the GPU (``tests/test_gpu_layers.py``)."""

import json
import os

import numpy as np
import pytest
import torch

HERE = os.path.join(os.path.dirname(__file__), "golden")
INDEX = json.load(open(os.path.join(HERE, "index.json")))
LAYERS = [e for e in INDEX["layers"] if e["name"].startswith("layer-")]
MODEL = [e for e in INDEX["layers"] if e["name"] == "transolver-tiny"][0]


def _load(module, arrays):
    sd = {k[3:]: torch.from_numpy(v) for k, v in arrays.items() if k.startswith("sd:")}
    module.load_state_dict(sd, strict=True)
    return module


def _close(a, b, rtol=1e-10):
    a, b = np.asarray(a), np.asarray(b)
    scale = max(np.abs(b).max(), 1e-30)
    return np.abs(a - b).max() <= rtol * scale


@pytest.mark.parametrize("entry", LAYERS, ids=[e["name"] for e in LAYERS])
def test_layer_matches_reference(entry):
    from flashslice_b200 import Physics_Attention_Irregular_Mesh
    arrays = dict(np.load(os.path.join(HERE, entry["file"])))
    layer = Physics_Attention_Irregular_Mesh(16, heads=2, dim_head=8, slice_num=8,
                                             **entry["kwargs"]).double()
    _load(layer, arrays)
    x = torch.from_numpy(arrays["in:x"]).requires_grad_(True)
    y, _ = layer(x)
    (y * torch.from_numpy(arrays["in:up"])).sum().backward()
    assert _close(y.detach().numpy(), arrays["out"])
    assert _close(x.grad.numpy(), arrays["grad:x"])
    for k, p in layer.named_parameters():
        if "pgrad:" + k in arrays:
            assert _close(p.grad.numpy(), arrays["pgrad:" + k]), k


def test_transolver_matches_reference():
    from flashslice_b200 import Transolver
    arrays = dict(np.load(os.path.join(HERE, MODEL["file"])))
    model = Transolver(**MODEL["kwargs"]).double()
    _load(model, arrays)
    y = model(torch.from_numpy(arrays["in:x"]), torch.from_numpy(arrays["in:fx"]))
    loss = (y ** 2).mean()
    loss.backward()
    assert _close(y.detach().numpy(), arrays["out"])
    assert abs(loss.item() - float(arrays["loss"])) <= 1e-10 * abs(float(arrays["loss"]))
    for k, p in model.named_parameters():
        if "pgrad:" + k in arrays:
            assert _close(p.grad.numpy(), arrays["pgrad:" + k], rtol=1e-9), k
