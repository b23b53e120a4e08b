"""Generate the golden fixtures in this directory from the reference itself.

Run in a container where the reference (Shizheng-Wen/flashslice v0.3.0) is
checked out, e.g. ``python tests/golden/make_golden.py /path/to/flashslice``.
It imports the reference package and

* runs its eager op math (``bench/parity_ops.py:59-79``: ``_membership`` and
  ``eager``) in float64 with torch autograd, per op: the slice forward and the
  backward of ``sum(z * dz) + sum(s * ds)``, the deslice forward and the
  backward of ``sum(out * dout)``; the inputs are seeded numpy draws shaped
  as ``parity_ops.Case`` builds them (``parity_ops.py:94-156``);
* runs its Triton kernels on the CPU under ``TRITON_INTERPRET=1`` in float32
  for the per-point statistics (``blocked.compute_stats``, online and
  two-pass) and the online deslice, which pins the (B, H, 2, N) layout and
  the (m, l) semantics;
* runs its eager ``Physics_Attention_Irregular_Mesh`` and ``Transolver`` in
  float64 on a seeded state dict, for the layer and model restatements.

The fixtures are small ``.npz`` files; the tests never import the reference.
"""

import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root):
    os.environ.setdefault("TRITON_INTERPRET", "1")
    sys.path.insert(0, root)
    import torch  # noqa: F401
    spec = importlib.util.spec_from_file_location(
        "ref_parity_ops", os.path.join(root, "bench", "parity_ops.py"))
    po = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(po)
    from flashslice.kernels import blocked, slice_ops
    slice_ops.set_tile_table("hopper")  # the table lookup queries CUDA otherwise
    import flashslice
    return po, blocked, slice_ops, flashslice


# name, B, N, H, D, DV, G, weight mode, bias
OP_CASES = [
    ("gd-g32-d32", 1, 24, 2, 32, 32, 32, "gd", True),
    ("hgd-g64-d32", 1, 20, 2, 32, 32, 64, "hgd", True),
    ("bhgd-g48-d40-dv24", 2, 11, 2, 40, 24, 48, "bhgd", True),
    ("bhgd-g160-d24-dv16-tinyN17-nobias", 1, 17, 2, 24, 16, 160, "bhgd", False),
    ("hgd-g40-masked", 1, 19, 2, 32, 32, 40, "hgd", True),
    ("gd-g1", 1, 21, 2, 32, 32, 1, "gd", True),
    ("bhgd-g520-d8-dv8-nobias", 1, 9, 1, 8, 8, 520, "bhgd", False),
    ("gd-n1-g16-d16", 1, 1, 2, 16, 16, 16, "gd", True),
]


def _case_inputs(rng, B, N, H, D, DV, G, mode, bias, Ht=12):
    r = lambda *s: rng.standard_normal(s)  # noqa: E731
    inp = {"x": r(B, N, H, D), "fx": r(B, N, H, DV),
           "tau": np.full(H, 0.7) + 0.1 * r(H), "tok": r(B, H, G, DV),
           "dz": r(B, H, G, DV), "ds": r(B, H, G), "dout": r(B, N, H, DV)}
    if mode == "gd":
        inp["W"] = r(G, D) / D ** 0.5
        inp["b"] = 0.1 * r(G) if bias else None
    elif mode == "hgd":
        inp["W"] = r(H, G, D) / D ** 0.5
        inp["b"] = 0.1 * r(H, G) if bias else None
    else:
        # weight = (t @ Wk) viewed (B, G, H, D) and permuted, as parity_ops.Case
        t = r(B, G, Ht)
        Wk = r(Ht, H * D) / (Ht * D) ** 0.25
        inp["W"] = np.ascontiguousarray(
            (t @ Wk).reshape(B, G, H, D).transpose(0, 2, 1, 3))
        inp["b"] = (np.ascontiguousarray((t @ (0.1 * r(Ht, H))).transpose(0, 2, 1))
                    if bias else None)
    return inp


def _ref_ops(po, torch, inp):
    """Per-op reference results in float64 via the reference's eager math."""
    T = lambda a: None if a is None else torch.tensor(a, dtype=torch.float64)  # noqa: E731
    res = {}

    def leaves():
        L = {k: T(inp[k]) for k in ("x", "fx", "W", "b", "tau", "tok")}
        for v in L.values():
            if v is not None:
                v.requires_grad_(True)
        return L

    # slice forward + backward of sum(z*dz) + sum(s*ds)
    L = leaves()
    sw = po._membership(L["x"], L["W"], L["b"], L["tau"])
    z = torch.einsum("bhng,bnhd->bhgd", sw, L["fx"])
    s = sw.sum(2)
    ((z * T(inp["dz"])).sum() + (s * T(inp["ds"])).sum()).backward()
    res["slice:z_num"], res["slice:s"] = z.detach().numpy(), s.detach().numpy()
    for k in ("x", "fx", "W", "b", "tau"):
        if L[k] is not None:
            res["slice:grad:" + k] = L[k].grad.numpy()
    # deslice forward + backward of sum(out*dout), through parity_ops.eager
    L = leaves()
    out, _, _ = po.eager(L["x"], L["fx"], L["W"], L["b"], L["tau"], None,
                         L["tok"], "deslice-first")
    (out * T(inp["dout"])).sum().backward()
    res["deslice:out"] = out.detach().numpy()
    for k in ("x", "W", "b", "tau", "tok"):
        if L[k] is not None:
            res["deslice:grad:" + k] = L[k].grad.numpy()
    return res


def _ref_kernels(blocked, slice_ops, torch, inp):
    """float32 outputs of the reference's Triton kernels, interpreted on CPU."""
    f = lambda a: torch.tensor(a, dtype=torch.float32)  # noqa: E731
    x, W, tau, tok = f(inp["x"]), f(inp["W"]), f(inp["tau"]), f(inp["tok"])
    G = W.shape[-2]
    b = f(inp["b"]) if inp["b"] is not None else torch.zeros(G)
    W, b = W.contiguous(), b.contiguous()
    res = {}
    blocked.set_stats_mode("online")
    res["kern:stats_online"] = blocked.compute_stats(x, W, b, tau).numpy()
    blocked.set_stats_mode("two-pass")
    res["kern:stats_twopass"] = blocked.compute_stats(x, W, b, tau).numpy()
    blocked.set_stats_mode("online")
    out, st = blocked._deslice_blk_impl(x, W, b, tau, tok, None, 0)
    res["kern:deslice_online_out"] = out.numpy()
    res["kern:deslice_online_stats"] = st.numpy()
    return res


def make_ops(po, blocked, slice_ops, torch):
    rng = np.random.RandomState(20261201)
    index = []
    for name, B, N, H, D, DV, G, mode, bias in OP_CASES:
        inp = _case_inputs(rng, B, N, H, D, DV, G, mode, bias)
        res = _ref_ops(po, torch, inp)
        if G * D <= 65536:
            res.update(_ref_kernels(blocked, slice_ops, torch, inp))
        arrays = {"in:" + k: v for k, v in inp.items() if v is not None}
        arrays.update(res)
        fn = "op_%s.npz" % name
        np.savez_compressed(os.path.join(HERE, fn), **arrays)
        index.append({"file": fn, "name": name, "B": B, "N": N, "H": H, "D": D,
                      "DV": DV, "G": G, "mode": mode, "bias": bias})
        print("wrote", fn)
    return index


def make_layer(torch, flashslice):
    """The eager physics-attention layer and a tiny Transolver, float64."""
    from flashslice.layers.physics_attention import Physics_Attention_Irregular_Mesh
    out = []
    torch.manual_seed(11)
    for name, kw in (("layer-tied", {}), ("layer-untied", {"untied_deslice": True}),
                     ("layer-notokattn", {"no_token_attention": True})):
        layer = Physics_Attention_Irregular_Mesh(16, heads=2, dim_head=8,
                                                 slice_num=8, **kw).double()
        x = torch.randn(1, 23, 16, dtype=torch.float64, requires_grad=True)
        up = torch.randn(1, 23, 16, dtype=torch.float64)
        y, _ = layer(x)
        (y * up).sum().backward()
        arrays = {"in:x": x.detach().numpy(), "in:up": up.numpy(),
                  "out": y.detach().numpy(), "grad:x": x.grad.numpy()}
        for k, v in layer.state_dict().items():
            arrays["sd:" + k] = v.numpy()
        for k, p in layer.named_parameters():
            if p.grad is not None:
                arrays["pgrad:" + k] = p.grad.numpy()
        fn = "%s.npz" % name
        np.savez_compressed(os.path.join(HERE, fn), **arrays)
        out.append({"file": fn, "name": name, "kwargs": kw})
        print("wrote", fn)
    torch.manual_seed(12)
    model = flashslice.Transolver(space_dim=3, fun_dim=1, out_dim=4, n_hidden=16,
                                  n_heads=2, n_layers=2, slice_num=8).double()
    xc = torch.rand(1, 20, 3, dtype=torch.float64)
    fv = torch.randn(1, 20, 1, dtype=torch.float64)
    y = model(xc, fv)
    loss = (y ** 2).mean()
    loss.backward()
    arrays = {"in:x": xc.numpy(), "in:fx": fv.numpy(), "out": y.detach().numpy(),
              "loss": np.array(loss.item())}
    for k, v in model.state_dict().items():
        arrays["sd:" + k] = v.numpy()
    for k, p in model.named_parameters():
        if p.grad is not None:
            arrays["pgrad:" + k] = p.grad.numpy()
    np.savez_compressed(os.path.join(HERE, "transolver-tiny.npz"), **arrays)
    out.append({"file": "transolver-tiny.npz", "name": "transolver-tiny",
                "kwargs": dict(space_dim=3, fun_dim=1, out_dim=4, n_hidden=16,
                               n_heads=2, n_layers=2, slice_num=8)})
    print("wrote transolver-tiny.npz")
    return out


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASHSLICE_REF", "")
    if not root or not os.path.isdir(root):
        raise SystemExit("usage: make_golden.py <path to the reference checkout>")
    po, blocked, slice_ops, flashslice = _import_reference(root)
    import torch
    torch.set_num_threads(4)
    meta = {"reference": "Shizheng-Wen/flashslice " + flashslice.__version__,
            "ops": make_ops(po, blocked, slice_ops, torch),
            "layers": make_layer(torch, flashslice)}
    with open(os.path.join(HERE, "index.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote index.json")


if __name__ == "__main__":
    main()
