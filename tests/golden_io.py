"""Loading the golden fixtures written by ``tests/golden/make_golden.py``."""

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def index():
    with open(os.path.join(GOLDEN, "index.json")) as f:
        return json.load(f)


def load(fn):
    with np.load(os.path.join(GOLDEN, fn)) as z:
        return {k: z[k] for k in z.files}


def op_inputs(arrs):
    """The op-case inputs; the bias is None when the case has none."""
    get = lambda k: arrs.get("in:" + k)  # noqa: E731
    return {k: get(k) for k in ("x", "fx", "W", "b", "tau", "tok", "dz", "ds", "dout")}


def relerr(a, ref):
    """Norm-wise relative error, as the reference's gates compute it
    (``bench/parity_ops.py:51-55``)."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    n = np.linalg.norm(ref)
    d = np.linalg.norm(a - ref)
    return float(d / n) if n > 0 else float(d)
