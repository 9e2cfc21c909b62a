"""Parity report: errors of the sm_100a path against the reference's float32
results (the golden vectors) and against float64 truth (the oracle), side by
side, with the reference's own float32 error against float64 for scale.

    python tests/parity_report.py            # needs a B200; prints a Markdown table

Each figure is max |a - b| / max |b| over the tensor (the parity tests'
measure; their bar is 1e-4). Gradient figures take the worst of the four atom
gradient columns, on the golden vectors' rows.
"""

import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle import cst_oracle as O  # noqa: E402
from tests.golden_cases import CASES, load  # noqa: E402
from tests.test_gpu_parity import make_layer, rel  # noqa: E402

NAMES = ["config1", "config2", "hierarchy", "config3", "config4s", "config5s"]


def report(name):
    d = load(name)
    layer = make_layer(name, d["p0"])
    x = torch.as_tensor(d["x"]).cuda().requires_grad_("dx" in d)
    y = layer(x)
    y.backward(torch.as_tensor(d["dy"]).cuda())
    torch.cuda.synchronize()
    out_axis, in_axis, spec = CASES[name]
    lay = O.decode(out_axis, in_axis, spec, d["p0"])
    W = O.weight64(lay)
    x64, dy64 = d["x"].astype(np.float64), d["dy"].astype(np.float64)
    rows = d.get("rows", slice(None))
    g64 = O.atom_gradients64(lay, dy64.T @ x64)[rows]
    grad = layer.atoms.p.grad.cpu().numpy()[rows]
    out = {"Y": (y.detach().cpu().numpy(), d["y"], x64 @ W.T)}
    if "dx" in d:
        out["dX"] = (x.grad.cpu().numpy(), d["dx"], dy64 @ W)
    out["grad"] = (grad, d["grad"], g64)
    lines = []
    for what, (new, ref32, truth) in out.items():
        if what == "grad":
            e32 = max(rel(new[:, c], ref32[:, c]) for c in range(4))
            e64 = max(rel(new[:, c], truth[:, c]) for c in range(4))
            r64 = max(rel(ref32[:, c], truth[:, c]) for c in range(4))
        else:
            e32, e64, r64 = rel(new, ref32), rel(new, truth), rel(ref32, truth)
        lines.append(f"| {name} | {what} | {e32:.2e} | {e64:.2e} | {r64:.2e} |")
    return lines


def main():
    print("| case | tensor | new vs reference fp32 | new vs fp64 | reference fp32 vs fp64 |")
    print("|---|---|---|---|---|")
    for name in NAMES:
        for line in report(name):
            print(line)


if __name__ == "__main__":
    main()
