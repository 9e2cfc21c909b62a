"""Pin the CPU oracle against vectors produced by the reference itself."""

import numpy as np
import pytest

from oracle import cst_oracle as O
from tests.golden_cases import CASES, field_lrs, load

NAMES = ["config1", "hierarchy", "config4s", "config3", "config2", "config5s"]


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-300))


@pytest.mark.parametrize("name", NAMES)
def test_routing_bit_exact(name):
    out_axis, in_axis, spec = CASES[name]
    d = load(name)
    table = O.routing_table(O.decode(out_axis, in_axis, spec, d["p0"]))
    for side in ("out", "in"):
        for key in ("level", "count", "first_tile"):
            np.testing.assert_array_equal(table[f"{side}_{key}"], d[f"route_{side}_{key}"])


@pytest.mark.parametrize("name", NAMES)
def test_factor_columns(name):
    out_axis, in_axis, spec = CASES[name]
    d = load(name)
    lay = O.decode(out_axis, in_axis, spec, np.asarray(d["p0"], np.float64), dtype=np.float64)
    cols = d["phi_cols"]
    phi_out = lay.out_prof.dense(lay.atoms)[:, cols] * lay.dec["amplitude"][cols]
    phi_in = lay.in_prof.dense(lay.atoms)[:, cols]
    assert rel(phi_out, d["phi_out"]) < 1e-12
    assert rel(phi_in, d["phi_in"]) < 1e-12
    # The support of every sampled column is exactly the routed footprint.
    assert ((phi_in != 0) == (d["phi_in"] != 0)).all()


@pytest.mark.parametrize("name", NAMES)
def test_forward_backward(name):
    out_axis, in_axis, spec = CASES[name]
    d = load(name)
    if name == "config5s":
        pytest.skip("covered by the float64 wide-atom test in test_oracle_wide")
    lay = O.decode(out_axis, in_axis, spec, d["p0"])
    x, dy = d["x"].astype(np.float64), d["dy"].astype(np.float64)
    W = O.weight64(lay)
    # The reference computes in float32; 1e-5 of the output scale bounds its rounding.
    assert rel(x @ W.T, d["y"]) < 1e-5
    if "dx" in d:
        assert rel(dy @ W, d["dx"]) < 1e-5
    grad = O.atom_gradients64(lay, dy.T @ x)
    if "rows" in d:
        grad = grad[d["rows"]]
    for c in range(4):
        assert rel(grad[:, c], d["grad"][:, c]) < 1e-5, c


def test_forward_backward_wide_folded():
    out_axis, in_axis, spec = CASES["config5s"]
    d = load("config5s")
    lay = O.decode(out_axis, in_axis, spec, d["p0"])
    # radius_max 256 on 512 sites: footprints of 3*256 sites fold onto the chart.
    assert (lay.out_prof.routing["count"] * lay.out_prof.routing["tile_sites"] > 512).any()
    x, dy = d["x"].astype(np.float64), d["dy"].astype(np.float64)
    W = O.weight64(lay)
    assert rel(x @ W.T, d["y"]) < 1e-5
    assert rel(dy @ W, d["dx"]) < 1e-5
    grad = O.atom_gradients64(lay, dy.T @ x)
    for c in range(4):
        assert rel(grad[:, c], d["grad"][:, c]) < 1e-5, c


@pytest.mark.parametrize("name", NAMES)
def test_optimizer_step(name):
    out_axis, in_axis, spec = CASES[name]
    d = load(name)
    rows = d.get("rows", slice(None))
    p0, grad = d["p0"][rows], d["grad"]
    lr = float(d["lr"])
    ratios = O.field_ratios(spec, field_lrs(d), lr)
    state = O.AdamState(0, np.zeros_like(grad), np.zeros_like(grad))
    p1 = O.optimizer_step(p0, grad, state, spec, lr=lr, field_ratios=ratios,
                          periods=(out_axis.period, in_axis.period))
    # torch's CPU sqrt is not correctly rounded: allow two float32 ulps (plus,
    # for the Polar pair whose norm is ~1, a 1e-9 absolute floor).
    ulp = np.spacing(np.abs(d["p1"]).astype(np.float32)).astype(np.float64)
    assert (np.abs(p1.astype(np.float64) - d["p1"]) <= 2 * ulp + 1e-9).all()
    assert (p1 != d["p1"]).mean() < 0.01


def test_reference_step_matches_golden_config1():
    out_axis, in_axis, spec = CASES["config1"]
    d = load("config1")
    state = O.AdamState(0, np.zeros((12, 4), np.float32), np.zeros((12, 4), np.float32))
    loss, y, dx, grad, p1 = O.reference_step(out_axis, in_axis, spec, d["p0"], d["x"],
                                             d["target"], state, lr=1e-3)
    assert rel(y, d["y"]) < 1e-5
    assert rel(dx, d["dx"]) < 1e-5
    for c in range(4):
        assert rel(grad[:, c], d["grad"][:, c]) < 1e-5
    np.testing.assert_allclose(p1, d["p1"], rtol=0, atol=1e-6)


def test_invalid_inputs_raise():
    out_axis, in_axis, spec = CASES["config1"]
    p = np.zeros((2, 4), np.float32)
    p[:, 0] = 0.1
    p[0, 1] = 1.5
    with pytest.raises(ValueError):
        O.decode(out_axis, in_axis, spec, p)
    p[0, 1] = np.nan
    with pytest.raises(ValueError):
        O.decode(out_axis, in_axis, spec, p)
    with pytest.raises(ValueError):
        O.Axis(12, base_tile_sites=5).validate()
