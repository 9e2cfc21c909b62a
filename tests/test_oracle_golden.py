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


def test_amplitude_decay_law():
    """The Polar amplitude decay of the oracle against the reference's own decay
    law (executor.py:18-41) on fixed inputs. The oracle's square roots are IEEE
    (correctly rounded) and torch's CPU ones are not (about 0.7% of float32
    inputs differ by one ulp), and t = new_r sqrt((1 - |u|)(1 + |u|)) amplifies
    a one-ulp change of u by |u| / (1 - u^2) as |u| -> 1. So: centers exact,
    s within two ulps, t within two ulps plus that conditioning times 4 ulps
    of u."""
    d = load("config3_decay")
    out = O.decay_amplitude(d["decay_previous"], d["decay_updated"], float(d["decay_amount"]))
    ref = d["decay_out"]
    np.testing.assert_array_equal(out[:, 2:], ref[:, 2:])
    ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    err = np.abs(out.astype(np.float64) - ref)
    assert (err[:, 0] <= 2 * ulp[:, 0]).all()
    r = np.hypot(ref[:, 0].astype(np.float64), ref[:, 1])
    u = np.clip(np.abs(ref[:, 0]) / r, 0, 1)
    cond = r * u / np.sqrt(np.maximum(1 - u * u, 2.0 ** -24)) * 4 * 2.0 ** -24
    assert (err[:, 1] <= 2 * ulp[:, 1] + cond).all()
    assert (out != ref).mean() < 0.02


def test_optimizer_steps_with_amplitude_decay():
    """Three reference CSTAdamW steps with amplitude_weight_decay on Polar rows.
    The decay itself is bit-exact (above); torch's CPU sqrt (one ulp off on a
    fraction of a percent of elements) reaches s through the Polar law with
    cancellation, so allow eight float32 ulps of the result (1e-9 floor)."""
    out_axis, in_axis, spec = CASES["config3"]
    d = load("config3_decay")
    p = d["p0"].copy()
    state = O.AdamState(0, np.zeros_like(p), np.zeros_like(p))
    lr, decay = float(d["lr"]), float(d["amplitude_weight_decay"])
    undecayed = O.optimizer_step(d["p0"], d["grads"][0], O.AdamState(0, np.zeros_like(p),
                                                                      np.zeros_like(p)),
                                 spec, lr=lr, periods=(out_axis.period, in_axis.period))
    assert np.abs(undecayed - d["p1"]).max() > 1e-7  # the decay matters at this size
    for step in range(3):
        p = O.optimizer_step(p, d["grads"][step], state, spec, lr=lr,
                             periods=(out_axis.period, in_axis.period),
                             amplitude_weight_decay=decay)
        ref = d[f"p{step + 1}"]
        ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
        assert (np.abs(p.astype(np.float64) - ref) <= 8 * ulp + 1e-9).all(), step
        assert (p != ref).mean() < 0.02


def test_amplitude_decay_rejects_rational_rows():
    out_axis, in_axis, spec = CASES["config1"]
    d = load("config1")
    state = O.AdamState(0, np.zeros_like(d["p0"]), np.zeros_like(d["p0"]))
    with pytest.raises(ValueError, match="Polar"):
        O.optimizer_step(d["p0"], d["grad"], state, spec, lr=1e-3, amplitude_weight_decay=0.1)


TRAJECTORIES = {
    "trajectory1": (O.Axis(8), O.Axis(16), O.Rational(radius_max=4.0)),
    "trajectory_mid": (O.Axis(256), O.Axis(256), O.Rational(radius_max=128.0)),
}


@pytest.mark.parametrize("name", sorted(TRAJECTORIES))
def test_reference_trajectory(name):
    """The oracle's reference-precision step, iterated, follows the reference's
    own training trajectory: every step's loss to 1e-6, the atoms to 1e-3
    (Adam normalises each coordinate's step, so a near-zero gradient whose
    last bits differ can move a coordinate by up to one step size)."""
    out_axis, in_axis, spec = TRAJECTORIES[name]
    d = load(name)
    lr, keep = float(d["lr"]), int(d["keep"])
    p = d["p0"].copy()
    state = O.AdamState(0, np.zeros_like(p), np.zeros_like(p))
    for step, want in enumerate(d["losses"]):
        loss, _, _, _, p = O.reference_step(out_axis, in_axis, spec, p, d["x"], d["target"],
                                            state, lr=lr, field_lrs=field_lrs(d) or None)
        assert abs(loss - want) <= 1e-6 * want, step
        if (step + 1) % keep == 0:
            ref = d["p_steps"][(step + 1) // keep - 1]
            assert np.abs(p - ref).max() <= 1e-3, step
            assert np.quantile(np.abs(p - ref), 0.999) <= 1e-5, step
