"""Axis/coordinate declarations of the committed golden cases.

Each entry restates the reference layer built by ``tests/golden/make_golden.py``.
"""

import os

import numpy as np

from oracle import cst_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CASES = {
    "config1": (O.Axis(8), O.Axis(16), O.Rational(radius_max=4.0)),
    "config2": (O.Axis(1024), O.Axis(1024), O.Rational(radius_max=512.0)),
    "config3": (O.Axis(1024), O.Axis(784, base_tile_sites=49), O.Polar()),
    "config4s": (O.Axis(1024), O.Axis(256), O.Rational(radius_max=128.0)),
    "config5s": (O.Axis(512), O.Axis(512), O.Rational(radius_max=256.0)),
    "hierarchy": (O.Axis(81, spacing=0.5, origin=-3.25, merge_factor=3),
                  O.Axis(54, origin=7.0, base_tile_sites=2, merge_factor=3),
                  O.Rational(radius_max=13.0)),
}


def load(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def field_lrs(d):
    if "field_amplitude" not in d:
        return {}
    return {"amplitude": float(d["field_amplitude"]),
            "radius_fraction": float(d["field_radius_fraction"])}
