"""Declarations mirroring torchcst's public kernel/chart factories for this path.

Same names, arguments and validation messages as the reference
(kernels/factories.py:86-99,125-134,197-239,403-460; kernels/spec.py:133-157;
kernels/radius_cell_mass.py:29-93; charts/presets.py:63-93), restricted to what
the radius cell-mass Linear hot path uses: product(cell_mass(ChebyshevSpec(M)))
on two fixed 1-D flat-torus regular grids with rational or Polar radius
coordinates. Everything here is metadata; nothing imports CUDA code.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


def _f32(value: float) -> float:
    """The value a float32 KernelState buffer holds, widened to double."""
    return float(np.float32(value))


@dataclass(frozen=True)
class ChebyshevSpec:
    modes: int = 8

    def __post_init__(self):
        if type(self.modes) is not int or not 1 <= self.modes <= 512:
            raise ValueError("ChebyshevSpec modes must be an integer in 1..512")


@dataclass(frozen=True)
class RadiusBounds:
    minimum: float
    birth: float
    maximum: float
    upper_floor: float

    def __post_init__(self):
        if not 0 < self.minimum <= self.birth <= self.maximum:
            raise ValueError("radius bounds must satisfy 0 < minimum <= birth <= maximum")
        if not self.minimum <= self.upper_floor <= self.maximum:
            raise ValueError("upper_floor must lie within the radius bounds")


@dataclass(frozen=True)
class CellMass:
    """RadiusIntegratedProfileBinding (kernels/spec.py:133-157)."""

    profile: ChebyshevSpec = field(default_factory=ChebyshevSpec)
    base_tile_sites: int = 1
    merge_factor: int = 2

    def __post_init__(self):
        if type(self.profile) is not ChebyshevSpec:
            raise ValueError(
                "radius cell integration requires a Chebyshev profile and shared physical radius")
        if type(self.base_tile_sites) is not int or self.base_tile_sites < 1:
            raise ValueError("base_tile_sites must be a positive integer")
        if type(self.merge_factor) is not int or self.merge_factor < 2:
            raise ValueError("merge_factor must be an integer at least two")


@dataclass(frozen=True)
class RationalRadius:
    """RationalRadiusSpec + its initialization settings (factories.py:197-239)."""

    radius_min: float = 0.5
    radius_birth: float = 4.0
    radius_max: float = 50.0
    amplitude_max: float = 32.0
    radius_fraction: float = 0.0
    amplitude_std: float = 0.1
    id: str = "rational_radius"
    revision: int = 8

    def __post_init__(self):
        for name in ("radius_min", "radius_birth", "radius_max", "amplitude_max"):
            v = getattr(self, name)
            if type(v) not in (int, float) or not math.isfinite(v) or v <= 0:
                raise ValueError(f"{name} must be positive and finite")
        if self.radius_min >= self.radius_max:
            raise ValueError("radius_min must be smaller than radius_max")
        if not self.radius_min <= self.radius_birth <= self.radius_max:
            raise ValueError("radius_birth must lie within its bounds")
        if (type(self.radius_fraction) not in (float, int)
                or not math.isfinite(self.radius_fraction)
                or not 0 <= self.radius_fraction <= 1):
            raise ValueError("radius_fraction must be a finite fraction in [0,1]")
        if (type(self.amplitude_std) not in (float, int)
                or not math.isfinite(self.amplitude_std) or self.amplitude_std < 0):
            raise ValueError("amplitude_std must be finite and nonnegative")

    optimizer_fields = (("amplitude", 0, 1), ("radius_fraction", 1, 2),
                        ("output_center", 2, 3), ("input_center", 3, 4))


@dataclass(frozen=True)
class PolarRadius:
    """PolarAmpRadiusSpec (rational envelope) + update settings (factories.py:403-460)."""

    amplitude_max: float
    w_c: float
    input_bounds: RadiusBounds
    output_bounds: RadiusBounds
    kappa: float = 3.0
    lower_kappa: float = 3.0
    upper_decay_power: float = 1.0
    alpha_init: float = 0.0
    radial_regularization: float = 0.1
    activity_gain: float = 1.0
    activity_mode: str = "finite_chord"
    dormant_expansion_rate: float = 0.0
    id: str = "polar_activity_radius"
    revision: int = 7

    def __post_init__(self):
        if not 0 <= self.alpha_init <= 1:
            raise ValueError("alpha_init must be in [0, 1]")
        if self.radial_regularization < 0:
            raise ValueError("radial_regularization must be nonnegative")
        if self.kappa <= 1 or self.upper_decay_power > 1:
            raise ValueError("kappa must exceed 1 and upper_decay_power must not exceed 1")
        if (self.activity_gain <= 0 or self.dormant_expansion_rate < 0
                or self.activity_mode not in ("finite_chord", "time_energy")):
            raise ValueError("invalid polar activity update settings")

    optimizer_fields = (("amplitude", 0, 2), ("output_center", 2, 3), ("input_center", 3, 4))


@dataclass(frozen=True)
class KernelSpec:
    """A separable cell-mass product kernel with its coordinate rule."""

    profiles: tuple
    coordinates: object
    composition: str = "separable"

    @property
    def revision(self):
        return self.coordinates.revision


@dataclass(frozen=True)
class RegularGrid:
    """A 1-D flat-torus regular grid chart (charts/presets.py:63-93)."""

    site_count: int
    spacing: float = 1.0
    origin: float = 0.0
    geometry: str = "flat_torus"

    @property
    def features(self):
        return self.site_count

    @property
    def period(self):
        return self.site_count * self.spacing


class chart_presets:  # noqa: N801 -- mirrors the reference module name
    @staticmethod
    def regular_grid(grid_shape, *, spacing=1.0, origin=0.0, geometry=None):
        if type(grid_shape) is tuple:
            if len(grid_shape) != 1:
                raise ValueError("radius cell masses require fixed one-dimensional torus grids")
            grid_shape = grid_shape[0]
        if type(grid_shape) is not int or grid_shape < 1:
            raise ValueError("grid_shape needs an int or a tuple of coordinate counts")
        if geometry != "flat_torus":
            raise ValueError("radius cell masses require fixed one-dimensional torus grids")
        if not (spacing > 0 and math.isfinite(spacing)) or not math.isfinite(origin):
            raise ValueError("spacing must be positive and origin finite")
        return RegularGrid(grid_shape, float(spacing), float(origin))


class kernels:  # noqa: N801 -- mirrors the reference module name
    @staticmethod
    def cell_mass(shape=None, *, base_tile_sites=1, merge_factor=2):
        return CellMass(ChebyshevSpec() if shape is None else shape, base_tile_sites,
                        merge_factor)

    @staticmethod
    def product(output_factor, input_factor=None, *, coordinates=None):
        if coordinates is None:
            raise ValueError("cell masses require Polar or rational radius coordinates")
        return KernelSpec((output_factor, output_factor if input_factor is None else input_factor),
                          coordinates)

    @staticmethod
    def rational_radius(*, radius_min=0.5, radius_birth=4.0, radius_max=50.0,
                        radius_fraction=0.0, amplitude_max=32.0, amplitude_std=0.1):
        return RationalRadius(radius_min, radius_birth, radius_max, amplitude_max,
                              radius_fraction, amplitude_std)

    @staticmethod
    def polar(*, amplitude_max, w_c, bounds=None, input_bounds=None, output_bounds=None,
              kappa=3.0, lower_kappa=None, upper_decay_power=1.0, alpha_init=0.0,
              radial_regularization=0.1, activity_gain=1.0, activity_mode="finite_chord",
              dormant_expansion_rate=0.0):
        if bounds is not None:
            if input_bounds is not None or output_bounds is not None:
                raise ValueError("use shared bounds or explicit input/output bounds")
            input_bounds = output_bounds = bounds
        if input_bounds is None:
            raise TypeError("coordinates require bounds or input_bounds")
        output_bounds = input_bounds if output_bounds is None else output_bounds
        if not isinstance(input_bounds, RadiusBounds) or not isinstance(output_bounds,
                                                                        RadiusBounds):
            raise ValueError("cell masses require RadiusBounds")
        return PolarRadius(amplitude_max, w_c, input_bounds, output_bounds, kappa,
                           kappa if lower_kappa is None else lower_kappa, upper_decay_power,
                           alpha_init, radial_regularization, activity_gain, activity_mode,
                           dormant_expansion_rate)


@dataclass(frozen=True)
class AxisDecl:
    """RadiusCellMassGrid: one validated axis (kernels/radius_cell_mass.py:16-26)."""

    site_count: int
    spacing: float
    origin: float
    base_tile_sites: int
    merge_factor: int
    modes: int

    @property
    def period(self):
        return self.site_count * self.spacing


def radius_cell_mass_axes(charts, kernel: KernelSpec):
    """Validate declarations (kernels/radius_cell_mass.py:29-93), output axis first."""
    if len(charts) != 2 or kernel.composition != "separable" or not isinstance(
            kernel.coordinates, (RationalRadius, PolarRadius)):
        raise ValueError("radius cell masses require the matching radius coordinate revision")
    axes = []
    for chart, binding in zip(charts, kernel.profiles):
        if type(chart) is not RegularGrid or chart.geometry != "flat_torus" or type(
                binding) is not CellMass:
            raise ValueError("radius cell masses require fixed one-dimensional torus grids")
        if chart.site_count % binding.base_tile_sites:
            raise ValueError("base_tile_sites must divide the chart site count")
        ratio = chart.site_count // binding.base_tile_sites
        while ratio > 1 and ratio % binding.merge_factor == 0:
            ratio //= binding.merge_factor
        if ratio != 1:
            raise ValueError("chart/base tile ratio must be a power of merge_factor")
        axes.append(AxisDecl(chart.site_count, chart.spacing, chart.origin,
                             binding.base_tile_sites, binding.merge_factor,
                             binding.profile.modes))
    coords = kernel.coordinates
    if isinstance(coords, RationalRadius):
        if any(coords.radius_max > a.period / 2 for a in axes):
            raise ValueError("radius bounds must fit each chart half-period")
    else:
        for axis, b in zip(axes, (coords.output_bounds, coords.input_bounds)):
            if b.maximum > axis.period / 2:
                raise ValueError("radius bounds must fit each chart half-period")
    return tuple(axes)
