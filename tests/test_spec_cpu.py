"""Declaration validation mirrors the reference messages (no device needed)."""

import pytest

from torchcst_b200 import ChebyshevSpec, RadiusBounds, chart_presets, kernels
from torchcst_b200.spec import radius_cell_mass_axes


def test_axes_validation_messages():
    g = chart_presets.regular_grid(12, geometry="flat_torus")
    k = kernels.product(kernels.cell_mass(ChebyshevSpec(8), base_tile_sites=5),
                        coordinates=kernels.rational_radius(radius_max=4.0))
    with pytest.raises(ValueError, match="base_tile_sites must divide"):
        radius_cell_mass_axes((g, g), k)
    k = kernels.product(kernels.cell_mass(ChebyshevSpec(8), base_tile_sites=2, merge_factor=3),
                        coordinates=kernels.rational_radius(radius_max=4.0))
    with pytest.raises(ValueError, match="power of merge_factor"):
        radius_cell_mass_axes((g, g), k)
    k = kernels.product(kernels.cell_mass(ChebyshevSpec(8)),
                        coordinates=kernels.rational_radius(radius_max=8.0))
    with pytest.raises(ValueError, match="half-period"):
        radius_cell_mass_axes((chart_presets.regular_grid(8, geometry="flat_torus"),) * 2, k)
    with pytest.raises(ValueError):
        chart_presets.regular_grid(8)
    with pytest.raises(ValueError):
        kernels.rational_radius(radius_fraction=1.5)


def test_config3_reading():
    out_f = kernels.cell_mass(ChebyshevSpec(modes=8))
    in_f = kernels.cell_mass(ChebyshevSpec(modes=8), base_tile_sites=49, merge_factor=2)
    coords = kernels.polar(amplitude_max=1.0, w_c=0.3, bounds=RadiusBounds(
        minimum=0.5, birth=4.0, maximum=50.0, upper_floor=1.0))
    axes = radius_cell_mass_axes(
        (chart_presets.regular_grid(1024, geometry="flat_torus"),
         chart_presets.regular_grid(784, geometry="flat_torus")),
        kernels.product(out_f, in_f, coordinates=coords))
    assert axes[1].base_tile_sites == 49 and axes[1].site_count == 784
