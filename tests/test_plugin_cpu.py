"""The torchcst backend plugin against the real reference package (CPU).

Registers the B200 Algorithm into torchcst's own registry, round-trips its
ExecutionPlan through JSON, checks that torchcst declarations convert to the
same native plan this package builds from its own declarations, and that a
reference CSTLinear routed to the plugin reports the missing sm_100 device
instead of running elsewhere. Needs the reference source tree; skipped where it
is absent (it is never present on the GPU box).
"""

import os
import sys

import pytest
import torch

# The reference source tree (its src/ directory), named by TORCHCST_REFERENCE_SRC;
# without it the tests run only where torchcst is importable already.
REF_SRC = os.environ.get("TORCHCST_REFERENCE_SRC")


@pytest.fixture(scope="module")
def tc():
    if REF_SRC:
        if not os.path.isdir(REF_SRC):
            pytest.skip("TORCHCST_REFERENCE_SRC is not a directory")
        if REF_SRC not in sys.path:
            sys.path.insert(0, REF_SRC)
    try:
        import torchcst
    except Exception as exc:  # pragma: no cover - depends on the container
        pytest.skip(f"torchcst not importable: {exc}")
    return torchcst


def _native_bytes(plan):
    import ctypes
    return (bytes(memoryview(plan.out_axis)), bytes(memoryview(plan.in_axis)),
            bytes(ctypes.string_at(ctypes.addressof(plan.coords), ctypes.sizeof(plan.coords))))


def test_register_plan_round_trip_and_duplicates(tc):
    from torchcst._backends.dispatch.select import FixedSelector
    from torchcst_b200 import plugin
    registry, plan = plugin.register()
    assert registry.loads_plan(registry.dumps_plan(plan)) == plan
    assert registry.validate_plan(plan).id == plugin.ALGORITHM_ID
    with pytest.raises(ValueError):
        registry.register(plugin.algorithm())
    FixedSelector(plan, registry=registry)
    with pytest.raises(ValueError):
        registry.validate_plan(plugin.plan(plugin.B200Recipe(validate="maybe")))


def _reference_layer(tc, n_out, n_in, coords, base_in=1, merge=2, atoms=16, seed=0):
    from torchcst import ChebyshevSpec, CSTLinear, chart_presets, kernels
    k = kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8), merge_factor=merge),
                        kernels.cell_mass(ChebyshevSpec(modes=8), base_tile_sites=base_in,
                                          merge_factor=merge),
                        coordinates=coords)
    torch.manual_seed(seed)
    return CSTLinear(charts=(chart_presets.regular_grid(n_out, geometry="flat_torus"),
                             chart_presets.regular_grid(n_in, geometry="flat_torus")),
                     atoms=atoms, kernel=k)


def test_declarations_convert_to_the_same_native_plan(tc):
    from torchcst import kernels as rk
    from torchcst.kernels.parameterizations.base import RadiusBounds as RB
    from torchcst_b200 import kernels, plugin
    from torchcst_b200 import runtime as R
    from torchcst_b200.spec import (CellMass, ChebyshevSpec, RadiusBounds, RegularGrid,
                                    radius_cell_mass_axes)
    cases = [
        ((8, 16, 1, 2), rk.rational_radius(radius_max=4.0, radius_fraction=0.0),
         kernels.rational_radius(radius_max=4.0)),
        ((1024, 1024, 1, 2), rk.rational_radius(radius_max=512.0, radius_fraction=0.0),
         kernels.rational_radius(radius_max=512.0)),
        ((1024, 784, 49, 2),
         rk.polar(amplitude_max=1.0, w_c=0.3, bounds=RB(minimum=0.5, birth=4.0, maximum=50.0,
                                                         upper_floor=1.0)),
         kernels.polar(amplitude_max=1.0, w_c=0.3,
                       bounds=RadiusBounds(minimum=0.5, birth=4.0, maximum=50.0,
                                           upper_floor=1.0))),
    ]
    for (n_out, n_in, base_in, merge), ref_coords, own_coords in cases:
        layer = _reference_layer(tc, n_out, n_in, ref_coords, base_in, merge)
        axes, spec = plugin.spec_from_reference(layer.cst_charts(), layer.kernel.declaration())
        own_kernel = kernels.product(CellMass(ChebyshevSpec(8), 1, merge),
                                     CellMass(ChebyshevSpec(8), base_in, merge),
                                     coordinates=own_coords)
        own_axes = radius_cell_mass_axes((RegularGrid(n_out), RegularGrid(n_in)), own_kernel)
        assert axes == own_axes
        assert _native_bytes(R.Plan.make(axes, spec)) == \
            _native_bytes(R.Plan.make(own_axes, own_kernel))


def test_reference_layer_routed_to_the_plugin_needs_sm100(tc):
    from torchcst import kernels as rk
    from torchcst_b200 import plugin
    layer = _reference_layer(tc, 8, 16, rk.rational_radius(radius_max=4.0, radius_fraction=0.0))
    layer.selector = plugin.selector()
    with pytest.raises(Exception, match="sm_100"):
        layer(torch.randn(4, 16))


def test_state_dict_round_trips_with_the_reference(tc):
    """A reference layer's state dict loads into the B200 layer and back
    unchanged (atoms under atom_state.atoms.p, reference row order)."""
    from torchcst import kernels as rk
    from torchcst_b200 import CSTLinear, ChebyshevSpec, chart_presets, kernels
    ref = _reference_layer(tc, 8, 16, rk.rational_radius(radius_max=4.0, radius_fraction=0.0),
                           atoms=12)
    ref_sd = ref.state_dict()
    own = CSTLinear(charts=(chart_presets.regular_grid(8, geometry="flat_torus"),
                            chart_presets.regular_grid(16, geometry="flat_torus")),
                    atoms=12,
                    kernel=kernels.product(kernels.cell_mass(ChebyshevSpec(modes=8)),
                                           coordinates=kernels.rational_radius(radius_max=4.0)))
    atoms_key = "atom_state.atoms.p"
    assert atoms_key in ref_sd and atoms_key in own.state_dict()
    own.load_state_dict({atoms_key: ref_sd[atoms_key]}, strict=False)
    assert torch.equal(own.atoms.p.detach(), ref_sd[atoms_key])
    with torch.no_grad():
        own.atoms.p.add_(0.125)
    ref.load_state_dict({atoms_key: own.state_dict()[atoms_key]}, strict=False)
    assert torch.equal(ref.state_dict()[atoms_key], own.atoms.p.detach())


def test_stand_in_declarations_convert_like_the_reference(tc):
    """tests/reference_decls.py (used where torchcst is absent) converts to the
    same native plan as the reference's own declarations of the same layers."""
    from tests import reference_decls as D
    from torchcst import kernels as rk
    from torchcst.kernels.parameterizations.base import RadiusBounds as RB
    from torchcst_b200 import plugin
    from torchcst_b200 import runtime as R
    cases = [
        ((8, 16, 1), rk.rational_radius(radius_max=4.0, radius_fraction=0.0),
         D.rational_kernel(4.0)),
        ((1024, 1024, 1), rk.rational_radius(radius_max=512.0, radius_fraction=0.0),
         D.rational_kernel(512.0)),
        ((1024, 784, 49),
         rk.polar(amplitude_max=1.0, w_c=0.3, bounds=RB(minimum=0.5, birth=4.0, maximum=50.0,
                                                         upper_floor=1.0)),
         D.polar_kernel()),
    ]
    for (n_out, n_in, base_in), ref_coords, stand_in in cases:
        layer = _reference_layer(tc, n_out, n_in, ref_coords, base_in)
        axes, spec = plugin.spec_from_reference(layer.cst_charts(), layer.kernel.declaration())
        axes2, spec2 = plugin.spec_from_reference((D.chart(n_out), D.chart(n_in)), stand_in)
        assert (axes, spec) == (axes2, spec2)
        assert _native_bytes(R.Plan.make(axes, spec)) == _native_bytes(R.Plan.make(axes2, spec2))


def test_update_algorithm_registers_and_needs_sm100(tc):
    """The atom_update Algorithm round-trips its plan, and a reference CSTAdamW
    routed to it on a CPU layer reports the missing sm_100 device."""
    from torchcst import CSTAdamW as RefAdamW
    from torchcst import kernels as rk
    from torchcst_b200 import plugin
    registry, _ = plugin.register()
    up = plugin.update_plan()
    assert registry.loads_plan(registry.dumps_plan(up)) == up
    assert registry.validate_plan(up).operation_id == "atom_update"
    layer = _reference_layer(tc, 8, 16, rk.rational_radius(radius_max=4.0, radius_fraction=0.0))
    opt = RefAdamW(layer.parameters(), model=layer, lr=1e-3,
                   update_selector=plugin.update_selector(registry))
    layer(torch.randn(4, 16)).square().mean().backward()
    with pytest.raises(ValueError, match="sm_100"):
        opt.step()


def test_auto_selector_falls_back_to_the_reference_choice(tc):
    """use_b200 routes a model's layers through the B200-first selector; without
    an sm_100 device the reference's own default plan runs, with identical
    results and gradients."""
    from torchcst import kernels as rk
    from torchcst_b200 import plugin
    coords = rk.rational_radius(radius_max=4.0, radius_fraction=0.0)
    a = _reference_layer(tc, 8, 16, coords, atoms=12)
    b = _reference_layer(tc, 8, 16, coords, atoms=12)
    model = torch.nn.Sequential(b, torch.nn.ReLU())
    assert plugin.use_b200(model) == 1
    x = torch.randn(4, 16)
    ya, yb = a(x), b(x)
    assert torch.equal(ya, yb)
    ya.square().sum().backward()
    yb.square().sum().backward()
    assert torch.equal(a.atoms.p.grad, b.atoms.p.grad)
    plugin.install()  # idempotent
    plugin.install()
